"""HybridAttention: the H3 attention wrapped into window softmax + linear branch.

Reference parity: src/models/hybrid_attention.py:32-255.

    softmax_output = orig.to_out( softmax_gate(x) * window_softmax(q, k, v) )
    linear_readout = output_gate(x) * RMSNorm( linear_attention(q_raw, k_raw, v_raw) )
    output         = softmax_output + to_out_linear(linear_readout)      # video rows only

`teacher_mode` passes straight through to the original attention; a window that covers
every frame is the original dense attention and switches the linear branch off.

This module's forward is the eager path (training, CPU oracle, teacher). The production
inference forward of a whole block -- fused kernels, concatenated projections, the window
kernel over the AttentionPlan -- is inference/engine.py, which reads the same parameters.
"""
import torch
from torch import nn

from vdn_minimax_h3_b200.models.h3 import _attention_kernels, apply_rotary_emb
from vdn_minimax_h3_b200.models.layout import SequenceLayout
from vdn_minimax_h3_b200.models.linear_branch import BidirectionalLinearBranch, OutputGate
from vdn_minimax_h3_b200.models.window import (ANCHOR_FRAME_MODES, full_cover, window_bounds,
                                               window_softmax_segments)

SOFTMAX_BACKENDS = ("auto", "kernel", "ref")


class HybridAttention(nn.Module):
    def __init__(self, orig_attn, hidden_size, delta_rule="sana_scaled", radius=4, chunk=0,
                 enable_softmax_gate=True, linear_head_dim=None, softmax_impl="auto",
                 anchor_frames="none", enable_text_state=False, bridge="alpha", a_fp32=True,
                 short_conv=()):
        super().__init__()
        if anchor_frames not in ANCHOR_FRAME_MODES:
            raise ValueError(f"anchor_frames={anchor_frames!r}; expected one of {ANCHOR_FRAME_MODES}")
        self.orig = orig_attn
        self.num_heads = orig_attn.heads
        self.head_dim = orig_attn.head_dim
        self.radius, self.chunk = radius, chunk
        self.softmax_impl = softmax_impl
        self.anchor_frames = anchor_frames
        self.enable_text_state = enable_text_state
        self.linear_attention_enabled = True
        self.layout: SequenceLayout = None
        self.teacher_mode = False
        self.inference_mode = False
        d_lin = linear_head_dim or self.head_dim
        self.linear_attention = BidirectionalLinearBranch(
            hidden_size, self.num_heads, d_lin, delta_rule=delta_rule, bridge=bridge,
            a_fp32=a_fp32, short_conv=short_conv)
        self.to_out_linear = nn.Linear(self.num_heads * d_lin, hidden_size, bias=False)
        self.enable_softmax_gate = enable_softmax_gate
        if enable_softmax_gate:
            self.softmax_gate = OutputGate(hidden_size, self.num_heads, init_value=0.99)

    @property
    def heads(self):
        return self.num_heads

    def bounds(self, layout=None):
        layout = layout or self.layout
        return window_bounds(layout.num_frames, self.radius, self.chunk)

    def forward(self, hidden_states, rotary_emb=None, attention_mask=None):
        if attention_mask is not None:
            raise ValueError("H3 packs one request per document; no attention mask expected")
        if hidden_states.shape[0] != 1:
            raise ValueError("HybridAttention assumes batch 1 (one packed document)")
        if self.teacher_mode:
            return self.orig(hidden_states, rotary_emb, attention_mask)
        return self.hybrid_forward(hidden_states[0], rotary_emb).unsqueeze(0)

    def hybrid_forward(self, x, rotary_emb):
        layout = self.layout
        bounds = self.bounds(layout) if layout is not None else None
        covered = layout is None or full_cover(bounds, layout.num_frames)
        scale = self.head_dim ** -0.5
        q, k, v, raw = self.orig.project(x, rotary_emb)
        ag = _attention_kernels() if self.softmax_impl != "ref" else None
        use_kernel = ag is not None and ag.kernel_path_ok(q, k, v)
        if self.softmax_impl == "kernel" and q.is_cuda and not use_kernel:
            raise RuntimeError("softmax_backend=kernel: the window kernel does not take these "
                               f"tensors (q {tuple(q.shape)} {q.dtype}); use auto or ref")
        if use_kernel:
            # sm_100a forward + backward kernels over the analytic plan (dense when covered)
            plan = (ag.dense_plan(x.shape[0], x.device) if covered
                    else ag.window_plan(layout, bounds, self.anchor_frames, x.device))
            soft = ag.window_attention_train(q, k, v, plan, scale)
            linear_active = not covered
        elif covered:
            import torch.nn.functional as F
            soft = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                                  v.transpose(0, 1)[None])[0].transpose(0, 1)
            linear_active = False
        else:
            soft = window_softmax_segments(q, k, v, layout, bounds, scale, self.anchor_frames)
            linear_active = True
        del q, k, v
        if self.enable_softmax_gate:
            flat = (soft * self.softmax_gate(x).to(soft.dtype)).reshape(x.shape[0], -1)
        else:
            flat = soft.reshape(x.shape[0], -1)
        out = self.orig.to_out[1](self.orig.to_out[0](flat.type_as(x)))
        if linear_active and self.linear_attention_enabled:
            vs, ve = layout.video_start, layout.video_end
            text_x = text_raw = None
            if self.enable_text_state:
                ts, te = layout.text_range
                text_x = x[ts:te]
                text_raw = tuple(t[ts:te] for t in raw)
            readout = self.linear_attention(
                x[vs:ve], layout.num_frames, layout.tokens_per_frame, bounds,
                tuple(t[vs:ve] for t in raw),
                frame_size=layout.frame_size if self.linear_attention.short_conv is not None else None,
                skip_ends=self.anchor_frames == "both", text_x=text_x, text_qkv_raw=text_raw,
                inference=False)
            if torch.is_grad_enabled():
                out = out.clone()
            out[vs:ve] += self.to_out_linear(readout.type_as(x))
        return out
