"""The inference engine: one DiT block as a short sequence of fused sm_100a kernels.

Per block (T packed rows, D = 5376, inner = 56 x 128):

    n1   = adaln_rmsnorm(x)                          norm.cu (+ per-frame sums of n1)
    qkvg = n1 @ [Wq; Wk; Wv; Wsgate; Wbeta; Wgdown]^T  gemm.cu, ONE GEMM for the three
                                                     projections and the three gate inputs;
    q, k = qk_prep(qkvg)                             its routed epilogue also writes the
                                                     QK-RMSNorm + 3D-RoPE'd q and k
    cat[:, :inner] = window_attention(q, k, v) * sigmoid(sgate)   attention.cu
    cat[video, inner:] = linear branch readout       linear_branch.cu chain
    x   += gate_msa[idx] * (cat @ [Wo | Wo_lin]^T + bo)  gemm.cu, K-concatenated O-proj and
                                                     to_out_linear, gated residual epilogue
    n2   = adaln_rmsnorm(x)
    h    = swiglu(n2 @ Wup^T + bup)                  gemm.cu, SwiGLU epilogue
    x   += gate_mlp[idx] * (h @ Wdown^T + bdown)     gemm.cu, gated residual epilogue

This is the arithmetic of the reference's fast_block_forward + HybridAttention
(src/models/ops/fused_block.py:93-111, src/models/hybrid_attention.py:178-255) with the
pointwise stretches folded into the GEMM epilogues. Packing the weights is one-way and
allocation-neutral: the packed buffers are built block by block and every original
parameter is re-pointed at a view of them, so the module tree (and LoRA/state-dict names)
keeps working and nothing is held twice.
"""
import types

import torch
import torch.nn.functional as F
from torch import nn

from vdn_minimax_h3_b200.models.h3 import H3Transformer
from vdn_minimax_h3_b200.models.hybrid_attention import HybridAttention
from vdn_minimax_h3_b200.models.layout import SequenceLayout
from vdn_minimax_h3_b200.models.window import AttentionPlan, full_cover
from vdn_minimax_h3_b200.ops import attention as attn_ops
from vdn_minimax_h3_b200.ops import gemm
from vdn_minimax_h3_b200.ops import linear_branch as lb
from vdn_minimax_h3_b200.ops import norm as norm_ops
from vdn_minimax_h3_b200.utils.profiling import SectionTimer


def _f32(t):
    return None if t is None else t.detach().float().contiguous()


class PackedBlock:
    """Concatenated / interleaved weights of one hybrid DiT block."""

    def __init__(self, block, cfg, fp8=False):
        attn = block.attn
        hybrid = isinstance(attn, HybridAttention)
        orig = attn.orig if hybrid else attn
        D, H, d = cfg.hidden_size, cfg.num_attention_heads, cfg.attention_head_dim
        inner = H * d
        self.hybrid = hybrid
        self.heads, self.head_dim, self.inner = H, d, inner
        dev = orig.to_q.weight.device
        dt = orig.to_q.weight.dtype
        # ---- QKV + gate inputs: one weight, one GEMM
        parts = [orig.to_q, orig.to_k, orig.to_v]
        extra = []
        self.has_sgate = hybrid and attn.enable_softmax_gate
        if self.has_sgate:
            extra.append(("sgate", attn.softmax_gate.up.weight, attn.softmax_gate.up.bias))
        if hybrid:
            br = attn.linear_attention
            extra.append(("beta", br.beta_proj.weight, None))
            extra.append(("ghid", br.output_gate.down.weight, None))
        def pad8(n):
            return (n + 7) // 8 * 8
        # every column group starts 16-byte aligned (a TMA / vector-load requirement)
        rows_pad = 3 * pad8(inner) + sum(pad8(w.shape[0]) for _, w, _ in extra)
        rows_pad = (rows_pad + 31) // 32 * 32   # whole 32-column groups (fp8 GEMM tiles)
        W = torch.zeros(rows_pad, D, device=dev, dtype=dt)
        b = torch.zeros(rows_pad, device=dev, dtype=torch.float32)
        off = 0
        self.cols = {}
        for name, lin in zip(("q", "k", "v"), parts):
            W[off:off + inner].copy_(lin.weight)
            if lin.bias is not None:
                b[off:off + inner].copy_(lin.bias.float())
            self.cols[name] = (off, off + inner)
            lin.weight.data = W[off:off + inner]
            off += pad8(inner)
        for name, w, bias in extra:
            n = w.shape[0]
            W[off:off + n].copy_(w)
            if bias is not None:
                b[off:off + n].copy_(bias.float())
            self.cols[name] = (off, off + n)
            w.data = W[off:off + n]
            off += pad8(n)
        self.w_qkvg, self.b_qkvg = W, b
        self.norm_q = _f32(orig.norm_q.weight)
        self.norm_k = _f32(orig.norm_k.weight)
        self.qk_eps = orig.norm_q.eps
        # ---- O-projection, K-concatenated with to_out_linear
        wo = orig.to_out[0].weight
        if hybrid:
            wl = attn.to_out_linear.weight
            Wo = torch.empty(D, inner + wl.shape[1], device=dev, dtype=dt)
            Wo[:, :inner].copy_(wo)
            Wo[:, inner:].copy_(wl)
            orig.to_out[0].weight.data = Wo[:, :inner]
            attn.to_out_linear.weight.data = Wo[:, inner:]
        else:
            Wo = wo.contiguous()
        self.w_o, self.b_o = Wo, _f32(orig.to_out[0].bias)
        # ---- feed-forward
        ff = block.ff
        self.ff_act = ff.activation
        up = ff.net[0].proj
        self.fp8 = fp8
        if fp8:
            from vdn_minimax_h3_b200.ops.fp8 import Fp8Weight
            self.w8_qkvg = Fp8Weight(self.w_qkvg, self.b_qkvg)
            if self.ff_act == "swiglu":
                self.w8_up = Fp8Weight(*gemm.interleave_swiglu_rows(up.weight.data, up.bias,
                                                                    tile=128))
            self.w8_down = Fp8Weight(ff.net[2].weight.data, ff.net[2].bias)
            self.w8_o = Fp8Weight(Wo, orig.to_out[0].bias)
        if self.ff_act == "swiglu":
            wi, bi = gemm.interleave_swiglu_rows(up.weight.data, up.bias)
            up.weight.data = wi   # NOTE: the module now holds the interleaved layout
            self.ff_interleaved = True
            self.w_up, self.b_up = wi, _f32(bi)
        else:
            self.ff_interleaved = False
            self.w_up, self.b_up = up.weight.data, _f32(up.bias)
        self.w_down, self.b_down = ff.net[2].weight.data, _f32(ff.net[2].bias)
        # ---- norms / modulation
        self.norm1 = _f32(block.norm1.weight)
        self.norm2 = _f32(block.norm2.weight)
        self.eps = block.norm1.eps
        self.adaln_w = block.adaln_proj.linear.weight.data
        self.adaln_b = _f32(block.adaln_proj.linear.bias)
        if hybrid:
            br = attn.linear_attention
            self.gate_up_w = br.output_gate.up.weight.data
            self.gate_up_b = _f32(br.output_gate.up.bias)


def _kernel_linear_forward(self, x):
    """nn.Linear.forward on the package's bf16 tcgen05 GEMM for bf16 CUDA rows (K a multiple
    of 8, 16-byte aligned rows), PyTorch otherwise."""
    w = self.weight
    if (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and x.shape[-1] % 8 == 0 and w.is_contiguous() and w.data_ptr() % 16 == 0):
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) == 1 and (x2.stride(0) * 2) % 16 == 0 and x2.data_ptr() % 16 == 0:
            return gemm.linear(x2, w, self.bias).view(*x.shape[:-1], w.shape[0])
    return F.linear(x, w, self.bias)


def route_outer_linears(model):
    """The Linears outside the block stack -- patch / audio / text embedders, the token
    refiner's projections and feed-forward, the video and audio output heads -- run on the
    bf16 GEMM kernel (instance-level forwards; parameters and their names are untouched).
    The refiner's attention already runs the dense plan of the attention kernel
    (models/h3.py: H3Attention). Returns the number of Linears routed."""
    names = ["proj_in", "audio_proj_in", "context_embedder", "proj_out", "audio_proj_out"]
    mods = [getattr(model, n) for n in names if hasattr(model, n)]
    for blk in model.token_refiner.refiner_blocks:
        mods += [m for m in blk.modules() if type(m) is nn.Linear]
    n = 0
    for m in mods:
        if type(m) is nn.Linear and not getattr(m, "_vdn_kernel_linear", False):
            m.forward = types.MethodType(_kernel_linear_forward, m)
            m._vdn_kernel_linear = True
            n += 1
    return n


class InferenceEngine:
    """Runs an H3Transformer (dense or hybrid) forward through the fused kernels."""

    def __init__(self, model: H3Transformer, fp8=False):
        """fp8=True: the QKV, FF-up and FF-down projections run on the block-scaled fp8
        GEMM (weights quantised once here, 128x128 blocks; activations quantised by the
        kernels that produce them, 1x128 blocks), as the reference's Fp8Linear conversion
        of the large Linears (src/models/ops/fp8_linear.py:286-323)."""
        self.model = model
        self.cfg = model.config
        self.fp8 = fp8
        self.outer_linears = route_outer_linears(model)
        self.blocks = []
        with torch.no_grad():
            for block in model.transformer_blocks:
                self.blocks.append(PackedBlock(block, self.cfg, fp8=fp8))
                if block.ff.activation == "swiglu":
                    block.ff.net[0].interleaved = 256
        self._plan_key = None
        self.plan = None
        self.dense_plan = None
        self._buffers = {}
        self._routes = {}
        self._cat_dirty = False
        self.timer = SectionTimer(False)

    # --------------------------------------------------------------------- helpers
    def _plans(self, attn, layout, T):
        key = (layout, attn.radius, attn.chunk, attn.anchor_frames) if attn is not None else (T,)
        if key != self._plan_key:
            dev = getattr(self, "compute_device", None)   # set when blocks stream from host
            if dev is None:
                dev = self.blocks[0].w_qkvg.device
            if attn is None or layout is None:
                from vdn_minimax_h3_b200.models.layout import SequenceLayout as SL
                lay = SL(seq_len=T, video_start=T, num_frames=0, tokens_per_frame=1)
                self.plan = AttentionPlan(lay, [], "none", device=dev, dense=True)
                self.covered = True
            else:
                bounds = attn.bounds(layout)
                self.covered = full_cover(bounds, layout.num_frames)
                self.plan = AttentionPlan(layout, bounds, attn.anchor_frames, device=dev,
                                          dense=self.covered)
                self.bounds = bounds
            self._plan_key = key
        return self.plan

    def _buf(self, name, shape, dtype, device, zero=False):
        b = self._buffers.get(name)
        if b is None or tuple(b.shape) != tuple(shape) or b.dtype != dtype or b.device != device:
            b = (torch.zeros if zero else torch.empty)(shape, dtype=dtype, device=device)
            self._buffers[name] = b
            if name == "cat":
                self._cat_dirty = False
        return b

    # ----------------------------------------------------------------------- block
    def block_forward(self, i, x, temb_act, adaln_idx, rope, layout):
        """x [T, D] bf16 updated in place."""
        pb = self.blocks[i]
        block = self.model.transformer_blocks[i]
        attn = block.attn
        cfg = self.cfg
        T, D = x.shape
        dev = x.device
        H, d, inner = pb.heads, pb.head_dim, pb.inner
        sec = self.timer.section
        # AdaLN table for this block: [n_t * MOD, 6D]
        with sec("adaln_table"):
            table = gemm.linear(temb_act, pb.adaln_w, pb.adaln_b).view(-1, 6 * D)
        linear_on = (pb.hybrid and layout is not None and attn.linear_attention_enabled
                     and not attn.teacher_mode)
        plan = self._plans(attn if pb.hybrid and not attn.teacher_mode else None, layout, T)
        linear_on = linear_on and not self.covered
        Fr = layout.num_frames if linear_on else 0
        S = layout.tokens_per_frame if linear_on else 1
        vs = layout.video_start if linear_on else 0
        n1 = self._buf("normed", (T, D), x.dtype, dev)
        f8 = pb.fp8 and x.is_cuda
        if f8:
            from vdn_minimax_h3_b200.ops import fp8 as fp8_ops
            nq = self._buf("normed_q", (T, D), torch.uint8, dev)
            nsf = self._buf("normed_sf", (fp8_ops.sf_bytes(T, D),), torch.uint8, dev)
        with sec("norm"):
            norm_ops.adaln_rmsnorm(x, pb.norm1, pb.eps, table, 0, D, adaln_idx,
                                   out=n1 if (linear_on or not f8) else False,
                                   fp8_out=(nq, nsf) if f8 else None)
            frame_sums = norm_ops.frame_sums(n1, Fr, S, 0, vs) if linear_on else None
        qkvg = self._buf("qkvg", (T, pb.w_qkvg.shape[0]), x.dtype, dev)
        c = pb.cols
        cos, sin = rope
        q = self._buf("q", (T, inner), x.dtype, dev)
        k = self._buf("k", (T, inner), x.dtype, dev)
        if f8 and fused_qk_ok(pb, cos):
            route = self._qkv_route(pb, qkvg, q, k)
            with sec("gemm_qkv"):
                fp8_ops.linear_routed_fp8(nq, nsf, pb.w8_qkvg, route, c["q"], c["k"], pb.norm_q,
                                          pb.norm_k, pb.qk_eps, cos, sin)
        elif fused_qk_ok(pb, cos):
            route = self._qkv_route(pb, qkvg, q, k)
            with sec("gemm_qkv"):
                gemm.linear_routed(n1, pb.w_qkvg, pb.b_qkvg, route, c["q"], c["k"], pb.norm_q,
                                   pb.norm_k, pb.qk_eps, cos, sin)
        else:
            with sec("gemm_qkv"):
                gemm.linear(n1, pb.w_qkvg, pb.b_qkvg, out=qkvg)
            with sec("qk_prep"):
                norm_ops.qk_prep(qkvg[:, c["q"][0]:c["q"][1]], H, pb.norm_q, pb.qk_eps, cos, sin,
                                 out=q)
                norm_ops.qk_prep(qkvg[:, c["k"][0]:c["k"][1]], H, pb.norm_k, pb.qk_eps, cos, sin,
                                 out=k)
        v = qkvg[:, c["v"][0]:c["v"][1]]
        kcat = pb.w_o.shape[1]
        cat = self._buf("cat", (T, kcat), x.dtype, dev, zero=True)
        sgate = qkvg[:, c["sgate"][0]:c["sgate"][1]] if pb.has_sgate else None
        with sec("attention"):
            attn_ops.window_attention(q.view(T, H, d), k.view(T, H, d), v.view(T, H, d), plan,
                                      d ** -0.5, gate_logits=sgate, out=cat[:, :inner])
        if pb.hybrid:
            if linear_on:
                with sec("linear_branch"):
                    self._linear_branch(pb, attn, layout, n1, qkvg, frame_sums, cat[:, inner:])
            elif self._cat_dirty:
                cat[:, inner:].zero_()
                self._cat_dirty = False
        with sec("gemm_o"):
            if f8:
                cq = self._buf("cat_q", tuple(cat.shape), torch.uint8, dev)
                csf = self._buf("cat_sf", (fp8_ops.sf_bytes(T, cat.shape[1]),), torch.uint8, dev)
                fp8_ops.quantize_act(cat, cq, csf)
                fp8_ops.linear_fp8_gated_residual(cq, csf, pb.w8_o, x, table[:, 2 * D:3 * D],
                                                  adaln_idx)
            else:
                gemm.linear_gated_residual(cat, pb.w_o, pb.b_o, x, table[:, 2 * D:3 * D],
                                           adaln_idx)
        n2 = n1
        if f8 and pb.ff_interleaved:
            with sec("norm"):
                norm_ops.adaln_rmsnorm(x, pb.norm2, pb.eps, table, 3 * D, 4 * D, adaln_idx,
                                       out=False, fp8_out=(nq, nsf))
            inter = pb.w8_up.shape[0] // 2
            hq = self._buf("h_q", (T, inter), torch.uint8, dev)
            hsf = self._buf("h_sf", (fp8_ops.sf_bytes(T, inter),), torch.uint8, dev)
            with sec("gemm_ff_up"):
                fp8_ops.linear_fp8_swiglu(nq, nsf, pb.w8_up, hq, hsf)
            with sec("gemm_ff_down"):
                fp8_ops.linear_fp8_gated_residual(hq, hsf, pb.w8_down, x, table[:, 5 * D:6 * D],
                                                  adaln_idx)
            return x
        with sec("norm"):
            norm_ops.adaln_rmsnorm(x, pb.norm2, pb.eps, table, 3 * D, 4 * D, adaln_idx, out=n2)
        with sec("gemm_ff_up"):
            if pb.ff_interleaved:
                h = gemm.linear_swiglu(n2, pb.w_up, pb.b_up)
            else:
                h = F.gelu(gemm.linear(n2, pb.w_up, pb.b_up).float(), approximate="tanh").to(x.dtype)
        with sec("gemm_ff_down"):
            gemm.linear_gated_residual(h, pb.w_down, pb.b_down, x, table[:, 5 * D:6 * D], adaln_idx)
        return x

    def _qkv_route(self, pb, qkvg, q, k):
        """Raw projection -> qkvg (all columns); normalised + rotated q/k -> q, k."""
        key = (qkvg.data_ptr(), tuple(qkvg.shape), q.data_ptr(), k.data_ptr(),
               tuple(sorted(pb.cols.items())))
        route = self._routes.get(key)
        if route is None:
            c = pb.cols
            route = gemm.ColumnRoute(qkvg.shape[1], planes=2)
            route.place(0, qkvg, plane=0)
            route.place(c["q"][0], q, plane=1)
            route.place(c["k"][0], k, plane=1)
            self._routes[key] = route
        return route

    def _linear_branch(self, pb, attn, layout, n1, qkvg, frame_sums, out):
        """The linear branch over the video rows, all heads; readout into `out` (video rows;
        anchor frames stay zero under anchors 'both')."""
        c = pb.cols
        H, d = pb.heads, pb.head_dim
        view = lambda name: qkvg[:, c[name][0]:c[name][1]]  # noqa: E731
        linear_branch_core(pb, attn, layout, self.bounds,
                           view("q").view(-1, H, d), view("k").view(-1, H, d),
                           view("v").view(-1, H, d), view("beta"), view("ghid"), frame_sums,
                           slice(0, H), out, n1.dtype)
        self._cat_dirty = True

    # --------------------------------------------------------------------- forward
    @torch.no_grad()
    def forward(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
                timestep_indices, token_tags, position_ids, video_indices, audio_indices,
                text_indices, layout: SequenceLayout = None, return_dict=False):
        m = self.model
        packed, temb, adaln_idx, rope = m.embed(
            hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
            timestep_indices, token_tags, position_ids, video_indices, audio_indices, text_indices)
        x = packed[0].contiguous()
        adaln_idx = adaln_idx.to(torch.int32).contiguous()
        temb_act = F.silu(temb.float()).to(x.dtype).contiguous()
        rope = (rope[0].contiguous(), rope[1].contiguous())
        if layout is None:
            first = next((b.attn for b in m.transformer_blocks if isinstance(b.attn, HybridAttention)), None)
            layout = None if first is None else first.layout
        for i in range(len(self.blocks)):
            self.block_forward(i, x, temb_act, adaln_idx, rope, layout)
        return m.head(x.unsqueeze(0), temb, timestep_indices, video_indices, audio_indices)

    __call__ = forward


def fused_qk_ok(pb, cos):
    """The QKV GEMM's routed epilogue handles 128-wide heads with full-width rotate-half
    RoPE on 128-column boundaries of the packed projection."""
    c = pb.cols
    return (cos.is_cuda and pb.head_dim == 128 and cos.shape[-1] == 128
            and cos.dtype == torch.float32 and c["q"][0] % 128 == 0 and c["k"][0] % 128 == 0)


def linear_branch_core(pb, attn, layout, bounds, q_raw, k_raw, v_raw, beta_logits, ghid,
                       frame_sums, heads, out, dtype, scatter=None):
    """The forward-only linear branch for a head range over every video row.

    q_raw/k_raw/v_raw [T, n, d] and beta_logits [T, n] cover the packed sequence (rows of
    the whole sequence, this head range); ghid [T, rank] is the output gate's low-rank
    hidden; frame_sums [F, D] fp32 are the per-frame sums of the attention input over the
    whole clip. Writes the gated, normalised readout of the generated frames into
    out[video rows] ([T, n*d] view); other rows are left untouched (zero). With
    scatter = (bases, _, rows_per_rank) the rows go to their Ulysses owners instead
    (`out` then only gives the row stride)."""
    br = attn.linear_attention
    n, d = heads.stop - heads.start, pb.head_dim
    ch = slice(heads.start * d, heads.stop * d)
    Fr, S = layout.num_frames, layout.tokens_per_frame
    vs = layout.video_start
    skip = attn.anchor_frames == "both"
    f0, f1 = (1, Fr - 1) if skip else (0, Fr)
    if f1 - f0 <= 0:
        return
    r0, r1 = vs + f0 * S, vs + f1 * S
    nF = f1 - f0
    conv = br.short_conv
    fs = layout.frame_size if conv is not None else None
    feats = []
    for t, proj in ((q_raw, "q"), (k_raw, "k"), (v_raw, "v")):
        t = t[r0:r1]
        if conv is not None and proj in conv.projs:
            w_sp, w_tm = conv.weights(proj, ch)
            feats.append(lb.conv_features(t, w_sp, w_tm, nF, fs, proj != "v"))
        else:
            feats.append(lb.activate(t, proj != "v"))
    qf, kf, vf = feats
    beta = torch.sigmoid(beta_logits[r0:r1].float())
    A, B = lb.frame_statistics(kf.view(nF, S, n, d), vf.view(nF, S, n, d), beta.view(nF, S, n),
                               a_fp32=br.a_fp32)
    del kf, vf
    alpha = br.alpha(frame_sums[f0:f1] / S, heads=None if n == pb.heads else heads)
    text_state = None
    if attn.enable_text_state:
        ts, te = layout.text_range
        text_raw = (q_raw[ts:te], k_raw[ts:te], v_raw[ts:te])
        text_beta = torch.sigmoid(beta_logits[ts:te].float())
        text_state = lb.text_state(br, text_raw, text_beta)
    trans, inj = lb.factor_apply(br.backend(S), alpha, A, B)
    prefix, suffix = lb.run_scans(trans, inj, text_state)
    bnd = bounds[f0:f1]
    if skip:
        bnd = [(lo - 1, hi - 1) for lo, hi in bnd]
    state = lb.gather(prefix, suffix, alpha, bnd, br.bridge, text_state, out_dtype=dtype)
    del prefix, suffix, trans, inj
    up_w = pb.gate_up_w[ch]
    up_b = None if pb.gate_up_b is None else pb.gate_up_b[ch]
    gate_logits = gemm.linear(ghid[r0:r1], up_w, up_b)
    if scatter is not None:
        lb.readout(qf.view(nF, S, n, d), state, br.norm.weight, gate_logits.view(-1, n, d),
                   br.norm.eps, out=out, gate_logits=True, scatter=(scatter[0], r0, scatter[2]))
    else:
        lb.readout(qf.view(nF, S, n, d), state, br.norm.weight, gate_logits.view(-1, n, d),
                   br.norm.eps, out=out[r0:r1], gate_logits=True)
