"""Ulysses sequence parallelism for the inference engine.

Reference parity: src/inference/utils/{ulysses.py, ulysses_runtime.py}. The residual stream
is sharded by packed-sequence row (ceil(T/P) rows per rank, the short shard last,
`sequence_splits`); inside attention one all-to-all turns "local rows x all heads" into
"all rows x local heads" (seq -> heads), every rank runs the window softmax and the linear
branch over the WHOLE sequence for its H/P heads, and a second all-to-all brings both
branches' outputs back to the row owners (heads -> seq). The per-frame means the linear
branch's alpha needs are partial sums per shard, all-reduced (N7 in the reference's
collective inventory). Embedding, token refiner and the output head run replicated, the
block residual is all-gathered once at the end.

`exchange` selects the transport: "nccl" (torch.distributed all_to_all_single, the
reference's own path) or "p2p" (this package's symmetric-memory peer kernels, see
parallel/symmetric.py) once those are installed.
"""
import math

import torch
import torch.distributed as dist

from vdn_minimax_h3_b200.inference.engine import InferenceEngine, linear_branch_core
from vdn_minimax_h3_b200.ops import attention as attn_ops
from vdn_minimax_h3_b200.ops import gemm
from vdn_minimax_h3_b200.ops import norm as norm_ops
from vdn_minimax_h3_b200.utils.profiling import SectionTimer


def sequence_splits(sequence_length, world_size):
    """Contiguous, nearly even shards, ceil(S/P) rows each, the short shard last."""
    if sequence_length <= 0 or world_size <= 0:
        raise ValueError("sequence_length and world_size must be positive")
    if world_size == 1:
        return (sequence_length,)
    chunk = math.ceil(sequence_length / world_size)
    last = sequence_length - chunk * (world_size - 1)
    if last <= 0:
        base, extra = divmod(sequence_length, world_size)
        return tuple(base + (r < extra) for r in range(world_size))
    return (chunk,) * (world_size - 1) + (last,)


def balanced_splits(total, parts):
    """Contiguous split of `total` with imbalance at most one (head ranges)."""
    if total <= 0 or parts <= 0 or parts > total:
        raise ValueError(f"need 0 < parts <= total; got total={total}, parts={parts}")
    base, extra = divmod(total, parts)
    return tuple(base + (r < extra) for r in range(parts))


class UlyssesRuntime:
    """Rank layout of one sequence-parallel group."""

    def __init__(self, group=None, profile=False):
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.timer = SectionTimer(profile)
        self.seq_len = None

    def configure(self, seq_len, num_heads):
        if num_heads % self.world_size:
            raise ValueError(f"{num_heads} heads are not divisible by {self.world_size} ranks")
        if self.seq_len == seq_len:
            return
        self.seq_len = seq_len
        self.splits = sequence_splits(seq_len, self.world_size)
        self.rows = math.ceil(seq_len / self.world_size)          # padded shard height
        self.local_start = sum(self.splits[:self.rank])
        self.local_end = self.local_start + self.splits[self.rank]
        self.heads_per_rank = num_heads // self.world_size

    def barrier(self):
        dist.barrier(group=self.group)

    def all_to_all(self, out, inp):
        dist.all_to_all_single(out, inp, group=self.group)

    def all_reduce(self, t, async_op=False):
        return dist.all_reduce(t, group=self.group, async_op=async_op)

    def all_gather_rows(self, local, out):
        dist.all_gather_into_tensor(out, local, group=self.group)


def init_ulysses(profile=False):
    if not dist.is_initialized():
        raise RuntimeError("init_process_group(nccl) before init_ulysses()")
    return UlyssesRuntime(profile=profile)


class UlyssesEngine:
    """Sequence-parallel forward over an InferenceEngine's packed weights (one rank)."""

    def __init__(self, engine: InferenceEngine, runtime: UlyssesRuntime, exchange="nccl"):
        self.engine = engine
        self.model = engine.model
        self.rt = runtime
        self.exchange = exchange
        self._bufs = {}

    def _buf(self, name, shape, dtype, device):
        b = self._bufs.get(name)
        if b is None or tuple(b.shape) != tuple(shape) or b.dtype != dtype:
            b = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[name] = b
        return b

    # ----------------------------------------------------------------------- block
    def block_forward(self, i, x, temb_act, adaln_idx, rope, layout):
        eng, rt = self.engine, self.rt
        pb = eng.blocks[i]
        attn = self.model.transformer_blocks[i].attn
        sec = rt.timer.section
        P, r = rt.world_size, rt.rank
        T = rt.seq_len
        C = rt.rows
        a0 = rt.local_start
        rows = x.shape[0]
        D = x.shape[1]
        H, d = pb.heads, pb.head_dim
        Hp = rt.heads_per_rank
        dev = x.device
        hybrid_on = pb.hybrid and not attn.teacher_mode and layout is not None
        plan = eng._plans(attn if hybrid_on else None, layout, T)
        linear_on = hybrid_on and attn.linear_attention_enabled and not eng.covered
        with sec("adaln_table"):
            table = gemm.linear(temb_act, pb.adaln_w, pb.adaln_b).view(-1, 6 * D)
        n1 = self._buf("n1", (rows, D), x.dtype, dev)
        with sec("norm"):
            norm_ops.adaln_rmsnorm(x, pb.norm1, pb.eps, table, 0, D, adaln_idx, out=n1)
        work = None
        if linear_on:
            fsum = norm_ops.frame_sums(n1, layout.num_frames, layout.tokens_per_frame, a0,
                                       layout.video_start)
            work = rt.all_reduce(fsum, async_op=True)
        qkvg = self._buf("qkvg", (rows, pb.w_qkvg.shape[0]), x.dtype, dev)
        with sec("gemm_qkv"):
            gemm.linear(n1, pb.w_qkvg, pb.b_qkvg, out=qkvg)
        c = pb.cols
        cos, sin = rope
        # ---- seq -> heads: pack [P, C, W] (q, k, v, q_raw, k_raw, sgate, beta, ghid per rank)
        rank_h = (c["ghid"][1] - c["ghid"][0]) if "ghid" in c else 0
        pad8 = lambda n: (n + 7) // 8 * 8  # noqa: E731  (every field 16-byte aligned)
        fields = [Hp * d] * 5 + [Hp if pb.has_sgate else 0, Hp if "beta" in c else 0, rank_h]
        widths = [pad8(w) for w in fields]
        W = sum(widths)
        send = self._buf("send", (P, C, W), x.dtype, dev)
        with sec("qk_prep+pack"):
            q = self._buf("q", (rows, H * d), x.dtype, dev)
            k = self._buf("k", (rows, H * d), x.dtype, dev)
            norm_ops.qk_prep(qkvg[:, c["q"][0]:c["q"][1]], H, pb.norm_q, pb.qk_eps, cos, sin, out=q)
            norm_ops.qk_prep(qkvg[:, c["k"][0]:c["k"][1]], H, pb.norm_k, pb.qk_eps, cos, sin, out=k)
            sv = send[:, :rows]
            hv = lambda t, w: t.view(rows, P, w).transpose(0, 1)  # noqa: E731
            srcs = [q, k, qkvg[:, c["v"][0]:c["v"][1]], qkvg[:, c["q"][0]:c["q"][1]],
                    qkvg[:, c["k"][0]:c["k"][1]]]
            srcs.append(qkvg[:, c["sgate"][0]:c["sgate"][1]] if pb.has_sgate else None)
            srcs.append(qkvg[:, c["beta"][0]:c["beta"][1]] if "beta" in c else None)
            off = 0
            for src, w, wp in zip(srcs, fields[:7], widths[:7]):
                if src is not None and w:
                    sv[:, :, off:off + w].copy_(hv(src, w))
                off += wp
            if rank_h:
                sv[:, :, off:off + rank_h].copy_(
                    qkvg[:, c["ghid"][0]:c["ghid"][1]].unsqueeze(0).expand(P, rows, rank_h))
        recv = self._buf("recv", (P, C, W), x.dtype, dev)
        with sec("a2a_dispatch"):
            rt.all_to_all(recv.view(-1), send.view(-1))
        full = recv.view(P * C, W)[:T]
        off = 0
        views = []
        for w, wp in zip(fields, widths):
            views.append(full[:, off:off + w])
            off += wp
        q_h, k_h, v_h, qr_h, kr_h, sg_h, bt_h, gh_h = views
        ret = self._buf("ret", (P * C, 2 * Hp * d), x.dtype, dev)
        with sec("attention"):
            attn_ops.window_attention(q_h.view(T, Hp, d), k_h.view(T, Hp, d), v_h.view(T, Hp, d),
                                      plan, d ** -0.5, gate_logits=sg_h if pb.has_sgate else None,
                                      out=ret[:T, :Hp * d])
        if pb.hybrid:
            ret[:T, Hp * d:].zero_()
            if linear_on:
                work.wait()
                with sec("linear_branch"):
                    linear_branch_core(pb, attn, layout, eng.bounds, qr_h.view(T, Hp, d),
                                       kr_h.view(T, Hp, d), v_h.view(T, Hp, d), bt_h, gh_h, fsum,
                                       slice(r * Hp, (r + 1) * Hp), ret[:T, Hp * d:], x.dtype)
        # ---- heads -> seq
        back = self._buf("back", (P, C, 2 * Hp * d), x.dtype, dev)
        with sec("a2a_return"):
            rt.all_to_all(back.view(-1), ret.view(-1))
        kcat = pb.w_o.shape[1]
        cat = self._buf("cat", (rows, kcat), x.dtype, dev)
        with sec("unpack"):
            nb = 2 if pb.hybrid else 1
            src = back[:, :rows].unflatten(-1, (2, Hp, d))[:, :, :nb]
            cat.view(rows, nb, P, Hp, d).copy_(src.permute(1, 2, 0, 3, 4))
        with sec("gemm_o"):
            gemm.linear_gated_residual(cat, pb.w_o, pb.b_o, x, table[:, 2 * D:3 * D], adaln_idx)
        n2 = n1
        with sec("norm"):
            norm_ops.adaln_rmsnorm(x, pb.norm2, pb.eps, table, 3 * D, 4 * D, adaln_idx, out=n2)
        with sec("gemm_ff_up"):
            h = gemm.linear_swiglu(n2, pb.w_up, pb.b_up)
        with sec("gemm_ff_down"):
            gemm.linear_gated_residual(h, pb.w_down, pb.b_down, x, table[:, 5 * D:6 * D], adaln_idx)
        return x

    # --------------------------------------------------------------------- forward
    @torch.no_grad()
    def forward(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
                timestep_indices, token_tags, position_ids, video_indices, audio_indices,
                text_indices, layout=None, return_dict=False):
        m, rt = self.model, self.rt
        T = position_ids.shape[0]
        rt.configure(T, m.config.num_attention_heads)
        packed, temb, adaln_idx, rope = m.embed(
            hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
            timestep_indices, token_tags, position_ids, video_indices, audio_indices, text_indices)
        if layout is None:
            from vdn_minimax_h3_b200.models.hybrid_attention import HybridAttention
            first = next((b.attn for b in m.transformer_blocks if isinstance(b.attn, HybridAttention)), None)
            layout = None if first is None else first.layout
        a, b = rt.local_start, rt.local_end
        x = packed[0, a:b].contiguous()
        idx = adaln_idx[a:b].to(torch.int32).contiguous()
        rope_l = (rope[0][a:b].contiguous(), rope[1][a:b].contiguous())
        temb_act = torch.nn.functional.silu(temb.float()).to(x.dtype).contiguous()
        for i in range(len(self.engine.blocks)):
            self.block_forward(i, x, temb_act, idx, rope_l, layout)
        full = self._buf("gather", (rt.world_size * rt.rows, x.shape[1]), x.dtype, x.device)
        local = self._buf("gather_local", (rt.rows, x.shape[1]), x.dtype, x.device)
        local[:x.shape[0]].copy_(x)
        rt.all_gather_rows(local, full)
        return m.head(full[:T].unsqueeze(0), temb, timestep_indices, video_indices, audio_indices)

    __call__ = forward
