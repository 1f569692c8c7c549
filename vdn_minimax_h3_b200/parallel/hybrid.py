"""Tensor parallel x Ulysses sequence parallel inference (e.g. TP=2 x Ulysses=4 on 8 GPUs).

The reference has no tensor parallelism; this is the layout of the hybrid configuration the
build targets. Ranks are r = s * tp + t: Ulysses shard s (rows [s*CS, (s+1)*CS), CS = tp*C,
C = ceil(T / world)) and tensor-parallel index t. Rank r owns residual rows
[r*C, (r+1)*C) (sequence-parallel TP: the residual is never replicated).

Per block, every exchange is a store issued by the kernel that produces the data:
  norm       AdaLN-RMSNorm of the own rows, written (E4M3 + scales, and bf16 for the
             per-frame sums) into BOTH ranks of the TP pair at row t*C: the all-gather of
             the column-parallel GEMM's input is done by its producer.
  QKV        column-parallel (this TP rank's H/tp heads; the low-rank gate input whole),
             routed epilogue: QK-norm + RoPE, and every head group written straight into
             its Ulysses destination's receive slab (peer memory).
  attention  + linear branch over all rows for H/world heads; epilogues store each output
             row into its row owner's O-projection input (row scatter).
  O-proj     row-parallel (this TP rank's heads along K); the epilogue stores bf16 partial
             rows into the owning TP rank's partial buffer: the reduce-scatter is done by
             the GEMM. A combine kernel adds both (bf16) partials, bias and the gated
             residual in fp32.
  FF         the same pattern: norm all-gather -> column-parallel SwiGLU (E4M3 out) ->
             row-parallel down projection with the partial-sum scatter -> combine.
Device flag barriers (parallel/symmetric.py) order each exchange inside the TP pair or the
Ulysses group; the per-frame sums for the linear branch's alpha are one NCCL all-reduce.
"""
import math

import torch
import torch.distributed as dist

from vdn_minimax_h3_b200.inference.engine import InferenceEngine, fused_qk_ok, linear_branch_core
from vdn_minimax_h3_b200.ops import attention as attn_ops
from vdn_minimax_h3_b200.ops import gemm
from vdn_minimax_h3_b200.ops import norm as norm_ops
from vdn_minimax_h3_b200.ops._ext import error_word, ext
from vdn_minimax_h3_b200.parallel.head import ShardedHead
from vdn_minimax_h3_b200.parallel.symmetric import SymmetricHeap
from vdn_minimax_h3_b200.utils.profiling import SectionTimer


class HybridRuntime:
    """Rank layout and process groups of TP x Ulysses."""

    def __init__(self, tp, profile=False):
        if not dist.is_initialized():
            raise RuntimeError("init_process_group(nccl) before HybridRuntime()")
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()
        if tp < 1 or self.world % tp:
            raise ValueError(f"tp={tp} does not divide world size {self.world}")
        self.tp = tp
        self.sp = self.world // tp
        self.tp_rank = self.rank % tp
        self.sp_rank = self.rank // tp
        # every rank creates every group, in the same order
        tp_groups = [dist.new_group([s * tp + t for t in range(tp)]) for s in range(self.sp)]
        sp_groups = [dist.new_group([s * tp + t for s in range(self.sp)]) for t in range(tp)]
        self.tp_group = tp_groups[self.sp_rank]
        self.sp_group = sp_groups[self.tp_rank]
        self.timer = SectionTimer(profile)
        self.seq_len = None

    def barrier(self):
        dist.barrier()

    def configure(self, T, heads):
        if heads % self.world:
            raise ValueError(f"{heads} heads are not divisible by {self.world} ranks")
        if self.seq_len == T:
            return
        self.seq_len = T
        self.C = math.ceil(T / self.world)             # residual rows per rank
        self.CS = self.C * self.tp                     # rows per Ulysses shard
        self.row0 = self.rank * self.C
        self.rows = max(0, min(T, self.row0 + self.C) - self.row0)
        self.shard0 = self.sp_rank * self.CS
        self.shard_rows = max(0, min(T, self.shard0 + self.CS) - self.shard0)
        self.heads_tp = heads // self.tp               # heads of this TP rank
        self.hp = heads // self.world                  # heads per rank after the all-to-all


def _pad(n, m):
    return (n + m - 1) // m * m


class TpBlock:
    """This TP rank's shard of a PackedBlock: column-parallel QKV / FF-up rows and
    row-parallel O / FF-down columns, bf16 and (optionally) block-scaled E4M3."""

    def __init__(self, pb, tp, t, fp8):
        H, d = pb.heads, pb.head_dim
        Ht = H // tp
        hs = slice(t * Ht * d, (t + 1) * Ht * d)
        c = pb.cols
        W, b = pb.w_qkvg, pb.b_qkvg
        parts, self.cols, off = [], {}, 0
        names = [("q", hs), ("k", hs), ("v", hs)]
        if "sgate" in c:
            names.append(("sgate", slice(t * Ht, (t + 1) * Ht)))
        if "beta" in c:
            names.append(("beta", slice(t * Ht, (t + 1) * Ht)))
        if "ghid" in c:
            names.append(("ghid", slice(0, c["ghid"][1] - c["ghid"][0])))
        for name, sl in names:
            lo = c[name][0]
            rows = W[lo + sl.start:lo + sl.stop]
            parts.append((name, rows, b[lo + sl.start:lo + sl.stop]))
        n_rows = _pad(sum(_pad(r.shape[0], 8) for _, r, _ in parts), 32)
        Wt = torch.zeros(n_rows, W.shape[1], device=W.device, dtype=W.dtype)
        bt = torch.zeros(n_rows, device=W.device, dtype=torch.float32)
        for name, rows, bias in parts:
            Wt[off:off + rows.shape[0]] = rows
            bt[off:off + rows.shape[0]] = bias
            self.cols[name] = (off, off + rows.shape[0])
            off += _pad(rows.shape[0], 8)
        self.w_qkvg, self.b_qkvg = Wt, bt
        # O: this TP rank's heads of the attention half and of the linear half (along K)
        inner = H * d
        if pb.hybrid:
            self.w_o = torch.cat([pb.w_o[:, hs], pb.w_o[:, inner + hs.start:inner + hs.stop]], 1).contiguous()
        else:
            self.w_o = pb.w_o[:, hs].contiguous()
        self.b_o = pb.b_o
        # FF: this rank's intermediate channels (value and gate rows), and down columns
        inter = pb.w_up.shape[0] // 2
        It = inter // tp
        wi = pb.w_up.view(inter // 128, 2, 128, -1)             # 256-interleaved [v | g]
        value = wi[:, 0].reshape(inter, -1)[t * It:(t + 1) * It]
        gate = wi[:, 1].reshape(inter, -1)[t * It:(t + 1) * It]
        bup = None
        if pb.b_up is not None:
            bi = pb.b_up.view(inter // 128, 2, 128)
            bup = torch.cat([bi[:, 0].reshape(-1)[t * It:(t + 1) * It],
                             bi[:, 1].reshape(-1)[t * It:(t + 1) * It]])
        up = torch.cat([value, gate], 0)
        self.w_up, self.b_up = gemm.interleave_swiglu_rows(up, bup)
        self.b_up = None if self.b_up is None else self.b_up.float().contiguous()
        self.w_down = pb.w_down[:, t * It:(t + 1) * It].contiguous()
        self.b_down = pb.b_down
        self.fp8 = fp8
        if fp8:
            from vdn_minimax_h3_b200.ops.fp8 import Fp8Weight
            self.w8_qkvg = Fp8Weight(self.w_qkvg, self.b_qkvg)
            self.w8_o = Fp8Weight(self.w_o)
            self.w8_up = Fp8Weight(*gemm.interleave_swiglu_rows(up, bup, tile=128))
            self.w8_down = Fp8Weight(self.w_down)


class HybridEngine:
    """TP x Ulysses forward over an InferenceEngine's packed weights (one rank, CUDA)."""

    def __init__(self, engine: InferenceEngine, runtime: HybridRuntime, fp8=False):
        self.engine = engine
        self.model = engine.model
        self.rt = runtime
        self.fp8 = fp8
        rt = runtime
        with torch.no_grad():
            self.tblocks = [TpBlock(pb, rt.tp, rt.tp_rank, fp8) for pb in engine.blocks]
        self._bufs = {}
        self._routes = {}
        self.tp_heap = None
        self.sp_heap = None
        self._heap_key = None
        self.head = ShardedHead()

    def _buf(self, name, shape, dtype, device):
        b = self._bufs.get(name)
        if b is None or tuple(b.shape) != tuple(shape) or b.dtype != dtype:
            b = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[name] = b
        return b

    # ---------------------------------------------------------------- buffers
    def _fields(self, tb):
        c = tb.cols
        hw = self.rt.hp * self.engine.blocks[0].head_dim
        f = [("q", hw), ("k", hw), ("v", hw), ("q_raw", hw), ("k_raw", hw)]
        for name in ("sgate", "beta", "ghid"):
            if name in c:
                f.append((name, _pad(c[name][1] - c[name][0], 8)))
        offs, o = {}, 0
        for name, w in f:
            offs[name] = (o, w)
            o += w
        return offs, o

    def _ensure_heaps(self, dev, D, W, kcat, inter, dtype):
        key = (D, W, kcat, inter, self.rt.seq_len)
        if self._heap_key == key:
            return
        self.close()
        rt = self.rt
        C, CS = rt.C, rt.CS
        from vdn_minimax_h3_b200.ops.fp8 import sf_bytes
        tp_specs = [((CS, D), dtype), ((CS, D), torch.uint8), ((sf_bytes(CS, D),), torch.uint8),
                    ((rt.tp, C, D), dtype)]
        self.tp_heap = SymmetricHeap(SymmetricHeap.required_bytes(tp_specs), rt.tp_group, dev)
        self.tp_heap.alloc("a", (CS, D), dtype)
        self.tp_heap.alloc("aq", (CS, D), torch.uint8)
        self.tp_heap.alloc("asf", (sf_bytes(CS, D),), torch.uint8)
        self.tp_heap.alloc("part", (rt.tp, C, D), dtype)
        sp_specs = [((rt.sp, CS, W), dtype), ((CS, kcat), dtype)]
        self.sp_heap = SymmetricHeap(SymmetricHeap.required_bytes(sp_specs), rt.sp_group, dev)
        self.sp_heap.alloc("recv", (rt.sp, CS, W), dtype)
        self.sp_heap.alloc("cat", (CS, kcat), dtype)
        self._heap_key = key
        self._routes.clear()

    def close(self):
        for heap in (self.tp_heap, self.sp_heap):
            if heap is not None:
                heap.barrier()
        torch.cuda.synchronize()
        for heap in (self.tp_heap, self.sp_heap):
            if heap is not None:
                heap.check()
                heap.close()
        self.tp_heap = self.sp_heap = None
        self._heap_key = None

    def _qkv_route(self, tb, offs, rows):
        key = (id(tb), rows)
        route = self._routes.get(key)
        if route is not None:
            return route
        rt = self.rt
        c = tb.cols
        d = self.engine.blocks[0].head_dim
        hw = rt.hp * d
        route = gemm.ColumnRoute(tb.w_qkvg.shape[0], planes=max(2, rt.sp))
        for u in range(rt.sp):
            slab = self.sp_heap.peer("recv", u)[rt.sp_rank, :rows]
            fv = lambda name: slab[:, offs[name][0]:offs[name][0] + offs[name][1]]  # noqa: E731
            route.place(c["q"][0] + u * hw, fv("q_raw"), plane=0)
            route.place(c["q"][0] + u * hw, fv("q"), plane=1)
            route.place(c["k"][0] + u * hw, fv("k_raw"), plane=0)
            route.place(c["k"][0] + u * hw, fv("k"), plane=1)
            route.place(c["v"][0] + u * hw, fv("v"), plane=0)
            for name in ("sgate", "beta", "ghid"):
                if name in offs:
                    lo, hi = c[name]
                    route.place(lo, slab[:, offs[name][0]:offs[name][0] + _pad(hi - lo, 8)], plane=u)
        self._routes[key] = route
        return route

    # ------------------------------------------------------------------ pieces
    def _norm_allgather(self, x, w, eps, table, shift, scale, idx, bf16_copy):
        """AdaLN norm of the own rows into both TP ranks' operand buffers."""
        rt, heap = self.rt, self.tp_heap
        peers = [r for r in range(rt.tp)]
        outs = [heap.peer("a", r) for r in peers] if bf16_copy else []
        qs = [heap.peer("aq", r) for r in peers] if self.fp8 else []
        sfs = [heap.peer("asf", r) for r in peers] if self.fp8 else []
        if rt.tp > 2:
            raise NotImplementedError("the producer-side all-gather covers TP pairs (tp=2)")
        if x.shape[0]:
            ext().adaln_rmsnorm_dst(x, w, float(eps), table, int(shift), int(scale), idx,
                                    rt.tp_rank * rt.C, outs, qs, sfs)
        heap.barrier()

    def _row_parallel(self, a, a_q, a_sf, w, w8, rows):
        """Partial products of the shard rows stored into their TP owners' partial slots."""
        rt, heap = self.rt, self.tp_heap
        bases = [heap.peer("part", r)[rt.tp_rank].data_ptr() for r in range(rt.tp)]
        tmpl = heap.local("part")[rt.tp_rank]
        if rows:
            if self.fp8:
                ext().gemm_f32_scatter(a_q, w8.q, a_sf, w8.sf, tmpl, bases, 0, rt.C,
                                       error_word(a_q.device))
            else:
                ext().gemm_f32_scatter(a, w, None, None, tmpl, bases, 0, rt.C, error_word(a.device))
        heap.barrier()

    def _combine(self, x, bias, gate, idx):
        part = self.tp_heap.local("part")
        if x.shape[0]:
            b = None if bias is None else bias.float().contiguous()
            if self.rt.tp == 1:
                raise NotImplementedError
            ext().residual_combine(x, part[0], part[1], b, gate, idx)

    # ------------------------------------------------------------------- block
    def block_forward(self, i, x, temb_act, adaln_idx, rope, rope_shard, layout):
        eng, rt = self.engine, self.rt
        pb, tb = eng.blocks[i], self.tblocks[i]
        attn = self.model.transformer_blocks[i].attn
        sec = rt.timer.section
        T, D = rt.seq_len, x.shape[1]
        d = pb.head_dim
        H = pb.heads
        hp = rt.hp
        hw = hp * d
        dev = x.device
        hybrid_on = pb.hybrid and not attn.teacher_mode and layout is not None
        plan = eng._plans(attn if hybrid_on else None, layout, T)
        linear_on = hybrid_on and attn.linear_attention_enabled and not eng.covered
        with sec("adaln_table"):
            table = gemm.linear(temb_act, pb.adaln_w, pb.adaln_b).view(-1, 6 * D)
        offs, W = self._fields(tb)
        kcat = tb.w_o.shape[1]
        self._ensure_heaps(dev, D, W, 2 * rt.heads_tp * d, tb.w_up.shape[0] // 2, x.dtype)
        tp_heap, sp_heap = self.tp_heap, self.sp_heap
        rows_s = rt.shard_rows
        # ---- norm1, all-gathered inside the TP pair by its producer
        with sec("norm"):
            self._norm_allgather(x, pb.norm1, pb.eps, table, 0, D, adaln_idx,
                                 bf16_copy=linear_on or not self.fp8)
        work = None
        if linear_on:
            own = tp_heap.local("a")[rt.tp_rank * rt.C:rt.tp_rank * rt.C + rt.rows]
            fsum = norm_ops.frame_sums(own, layout.num_frames, layout.tokens_per_frame, rt.row0,
                                       layout.video_start)
            work = dist.all_reduce(fsum, async_op=True)
        # ---- QKV (column-parallel) routed into the Ulysses slabs
        cos, sin = rope_shard
        route = self._qkv_route(tb, offs, rows_s)
        c = tb.cols
        with sec("gemm_qkv"):
            if rows_s:
                if self.fp8:
                    from vdn_minimax_h3_b200.ops import fp8 as fp8_ops
                    fp8_ops.linear_routed_fp8(tp_heap.local("aq")[:rows_s], tp_heap.local("asf"),
                                              tb.w8_qkvg, route, c["q"], c["k"], pb.norm_q,
                                              pb.norm_k, pb.qk_eps, cos, sin)
                else:
                    gemm.linear_routed(tp_heap.local("a")[:rows_s], tb.w_qkvg, tb.b_qkvg, route,
                                       c["q"], c["k"], pb.norm_q, pb.norm_k, pb.qk_eps, cos, sin)
        with sec("a2a_dispatch"):
            sp_heap.barrier()
        recv = sp_heap.local("recv")
        full = recv.view(rt.sp * rt.CS, W)[:T]
        fv = lambda name, a=0, n=None: full[:, offs[name][0] + a:offs[name][0] + a + (  # noqa: E731
            offs[name][1] if n is None else n)]
        u = rt.tp_rank  # placeholder to keep names short below
        del u
        su = rt.sp_rank  # this rank's position in its Ulysses group
        sg = fv("sgate", su * hp, hp) if "sgate" in offs else None
        bt = fv("beta", su * hp, hp) if "beta" in offs else None
        gh = fv("ghid", 0, c["ghid"][1] - c["ghid"][0]) if "ghid" in offs else None
        cat_peers = [sp_heap.peer("cat", r) for r in range(rt.sp)]
        cat_local = sp_heap.local("cat")
        scat = lambda col, row0: ([t.data_ptr() + 2 * col for t in cat_peers], row0, rt.CS)  # noqa: E731
        head0 = rt.tp_rank * rt.heads_tp + su * hp      # global head index of this rank's slice
        with sec("attention"):
            attn_ops.window_attention(fv("q").view(T, hp, d), fv("k").view(T, hp, d),
                                      fv("v").view(T, hp, d), plan, d ** -0.5, gate_logits=sg,
                                      out=cat_local[:, su * hw:(su + 1) * hw],
                                      scatter=scat(su * hw, 0))
        if pb.hybrid:
            if linear_on:
                work.wait()
                lin_col = rt.heads_tp * d + su * hw
                with sec("linear_branch"):
                    linear_branch_core(pb, attn, layout, eng.bounds, fv("q_raw").view(T, hp, d),
                                       fv("k_raw").view(T, hp, d), fv("v").view(T, hp, d), bt, gh,
                                       fsum, slice(head0, head0 + hp),
                                       cat_local[:, lin_col:lin_col + hw], x.dtype,
                                       scatter=scat(lin_col, None))
            else:
                cat_local[:rows_s, rt.heads_tp * d:].zero_()
        with sec("a2a_return"):
            sp_heap.barrier()
        cat = cat_local[:rows_s, :kcat]
        # ---- O-projection (row-parallel) -> partial-sum scatter -> combine
        with sec("gemm_o"):
            cq = csf = None
            if self.fp8:
                from vdn_minimax_h3_b200.ops import fp8 as fp8_ops
                cq = self._buf("cat_q", (rt.CS, kcat), torch.uint8, dev)[:rows_s]
                csf = self._buf("cat_sf", (fp8_ops.sf_bytes(rt.CS, kcat),), torch.uint8, dev)
                if rows_s:
                    fp8_ops.quantize_act(cat, cq, csf)
            self._row_parallel(cat, cq, csf, tb.w_o, getattr(tb, "w8_o", None), rows_s)
            self._combine(x, tb.b_o, table[:, 2 * D:3 * D], adaln_idx)
        # ---- FF: norm2 all-gather -> SwiGLU (column-parallel) -> down (row-parallel)
        with sec("norm"):
            self._norm_allgather(x, pb.norm2, pb.eps, table, 3 * D, 4 * D, adaln_idx,
                                 bf16_copy=not self.fp8)
        inter_t = tb.w_up.shape[0] // 2
        with sec("gemm_ff_up"):
            if self.fp8:
                from vdn_minimax_h3_b200.ops import fp8 as fp8_ops
                hq = self._buf("h_q", (rt.CS, inter_t), torch.uint8, dev)[:rows_s]
                hsf = self._buf("h_sf", (fp8_ops.sf_bytes(rt.CS, inter_t),), torch.uint8, dev)
                h = None
                if rows_s:
                    fp8_ops.linear_fp8_swiglu(tp_heap.local("aq")[:rows_s], tp_heap.local("asf"),
                                              tb.w8_up, hq, hsf)
            else:
                hq = hsf = None
                h = gemm.linear_swiglu(tp_heap.local("a")[:rows_s], tb.w_up, tb.b_up) if rows_s else None
        with sec("gemm_ff_down"):
            self._row_parallel(h, hq, hsf, tb.w_down, getattr(tb, "w8_down", None), rows_s)
            self._combine(x, tb.b_down, table[:, 5 * D:6 * D], adaln_idx)
        return x

    # ----------------------------------------------------------------- forward
    @torch.no_grad()
    def forward(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
                timestep_indices, token_tags, position_ids, video_indices, audio_indices,
                text_indices, layout=None, return_dict=False):
        m, rt = self.model, self.rt
        T = position_ids.shape[0]
        rt.configure(T, m.config.num_attention_heads)
        for pb in self.engine.blocks:
            if not fused_qk_ok(pb, torch.empty(0, 128, device="cuda")):
                raise NotImplementedError("TP x Ulysses needs 128-wide heads on 128-column boundaries")
        packed, temb, adaln_idx, rope = m.embed(
            hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
            timestep_indices, token_tags, position_ids, video_indices, audio_indices, text_indices)
        if layout is None:
            from vdn_minimax_h3_b200.models.hybrid_attention import HybridAttention
            first = next((b.attn for b in m.transformer_blocks if isinstance(b.attn, HybridAttention)), None)
            layout = None if first is None else first.layout
        a, b = rt.row0, rt.row0 + rt.rows
        x = packed[0, a:b].contiguous()
        idx = adaln_idx[a:b].to(torch.int32).contiguous()
        s0, s1 = rt.shard0, rt.shard0 + rt.shard_rows
        rope_shard = (rope[0][s0:s1].contiguous(), rope[1][s0:s1].contiguous())
        temb_act = torch.nn.functional.silu(temb.float()).to(x.dtype).contiguous()
        for i in range(len(self.engine.blocks)):
            self.block_forward(i, x, temb_act, idx, rope, rope_shard, layout)
        # N6: the head on this rank's own video / audio rows, outputs gathered
        bounds = [(min(T, p * rt.C), min(T, (p + 1) * rt.C)) for p in range(rt.world)]
        with rt.timer.section("head"):
            return self.head(m, x, bounds, rt.rank, temb, timestep_indices, video_indices,
                             audio_indices)

    __call__ = forward
