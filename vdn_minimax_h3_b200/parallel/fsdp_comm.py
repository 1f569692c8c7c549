"""FSDP2 gradient reduce-scatter and parameter all-gather over symmetric memory instead of
NCCL.

FSDP2 (torch.distributed.fsdp.fully_shard) lets a module replace its reduce-scatter with a
`ReduceScatter` comm object that also allocates the buffers. `SymmetricReduceScatter`
hands FSDP its reduce-scatter INPUT buffers from a ring of slots in a symmetric heap
(parallel/symmetric.py: every rank's copy mapped into every other rank), so FSDP's gradient
copy-in writes straight into memory the peers can read. The reduce-scatter itself is then
one kernel per rank (csrc/symmetric.cu: symm_reduce_scatter): the owner of shard r reads
shard r of every rank's input over NVLink, sums in fp32 and applies the op's scale (1/P for
AVG) as it stores -- no NCCL, no intermediate buffer -- between two device flag barriers
(the first makes every rank's copy-in visible, the second keeps a rank from reusing its slot
while peers still read it). It runs on FSDP's reduce-scatter stream, so it overlaps the
backward of the next block like the NCCL call it replaces.

`SymmetricAllGather` is the parameter all-gather: FSDP keeps its own output buffer (its
copy-in already put this rank's shard at the rank's slice); the comm copies that shard into
a slot of a symmetric heap, passes one device flag barrier, and one kernel
(csrc/symmetric.cu: symm_all_gather) pulls every peer's shard over NVLink into the output,
all on FSDP's all-gather stream. Two slots suffice without a closing barrier: a rank writes
slot k again only after passing the barrier of the gather after k, which every rank reaches
only once its pull of gather k is done (stream order).

Reference: the implicit all-gather / reduce-scatter of FSDP2 in
src/training/fsdp_stage.py:392-451 (NCCL). What is NOT done here: the all-gather fused into
the first consuming GEMM (the gathered parameters still land in FSDP's unsharded buffer).

A slot is reused only after the event recorded behind its closing barrier, waited on by the
stream that allocates it again. Anything the kernel does not take (non-fp32 dtype, an op
other than SUM / AVG, a bucket larger than a slot, misaligned shard sizes, CPU tensors)
falls back to torch.distributed.reduce_scatter_tensor.
"""
import math

import torch
import torch.distributed as dist
from torch.distributed.fsdp._fully_shard._fsdp_collectives import AllGather, ReduceScatter


class SymmetricReduceScatter(ReduceScatter):
    def __init__(self, group, device, slot_numel, slots=4):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.slots = slots
        self.slot_numel = int(math.ceil(slot_numel / 64) * 64)
        self.heap = None
        self._events = [None] * slots
        self._next = 0
        self._slot_of = {}            # data_ptr of a handed-out input -> slot
        self._expect_output = False
        self._srcs = {}
        self.calls = self.fallbacks = 0
        if self.enabled():
            from vdn_minimax_h3_b200.parallel.symmetric import SymmetricHeap
            specs = [((self.slot_numel,), torch.float32)] * slots
            # ranks meet here once per unit per backward; a long limit, still bounded
            self.heap = SymmetricHeap(SymmetricHeap.required_bytes(specs), group, self.device,
                                      timeout_s=120.0)
            for i in range(slots):
                self.heap.alloc(f"rs{i}", (self.slot_numel,), torch.float32)

    def enabled(self):
        return self.device.type == "cuda" and 1 < self.world <= 8 and self.slot_numel > 0

    # FSDP calls allocate exactly twice per reduce-scatter: the input (compute stream), then
    # the output (reduce-scatter stream); only inputs ever live in a slot.
    def allocate(self, size, *, dtype, device):
        numel = math.prod(int(s) for s in size)
        is_output, self._expect_output = self._expect_output, not self._expect_output
        if is_output or self.heap is None or dtype != torch.float32 or \
                numel > self.slot_numel or numel % (4 * self.world):
            return torch.empty(*size, dtype=dtype, device=device)
        slot = self._next
        self._next = (self._next + 1) % self.slots
        if self._events[slot] is not None:
            torch.cuda.current_stream(device).wait_event(self._events[slot])
        buf = self.heap.local(f"rs{slot}")[:numel].view(*size)
        self._slot_of[buf.data_ptr()] = slot
        return buf

    def _same_group(self, group):
        if group is self.group:
            return True
        return dist.get_process_group_ranks(group) == dist.get_process_group_ranks(self.group)

    def close(self):
        if self.heap is not None:
            torch.cuda.synchronize(self.device)
            self.heap.check()
            self.heap.close()
            self.heap = None

    def __call__(self, output_tensor, input_tensor, group, op, async_op=False):
        slot = self._slot_of.pop(input_tensor.data_ptr(), None)
        scale = {dist.ReduceOp.SUM: 1.0, dist.ReduceOp.AVG: 1.0 / self.world}.get(op)
        if (slot is None or scale is None or not self._same_group(group) or async_op
                or output_tensor.dtype != torch.float32 or not output_tensor.is_contiguous()):
            self.fallbacks += 1
            return dist.reduce_scatter_tensor(output_tensor, input_tensor, group=group, op=op,
                                              async_op=async_op)
        from vdn_minimax_h3_b200.ops._ext import ext
        srcs = self._srcs.get(slot)
        if srcs is None:
            srcs = self._srcs[slot] = [self.heap.peer(f"rs{slot}", p).data_ptr()
                                       for p in range(self.world)]
        n = output_tensor.numel()
        self.heap.barrier()                      # every rank's copy-in is visible
        ext().symm_reduce_scatter(srcs, self.rank * n, output_tensor, scale)
        self.heap.barrier()                      # peers are done reading this rank's slot
        self._events[slot] = torch.cuda.current_stream(self.device).record_event()
        self.calls += 1
        return None


def trainable_reduce_numel(param_groups, world):
    """Largest reduce-scatter input (fp32 elements) FSDP will form for one of the parameter
    groups (one list per fully_shard unit): the dim-0-padded sizes of the parameters that
    take gradients."""
    best = 0
    for params in param_groups:
        total = 0
        for p in params:
            if p.requires_grad:
                d0 = p.shape[0] if p.dim() else 1
                total += math.ceil(d0 / world) * world * (p.numel() // max(d0, 1))
        best = max(best, total)
    return best


class SymmetricAllGather(AllGather):
    """FSDP2 parameter all-gather: shard -> symmetric slot, flag barrier, peer-pull kernel."""

    def __init__(self, group, device, slot_bytes, slots=2):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.slots = max(2, int(slots))
        self.slot_bytes = int(math.ceil(slot_bytes / 256) * 256)
        self.heap = None
        self._next = 0
        self._srcs = {}
        self.calls = self.fallbacks = 0
        if self.enabled():
            from vdn_minimax_h3_b200.parallel.symmetric import SymmetricHeap
            specs = [((self.slot_bytes,), torch.uint8)] * self.slots
            self.heap = SymmetricHeap(SymmetricHeap.required_bytes(specs), group, self.device,
                                      timeout_s=120.0)
            for i in range(self.slots):
                self.heap.alloc(f"ag{i}", (self.slot_bytes,), torch.uint8)

    def enabled(self):
        return self.device.type == "cuda" and 1 < self.world <= 8 and self.slot_bytes > 0

    def allocate(self, size, *, dtype, device):
        return torch.empty(*size, dtype=dtype, device=device)

    def _same_group(self, group):
        if group is self.group:
            return True
        return dist.get_process_group_ranks(group) == dist.get_process_group_ranks(self.group)

    def close(self):
        if self.heap is not None:
            torch.cuda.synchronize(self.device)
            self.heap.check()
            self.heap.close()
            self.heap = None

    def __call__(self, output_tensor, input_tensor, group, async_op=False):
        shard = input_tensor.numel() * input_tensor.element_size()
        in_place = (output_tensor.is_contiguous() and input_tensor.is_contiguous()
                    and output_tensor.numel() == input_tensor.numel() * self.world
                    and input_tensor.data_ptr() == output_tensor.data_ptr() + self.rank * shard)
        if (self.heap is None or async_op or not in_place or not self._same_group(group)
                or shard > self.slot_bytes or output_tensor.data_ptr() % 16):
            self.fallbacks += 1
            return dist.all_gather_into_tensor(output_tensor, input_tensor, group=group,
                                               async_op=async_op)
        from vdn_minimax_h3_b200.ops._ext import ext
        slot = self._next
        self._next = (self._next + 1) % self.slots
        local = self.heap.local(f"ag{slot}")[:shard]
        local.copy_(input_tensor.view(-1).view(torch.uint8))
        srcs = self._srcs.get(slot)
        if srcs is None:
            srcs = self._srcs[slot] = [self.heap.peer(f"ag{slot}", p).data_ptr()
                                       for p in range(self.world)]
        self.heap.barrier()                      # every rank's shard is in its slot
        ext().symm_all_gather(srcs, self.rank, output_tensor, shard)
        self.calls += 1
        return None


def gather_shard_bytes(param_groups, world, elem_bytes=4):
    """Largest per-rank all-gather shard (bytes) FSDP will form for one of the parameter
    groups: the dim-0-padded shard of every parameter, at `elem_bytes` per element (an upper
    bound for the bf16 / fp32 mixed-precision gathers)."""
    best = 0
    for params in param_groups:
        total = 0
        for p in params:
            d0 = p.shape[0] if p.dim() else 1
            total += math.ceil(d0 / world) * (p.numel() // max(d0, 1))
        best = max(best, total * elem_bytes)
    return best
