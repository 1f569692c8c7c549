"""Symmetric device memory for one node's ranks (CUDA IPC over NVLink / NVSwitch).

Every rank allocates the same layout (a bump allocator over one cudaMalloc'd region, the
same sequence of `alloc` calls on every rank), exports an IPC handle, and maps every peer's
region. `peer(name, r)` is then a tensor view of rank r's copy of buffer `name`, usable as a
store destination by this GPU's kernels: the routed GEMM epilogue, the attention and readout
row scatters. `barrier()` is a device-side flag barrier over the same mapping (one warp,
bounded wait, error word on timeout) that orders the peer stores of all ranks.

This replaces the reference's NCCL all_to_all_single exchanges
(src/inference/utils/ulysses_runtime.py:298-305, 348-355, 407-412, 426-476) with stores
issued by the kernels that produce the data.
"""
import torch
import torch.distributed as dist

from vdn_minimax_h3_b200.ops._ext import check_device_error, error_word, ext

_ALIGN = 256


class SymmetricHeap:
    """One IPC-exported region per rank, mapped into every rank of `group`."""

    def __init__(self, nbytes, group=None, device=None, timeout_s=10.0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("symmetric heaps span at most 8 ranks (one NVLink node)")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.timeout_ns = int(timeout_s * 1e9)
        # flags: world slots written by the peers + one epoch counter, then the data region
        self._flag_bytes = _ALIGN
        self.nbytes = self._flag_bytes + (nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
        dev = self.device.index
        ptr, handle = ext().symm_alloc(self.nbytes, dev)
        self._own = ptr
        handles = [None] * self.world
        dist.all_gather_object(handles, (self.rank, handle), group=group)
        self.ptrs = []
        for r, (src, h) in enumerate(handles):
            assert src == r
            self.ptrs.append(ptr if r == self.rank else ext().symm_open(h, dev))
        self._peer_flags = torch.tensor([p for p in self.ptrs], dtype=torch.int64,
                                        device=self.device)
        self._offset = self._flag_bytes
        self._bufs = {}
        self._closed = False

    # ------------------------------------------------------------------ allocation
    def alloc(self, name, shape, dtype):
        """Reserve `name` (same call order on every rank); returns the local tensor."""
        if name in self._bufs:
            raise ValueError(f"{name} already allocated")
        n = torch.Size(shape).numel() * torch.empty((), dtype=dtype).element_size()
        off = self._offset
        if off + n > self.nbytes:
            raise MemoryError(f"symmetric heap full: {name} needs {n} B at {off} of {self.nbytes}")
        self._offset = off + (n + _ALIGN - 1) // _ALIGN * _ALIGN
        self._bufs[name] = (off, tuple(shape), dtype, n)
        return self.peer(name, self.rank)

    def peer(self, name, rank):
        """Rank `rank`'s copy of buffer `name` as a tensor on this device."""
        off, shape, dtype, n = self._bufs[name]
        raw = ext().bytes_at(self.ptrs[rank] + off, n, self.device.index)
        return raw.view(dtype).view(shape)

    def local(self, name):
        return self.peer(name, self.rank)

    # --------------------------------------------------------------------- barrier
    def barrier(self):
        """All ranks' earlier stores on their current streams (peer stores included) are
        visible everywhere once every rank's barrier kernel returns."""
        flags = self.ptrs[self.rank]
        ext().symm_barrier(flags + 8 * self.world, flags, self._peer_flags, self.rank,
                           self.timeout_ns, error_word(self.device))

    def check(self):
        check_device_error(self.device)

    def close(self):
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                ext().symm_close(p, self.device.index)
        ext().symm_free(self._own, self.device.index)
        self._closed = True

    @staticmethod
    def required_bytes(specs):
        """Heap size for a list of (shape, dtype)."""
        total = 0
        for shape, dtype in specs:
            n = torch.Size(shape).numel() * torch.empty((), dtype=dtype).element_size()
            total += (n + _ALIGN - 1) // _ALIGN * _ALIGN
        return total
