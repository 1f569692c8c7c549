"""Block-streamed inference: the DiT blocks' weights live in pinned host memory, and each block
comes onto the GPU only while it runs; the next block is copied on a side stream while the
current one computes.

Reference parity: src/inference/infer_diffusers.py:42-63 (`--offload_dit`: diffusers group
offloading at block level, one block per group, `use_stream=True`; "a 24 GB card needs it:
345 frames then peak at 22 GB"). There the unit is a diffusers block; here it is one
InferenceEngine block: its packed weights (`PackedBlock`, fp8 copies included) and its
module's parameters and buffers. Those alias one another (the packed QKV and O weights are
the storage of the module's Linears), so the streamer moves STORAGES, not tensors: every
distinct storage reachable from a block is copied once, and every tensor is re-pointed at a
view of that copy with its own offset, size and strides, so the aliasing survives the trip.
A storage reachable from two blocks (a tied tensor) stays resident.

    engine = InferenceEngine(model, fp8=...)
    enable_block_offload(engine)          # weights to host; engine.block_forward streams

Per block: `acquire(i)` makes block i resident (waits for its prefetch, or copies it now) and
starts the copy of block i+1 (block 0 after the last, for the next model evaluation);
`release(i)` re-points block i at its host copy, which frees its device storage once the
compute stream has passed the block (the storage is recorded on that stream). At most two
blocks' weights are on the device at a time. On a CPU engine the same steps run with plain
copies (that is what the CPU tests exercise).
"""
import torch

from vdn_minimax_h3_b200.ops.fp8 import Fp8Weight


def _refs(pb, module):
    """Every tensor a block's forward reads: PackedBlock attributes (and their Fp8Weight
    parts) and the block module's parameters and buffers."""
    out = []
    for v in vars(pb).values():
        if torch.is_tensor(v):
            out.append(v)
        elif isinstance(v, Fp8Weight):
            out.extend(t for t in (v.q, v.sf, v.bias) if t is not None)
    out.extend(module.parameters())
    out.extend(module.buffers())
    seen, uniq = set(), []
    for t in out:
        if id(t) not in seen:
            seen.add(id(t))
            uniq.append(t)
    return uniq


def _storage_key(t):
    return (t.device.type, t.device.index, t.untyped_storage().data_ptr())


def _view(base, t_meta):
    dtype, offset, size, stride = t_meta
    return torch.empty(0, dtype=dtype, device=base.device).set_(
        base.untyped_storage(), offset, size, stride)


class _Block:
    """One block's storages (host copies) and the tensors that view them."""

    def __init__(self, tensors, shared):
        self.groups = {}          # storage key -> [host uint8 copy, [(tensor, meta)]]
        for t in tensors:
            key = _storage_key(t)
            if key in shared or t.numel() == 0:
                continue
            meta = (t.dtype, t.storage_offset(), tuple(t.shape), tuple(t.stride()))
            g = self.groups.get(key)
            if g is None:
                st = t.untyped_storage()
                flat = torch.empty(0, dtype=torch.uint8, device=t.device).set_(st, 0, (st.nbytes(),))
                host = torch.empty(st.nbytes(), dtype=torch.uint8,
                                   pin_memory=torch.cuda.is_available())
                host.copy_(flat)
                g = self.groups[key] = [host, []]
            g[1].append((t, meta))
        self.event = None
        self.resident = False

    def nbytes(self):
        return sum(g[0].numel() for g in self.groups.values())

    def bind_host(self):
        for host, members in self.groups.values():
            for t, meta in members:
                t.data = _view(host, meta)
        self.resident = False

    def bind_device(self, device, copy_stream, compute_stream):
        """Copy every storage to `device` (on `copy_stream` when given) and re-point the
        tensors; returns after queueing the copies."""
        for host, members in self.groups.values():
            dev = torch.empty(host.numel(), dtype=torch.uint8, device=device)
            if copy_stream is not None:
                dev.record_stream(compute_stream)   # freed only after the compute stream's use
                dev.copy_(host, non_blocking=True)
            else:
                dev.copy_(host)
            for t, meta in members:
                t.data = _view(dev, meta)
        self.resident = True


class BlockStreamer:
    """Keeps a sequence of blocks' weights on the host and streams them per block.
    `per_block[i]` lists every tensor block i reads."""

    def __init__(self, per_block, device):
        self.device = torch.device(device)
        owners = {}
        for i, ts in enumerate(per_block):
            for t in ts:
                owners.setdefault(_storage_key(t), set()).add(i)
        shared = {k for k, v in owners.items() if len(v) > 1}
        self.blocks = [_Block(ts, shared) for ts in per_block]
        for b in self.blocks:
            b.bind_host()
        cuda = self.device.type == "cuda"
        self.copy_stream = torch.cuda.Stream(self.device) if cuda else None
        if cuda:
            torch.cuda.empty_cache()

    def host_bytes(self):
        return sum(b.nbytes() for b in self.blocks)

    def _compute_stream(self):
        return torch.cuda.current_stream(self.device) if self.copy_stream is not None else None

    def _prefetch(self, i):
        b = self.blocks[i]
        if b.resident:
            return
        if self.copy_stream is None:
            b.bind_device(self.device, None, None)
            return
        compute = self._compute_stream()
        self.copy_stream.wait_stream(compute)     # its previous use of the memory is done
        with torch.cuda.stream(self.copy_stream):
            b.bind_device(self.device, self.copy_stream, compute)
            b.event = torch.cuda.Event()
            b.event.record(self.copy_stream)

    def acquire(self, i):
        b = self.blocks[i]
        if not b.resident:
            self._prefetch(i)
        if b.event is not None:
            self._compute_stream().wait_event(b.event)
            b.event = None
        n = len(self.blocks)
        if n > 1:
            self._prefetch((i + 1) % n)

    def release(self, i):
        self.blocks[i].bind_host()


def enable_block_offload(engine, device=None):
    """Stream `engine`'s DiT blocks from pinned host memory (see the module docstring).
    Returns the BlockStreamer; `engine.block_forward` is wrapped on this instance only."""
    if getattr(engine, "offload", None) is not None:
        return engine.offload
    if device is None:
        device = engine.blocks[0].w_qkvg.device
    per_block = [_refs(engine.blocks[i], engine.model.transformer_blocks[i])
                 for i in range(len(engine.blocks))]
    streamer = BlockStreamer(per_block, device)
    engine.offload = streamer
    engine.compute_device = torch.device(device)
    resident_forward = engine.block_forward

    def block_forward(i, *args, **kwargs):
        streamer.acquire(i)
        try:
            return resident_forward(i, *args, **kwargs)
        finally:
            streamer.release(i)

    engine.block_forward = block_forward
    return streamer


def enable_module_offload(model, device):
    """Stream an eager H3Transformer's DiT blocks (its `transformer_blocks`, parameters and
    buffers) from pinned host memory through forward hooks, the same way as
    `enable_block_offload` does for the fused engine; everything outside the blocks must
    already be on `device`. Returns the BlockStreamer (also `model._vdn_offload`)."""
    if getattr(model, "_vdn_offload", None) is not None:
        return model._vdn_offload
    blocks = list(model.transformer_blocks)
    per_block = []
    for blk in blocks:
        seen, ts = set(), []
        for t in list(blk.parameters()) + list(blk.buffers()):
            if id(t) not in seen:
                seen.add(id(t))
                ts.append(t)
        per_block.append(ts)
    streamer = BlockStreamer(per_block, device)
    for i, blk in enumerate(blocks):
        blk.register_forward_pre_hook(lambda mod, args, i=i: streamer.acquire(i))
        blk.register_forward_hook(lambda mod, args, out, i=i: streamer.release(i))
    model._vdn_offload = streamer
    return streamer
