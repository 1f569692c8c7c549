"""The FSDP2 reduce-scatter and all-gather comms on CPU: the reduce-scatter's allocate() hands
out one buffer per call in FSDP's input / output order (only inputs may ever come from a
slot), and set on every fully_shard unit the two comms leave the gradients of 2 gloo ranks
exactly as stock FSDP2 makes them (on CPU every call takes the torch.distributed fallback)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.Tanh(), torch.nn.Linear(32, 8))


def _grads(custom):
    from torch.distributed.fsdp import fully_shard
    from vdn_minimax_h3_b200.parallel.fsdp_comm import SymmetricAllGather, SymmetricReduceScatter
    m = _model()
    fully_shard(m[0])
    fully_shard(m[2])
    fully_shard(m)
    comm = None
    if custom:
        comm = SymmetricReduceScatter(dist.group.WORLD, "cpu", 1024)
        comm.gather = SymmetricAllGather(dist.group.WORLD, "cpu", 4096)
        for u in (m[0], m[2], m):
            u.set_custom_reduce_scatter(comm)
            u.set_custom_all_gather(comm.gather)
    torch.manual_seed(10 + dist.get_rank())
    x = torch.randn(5, 16)
    m(x).square().sum().backward()
    out = {n: p.grad.full_tensor() for n, p in m.named_parameters()}
    return out, comm


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ref, _ = _grads(False)
        got, comm = _grads(True)
        same = all(torch.equal(ref[k], got[k]) for k in ref)
        q.put((rank, same and comm.fallbacks > 0 and not comm.enabled()
               and comm.gather.fallbacks > 0 and not comm.gather.enabled()))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_comm_with_fsdp2_on_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    assert res == {0: True, 1: True}, res


def test_allocate_alternates_input_and_output():
    from vdn_minimax_h3_b200.parallel.fsdp_comm import SymmetricReduceScatter
    c = SymmetricReduceScatter.__new__(SymmetricReduceScatter)
    c.heap, c._expect_output, c.slot_numel, c.world = None, False, 1024, 2
    shapes = []
    for _ in range(3):
        shapes.append(tuple(c.allocate((64,), dtype=torch.float32, device="cpu").shape))
        shapes.append(tuple(c.allocate((32,), dtype=torch.float32, device="cpu").shape))
    assert shapes == [(64,), (32,)] * 3 and c._expect_output is False


def test_shard_sizing_helpers():
    """The slot sizes cover FSDP's dim-0-padded shards: reduce-scatter inputs count only
    parameters that take gradients (fp32 elements), all-gather shards count every parameter
    (bytes at the given element size)."""
    from vdn_minimax_h3_b200.parallel.fsdp_comm import gather_shard_bytes, trainable_reduce_numel
    w = torch.nn.Parameter(torch.zeros(40, 256))          # 40 rows over 3 ranks -> 14 per rank
    b = torch.nn.Parameter(torch.zeros(40))
    frozen = torch.nn.Parameter(torch.zeros(9, 16), requires_grad=False)
    groups = [[w, b, frozen], [torch.nn.Parameter(torch.zeros(8, 8))]]
    assert trainable_reduce_numel(groups, 3) == 14 * 3 * 256 + 14 * 3
    assert gather_shard_bytes(groups, 3, elem_bytes=2) == (14 * 256 + 14 + 3 * 16) * 2
    assert gather_shard_bytes(groups, 3) == (14 * 256 + 14 + 3 * 16) * 4


def test_all_gather_falls_back_when_not_in_place():
    """Without a heap (CPU) or when FSDP's input is not the output's own rank slice, the
    gather goes to torch.distributed and is counted as a fallback."""
    from vdn_minimax_h3_b200.parallel import fsdp_comm
    c = fsdp_comm.SymmetricAllGather.__new__(fsdp_comm.SymmetricAllGather)
    c.heap, c.world, c.rank, c.group, c.slot_bytes = None, 2, 1, None, 1 << 20
    c.calls = c.fallbacks = 0
    seen = []
    orig = fsdp_comm.dist.all_gather_into_tensor
    fsdp_comm.dist.all_gather_into_tensor = lambda out, inp, group=None, async_op=False: seen.append(
        (out.shape, inp.shape)) or None
    try:
        out = torch.zeros(8)
        assert c(out, out[4:], None) is None
        assert c(out, torch.zeros(4), None) is None      # not in place
    finally:
        fsdp_comm.dist.all_gather_into_tensor = orig
    assert c.fallbacks == 2 and c.calls == 0 and len(seen) == 2
    assert c.allocate((3, 5), dtype=torch.bfloat16, device="cpu").shape == (3, 5)
