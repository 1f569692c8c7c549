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
