"""Ulysses on 2 GPUs: the sequence-parallel engine (NCCL all-to-all, or the symmetric-memory
exchange fused into the producing kernels) equals the single-GPU engine on a reduced geometry
with head_dim 128 and the released transform; the symmetric heap moves bytes between ranks.
Each rank is its own process on its own GPU. Skipped with < 2 GPUs."""
import copy
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, exchange, softmax_ranks=0):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from tests.test_model_cpu import _forward_inputs, tiny_model
        from vdn_minimax_h3_b200.inference.engine import InferenceEngine
        from vdn_minimax_h3_b200.inference.render import render_geometry
        from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID
        from vdn_minimax_h3_b200.models.h3 import H3Config
        from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
        from vdn_minimax_h3_b200.ops._ext import check_device_error
        from vdn_minimax_h3_b200.parallel.ulysses import UlyssesEngine, init_ulysses
        cfg = H3Config(hidden_size=256, num_layers=2, num_attention_heads=max(4, world),
                       attention_head_dim=128,
                       in_channels=8, text_dim=96, time_embed_dim=64, time_freq_dim=32,
                       ff_inner_dim=512, num_refiner_layers=1, rope_axes_dim=(32, 48, 48))
        model = tiny_model(RELEASED_HYBRID, cfg)
        geo = render_geometry(cfg, 5, latent_h=8, latent_w=12, audio=True, num_latent_frames=17)
        geo.num_audio_latents = 6
        kw, layout = _forward_inputs(cfg, geo, 24)
        gm = model.to(device=dev, dtype=torch.bfloat16)
        gm.time_embedder.float()
        for blk in gm.transformer_blocks:
            blk.attn.linear_attention.alpha.float()
        set_layout(gm, layout)
        kwg = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in kw.items()}
        with torch.no_grad():
            single = InferenceEngine(copy.deepcopy(gm))
            ref_v, _ = single(**kwg, layout=layout)
            sp = UlyssesEngine(InferenceEngine(gm), init_ulysses(softmax_ranks=softmax_ranks),
                               exchange=exchange)
            out_v, _ = sp(**kwg, layout=layout)
            out_v2, _ = sp(**kwg, layout=layout)
            sp.close()
        torch.cuda.synchronize()
        check_device_error()
        err = ((out_v.float() - ref_v.float()).norm() / ref_v.float().norm()).item()
        if not torch.equal(out_v, out_v2):
            err = "second forward differs from the first"
        q.put((rank, err))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def _heap_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from vdn_minimax_h3_b200.parallel.symmetric import SymmetricHeap
        heap = SymmetricHeap(1 << 20, device=dev, timeout_s=20.0)
        buf = heap.alloc("x", (world, 1000), torch.float32)
        for it in range(3):
            for p in range(world):   # write my row into every rank's copy
                heap.peer("x", p)[rank].fill_(100 * it + rank)
            heap.barrier()
            torch.cuda.synchronize()
            want = torch.tensor([100 * it + r for r in range(world)], dtype=torch.float32, device=dev)
            ok = torch.equal(buf[:, 0], want) and torch.equal(buf[:, -1], want)
            heap.barrier()   # nobody overwrites before everyone has read
            if not ok:
                break
        heap.check()
        heap.close()
        q.put((rank, ok))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def _spawn(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=280)
    return dict(q.get(timeout=10) for _ in range(world))


TWO_GPUS = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                              reason="needs 2 GPUs")


@TWO_GPUS
@pytest.mark.timeout(300)
def test_symmetric_heap_two_gpus():
    res = _spawn(_heap_worker, 2)
    assert all(v is True for v in res.values()), res


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,exchange,softmax_ranks", [
    (2, "nccl", 0), (2, "p2p", 0), (2, "nccl", 1), (2, "p2p", 1), (4, "p2p", 3), (4, "nccl", 1),
    (8, "p2p", 0), (8, "p2p", 5), (8, "nccl", 5)])
def test_ulysses_match_single(world, exchange, softmax_ranks):
    """Plain Ulysses (softmax_ranks 0) and branch parallel: with 4 heads on 4 GPUs,
    3 softmax ranks hold 2 + 1 + 1 heads and 1 linear rank all 4 (uneven splits); on 8 GPUs
    (8 heads) the shipped B200 layout 5 + 3 (softmax heads 2,2,2,1,1; linear 3,3,2)."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _spawn(_worker, world, exchange, softmax_ranks)
    assert all(isinstance(v, float) and v < 2e-2 for v in res.values()), res


def _hybrid_worker(rank, world, port, q, tp, fp8):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from tests.test_model_cpu import _forward_inputs, tiny_model
        from vdn_minimax_h3_b200.inference.engine import InferenceEngine
        from vdn_minimax_h3_b200.inference.render import render_geometry
        from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID
        from vdn_minimax_h3_b200.models.h3 import H3Config
        from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
        from vdn_minimax_h3_b200.ops._ext import check_device_error
        from vdn_minimax_h3_b200.parallel.hybrid import HybridEngine, HybridRuntime
        cfg = H3Config(hidden_size=512, num_layers=2, num_attention_heads=8, attention_head_dim=128,
                       in_channels=8, text_dim=96, time_embed_dim=64, time_freq_dim=32,
                       ff_inner_dim=1024, num_refiner_layers=1, rope_axes_dim=(32, 48, 48))
        model = tiny_model(RELEASED_HYBRID, cfg)
        geo = render_geometry(cfg, 5, latent_h=8, latent_w=12, audio=True, num_latent_frames=17)
        geo.num_audio_latents = 6
        kw, layout = _forward_inputs(cfg, geo, 24)
        gm = model.to(device=dev, dtype=torch.bfloat16)
        gm.time_embedder.float()
        for blk in gm.transformer_blocks:
            blk.attn.linear_attention.alpha.float()
        set_layout(gm, layout)
        kwg = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in kw.items()}
        with torch.no_grad():
            single = InferenceEngine(copy.deepcopy(gm), fp8=fp8)
            ref_v, _ = single(**kwg, layout=layout)
            hp = HybridEngine(InferenceEngine(gm, fp8=fp8), HybridRuntime(tp), fp8=fp8)
            out_v, _ = hp(**kwg, layout=layout)
            out_v2, _ = hp(**kwg, layout=layout)
            hp.close()
        torch.cuda.synchronize()
        check_device_error()
        err = ((out_v.float() - ref_v.float()).norm() / ref_v.float().norm()).item()
        if not torch.equal(out_v, out_v2):
            err = "second forward differs from the first"
        q.put((rank, err))
    except Exception as exc:  # noqa: BLE001
        import traceback
        q.put((rank, repr(exc) + traceback.format_exc()[-1500:]))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,tp,fp8", [(2, 2, False), (2, 2, True), (4, 2, True), (8, 2, True)])
def test_tp_ulysses_match_single(world, tp, fp8):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _spawn(_hybrid_worker, world, tp, fp8)
    tol = 4e-2 if fp8 else 2e-2
    assert all(isinstance(v, float) and v < tol for v in res.values()), res


def _fsdp_comm_worker(rank, world, port, q, gather):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard
        from vdn_minimax_h3_b200.ops._ext import check_device_error
        from vdn_minimax_h3_b200.parallel.fsdp_comm import (SymmetricAllGather, SymmetricReduceScatter,
                                                            gather_shard_bytes, trainable_reduce_numel)

        def grads(custom, steps=3):
            torch.manual_seed(0)
            m = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(),
                                    torch.nn.Linear(512, 256), torch.nn.GELU(),
                                    torch.nn.Linear(256, 40)).to(dev)
            mp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32) \
                if gather else None
            kw = {"mp_policy": mp} if mp is not None else {}
            for i in (0, 2, 4):
                fully_shard(m[i], **kw)
            fully_shard(m, **kw)
            comms = []
            if custom:
                groups = [list(m[i].parameters()) for i in (0, 2, 4)]
                rs = SymmetricReduceScatter(dist.group.WORLD, dev,
                                            trainable_reduce_numel(groups, world), slots=2)
                comms.append(rs)
                for u in (m[0], m[2], m[4], m):
                    u.set_custom_reduce_scatter(rs)
                if gather:
                    ag = SymmetricAllGather(dist.group.WORLD, dev, gather_shard_bytes(groups, world))
                    comms.append(ag)
                    for u in (m[0], m[2], m[4], m):
                        u.set_custom_all_gather(ag)
            out = []
            for s in range(steps):     # more steps than slots: the slot rings are reused
                torch.manual_seed(100 * s + rank)
                loss = m(torch.randn(64, 256, device=dev)).float().square().mean()
                loss.backward()
                g = {n: p.grad.full_tensor().clone() for n, p in m.named_parameters()}
                g["loss"] = loss.detach().reshape(1)
                out.append(g)
                m.zero_grad(set_to_none=True)
            torch.cuda.synchronize()
            return out, comms

        ref, _ = grads(False)
        got, comms = grads(True)
        check_device_error()
        err = max(((a[k] - b[k]).norm() / b[k].norm()).item() for a, b in zip(got, ref) for k in b)
        bad = [f"{type(c).__name__} calls {c.calls} fallbacks {c.fallbacks}" for c in comms
               if c.calls == 0 or c.fallbacks]
        res = err if not bad else f"err {err}; " + "; ".join(bad)
        for c in comms:
            c.close()
        q.put((rank, res))
    except Exception as exc:  # noqa: BLE001
        import traceback
        q.put((rank, repr(exc) + traceback.format_exc()[-1500:]))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
def test_fsdp_symmetric_reduce_scatter(world):
    """FSDP2 with its gradient reduce-scatter over symmetric memory (the owner pulls its shard
    from every rank and sums; parallel/fsdp_comm.py) gives the stock NCCL gradients, over
    three backward passes that reuse the slot ring."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _spawn(_fsdp_rs_worker, world)
    assert all(isinstance(v, float) and v < 1e-5 for v in res.values()), res


def _fsdp_rs_worker(rank, world, port, q):
    _fsdp_comm_worker(rank, world, port, q, gather=False)


def _fsdp_ag_worker(rank, world, port, q):
    _fsdp_comm_worker(rank, world, port, q, gather=True)


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
def test_fsdp_symmetric_all_gather(world):
    """FSDP2 (bf16 parameters) with both its parameter all-gather (shard -> symmetric slot,
    flag barrier, peer-pull kernel) and its gradient reduce-scatter over symmetric memory
    gives the stock NCCL losses and gradients -- the gather moves bytes, so they match
    exactly -- over three steps that reuse both slot rings."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _spawn(_fsdp_ag_worker, world)
    assert all(isinstance(v, float) and v < 1e-5 for v in res.values()), res
