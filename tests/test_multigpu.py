"""Ulysses on 2 GPUs (NCCL): the sequence-parallel engine equals the single-GPU engine on a
reduced geometry with head_dim 128 and the released transform. Skipped with < 2 GPUs."""
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


def _worker(rank, world, port, q):
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
        cfg = H3Config(hidden_size=256, num_layers=2, num_attention_heads=4, attention_head_dim=128,
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
            sp = UlyssesEngine(InferenceEngine(gm), init_ulysses())
            out_v, _ = sp(**kwg, layout=layout)
        torch.cuda.synchronize()
        check_device_error()
        err = ((out_v.float() - ref_v.float()).norm() / ref_v.float().norm()).item()
        q.put((rank, err))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.timeout(300)
def test_ulysses_two_gpus_match_single():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=280)
    res = dict(q.get() for _ in range(2))
    assert all(isinstance(v, float) and v < 2e-2 for v in res.values()), res
