"""Ulysses sequence parallelism on CPU ranks (gloo, world 2): the sharded engine forward
equals the single-process engine forward, and the split helpers match the reference's rules."""
import copy
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vdn_minimax_h3_b200.parallel.ulysses import balanced_splits, sequence_splits


def test_sequence_splits():
    assert sequence_splits(10, 1) == (10,)
    assert sequence_splits(104766, 8) == (13096,) * 7 + (104766 - 7 * 13096,)
    assert sum(sequence_splits(17, 5)) == 17
    assert balanced_splits(56, 3) == (19, 19, 18)
    with pytest.raises(ValueError):
        balanced_splits(2, 3)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q, softmax_ranks=0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tests.test_model_cpu import _forward_inputs, tiny_model
        from vdn_minimax_h3_b200.inference.engine import InferenceEngine
        from vdn_minimax_h3_b200.inference.render import render_geometry
        from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID
        from vdn_minimax_h3_b200.models.h3 import H3Config
        from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
        from vdn_minimax_h3_b200.parallel.ulysses import UlyssesEngine, init_ulysses
        cfg = H3Config(hidden_size=128, num_layers=2, num_attention_heads=2, attention_head_dim=64,
                       in_channels=8, text_dim=96, time_embed_dim=64, time_freq_dim=32,
                       ff_inner_dim=256, num_refiner_layers=1, rope_axes_dim=(16, 24, 24))
        model = tiny_model(RELEASED_HYBRID, cfg)
        geo = render_geometry(cfg, 5, latent_h=8, latent_w=12, audio=True, num_latent_frames=17)
        geo.num_audio_latents = 6
        kw, layout = _forward_inputs(cfg, geo, 11)
        set_layout(model, layout)
        with torch.no_grad():
            ref_v, ref_a = InferenceEngine(copy.deepcopy(model))(**kw, layout=layout)
            eng = UlyssesEngine(InferenceEngine(model), init_ulysses(softmax_ranks=softmax_ranks))
            out_v, out_a = eng(**kw, layout=layout)
        err = max(((out_v - ref_v).norm() / ref_v.norm()).item(),
                  ((out_a - ref_a).norm() / ref_a.norm()).item())
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,softmax_ranks", [(2, 0), (2, 1), (3, 1), (3, 2)])
def test_ulysses_matches_single_process(world, softmax_ranks):
    """softmax_ranks = 0 is plain Ulysses; otherwise branch parallel, with uneven head
    splits at world 3 (1 softmax rank with 2 heads + 2 linear ranks with 1 head each, and
    2 + 1)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, softmax_ranks))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=280)
    results = {}
    while not q.empty():
        r, e = q.get()
        results[r] = e
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert len(results) == world
    assert max(results.values()) < 1e-4, results


def test_sharded_head_plan_cache_follows_the_tensor():
    """The head's row cuts are cached per index tensor: the same tensor hits the cache, an
    in-place change or a new tensor with other rows (even one of the same size) is re-cut."""
    import torch
    from vdn_minimax_h3_b200.parallel.head import ShardedHead
    head = ShardedHead()
    bounds = [(0, 10), (10, 20), (20, 30)]
    a = torch.tensor([2, 3, 11, 12, 13, 25])
    assert head._plan(a, bounds) == [(0, 2), (2, 5), (5, 6)]
    assert head._plan(a, bounds) is head._plan(a, bounds)
    a[2:] = torch.tensor([21, 22, 23, 24])                  # in place: version changes
    assert head._plan(a, bounds) == [(0, 2), (2, 2), (2, 6)]
    del a
    b = torch.tensor([0, 1, 2, 3, 4, 29])                   # same size, other rows
    assert head._plan(b, bounds) == [(0, 5), (5, 5), (5, 6)]
    assert head._plan(b, [(0, 3), (3, 30)]) == [(0, 3), (3, 6)]
