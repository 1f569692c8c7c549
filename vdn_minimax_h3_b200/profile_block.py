"""Per-section device-time breakdown of the full-size inference engine.

    python -m vdn_minimax_h3_b200.profile_block [--nfe 2] [--num-layers 50]
    torchrun --nproc-per-node N -m vdn_minimax_h3_b200.profile_block [--exchange p2p|nccl]

Builds the synthetic full-geometry model, runs one warm-up NFE, then `--nfe` NFE with the
CUDA-event section timer on (the engine's on one GPU, the Ulysses runtime's under torchrun)
and prints ms per NFE per section as JSON (rank 0 prints every rank's line).
"""
import argparse
import datetime
import json
import os

import torch


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--nfe", type=int, default=2)
    p.add_argument("--num-layers", type=int, default=50)
    p.add_argument("--exchange", choices=("p2p", "nccl"), default="p2p")
    p.add_argument("--fp8", action="store_true")
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--softmax-ranks", type=int, default=0)
    p.add_argument("--kernel-table", action="store_true",
                   help="also run one NFE under torch.profiler and print its device-time table "
                        "(kernels, copies) and the host calls that synchronise")
    a = p.parse_args(argv)
    import bench  # noqa: F401  (same synthetic request as the headline bench)
    from vdn_minimax_h3_b200.inference.assemble import build_inference_engine, build_synthetic_model
    from vdn_minimax_h3_b200.inference.render import generate_latents
    from vdn_minimax_h3_b200.models.h3 import h3_full_config
    from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    cfg = h3_full_config()
    cfg.num_layers = a.num_layers
    model, _ = build_synthetic_model(cfg, device=dev)
    engine = build_inference_engine(model, fp8=a.fp8)
    transformer, timer = engine, engine.timer
    if world > 1 and a.tp > 1:
        from vdn_minimax_h3_b200.parallel.hybrid import HybridEngine, HybridRuntime
        rt = HybridRuntime(a.tp)
        transformer = HybridEngine(engine, rt, fp8=a.fp8)
        timer = rt.timer
    elif world > 1:
        from vdn_minimax_h3_b200.parallel.ulysses import UlyssesEngine, init_ulysses
        rt = init_ulysses(softmax_ranks=a.softmax_ranks)
        transformer = UlyssesEngine(engine, rt, exchange=a.exchange)
        timer = rt.timer
    emb = torch.randn(800, cfg.text_dim, device=dev, dtype=torch.bfloat16)
    on_layout = lambda lay: set_layout(model, lay)  # noqa: E731
    generate_latents(transformer, emb, 345, 1, 0, dev, cfg, on_layout=on_layout)
    timer.enabled = True
    generate_latents(transformer, emb, 345, a.nfe, 0, dev, cfg, on_layout=on_layout)
    rep = timer.report()
    if a.kernel_table and (world == 1 or torch.distributed.get_rank() == 0):
        from torch.profiler import ProfilerActivity, profile
        timer.enabled = False
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            generate_latents(transformer, emb, 345, 1, 0, dev, cfg, on_layout=on_layout)
            torch.cuda.synchronize()
        ka = prof.key_averages()
        print(ka.table(sort_by="cuda_time_total", row_limit=45, max_name_column_width=70),
              flush=True)
        syncs = [e for e in ka if any(s in e.key for s in ("Synchronize", "Memcpy", "item",
                                                           "_local_scalar_dense", "nonzero"))]
        for e in syncs:
            print(json.dumps({"host_call": e.key, "count": e.count,
                              "cpu_ms": round(e.cpu_time_total / 1e3, 3)}), flush=True)
        timer.enabled = True
    per_nfe = {k: round(v / a.nfe, 2) for k, v in rep.items()}
    line = {"ms_per_nfe_by_section": per_nfe, "total_ms_per_nfe": round(sum(per_nfe.values()), 1),
            "num_layers": a.num_layers, "world": world, "fp8": a.fp8, "tp": a.tp}
    if world > 1:
        import torch.distributed as dist
        lines = [None] * world
        dist.all_gather_object(lines, line)
        transformer.close()
        if dist.get_rank() == 0:
            for r, ln in enumerate(lines):
                print(json.dumps({"rank": r, **ln}), flush=True)
        dist.destroy_process_group()
    else:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
