"""Per-section device-time breakdown of the full-size inference engine on one GPU.

    python -m vdn_minimax_h3_b200.profile_block [--nfe 2] [--num-layers 50]

Builds the synthetic full-geometry model, runs one warm-up NFE, then `--nfe` NFE with the
engine's CUDA-event section timer on, and prints ms per NFE per section as JSON.
"""
import argparse
import json

import torch


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--nfe", type=int, default=2)
    p.add_argument("--num-layers", type=int, default=50)
    a = p.parse_args(argv)
    import bench  # noqa: F401  (same synthetic request as the headline bench)
    from vdn_minimax_h3_b200.inference.assemble import build_inference_engine, build_synthetic_model
    from vdn_minimax_h3_b200.inference.render import generate_latents
    from vdn_minimax_h3_b200.models.h3 import h3_full_config
    from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
    cfg = h3_full_config()
    cfg.num_layers = a.num_layers
    dev = torch.device("cuda", 0)
    model, _ = build_synthetic_model(cfg, device=dev)
    engine = build_inference_engine(model)
    emb = torch.randn(800, cfg.text_dim, device=dev, dtype=torch.bfloat16)
    generate_latents(engine, emb, 345, 1, 0, dev, cfg, on_layout=lambda l: set_layout(model, l))
    engine.timer.enabled = True
    generate_latents(engine, emb, 345, a.nfe, 0, dev, cfg, on_layout=lambda l: set_layout(model, l))
    rep = engine.timer.report()
    per_nfe = {k: round(v / a.nfe, 2) for k, v in rep.items()}
    print(json.dumps({"ms_per_nfe_by_section": per_nfe, "total_ms_per_nfe": round(sum(per_nfe.values()), 1),
                      "num_layers": a.num_layers}), flush=True)


if __name__ == "__main__":
    main()
