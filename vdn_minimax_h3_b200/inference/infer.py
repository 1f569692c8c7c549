"""Single-GPU render entry point.

    python -m vdn_minimax_h3_b200.inference.infer --config configs/inference/8nfe_tuned_fp8.yaml \
        checkpoint=... render.prompt_file=... render.out=clip.mp4 [synthetic_base=true]

config -> assemble (checkpoint + base, or the synthetic random-init model) -> warm-up NFEs
-> timed render (device-synchronised per-NFE times) -> decode (stand-in decoders) -> mp4
with the soundtrack muxed in -> optional record JSON. `kernels.inference_kernels=false`
(the configs' rung 0, 8nfe.yaml / 50nfe.yaml) renders with the eager model -- the released
arithmetic, `kernels.softmax_backend` choosing the window path -- instead of the fused
engine; `true` (the `_tuned` rungs) runs the fused sm_100a engine, in fp8 when
`precision.fp8.enabled`. Reference parity: src/inference/infer.py:28-73 and the config
ladder of configs/inference/8nfe*.yaml.
"""
import json
import os
import subprocess
import sys
import time

import torch

from vdn_minimax_h3_b200.config import load_config
from vdn_minimax_h3_b200.config.schemas import (InferenceConfig, validate_ablation, validate_kernels,
                                                validate_single_process)


def assemble(cfg, device):
    from vdn_minimax_h3_b200.inference.assemble import (build_from_checkpoint, build_inference_engine,
                                                        build_synthetic_model)
    from vdn_minimax_h3_b200.inference.lora import load_external_lora, merge_lora_state
    from vdn_minimax_h3_b200.models.hybrid_transform import set_teacher_mode
    if cfg.checkpoint:
        from vdn_minimax_h3_b200.checkpoints import load_checkpoint
        art = load_checkpoint(cfg.checkpoint)
        model = build_from_checkpoint(art, device=device, base_source=cfg.base_source,
                                      init="random" if cfg.synthetic_base else "load")
    else:
        model, _ = build_synthetic_model(device=device)
    for ext in cfg.external_loras:
        state, scale, _ = load_external_lora(ext.path, ext.alpha)
        merge_lora_state(model, state, scale)
    if cfg.behavior.teacher_mode:
        set_teacher_mode(model, True)
    from vdn_minimax_h3_b200.models.hybrid_transform import set_softmax_backend
    set_softmax_backend(model, cfg.kernels.softmax_backend)
    if cfg.ablation.enabled:
        from vdn_minimax_h3_b200.models.hybrid_transform import iter_hybrids
        for attn in iter_hybrids(model):
            for k, v in cfg.ablation.overrides.items():
                if not hasattr(attn, k):
                    raise ValueError(f"ablation override {k!r} is not a hybrid attention field")
                setattr(attn, k, v)
    if not cfg.kernels.inference_kernels:
        # rung 0: the eager model itself (returned as the engine, so callers run it)
        if cfg.runtime.offload_blocks:
            from vdn_minimax_h3_b200.inference.offload import enable_module_offload
            enable_module_offload(model, device)
        return model, model
    engine = build_inference_engine(model, fp8=cfg.precision.fp8.enabled)
    if cfg.runtime.offload_blocks:
        from vdn_minimax_h3_b200.inference.offload import enable_block_offload
        enable_block_offload(engine)
    return model, engine


def render(cfg, model, engine, device, runtime=None, transformer=None, on_step=None):
    from vdn_minimax_h3_b200.inference.prompt_cache import load_prompt
    from vdn_minimax_h3_b200.inference.render import generate_latents
    from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
    emb, _, conditions = load_prompt(cfg.render.prompt_file, device)
    transformer = transformer or engine
    kw = dict(video_shift=cfg.render.video_shift, audio_shift=cfg.render.audio_shift,
              conditions=conditions, on_layout=lambda lay: set_layout(model, lay),
              barrier=runtime.barrier if runtime is not None else None, on_step=on_step)
    if cfg.render.warmup_steps:
        generate_latents(transformer, emb, cfg.render.num_frames, cfg.render.warmup_steps,
                         cfg.render.seed, device, model.config, **kw)
    steps = []
    t0 = time.perf_counter()
    lat, aud = generate_latents(transformer, emb, cfg.render.num_frames, cfg.render.num_steps,
                                cfg.render.seed, device, model.config, step_seconds=steps, **kw)
    return lat, aud, steps, time.perf_counter() - t0


def main(argv=None):
    cfg = load_config(InferenceConfig, argv, (validate_kernels, validate_ablation,
                                              validate_single_process))
    device = torch.device(cfg.render.device)
    torch.cuda.set_device(device)
    t_start = time.perf_counter()
    model, engine = assemble(cfg, device)
    t_setup = time.perf_counter() - t_start
    lat, aud, steps, denoise = render(cfg, model, engine, device)
    from vdn_minimax_h3_b200.inference.vae import decode_and_save
    t0 = time.perf_counter()
    decode_and_save(lat, aud, cfg.render.out)
    t_decode = time.perf_counter() - t0
    if cfg.render.save_latents:
        os.makedirs(cfg.render.latents_root, exist_ok=True)
        torch.save({"latents": lat.cpu(), "audio": aud.cpu()},
                   os.path.join(cfg.render.latents_root, os.path.basename(cfg.render.out) + ".pt"))
    print(f"timing: setup {t_setup:.1f}s, denoise {denoise:.2f}s ({cfg.render.num_steps} NFE, "
          f"{denoise / cfg.render.num_steps:.2f} s/NFE), decode+encode {t_decode:.1f}s", flush=True)
    if cfg.render.record:
        from vdn_minimax_h3_b200.config.loader import resolved_dict
        try:
            commit = subprocess.run(["git", "rev-parse", "HEAD"], capture_output=True, text=True).stdout.strip()
        except OSError:
            commit = None
        rec = {"config": resolved_dict(cfg), "step_seconds": steps, "denoise_s": denoise,
               "setup_s": t_setup, "decode_s": t_decode, "git_commit": commit,
               "fp8": cfg.precision.fp8.enabled,
               "engine": ("fused sm_100a kernels" if cfg.kernels.inference_kernels
                          else f"eager model (softmax_backend={cfg.kernels.softmax_backend})")}
        with open(cfg.render.out + ".inference.json", "w") as f:
            json.dump(rec, f, indent=2)
    return 0


if __name__ == "__main__":
    sys.exit(main())
