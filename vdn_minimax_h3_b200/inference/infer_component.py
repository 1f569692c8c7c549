"""Render through an exported model component -- the portable single-GPU path.

    python -m vdn_minimax_h3_b200.inference.infer_component COMPONENT_DIR [PROMPT]
        [--out results/component.mp4] [--steps 8] [--frames 345]
        [--first first.png] [--last last.png] [--offload_dit] [--model_root PATH|hub]
        [--random-base-seed N] [--seed 0] [--device cuda]

COMPONENT_DIR is what `python -m vdn_minimax_h3_b200.export.component CKPT` writes:
config.json plus the flattened `modeling_vdn_h3.py`. The modeling file is imported from
that directory (it needs no package), the component class assembles the transformer
(base + hybrid branch + merged adapters) and the transformer runs its eager bf16 forward:
no fp8, no fused block engine, no sequence parallelism. PROMPT is text (encoded by the
Qwen3-VL conditioner with --model_root, else by the weight-free stand-in) or a prompt-cache
.pt file written by encode_prompt / encode_keyframes. --first / --last add keyframes
(fl2va / i2va / l2va), put on the canvas and encoded like encode_keyframes does.
--offload_dit keeps the DiT blocks in pinned host memory and streams each onto the GPU
while it runs (the next one copied on a side stream), for a card that cannot hold the
transformer. The latents are decoded and written as one mp4 with the soundtrack muxed in
(inference/vae.py decoders: stand-ins for the external VAEs).

Reference parity: src/inference/infer_diffusers.py:40-131 (the published-component render:
`ModularPipeline.from_pretrained(...)`, text encoder and decoders offloaded, `--offload_dit`
block-level group offloading, `encode_video` with audio). diffusers is not part of this
stack; the component directory, the sampler of inference/render.py and the muxer stand in
for the pipeline blocks.
"""
import argparse
import os
import sys
import time

import torch

FPS = 24
DEFAULT_PROMPT = "Waves roll onto a beach at sunset while gulls call over the surf."


def load_transformer(component_dir, random_base_seed=None, dtype=torch.bfloat16):
    """The component's model, assembled by the class in the component's own modeling file.
    Returns (component module, transformer in `dtype` on the CPU; the alpha island fp32)."""
    from vdn_minimax_h3_b200.export.component import load_component_module
    mod = load_component_module(component_dir)
    comp = mod.VDNMiniMaxH3Transformer3DModel.from_pretrained(
        component_dir, device="cpu", random_base_seed=random_base_seed)
    model = comp.transformer.to(dtype)
    for blk in model.transformer_blocks:
        alpha = getattr(getattr(blk.attn, "linear_attention", None), "alpha", None)
        if alpha is not None:
            alpha.float()
    return mod, model.eval()


def place(model, device, offload_dit=False):
    """The whole transformer on `device`, or (offload_dit) everything but the DiT blocks,
    which then stream from pinned host memory block by block."""
    if not offload_dit:
        return model.to(device), None
    from vdn_minimax_h3_b200.inference.offload import enable_module_offload
    blocks = model.transformer_blocks
    for name, child in model.named_children():
        if child is not blocks:
            child.to(device)
    for name, p in list(model.named_parameters(recurse=False)):
        p.data = p.data.to(device)
    for name, b in list(model.named_buffers(recurse=False)):
        setattr(model, name, b.to(device))
    return model, enable_module_offload(model, device)


def prompt_inputs(prompt, first, last, model_root, device, seed, width):
    """-> (prompt_embeds [L, D] bf16, conditions or None, (latent_h, latent_w) or None)."""
    from vdn_minimax_h3_b200.inference.encoders import (VAE_SPATIAL, KeyframeVaeStandIn,
                                                        StandInConditioner, build_presentation,
                                                        make_conditioner, put_on_canvas)
    if prompt and prompt.endswith(".pt") and os.path.isfile(prompt):
        from vdn_minimax_h3_b200.inference.prompt_cache import load_prompt
        emb, _, conditions = load_prompt(prompt, device)
        return emb, conditions, None
    cond = make_conditioner(model_root, device, seed) if model_root else \
        StandInConditioner(seed=seed, width=width)
    images, canvas, anchors = [], None, []
    if first or last:
        from PIL import Image
        pairs = [(a, p) for a, p in (("first", first), ("last", last)) if p]
        anchors = [a for a, _ in pairs]
        images, height, width_px = put_on_canvas([Image.open(p) for _, p in pairs])
        canvas = (height // VAE_SPATIAL, width_px // VAE_SPATIAL)
    ids, _ = build_presentation(cond, prompt or DEFAULT_PROMPT, images)
    emb = cond.encode(ids, images).to(device, torch.bfloat16)
    conditions = None
    if images:
        vae = KeyframeVaeStandIn(seed)
        conditions = (tuple(anchors), [vae.encode(im).to(device) for im in images])
    return emb, conditions, canvas


def render(component_dir, prompt=None, out="results/component.mp4", steps=8, frames=345,
           first=None, last=None, offload_dit=False, model_root=None, random_base_seed=None,
           seed=0, device="cuda", latent_hw=None, num_latent_frames=None):
    """One clip through the component; returns a dict of what was written and the timings."""
    from vdn_minimax_h3_b200.inference.render import LATENT_H, LATENT_W, generate_latents
    from vdn_minimax_h3_b200.inference.vae import decode_and_save
    device = torch.device(device)
    t0 = time.perf_counter()
    mod, model = load_transformer(component_dir, random_base_seed)
    model, streamer = place(model, device, offload_dit)
    set_layout = getattr(mod, "set_layout", None)
    if set_layout is None:
        from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
    t_load = time.perf_counter() - t0
    emb, conditions, canvas = prompt_inputs(prompt, first, last, model_root, device, seed,
                                            model.config.text_dim)
    lh, lw = latent_hw or canvas or (LATENT_H, LATENT_W)
    per_step = []
    t1 = time.perf_counter()
    lat, aud = generate_latents(model, emb, frames, steps, seed, device, model.config,
                                conditions=conditions, latent_h=lh, latent_w=lw,
                                on_layout=lambda lay: set_layout(model, lay),
                                step_seconds=per_step, num_latent_frames=num_latent_frames)
    t_denoise = time.perf_counter() - t1
    timings = {}
    path = decode_and_save(lat, aud, out, timings=timings)
    return {"out": path, "frames": timings.get("frames"), "load_s": t_load,
            "denoise_s": t_denoise, "step_seconds": per_step,
            "offload_host_bytes": streamer.host_bytes() if streamer is not None else 0,
            **{k: v for k, v in timings.items() if k.endswith("_s")}}


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("component", help="component directory (config.json + modeling_vdn_h3.py)")
    p.add_argument("prompt", nargs="?", default=None,
                   help="prompt text, or a prompt-cache .pt (encode_prompt / encode_keyframes)")
    p.add_argument("--out", default="results/component.mp4")
    p.add_argument("--steps", type=int, default=8, help="model evaluations (NFE)")
    p.add_argument("--frames", type=int, default=345, help="snapped up to the next 17n+5")
    p.add_argument("--first", help="keyframe the video starts from")
    p.add_argument("--last", help="keyframe the video ends on")
    p.add_argument("--offload_dit", action="store_true",
                   help="stream the DiT blocks onto the GPU one at a time")
    p.add_argument("--model_root", default=None,
                   help="MiniMax-H3 snapshot (or `hub`) for the Qwen3-VL conditioner; "
                        "default: the weight-free stand-in")
    p.add_argument("--random-base-seed", type=int, default=None,
                   help="random backbone instead of the base weights (offline tests)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", default="cuda")
    args = p.parse_args(argv)
    if args.device.startswith("cuda"):
        torch.cuda.set_device(torch.device(args.device))
    rec = render(args.component, args.prompt, args.out, args.steps, args.frames, args.first,
                 args.last, args.offload_dit, args.model_root, args.random_base_seed,
                 args.seed, args.device)
    nfe = max(len(rec["step_seconds"]), 1)
    print(f"wrote {rec['out']}: {rec['frames']} frames; load {rec['load_s']:.1f}s, denoise "
          f"{rec['denoise_s']:.2f}s ({rec['denoise_s'] / nfe:.2f} s/NFE), decode "
          f"{rec.get('decode_s', 0):.1f}s, encode {rec.get('encode_s', 0):.1f}s", flush=True)
    return rec


if __name__ == "__main__":
    main()
    sys.exit(0)
