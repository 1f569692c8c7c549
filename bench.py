"""Headline benchmark: VDN-H3 T2VA denoising of a 14.4 s clip (345 frames, 768x1344,
102 latent frames, 104,766 packed rows), 8 NFE, random-init weights of the full
architecture, synthetic latents and prompt embeddings.

Default: the block-scaled fp8 configuration (E4M3 projections with 1x128 activation /
128x128 weight scales; attention and the linear branch in bf16), tensor parallel 2 x
Ulysses N/2 on N >= 2 GPUs -- the precision of the published headline numbers (MXFP8) and
the hybrid layout of the fp8 configuration. `--bf16` runs every GEMM in bf16 with plain
Ulysses over N GPUs.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference] [--bf16]
    torchrun --nproc-per-node N ... bench.py --gpus N ...

One "step" is one NFE (one transformer forward + the scheduler's Euler step) of the
8-step schedule; W untimed steps, then exactly K steps timed with CUDA events between a
barrier + synchronize on both sides, max over ranks. `value` is the denoise time of a whole
8-NFE clip (ms_per_step * 8), in seconds (lower is better). `e2e` runs the public API
(inference.render.generate_latents) for a full 8-NFE render with the inputs copied from
pinned host memory and the latents read back each run. Rank 0 prints one JSON line.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import torch

BASELINE = {1: 47.6, 2: 25.9, 4: 13.1, 8: 6.9}     # published SGLang MXFP8 denoise s, 8 NFE, B200 (reference README.md:133)
METRIC = "denoise s per 14.4s clip, 8 steps (e2e s alongside)"
NUM_FRAMES, TEXT_LEN, NFE = 345, 800, 8


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--fp8", action="store_true", default=True,
                   help="block-scaled fp8 projections (default)")
    p.add_argument("--bf16", dest="fp8", action="store_false",
                   help="bf16 projections, Ulysses over all GPUs")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--tp", type=int, default=None,
                   help="tensor-parallel degree (TP x Ulysses); default 2 with fp8 on an even "
                        "number of GPUs, else 1")
    p.add_argument("--exchange", choices=("p2p", "nccl"), default="p2p",
                   help="Ulysses exchange: symmetric-memory stores fused into the producing "
                        "kernels (p2p) or NCCL all_to_all_single (nccl)")
    p.add_argument("--softmax-ranks", type=int, default=0,
                   help="branch-parallel Ulysses: this many ranks run the window softmax, the "
                        "rest the linear branch (0 = every rank runs both for its heads)")
    p.add_argument("--num-layers", type=int, default=None, help=argparse.SUPPRESS)
    return p.parse_args(argv)


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.rows = []
        self.proc = None
        try:
            props = torch.cuda.get_device_properties(device)
            self.target = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        except Exception:
            self.target = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.target:
            cmd += ["-i", self.target]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm = sorted(float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit())
        mx = max((float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()),
                 default=None)
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in self.rows if len(r) >= 9 for n, v in zip(names, r[5:9])
                          if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(sm)}


# ------------------------------------------------------------------------------ arms
def reference_arm(args):
    """The reference's own stack, unmodified, through its public API -- if it imports."""
    ref = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    why = None
    if not os.path.isdir(ref):
        why = "baseline/_ref not installed"
    else:
        sys.path.insert(0, ref)
        try:
            import src.inference.render  # noqa: F401  (the reference's render entry)
        except Exception as exc:  # noqa: BLE001
            why = (f"reference needs its patched diffusers MiniMax-H3 backbone, peft, omegaconf and "
                   f"flash-attn-4, none installable offline; import failed: {type(exc).__name__}: {exc}")
    if why:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return 0
    raise SystemExit("reference arm imported unexpectedly; no runner is wired for it")


def main(argv=None):
    args = parse(argv)
    if args.impl == "reference":
        return reference_arm(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.tp is None:
        args.tp = 2 if (args.fp8 and world >= 2 and world % 2 == 0
                        and not args.softmax_ranks) else 1
    if args.softmax_ranks and args.tp > 1:
        raise SystemExit("--softmax-ranks is a Ulysses-only layout; use --tp 1")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    runtime = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    from vdn_minimax_h3_b200.inference.assemble import build_inference_engine, build_synthetic_model
    from vdn_minimax_h3_b200.inference.render import build_inputs, generate_latents, render_geometry
    from vdn_minimax_h3_b200.models.h3 import h3_full_config
    from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
    from vdn_minimax_h3_b200.models.layout import patchify_video_latents
    from vdn_minimax_h3_b200.models.scheduler import FlowMatchEulerScheduler
    from vdn_minimax_h3_b200.ops import _ext

    cfg = h3_full_config()
    if args.num_layers:
        cfg.num_layers = args.num_layers
    model, build_s = build_synthetic_model(cfg, device=dev, seed=args.seed)
    engine = build_inference_engine(model, fp8=args.fp8)
    transformer = engine
    if world > 1 and args.tp > 1:
        from vdn_minimax_h3_b200.parallel.hybrid import HybridEngine, HybridRuntime
        runtime = HybridRuntime(args.tp)
        transformer = HybridEngine(engine, runtime, fp8=args.fp8)
    elif world > 1:
        from vdn_minimax_h3_b200.parallel.ulysses import UlyssesEngine, init_ulysses
        runtime = init_ulysses(softmax_ranks=args.softmax_ranks)
        transformer = UlyssesEngine(engine, runtime, exchange=args.exchange)

    # ---- synthetic request: prompt embeddings + noise for a 14.4 s clip
    g = torch.Generator().manual_seed(args.seed + 100)
    prompt_host = torch.randn(TEXT_LEN, cfg.text_dim, generator=g).to(torch.bfloat16).pin_memory()
    geo = render_geometry(cfg, NUM_FRAMES)
    video_host = torch.randn(1, geo.channels, geo.num_latent_frames, geo.latent_h, geo.latent_w,
                             generator=g).pin_memory()
    audio_host = torch.randn(geo.num_audio_latents * 2, 32, generator=g).pin_memory()

    packed, layout, idx = build_inputs(geo, TEXT_LEN, dev)
    set_layout(model, layout)
    emb = prompt_host.to(dev, non_blocking=True)[None]
    video_rows = patchify_video_latents(video_host.to(dev), geo.patch)
    audio_rows = audio_host.to(dev)
    sched, a_sched = FlowMatchEulerScheduler(12.0), FlowMatchEulerScheduler(3.0)
    sched.set_timesteps(NFE + 1, device=dev)
    a_sched.set_timesteps(NFE + 1, device=dev)
    S = int(packed.position_ids.shape[0])

    def step(i):
        nonlocal video_rows, audio_rows
        k = i % NFE
        t, a_t = float(sched.timesteps[k]), float(a_sched.timesteps[k])
        row_t = torch.full((S,), t, dtype=torch.float32, device=dev)
        row_t[idx["audio_indices"]] = a_t
        timestep, t_idx = torch.unique(row_t, sorted=True, return_inverse=True)
        v, a = transformer(hidden_states=video_rows[None], audio_hidden_states=audio_rows[None],
                           encoder_hidden_states=emb, timestep=timestep, timestep_indices=t_idx,
                           token_tags=idx["token_tags"], position_ids=idx["position_ids"],
                           video_indices=idx["video_indices"], audio_indices=idx["audio_indices"],
                           text_indices=idx["text_indices"], return_dict=False)
        video_rows = sched.step(v[0].float(), t, video_rows, index=k)
        audio_rows = a_sched.step(a[0].float(), a_t, audio_rows, index=k)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for i in range(args.warmup):
        step(i)
    _ext.check_device_error(dev)
    barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    launches0 = _ext.LAUNCHES[0]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        step(args.warmup + i)
    e1.record()
    torch.cuda.synchronize(dev)
    barrier()
    clock_info = clocks.stop()
    launches = _ext.LAUNCHES[0] - launches0
    _ext.check_device_error(dev)
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    value = ms * NFE / 1000.0

    e2e = None
    if not args.no_e2e:
        # The public API end to end: inputs from pinned host memory, the 8-NFE render
        # (inference.render.generate_latents), then inference.vae.decode_and_save -- the
        # video decoder stand-in (the VAE's geometry and ~700 TFLOP of convolutions, frames
        # split across the ranks), OpenCV's mp4 encode (each rank encodes its own frames,
        # rank 0 joins the segments) and the PCM soundtrack muxed into the same file on
        # rank 0. Wall clock, both ends synchronised, max over ranks. d2h counts every
        # frame of the clip once (each rank copies its share).
        from vdn_minimax_h3_b200.inference.vae import (AudioDecoderStandIn, VideoDecoderStandIn,
                                                       decode_and_save, decode_frames)
        vdec, adec = VideoDecoderStandIn(geo.channels), AudioDecoderStandIn(32)
        decode_frames(video_host[:, :, :7].to(dev), vdec)        # warm-up: kernels, autotune
        out_path = os.path.join("/tmp", f"vdn_bench_{os.getpid()}.mp4")
        barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        emb_d = prompt_host.to(dev, non_blocking=True)
        vid_d = patchify_video_latents(video_host.to(dev, non_blocking=True), geo.patch)
        aud_d = audio_host.to(dev, non_blocking=True)
        lat, aud = generate_latents(transformer, emb_d, NUM_FRAMES, NFE, args.seed, dev, cfg,
                                    initial_noise=(vid_d, aud_d),
                                    on_layout=lambda lay: set_layout(model, lay))
        torch.cuda.synchronize(dev)
        t_lat = time.perf_counter()
        timings = {}
        decode_and_save(lat, aud, out_path, vdec, adec, timings=timings)
        torch.cuda.synchronize(dev)
        barrier()
        t1 = time.perf_counter()
        e2e_s, denoise_s = t1 - t0, t_lat - t0
        if world > 1:
            t = torch.tensor([e2e_s, denoise_s], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_s, denoise_s = (float(x) for x in t.tolist())
        mp4_bytes = os.path.getsize(out_path) if rank == 0 and os.path.exists(out_path) else 0
        if rank == 0 and os.path.exists(out_path):
            os.remove(out_path)
        bi = (prompt_host.numel() * prompt_host.element_size() + video_host.numel() * 4
              + audio_host.numel() * 4)
        frames = timings.get("frames", 0)
        bo = frames * geo.latent_h * 16 * geo.latent_w * 16 * 3 if rank == 0 else 0
        e2e = {"value": round(e2e_s, 3), "unit": "s", "h2d_bytes_per_step": bi // NFE,
               "d2h_bytes_per_step": bo // NFE, "denoise_s": round(denoise_s, 3),
               "decode_s": round(timings.get("decode_s", 0.0), 3),
               "encode_s": round(timings.get("encode_s", 0.0), 3),
               "mux_s": round(timings.get("mux_s", 0.0), 3), "frames": frames,
               "mp4_bytes": mp4_bytes,
               "note": "one clip through inference.render.generate_latents and "
                       "inference.vae.decode_and_save: H2D of the inputs, 8 NFE, decode by the "
                       "VAE-geometry decoder STAND-IN (random weights, ~700 TFLOP), uint8 "
                       "frames to the host (each rank its share), OpenCV mp4v encode per rank, "
                       "segments joined and PCM audio muxed into the mp4 on rank 0"}
        _ext.check_device_error(dev)

    if rank == 0:
        base = BASELINE.get(world)
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
            "higher_is_better": False, "scaling": "strong",
            "vs_baseline": round(value / base, 3) if base else None,
            "dtype": ("fp8 (E4M3 block-scaled projections: 1x128 activation / 128x128 weight "
                      "scales; bf16 attention, linear branch, norms)") if args.fp8 else "bf16",
            "data": "synthetic (random-normal latents and prompt embeddings; random-init weights)",
            "config": {"model": f"VDN-H3 (MiniMax-H3 geometry, {cfg.num_layers} blocks, hidden "
                                f"{cfg.hidden_size}, {cfg.num_attention_heads}x{cfg.attention_head_dim} heads, "
                                "c1 window + vdn_solve linear branch, LoRA default+turbo merged)",
                       "global_batch": 1, "seq_len": S, "num_frames": NUM_FRAMES,
                       "latent_frames": geo.num_latent_frames, "text_len": TEXT_LEN, "nfe": NFE,
                       "parallelism": ("single-gpu" if world == 1 else
                                       f"tp{args.tp}xulysses{world // args.tp}" if args.tp > 1
                                       else f"ulysses{world}" + (
                                           f" (branch parallel {args.softmax_ranks} softmax + "
                                           f"{world - args.softmax_ranks} linear ranks)"
                                           if args.softmax_ranks else "")),
                       "exchange": None if world == 1 else ("p2p" if args.tp > 1 else args.exchange),
                       "baseline_config": ("block-scaled fp8, TP=2 x Ulysses (BASELINE config 3)"
                                           if args.fp8 else "bf16 Ulysses (BASELINE config 2)"),
                       "l2": "inputs larger than L2 (the weights, 33-66 GB, stream every step)"},
            "clocks": clock_info, "gpu_launches": launches, "e2e": e2e,
            "build_s": round(build_s, 1),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        transformer.close()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
