"""Training throughput: Stage B (LoRA `default` + linear branch against the dense teacher)
or Stage DMD (few-step generator, frozen real score, trainable fake score on one model).

    python bench_train.py [--stage b|dmd] [--steps K --warmup W] [--kernels on|off]   # 1 GPU
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench_train.py --gpus N --steps K --warmup W            # N GPUs, FSDP2

`--kernels off` is the labelled baseline arm: the same model and loop with every sm_100a
training kernel switched off (attention through PyTorch SDPA, the linear branch's scans /
SPD factor / short conv and the AdaLN norm in eager PyTorch, every Linear's forward, dgrad
and wgrad through cuBLAS), i.e. PyTorch FSDP2 + NCCL + cuBLAS / cuDNN. With `--kernels on`
the Linears run on the package's tcgen05 GEMM (ops/linear_grad.py).

Stage DMD (`--stage dmd`): each step is one DMD2 sub-iteration on every rank -- the
generator's own rollout of k grid steps (k the rank-shared index of that iteration, 8-step
grid), then on a generator turn the DM-loss update of `turbo` (generator x0 with a graph,
real and fake score x0) and on every turn the fake score's flow-matching update
(training.trainers.dmd_sub_iteration). Timed steps follow the 1 : 5 turn schedule from the
first generator turn; the line reports each turn kind's time and the whole-cycle rate
(1 generator + 5 fake sub-iterations).

One step on every rank = one synthetic clip (per-GPU batch 1) of the headline training
shape: 81 latent frames at the inference spatial latent size (48 x 84 -> 24 x 42 tokens per
frame), the matching audio latents and an 800 x 5120 prompt; the full VDN-H3 geometry with
random weights (backbone frozen; trainable: the hybrid branch and a rank-64 LoRA on the DiT
and refiner attention); FSDP2 with per-block activation checkpointing (checkpointed activations in pinned host
memory, the Stage B default `distributed.offload_activations=true`); the dense teacher
forward (no grad), the student forward + backward, gradient clipping and the AdamW step are
all inside the timed region. Timing: W untimed steps, then K steps between a barrier +
device synchronisation, CUDA events, max over ranks. Rank 0 prints one JSON line whose
`value` is the whole job's samples per second. `--tiny` swaps in a two-block model for CPU
tests (its numbers mean nothing). `VDN_PROF_STEP=n` (or H3_PROF_STEP) runs warm-up step n
(1-based) under torch.profiler and prints its kernel table; timed steps are never profiled.

Reference parity: the Stage B loop of src/training/train_stage_b.py:175-450 (here through
vdn_minimax_h3_b200.training: the same batch packing, teacher velocity, student forward,
loss and optimizer groups as `training.trainers.run_stage_b`).
"""
import argparse
import datetime
import json
import os
import sys
import time

import torch
import torch.distributed as dist
import torch.nn.functional as F

LORA_TARGETS = ["attn.orig.to_q", "attn.orig.to_k", "attn.orig.to_v", "attn.orig.to_out.0",
                "token_refiner.refiner_blocks.*.attn.to_q", "token_refiner.refiner_blocks.*.attn.to_k",
                "token_refiner.refiner_blocks.*.attn.to_v",
                "token_refiner.refiner_blocks.*.attn.to_out.0"]


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--latent-frames", type=int, default=81)
    p.add_argument("--lora-rank", type=int, default=64)
    p.add_argument("--no-offload", dest="offload", action="store_false",
                   help="keep checkpointed activations on the GPU (the Stage B default, "
                        "distributed.offload_activations=true, saves them to pinned host memory)")
    p.add_argument("--ac", choices=("block", "two-level"), default="block",
                   help="activation checkpointing: per block (the headline training setup), or per block "
                        "with the attention and feed-forward as inner regions")
    p.add_argument("--num-layers", type=int, default=None,
                   help="diagnostic only: fewer DiT blocks (the printed number is then not the "
                        "benchmark's)")
    p.add_argument("--stage", choices=("b", "dmd"), default="b")
    p.add_argument("--kernels", choices=("on", "off"), default="on",
                   help="off: the labelled baseline (PyTorch / cuBLAS / cuDNN for every op)")
    p.add_argument("--linears", choices=("kernel", "cublas"), default="kernel",
                   help="with --kernels on: the Linears' forward / dgrad / wgrad on the package's "
                        "GEMM (default) or on cuBLAS (isolates the GEMM's share of the step)")
    p.add_argument("--tiny", action="store_true", help="two-block model (CPU tests only)")
    return p.parse_args(argv)


def host_available_gib():
    """MemAvailable of this host in GiB (None where /proc/meminfo is absent)."""
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) / 2 ** 20
    except OSError:
        return None
    return None


def _linear_calls():
    """Linear forwards issued so far on the GEMM kernel vs on F.linear (ops/linear_grad.py)."""
    from vdn_minimax_h3_b200.ops import linear_grad
    return dict(linear_grad.STATS)


def main(argv=None):
    args = parse(argv)
    from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID, TINY_HYBRID, build_model, make_spec
    from vdn_minimax_h3_b200.models.h3 import h3_full_config, h3_tiny_config
    from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
    from vdn_minimax_h3_b200.models.lora import inject_lora
    from vdn_minimax_h3_b200.training import fsdp_stage as fs
    from vdn_minimax_h3_b200.training.batch import pack_noisy_batch
    from vdn_minimax_h3_b200.training.dataset import SyntheticLatentDataset
    from vdn_minimax_h3_b200.utils.activation_checkpointing import enable_block_checkpointing

    timing_phases = [False]

    def phase(name):
        """fs.phase when the step is being broken down, else a no-op context."""
        import contextlib
        return fs.phase(name) if timing_phases[0] else contextlib.nullcontext()

    if args.linears == "cublas":
        from vdn_minimax_h3_b200.ops import linear_grad
        linear_grad.LINEAR_KERNELS = False
    if args.kernels == "off":
        from vdn_minimax_h3_b200.ops import attention_grad, linear_branch_grad, linear_grad, norm_grad
        attention_grad.ATTENTION_KERNELS = False
        linear_branch_grad.USE_KERNELS = False
        linear_grad.LINEAR_KERNELS = False
        norm_grad.NORM_KERNELS = False
    cuda = torch.cuda.is_available()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(device)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        dist.init_process_group("nccl" if cuda else "gloo", timeout=datetime.timedelta(seconds=900),
                                **({"device_id": device} if cuda else {}))
    world, rank = dist.get_world_size(), dist.get_rank()
    torch.manual_seed(args.seed)

    cfg = h3_tiny_config() if args.tiny else h3_full_config()
    if args.num_layers:
        cfg.num_layers = args.num_layers
    hybrid = TINY_HYBRID if args.tiny else RELEASED_HYBRID
    t0 = time.perf_counter()
    spec = make_spec(cfg, hybrid, dtype="float32" if args.tiny else "bfloat16")
    model = build_model(spec, device="cpu" if args.tiny else device, init="random", seed=args.seed)
    inject_lora(model, "default", args.lora_rank, args.lora_rank, LORA_TARGETS)
    if args.stage == "dmd":
        # generator adapter `turbo` (trainable), fake-score adapter `fake` (trainable, B = 0);
        # the backbone, the hybrid branch and `default` are frozen (the Stage DMD trainables)
        inject_lora(model, "turbo", args.lora_rank, args.lora_rank, LORA_TARGETS, init_b_zero=False)
        inject_lora(model, "fake", 128, 128, LORA_TARGETS, init_b_zero=True)
        select = lambda n, p: ".lora_A.turbo." in n or ".lora_B.turbo." in n or \
            ".lora_A.fake." in n or ".lora_B.fake." in n  # noqa: E731
    else:
        select = fs.trainable_select(include_lora=True)
    for n, p in model.named_parameters():
        p.requires_grad_(select(n, p))
    model.to(device)
    if world > 1 or cuda:
        # one GPU is a 1-rank FSDP2 mesh: bf16 compute with fp32 trainables, as on N ranks
        fs.shard_model(model, device, None, activation_checkpointing=True,
                       split_ac=args.ac == "two-level")
    else:
        enable_block_checkpointing(model, split=args.ac == "two-level")
    if args.stage == "dmd":
        gen_params = [p for n, p in model.named_parameters() if p.requires_grad and ".turbo." in n]
        fake_params = [p for n, p in model.named_parameters() if p.requires_grad and ".fake." in n]
        optimizer = torch.optim.AdamW([{"params": gen_params}, {"params": fake_params}], lr=1e-5,
                                      weight_decay=0.0)
    else:
        groups = fs.build_param_groups(model, 1e-4, big_scale=0.4, small_scale=2.0, lora_scale=1.0)
        optimizer = torch.optim.AdamW(groups, lr=1e-4, weight_decay=0.0)
    trainable = [p for p in model.parameters() if p.requires_grad]
    gens = fs.make_generators(args.seed, rank, device)
    if args.tiny:
        shape, n_audio, text_len, text_dim = (cfg.in_channels, 3, 16, 16), 4, 8, cfg.text_dim
    else:
        shape = (cfg.in_channels, args.latent_frames, 48, 84)
        n_audio = max(8, args.latent_frames * 455 // 102)
        text_len, text_dim = 800, cfg.text_dim
    data = SyntheticLatentDataset(args.warmup + args.steps, shape, n_audio, text_len, text_dim,
                                  seed=args.seed + rank)
    build_s = time.perf_counter() - t0
    if args.offload and cuda:
        # checkpointed block inputs go to pinned host memory: refuse to start on a host that
        # cannot hold them twice over rather than exhaust the machine's memory
        rows = shape[1] * (shape[2] // 2) * (shape[3] // 2) + n_audio + text_len
        # measured on one B200: ~2 block inputs' worth (bf16) saved per block
        need = 2 * cfg.num_layers * rows * cfg.hidden_size * 2 / 2 ** 30
        avail = host_available_gib()
        if avail is not None and avail < 2 * need + 64:
            raise SystemExit(f"activation offload needs ~{need:.0f} GiB of pinned host memory "
                             f"(2x + 64 GiB margin); {avail:.0f} GiB available: pass --no-offload "
                             f"or use more ranks")

    saved = {}

    def step(i):
        with phase("pack"):
            batch = pack_noisy_batch(data[i], device, gens["noise"], gens["sigma"])
            set_layout(model, batch["layout"])
        with phase("teacher"):
            tv, ta = fs.teacher_velocity(model, batch["inputs"], adapters=True)
        before = torch.cuda.memory_allocated() if cuda else 0
        with phase("student_forward"):
            sv, sa = fs.student_forward(model, batch["inputs"], args.offload and cuda)
        if cuda and "per_block_gib" not in saved:
            # device memory the graph keeps between forward and backward, per block
            saved["per_block_gib"] = round((torch.cuda.memory_allocated() - before)
                                           / cfg.num_layers / 2 ** 30, 3)
        loss = F.mse_loss(sv[0].float(), tv) + 0.5 * F.mse_loss(sa[0].float(), ta)
        loss, _ = fs.finite_or_zero(loss)
        with phase("backward"):
            loss.backward()
        with phase("optimizer"):
            fs.clip_gradients(trainable, 1.0)
            optimizer.step()
            optimizer.zero_grad(set_to_none=True)
        return loss

    kinds = {}
    if args.stage == "dmd":
        from vdn_minimax_h3_b200.training import dmd as dmd_lib
        from vdn_minimax_h3_b200.training.batch import PackedPrompt, initial_noise
        from vdn_minimax_h3_b200.training.trainers import dmd_sub_iteration
        roles = dmd_lib.Roles(model, "vdn", "default", "turbo", "fake")
        schedule = dmd_lib.FewStepSchedule(8, 12.0, 3.0)
        video_shape = shape

        def turn_of(i):
            # warm-up: a generator turn then fake turns when W >= 2, one fake turn when W == 1;
            # then the 1:5 schedule from its first generator turn
            if i < args.warmup:
                return dmd_lib.GENERATOR_TURN if (i == 0 and args.warmup >= 2) else dmd_lib.FAKE_TURN
            return dmd_lib.turn(i - args.warmup, 0, 5)

        def step(i):
            packed = PackedPrompt(data[i]["prompt_embeds"], video_shape, n_audio, device)
            set_layout(model, packed.layout)
            k = dmd_lib.shared_rollout_index(args.seed, i, schedule.num_steps)
            v0, a0 = initial_noise(video_shape, n_audio, gens["noise"], device)
            with phase("rollout"):
                xv, xa = dmd_lib.rollout(model, roles, schedule, packed, v0, a0, k)
            with phase(f"{turn_of(i)}_turn"):
                rec = dmd_sub_iteration(model, roles, schedule, packed, xv, xa, k, turn_of(i), gens,
                                    optimizer, gen_params, fake_params, gen_lr=1e-5, fake_lr=1e-5,
                                    u_range=(0.02, 0.98), shifts=(12.0, 3.0), audio_weight=0.5,
                                    clips=(1.0, 1.0))
            kinds.setdefault("rollout_k", []).append(k)
            return torch.tensor(rec["fake_loss"])

    from vdn_minimax_h3_b200.utils.profiling import step_profiler
    phases = {}
    for i in range(args.warmup):
        timing_phases[0] = i == args.warmup - 1    # the last warm-up step is broken down
        fs.phase_reset()
        with step_profiler(i + 1, row_limit=40):   # VDN_PROF_STEP=n: warm-up step n only
            step(i)
        phases = fs.phase_fields("")
    timing_phases[0] = False
    kinds.clear()
    clocks = None
    if cuda:
        from bench import ClockSampler
        clocks = ClockSampler(device)
        clocks.start()
    dist.barrier()
    per_step = []
    if cuda:
        torch.cuda.synchronize()
        events = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        events[0].record()
    else:
        t_start = time.perf_counter()
    loss = None
    for i in range(args.steps):
        t_i = time.perf_counter()
        loss = step(args.warmup + i)
        if cuda:
            events[i + 1].record()
        else:
            per_step.append((time.perf_counter() - t_i) * 1e3)
    if cuda:
        torch.cuda.synchronize()
        per_step = [events[i].elapsed_time(events[i + 1]) for i in range(args.steps)]
        ms = events[0].elapsed_time(events[-1])
        clock_info = clocks.stop()
    else:
        ms = (time.perf_counter() - t_start) * 1e3
    dist.barrier()
    t = torch.tensor([ms] + per_step, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, per_step = float(t[0].item()), [float(x) for x in t[1:].tolist()]
    if rank == 0:
        stage_name = ("Stage DMD: DMD2 sub-iterations, generator:fake 1:5, 8-step grid"
                      if args.stage == "dmd" else "Stage B: LoRA + hybrid branch")
        line = {
            "metric": f"train samples/s ({stage_name}, FSDP2)",
            "value": round(world * args.steps / (ms / 1e3), 4), "unit": "samples/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 1), "higher_is_better": True, "scaling": "weak",
            "dtype": "bf16 params (fp32 master for trainables), fp32 loss",
            "data": "synthetic (random-normal latents and prompt embeddings; random-init weights)",
            "config": {"model": "tiny" if args.tiny else "VDN-H3 (50 blocks, hidden 5376, 56x128 heads)",
                       "per_gpu_batch": 1, "latent_frames": shape[1],
                       "latent_hw": list(shape[2:]), "lora_rank": args.lora_rank,
                       "parallelism": f"fsdp2 x{world}" if world > 1 else "single-gpu",
                       "activation_checkpointing": "per block" if args.ac == "block"
                       else "per block + attn/ff regions",
                       "num_layers": cfg.num_layers,
                       "activation_offload": bool(args.offload and cuda)},
            "loss": float(loss.item()) if loss is not None else None,
            "kernels": args.kernels,
            "linears": "cublas" if args.kernels == "off" else args.linears,
            "linear_calls": _linear_calls(),
            "reduce_scatter": ("symmetric memory (own kernel)" if getattr(
                getattr(model, "_vdn_reduce_comm", None), "calls", 0) else "nccl"),
            "all_gather": ("symmetric memory (own kernel)" if getattr(
                getattr(model, "_vdn_gather_comm", None), "calls", 0) else "nccl"),
            "phases_s": phases,
            "phases_note": "wall seconds of the last warm-up step (synchronising timers, not in the timed steps)",
            "step_ms": [round(x, 1) for x in per_step],
            "build_s": round(build_s, 1),
        }
        if args.stage == "dmd" and per_step:
            from vdn_minimax_h3_b200.training import dmd as dmd_lib
            gen = [ms_i for j, ms_i in enumerate(per_step) if dmd_lib.turn(j, 0, 5) == dmd_lib.GENERATOR_TURN]
            fake = [ms_i for j, ms_i in enumerate(per_step) if dmd_lib.turn(j, 0, 5) != dmd_lib.GENERATOR_TURN]
            if gen and fake:
                tg, tf = sum(gen) / len(gen), sum(fake) / len(fake)
                line["generator_turn_ms"], line["fake_turn_ms"] = round(tg, 1), round(tf, 1)
                # one 1:5 cycle = 1 generator + 5 fake sub-iterations, one clip per rank each
                line["cycle_samples_per_s"] = round(world * 6 / ((tg + 5 * tf) / 1e3), 4)
            line["rollout_k"] = kinds.get("rollout_k")
        if cuda:
            line["clocks"] = clock_info
            line["peak_gib"] = round(torch.cuda.max_memory_allocated() / 2 ** 30, 1)
            line["saved_per_block_gib"] = saved.get("per_block_gib")
        print(json.dumps(line), flush=True)
    fs.close_comms(model)
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
