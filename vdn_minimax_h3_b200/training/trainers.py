"""The four training stages.

  Stage A1  per-layer alignment (reference src/training/train_stage_a1.py:50-395): the dense
            teacher trunk runs under no_grad with teacher_mode; a forward hook on every
            HybridAttention re-runs the hybrid on the detached input and backpropagates the
            normalised error sum((s - t)^2) / sum(t^2) at once (one layer's graph alive at a
            time). Gradients are all-reduced (AVG); ZeRO-1: layer i's optimizer lives on rank
            i % world, which steps it and broadcasts the parameters. Per-layer clipping.
  Stage A2  end-to-end alignment under FSDP2 to the teacher velocity, video + weighted audio
            MSE, non-finite losses zeroed through the graph (train_stage_a2.py:43-296).
  Stage B   A2 plus the `default` LoRA on the DiT/refiner attention projections; objective
            `teacher` (teacher velocity) or `diffusion` (data-ward velocity) with per-modality
            lambda mixing, `excess_vs_teacher` logged (train_stage_b.py:52-450).
  Stage DMD DMD2 without a GAN (train_stage_dmd.py:103-514, training/dmd.py): generator =
            VDN + default + turbo, real score = dense teacher or VDN, fake score = real + a
            rank-128 `fake` adapter (B = 0 at init); fake-only warm-up, then one generator
            update per `fake_updates_per_step` sub-iterations.

All four share training/fsdp_stage.py. Every stage writes `metrics.jsonl` on rank 0 and
saves v2 artifacts (weights every `save_every`, train states with name-keyed optimizer
state and per-rank RNG). `synthetic` as a base source means a random-init backbone.
"""
import json
import math
import os
import time
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.nn.functional as F

from vdn_minimax_h3_b200.config.loader import resolved_dict
from vdn_minimax_h3_b200.models.factory import build_model, load_model_weights, resolve_model_spec
from vdn_minimax_h3_b200.models.hybrid_transform import (hybrid_new_parameters, is_transform_parameter,
                                                         iter_hybrids, set_layout, set_teacher_mode)
from vdn_minimax_h3_b200.models.lora import inject_lora, set_active_adapters
from vdn_minimax_h3_b200.models.model_spec import AdapterSpec, ModelSpec
from vdn_minimax_h3_b200.training import dmd as dmd_lib
from vdn_minimax_h3_b200.training import fsdp_stage as fs
from vdn_minimax_h3_b200.training.batch import PackedPrompt, initial_noise, pack_noisy_batch, sample_paired_timesteps
from vdn_minimax_h3_b200.utils import run_lock
from vdn_minimax_h3_b200.utils.lr_schedule import check_schedule_stamp, lr_at, schedule_stamp
from vdn_minimax_h3_b200.utils.profiling import debug_memory_line, step_profiler
from vdn_minimax_h3_b200.utils.watchdog import Heartbeat


# ----------------------------------------------------------------------------- common
def _dist_setup(seed):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
        backend = "nccl"
    else:
        device = torch.device("cpu")
        backend = "gloo"
    if not dist.is_initialized():
        import datetime
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=900),
                                **({"device_id": device} if backend == "nccl" else {}))
    torch.manual_seed(seed)
    return world, dist.get_rank(), device


def _init_mode(source):
    return "random" if source == "synthetic" else "load"


def _metrics_writer(out_dir):
    path = os.path.join(out_dir, "metrics.jsonl")

    def write(rec):
        if fs.rank0():
            with open(path, "a") as f:
                f.write(json.dumps(rec) + "\n")
    return write


def _reduce_metrics(values, device):
    keys = sorted(values)
    t = torch.tensor([float(values[k]) for k in keys], dtype=torch.float64, device=device)
    if dist.is_initialized():
        dist.all_reduce(t)
        t /= dist.get_world_size()
    return dict(zip(keys, t.tolist()))


def _load_dataset(cfg, video_shape=None, text_only=False):
    from vdn_minimax_h3_b200.training.dataset import H3LatentT2VADataset, SyntheticLatentDataset
    idx = cfg.data.index_file
    if idx.startswith("synthetic:"):
        # synthetic:<n>:<C>x<F>x<h>x<w>:<audio latents>:<text_len>:<text_dim>
        _, n, geo, na, tl, td = idx.split(":")
        C, F_, h, w = (int(v) for v in geo.split("x"))
        return SyntheticLatentDataset(int(n), (C, F_, h, w), int(na), int(tl), int(td),
                                      text_only=text_only)
    return H3LatentT2VADataset(idx, text_only=text_only)


def _prepare_trainables(model, select):
    for name, p in model.named_parameters():
        p.requires_grad_(bool(select(name, p)))
        if p.requires_grad:
            p.data = p.data.float()     # fp32 masters for everything that trains


def _sched_args(opt, max_steps):
    return SimpleNamespace(lr=opt.lr, min_lr=opt.min_lr, warmup_steps=opt.warmup_steps,
                           max_steps=max_steps)


# ---------------------------------------------------------------------------- A2 / B
def _fsdp_stage(cfg, stage):
    """The shared loop of A2 and B."""
    out = cfg.checkpoint.output_dir
    fs.refuse_if_guarded(out, os.path.join(out, "DONE"), getattr(cfg.training, "ignore_stopped", False))
    world, rank, device = _dist_setup(cfg.training.seed)
    if rank == 0:
        run_lock.acquire(out)
    from vdn_minimax_h3_b200.checkpoints.loader import load_checkpoint
    seed_art = load_checkpoint(cfg.initialization.checkpoint)
    spec = ModelSpec.from_dict(seed_art.model_spec)
    lora_cfg = getattr(cfg, "lora", None)
    if stage == "b" and lora_cfg is not None and not spec.adapters:
        spec.adapters = [AdapterSpec("lora", 1, {"rank": lora_cfg.rank, "alpha": lora_cfg.alpha,
                                                 "targets": list(lora_cfg.targets), "name": "default"})]
    spec_dict = spec.to_dict()
    src = cfg.initialization.base_source or spec.base.source
    model = build_model(spec, device="cpu", base_source=src, init=_init_mode(src), seed=cfg.training.seed)
    load_model_weights(model, {k: v for k, v in seed_art.weights.items() if ".lora_" not in k}, strict=False)
    for a in spec.adapters:
        c = a.config
        inject_lora(model, c.get("name", "default"), c["rank"], c["alpha"], c["targets"])
    lora_w = {k: v for k, v in seed_art.weights.items() if ".lora_" in k}
    if lora_w:
        load_model_weights(model, lora_w, strict=False)
    select = fs.trainable_select(include_lora=stage == "b")
    _prepare_trainables(model, select)
    if getattr(cfg.training, "freeze_softmax_gate", False):
        for attn in iter_hybrids(model):
            if attn.enable_softmax_gate:
                attn.softmax_gate.requires_grad_(False)
    model.to(device)
    resume = fs.find_resume(out, spec_dict, model) if cfg.training.auto_resume else fs.Resume()
    from vdn_minimax_h3_b200.utils.distributed import broadcast_and_verify_init
    if world > 1:
        broadcast_and_verify_init(model, [p for n, p in model.named_parameters() if p.requires_grad], device)
    if world > 1 or torch.device(device).type == "cuda":
        # one rank on a GPU is a 1-rank FSDP2 mesh too: its mixed-precision policy is what
        # runs a bf16 backbone with fp32 trainables (and fp32 alpha modules)
        fs.shard_model(model, device, cfg.distributed.shard_size, cfg.distributed.activation_checkpointing)
    opt_cfg = cfg.optimizer
    big = getattr(opt_cfg, "big_lr_scale", getattr(opt_cfg, "branch_lr_scale", 1.0))
    groups = fs.build_param_groups(model, opt_cfg.lr, big_scale=big, small_scale=opt_cfg.small_lr_scale,
                                   small_eps=opt_cfg.small_eps, lora_scale=1.0)
    optimizer = torch.optim.AdamW(groups, lr=opt_cfg.lr, weight_decay=opt_cfg.weight_decay)
    gens = fs.make_generators(cfg.training.seed, rank, device)
    cursor = fs.restore_optimizer_and_rng(resume, model, optimizer, gens)
    sched = _sched_args(opt_cfg, cfg.training.max_steps)
    if resume.artifact is not None and resume.artifact.resolved_training_config:
        check_schedule_stamp(resume.artifact.metadata.get("schedule"), sched, rank, resume.step)
    dataset = _load_dataset(cfg)
    loader, sampler = fs.make_loader(dataset, world, rank, cfg.training.seed,
                                      getattr(cfg.data, "num_workers", 0))
    sampler.skip = cursor
    write = _metrics_writer(out)
    trainable = [p for p in model.parameters() if p.requires_grad]
    step = resume.step
    objective = getattr(cfg.training, "objective", "teacher")
    it = iter(loader)
    hb = Heartbeat(interval_s=1.0, timeout_s=120.0).start() if world > 1 else None
    while step < cfg.training.max_steps:
        if hb is not None:
            hb.check()      # a dead or stalled peer is reported before this step's collectives
        fs.phase_reset()
        try:
            sample = next(it)
        except StopIteration:
            sampler.skip = 0
            sampler.sampler.set_epoch(step)
            it = iter(loader)
            sample = next(it)
        t0 = time.perf_counter()
        prof_ctx = step_profiler(step + 1, print_fn=lambda m: print(m, flush=True) if fs.rank0() else None)
        prof_ctx.__enter__()
        with fs.phase("pack"):
            batch = pack_noisy_batch(sample, device, gens["noise"], gens["sigma"])
            set_layout(model, batch["layout"])
        with fs.phase("teacher"):
            tv, ta = fs.teacher_velocity(model, batch["inputs"], adapters=stage == "b")
        with fs.phase("student"):
            sv, sa = fs.student_forward(model, batch["inputs"], cfg.distributed.offload_activations)
            sv, sa = sv[0].float(), sa[0].float()
            w_a = cfg.training.audio_loss_weight
            loss_teacher = F.mse_loss(sv, tv) + w_a * F.mse_loss(sa, ta)
            with torch.no_grad():
                data_v = F.mse_loss(sv, batch["target_video_rows"])
                data_a = F.mse_loss(sa, batch["target_audio_rows"])
                teacher_data = F.mse_loss(tv, batch["target_video_rows"])
            if stage == "b" and objective == "diffusion":
                loss = F.mse_loss(sv, batch["target_video_rows"]) + w_a * F.mse_loss(sa, batch["target_audio_rows"])
            else:
                loss = loss_teacher
            if stage == "b":
                lv, la = cfg.training.lambda_diffusion_video, cfg.training.lambda_diffusion_audio
                if lv:
                    loss = loss + lv * F.mse_loss(sv, batch["target_video_rows"])
                if la:
                    loss = loss + la * F.mse_loss(sa, batch["target_audio_rows"])
            loss, finite = fs.finite_or_zero(loss)
        with fs.phase("backward"):
            loss.backward()
        lr = lr_at(step, sched)
        fs.set_group_lrs(optimizer, lr)
        gnorm = fs.clip_gradients(trainable, opt_cfg.grad_clip)
        optimizer.step()
        optimizer.zero_grad(set_to_none=True)
        prof_ctx.__exit__(None, None, None)
        step += 1
        m = _reduce_metrics({"loss": loss.item(), "loss_teacher": loss_teacher.item(),
                             "data_video": data_v.item(), "data_audio": data_a.item(),
                             "excess_vs_teacher": (data_v - teacher_data).item(),
                             "finite": float(finite)}, device)
        rec = {"step": step, "lr": lr, "grad_norm": gnorm, "step_s": time.perf_counter() - t0,
               **m, **fs.phase_fields()}
        if torch.cuda.is_available():
            rec["peak_gib"] = torch.cuda.max_memory_allocated() / 2 ** 30
        write(rec)
        select_w = fs.trainable_select(include_lora=stage == "b")
        if step % cfg.checkpoint.save_every == 0 or step in cfg.checkpoint.early_saves or step == cfg.training.max_steps:
            name = ("hybrid_lora" if stage == "b" else "hybrid") + f"_step{step:06d}.pt"
            fs.save_weights_artifact(model, out, name, stage, step, spec_dict, select_w)
            fs.save_train_state(model, optimizer, select_w, stage, step, spec_dict, resolved_dict(cfg),
                                gens, out, f"train_state_step{step:06d}.pt",
                                data_cursor=(step * world) % max(len(dataset), 1) // world,
                                extra={"schedule": schedule_stamp(sched)},
                                keep_states=cfg.checkpoint.keep_states)
    if hb is not None:
        hb.stop()
    fs.close_comms(model)
    if fs.rank0():
        open(os.path.join(out, "DONE"), "w").close()
        run_lock.release(out)
    return step


def run_stage_a2(cfg):
    return _fsdp_stage(cfg, "a2")


def run_stage_b(cfg):
    return _fsdp_stage(cfg, "b")


# -------------------------------------------------------------------------------- A1
class AlignHook:
    """Forward hook on a HybridAttention running in teacher_mode: re-run the hybrid on the
    detached input and backpropagate the normalised alignment error of this layer now."""

    def __init__(self, layer_index):
        self.index = layer_index
        self.losses = []

    def __call__(self, module, args, output):
        if not torch.is_grad_enabled() and not getattr(module, "_align_active", False):
            return None
        hidden, rotary = args[0], args[1] if len(args) > 1 else None
        target = output.detach()
        with torch.enable_grad():
            student = module.hybrid_forward(hidden[0].detach(), rotary)
            err = (student.float() - target[0].float()).pow(2).sum() / target.float().pow(2).sum().clamp_min(1e-12)
            err.backward()
        self.losses.append(err.item())
        if not dist.is_initialized() or dist.get_rank() == 0:
            debug_memory_line(f"block {self.index:2d}")
        return None


def _bucketed(tensors, collective):
    """Runs `collective` once per dtype on one flat buffer holding all of `tensors`, then
    copies the result back (one NCCL call per layer instead of one per parameter)."""
    by_dtype = {}
    for t in tensors:
        by_dtype.setdefault(t.dtype, []).append(t)
    for group in by_dtype.values():
        flat = torch.cat([t.reshape(-1) for t in group])
        collective(flat)
        offset = 0
        for t in group:
            t.copy_(flat[offset:offset + t.numel()].view_as(t))
            offset += t.numel()


def run_stage_a1(cfg):
    out = cfg.checkpoint.output_dir
    fs.refuse_if_guarded(out, os.path.join(out, "DONE"))
    world, rank, device = _dist_setup(cfg.training.seed)
    if rank == 0:
        run_lock.acquire(out)
    from vdn_minimax_h3_b200.models.factory import h3_config_from_resolved
    from vdn_minimax_h3_b200.models.h3 import h3_full_config
    base = cfg.model.base
    from vdn_minimax_h3_b200.models.h3 import H3Config
    loaded = (H3Config.from_dict(dict(cfg.model.base.config_overrides)).to_dict()
              if cfg.model.base.config_overrides else h3_full_config().to_dict())
    section = {"base": dict(library=base.library, class_name=base.class_name, source=base.source,
                            subfolder=base.subfolder, revision=base.revision, dtype=base.dtype),
               "architecture": resolved_dict(cfg)["model"]["architecture"]}
    spec = resolve_model_spec(section, loaded)
    spec_dict = spec.to_dict()
    model = build_model(spec, device="cpu", init=_init_mode(base.source), seed=cfg.training.seed)
    if cfg.training.truncate_blocks:
        model.transformer_blocks = model.transformer_blocks[:cfg.training.truncate_blocks]
    select = fs.trainable_select(include_lora=False)
    _prepare_trainables(model, select)
    if cfg.training.freeze_softmax_gate:
        for attn in iter_hybrids(model):
            if attn.enable_softmax_gate:
                attn.softmax_gate.requires_grad_(False)
    model.to(device)
    if torch.device(device).type == "cuda":
        from vdn_minimax_h3_b200.ops.linear_grad import route_training_linears
        route_training_linears(model)
    if world > 1:
        from vdn_minimax_h3_b200.utils.distributed import broadcast_and_verify_init
        broadcast_and_verify_init(model, [p for p in model.parameters() if p.requires_grad], device)
    layers = hybrid_new_parameters(model)
    hooks = []
    for (idx, _), attn in zip(layers, iter_hybrids(model)):
        h = AlignHook(idx)
        attn._align_active = True
        hooks.append(h)
        attn.register_forward_hook(h)
    set_teacher_mode(model, True)
    opt_cfg = cfg.optimizer
    # ZeRO-1: the optimizer of layer i lives on rank i % world
    optimizers = {}
    for (idx, named), attn in zip(layers, iter_hybrids(model)):
        if idx % world != rank:
            continue
        params = [p for _, p in named if p.requires_grad]
        groups = fs.build_param_groups(model, opt_cfg.lr, big_scale=opt_cfg.big_lr_scale,
                                       small_scale=opt_cfg.small_lr_scale, small_eps=opt_cfg.small_eps,
                                       select=lambda n, p, ok={id(q) for q in params}: id(p) in ok)
        optimizers[idx] = torch.optim.AdamW(groups, lr=opt_cfg.lr, weight_decay=opt_cfg.weight_decay)
    sched = _sched_args(opt_cfg, cfg.training.max_steps)
    gens = fs.make_generators(cfg.training.seed, rank, device)
    dataset = _load_dataset(cfg)
    loader, sampler = fs.make_loader(dataset, world, rank, cfg.training.seed,
                                      getattr(cfg.data, "num_workers", 0))
    write = _metrics_writer(out)
    step = 0
    it = iter(loader)
    while step < cfg.training.max_steps:
        try:
            sample = next(it)
        except StopIteration:
            it = iter(loader)
            sample = next(it)
        for h in hooks:
            h.losses.clear()
        batch = pack_noisy_batch(sample, device, gens["noise"], gens["sigma"])
        set_layout(model, batch["layout"])
        with torch.no_grad():
            model(**batch["inputs"])               # teacher trunk; the hooks train each layer
        lr = lr_at(step, sched)
        norms = {}
        for (idx, named), attn in zip(layers, iter_hybrids(model)):
            params = [p for _, p in named if p.requires_grad]
            if world > 1:
                for p in params:
                    if p.grad is None:
                        p.grad = torch.zeros_like(p)
                _bucketed([p.grad for p in params],
                          lambda flat: dist.all_reduce(flat, op=dist.ReduceOp.AVG))
            norms[idx] = fs.clip_gradients(params, opt_cfg.grad_clip)
            if idx in optimizers:
                fs.set_group_lrs(optimizers[idx], lr)
                optimizers[idx].step()
            for p in params:
                p.grad = None
            if world > 1:
                _bucketed([p.data for p in params], lambda flat, src=idx % world: dist.broadcast(flat, src=src))
        step += 1
        rel = _reduce_metrics({f"rel_{h.index}": (h.losses[-1] if h.losses else 0.0) for h in hooks}, device)
        write({"step": step, "lr": lr, "rel_mean": sum(rel.values()) / max(len(rel), 1),
               **rel, **{f"grad_norm_{k}": v for k, v in norms.items()}})
        if step % cfg.checkpoint.save_every == 0 or step in cfg.checkpoint.early_saves or step == cfg.training.max_steps:
            meta = {"truncated": True} if cfg.training.truncate_blocks else {}
            fs.save_weights_artifact(model, out, f"hybrid_step{step:06d}.pt", "a1", step, spec_dict,
                                     select, metadata=meta)
    set_teacher_mode(model, False)
    if fs.rank0():
        open(os.path.join(out, "DONE"), "w").close()
        run_lock.release(out)
    return step


# ------------------------------------------------------------------------------- DMD
def dmd_sub_iteration(model, roles, schedule, packed, xv, xa, k, kind, gens, optimizer,
                      gen_params, fake_params, gen_lr, fake_lr, u_range, shifts, audio_weight,
                      clips):
    """One Stage-DMD sub-iteration after the rollout (xv, xa at grid step k): on a generator
    turn the DM-loss update of `turbo` (generator x0 with a graph, real and fake score x0 at a
    fresh (x_t, t), the distribution-matching gradient); on every turn the fake score's
    flow-matching update on the detached generator sample. Optimizer group 0 is the
    generator's, group 1 the fake score's. Returns the turn's metrics."""
    rec = {}
    dev = xv.device
    if kind == dmd_lib.GENERATOR_TURN:
        x0v, x0a = dmd_lib.generator_x0(model, roles, schedule, packed, xv, xa, k, build_graph=True)
        t_v, t_a, _ = sample_paired_timesteps(gens["sigma"], *u_range, *shifts)
        nv = torch.randn(x0v.shape, generator=gens["noise"], device=dev)
        na = torch.randn(x0a.shape, generator=gens["noise"], device=dev)
        xt_v, xt_a = dmd_lib.noised(x0v.detach(), t_v, nv), dmd_lib.noised(x0a.detach(), t_a, na)
        rv, ra = dmd_lib.score_x0(model, roles, dmd_lib.REAL, packed, xt_v, xt_a, t_v, t_a)
        fv, fa = dmd_lib.score_x0(model, roles, dmd_lib.FAKE, packed, xt_v, xt_a, t_v, t_a)
        lv, normv, gapv = dmd_lib.distribution_matching_loss(x0v, rv, fv)
        la, _, _ = dmd_lib.distribution_matching_loss(x0a, ra, fa)
        loss, _ = fs.finite_or_zero(lv + audio_weight * la)
        dmd_lib.require_role(roles, dmd_lib.GENERATOR, "generator backward")
        loss.backward()
        for p in fake_params:
            p.grad = None
        optimizer.param_groups[0]["lr"] = gen_lr
        optimizer.param_groups[1]["lr"] = 0.0
        rec.update(dm_loss=loss.item(), dm_norm_video=normv.item(), dm_gap_video=gapv.item(),
                   grad_norm_turbo=fs.clip_gradients(gen_params, clips[0]))
        optimizer.step()
        optimizer.zero_grad(set_to_none=True)
        x0v, x0a = x0v.detach(), x0a.detach()
    else:
        x0v, x0a = dmd_lib.generator_x0(model, roles, schedule, packed, xv, xa, k, build_graph=False)
    # fake-score flow-matching update on the (detached) generator sample
    roles.set(dmd_lib.FAKE)
    t_v, t_a, _ = sample_paired_timesteps(gens["sigma"], *u_range, *shifts)
    nv = torch.randn(x0v.shape, generator=gens["noise"], device=dev)
    na = torch.randn(x0a.shape, generator=gens["noise"], device=dev)
    vel_v, vel_a = model(**packed.inputs(dmd_lib.noised(x0v, t_v, nv), dmd_lib.noised(x0a, t_a, na), t_v, t_a))
    floss = dmd_lib.fake_regression_loss(vel_v[0].float(), x0v, nv) + \
        audio_weight * dmd_lib.fake_regression_loss(vel_a[0].float(), x0a, na)
    floss, _ = fs.finite_or_zero(floss)
    floss.backward()
    for p in gen_params:
        p.grad = None
    optimizer.param_groups[0]["lr"] = 0.0
    optimizer.param_groups[1]["lr"] = fake_lr
    rec.update(fake_loss=floss.item(), grad_norm_fake=fs.clip_gradients(fake_params, clips[1]))
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    return rec


def run_stage_dmd(cfg):
    out = cfg.checkpoint.output_dir
    fs.refuse_if_guarded(out, os.path.join(out, "DONE"), cfg.training.ignore_stopped)
    world, rank, device = _dist_setup(cfg.training.seed)
    if rank == 0:
        run_lock.acquire(out)
    from vdn_minimax_h3_b200.checkpoints.loader import load_checkpoint
    seed_art = load_checkpoint(cfg.initialization.checkpoint)
    spec = ModelSpec.from_dict(seed_art.model_spec)
    src = cfg.initialization.base_source or spec.base.source
    model = build_model(spec, device="cpu", base_source=src, init=_init_mode(src), seed=cfg.training.seed)
    load_model_weights(model, {k: v for k, v in seed_art.weights.items() if ".lora_" not in k}, strict=False)
    targets = ["attn.orig.to_q", "attn.orig.to_k", "attn.orig.to_v", "attn.orig.to_out.0"]
    vdn_cfg = spec.adapters[0].config if spec.adapters else {"rank": 64, "alpha": 64, "targets": targets}
    inject_lora(model, "default", vdn_cfg["rank"], vdn_cfg["alpha"], vdn_cfg["targets"])
    lora_w = {k: v for k, v in seed_art.weights.items() if ".lora_" in k}
    if lora_w:
        load_model_weights(model, lora_w, strict=False)
    tb = cfg.turbo
    inject_lora(model, tb.adapter_name, vdn_cfg["rank"], vdn_cfg["alpha"], vdn_cfg["targets"], init_b_zero=False)
    if tb.checkpoint and tb.checkpoint != "synthetic":
        from vdn_minimax_h3_b200.inference.lora import load_external_lora
        state, _, _ = load_external_lora(tb.checkpoint)
        renamed = {k.replace(".lora_A.", f".lora_A.{tb.adapter_name}.").replace(".lora_B.", f".lora_B.{tb.adapter_name}.")
                   .replace(".attn.", ".attn.orig.", 1): v for k, v in state.items()}
        load_model_weights(model, renamed, strict=False)
    d = cfg.dmd
    inject_lora(model, d.fake_adapter_name, d.fake_rank, d.fake_rank, vdn_cfg["targets"], init_b_zero=True)

    def select(name, p):
        return f".lora_A.{tb.adapter_name}." in name or f".lora_B.{tb.adapter_name}." in name or \
            f".lora_A.{d.fake_adapter_name}." in name or f".lora_B.{d.fake_adapter_name}." in name
    _prepare_trainables(model, select)
    model.to(device)
    if world > 1:
        from vdn_minimax_h3_b200.utils.distributed import broadcast_and_verify_init
        broadcast_and_verify_init(model, [p for p in model.parameters() if p.requires_grad], device)
    if world > 1 or torch.device(device).type == "cuda":
        fs.shard_model(model, device, cfg.distributed.shard_size, cfg.distributed.activation_checkpointing)
    gen_params = [p for n, p in model.named_parameters() if p.requires_grad and f".{tb.adapter_name}." in n]
    fake_params = [p for n, p in model.named_parameters() if p.requires_grad and f".{d.fake_adapter_name}." in n]
    o = cfg.optimizer
    optimizer = torch.optim.AdamW([{"params": gen_params, "name": "turbo"},
                                   {"params": fake_params, "name": "fake"}], lr=o.lr, weight_decay=o.weight_decay)
    roles = dmd_lib.Roles(model, d.real_score, "default", tb.adapter_name, d.fake_adapter_name)
    schedule = dmd_lib.FewStepSchedule(tb.num_steps, tb.video_shift, tb.audio_shift)
    gens = fs.make_generators(cfg.training.seed, rank, device)
    dataset = _load_dataset(cfg, text_only=True)
    loader, sampler = fs.make_loader(dataset, world, rank, cfg.training.seed,
                                      getattr(cfg.data, "num_workers", 0))
    g = cfg.generation
    from vdn_minimax_h3_b200.models.layout import align_num_frames, audio_latent_num_frames, video_latent_num_frames
    nf = align_num_frames(g.num_frames)
    video_shape = (model.config.in_channels, video_latent_num_frames(nf), g.latent_height, g.latent_width)
    n_audio = audio_latent_num_frames(nf)
    gen_sched = SimpleNamespace(lr=o.lr, min_lr=o.min_lr, warmup_steps=o.warmup_steps, max_steps=cfg.training.max_steps)
    fake_sched = SimpleNamespace(lr=o.fake_lr, min_lr=o.fake_min_lr, warmup_steps=o.fake_warmup_steps,
                                 max_steps=cfg.training.max_steps * d.fake_updates_per_step + d.fake_warmup_steps)
    write = _metrics_writer(out)
    gen_step = fake_step = iteration = 0
    it = iter(loader)
    while gen_step < cfg.training.max_steps:
        try:
            sample = next(it)
        except StopIteration:
            it = iter(loader)
            sample = next(it)
        kind = dmd_lib.turn(fake_step, d.fake_warmup_steps, d.fake_updates_per_step)
        packed = PackedPrompt(sample["prompt_embeds"], video_shape, n_audio, device)
        set_layout(model, packed.layout)
        k = dmd_lib.shared_rollout_index(cfg.training.seed, iteration, schedule.num_steps)
        v0, a0 = initial_noise(video_shape, n_audio, gens["noise"], device)
        xv, xa = dmd_lib.rollout(model, roles, schedule, packed, v0, a0, k)
        rec = {"iteration": iteration, "turn": kind, "rollout_k": k}
        rec.update(dmd_sub_iteration(
            model, roles, schedule, packed, xv, xa, k, kind, gens, optimizer, gen_params, fake_params,
            gen_lr=lr_at(gen_step, gen_sched), fake_lr=lr_at(fake_step, fake_sched),
            u_range=(d.u_min, d.u_max), shifts=(tb.video_shift, tb.audio_shift),
            audio_weight=cfg.training.audio_loss_weight, clips=(o.grad_clip, o.fake_grad_clip)))
        if kind == dmd_lib.GENERATOR_TURN:
            gen_step += 1
        fake_step += 1
        iteration += 1
        rec.update(gen_step=gen_step, fake_step=fake_step)
        write(rec)
        if kind == dmd_lib.GENERATOR_TURN and (gen_step % cfg.checkpoint.save_every == 0 or gen_step == cfg.training.max_steps):
            fs.save_weights_artifact(model, out, f"turbo_step{gen_step:06d}.pt", "dmd", gen_step,
                                     spec.to_dict(), lambda n, p: f".{tb.adapter_name}." in n and "lora_" in n,
                                     metadata={"fake_step": fake_step, "iteration": iteration})
    set_active_adapters(model, ["default", tb.adapter_name])
    if fs.rank0():
        open(os.path.join(out, "DONE"), "w").close()
        run_lock.release(out)
    return gen_step
