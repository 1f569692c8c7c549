"""The machinery every FSDP2 stage shares: phase timers, teacher / student forwards, run
guards, fingerprinted weight saves, resumable train states, two-phase resume, sharding,
parameter groups, clipping, data loading and RNG streams.

Reference parity: src/training/fsdp_stage.py:38-507. Sharding is torch's FSDP2
(`fully_shard`) per DiT block and per refiner block with a (replicate, shard) device mesh
for HSDP, bf16 compute with fp32 reduction, and the alpha modules in their own fp32 policy;
two-level activation checkpointing (utils/activation_checkpointing.py); saved activations
optionally offloaded to pinned host memory.
"""
import glob
import os
import re
import time
from collections import OrderedDict, defaultdict
from contextlib import contextmanager

import torch
import torch.distributed as dist

from vdn_minimax_h3_b200.checkpoints.schema import CheckpointArtifact
from vdn_minimax_h3_b200.checkpoints.writer import save_checkpoint
from vdn_minimax_h3_b200.models.hybrid_transform import is_transform_parameter, set_teacher_mode
from vdn_minimax_h3_b200.models.lora import set_adapters_enabled
from vdn_minimax_h3_b200.utils import run_lock
from vdn_minimax_h3_b200.utils.lr_classes import lr_class_map
from vdn_minimax_h3_b200.utils.samplers import SkipFirst

# ------------------------------------------------------------------------------ timers
_PHASES = OrderedDict()


def phase_reset():
    _PHASES.clear()


class phase:
    """Synchronising wall-clock timer of one named phase of a step (device work included)."""

    def __init__(self, name):
        self.name = name

    def __enter__(self):
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        _PHASES[self.name] = _PHASES.get(self.name, 0.0) + time.perf_counter() - self.t0
        return False


def phase_fields(prefix="t_"):
    return {prefix + k: round(v, 3) for k, v in _PHASES.items()}


# ------------------------------------------------------------------------- forwards
@torch.no_grad()
def teacher_velocity(model, inputs, adapters=False):
    """The dense teacher (teacher_mode, adapters off when `adapters`) on the same inputs."""
    set_teacher_mode(model, True)
    if adapters:
        set_adapters_enabled(model, False)
    try:
        v, a = model(**inputs)
        return v[0].detach().float(), a[0].detach().float()
    finally:
        set_teacher_mode(model, False)
        if adapters:
            set_adapters_enabled(model, True)
        if torch.cuda.is_available():
            torch.cuda.empty_cache()


def student_forward(model, inputs, offload_activations):
    if offload_activations:
        with torch.autograd.graph.save_on_cpu(pin_memory=torch.cuda.is_available()):
            return model(**inputs)
    return model(**inputs)


def finite_or_zero(loss):
    """A non-finite loss becomes 0 * loss THROUGH the graph, so every rank still reaches the
    same reduce-scatters (a skipped backward would desynchronise FSDP)."""
    if torch.isfinite(loss):
        return loss, True
    return loss * 0.0 if torch.isfinite(loss * 0.0) else torch.nan_to_num(loss) * 0.0, False


# --------------------------------------------------------------------------- guards
def rank0():
    return not dist.is_initialized() or dist.get_rank() == 0


def refuse_if_guarded(out_dir, done_path=None, ignore_stopped=False):
    """Before any model is loaded: a STOPPED marker, a finished run, or a live lock holder
    end the job with a message instead of overwriting anything."""
    if os.path.exists(os.path.join(out_dir, "STOPPED")) and not ignore_stopped:
        raise SystemExit(f"{out_dir}/STOPPED exists; remove it (or ignore_stopped=true) to continue")
    if done_path and os.path.exists(done_path):
        raise SystemExit(f"{done_path} exists: this run already finished")
    holder = run_lock.check(out_dir)
    if holder is not None:
        raise SystemExit(f"{out_dir} is locked by job {holder['job_id']}")


# ---------------------------------------------------------------------- saving
def _full(t):
    return t.full_tensor() if hasattr(t, "full_tensor") else t


def gather_named(model, select):
    """{name: full fp32 CPU tensor} of the selected parameters; every rank takes part in the
    all-gathers, rank 0 keeps the result."""
    out = {}
    for name, p in model.named_parameters():
        if select(name, p):
            full = _full(p.detach())
            if rank0():
                out[name] = full.float().cpu().clone()
    return out


def fingerprint(weights):
    return {k: float(v.double().sum()) for k, v in weights.items()}


def verify_fingerprint(saved_path, weights):
    """Re-read a save and compare an fp64 fingerprint of every tensor."""
    back = torch.load(saved_path, map_location="cpu", weights_only=True)["weights"]
    want, got = fingerprint(weights), fingerprint(back)
    bad = [k for k in want if got.get(k) != want[k]]
    if bad:
        raise RuntimeError(f"{saved_path}: {len(bad)} tensors changed on disk, e.g. {bad[:3]}")


def save_weights_artifact(model, out_dir, filename, stage, step, spec_dict, select, metadata=None):
    weights = gather_named(model, select)
    path = None
    if rank0():
        meta = {"stage": stage, "step": step, **(metadata or {})}
        art = CheckpointArtifact(kind="weights", model_spec=spec_dict, weights=weights, metadata=meta)
        path = save_checkpoint(art, os.path.join(out_dir, filename))
        verify_fingerprint(path, weights)
    if dist.is_initialized():
        dist.barrier()
    return path


def _rng_state(generators):
    state = {"torch": torch.get_rng_state()}
    if torch.cuda.is_available():
        state["cuda"] = torch.cuda.get_rng_state()
    for k, g in generators.items():
        state[k] = g.get_state()
    return state


def save_train_state(model, optimizer, select, stage, step, spec_dict, resolved_config, generators,
                     out_dir, filename, data_cursor=0, epoch=0, extra=None, keep_states=3):
    """Weights + name-keyed optimizer moments (full tensors) + per-rank RNG + config."""
    weights = gather_named(model, select)
    names = {id(p): n for n, p in model.named_parameters()}
    opt_state = {}
    for group in optimizer.param_groups:
        for p in group["params"]:
            st = optimizer.state.get(p)
            if not st:
                continue
            full = {k: (_full(v).float().cpu().clone() if torch.is_tensor(v) and v.dim() > 0 else
                        (v.cpu() if torch.is_tensor(v) else v)) for k, v in st.items()}
            if rank0():
                opt_state[names[id(p)]] = full
    rng = _rng_state(generators)
    rngs = [None] * (dist.get_world_size() if dist.is_initialized() else 1)
    if dist.is_initialized():
        dist.all_gather_object(rngs, rng)
    else:
        rngs = [rng]
    path = None
    if rank0():
        meta = {"stage": stage, "epoch": epoch, "data_cursor": data_cursor,
                "world_size": len(rngs), **(extra or {})}
        art = CheckpointArtifact(kind="train_state", model_spec=spec_dict, weights=weights,
                                 optimizer=opt_state, step=step, rng_state={"per_rank": rngs},
                                 resolved_training_config=resolved_config, metadata=meta)
        path = save_checkpoint(art, os.path.join(out_dir, filename))
        states = sorted(glob.glob(os.path.join(out_dir, "train_state_step*.pt")))
        for old in states[:-keep_states]:
            os.remove(old)
    if dist.is_initialized():
        dist.barrier()
    return path


# --------------------------------------------------------------------------- resume
class Resume:
    def __init__(self):
        self.path = None
        self.step = 0
        self.artifact = None


def _step_of(path):
    m = re.search(r"step(\d+)", os.path.basename(path))
    return int(m.group(1)) if m else -1


def find_resume(out_dir, spec_dict, model):
    """Phase one (before sharding): the newest train_state (else weights) in out_dir, its
    weights copied into the model. A ModelSpec that differs from this run's is refused."""
    from vdn_minimax_h3_b200.checkpoints.loader import load_checkpoint
    r = Resume()
    cands = sorted(glob.glob(os.path.join(out_dir, "train_state_step*.pt")), key=_step_of)
    if not cands:
        cands = sorted(glob.glob(os.path.join(out_dir, "*_step*.pt")), key=_step_of)
    if not cands:
        return r
    art = load_checkpoint(cands[-1])
    if art.model_spec != spec_dict:
        raise RuntimeError(f"{cands[-1]} was written for a different ModelSpec; refusing to resume")
    params = dict(model.named_parameters())
    with torch.no_grad():
        for k, v in art.weights.items():
            if k in params:
                params[k].copy_(v.to(params[k].dtype))
    r.path, r.step, r.artifact = cands[-1], (art.step or _step_of(cands[-1])), art
    return r


def restore_optimizer_and_rng(resume, model, optimizer, generators):
    """Phase two (after sharding and optimizer construction): moments distributed onto the
    shards, RNG restored for this rank (when the world size matches)."""
    art = resume.artifact
    if art is None or art.kind != "train_state":
        return 0
    names = {n: p for n, p in model.named_parameters()}
    for name, st in (art.optimizer or {}).items():
        p = names.get(name)
        if p is None:
            continue
        new = {}
        for k, v in st.items():
            if torch.is_tensor(v) and v.dim() > 0:
                if hasattr(p, "device_mesh"):
                    from torch.distributed.tensor import distribute_tensor
                    new[k] = distribute_tensor(v.to(p.device), p.device_mesh, p.placements)
                else:
                    new[k] = v.to(p.device)
            else:
                new[k] = v
        optimizer.state[p] = new
    rngs = art.rng_state.get("per_rank", [])
    rank = dist.get_rank() if dist.is_initialized() else 0
    if len(rngs) == (dist.get_world_size() if dist.is_initialized() else 1):
        st = rngs[rank]
        torch.set_rng_state(st["torch"])
        if "cuda" in st and torch.cuda.is_available():
            torch.cuda.set_rng_state(st["cuda"])
        for k, g in generators.items():
            if k in st:
                g.set_state(st[k])
    return int(art.metadata.get("data_cursor", 0))


# ------------------------------------------------------------------------- sharding
def shard_model(model, device, shard_size=None, activation_checkpointing=True, split_ac=True,
                param_dtype=torch.bfloat16, reduce_dtype=torch.float32, symmetric_reduce=None,
                kernel_linears=True, symmetric_gather=None):
    """fully_shard each refiner block and DiT block (alpha modules first, in fp32), then the
    root; HSDP when the world is larger than `shard_size`. On CUDA every nn.Linear first gets
    the GEMM-kernel forward / dgrad / wgrad of ops/linear_grad.py (`kernel_linears`; the
    module switch linear_grad.LINEAR_KERNELS turns it off at run time). With `symmetric_reduce` (default:
    on for CUDA shard groups of 2-8 ranks) the gradient reduce-scatter of every unit runs over
    symmetric memory (parallel/fsdp_comm.py) instead of NCCL, and with `symmetric_gather`
    (same default) the parameter all-gather as well -- both only when the shard group's ranks
    share one host (CUDA IPC); the comm objects are kept as
    `model._vdn_reduce_comm` / `model._vdn_gather_comm` (`close_comms(model)` before
    destroying the process group)."""
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard
    from vdn_minimax_h3_b200.utils.activation_checkpointing import enable_block_checkpointing
    world = dist.get_world_size()
    shard = min(shard_size or world, world)
    if world % shard:
        raise ValueError(f"world {world} is not a multiple of shard_size {shard}")
    dev_type = torch.device(device).type
    if kernel_linears and dev_type == "cuda":
        from vdn_minimax_h3_b200.ops.linear_grad import route_training_linears
        route_training_linears(model)
    if world // shard > 1:
        mesh = init_device_mesh(dev_type, (world // shard, shard), mesh_dim_names=("replicate", "shard"))
    else:
        mesh = init_device_mesh(dev_type, (world,), mesh_dim_names=("shard",))
    if activation_checkpointing:
        enable_block_checkpointing(model, split=split_ac)
    mp = MixedPrecisionPolicy(param_dtype=param_dtype, reduce_dtype=reduce_dtype)
    mp32 = MixedPrecisionPolicy(param_dtype=torch.float32, reduce_dtype=torch.float32)
    for block in model.transformer_blocks:
        alpha = getattr(getattr(block.attn, "linear_attention", None), "alpha", None)
        if alpha is not None:
            fully_shard(alpha, mesh=mesh, mp_policy=mp32)
        fully_shard(block, mesh=mesh, mp_policy=mp)
    for blk in model.token_refiner.refiner_blocks:
        fully_shard(blk, mesh=mesh, mp_policy=mp)
    fully_shard(model, mesh=mesh, mp_policy=mp)
    one_host = dev_type == "cuda" and 1 < shard <= 8 and _group_on_one_host(mesh.get_group("shard"))
    if symmetric_reduce is None:
        symmetric_reduce = one_host
    if symmetric_reduce:
        from torch.distributed.fsdp import FSDPModule
        from vdn_minimax_h3_b200.parallel.fsdp_comm import SymmetricReduceScatter, trainable_reduce_numel
        units = [m for m in model.modules() if isinstance(m, FSDPModule)]
        blocks = list(model.transformer_blocks) + list(model.token_refiner.refiner_blocks)
        in_blocks = {id(p) for b in blocks for p in b.parameters()}
        groups = [list(b.parameters()) for b in blocks]      # (a block's alpha unit included)
        groups.append([p for p in model.parameters() if id(p) not in in_blocks])
        shard_group = mesh.get_group("shard")
        comm = SymmetricReduceScatter(shard_group, device, trainable_reduce_numel(groups, shard))
        if comm.enabled():
            for u in units:
                u.set_custom_reduce_scatter(comm)
        model._vdn_reduce_comm = comm
    if symmetric_gather is None:
        symmetric_gather = one_host
    if symmetric_gather:
        from torch.distributed.fsdp import FSDPModule
        from vdn_minimax_h3_b200.parallel.fsdp_comm import SymmetricAllGather, gather_shard_bytes
        units = [m for m in model.modules() if isinstance(m, FSDPModule)]
        blocks = list(model.transformer_blocks) + list(model.token_refiner.refiner_blocks)
        in_blocks = {id(p) for b in blocks for p in b.parameters()}
        groups = [list(b.parameters()) for b in blocks]
        groups.append([p for p in model.parameters() if id(p) not in in_blocks])
        comm = SymmetricAllGather(mesh.get_group("shard"), device, gather_shard_bytes(groups, shard))
        if comm.enabled():
            for u in units:
                u.set_custom_all_gather(comm)
        model._vdn_gather_comm = comm
    return model


def _group_on_one_host(group):
    """True when every rank of `group` runs on this host (the symmetric heaps map peers'
    memory through CUDA IPC, which does not cross nodes)."""
    import socket
    names = [None] * dist.get_world_size(group)
    dist.all_gather_object(names, socket.gethostname(), group=group)
    return len(set(names)) == 1


def close_comms(model):
    """Release the symmetric heaps of the FSDP comms `shard_model` installed."""
    for name in ("_vdn_reduce_comm", "_vdn_gather_comm"):
        comm = getattr(model, name, None)
        if comm is not None:
            comm.close()


def trainable_select(include_lora=True, adapter_names=None):
    def select(name, p):
        if "lora_" in name:
            if not include_lora:
                return False
            return adapter_names is None or any(f".lora_A.{a}." in name or f".lora_B.{a}." in name
                                                for a in adapter_names)
        return is_transform_parameter(name)
    return select


def build_param_groups(model, base_lr, big_scale=1.0, small_scale=1.0, small_eps=None,
                       lora_scale=1.0, select=None):
    """AdamW groups: lora, branch_big, branch_small (structural classes, utils/lr_classes)."""
    classes = lr_class_map(model)
    groups = defaultdict(list)
    for name, p in model.named_parameters():
        if not p.requires_grad or (select is not None and not select(name, p)):
            continue
        if "lora_" in name:
            groups["lora"].append(p)
        else:
            groups["branch_" + classes.get(id(p), "big")].append(p)
    out = []
    for name, params in groups.items():
        scale = {"lora": lora_scale, "branch_big": big_scale, "branch_small": small_scale}[name]
        g = {"params": params, "name": name, "lr_scale": scale, "lr": base_lr * scale}
        if name == "branch_small" and small_eps is not None:
            g["eps"] = small_eps
        out.append(g)
    return out


def set_group_lrs(optimizer, lr):
    for g in optimizer.param_groups:
        g["lr"] = lr * g.get("lr_scale", 1.0)


def clip_gradients(params, grad_clip):
    """Global-norm clipping that also works on sharded (DTensor) gradients."""
    params = [p for p in params if p.grad is not None]
    if not params or grad_clip <= 0:
        return 0.0
    norm = torch.nn.utils.clip_grad_norm_(params, grad_clip)
    return float(_full(norm)) if torch.is_tensor(norm) else float(norm)


def make_loader(dataset, world, rank, seed, num_workers=0, pin_memory=None):
    """One clip per rank per step (DistributedSampler behind SkipFirst for resumes).
    `num_workers` reader processes (the config's data.num_workers) keep the next clips'
    latents loading while the step runs; on CUDA the batches land in pinned host memory so
    the copies to the GPU are DMA transfers."""
    from torch.utils.data import DataLoader, DistributedSampler
    from vdn_minimax_h3_b200.training.dataset import collate_single
    if pin_memory is None:
        pin_memory = torch.cuda.is_available()
    sampler = SkipFirst(DistributedSampler(dataset, num_replicas=world, rank=rank, shuffle=True, seed=seed))
    # workers come from a forkserver, not a fork of this (multi-threaded: NCCL, heartbeat)
    # process, which can leave a lock held in the child
    extra = ({"persistent_workers": True, "prefetch_factor": 2,
              "multiprocessing_context": "forkserver"} if num_workers > 0 else {})
    loader = DataLoader(dataset, batch_size=1, sampler=sampler, num_workers=num_workers,
                        collate_fn=collate_single, pin_memory=pin_memory, **extra)
    return loader, sampler


def make_generators(seed, rank, device):
    dev = torch.device(device)
    noise = torch.Generator(device=dev).manual_seed(seed * 1000 + rank)
    sigma = torch.Generator().manual_seed(seed * 1000 + rank + 7)
    return {"noise": noise, "sigma": sigma}
