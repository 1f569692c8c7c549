"""Training stack on CPU: schedule and DMD maths, live LoRA, and tiny end-to-end runs of
stages A1, A2, B and DMD (gloo; one rank, and two ranks under FSDP2 for A2)."""
import glob
import json
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vdn_minimax_h3_b200.config import load_config
from vdn_minimax_h3_b200.config.schemas import StageA1Config, StageA2Config, StageBConfig, StageDMDConfig
from vdn_minimax_h3_b200.models.factory import TINY_HYBRID, build_model, make_spec
from vdn_minimax_h3_b200.models.h3 import h3_tiny_config
from vdn_minimax_h3_b200.models.lora import inject_lora, merge_and_unload, set_active_adapters
from vdn_minimax_h3_b200.training import dmd
from vdn_minimax_h3_b200.training.batch import euler_blend, few_step_sigmas, few_step_timesteps
from vdn_minimax_h3_b200.utils.lr_schedule import check_schedule_stamp, lr_at, schedule_stamp
from types import SimpleNamespace

TINY_DATA = "synthetic:4:16x3x16x16:4:8:256"


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_lr_schedule():
    a = SimpleNamespace(lr=1.0, min_lr=0.1, warmup_steps=4, max_steps=14)
    assert lr_at(0, a) == 0.25 and lr_at(3, a) == 1.0
    assert abs(lr_at(14, a) - 0.1) < 1e-9
    assert check_schedule_stamp(schedule_stamp(a), SimpleNamespace(lr=2.0, min_lr=0.1, warmup_steps=4, max_steps=14), rank=1) \
        == {"lr": (1.0, 2.0)}


def test_dmd_maths():
    assert dmd.turn(0, 2, 3) == dmd.WARMUP_TURN
    assert [dmd.turn(k, 2, 3) for k in range(2, 8)] == ["generator", "fake", "fake"] * 2
    assert dmd.shared_rollout_index(3, 17, 8) == dmd.shared_rollout_index(3, 17, 8)
    x0_g = torch.randn(50, requires_grad=True)
    x0_r, x0_f = torch.randn(50), torch.randn(50)
    loss, norm, _ = dmd.distribution_matching_loss(x0_g, x0_r, x0_f)
    loss.backward()
    g = (x0_f - x0_r) / (x0_g.detach() - x0_r).abs().mean()
    assert torch.allclose(x0_g.grad, g / 50, atol=1e-6)
    sched = dmd.FewStepSchedule(8, 12.0, 3.0)
    tv, _ = few_step_timesteps(8, 12.0, 3.0)
    sv, _ = few_step_sigmas(8, 12.0, 3.0)
    x, v = torch.randn(10), torch.randn(10)
    a, _ = sched.step(2, x, torch.zeros(1), v, torch.zeros(1))
    assert torch.allclose(a, euler_blend(x, v, tv[2], sv[2], sv[3]))


def test_live_lora_roles_and_merge():
    torch.manual_seed(0)
    cfg = h3_tiny_config()
    model = build_model(make_spec(cfg, TINY_HYBRID, dtype="float32"), init="random")
    targets = ["attn.orig.to_q", "attn.orig.to_v"]
    assert inject_lora(model, "default", 4, 4, targets, init_b_zero=False) == 2 * cfg.num_layers
    inject_lora(model, "fake", 2, 2, targets, init_b_zero=False)
    names = [n for n, _ in model.named_parameters() if "lora_A" in n]
    assert "transformer_blocks.0.attn.orig.to_q.lora_A.default.weight" in names
    lin = model.transformer_blocks[0].attn.orig.to_q
    x = torch.randn(3, cfg.hidden_size)
    set_active_adapters(model, ["default"])
    y_default = lin(x)
    set_active_adapters(model, [])
    assert torch.allclose(lin(x), lin.base_layer(x))
    set_active_adapters(model, ["default"])
    merge_and_unload(model)
    assert torch.allclose(model.transformer_blocks[0].attn.orig.to_q(x), y_default, atol=1e-5)


def _seed_checkpoint(path):
    from vdn_minimax_h3_b200.checkpoints import CheckpointArtifact, save_checkpoint
    from vdn_minimax_h3_b200.models.hybrid_transform import hybrid_new_parameters
    torch.manual_seed(0)
    spec = make_spec(h3_tiny_config(), TINY_HYBRID, source="synthetic", dtype="float32")
    model = build_model(spec, init="random")
    w = {n: p.detach().clone() for _, ps in hybrid_new_parameters(model) for n, p in ps}
    save_checkpoint(CheckpointArtifact("weights", spec.to_dict(), w), path)
    return path


def _run_stage(stage, argv, world=1, rank=0, port=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port or _port()),
                      WORLD_SIZE=str(world), RANK=str(rank), LOCAL_RANK="0")
    from vdn_minimax_h3_b200.training import trainers
    schema, fn = {"a1": (StageA1Config, trainers.run_stage_a1), "a2": (StageA2Config, trainers.run_stage_a2),
                  "b": (StageBConfig, trainers.run_stage_b), "dmd": (StageDMDConfig, trainers.run_stage_dmd)}[stage]
    try:
        return fn(load_config(schema, argv))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _metrics(out):
    with open(os.path.join(out, "metrics.jsonl")) as f:
        return [json.loads(line) for line in f]


@pytest.mark.timeout(300)
def test_stage_a1_tiny(tmp_path):
    out = str(tmp_path / "a1")
    cfg = h3_tiny_config().to_dict()
    argv = ["model.base.source=synthetic", f"data.index_file={TINY_DATA}", f"checkpoint.output_dir={out}",
            "training.max_steps=2", "checkpoint.save_every=2", "checkpoint.early_saves=[]",
            "model.architecture.hybrid_attention.softmax_attention.radius=0",
            "model.architecture.hybrid_attention.softmax_attention.chunk=2",
            "model.architecture.hybrid_attention.linear_attention.delta_rule=sana_scaled",
            "model.architecture.hybrid_attention.linear_attention.short_conv.targets=[]",
            "model.base.dtype=float32", "model.base.config_overrides=" + json.dumps(cfg)]
    assert _run_stage("a1", argv) == 2
    m = _metrics(out)
    assert len(m) == 2 and all(r["rel_mean"] >= 0 for r in m)
    assert os.path.exists(os.path.join(out, "hybrid_step000002.pt")) and os.path.exists(os.path.join(out, "DONE"))


@pytest.mark.timeout(300)
def test_stage_a2_resume_and_b(tmp_path):
    seed = _seed_checkpoint(str(tmp_path / "seed.pt"))
    out = str(tmp_path / "a2")
    base = [f"initialization.checkpoint={seed}", f"data.index_file={TINY_DATA}", f"checkpoint.output_dir={out}",
            "checkpoint.save_every=1", "checkpoint.early_saves=[]", "distributed.offload_activations=false"]
    assert _run_stage("a2", base + ["training.max_steps=1"]) == 1
    os.remove(os.path.join(out, "DONE"))
    assert _run_stage("a2", base + ["training.max_steps=2"]) == 2        # resumes at step 1
    steps = [r["step"] for r in _metrics(out)]
    assert steps == [1, 2]
    art = torch.load(sorted(glob.glob(os.path.join(out, "train_state_step*.pt")))[-1], weights_only=True)
    assert art["step"] == 2 and all(isinstance(k, str) for k in art["optimizer"])
    outb = str(tmp_path / "b")
    argv = [f"initialization.checkpoint={os.path.join(out, 'hybrid_step000002.pt')}",
            f"data.index_file={TINY_DATA}", f"checkpoint.output_dir={outb}", "training.max_steps=1",
            "checkpoint.save_every=1", "distributed.offload_activations=false",
            "lora.rank=4", "lora.alpha=4", "lora.targets=[attn.orig.to_q,attn.orig.to_v]"]
    assert _run_stage("b", argv) == 1
    w = torch.load(os.path.join(outb, "hybrid_lora_step000001.pt"), weights_only=True)
    assert any(".lora_A.default." in k for k in w["weights"]) and w["model_spec"]["adapters"]


@pytest.mark.timeout(300)
def test_stage_dmd_tiny(tmp_path):
    seed = _seed_checkpoint(str(tmp_path / "seed.pt"))
    out = str(tmp_path / "dmd")
    argv = [f"initialization.checkpoint={seed}", "data.index_file=synthetic:4:16x3x16x16:4:8:256",
            f"checkpoint.output_dir={out}", "turbo.checkpoint=synthetic", "turbo.num_steps=2",
            "dmd.fake_rank=4", "dmd.fake_warmup_steps=1", "dmd.fake_updates_per_step=2",
            "training.max_steps=1", "checkpoint.save_every=1", "generation.num_frames=5",
            "generation.latent_height=16", "generation.latent_width=16", "distributed.offload_activations=false"]
    assert _run_stage("dmd", argv) == 1
    m = _metrics(out)
    assert [r["turn"] for r in m][:2] == ["warmup", "generator"]
    assert all(r["fake_loss"] == r["fake_loss"] for r in m)


def _fsdp_worker(rank, world, port, seed, out, q):
    try:
        steps = _run_stage("a2", [f"initialization.checkpoint={seed}", f"data.index_file={TINY_DATA}",
                                  f"checkpoint.output_dir={out}", "training.max_steps=2", "checkpoint.save_every=2",
                                  "checkpoint.early_saves=[]", "distributed.offload_activations=false",
                                  "distributed.shard_size=2"], world=world, rank=rank, port=port)
        q.put((rank, steps))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))


def test_debug_mem_lines(tmp_path, monkeypatch, capsys):
    """H3_DEBUG_MEM (reference train_stage_a1.py:92-94) prints one memory line per aligned block."""
    monkeypatch.setenv("H3_DEBUG_MEM", "1")
    out = str(tmp_path / "a1m")
    cfg = h3_tiny_config().to_dict()
    argv = ["model.base.source=synthetic", f"data.index_file={TINY_DATA}", f"checkpoint.output_dir={out}",
            "training.max_steps=1", "checkpoint.save_every=1", "checkpoint.early_saves=[]",
            "model.architecture.hybrid_attention.softmax_attention.radius=0",
            "model.architecture.hybrid_attention.softmax_attention.chunk=2",
            "model.architecture.hybrid_attention.linear_attention.delta_rule=sana_scaled",
            "model.architecture.hybrid_attention.linear_attention.short_conv.targets=[]",
            "model.base.dtype=float32", "model.base.config_overrides=" + json.dumps(cfg)]
    assert _run_stage("a1", argv) == 1
    lines = [ln for ln in capsys.readouterr().out.splitlines() if "alloc=" in ln]
    assert any(ln.strip().startswith("block  0: alloc=") for ln in lines), lines
    assert all("peak=" in ln and ln.endswith("GiB") for ln in lines)


@pytest.mark.timeout(300)
def test_stage_a2_fsdp2_two_ranks(tmp_path):
    seed = _seed_checkpoint(str(tmp_path / "seed.pt"))
    out = str(tmp_path / "a2f")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_fsdp_worker, args=(r, 2, port, seed, out, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=280)
    res = dict(q.get() for _ in range(2))
    assert res == {0: 2, 1: 2}, res
    assert os.path.exists(os.path.join(out, "hybrid_step000002.pt"))


def test_step_profiler_env(tmp_path, monkeypatch, capsys):
    """VDN_PROF_STEP=N (the reference's H3_PROF_STEP) prints a profiler table for step N."""
    monkeypatch.setenv("H3_PROF_STEP", "1")
    seed = _seed_checkpoint(str(tmp_path / "seed.pt"))
    out = str(tmp_path / "a2")
    argv = [f"initialization.checkpoint={seed}", f"data.index_file={TINY_DATA}",
            f"checkpoint.output_dir={out}", "training.max_steps=1", "checkpoint.save_every=1",
            "checkpoint.early_saves=[]", "distributed.offload_activations=false"]
    assert _run_stage("a2", argv) == 1
    assert "profile of step 1" in capsys.readouterr().out


def _bucket_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from vdn_minimax_h3_b200.training.trainers import _bucketed
        g = torch.Generator().manual_seed(rank)
        ts = [torch.randn(3, 5, generator=g), torch.randn(7, generator=g).bfloat16(),
              torch.randn(2, 2, generator=g)]
        want = [t.clone() for t in ts]
        for t in want:
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
        _bucketed(ts, lambda flat: dist.all_reduce(flat, op=dist.ReduceOp.SUM))
        same = all(torch.equal(a, b) for a, b in zip(ts, want))
        params = [torch.full((4,), float(rank)), torch.full((2, 3), float(rank)).bfloat16()]
        _bucketed(params, lambda flat: dist.broadcast(flat, src=1))
        q.put((rank, same and all(bool((p == 1).all()) for p in params)))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))


@pytest.mark.timeout(120)
def test_a1_bucketed_collectives_two_ranks():
    """Stage A1's per-layer buckets (one collective per dtype over a flat buffer) give the
    same all-reduce sums as per-tensor calls, and the broadcast leaves every rank with the
    owner's values, on 2 gloo ranks with mixed fp32 / bf16 tensors."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_bucket_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    assert res == {0: True, 1: True}


def test_train_cli_validates_every_stage(capsys):
    """`train <stage> --config ... --validate-only` loads and validates each shipped stage
    config and exits 0; an unknown stage is refused (the module entry checked once through
    `python -m`)."""
    import subprocess
    import sys
    from vdn_minimax_h3_b200.training import train
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cases = {"a1": ["configs/training/stage_a1_c1_vdn_anchor.yaml", "data.index_file=i"],
             "a2": ["configs/training/stage_a2_c1_vdn_anchor.yaml", "data.index_file=i"],
             "b": ["configs/training/stage_b_c1_vdn_anchor.yaml", "data.index_file=i"],
             "dmd": ["configs/training/stage_dmd_vdn.yaml", "data.index_file=i", "turbo.checkpoint=t"]}
    for stage, (cfg, *over) in cases.items():
        with pytest.raises(SystemExit) as ex:
            train.main([stage, "--config", os.path.join(root, cfg), *over, "--validate-only"])
        assert ex.value.code == 0 and "config ok" in capsys.readouterr().err, stage
    with pytest.raises(SystemExit) as ex:
        train.main(["c"])
    assert "usage" in str(ex.value.code)
    r = subprocess.run([sys.executable, "-m", "vdn_minimax_h3_b200.training.train", "b", "--config",
                        "configs/training/stage_b_c1_vdn_anchor.yaml", "data.index_file=i",
                        "--print-config"], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "index_file: i" in r.stdout, r.stderr[-1500:]


@pytest.mark.timeout(300)
def test_train_cli_runs_stage_a1(tmp_path):
    from vdn_minimax_h3_b200.training import train
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_port()), WORLD_SIZE="1", RANK="0",
                      LOCAL_RANK="0")
    out = str(tmp_path / "a1")
    cfg = h3_tiny_config().to_dict()
    argv = ["a1", "model.base.source=synthetic", f"data.index_file={TINY_DATA}",
            f"checkpoint.output_dir={out}", "training.max_steps=1", "checkpoint.save_every=1",
            "checkpoint.early_saves=[]",
            "model.architecture.hybrid_attention.softmax_attention.radius=0",
            "model.architecture.hybrid_attention.softmax_attention.chunk=2",
            "model.architecture.hybrid_attention.linear_attention.delta_rule=sana_scaled",
            "model.architecture.hybrid_attention.linear_attention.short_conv.targets=[]",
            "model.base.dtype=float32", "model.base.config_overrides=" + json.dumps(cfg)]
    assert train.main(argv) == 1
    assert os.path.exists(os.path.join(out, "DONE"))
