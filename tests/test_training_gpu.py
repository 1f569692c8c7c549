"""The training stages on a B200 (one rank, NCCL): tiny Stage B (LoRA + branch) and DMD
runs take optimizer steps on CUDA with finite losses."""
import os

import pytest
import torch

from tests.test_training_cpu import TINY_DATA, _metrics, _run_stage, _seed_checkpoint

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.mark.timeout(600)
def test_stage_b_and_dmd_on_gpu(tmp_path):
    seed = _seed_checkpoint(str(tmp_path / "seed.pt"))
    outb = str(tmp_path / "b")
    argv = [f"initialization.checkpoint={seed}", f"data.index_file={TINY_DATA}",
            f"checkpoint.output_dir={outb}", "training.max_steps=2", "checkpoint.save_every=2",
            "checkpoint.early_saves=[]", "distributed.offload_activations=false",
            "lora.rank=4", "lora.alpha=4", "lora.targets=[attn.orig.to_q,attn.orig.to_v]"]
    assert _run_stage("b", argv) == 2
    m = _metrics(outb)
    assert [r["step"] for r in m] == [1, 2]
    assert all(r["finite"] == 1.0 and r["loss"] == r["loss"] for r in m)
    assert all(r.get("peak_gib", 0) > 0 for r in m)          # ran on the GPU
    outd = str(tmp_path / "dmd")
    argv = [f"initialization.checkpoint={seed}", f"data.index_file={TINY_DATA}",
            f"checkpoint.output_dir={outd}", "turbo.checkpoint=synthetic", "turbo.num_steps=2",
            "dmd.fake_rank=4", "dmd.fake_warmup_steps=1", "dmd.fake_updates_per_step=2",
            "training.max_steps=1", "checkpoint.save_every=1", "generation.num_frames=5",
            "generation.latent_height=16", "generation.latent_width=16",
            "distributed.offload_activations=false"]
    assert _run_stage("dmd", argv) == 1
    assert os.path.isfile(os.path.join(outd, "DONE"))
