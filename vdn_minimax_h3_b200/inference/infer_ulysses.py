"""Multi-GPU render entry point (one process per GPU, Ulysses sequence parallel).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m vdn_minimax_h3_b200.inference.infer_ulysses \
        --config configs/inference/8nfe_tuned_fp8_ulysses_b200.yaml render.prompt_file=... render.out=...

init NCCL -> assemble on every rank -> UlyssesEngine -> barrier -> warm-up -> timed render
(device-synchronised, max over ranks) -> rank-0 decode + save -> timing line.
Reference parity: src/inference/infer_ulysses.py:43-184.
"""
import datetime
import os
import sys
import time

import torch
import torch.distributed as dist

from vdn_minimax_h3_b200.config import load_config
from vdn_minimax_h3_b200.config.schemas import (InferenceConfig, validate_ablation, validate_kernels,
                                                validate_parallel)


def main(argv=None):
    t_start = time.perf_counter()
    cfg = load_config(InferenceConfig, argv, (validate_kernels, validate_ablation, validate_parallel))
    if not cfg.kernels.inference_kernels:
        raise ValueError("the sequence / tensor parallel engines run the fused kernels: "
                         "kernels.inference_kernels=false is a single-GPU (infer.py) setting")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    from vdn_minimax_h3_b200.inference.infer import assemble, render
    model, engine = assemble(cfg, device)
    par = cfg.parallel
    if par.tensor_parallel > 1:
        if par.softmax_ranks:
            raise ValueError("parallel.softmax_ranks (branch parallel) needs tensor_parallel = 1")
        from vdn_minimax_h3_b200.parallel.hybrid import HybridEngine, HybridRuntime
        runtime = HybridRuntime(par.tensor_parallel, profile=par.profile)
        sp = HybridEngine(engine, runtime, fp8=cfg.precision.fp8.enabled)
    else:
        from vdn_minimax_h3_b200.parallel.ulysses import UlyssesEngine, init_ulysses
        runtime = init_ulysses(profile=par.profile, softmax_ranks=par.softmax_ranks)
        sp = UlyssesEngine(engine, runtime, exchange=par.exchange)
    runtime.barrier()
    # host-side liveness: a rank that dies or stalls is reported before the next NFE launches
    from vdn_minimax_h3_b200.utils.watchdog import Heartbeat
    hb = Heartbeat(interval_s=1.0, timeout_s=120.0).start()
    t_setup = time.perf_counter() - t_start
    lat, aud, steps, denoise = render(cfg, model, engine, device, runtime=runtime, transformer=sp,
                                      on_step=lambda i: hb.check())
    hb.check()
    d = torch.tensor([denoise], device=device)
    dist.all_reduce(d, op=dist.ReduceOp.MAX)
    # every rank decodes a share of the frames; rank 0 gathers them and writes the mp4
    from vdn_minimax_h3_b200.inference.vae import decode_and_save
    t0 = time.perf_counter()
    decode_and_save(lat, aud, cfg.render.out)
    t_decode = time.perf_counter() - t0
    runtime.barrier()
    if dist.get_rank() == 0:
        prof = runtime.timer.report() if cfg.parallel.profile else {}
        print(f"Ulysses timing ({dist.get_world_size()} GPUs): setup {t_setup:.1f}s, denoise "
              f"{float(d.item()):.2f}s ({cfg.render.num_steps} NFE), decode+encode {t_decode:.1f}s, "
              f"E2E {time.perf_counter() - t_start:.1f}s" + (f", sections {prof}" if prof else ""),
              flush=True)
    hb.stop()
    sp.close()   # symmetric-memory heaps are released on every rank before NCCL goes away
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
