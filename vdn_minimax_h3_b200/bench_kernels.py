"""Kernel micro-benchmarks on the VDN-H3 shapes (one GPU, CUDA-event timing).

    python -m vdn_minimax_h3_b200.bench_kernels --gemm
    python -m vdn_minimax_h3_b200.bench_kernels --attention
    python -m vdn_minimax_h3_b200.bench_kernels --linear
    python -m vdn_minimax_h3_b200.bench_kernels --linear-train
    python -m vdn_minimax_h3_b200.bench_kernels --gemm-train

Each case runs 3 warm-up launches and times 10 with CUDA events on the launching stream;
operands are larger than the 126 MB L2 for the full-size shapes. Library baselines
(cuBLAS through torch.matmul, cuDNN/flash SDPA) run beside the package's kernels.
"""
import argparse
import json

import torch

M_ROWS = 104766  # packed rows of a 14.4 s T2VA clip (800 text + 1150 audio + 102*1008 video)


def timed(fn, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(True), torch.cuda.Event(True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


def bench_gemm():
    from vdn_minimax_h3_b200.ops import gemm
    from vdn_minimax_h3_b200.ops._ext import check_device_error
    rows = []
    for name, n, k in [("qkv", 21504, 5376), ("o_proj", 5376, 7168), ("ff_up", 28672, 5376),
                       ("ff_down", 5376, 14336), ("square", 8192, 8192)]:
        m = 8192 if name == "square" else M_ROWS
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) / k ** 0.5
        out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        ours = timed(lambda: gemm.linear(x, w, out=out))
        check_device_error()
        lib = timed(lambda: torch.matmul(x, w.t(), out=out))
        flop = 2.0 * m * n * k
        row = dict(case=name, M=m, N=n, K=k, ours_ms=ours, ours_tflops=flop / ours / 1e9,
                   cublas_ms=lib, cublas_tflops=flop / lib / 1e9)
        if name == "ff_up":
            wi, _ = gemm.interleave_swiglu_rows(w)
            row["swiglu_ms"] = timed(lambda: gemm.linear_swiglu(x, wi))
        rows.append(row)
        print(json.dumps(row), flush=True)
        del x, w, out
        torch.cuda.empty_cache()
    return rows


def bench_gemm_train(rows_t=82809):
    """The three products of each training Linear at the Stage-B shape (81 latent frames:
    82,809 packed rows): forward x W^T, dgrad dy W (W read MN-major) and wgrad dy^T x (both
    read MN-major, contraction over the rows), the package's GEMM against cuBLAS
    (torch.matmul on the same stored tensors)."""
    from vdn_minimax_h3_b200.ops import gemm
    from vdn_minimax_h3_b200.ops._ext import check_device_error
    rows = []
    for name, n, k in [("q_k_v", 7168, 5376), ("o_proj", 5376, 7168), ("ff_up", 28672, 5376),
                       ("ff_down", 5376, 14336)]:
        m = rows_t
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) / k ** 0.5
        dy = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
        y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        dx = torch.empty(m, k, device="cuda", dtype=torch.bfloat16)
        dw = torch.empty(n, k, device="cuda", dtype=torch.bfloat16)
        flop = 2.0 * m * n * k
        row = dict(case=name, T=m, out=n, inp=k)
        for prod, ours, lib in (
                ("fwd", lambda: gemm.linear(x, w, out=y), lambda: torch.matmul(x, w.t(), out=y)),
                ("dgrad", lambda: gemm.linear_dgrad(dy, w, out=dx), lambda: torch.matmul(dy, w, out=dx)),
                ("wgrad", lambda: gemm.linear_wgrad(dy, x, out=dw), lambda: torch.matmul(dy.t(), x, out=dw))):
            t_ours = timed(ours)
            check_device_error()
            t_lib = timed(lib)
            row[f"{prod}_ms"] = round(t_ours, 3)
            row[f"{prod}_tflops"] = round(flop / t_ours / 1e9, 1)
            row[f"{prod}_cublas_ms"] = round(t_lib, 3)
            row[f"{prod}_cublas_tflops"] = round(flop / t_lib / 1e9, 1)
        rows.append(row)
        print(json.dumps(row), flush=True)
        del x, w, dy, y, dx, dw
        torch.cuda.empty_cache()
    return rows


def bench_gemm_fp8():
    """Block-scaled fp8 GEMMs on the H3 shapes (and cuBLAS fp8 via torch._scaled_mm with
    row/column scales as the library baseline)."""
    from vdn_minimax_h3_b200.ops import fp8
    from vdn_minimax_h3_b200.ops._ext import check_device_error
    from vdn_minimax_h3_b200.ops.gemm import interleave_swiglu_rows
    rows = []
    for name, n, k in [("qkv", 21504, 5376), ("ff_up_swiglu", 28672, 5376), ("ff_down", 5376, 14336),
                       ("o_proj", 5376, 14336)]:
        m = M_ROWS
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) / k ** 0.5
        xq, xsf = fp8.quantize_act(x)
        if name == "ff_up_swiglu":
            fw = fp8.Fp8Weight(interleave_swiglu_rows(w, None, tile=128)[0])
            hq = torch.empty(m, n // 2, dtype=torch.uint8, device="cuda")
            hsf = torch.empty(fp8.sf_bytes(m, n // 2), dtype=torch.uint8, device="cuda")
            ours = timed(lambda: fp8.linear_fp8_swiglu(xq, xsf, fw, hq, hsf))
        else:
            fw = fp8.Fp8Weight(w)
            out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            ours = timed(lambda: fp8.linear_fp8(xq, xsf, fw, out))
        check_device_error()
        a8 = xq.view(torch.float8_e4m3fn)
        b8 = fw.q.view(torch.float8_e4m3fn)
        sa = torch.ones(m, 1, device="cuda")
        sb = torch.ones(1, n, device="cuda")
        try:
            lib = timed(lambda: torch._scaled_mm(a8, b8.t(), scale_a=sa, scale_b=sb,
                                                 out_dtype=torch.bfloat16))
        except Exception as exc:  # noqa: BLE001
            lib = float("nan")
            print(json.dumps({"scaled_mm_error": repr(exc)[:200]}), flush=True)
        quant = timed(lambda: fp8.quantize_act(x, xq, xsf))
        flop = 2.0 * m * n * k
        row = dict(case=name, M=m, N=n, K=k, ours_ms=ours, ours_tflops=flop / ours / 1e9,
                   cublas_fp8_rowwise_ms=lib, cublas_tflops=flop / lib / 1e9, quant_act_ms=quant)
        rows.append(row)
        print(json.dumps(row), flush=True)
        del x, w, xq, xsf, fw
        torch.cuda.empty_cache()
    return rows


def bench_norm():
    """AdaLN-RMSNorm, frame sums and QK-prep on the full packed sequence (HBM-bound)."""
    from vdn_minimax_h3_b200.ops import norm
    from vdn_minimax_h3_b200.models.h3 import RotaryEmbedding3D
    T, D, F, S = M_ROWS, 5376, 102, 1008
    x = torch.randn(T, D, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(x)
    w = torch.rand(D, device="cuda") + 0.5
    table = torch.randn(6, 6 * D, device="cuda", dtype=torch.bfloat16) * 0.1
    idx = torch.randint(0, 6, (T,), device="cuda", dtype=torch.int32)
    rows = []
    ms = timed(lambda: norm.adaln_rmsnorm(x, w, 1e-6, table, 0, D, idx, out=out))
    rows.append(dict(case="adaln_rmsnorm", ms=ms, gbps=2 * x.numel() * 2 / ms / 1e6))
    ms = timed(lambda: norm.frame_sums(x, F, S, 0, T - F * S))
    rows.append(dict(case="frame_sums", ms=ms, gbps=F * S * D * 2 / ms / 1e6))
    pos = torch.stack([torch.arange(T) // 1008, (torch.arange(T) // 42) % 24, torch.arange(T) % 42], 1)
    cos, sin = RotaryEmbedding3D((32, 48, 48))(pos.cuda())
    src = torch.randn(T, 7168, device="cuda", dtype=torch.bfloat16)
    qo = torch.empty_like(src)
    nw = torch.rand(128, device="cuda") + 0.5
    ms = timed(lambda: norm.qk_prep(src, 56, nw, 1e-6, cos, sin, out=qo))
    rows.append(dict(case="qk_prep", ms=ms, gbps=2 * src.numel() * 2 / ms / 1e6))
    for r in rows:
        print(json.dumps(r), flush=True)
    return rows


def bench_linear_train(frames=81, heads=56):
    """Training stages of the linear branch, forward + backward at the Stage-B training
    shape (81 latent frames, 56 heads): the SPD factor and the two scans through
    ops/linear_branch_grad.py (kernels forward, adjoint scan backward) vs autograd through
    the eager PyTorch ops (Cholesky + triangular solve, one batched product per frame); then
    the short conv of one projection (24 x 42 grid, SiLU + L2), two-pass kernels forward and
    conv_bwd.cu backward vs autograd through the eager bf16 conv."""
    from vdn_minimax_h3_b200.models import scan as scan_ref
    from vdn_minimax_h3_b200.models.delta_rule import VdnDelta
    from vdn_minimax_h3_b200.ops import linear_branch_grad as lbg
    from vdn_minimax_h3_b200.ops._ext import LAUNCHES, check_device_error
    torch.manual_seed(0)
    F, H, d = frames, heads, 128
    k = torch.nn.functional.normalize(torch.randn(F, H, 256, d, device="cuda"), dim=-1)
    A = torch.matmul(k.transpose(-1, -2), k)
    del k
    B = torch.randn(F, H, d, d, device="cuda")
    alpha = torch.rand(F, H, d, device="cuda") * 0.5 + 0.45
    start = torch.randn(H, d, d, device="cuda") * 0.1
    g_pre, g_suf = torch.randn(2, F, H, d, d, device="cuda")
    backend = VdnDelta()
    leaves = [t.requires_grad_() for t in (alpha, A, B, start)]

    def step(factor, scan):
        trans, inj = factor(backend, *leaves[:3])
        pre, suf = scan(trans, inj, leaves[3])
        torch.autograd.backward([pre, suf], [g_pre, g_suf])
        for t in leaves:
            t.grad = None

    rows = []
    for name, factor, scan in (
            ("kernels", lbg.vdn_factor, lbg.scans),
            ("eager", lambda b, *a: b.factor_apply(*a), scan_ref.run_scans)):
        n0 = LAUNCHES[0]
        ms = timed(lambda: step(factor, scan), iters=5, warmup=3)
        check_device_error()
        rows.append({"stage": "factor+scans fwd+bwd", "impl": name, "frames": F, "heads": H,
                     "ms": round(ms, 3), "own_launches_per_iter": (LAUNCHES[0] - n0) // 8})
    del A, B, alpha, start, g_pre, g_suf, leaves
    # the short conv of one projection (k or v), forward + backward
    from vdn_minimax_h3_b200.models.linear_branch import conv_features_reference
    gh, gw = 24, 42
    N, C = F * gh * gw, H * d
    tokens = torch.randn(N, H, d, device="cuda", dtype=torch.bfloat16)
    w_sp = (torch.randn(C, 5, 5, device="cuda") * 0.2).to(torch.bfloat16)
    w_tm = (torch.randn(C, 5, device="cuda") * 0.45).to(torch.bfloat16)
    up = torch.randn(N, H, d, device="cuda", dtype=torch.bfloat16)
    x = tokens.requires_grad_()
    ws, wt = w_sp.requires_grad_(), w_tm.requires_grad_()

    def conv_step(fn):
        out = fn(x, ws, wt, F, (gh, gw), True)
        out.backward(up)
        x.grad = ws.grad = wt.grad = None

    for name, fn in (("kernels", lbg.conv_features), ("eager", conv_features_reference)):
        n0 = LAUNCHES[0]
        ms = timed(lambda: conv_step(fn), iters=5, warmup=3)
        check_device_error()
        rows.append({"stage": "short conv fwd+bwd (one projection)", "impl": name, "frames": F,
                     "heads": H, "grid": [gh, gw], "ms": round(ms, 3),
                     "own_launches_per_iter": (LAUNCHES[0] - n0) // 8})
    for r in rows:
        print(json.dumps(r), flush=True)
    return rows


def profile_small():
    """Single launches on small inputs, for a one-pass-per-kernel profiler capture."""
    from vdn_minimax_h3_b200.models.delta_rule import VdnDelta
    from vdn_minimax_h3_b200.models.layout import SequenceLayout
    from vdn_minimax_h3_b200.models.window import AttentionPlan, window_bounds
    from vdn_minimax_h3_b200.ops import attention, linear_branch as lb
    from vdn_minimax_h3_b200.ops import gemm
    from vdn_minimax_h3_b200.ops._ext import check_device_error
    xa = torch.randn(16384, 5376, device="cuda", dtype=torch.bfloat16)
    wa = torch.randn(5376, 5376, device="cuda", dtype=torch.bfloat16) / 70
    gemm.linear(xa, wa)
    from vdn_minimax_h3_b200.ops import fp8
    w8 = fp8.Fp8Weight(torch.randn(21504, 5376, device="cuda", dtype=torch.bfloat16) / 70)
    xq = torch.empty(16384, 5376, device="cuda", dtype=torch.uint8)
    xsf = torch.empty(fp8.sf_bytes(16384, 5376), device="cuda", dtype=torch.uint8)
    fp8.quantize_act(xa, xq, xsf)
    fp8.linear_fp8(xq, xsf, w8, torch.empty(16384, 21504, device="cuda", dtype=torch.bfloat16))
    Fr, S, H = 20, 1008, 8
    lay = SequenceLayout(seq_len=1950 + Fr * S, video_start=1950, num_frames=Fr, tokens_per_frame=S,
                         frame_height=24, frame_width=42, text_start=0, text_len=800)
    plan = AttentionPlan(lay, window_bounds(Fr, 1, 5), "both", device="cuda")
    q = torch.randn(lay.seq_len, H, 128, device="cuda", dtype=torch.bfloat16)
    attention.window_attention(q, q, q, plan, 128 ** -0.5)
    A = torch.randn(256, 128, 128, device="cuda") * 0.01
    A = A @ A.transpose(-1, -2)
    lb.factor_apply(VdnDelta(S), torch.rand(256, 128, device="cuda"), A.view(16, 16, 128, 128),
                    torch.randn(16, 16, 128, 128, device="cuda"))
    # short conv at full head count over 20 frames (289 MB in, above L2): about one wave
    Hc = 56
    x = torch.randn(Fr * S, Hc, 128, device="cuda", dtype=torch.bfloat16)
    lb.conv_features(x, torch.randn(Hc * 128, 5, 5, device="cuda"),
                     torch.randn(Hc * 128, 5, device="cuda"), Fr, (24, 42), True)
    torch.cuda.synchronize()
    check_device_error()
    print("profile-small ok", flush=True)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gemm", action="store_true")
    p.add_argument("--attention", action="store_true")
    p.add_argument("--gemm-train", action="store_true",
                   help="training Linear products (forward, dgrad, wgrad) vs cuBLAS at the Stage-B shape")
    p.add_argument("--gemm-train-small", action="store_true",
                   help="the same products at 8,192 rows (ncu-sized)")
    p.add_argument("--attention-train-small", action="store_true",
                   help="training attention forward + backward on 20 frames x 16 heads (ncu-sized, tensors above L2)")
    p.add_argument("--attention-train", action="store_true",
                   help="training attention forward + backward at the Stage-B shape vs SDPA")
    p.add_argument("--attention-ab", action="store_true",
                   help="window attention against cuDNN / flash SDPA on the same plan segments")
    p.add_argument("--trace-variant", type=int, default=None,
                   help="kernel variant for --attention-trace (default: the current one)")
    p.add_argument("--linear", action="store_true")
    p.add_argument("--linear-heads", type=int, nargs="*", default=[56],
                   help="head counts for --linear (7 = one rank's share at 8-way Ulysses)")
    p.add_argument("--norm", action="store_true")
    p.add_argument("--linear-train", action="store_true",
                   help="SPD factor + scans forward and backward at the training shape")
    p.add_argument("--gemm-fp8", action="store_true")
    p.add_argument("--gemm-fp8-trace", action="store_true",
                   help="fp8 GEMM wait-cycle counters (QKV shape)")
    p.add_argument("--attention-trace", action="store_true",
                   help="clock64 phase durations of CTA 0's attention pipeline")
    p.add_argument("--profile-small", action="store_true",
                   help="one launch each of window attention, SPD inverse and conv features on "
                        "small inputs (an ncu-sized driver)")
    p.add_argument("--attention-small", action="store_true",
                   help="window attention on 20 frames x 8 heads (an ncu-sized case)")
    p.add_argument("--linear-small", action="store_true",
                   help="conv features + SPD inverse on 8 frames (an ncu-sized case)")
    a = p.parse_args(argv)
    if a.gemm:
        bench_gemm()
    if a.attention:
        from vdn_minimax_h3_b200.ops.attention import bench_attention
        bench_attention(timed)
    if a.attention_train:
        from vdn_minimax_h3_b200.ops.attention_grad import bench_attention_train
        bench_attention_train(timed)
    if a.gemm_train:
        bench_gemm_train()
    if a.gemm_train_small:
        bench_gemm_train(8192)
    if a.attention_train_small:
        from vdn_minimax_h3_b200.ops.attention_grad import bench_attention_train
        bench_attention_train(timed, frames=20, heads=16)
    if a.attention_ab:
        from vdn_minimax_h3_b200.ops.attention import bench_attention_vs_cudnn
        bench_attention_vs_cudnn(timed)
    if a.linear:
        from vdn_minimax_h3_b200.ops.linear_branch import bench_linear
        for h in a.linear_heads:
            bench_linear(timed, heads=h)
    if a.norm:
        bench_norm()
    if a.linear_train:
        bench_linear_train()
    if a.gemm_fp8:
        bench_gemm_fp8()
    if a.gemm_fp8_trace:
        from vdn_minimax_h3_b200.ops.fp8 import trace_gemm_fp8
        trace_gemm_fp8()
    if a.attention_trace:
        from vdn_minimax_h3_b200.ops.attention import trace_attention
        trace_attention(variant=a.trace_variant)
    if a.profile_small:
        profile_small()
    if a.attention_small:
        from vdn_minimax_h3_b200.ops.attention import bench_attention
        bench_attention(timed, frames=20, heads=8)
    if a.linear_small:
        from vdn_minimax_h3_b200.ops.linear_branch import bench_linear
        bench_linear(lambda fn: (fn(), torch.cuda.synchronize(), 0.0)[2], frames=8)


if __name__ == "__main__":
    main()
