"""Block-scaled fp8 kernels vs their fp32 oracles (dequantise, matmul in fp32)."""
import pytest
import torch

from vdn_minimax_h3_b200.ops import fp8
from vdn_minimax_h3_b200.ops._ext import check_device_error
from vdn_minimax_h3_b200.ops.gemm import interleave_swiglu_rows

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,K", [(130, 256), (1000, 5376)])
def test_quant_rows_matches_oracle(M, K):
    torch.manual_seed(0)
    x = (torch.randn(M, K, device="cuda") * torch.rand(M, 1, device="cuda") * 10).to(torch.bfloat16)
    q, sf = fp8.quantize_act(x)
    torch.cuda.synchronize()
    qr, sfr = fp8.quantize_act(x.cpu())
    assert torch.equal(fp8.sf_unblock(sf.cpu(), M, K, 128), fp8.sf_unblock(sfr, M, K, 128))
    mism = (q.cpu() != qr).float().mean().item()
    assert mism < 1e-4, mism


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (300, 544, 384), (2048, 5376, 5376)])
def test_gemm_fp8_store(M, N, K):
    torch.manual_seed(1)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    b = torch.randn(N, device="cuda")
    xq, xsf = fp8.quantize_act(x)
    fw = fp8.Fp8Weight(w, b)
    y = fp8.linear_fp8(xq, xsf, fw)
    torch.cuda.synchronize()
    check_device_error()
    ref = fp8.dequantize(xq, xsf, 128) @ fw.dequantized().t() + b
    assert _rel(y, ref) < 8e-3
    assert _rel(y, x.float() @ w.float().t() + b) < 0.06


def test_gemm_fp8_residual():
    torch.manual_seed(2)
    M, N, K = 333, 512, 256
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / 16
    fw = fp8.Fp8Weight(w)
    xq, xsf = fp8.quantize_act(x)
    res = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    table = torch.randn(3, N, device="cuda", dtype=torch.bfloat16)
    idx = torch.randint(0, 3, (M,), device="cuda", dtype=torch.int32)
    ref = res.float() + table.float()[idx.long()] * (fp8.dequantize(xq, xsf, 128) @ fw.dequantized().t())
    fp8.linear_fp8_gated_residual(xq, xsf, fw, res, table, idx)
    torch.cuda.synchronize()
    check_device_error()
    assert _rel(res, ref) < 8e-3


def test_gemm_fp8_swiglu_quant():
    torch.manual_seed(3)
    M, I, K = 500, 512, 384
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2 * I, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    wi, _ = interleave_swiglu_rows(w, None, tile=128)
    fw = fp8.Fp8Weight(wi)
    xq, xsf = fp8.quantize_act(x)
    q, sf = fp8.linear_fp8_swiglu(xq, xsf, fw)
    torch.cuda.synchronize()
    check_device_error()
    h = fp8.dequantize(q, sf, 128)
    y = (fp8.dequantize(xq, xsf, 128) @ fw.dequantized().t()).view(M, 2 * I // 128, 2, 64)
    ref = (y[:, :, 0] * torch.nn.functional.silu(y[:, :, 1])).reshape(M, I)
    assert _rel(h, ref) < 0.05


def test_engine_fp8_close_to_bf16():
    """The fp8 engine (QKV, FF-up, FF-down on the block-scaled GEMM) stays close to the bf16
    engine on a reduced hybrid geometry with 128-wide heads."""
    import copy
    from tests.test_model_cpu import _forward_inputs, tiny_model
    from vdn_minimax_h3_b200.inference.engine import InferenceEngine
    from vdn_minimax_h3_b200.inference.render import render_geometry
    from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID
    from vdn_minimax_h3_b200.models.h3 import H3Config
    from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
    cfg = H3Config(hidden_size=512, num_layers=2, num_attention_heads=4, attention_head_dim=128,
                   in_channels=8, text_dim=96, time_embed_dim=64, time_freq_dim=32,
                   ff_inner_dim=1024, num_refiner_layers=1, rope_axes_dim=(32, 48, 48))
    model = tiny_model(RELEASED_HYBRID, cfg)
    geo = render_geometry(cfg, 5, latent_h=8, latent_w=12, audio=True, num_latent_frames=9)
    geo.num_audio_latents = 6
    kw, layout = _forward_inputs(cfg, geo, 24)
    gm = model.to(device="cuda", dtype=torch.bfloat16)
    gm.time_embedder.float()
    for blk in gm.transformer_blocks:
        blk.attn.linear_attention.alpha.float()
    set_layout(gm, layout)
    kwg = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in kw.items()}
    with torch.no_grad():
        ref_v, _ = InferenceEngine(copy.deepcopy(gm))(**kwg, layout=layout)
        out_v, _ = InferenceEngine(gm, fp8=True)(**kwg, layout=layout)
    torch.cuda.synchronize()
    check_device_error()
    err = _rel(out_v, ref_v)
    print(f"fp8 engine vs bf16 engine: {err:.3e}")
    # budget: an E4M3 operand carries a relative rounding error of RMS 2^-3 / sqrt(12) =
    # 3.6e-2; a GEMM with both operands quantised, ~5.1e-2 on its output. The block output
    # adds that error to a residual stream that carries most of the signal, so the whole
    # engine must stay well under one GEMM's error.
    assert err < 3.0e-2
