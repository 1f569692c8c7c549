"""Block-scaled fp8 host logic: exponent rule, blocked scale-factor layout, the fp32 oracles."""
import torch

from vdn_minimax_h3_b200.ops import fp8
from vdn_minimax_h3_b200.ops.gemm import interleave_swiglu_rows


def test_e8_exponent_rule():
    amax = torch.tensor([448.0, 449.0, 224.0, 1.0, 0.0, 896.0, 3e-30])
    e = fp8.e8_exponent(amax)
    assert e.tolist()[:6] == [0, 1, -1, -8, -127, 1]
    assert (amax / torch.pow(2.0, e.float()) <= 448.0).all()


def test_sf_layout_round_trip():
    torch.manual_seed(0)
    for tile_rows in (128, 256):
        e = torch.randint(-20, 20, (300, 16), dtype=torch.int32)
        sf = fp8.sf_blocked(e, tile_rows)
        assert sf.numel() % 512 == 0
        assert torch.equal(fp8.sf_unblock(sf, 300, 16 * 32, tile_rows), e)
    # the atom formula of the kernels: row 37, block 5 of K=512 (16 blocks)
    e = torch.zeros(128, 16, dtype=torch.int32)
    e[37, 5] = 9
    sf = fp8.sf_blocked(e, 128)
    off = (0 * 4 + 5 // 4) * 512 + (37 % 32) * 16 + (37 // 32) * 4 + 5 % 4
    assert int(sf[off]) == 9 + 127


def test_fp8_linear_oracle_close_to_bf16():
    torch.manual_seed(1)
    x = torch.randn(100, 256)
    w = torch.randn(96, 256) / 16
    xq, xsf = fp8.quantize_act(x)
    fw = fp8.Fp8Weight(w, torch.randn(96))
    y = fp8.linear_fp8(xq, xsf, fw).float()
    ref = x @ w.t() + fw.bias
    rel = ((y - ref).norm() / ref.norm()).item()
    assert rel < 0.06, rel


def test_fp8_swiglu_oracle():
    torch.manual_seed(2)
    x = torch.randn(64, 256)
    w = torch.randn(512, 256) / 16
    wi, _ = interleave_swiglu_rows(w, None, tile=128)
    xq, xsf = fp8.quantize_act(x)
    q, sf = fp8.linear_fp8_swiglu(xq, xsf, fp8.Fp8Weight(wi))
    h = fp8.dequantize(q, sf, 128)
    a = x @ w.t()
    ref = a[:, :256] * torch.nn.functional.silu(a[:, 256:])
    assert ((h - ref).norm() / ref.norm()).item() < 0.1
