"""Linear-branch kernels vs their fp32 PyTorch references, and the whole inference engine on
the GPU vs the eager CPU model at a reduced geometry (head_dim 128, released transform)."""
import copy

import pytest
import torch

from vdn_minimax_h3_b200.models import scan as scan_ref
from vdn_minimax_h3_b200.models.delta_rule import VdnDelta, VdnScaledDelta
from vdn_minimax_h3_b200.models.linear_branch import activate as activate_ref
from vdn_minimax_h3_b200.models.linear_branch import conv_features_reference
from vdn_minimax_h3_b200.models.window import window_bounds
from vdn_minimax_h3_b200.ops import linear_branch as lb
from vdn_minimax_h3_b200.ops._ext import check_device_error

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("l2", [True, False])
def test_activate(l2):
    torch.manual_seed(0)
    full = torch.randn(300, 3 * 128 + 64, device="cuda", dtype=torch.bfloat16)
    x = full[:, :3 * 128].view(300, 3, 128)
    out = lb.activate(x, l2)
    check_device_error()
    assert _rel(out, activate_ref(x.float().cpu(), l2)) < 1e-2


@pytest.mark.parametrize("two_pass", [True, False])
@pytest.mark.parametrize("F,gh,gw,H,l2", [(7, 5, 6, 2, True), (18, 4, 3, 1, False),
                                          (9, 24, 42, 9, True)])
def test_conv_features(F, gh, gw, H, l2, two_pass):
    torch.manual_seed(0)
    x = torch.randn(F * gh * gw, H, 128, device="cuda", dtype=torch.bfloat16)
    w_sp = torch.randn(H * 128, 5, 5, device="cuda") / 5
    w_tm = torch.randn(H * 128, 5, device="cuda") / 2
    out = lb.conv_features(x, w_sp, w_tm, F, (gh, gw), l2, two_pass=two_pass)
    check_device_error()
    ref = conv_features_reference(x.float().cpu(), w_sp.cpu(), w_tm.cpu(), F, (gh, gw), l2)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("F,S,H", [(3, 100, 2), (2, 1008, 1)])
def test_frame_stats(F, S, H):
    torch.manual_seed(0)
    k = torch.nn.functional.normalize(torch.randn(F * S, H, 128, device="cuda"), dim=-1).to(torch.bfloat16)
    v = torch.randn(F * S, H, 128, device="cuda", dtype=torch.bfloat16)
    beta = torch.rand(F * S, H, device="cuda")
    A, B = lb.frame_statistics(k.view(F, S, H, 128), v.view(F, S, H, 128), beta.view(F, S, H))
    check_device_error()
    Ar, Br = scan_ref.frame_statistics(k.float().cpu().view(F, S, H, 128).permute(0, 2, 1, 3),
                                       v.float().cpu().view(F, S, H, 128).permute(0, 2, 1, 3),
                                       beta.cpu().view(F, S, H).permute(0, 2, 1))
    A = 0.5 * (A + A.transpose(-1, -2))
    assert _rel(A, Ar) < 1e-4
    assert _rel(B, Br) < 1e-2


@pytest.mark.parametrize("rule", [VdnDelta, VdnScaledDelta])
def test_spd_factor(rule):
    torch.manual_seed(0)
    F, H, S = 3, 2, 200
    k = torch.nn.functional.normalize(torch.randn(F, H, S, 128), dim=-1)
    beta = torch.rand(F, H, S)
    A = torch.einsum("fhsk,fhs,fhsl->fhkl", k, beta, k)
    B = torch.randn(F, H, 128, 128)
    alpha = torch.rand(F, H, 128) * 0.5 + 0.5
    backend = rule(S)
    tr, inj = lb.factor_apply(backend, alpha.cuda(), A.cuda(), B.cuda())
    check_device_error()
    tr_r, inj_r = backend.factor_apply(alpha.double(), A.double(), B.double())
    assert _rel(tr, tr_r) < 1e-4
    assert _rel(inj, inj_r) < 1e-4


@pytest.mark.parametrize("cluster", [0, 1, 2, 4, 8, -2])
@pytest.mark.parametrize("with_start", [False, True])
def test_scan(with_start, cluster):
    """The single-CTA scan and the cluster-split scan (state columns over 2/4/8 CTAs
    exchanged through distributed shared memory) match the fp64 recurrence."""
    from vdn_minimax_h3_b200.ops._ext import ext
    torch.manual_seed(0)
    F, H = 9, 3
    trans = torch.randn(F, H, 128, 128) * 0.08
    inj = torch.randn(F, H, 128, 128)
    start = torch.randn(H, 128, 128) if with_start else None
    ext().lb_scan_set_cluster(cluster)
    try:
        p, s = lb.run_scans(trans.cuda(), inj.cuda(), None if start is None else start.cuda())
        check_device_error()
    finally:
        ext().lb_scan_set_cluster(0)
    pr, sr = scan_ref.run_scans(trans.double(), inj.double(), None if start is None else start.double())
    assert _rel(p, pr) < 1e-4
    assert _rel(s, sr) < 1e-4


@pytest.mark.parametrize("bridge,text", [("alpha", False), ("alpha", True), ("none", False)])
def test_gather(bridge, text):
    torch.manual_seed(0)
    F, H = 12, 2
    prefix = torch.randn(F, H, 128, 128)
    suffix = torch.randn(F, H, 128, 128)
    alpha = torch.rand(F, H, 128) * 0.5 + 0.5
    ts = torch.randn(H, 128, 128) if text else None
    bounds = window_bounds(F, 1, 3)
    out = lb.gather(prefix.cuda(), suffix.cuda(), alpha.cuda(), bounds, bridge,
                    None if ts is None else ts.cuda())
    check_device_error()
    ref = scan_ref.gather_linear_state(prefix, suffix, alpha, bounds, bridge=bridge, text_state=ts)
    assert _rel(out, ref) < 1e-2


def test_readout():
    torch.manual_seed(0)
    F, S, H = 3, 200, 2
    q = torch.randn(F * S, H, 128, device="cuda", dtype=torch.bfloat16)
    state = (torch.randn(F, H, 128, 128, device="cuda") * 0.1).to(torch.bfloat16)
    w = torch.randn(128, device="cuda")
    gate = torch.randn(F * S, H, 128, device="cuda", dtype=torch.bfloat16)
    big = torch.zeros(F * S + 10, 2 * H * 128, device="cuda", dtype=torch.bfloat16)
    out = big[5:5 + F * S, H * 128:]
    lb.readout(q.view(F, S, H, 128), state, w, gate, 1e-6, out=out, gate_logits=True)
    check_device_error()
    ref = lb.readout_reference(q.cpu().view(F, S, H, 128), state.cpu(), w.cpu(), gate.cpu(), 1e-6, True)
    assert _rel(out, ref) < 2e-2
    assert big[:5].abs().max().item() == 0 and big[:, :H * 128].abs().max().item() == 0


@torch.no_grad()
def test_engine_gpu_matches_cpu_eager():
    from vdn_minimax_h3_b200.inference.engine import InferenceEngine
    from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID
    from vdn_minimax_h3_b200.models.h3 import H3Config
    from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
    from tests.test_model_cpu import _forward_inputs, tiny_model
    from vdn_minimax_h3_b200.inference.render import render_geometry
    cfg = H3Config(hidden_size=256, num_layers=2, num_attention_heads=2, attention_head_dim=128,
                   in_channels=8, text_dim=96, time_embed_dim=64, time_freq_dim=32,
                   ff_inner_dim=512, num_refiner_layers=1, rope_axes_dim=(32, 48, 48))
    model = tiny_model(RELEASED_HYBRID, cfg)
    geo = render_geometry(cfg, 5, latent_h=8, latent_w=12, audio=True, num_latent_frames=17)
    geo.num_audio_latents = 6
    kw, layout = _forward_inputs(cfg, geo, 24)
    set_layout(model, layout)
    ref_v, ref_a = model(**kw)
    gmodel = copy.deepcopy(model).to(device="cuda", dtype=torch.bfloat16)
    gmodel.time_embedder.float()
    for blk in gmodel.transformer_blocks:
        blk.attn.linear_attention.alpha.float()
    eager = copy.deepcopy(gmodel)
    eng = InferenceEngine(gmodel)
    kwg = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in kw.items()}
    out_v, out_a = eng(**kwg, layout=layout)
    check_device_error()
    # budget: the round-off of the same model run eagerly in bf16 on this GPU (every op
    # rounds to bf16 there too); the fused kernels keep more of each chain in fp32, so they
    # must land within a small multiple of it
    set_layout(eager, layout)
    bf_v, bf_a = eager(**kwg)
    budget_v = 1.5 * _rel(bf_v, ref_v) + 2e-3
    budget_a = 1.5 * _rel(bf_a, ref_a) + 2e-3
    print(f"engine vs fp32: video {_rel(out_v, ref_v):.2e} (budget {budget_v:.2e}), "
          f"audio {_rel(out_a, ref_a):.2e} (budget {budget_a:.2e})")
    assert _rel(out_v, ref_v) < budget_v
    assert _rel(out_a, ref_a) < budget_a
