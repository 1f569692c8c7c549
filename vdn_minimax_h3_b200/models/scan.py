"""Frame statistics, the bidirectional scans and the boundary gather (fp32 oracle).

Reference parity: src/models/linear_attention/scan.py.
  frame_statistics    A[f,h] = sum_s beta k k^T (fp32, symmetrised), B[f,h] = sum_s beta v k^T
                      (scan.py:19-42,121-167)
  run_scans           prefix[t] = frames 0..t, suffix[t] = frames t..F-1, each
                      S_t = S_{t-1} T_t + inj_t from the (half) text state (scan.py:170-207)
  gather_linear_state prefix[lo-1] + suffix[hi+1], decayed into the query frame by
                      prod alpha over the skipped frames (bridge "alpha"), text state at the
                      clip ends (scan.py:260-396)

The CUDA inference path (ops/linear_branch.py) runs each of these as sm_100a kernels; these
functions are what they are tested against and what training differentiates through.
"""
import torch

BRIDGE_MODES = ("alpha", "none")


def frame_statistics(kf, vf, beta, a_fp32=True):
    """kf, vf [F, H, S, d]; beta [F, H, S] -> A [F,H,d,d] fp32 (symmetric), B [F,H,dv,d]."""
    with torch.autocast(device_type=kf.device.type, enabled=False):
        if a_fp32:
            k32 = kf.float()
            A = torch.matmul((k32 * beta.unsqueeze(-1).float()).transpose(-1, -2), k32)
        else:
            A = torch.matmul((kf * beta.unsqueeze(-1).to(kf.dtype)).transpose(-1, -2), kf).float()
        A = 0.5 * (A + A.transpose(-1, -2))
        vb = vf * beta.unsqueeze(-1).to(vf.dtype)
        B = torch.matmul(vb.transpose(-1, -2), kf).float()
    return A, B


def run_scans(transitions, injections, text_state=None):
    """Serial recurrences over frames in both directions. [F,H,d,d] fp32 in and out."""
    with torch.autocast(device_type=transitions.device.type, enabled=False):
        F_ = transitions.shape[0]
        start = (torch.zeros_like(injections[0]) if text_state is None
                 else text_state.to(injections.dtype))
        fwd, state = [], start
        for f in range(F_):
            state = state @ transitions[f] + injections[f]
            fwd.append(state)
        rev, state = [None] * F_, start
        for f in range(F_ - 1, -1, -1):
            state = state @ transitions[f] + injections[f]
            rev[f] = state
        return torch.stack(fwd), torch.stack(rev)


def gather_indices(bounds, num_frames, device):
    last_before = torch.tensor([lo for lo, _ in bounds], device=device) - 1
    first_after = torch.tensor([hi for _, hi in bounds], device=device) + 1
    return dict(
        before_idx=last_before.clamp(min=0), after_idx=first_after.clamp(max=num_frames - 1),
        has_before=last_before >= 0, has_after=first_after < num_frames,
        bridge_before=(last_before + 1).clamp(min=0), bridge_after=first_after.clamp(max=num_frames),
        frames=torch.arange(num_frames, device=device))


def gather_linear_state(prefix, suffix, alpha, bounds, bridge="alpha", text_state=None,
                        out_dtype=None):
    """Everything outside each query frame's window, in that frame's reference. [F,H,dv,dk]."""
    assert bridge in BRIDGE_MODES, bridge
    idx = gather_indices(bounds, prefix.shape[0], prefix.device)
    before = prefix[idx["before_idx"]]
    after = suffix[idx["after_idx"]]
    if text_state is not None:
        ts = text_state.to(before.dtype)
        before = torch.where(idx["has_before"].view(-1, 1, 1, 1), before, ts)
        after = torch.where(idx["has_after"].view(-1, 1, 1, 1), after, ts)
    if bridge == "alpha":
        log_a = torch.log(alpha.clamp_min(1e-12))
        pre = torch.cat([torch.zeros_like(log_a[:1]), log_a.cumsum(0)])
        fr = idx["frames"]
        a_before = torch.exp(pre[fr + 1] - pre[idx["bridge_before"]])
        a_after = torch.exp(pre[idx["bridge_after"]] - pre[fr])
        before = before * a_before.unsqueeze(2)
        after = after * a_after.unsqueeze(2)
    if text_state is not None:
        out = before + after
    else:
        out = (before * idx["has_before"].view(-1, 1, 1, 1)
               + after * idx["has_after"].view(-1, 1, 1, 1))
    return out if out_dtype is None else out.to(out_dtype)
