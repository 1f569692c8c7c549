"""Delta-rule state-update backends: how one frame's statistics A = k^T diag(beta) k and
B = v^T diag(beta) k become the scan's transition and injection.

Reference parity: src/models/linear_attention/delta_rule.py:6-94.
  SanaDelta       T = diag(alpha)(I - A/S),   inj = B/sqrt(S)
  VdnDelta        T = diag(alpha)(I + A)^-1,  inj = B (I + A)^-1      (released rule)
  VdnScaledDelta  T = diag(alpha)(I + A/S)^-1, inj = (B/sqrt(S)) (I + A/S)^-1

`factor_apply` here is the fp32 PyTorch oracle (Cholesky, one triangular solve and a
product, as the reference does). The CUDA path (ops/linear_branch.py) replaces it with a
one-CTA-per-matrix SPD inverse kernel; `step_ref` replays one recurrence step for tests.
"""
import torch


class SanaDelta:
    def __init__(self, tokens_per_frame):
        self.inv_tokens = 1.0 / tokens_per_frame
        self.inv_sqrt_tokens = self.inv_tokens ** 0.5

    def factor_apply(self, alpha, A_raw, B_raw):
        eye = torch.eye(A_raw.shape[-1], device=A_raw.device, dtype=A_raw.dtype)
        transition = alpha.unsqueeze(-1) * (eye - self.inv_tokens * A_raw)
        return transition, self.inv_sqrt_tokens * B_raw

    def step_ref(self, state, alpha, A_raw, B_raw):
        t, inj = self.factor_apply(alpha, A_raw, B_raw)
        return state @ t + inj


class VdnDelta:
    a_scale = 1.0
    b_scale = 1.0

    def __init__(self, tokens_per_frame=None):
        pass

    def inverse(self, A32):
        eye = torch.eye(A32.shape[-1], device=A32.device, dtype=torch.float32).expand_as(A32)
        chol = torch.linalg.cholesky(A32 * self.a_scale + eye)
        linv = torch.linalg.solve_triangular(chol, eye, upper=False, left=True)
        return linv.transpose(-1, -2) @ linv

    def factor_apply(self, alpha, A_raw, B_raw):
        inv = self.inverse(A_raw.float())
        transition = alpha.unsqueeze(-1) * inv
        injection = (B_raw.float() * self.b_scale) @ inv
        return transition.to(A_raw.dtype), injection.to(B_raw.dtype)

    def step_ref(self, state, alpha, A_raw, B_raw):
        t, inj = self.factor_apply(alpha, A_raw, B_raw)
        return state @ t + inj


class VdnScaledDelta(VdnDelta):
    def __init__(self, tokens_per_frame):
        super().__init__(tokens_per_frame)
        self.a_scale = 1.0 / tokens_per_frame
        self.b_scale = self.a_scale ** 0.5


# keys are the checkpoint enum checkpoints.key_mapping.DELTA_RULE_VALUES
DELTA_BACKENDS = {"sana_scaled": SanaDelta, "vdn_solve": VdnDelta, "vdn_scaled": VdnScaledDelta}
