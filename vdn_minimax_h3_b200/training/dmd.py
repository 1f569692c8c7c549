"""DMD2 (no GAN) for Stage DMD: three roles on ONE model (generator / real score / fake
score as switches of teacher_mode and the active adapter set), the few-step sampler the
generator is trained through, the distribution-matching loss and the fake-score regression.

Reference parity: src/training/dmd.py:33-207 (same role table, same loss definitions, the
rank-shared rollout index that keeps collective counts equal on every rank, the
role-restoring score forward so a checkpoint recompute never runs under the wrong role).
Pure functions over fp32 packed rows: testable on CPU.
"""
import torch
import torch.nn.functional as F

from vdn_minimax_h3_b200.models.hybrid_transform import set_teacher_mode
from vdn_minimax_h3_b200.models.lora import set_active_adapters
from vdn_minimax_h3_b200.training.batch import euler_blend, few_step_sigmas, few_step_timesteps, x0_from_velocity

REAL_SCORES = ("dense", "vdn")
GENERATOR, REAL, FAKE = "generator", "real", "fake"
WARMUP_TURN, GENERATOR_TURN, FAKE_TURN = "warmup", "generator", "fake"


def turn(fake_step, warmup_steps, updates_per_step):
    if fake_step < warmup_steps:
        return WARMUP_TURN
    return GENERATOR_TURN if (fake_step - warmup_steps) % updates_per_step == 0 else FAKE_TURN


class Roles:
    def __init__(self, model, real_score, vdn_adapter="default", turbo_adapter="turbo",
                 fake_adapter="fake"):
        if real_score not in REAL_SCORES:
            raise ValueError(f"real_score must be one of {REAL_SCORES}, got {real_score!r}")
        dense = real_score == "dense"
        self.model, self.real_score = model, real_score
        self.table = {
            GENERATOR: (False, [vdn_adapter, turbo_adapter]),
            REAL: (True, []) if dense else (False, [vdn_adapter]),
            FAKE: (True, [fake_adapter]) if dense else (False, [vdn_adapter, fake_adapter]),
        }
        self.current = None

    def teacher_mode(self, role):
        return self.table[role][0]

    def adapters(self, role):
        return list(self.table[role][1])

    def set(self, role):
        teacher, adapters = self.table[role]
        set_teacher_mode(self.model, teacher)
        set_active_adapters(self.model, adapters)
        self.current = role


class FewStepSchedule:
    def __init__(self, num_steps, video_shift, audio_shift):
        self.num_steps = int(num_steps)
        self.t_v, self.t_a = few_step_timesteps(num_steps, video_shift, audio_shift)
        self.sigma_v, self.sigma_a = few_step_sigmas(num_steps, video_shift, audio_shift)

    def times(self, i):
        return float(self.t_v[i]), float(self.t_a[i])

    def step(self, i, video_rows, audio_rows, vel_v, vel_a):
        return (euler_blend(video_rows, vel_v, self.t_v[i], self.sigma_v[i], self.sigma_v[i + 1]),
                euler_blend(audio_rows, vel_a, self.t_a[i], self.sigma_a[i], self.sigma_a[i + 1]))

    def x0(self, i, video_rows, audio_rows, vel_v, vel_a):
        return (x0_from_velocity(video_rows, vel_v, self.t_v[i]),
                x0_from_velocity(audio_rows, vel_a, self.t_a[i]))


def sample_rollout_index(generator, num_steps):
    return int(torch.randint(num_steps, (), generator=generator))


def shared_rollout_index(seed, iteration, num_steps):
    """Identical on every rank and a pure function of (seed, iteration): the number of
    forwards (hence FSDP all-gathers) a rank issues must not differ across ranks."""
    g = torch.Generator().manual_seed(int(seed) * 100031 + int(iteration))
    return sample_rollout_index(g, num_steps)


@torch.no_grad()
def rollout(model, roles, schedule, packed, video_rows, audio_rows, steps):
    roles.set(GENERATOR)
    for i in range(steps):
        t_v, t_a = schedule.times(i)
        v, a = model(**packed.inputs(video_rows, audio_rows, t_v, t_a))
        video_rows, audio_rows = schedule.step(i, video_rows, audio_rows, v[0].float(), a[0].float())
    return video_rows, audio_rows


def generator_x0(model, roles, schedule, packed, video_rows, audio_rows, index, build_graph=True,
                 forward=None):
    roles.set(GENERATOR)
    t_v, t_a = schedule.times(index)
    inputs = packed.inputs(video_rows, audio_rows, t_v, t_a)
    if build_graph:
        v, a = (forward or model)(**inputs)
    else:
        with torch.no_grad():
            v, a = model(**inputs)
    return schedule.x0(index, video_rows, audio_rows, v[0].float(), a[0].float())


def noised(x0, t, noise):
    return t * x0 + (1.0 - t) * noise


@torch.no_grad()
def score_x0(model, roles, role, packed, x_v, x_a, t_v, t_a):
    previous = roles.current
    roles.set(role)
    try:
        v, a = model(**packed.inputs(x_v, x_a, t_v, t_a))
        return x0_from_velocity(x_v, v[0].float(), t_v), x0_from_velocity(x_a, a[0].float(), t_a)
    finally:
        if previous is not None:
            roles.set(previous)


def require_role(roles, role, what):
    if roles.current != role:
        raise RuntimeError(f"{what} needs the {role!r} role live for the checkpoint recompute, "
                           f"but {roles.current!r} is active")


def distribution_matching_loss(x0_g, x0_r, x0_f):
    """g = (x0_fake - x0_real) / mean|x0_g - x0_real|, as 0.5 * MSE against (x0_g - g)."""
    with torch.no_grad():
        det = x0_g.detach()
        normaliser = (det - x0_r).abs().mean()
        g = (x0_f - x0_r) / normaliser.clamp_min(1e-6)
        target = det - g
        gap = (x0_f - x0_r).pow(2).mean().sqrt()
    return 0.5 * F.mse_loss(x0_g, target), normaliser, gap


def fake_regression_loss(velocity_pred, x0, noise):
    return F.mse_loss(velocity_pred, x0 - noise)
