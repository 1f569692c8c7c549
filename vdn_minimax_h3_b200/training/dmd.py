"""Stage-DMD building blocks (distribution-matching distillation, DMD2 without the GAN
term): the turn schedule, the three roles of the one sharded model, the generator's
few-step sampler, and the two losses. Everything is plain functions over fp32 packed rows,
so the arithmetic is checked on CPU.

Behaviour parity: src/training/dmd.py:33-207 -- the same role table (generator = VDN +
`default` + `turbo`; real score = dense teacher or VDN + `default`; fake score = the real
score's architecture + `fake`), the same loop shape (fake-only warm-up, then one generator
update per `updates_per_step` fake updates), the same DM gradient. The rollout index is
drawn from a hash of (seed, iteration), so every rank draws the same one without talking.
"""
import hashlib
from contextlib import contextmanager
from typing import Dict, List, NamedTuple

import torch
import torch.nn.functional as F

from vdn_minimax_h3_b200.models.hybrid_transform import set_teacher_mode
from vdn_minimax_h3_b200.models.lora import set_active_adapters
from vdn_minimax_h3_b200.training.batch import euler_blend, few_step_sigmas, few_step_timesteps, x0_from_velocity

REAL_SCORES = ("dense", "vdn")
GENERATOR, REAL, FAKE = "generator", "real", "fake"
WARMUP_TURN, GENERATOR_TURN, FAKE_TURN = "warmup", "generator", "fake"


def turn(fake_step: int, warmup_steps: int, updates_per_step: int) -> str:
    """Kind of sub-iteration number `fake_step` (the saved counter, so a resume lands on
    the right kind). Every sub-iteration updates the fake score once; after the warm-up the
    first of every `updates_per_step` also updates the generator on the same sample."""
    past_warmup = fake_step - warmup_steps
    if past_warmup < 0:
        return WARMUP_TURN
    _, position = divmod(past_warmup, updates_per_step)
    return GENERATOR_TURN if position == 0 else FAKE_TURN


class RoleState(NamedTuple):
    teacher_mode: bool           # dense backbone attention (no hybrid branch) when True
    adapters: List[str]          # LoRA adapters active in that role


class Roles:
    """The role table and the switch between roles. Switching flips teacher_mode and the
    active adapter set only; requires_grad is FSDP's business and is not touched."""

    def __init__(self, model, real_score, vdn_adapter="default", turbo_adapter="turbo",
                 fake_adapter="fake"):
        if real_score not in REAL_SCORES:
            raise ValueError(f"real_score must be one of {REAL_SCORES}, got {real_score!r}")
        self.model, self.real_score = model, real_score
        # the real score's architecture: the dense teacher, or the hybrid with `default`
        real = RoleState(True, []) if real_score == "dense" else RoleState(False, [vdn_adapter])
        self.table: Dict[str, RoleState] = {
            GENERATOR: RoleState(False, [vdn_adapter, turbo_adapter]),
            REAL: real,
            FAKE: RoleState(real.teacher_mode, real.adapters + [fake_adapter]),
        }
        self.current = None

    def teacher_mode(self, role):
        return self.table[role].teacher_mode

    def adapters(self, role):
        return list(self.table[role].adapters)

    def set(self, role):
        state = self.table[role]
        set_teacher_mode(self.model, state.teacher_mode)
        set_active_adapters(self.model, list(state.adapters))
        self.current = role

    @contextmanager
    def borrowed(self, role):
        """Run under `role`, then put back whichever role was live (activation
        checkpointing recomputes the generator's blocks under the role live at backward
        time, so a score forward between its forward and backward must not leave its own)."""
        previous = self.current
        self.set(role)
        try:
            yield
        finally:
            if previous is not None:
                self.set(previous)


class FewStepSchedule:
    """The generator's sampling grid for both modalities: forward times t and sigmas."""

    def __init__(self, num_steps, video_shift, audio_shift):
        self.num_steps = int(num_steps)
        self.t_v, self.t_a = few_step_timesteps(num_steps, video_shift, audio_shift)
        self.sigma_v, self.sigma_a = few_step_sigmas(num_steps, video_shift, audio_shift)

    def times(self, i):
        return float(self.t_v[i]), float(self.t_a[i])

    def step(self, i, video_rows, audio_rows, vel_v, vel_a):
        """Euler step from grid point i to i + 1, both modalities."""
        grids = ((video_rows, vel_v, self.t_v, self.sigma_v), (audio_rows, vel_a, self.t_a, self.sigma_a))
        return tuple(euler_blend(x, v, t[i], sg[i], sg[i + 1]) for x, v, t, sg in grids)

    def x0(self, i, video_rows, audio_rows, vel_v, vel_a):
        return (x0_from_velocity(video_rows, vel_v, self.t_v[i]),
                x0_from_velocity(audio_rows, vel_a, self.t_a[i]))


def sample_rollout_index(generator, num_steps):
    return int(torch.randint(num_steps, (), generator=generator))


def shared_rollout_index(seed, iteration, num_steps):
    """The grid step that gets the gradient this iteration: a pure function of (seed,
    iteration), identical on every rank without communication (the index sets how many
    forwards, hence FSDP all-gathers, a rank runs, and ranks must agree on that count)."""
    digest = hashlib.blake2b(f"dmd-rollout:{int(seed)}:{int(iteration)}".encode(), digest_size=8)
    return int.from_bytes(digest.digest(), "little") % int(num_steps)


def _velocities(model, packed, x_v, x_a, t_v, t_a, forward=None):
    v, a = (forward or model)(**packed.inputs(x_v, x_a, t_v, t_a))
    return v[0].float(), a[0].float()


@torch.no_grad()
def rollout(model, roles, schedule, packed, video_rows, audio_rows, steps):
    """The generator's own first `steps` Euler steps from noise, without a graph."""
    roles.set(GENERATOR)
    for i in range(steps):
        vel = _velocities(model, packed, video_rows, audio_rows, *schedule.times(i))
        video_rows, audio_rows = schedule.step(i, video_rows, audio_rows, *vel)
    return video_rows, audio_rows


def generator_x0(model, roles, schedule, packed, video_rows, audio_rows, index, build_graph=True,
                 forward=None):
    """The generator's x0 prediction at grid step `index`, with a graph when `build_graph`."""
    roles.set(GENERATOR)
    times = schedule.times(index)
    if build_graph:
        vel = _velocities(model, packed, video_rows, audio_rows, *times, forward=forward)
    else:
        with torch.no_grad():
            vel = _velocities(model, packed, video_rows, audio_rows, *times)
    return schedule.x0(index, video_rows, audio_rows, *vel)


def noised(x0, t, noise):
    """x_t on the flow path: t * x0 + (1 - t) * eps."""
    return noise + t * (x0 - noise)


@torch.no_grad()
def score_x0(model, roles, role, packed, x_v, x_a, t_v, t_a):
    """x0 of the real or fake score at (x_t, t); the live role is restored afterwards."""
    with roles.borrowed(role):
        vel_v, vel_a = _velocities(model, packed, x_v, x_a, t_v, t_a)
    return x0_from_velocity(x_v, vel_v, t_v), x0_from_velocity(x_a, vel_a, t_a)


def require_role(roles, role, what):
    if roles.current != role:
        raise RuntimeError(f"{what}: the checkpoint recompute would run as {roles.current!r}; "
                           f"switch to {role!r} before the backward")


def distribution_matching_loss(x0_g, x0_r, x0_f):
    """DMD's generator gradient for one modality: d loss / d x0_g = g / numel with
    g = (x0_fake - x0_real) / mean|x0_g - x0_real|. Written as <x0_g, g> / numel plus a
    constant, so its value is 0.5 * mean(g^2). Returns (loss, normaliser, rms(x0_f - x0_r))."""
    with torch.no_grad():
        diff = x0_f - x0_r
        normaliser = (x0_g.detach() - x0_r).abs().mean()
        g = diff / normaliser.clamp_min(1e-6)
        offset = 0.5 * g.square().mean() - (x0_g.detach() * g).mean()
        gap = diff.square().mean().sqrt()
    return (x0_g * g).mean() + offset, normaliser, gap


def fake_regression_loss(velocity_pred, x0, noise):
    """Flow-matching loss of the fake score on generator samples: target velocity x0 - eps."""
    return F.mse_loss(velocity_pred, x0 - noise)
