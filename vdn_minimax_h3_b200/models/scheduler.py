"""Flow-matching Euler scheduler with the exponential time shift.

Conventions (reference src/training/t2va_batch.py:24-58,192-215 and dmd.py:13-17):
t = 1 - sigma; x_t = t * x0 + (1 - t) * eps; the model predicts the data-ward velocity
v = x0 - eps; x0 = x_t + (1 - t) * v; one Euler step is the blend r * x_t + (1 - r) * x0
with r = sigma_next / sigma taken from the sigma grid. The grid is uniform in u and
shifted sigma' = s*u / (1 + (s-1)*u) (shift 12 for video, 3 for audio,
src/config/inference.py:83-84). `set_timesteps(n + 1)` makes n model evaluations, the
terminal sigma 0 included as the last grid point (render.py:100-105).
"""
import torch


def shifted_sigmas(num_points, shift):
    base = torch.linspace(1.0, 0.0, num_points, dtype=torch.float32)
    return shift * base / (1 + (shift - 1) * base)


class FlowMatchEulerScheduler:
    def __init__(self, shift=12.0):
        if shift <= 0:
            raise ValueError("shift must be positive")
        self.shift = float(shift)
        self.sigmas = None
        self.timesteps = None

    def set_timesteps(self, num_points, device=None):
        """`num_points` sigma grid points (terminal 0 included): num_points - 1 NFE."""
        if num_points < 2:
            raise ValueError("need at least 2 grid points (one model evaluation)")
        self.sigmas = shifted_sigmas(num_points, self.shift).to(device)
        self.timesteps = 1.0 - self.sigmas[:-1]
        self._index = {float(t): i for i, t in enumerate(self.timesteps.tolist())}
        return self.timesteps

    def index_of(self, t):
        return self._index[float(t)]

    def step(self, velocity, t, sample, index=None):
        """One Euler step from grid point `index` (looked up from t when omitted)."""
        i = self.index_of(t) if index is None else index
        sigma, sigma_next = self.sigmas[i], self.sigmas[i + 1]
        t = torch.as_tensor(1.0 - sigma, dtype=sample.dtype, device=sample.device)
        denoised = sample + (1 - t) * velocity
        ratio = (sigma_next / sigma).to(sample.dtype)
        return ratio * sample + (1.0 - ratio) * denoised

    @staticmethod
    def scale_noise(sample, t, noise):
        """Forward process at t: t * x0 + (1 - t) * eps."""
        return t * sample + (1.0 - t) * noise
