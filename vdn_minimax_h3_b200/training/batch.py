"""Shared packing for the trainers: latent sample -> noisy packed model inputs, and the
few-step sampler side used by Stage DMD.

Reference parity: src/training/t2va_batch.py:24-285 -- the `[text | audio | video]` layout,
the inference-locked (12u, 3u) sigma pairing, the data-ward velocity target (x0 - eps),
per-row timesteps -> (unique, index), PackedPrompt reused across every forward of an
iteration, the scheduler's Euler blend, x0 from velocity.
"""
import torch

from vdn_minimax_h3_b200.models.layout import (AUDIO_CHANNELS, build_packed_sequence, layout_from_indices,
                                               patchify_video_latents)

PATCH_SIZE = (1, 2, 2)
VIDEO_SHIFT, AUDIO_SHIFT = 12.0, 3.0


def sample_sigmas(generator):
    """One u per step through both shifts: sigma' = s*u / (1 + (s-1)*u)."""
    u = torch.rand((), generator=generator).clamp(1e-4, 1.0)
    sv = VIDEO_SHIFT * u / (1 + (VIDEO_SHIFT - 1) * u)
    sa = AUDIO_SHIFT * u / (1 + (AUDIO_SHIFT - 1) * u)
    return float(sv), float(sa)


def few_step_sigmas(num_steps, video_shift, audio_shift):
    if num_steps < 1:
        raise ValueError(f"few-step schedule needs num_steps >= 1, got {num_steps}")
    if video_shift <= 0 or audio_shift <= 0:
        raise ValueError("few-step scheduler shifts must be positive")
    base = torch.linspace(1.0, 0.0, num_steps + 1, dtype=torch.float32)
    return (video_shift * base / (1 + (video_shift - 1) * base),
            audio_shift * base / (1 + (audio_shift - 1) * base))


def few_step_timesteps(num_steps, video_shift, audio_shift):
    sv, sa = few_step_sigmas(num_steps, video_shift, audio_shift)
    return 1.0 - sv[:-1], 1.0 - sa[:-1]


def sample_few_step_timesteps(generator, num_steps, video_shift, audio_shift):
    v, a = few_step_timesteps(num_steps, video_shift, audio_shift)
    i = int(torch.randint(len(v), (), generator=generator))
    return float(v[i]), float(a[i]), i


def sample_paired_timesteps(generator, u_min, u_max, video_shift, audio_shift):
    if not (0.0 <= u_min < u_max <= 1.0):
        raise ValueError(f"need 0 <= u_min < u_max <= 1, got [{u_min}, {u_max}]")
    u = u_min + (u_max - u_min) * float(torch.rand((), generator=generator))
    sv = video_shift * u / (1 + (video_shift - 1) * u)
    sa = audio_shift * u / (1 + (audio_shift - 1) * u)
    return 1.0 - sv, 1.0 - sa, u


def x0_from_velocity(sample, velocity, timestep):
    t = torch.as_tensor(timestep, dtype=sample.dtype, device=sample.device)
    return sample + (1 - t) * velocity


def euler_blend(sample, velocity, timestep, sigma, sigma_next):
    denoised = x0_from_velocity(sample, velocity, timestep)
    sigma = torch.as_tensor(sigma, dtype=sample.dtype, device=sample.device)
    sigma_next = torch.as_tensor(sigma_next, dtype=sample.dtype, device=sample.device)
    r = sigma_next / sigma
    return r * sample + (1.0 - r) * denoised


def build_layout(text_len, video_shape, num_audio_latents, device):
    """t2va `[text | audio | video]`, no conditioning rows."""
    _, F_, h, w = video_shape
    packed = build_packed_sequence(text_len, F_, h // PATCH_SIZE[1], w // PATCH_SIZE[2], num_audio_latents)
    return tuple(t.to(device) for t in (packed.position_ids, packed.token_tags, packed.video_indices,
                                        packed.audio_indices, packed.text_indices))


def _timestep_pair(seq_len, audio_indices, t_v, t_a, device):
    row_t = torch.full((seq_len,), float(t_v), dtype=torch.float32, device=device)
    if audio_indices.numel():
        row_t[audio_indices] = float(t_a)
    return torch.unique(row_t, sorted=True, return_inverse=True)


class PackedPrompt:
    """One prompt's packed geometry, built once per iteration and reused by every forward."""

    def __init__(self, prompt_embeds, video_shape, num_audio_latents, device):
        self.prompt_embeds = prompt_embeds.to(device, torch.bfloat16, non_blocking=True)[None]
        self.video_shape = tuple(video_shape)
        self.num_audio_latents = int(num_audio_latents)
        self.device = device
        (self.position_ids, self.token_tags, self.video_indices, self.audio_indices,
         self.text_indices) = build_layout(prompt_embeds.shape[0], self.video_shape,
                                           self.num_audio_latents, device)
        _, F_, h, w = self.video_shape
        gh, gw = h // PATCH_SIZE[1], w // PATCH_SIZE[2]
        self.seq_len = int(self.position_ids.shape[0])
        self.layout = layout_from_indices(self.video_indices, F_, gh * gw, seq_len=self.seq_len,
                                          frame_size=(gh, gw), text_indices=self.text_indices)
        self.num_video_rows = int(self.video_indices.numel())

    def inputs(self, video_rows, audio_rows, t_v, t_a):
        if not (0.0 <= float(t_v) < 1.0 and 0.0 <= float(t_a) < 1.0):
            raise ValueError(f"model-evaluation timesteps must be in [0, 1), got {t_v}, {t_a}")
        if video_rows.shape[0] != self.num_video_rows:
            raise ValueError("video rows do not match the packed geometry")
        if audio_rows.shape[0] != self.num_audio_latents * AUDIO_CHANNELS:
            raise ValueError("audio rows do not match the packed geometry")
        timestep, t_idx = _timestep_pair(self.seq_len, self.audio_indices, t_v, t_a, self.device)
        return dict(hidden_states=video_rows[None], audio_hidden_states=audio_rows[None],
                    encoder_hidden_states=self.prompt_embeds, timestep=timestep,
                    timestep_indices=t_idx, token_tags=self.token_tags,
                    position_ids=self.position_ids, video_indices=self.video_indices,
                    audio_indices=self.audio_indices, text_indices=self.text_indices,
                    return_dict=False)


def pack_noisy_batch(sample, device, noise_generator, sigma_generator, fixed_timesteps=None):
    """Dataset sample -> model inputs, fp32 velocity targets, the two timesteps, the layout."""
    # from the loader's pinned buffers these are asynchronous DMA copies
    video = sample["video_latents"].to(device, torch.float32, non_blocking=True)[None]
    audio = sample["audio_latents"].to(device, torch.float32, non_blocking=True)   # (2, 32, A)
    emb = sample["prompt_embeds"]
    audio_rows = audio.permute(0, 2, 1).reshape(-1, audio.shape[1])
    pp = PackedPrompt(emb, tuple(video.shape[1:]), audio.shape[-1], device)
    if fixed_timesteps is None:
        sv, sa = sample_sigmas(sigma_generator)
        t_v, t_a = 1.0 - sv, 1.0 - sa
    else:
        t_v, t_a = map(float, fixed_timesteps)
    noise_v = torch.randn(video.shape, generator=noise_generator, device=device, dtype=torch.float32)
    noise_a = torch.randn(audio_rows.shape, generator=noise_generator, device=device, dtype=torch.float32)
    noisy_video = patchify_video_latents(t_v * video + (1.0 - t_v) * noise_v, PATCH_SIZE)
    noisy_audio = t_a * audio_rows + (1.0 - t_a) * noise_a
    target_video = patchify_video_latents(video - noise_v, PATCH_SIZE)
    target_audio = audio_rows - noise_a
    return dict(inputs=pp.inputs(noisy_video, noisy_audio, t_v, t_a), target_video_rows=target_video,
                target_audio_rows=target_audio, t_v=t_v, t_a=t_a, layout=pp.layout)


def initial_noise(video_shape, num_audio_latents, generator, device):
    video = torch.randn((1, *video_shape), generator=generator, device=device, dtype=torch.float32)
    audio = torch.randn((num_audio_latents * AUDIO_CHANNELS, 32), generator=generator, device=device,
                        dtype=torch.float32)
    return patchify_video_latents(video, PATCH_SIZE), audio
