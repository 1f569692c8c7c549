"""The sampler: packed layout, seeded noise, the denoising loop, unpatchify.

Reference parity: src/inference/render.py:32-163 (`generate_latents`): the t2va /
keyframe (i2va, l2va, fl2va) / ref2va layouts, one layout per generation, two shifted
schedulers (12 video / 3 audio), conditioning noise drawn first, conditions pinned at
t = 0.999, per-row timesteps -> (unique timesteps, indices), Euler steps of the generated
rows only, device-synchronised per-NFE timing, and the channel-major audio rows.

`transformer` is any callable with the H3 forward signature: the eager H3Transformer, an
InferenceEngine, or a Ulysses/TP-parallel engine.
"""
import time
from dataclasses import dataclass

import torch

from vdn_minimax_h3_b200.models.layout import (AUDIO_CHANNELS, AUDIO_WIDTH, align_num_frames,
                                               audio_latent_num_frames, build_packed_sequence,
                                               layout_from_indices, patchify_video_latents,
                                               unpatchify_video_rows, video_latent_num_frames)
from vdn_minimax_h3_b200.models.scheduler import FlowMatchEulerScheduler

LATENT_H, LATENT_W = 48, 84           # the 768x1344 canvas through the 16x spatial VAE
KEYFRAME_NOISE_AUG = 0.999
PIXEL_MEAN, PIXEL_STD = (0.485, 0.456, 0.406), (0.229, 0.224, 0.225)
KEYFRAME_SLOTS = {"first": 0, "last": -1}


@dataclass
class RenderGeometry:
    num_frames: int
    num_latent_frames: int
    num_audio_latents: int
    latent_h: int
    latent_w: int
    channels: int
    patch: tuple

    @property
    def grid(self):
        return self.latent_h // self.patch[1], self.latent_w // self.patch[2]


def render_geometry(model_config, num_frames, latent_h=LATENT_H, latent_w=LATENT_W, audio=True,
                    num_latent_frames=None):
    """Geometry of a render; `num_latent_frames` overrides the 17n+5 -> 5n+2 rule (tests)."""
    nf = align_num_frames(num_frames)
    nlf = video_latent_num_frames(nf) if num_latent_frames is None else int(num_latent_frames)
    return RenderGeometry(num_frames=nf, num_latent_frames=nlf,
                          num_audio_latents=audio_latent_num_frames(nf) if audio else 0,
                          latent_h=latent_h, latent_w=latent_w,
                          channels=model_config.in_channels, patch=tuple(model_config.patch_size))


def build_inputs(geo: RenderGeometry, text_len, device, conditions=None):
    """Packed layout + SequenceLayout for a request; conditions = (anchors, latents)."""
    anchors, cond_latents = conditions if conditions else ((), [])
    gh, gw = geo.grid
    cond_grids, slots = [], []
    for a, c in zip(anchors, cond_latents):
        cond_grids.append((c.shape[-2] // geo.patch[1], c.shape[-1] // geo.patch[2]))
        slot = KEYFRAME_SLOTS.get(a, None)
        slots.append(geo.num_latent_frames - 1 if slot == -1 else (slot if slot is not None
                                                                   else -(len(slots) + 1)))
    packed = build_packed_sequence(text_len, geo.num_latent_frames, gh, gw, geo.num_audio_latents,
                                   condition_grids=cond_grids, keyframe_positions=slots)
    n_cond = packed.num_condition_rows
    layout = layout_from_indices(packed.video_indices[n_cond:], geo.num_latent_frames, gh * gw,
                                 seq_len=int(packed.position_ids.shape[0]), frame_size=(gh, gw),
                                 text_indices=packed.text_indices)
    dev = {k: getattr(packed, k).to(device) for k in
           ("position_ids", "token_tags", "video_indices", "audio_indices", "text_indices")}
    return packed, layout, dev


@torch.no_grad()
def generate_latents(transformer, prompt_embeds, num_frames, num_steps, seed, device,
                     model_config, video_shift=12.0, audio_shift=3.0, step_seconds=None,
                     conditions=None, latent_h=LATENT_H, latent_w=LATENT_W, audio=True,
                     on_layout=None, barrier=None, initial_noise=None, num_latent_frames=None,
                     on_step=None):
    """The denoising loop. Returns (latents [1, C, F, H, W] fp32, audio [2, 32, A] fp32).

    on_layout(layout) is called once before the loop (the hybrid's set_layout);
    barrier() (multi-GPU) runs before and after the loop; `step_seconds` (a list) gets the
    device-synchronised time of every NFE; `initial_noise` (video_rows, audio_rows) replaces
    the seeded draw (the e2e bench copies it from pinned host memory); `on_step(i)` runs on
    the host before each NFE is launched (the multi-GPU entry's heartbeat check)."""
    geo = render_geometry(model_config, num_frames, latent_h, latent_w, audio, num_latent_frames)
    text_len = prompt_embeds.shape[0]
    packed, layout, idx = build_inputs(geo, text_len, device, conditions)
    if on_layout is not None:
        on_layout(layout)
    sched, a_sched = FlowMatchEulerScheduler(video_shift), FlowMatchEulerScheduler(audio_shift)
    sched.set_timesteps(num_steps + 1, device=device)
    a_sched.set_timesteps(num_steps + 1, device=device)
    gen = torch.Generator(device).manual_seed(seed)
    n_cond = packed.num_condition_rows
    cond_rows = []
    if conditions:
        for c in conditions[1]:
            noise = torch.randn(c.shape, generator=gen, device=device, dtype=torch.float32)
            noised = sched.scale_noise(c.to(device, torch.float32), KEYFRAME_NOISE_AUG, noise)
            cond_rows.append(patchify_video_latents(noised, geo.patch))
    if initial_noise is None:
        latents = torch.randn((1, geo.channels, geo.num_latent_frames, geo.latent_h, geo.latent_w),
                              generator=gen, device=device, dtype=torch.float32)
        video_rows = patchify_video_latents(latents, geo.patch)
        audio_rows = torch.randn((geo.num_audio_latents * AUDIO_CHANNELS, AUDIO_WIDTH),
                                 generator=gen, device=device, dtype=torch.float32)
    else:
        video_rows, audio_rows = initial_noise
    if cond_rows:
        video_rows = torch.cat(cond_rows + [video_rows])
    if barrier is not None:
        barrier()
    S = int(packed.position_ids.shape[0])
    emb = prompt_embeds.to(device)[None]
    vid_idx, aud_idx = idx["video_indices"], idx["audio_indices"]
    for i in range(num_steps):
        if on_step is not None:
            on_step(i)
        t = float(sched.timesteps[i])
        a_t = float(a_sched.timesteps[i])
        started = time.perf_counter()
        row_t = torch.full((S,), t, dtype=torch.float32, device=device)
        if n_cond:
            row_t[vid_idx[:n_cond]] = max(t, KEYFRAME_NOISE_AUG)
        if aud_idx.numel():
            row_t[aud_idx] = a_t
        timestep, t_idx = torch.unique(row_t, sorted=True, return_inverse=True)
        v_pred, a_pred = transformer(
            hidden_states=video_rows[None], audio_hidden_states=audio_rows[None],
            encoder_hidden_states=emb, timestep=timestep, timestep_indices=t_idx,
            token_tags=idx["token_tags"], position_ids=idx["position_ids"],
            video_indices=vid_idx, audio_indices=aud_idx, text_indices=idx["text_indices"],
            return_dict=False)
        video_rows[n_cond:] = sched.step(v_pred[0, n_cond:].float(), t, video_rows[n_cond:], index=i)
        if aud_idx.numel():
            audio_rows = a_sched.step(a_pred[0].float(), a_t, audio_rows, index=i)
        if step_seconds is not None:
            if torch.device(device).type == "cuda":
                torch.cuda.synchronize(device)
            step_seconds.append(time.perf_counter() - started)
    if barrier is not None:
        if torch.device(device).type == "cuda":
            torch.cuda.synchronize(device)
        barrier()
    gh, gw = geo.grid
    latents = unpatchify_video_rows(video_rows[n_cond:], geo.channels, geo.num_latent_frames,
                                    geo.latent_h, geo.latent_w, geo.patch)
    audio_latents = audio_rows.reshape(AUDIO_CHANNELS, geo.num_audio_latents, AUDIO_WIDTH) \
        .permute(0, 2, 1).contiguous()
    return latents, audio_latents
