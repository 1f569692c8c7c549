"""Decode-and-save with decoder STAND-INS of the right geometry.

The H3 video VAE (24 latent channels, 16x spatial, 17n+5 <- 5n+2 temporal) and the stereo
audio VAE are external to the reference (diffusers, absent here) and are not part of this
package. To keep the render path whole, `VideoDecoderStandIn` / `AudioDecoderStandIn` map
latents to pixels / samples with the same shapes using random weights: a 1x1x1 projection
to 3 x 16 x 16 channels + depth-to-space, a 17-from-5 temporal upsampling and a tanh, and a
linear audio head. They are labelled stand-ins everywhere they are used; their output is
not a picture of anything.

decode_and_save mirrors reference src/inference/render.py:166-198: decode, pixel
de-normalisation, uint8 frames, atomic `.partial.mp4` -> rename. Video goes through
OpenCV's mp4 writer; the soundtrack is written beside it as a 16-bit PCM `.wav` (no muxer
is available offline).
"""
import os
import wave

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from vdn_minimax_h3_b200.inference.render import PIXEL_MEAN, PIXEL_STD
from vdn_minimax_h3_b200.models.layout import FPS

AUDIO_SAMPLE_RATE = 48000


class VideoDecoderStandIn(nn.Module):
    def __init__(self, latent_channels=24, spatial=16, seed=0):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.spatial = spatial
        self.proj = nn.Parameter(torch.randn(3 * spatial * spatial, latent_channels, generator=g)
                                 / latent_channels ** 0.5)

    def forward(self, latents):
        """[1, C, F, h, w] -> [1, 3, 17n+5, 16h, 16w] in [-1, 1]."""
        b, c, f, h, w = latents.shape
        x = torch.einsum("oc,bcfhw->bofhw", self.proj.to(latents.dtype), latents)
        x = x.reshape(b, 3, self.spatial, self.spatial, f, h, w).permute(0, 1, 4, 5, 2, 6, 3)
        x = x.reshape(b, 3, f, h * self.spatial, w * self.spatial)
        n = (f - 2) // 5
        frames = 17 * n + 5
        x = F.interpolate(x, size=(frames, x.shape[-2], x.shape[-1]), mode="trilinear",
                          align_corners=True) if frames != f else x
        return torch.tanh(x)


class AudioDecoderStandIn(nn.Module):
    def __init__(self, width=32, samples_per_latent=AUDIO_SAMPLE_RATE // 40, seed=1):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.spl = samples_per_latent
        self.proj = nn.Parameter(torch.randn(samples_per_latent, width, generator=g) / width ** 0.5)

    def forward(self, audio_latents):
        """[2, 32, A] -> [2, A * samples_per_latent] in [-1, 1]."""
        y = torch.einsum("sw,cwa->cas", self.proj.to(audio_latents.dtype), audio_latents)
        return torch.tanh(y.reshape(audio_latents.shape[0], -1))


@torch.no_grad()
def decode(latents, audio_latents, video_decoder, audio_decoder):
    dev = latents.device
    video = video_decoder.to(dev)(latents.float())
    mean = torch.tensor(PIXEL_MEAN, device=dev).view(1, -1, 1, 1, 1)
    std = torch.tensor(PIXEL_STD, device=dev).view(1, -1, 1, 1, 1)
    video = (video.float() * std + mean).clamp(0, 1)
    audio = audio_decoder.to(dev)(audio_latents.float()).clamp(-1, 1)
    frames = (video[0].permute(1, 2, 3, 0) * 255).round().to(torch.uint8).cpu()  # (F, H, W, 3)
    return frames, audio.cpu()


def write_mp4(frames, path, fps=FPS):
    import cv2
    h, w = frames.shape[1], frames.shape[2]
    writer = cv2.VideoWriter(path, cv2.VideoWriter_fourcc(*"mp4v"), fps, (w, h))
    if not writer.isOpened():
        raise RuntimeError(f"cannot open an mp4 writer for {path}")
    for f in frames.numpy():
        writer.write(f[:, :, ::-1])  # RGB -> BGR
    writer.release()


def write_wav(audio, path, rate=AUDIO_SAMPLE_RATE):
    pcm = (audio.clamp(-1, 1).numpy().T * 32767).astype(np.int16)
    with wave.open(path, "wb") as w:
        w.setnchannels(pcm.shape[1])
        w.setsampwidth(2)
        w.setframerate(rate)
        w.writeframes(pcm.tobytes())


def decode_and_save(latents, audio_latents, out_path, video_decoder=None, audio_decoder=None):
    video_decoder = video_decoder or VideoDecoderStandIn(latents.shape[1])
    audio_decoder = audio_decoder or AudioDecoderStandIn(audio_latents.shape[1])
    frames, audio = decode(latents, audio_latents, video_decoder, audio_decoder)
    os.makedirs(os.path.dirname(os.path.abspath(out_path)) or ".", exist_ok=True)
    stem, ext = os.path.splitext(out_path)
    partial = f"{stem}.partial{ext}"
    write_mp4(frames, partial)
    os.replace(partial, out_path)
    write_wav(audio, f"{stem}.partial.wav")
    os.replace(f"{stem}.partial.wav", f"{stem}.wav")
    return out_path
