"""Decode-and-save with decoder STAND-INS of the real VAEs' geometry and a realistic cost.

The H3 video VAE (24 latent channels, 16x spatial, 17n+5 pixel frames from 5n+2 latent
frames) and the stereo audio VAE are external to the reference (diffusers, absent here).
`VideoDecoderStandIn` is a random-init decoder with that geometry and the compute of a
video VAE decoder of the usual shape:
  * latent resolution: a 3x3x3 conv 24 -> 384 channels and a residual block of two 3x3x3
    convs (temporal mixing happens here, where it is cheap);
  * the temporal map 5n+2 -> 17n+5 (pixel frame p reads latent frame p * F_lat // F_pix);
  * four per-frame stages, each a 2x nearest upsample, a 3x3 conv and a residual block of
    two 3x3 convs, at 384 / 384 / 192 / 96 channels, then a 3x3 conv to RGB and a tanh:
    ~700 TFLOP for a 14.4 s 768 x 1344 clip (`flops()`).
Pixel frames are decoded in chunks (bounded memory) and, under sequence parallelism, split
across the ranks and gathered on rank 0. `AudioDecoderStandIn` maps the 32-wide audio
latents to 48 kHz stereo samples. Both are labelled stand-ins wherever they run; their
output is not a picture or a sound of anything.

decode_and_save follows reference src/inference/render.py:166-198: decode, pixel
de-normalisation, uint8 frames, atomic `.partial.mp4` -> rename; the soundtrack is muxed into
the same mp4 as 16-bit PCM (inference/mp4mux.py) after OpenCV encodes the video track --
frame ranges in parallel threads, joined into one track by the same muxer.
"""
import os
import time

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from vdn_minimax_h3_b200.inference.render import PIXEL_MEAN, PIXEL_STD
from vdn_minimax_h3_b200.models.layout import FPS

AUDIO_SAMPLE_RATE = 48000
VIDEO_WIDTHS = (384, 384, 192, 96)


def pixel_frames(latent_frames):
    """17n+5 pixel frames for 5n+2 latent frames (other counts: 3.4x, rounded down)."""
    n, rest = divmod(latent_frames - 2, 5)
    return 17 * n + 5 if rest == 0 and latent_frames >= 2 else max(1, latent_frames * 17 // 5)


class _Res(nn.Module):
    def __init__(self, conv, ch):
        super().__init__()
        self.a, self.b = conv(ch, ch), conv(ch, ch)

    def forward(self, x):
        return x + self.b(F.silu(self.a(F.silu(x))))


class VideoDecoderStandIn(nn.Module):
    def __init__(self, latent_channels=24, widths=VIDEO_WIDTHS, seed=0, chunk_frames=8):
        super().__init__()
        conv3 = lambda i, o: nn.Conv3d(i, o, 3, padding=1)  # noqa: E731
        conv2 = lambda i, o: nn.Conv2d(i, o, 3, padding=1)  # noqa: E731
        with torch.random.fork_rng(devices=[]):
            torch.manual_seed(seed)
            self.conv_in = conv3(latent_channels, widths[0])
            self.res_in = _Res(conv3, widths[0])
            chans = (widths[0],) + tuple(widths)
            self.ups = nn.ModuleList(nn.ModuleList([conv2(ci, co), _Res(conv2, co)])
                                     for ci, co in zip(chans[:-1], chans[1:]))
            self.conv_out = conv2(widths[-1], 3)
        self.spatial = 2 ** len(widths)
        self.chunk_frames = chunk_frames

    def flops(self, latent_shape):
        """Multiply-add FLOPs of one decode of latents [1, C, F, h, w]."""
        _, c, f, h, w = latent_shape
        w0 = self.conv_in.out_channels
        total = 2 * f * h * w * 27 * (c * w0 + 2 * w0 * w0)
        p, hh, ww = pixel_frames(f), h, w
        for conv, _ in self.ups:
            hh, ww = 2 * hh, 2 * ww
            ci, co = conv.in_channels, conv.out_channels
            total += 2 * p * hh * ww * 9 * (ci * co + 2 * co * co)
        return total + 2 * p * hh * ww * 9 * self.conv_out.in_channels * 3

    def prepare(self, device):
        """Moves to `device`; on CUDA bf16 weights in the channels-last layouts cuDNN's
        tensor-core convolutions prefer (3-D stage channels_last_3d, 2-D stages channels_last)."""
        self.to(device)
        if torch.device(device).type == "cuda":
            self.to(dtype=torch.bfloat16)
            for m in (self.conv_in, self.res_in):
                m.to(memory_format=torch.channels_last_3d)
            for m in (self.ups, self.conv_out):
                m.to(memory_format=torch.channels_last)
        return self

    def latent_stage(self, latents):
        x = latents.to(self.conv_in.weight.dtype)
        if x.is_cuda:
            x = x.contiguous(memory_format=torch.channels_last_3d)
        return self.res_in(self.conv_in(x))

    def frames(self, z, p0, p1, num_pixel):
        """Pixel frames [p0, p1) in [-1, 1], [n, 3, H, W], from the latent-stage output z."""
        f = z.shape[2]
        idx = (torch.arange(p0, p1, device=z.device) * f) // num_pixel
        x = z[0].index_select(1, idx).transpose(0, 1)          # [n, C, h, w]
        if x.is_cuda:
            x = x.contiguous(memory_format=torch.channels_last)
        for conv, res in self.ups:
            x = res(conv(F.interpolate(x, scale_factor=2.0, mode="nearest")))
        return torch.tanh(self.conv_out(F.silu(x)))

    def forward(self, latents):
        """[1, C, F, h, w] -> [1, 3, 17n+5, 16h, 16w] in [-1, 1] (all frames, one rank)."""
        z = self.latent_stage(latents)
        P = pixel_frames(latents.shape[2])
        out = [self.frames(z, a, min(a + self.chunk_frames, P), P)
               for a in range(0, P, self.chunk_frames)]
        return torch.cat(out).transpose(0, 1)[None]


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


def _to_uint8(video):
    """[n, 3, H, W] in [-1, 1] -> uint8 [n, H, W, 3] after the pixel de-normalisation."""
    mean = torch.tensor(PIXEL_MEAN, device=video.device).view(1, -1, 1, 1)
    std = torch.tensor(PIXEL_STD, device=video.device).view(1, -1, 1, 1)
    pix = (video.float() * std + mean).clamp(0, 1)
    return (pix * 255).round().to(torch.uint8).permute(0, 2, 3, 1)


def _ranks(group, single=False):
    import torch.distributed as dist
    on = not single and dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if on else 1
    return (dist.get_rank(group) if world > 1 else 0), world


@torch.no_grad()
def decode_share(latents, video_decoder, rank=0, world=1):
    """This rank's contiguous share of the pixel frames, uint8 [n, H, W, 3] on the latents'
    device, and the total pixel frame count P (shares of ceil(P / world) frames)."""
    dev = latents.device
    dec = video_decoder.prepare(dev)
    z = dec.latent_stage(latents)
    P = pixel_frames(latents.shape[2])
    share = -(-P // world)
    p0, p1 = min(rank * share, P), min((rank + 1) * share, P)
    parts = [_to_uint8(dec.frames(z, a, min(a + dec.chunk_frames, p1), P))
             for a in range(p0, p1, dec.chunk_frames)]
    H, W = latents.shape[3] * dec.spatial, latents.shape[4] * dec.spatial
    mine = torch.cat(parts) if parts else torch.empty(0, H, W, 3, dtype=torch.uint8, device=dev)
    return mine, P


@torch.no_grad()
def decode_frames(latents, video_decoder, group=None, single=False):
    """uint8 frames [P, H, W, 3] on the host of rank 0 (None elsewhere). Under an initialised
    process group (unless `single`) every rank decodes a contiguous share of the pixel frames
    and rank 0 gathers them."""
    import torch.distributed as dist
    rank, world = _ranks(group, single)
    mine, P = decode_share(latents, video_decoder, rank, world)
    dev = mine.device
    H, W = mine.shape[1], mine.shape[2]
    share = -(-P // world)
    if world == 1:
        return mine.cpu()
    pad = torch.zeros(share, H, W, 3, dtype=torch.uint8, device=dev)
    pad[:mine.shape[0]].copy_(mine)
    full = torch.empty(world * share, H, W, 3, dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(full, pad, group=group)
    return full[:P].cpu() if rank == 0 else None


@torch.no_grad()
def decode(latents, audio_latents, video_decoder, audio_decoder):
    """One process decodes everything: (uint8 frames [P, H, W, 3], audio [2, samples]) on
    the host."""
    frames = decode_frames(latents, video_decoder, single=True)
    audio = audio_decoder.to(latents.device)(audio_latents.float()).clamp(-1, 1)
    return frames, audio.cpu()


def write_mp4(frames, path, fps=FPS):
    import cv2
    h, w = frames.shape[1], frames.shape[2]
    writer = cv2.VideoWriter(path, cv2.VideoWriter_fourcc(*"mp4v"), fps, (w, h))
    if not writer.isOpened():
        raise RuntimeError(f"cannot open an mp4 writer for {path}")
    for f in frames.numpy():
        writer.write(np.ascontiguousarray(f[:, :, ::-1]))  # RGB -> BGR
    writer.release()


def encode_mp4(frames, fps=FPS, workers=None, min_frames=8):
    """The bytes of a video-only mp4 of `frames` ([P, H, W, 3] uint8): contiguous frame
    ranges are encoded by parallel OpenCV writers (the encoder releases the GIL), each range
    starting on a key frame, and joined into one track (mp4mux.concat_video_segments)."""
    import tempfile
    from concurrent.futures import ThreadPoolExecutor
    from vdn_minimax_h3_b200.inference.mp4mux import concat_video_segments
    P = frames.shape[0]
    workers = workers or min(16, os.cpu_count() or 1)
    k = max(1, min(workers, P // max(min_frames, 1)))
    cuts = [round(i * P / k) for i in range(k + 1)]
    with tempfile.TemporaryDirectory(prefix="vdn_mp4_") as tmp:
        paths = [os.path.join(tmp, f"seg{i}.mp4") for i in range(k)]
        with ThreadPoolExecutor(k) as pool:
            list(pool.map(lambda i: write_mp4(frames[cuts[i]:cuts[i + 1]], paths[i], fps), range(k)))
        segments = []
        for path in paths:
            with open(path, "rb") as f:
                segments.append(f.read())
    return concat_video_segments(segments)


def mux_pcm(video_mp4, audio, rate=AUDIO_SAMPLE_RATE):
    """The mp4 bytes `video_mp4` with `audio` ([channels, samples] in [-1, 1]) added as a
    16-bit PCM track."""
    from vdn_minimax_h3_b200.inference.mp4mux import add_pcm_track
    pcm = (audio.clamp(-1, 1).numpy().T * 32767).astype(np.int16)
    return add_pcm_track(video_mp4, pcm, rate)


@torch.no_grad()
def decode_and_save(latents, audio_latents, out_path, video_decoder=None, audio_decoder=None,
                    group=None, timings=None):
    """Decodes and writes one mp4 with sound on rank 0; returns the path there and None on
    the other ranks. Under an initialised process group every rank of `group` decodes a
    contiguous share of the frames, copies only that share to its host and encodes it there
    (its own key frame first); rank 0 gathers the encoded segments -- a few MB instead of
    the raw frames -- and joins them into one track (mp4mux.concat_video_segments).
    `timings` (a dict) receives the seconds spent decoding (to host), encoding (with the
    segment gather and join) and muxing on this rank."""
    video_decoder = video_decoder or VideoDecoderStandIn(latents.shape[1])
    audio_decoder = audio_decoder or AudioDecoderStandIn(audio_latents.shape[1])
    rank, world = _ranks(group)
    t0 = time.perf_counter()
    mine, P = decode_share(latents, video_decoder, rank, world)
    frames = mine.cpu()
    audio = audio_decoder.to(latents.device)(audio_latents.float()).clamp(-1, 1).cpu() \
        if rank == 0 else None
    t1 = time.perf_counter()
    if world == 1:
        video = encode_mp4(frames)
    else:
        import torch.distributed as dist
        from vdn_minimax_h3_b200.inference.mp4mux import concat_video_segments
        threads = max(1, (os.cpu_count() or 1) // world)
        seg = encode_mp4(frames, workers=threads) if frames.shape[0] else b""
        segs = [None] * world
        dist.all_gather_object(segs, seg, group=group)
        if rank != 0:
            if timings is not None:
                timings.update(decode_s=t1 - t0, encode_s=time.perf_counter() - t1)
            return None
        video = concat_video_segments([x for x in segs if x])
    os.makedirs(os.path.dirname(os.path.abspath(out_path)) or ".", exist_ok=True)
    stem, ext = os.path.splitext(out_path)
    partial = f"{stem}.partial{ext}"
    t2 = time.perf_counter()
    with open(partial, "wb") as f:
        f.write(mux_pcm(video, audio))
    os.replace(partial, out_path)
    if timings is not None:
        timings.update(decode_s=t1 - t0, encode_s=t2 - t1, mux_s=time.perf_counter() - t2,
                       frames=int(P))
    return out_path
