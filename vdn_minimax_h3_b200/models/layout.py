"""Packed-sequence geometry: the `[text | conditions | audio | video]` layout every forward
consumes, and the SequenceLayout view of it that both attention branches read.

Reference parity:
  * SequenceLayout / layout_from_indices: src/models/sequence_layout.py:9-88.
  * The packed layout itself is built in the reference by diffusers'
    MiniMaxH3PrepareLayoutStep.build_packed_sequence (called from
    src/inference/render.py:68-77 and src/training/t2va_batch.py:72-90). That builder is
    not part of the reference tree, so `build_packed_sequence` here is this package's own
    statement of the layout, with the properties the reference relies on: text rows
    first and contiguous, then one block of rows per conditioning frame or reference
    image, then the audio rows, then the generated video rows contiguous and t-major at
    the end (render.py:40-47; docs/inference.md:147-155).
  * Frame arithmetic (17n+5 pixel frames -> 5n+2 latent frames; 40 audio latents per
    second at 24 fps) follows the comments in src/inference/render.py:24,54-59 and
    src/training/dataset_h3_latents.py:5-9.
"""
from dataclasses import dataclass

import torch

VIDEO_TAG, TEXT_TAG, AUDIO_TAG = 0, 1, 2
MODALITY_NUM = 3
FPS = 24
AUDIO_LATENTS_PER_SECOND = 40
AUDIO_CHANNELS = 2
AUDIO_WIDTH = 32


@dataclass(frozen=True)
class SequenceLayout:
    """Where everything sits in one packed document (batch 1)."""
    seq_len: int
    video_start: int
    num_frames: int
    tokens_per_frame: int
    frame_height: int = 0
    frame_width: int = 0
    text_start: int = 0
    text_len: int = 0

    @property
    def video_end(self):
        return self.video_start + self.num_frames * self.tokens_per_frame

    @property
    def text_range(self):
        if not self.text_len:
            raise ValueError("this layout carries no text rows; pass text_indices to "
                             "layout_from_indices (the linear branch's text state needs them)")
        return self.text_start, self.text_start + self.text_len

    @property
    def frame_size(self):
        if not (self.frame_height and self.frame_width):
            raise ValueError("this layout carries no spatial grid; pass frame_size=(H, W)")
        if self.frame_height * self.frame_width != self.tokens_per_frame:
            raise ValueError(f"grid {self.frame_height}x{self.frame_width} != "
                             f"{self.tokens_per_frame} tokens/frame")
        return self.frame_height, self.frame_width

    def global_index(self, device):
        """Rows outside the video span (text, conditions, audio): dense in the softmax."""
        idx = torch.arange(self.seq_len, device=device)
        return torch.cat([idx[:self.video_start], idx[self.video_end:]])

    def global_ranges(self):
        """The non-video rows as at most two half-open ranges."""
        return [r for r in ((0, self.video_start), (self.video_end, self.seq_len)) if r[0] < r[1]]


def layout_from_indices(video_indices, num_latent_frames, tokens_per_frame, seq_len,
                        frame_size=None, text_indices=None):
    """SequenceLayout from the builder's index tensors, verifying contiguity."""
    video_start = int(video_indices[0].item())
    if int(video_indices[-1].item()) - video_start + 1 != video_indices.numel():
        raise ValueError("video rows are not contiguous in the packed sequence")
    if video_indices.numel() != num_latent_frames * tokens_per_frame:
        raise ValueError(f"{video_indices.numel()} video rows != {num_latent_frames} frames x "
                         f"{tokens_per_frame} tokens/frame")
    height, width = frame_size or (0, 0)
    if frame_size and height * width != tokens_per_frame:
        raise ValueError(f"frame_size {height}x{width} != {tokens_per_frame} tokens/frame")
    text_start, text_len = 0, 0
    if text_indices is not None and text_indices.numel():
        text_start = int(text_indices[0].item())
        if int(text_indices[-1].item()) - text_start + 1 != text_indices.numel():
            raise ValueError("text rows are not contiguous in the packed sequence")
        text_len = int(text_indices.numel())
    return SequenceLayout(seq_len=seq_len, video_start=video_start,
                          num_frames=num_latent_frames, tokens_per_frame=tokens_per_frame,
                          frame_height=height, frame_width=width,
                          text_start=text_start, text_len=text_len)


# ----------------------------------------------------------------------- frame arithmetic
def align_num_frames(num_frames, group=17, tail=5):
    """Round a pixel-frame count down to the 17n+5 grid the video VAE codes (min 5)."""
    if num_frames < tail:
        return tail
    return (num_frames - tail) // group * group + tail


def video_latent_num_frames(num_frames, group=17, tail=5):
    """17n+5 pixel frames -> 5n+2 latent frames (every 17 frames code as 5 latents)."""
    n = (align_num_frames(num_frames, group, tail) - tail) // group
    return 5 * n + 2


def audio_latent_num_frames(num_frames, fps=FPS, rate=AUDIO_LATENTS_PER_SECOND):
    """Audio latents covering `num_frames` video frames (40 per second at 24 fps)."""
    return int(round(num_frames * rate / fps))


# ------------------------------------------------------------------------------ patches
def patchify_video_latents(latents, patch=(1, 2, 2)):
    """[B, C, F, H, W] -> rows [F*(H/ph)*(W/pw), C*pt*ph*pw], t-major, channel-major patch."""
    b, c, f, h, w = latents.shape
    pt, ph, pw = patch
    x = latents.reshape(b, c, f // pt, pt, h // ph, ph, w // pw, pw)
    x = x.permute(0, 2, 4, 6, 1, 3, 5, 7)
    return x.reshape(b * (f // pt) * (h // ph) * (w // pw), c * pt * ph * pw)


def unpatchify_video_rows(rows, channels, frames, height, width, patch=(1, 2, 2)):
    """Inverse of patchify_video_latents for batch 1."""
    pt, ph, pw = patch
    x = rows.reshape(1, frames // pt, height // ph, width // pw, channels, pt, ph, pw)
    x = x.permute(0, 4, 1, 5, 2, 6, 3, 7)
    return x.reshape(1, channels, frames, height, width).contiguous()


# ------------------------------------------------------------------------ packed layout
@dataclass
class PackedLayout:
    position_ids: torch.Tensor    # [S, 3] int64 (t, h, w)
    token_tags: torch.Tensor      # [S] int64
    video_indices: torch.Tensor   # conditioning rows first, then the generated rows
    audio_indices: torch.Tensor
    text_indices: torch.Tensor
    num_condition_rows: int
    condition_frames: int

    def as_tuple(self):
        return (self.position_ids, self.token_tags, self.video_indices, self.audio_indices,
                self.text_indices, self.num_condition_rows, self.condition_frames)


def build_packed_sequence(text_len, num_latent_frames, grid_h, grid_w, num_audio_latents,
                          audio_channels=AUDIO_CHANNELS, condition_grids=(),
                          keyframe_positions=()):
    """The packed document `[text | conditions | audio | video]`.

    text_len            prompt rows (tag TEXT); positions (i, i, i) in order.
    condition_grids     one (h, w) grid per conditioning block (keyframes or reference
                        images); each block is one frame of rows tagged VIDEO and sits
                        between the text and the audio, outside the generated span.
    keyframe_positions  the latent time index each conditioning block is anchored at
                        (i2va: 0; l2va: F-1; references: negative slots before frame 0).
    audio rows          `audio_channels * num_audio_latents` rows of width 32, channel
                        major, tag AUDIO; positions (t_audio, 0, 0) on the video clock.
    video rows          F * grid_h * grid_w rows, t-major, positions (t, h, w).

    Returns a PackedLayout; `video_indices` lists the conditioning rows first (as the
    reference's builder does), so `video_indices[num_condition_rows:]` is the generated
    span that SequenceLayout describes.
    """
    pos, tags = [], []
    text_pos = torch.arange(text_len, dtype=torch.long)
    pos.append(torch.stack([text_pos, text_pos, text_pos], dim=1))
    tags.append(torch.full((text_len,), TEXT_TAG, dtype=torch.long))
    offset = text_len
    t_base = text_len  # video clock starts after the prompt's positions

    cond_rows = []
    for block, (h, w) in enumerate(condition_grids):
        t_slot = keyframe_positions[block] if block < len(keyframe_positions) else -(block + 1)
        hh, ww = torch.meshgrid(torch.arange(h), torch.arange(w), indexing="ij")
        tt = torch.full_like(hh, t_base + t_slot)
        pos.append(torch.stack([tt.flatten(), hh.flatten(), ww.flatten()], dim=1))
        tags.append(torch.full((h * w,), VIDEO_TAG, dtype=torch.long))
        cond_rows.append(torch.arange(offset, offset + h * w))
        offset += h * w

    n_audio = audio_channels * num_audio_latents
    audio_idx = torch.arange(offset, offset + n_audio)
    if n_audio:
        a_t = torch.arange(num_audio_latents).repeat(audio_channels)
        a_t = t_base + (a_t * num_latent_frames) // max(num_audio_latents, 1)
        pos.append(torch.stack([a_t, torch.zeros_like(a_t), torch.full_like(a_t, -1)], dim=1))
        tags.append(torch.full((n_audio,), AUDIO_TAG, dtype=torch.long))
    offset += n_audio

    n_video = num_latent_frames * grid_h * grid_w
    tt, hh, ww = torch.meshgrid(torch.arange(num_latent_frames), torch.arange(grid_h),
                                torch.arange(grid_w), indexing="ij")
    pos.append(torch.stack([tt.flatten() + t_base, hh.flatten(), ww.flatten()], dim=1))
    tags.append(torch.full((n_video,), VIDEO_TAG, dtype=torch.long))
    video_idx = torch.arange(offset, offset + n_video)
    offset += n_video

    num_condition_rows = sum(h * w for h, w in condition_grids)
    video_indices = torch.cat(cond_rows + [video_idx]) if cond_rows else video_idx
    return PackedLayout(
        position_ids=torch.cat(pos).long(), token_tags=torch.cat(tags).long(),
        video_indices=video_indices, audio_indices=audio_idx,
        text_indices=torch.arange(0, text_len), num_condition_rows=num_condition_rows,
        condition_frames=len(condition_grids))


def layout_for(packed: PackedLayout, num_latent_frames, grid_h, grid_w):
    """SequenceLayout of a PackedLayout's generated video span."""
    return layout_from_indices(packed.video_indices[packed.num_condition_rows:],
                               num_latent_frames, grid_h * grid_w,
                               seq_len=int(packed.position_ids.shape[0]),
                               frame_size=(grid_h, grid_w), text_indices=packed.text_indices)
