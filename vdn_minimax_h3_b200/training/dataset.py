"""The latents dataset: an index jsonl of `latent_path`s; sidecars by path arithmetic
(<root>/video/<name>, <root>/audio/<name>, <root>/text/<name>), one fixed latent shape per
dataset, a text-only mode for Stage DMD (reference src/training/dataset_h3_latents.py), and
a synthetic dataset of the same record layout for runs with no data on disk."""
import json
import os

import torch
from torch.utils.data import Dataset


class H3LatentT2VADataset(Dataset):
    def __init__(self, index_file, text_only=False):
        self.text_only = text_only
        self.records = []
        with open(index_file) as f:
            for line in f:
                rec = json.loads(line)
                if "error" not in rec:
                    self.records.append(rec["latent_path"])
        if not self.records:
            raise RuntimeError(f"no usable rows in {index_file}")
        first = torch.load(self.records[0], map_location="cpu", weights_only=True)
        self.video_shape = tuple(first.shape)

    def __len__(self):
        return len(self.records)

    def __getitem__(self, idx):
        vp = self.records[idx]
        base, name = os.path.dirname(os.path.dirname(vp)), os.path.basename(vp)
        text = torch.load(os.path.join(base, "text", name), map_location="cpu", weights_only=True)
        if self.text_only:
            return {"prompt_embeds": text["prompt_embeds"], "text_token_tags": text["text_token_tags"]}
        video = torch.load(vp, map_location="cpu", weights_only=True)
        audio = torch.load(os.path.join(base, "audio", name), map_location="cpu", weights_only=True)
        if tuple(video.shape) != self.video_shape:
            raise ValueError(f"{vp}: shape {tuple(video.shape)} != {self.video_shape}")
        return {"video_latents": video, "audio_latents": audio, "prompt_embeds": text["prompt_embeds"],
                "text_token_tags": text["text_token_tags"]}


class SyntheticLatentDataset(Dataset):
    """Random-normal clips of a fixed geometry (deterministic per index)."""

    def __init__(self, length, video_shape=(24, 81, 48, 84), num_audio_latents=455, text_len=800,
                 text_dim=5120, seed=0, text_only=False):
        self.length, self.video_shape = length, tuple(video_shape)
        self.num_audio_latents, self.text_len, self.text_dim = num_audio_latents, text_len, text_dim
        self.seed, self.text_only = seed, text_only

    def __len__(self):
        return self.length

    def __getitem__(self, idx):
        g = torch.Generator().manual_seed(self.seed * 1000003 + idx)
        out = {"prompt_embeds": torch.randn(self.text_len, self.text_dim, generator=g).to(torch.bfloat16),
               "text_token_tags": torch.ones(self.text_len, dtype=torch.long)}
        if not self.text_only:
            out["video_latents"] = torch.randn(self.video_shape, generator=g).to(torch.bfloat16)
            out["audio_latents"] = torch.randn(2, 32, self.num_audio_latents, generator=g).to(torch.bfloat16)
        return out


def write_synthetic_dataset(root, n, video_shape, num_audio_latents, text_len, text_dim, seed=0):
    """Materialise a SyntheticLatentDataset in the on-disk layout; returns the index path."""
    ds = SyntheticLatentDataset(n, video_shape, num_audio_latents, text_len, text_dim, seed)
    for sub in ("video", "audio", "text"):
        os.makedirs(os.path.join(root, sub), exist_ok=True)
    index = os.path.join(root, "index.jsonl")
    with open(index, "w") as f:
        for i in range(n):
            s = ds[i]
            name = f"clip{i:05d}.pt"
            torch.save(s["video_latents"], os.path.join(root, "video", name))
            torch.save(s["audio_latents"], os.path.join(root, "audio", name))
            torch.save({"prompt_embeds": s["prompt_embeds"], "text_token_tags": s["text_token_tags"]},
                       os.path.join(root, "text", name))
            f.write(json.dumps({"latent_path": os.path.join(root, "video", name)}) + "\n")
    return index


def collate_single(samples):
    assert len(samples) == 1
    return samples[0]
