"""Conditioning encoders for the prompt cache: the text/vision conditioner (Qwen3-VL hidden
state after decoder layer 50), the keyframe / reference image presentation, and the VAE
encode of keyframes.

Reference parity: src/inference/encode_prompt.py:29-52 (t2va text), encode_keyframes.py:
75-156 (canvas, reference sizing, `<Picture i>` presentation, vision rows tagged VIDEO),
encode_keyframes.py:224-229 (seed-42 posterior sample of each keyframe).

Two encoder back ends share one interface (`encode(token_ids, images) -> (L, 5120) bf16`):
  * `Qwen3VLConditioner` loads a MiniMax-H3 snapshot (processor/, text_encoder/) through
    transformers and returns `hidden_states[50]`, exactly the reference's call;
  * `StandInConditioner` needs no weights: a byte-level tokenizer and seeded embedding
    tables (token rows; vision rows from 14x14-pixel patch means through a seeded
    projection). It produces caches of the right shapes, tags and modes for offline runs
    and tests; its embeddings carry no meaning.
`KeyframeVaeStandIn` plays the MiniMax-H3 VAE's encoder geometry (16x spatial
compression, 24 latent channels, one latent frame per image) for offline caches.
"""
import math

import numpy as np
import torch

TEXT_ENCODER_LAYER = 50
VIDEO_TAG, TEXT_TAG = 0, 1
EMBED_WIDTH = 5120
CANVAS_MULTIPLE, CANVAS_SHORT_EDGE, CANVAS_MAX_PIXELS = 32, 768, 768 * 1344
MAX_ASPECT = 4
REFERENCE_SHORT_EDGE = 768
KEYFRAME_ENCODE_SEED = 42
VAE_SPATIAL, LATENT_CHANNELS = 16, 24
PIXEL_MEAN, PIXEL_STD = 0.5, 0.5

# the opening line MiniMax-H3 expects per keyframe mode (a substring marker, the full line)
KEYFRAME_INSTRUCTIONS = {
    ("first",): ("is fully referenced",
                 "For the target video, at 0.00 seconds into the target video, "
                 "<Picture 1> (from [Shot 1]) is fully referenced."),
    ("last",): ("How the reference pictures align",
                "How the reference pictures align with the target video — <Picture 1> "
                "(from [Shot N]) aligns with the S.SS-second mark of the target video."),
    ("first", "last"): ("How the reference pictures align",
                        "How the reference pictures align with the target video — "
                        "Picture 1 (from Shot 1) aligns with the 0.00-second mark of the "
                        "target video; Picture 2 (from Shot N) aligns with the S.SS-second "
                        "mark of the target video."),
}


# ------------------------------------------------------------------------------ geometry
def resolve_canvas_size(width, height, multiple=CANVAS_MULTIPLE, short_edge=CANVAS_SHORT_EDGE,
                        max_pixels=CANVAS_MAX_PIXELS):
    """Canvas (height, width) of an image's aspect ratio: the short side `short_edge`, both
    sides multiples of `multiple`, the long side shortened (in steps of `multiple`) until
    the area fits `max_pixels`. 16:9 -> (768, 1344), the H3 render canvas."""
    if width <= 0 or height <= 0:
        raise ValueError("image sides must be positive")
    landscape = width >= height
    long_side = max(width, height) * short_edge / min(width, height)
    short = max(multiple, round(short_edge / multiple) * multiple)
    long_ = max(short, round(long_side / multiple) * multiple)
    while long_ * short > max_pixels and long_ > short:
        long_ -= multiple
    return (short, long_) if landscape else (long_, short)


def put_on_canvas(images):
    """The canvas follows the first image's aspect ratio; the first image is stretched onto
    it, every other one scaled to cover it and centre-cropped. -> (images, height, width)."""
    from PIL import Image
    height, width = resolve_canvas_size(*images[0].size)
    out = []
    for i, im in enumerate(images):
        im = im.convert("RGB")
        if im.size == (width, height):
            out.append(im)
        elif i == 0:
            out.append(im.resize((width, height), Image.Resampling.LANCZOS))
        else:
            scale = max(width / im.size[0], height / im.size[1])
            size = (max(width, round(im.size[0] * scale)), max(height, round(im.size[1] * scale)))
            left, top = (size[0] - width) // 2, (size[1] - height) // 2
            out.append(im.resize(size, Image.Resampling.LANCZOS)
                       .crop((left, top, left + width, top + height)))
    return out, height, width


def normalize_references(images, short_edge=REFERENCE_SHORT_EDGE):
    """Each reference on a short edge of `short_edge` at its own aspect ratio (sides rounded
    to the canvas multiple, LANCZOS); aspect ratios beyond 4:1 are refused."""
    from PIL import Image
    out = []
    for im in images:
        im = im.convert("RGB")
        w, h = im.size
        if w > MAX_ASPECT * h or h > MAX_ASPECT * w:
            raise ValueError(f"a reference image must be within 1:{MAX_ASPECT} and "
                             f"{MAX_ASPECT}:1, got {w}x{h}")
        scale = short_edge / min(w, h)
        target = tuple(max(CANVAS_MULTIPLE, round(s * scale / CANVAS_MULTIPLE) * CANVAS_MULTIPLE)
                       for s in (w, h))
        out.append(im if im.size == target else im.resize(target, Image.Resampling.LANCZOS))
    return out


def check_instruction(prompt, anchors):
    """True when the prompt opens with the keyframe mode's instruction line (the reference
    warns, never refuses)."""
    marker, _ = KEYFRAME_INSTRUCTIONS[tuple(anchors)]
    opening = next((line for line in prompt.splitlines() if line.strip()), "")
    return marker.lower() in opening.lower()


# ---------------------------------------------------------------------------- encoders
class StandInConditioner:
    """Weight-free conditioner with the real one's interface and output geometry."""

    PATCH = 14
    MERGE = 2          # vision tokens per 28x28 pixels, like Qwen3-VL's 2x2 patch merge
    VOCAB = 256 + 3    # bytes + <|vision_start|>, <|image_pad|>, <|vision_end|>

    def __init__(self, width=EMBED_WIDTH, seed=0):
        g = torch.Generator().manual_seed(seed)
        self.width = width
        self.table = torch.randn(self.VOCAB, width, generator=g) * 0.02
        self.pos = torch.randn(4096, width, generator=g) * 0.01
        self.proj = torch.randn(3 * self.PATCH * self.PATCH * self.MERGE ** 2, width,
                                generator=g) / math.sqrt(3 * (self.PATCH * self.MERGE) ** 2)
        self.vision_start, self.image_pad, self.vision_end = 256, 257, 258

    def tokenize(self, text):
        return list(text.encode("utf-8"))

    def image_tokens(self, image):
        side = self.PATCH * self.MERGE
        return max(1, image.size[0] // side) * max(1, image.size[1] // side)

    def _vision_rows(self, image):
        side = self.PATCH * self.MERGE
        a = torch.from_numpy(np.asarray(image.convert("RGB"), dtype=np.float32) / 255.0)
        gh, gw = max(1, a.shape[0] // side), max(1, a.shape[1] // side)
        a = a[:gh * side, :gw * side]
        if a.shape[0] < side or a.shape[1] < side:
            a = torch.nn.functional.pad(a, (0, 0, 0, side - a.shape[1], 0, side - a.shape[0]))
        patches = a.reshape(gh, side, gw, side, 3).permute(0, 2, 1, 3, 4).reshape(gh * gw, -1)
        return (patches - PIXEL_MEAN) / PIXEL_STD @ self.proj

    @torch.no_grad()
    def encode(self, token_ids, images=()):
        ids = torch.tensor(token_ids, dtype=torch.long)
        emb = self.table[ids].clone()
        pad_rows = (ids == self.image_pad).nonzero().flatten()
        vis = [self._vision_rows(im) for im in images]
        if vis:
            v = torch.cat(vis)
            if v.shape[0] != pad_rows.numel():
                raise ValueError("vision rows do not match the <|image_pad|> tokens")
            emb[pad_rows] += v
        n = emb.shape[0]
        emb += self.pos[torch.arange(n) % self.pos.shape[0]]
        return emb.to(torch.bfloat16)


class Qwen3VLConditioner:
    """The MiniMax-H3 conditioner from a local snapshot (processor/, text_encoder/):
    hidden state after decoder layer 50, the prompt verbatim, no special tokens."""

    def __init__(self, model_root, device="cuda:0"):
        from transformers import Qwen3VLForConditionalGeneration, Qwen3VLProcessor
        self.processor = Qwen3VLProcessor.from_pretrained(model_root, subfolder="processor")
        self.model = Qwen3VLForConditionalGeneration.from_pretrained(
            model_root, subfolder="text_encoder", dtype=torch.bfloat16).to(device)
        self.model.eval().requires_grad_(False)
        self.device = device
        tok = self.processor.tokenizer
        self.vision_start = tok.convert_tokens_to_ids("<|vision_start|>")
        self.image_pad = tok.convert_tokens_to_ids("<|image_pad|>")
        self.vision_end = tok.convert_tokens_to_ids("<|vision_end|>")
        self._vision = None

    def tokenize(self, text):
        return self.processor.tokenizer(text, add_special_tokens=False)["input_ids"]

    def prepare_images(self, images):
        vision = self.processor.image_processor(images=list(images), return_tensors="pt")
        self._vision = {"pixel_values": vision["pixel_values"],
                        "image_grid_thw": vision["image_grid_thw"]}
        merge = self.processor.image_processor.merge_size ** 2
        return [int(t.prod()) // merge for t in vision["image_grid_thw"]]

    @torch.no_grad()
    def encode(self, token_ids, images=()):
        dev = self.device
        ids = torch.tensor([token_ids], dtype=torch.long, device=dev)
        mm = torch.tensor(self.processor.create_mm_token_type_ids([token_ids]), dtype=torch.long,
                          device=dev)
        kw = {}
        if images:
            kw = {k: (v.to(dev, self.model.dtype) if k.startswith("pixel_") else v.to(dev))
                  for k, v in self._vision.items()}
        out = self.model.model(input_ids=ids, attention_mask=torch.ones_like(ids),
                               mm_token_type_ids=mm, use_cache=False, output_hidden_states=True,
                               **kw)
        return out.hidden_states[TEXT_ENCODER_LAYER][0].to(torch.bfloat16).cpu()


def make_conditioner(model_root=None, device="cuda:0", seed=0):
    """The Qwen3-VL conditioner when a snapshot is given ("hub": the MiniMax-H3 snapshot,
    fetched on first use), else the stand-in."""
    if not model_root:
        return StandInConditioner(seed=seed)
    from vdn_minimax_h3_b200.paths import resolve_repo_path, upstream_snapshot
    root = upstream_snapshot("processor", "text_encoder") if model_root == "hub" else \
        resolve_repo_path(model_root)
    return Qwen3VLConditioner(root, device)


def build_presentation(cond, prompt, images=()):
    """`"<Picture i>: "` + vision block per image, then the prompt verbatim. Label and
    prompt rows are tagged TEXT, vision rows (start, pads, end) VIDEO.
    -> (token_ids, token_tags)."""
    counts = (cond.prepare_images(images) if hasattr(cond, "prepare_images") and images
              else [cond.image_tokens(im) for im in images])
    ids, tags = [], []
    for i, n in enumerate(counts):
        label = cond.tokenize(f"<Picture {i + 1}>: ")
        vision = [cond.vision_start] + [cond.image_pad] * n + [cond.vision_end]
        ids += label + vision
        tags += [TEXT_TAG] * len(label) + [VIDEO_TAG] * len(vision)
    body = cond.tokenize(prompt)
    ids += body
    tags += [TEXT_TAG] * len(body)
    return ids, tags


# ------------------------------------------------------------------------------- VAE
class KeyframeVaeStandIn:
    """Keyframe -> (1, 24, 1, H/16, W/16) fp32 latent with the MiniMax-H3 VAE's geometry:
    pixels normalised with (0.5, 0.5), 16x16 patch means through a seeded 3 -> 48 projection
    (mean and log-variance halves), one posterior sample under `seed` (42, as the
    reference's keyframe encode), rounded through fp16."""

    def __init__(self, seed=0):
        g = torch.Generator().manual_seed(seed + 7)
        self.proj = torch.randn(3 * VAE_SPATIAL * VAE_SPATIAL, 2 * LATENT_CHANNELS,
                                generator=g) / VAE_SPATIAL

    @torch.no_grad()
    def encode(self, image, seed=KEYFRAME_ENCODE_SEED):
        a = torch.from_numpy(np.asarray(image.convert("RGB"), dtype=np.float32) / 255.0)
        H, W = a.shape[0] // VAE_SPATIAL, a.shape[1] // VAE_SPATIAL
        a = (a[:H * VAE_SPATIAL, :W * VAE_SPATIAL] - PIXEL_MEAN) / PIXEL_STD
        patches = a.reshape(H, VAE_SPATIAL, W, VAE_SPATIAL, 3).permute(0, 2, 1, 3, 4)
        stats = patches.reshape(H * W, -1) @ self.proj
        mean, logvar = stats[:, :LATENT_CHANNELS], stats[:, LATENT_CHANNELS:].clamp(-30, 20)
        g = torch.Generator().manual_seed(seed)
        z = mean + torch.exp(0.5 * logvar) * torch.randn(mean.shape, generator=g)
        z = z.to(torch.float16).float()
        return z.t().reshape(1, LATENT_CHANNELS, 1, H, W)
