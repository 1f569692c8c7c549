"""Inference plumbing on CPU: prompt cache, conditioning layouts (i2va / fl2va / ref2va),
LoRA merge semantics, decode-and-save stand-ins."""
import os

import pytest
import torch

from vdn_minimax_h3_b200.inference.lora import merge_lora_state, random_lora_state, translate_original_layout
from vdn_minimax_h3_b200.inference.prompt_cache import conditioning_mode, load_prompt, save_prompt, synthetic_prompt
from vdn_minimax_h3_b200.inference.render import build_inputs, generate_latents, render_geometry
from vdn_minimax_h3_b200.inference.vae import decode_and_save
from vdn_minimax_h3_b200.models.factory import TINY_HYBRID, build_model, make_spec
from vdn_minimax_h3_b200.models.h3 import h3_tiny_config
from vdn_minimax_h3_b200.models.hybrid_transform import set_layout


def test_prompt_cache_round_trip(tmp_path):
    p = synthetic_prompt(12, 256, anchors=("first", "last"), latent_hw=(16, 16), channels=16)
    path = save_prompt(str(tmp_path / "p.pt"), p["prompt"], p["prompt_embeds"], p["text_token_tags"],
                       p["keyframe_anchors"], p["condition_latents"])
    emb, tags, cond = load_prompt(path, "cpu")
    assert emb.dtype == torch.bfloat16 and emb.shape == (12, 256)
    assert conditioning_mode(cond[0]) == "fl2va" and len(cond[1]) == 2
    assert conditioning_mode(("ref", "ref")) == "ref2va" and conditioning_mode(()) == "t2va"


def test_keyframe_layout_and_render():
    cfg = h3_tiny_config()
    torch.manual_seed(0)
    model = build_model(make_spec(cfg, TINY_HYBRID, dtype="float32"), init="random")
    geo = render_geometry(cfg, 5, latent_h=16, latent_w=16, audio=True, num_latent_frames=4)
    geo.num_audio_latents = 3
    cond = [torch.randn(1, 16, 1, 16, 16)]
    packed, layout, idx = build_inputs(geo, 8, "cpu", conditions=(("first",), cond))
    assert packed.num_condition_rows == 64 and layout.video_start == 8 + 64 + 6
    emb = torch.randn(8, 256)
    lat, aud = generate_latents(model, emb, 5, 2, 3, "cpu", cfg, video_shift=1.0, audio_shift=1.0,
                                conditions=(("first",), cond), latent_h=16, latent_w=16,
                                audio=False, num_latent_frames=4,
                                on_layout=lambda lay: set_layout(model, lay))
    assert lat.shape == (1, 16, 4, 16, 16) and torch.isfinite(lat).all()


def test_lora_merge_reroot_and_translation():
    cfg = h3_tiny_config()
    model = build_model(make_spec(cfg, TINY_HYBRID, dtype="float32"), init="random")
    w = model.transformer_blocks[0].attn.orig.to_q.weight.detach().clone()
    state = random_lora_state(model, 4, targets=("to_q",), seed=1)
    a = state["transformer_blocks.0.attn.to_q.lora_A.default.weight"]
    b = state["transformer_blocks.0.attn.to_q.lora_B.default.weight"]
    assert merge_lora_state(model, state, scale=0.5) == cfg.num_layers
    assert torch.allclose(model.transformer_blocks[0].attn.orig.to_q.weight, w + 0.5 * (b @ a), atol=1e-5)
    orig = {"blocks.0.attn.qkv_proj.lora_A.weight": torch.ones(2, 4),
            "blocks.0.attn.qkv_proj.lora_B.weight": torch.arange(6.).view(6, 1).repeat(1, 2),
            "blocks.0.mlp.fc1.lora_B.weight": torch.cat([torch.zeros(2, 2), torch.ones(2, 2)])}
    tr = translate_original_layout(orig)
    assert torch.equal(tr["transformer_blocks.0.attn.to_k.lora_B.weight"][:, 0], torch.tensor([2., 3.]))
    assert torch.equal(tr["transformer_blocks.0.ff.net.0.proj.lora_B.weight"][:2], torch.ones(2, 2))


def test_decode_and_save(tmp_path):
    """17n+5 pixel frames at 16x the latent size, written as one mp4 whose second track is
    the 48 kHz stereo PCM soundtrack (muxed here, no external muxer)."""
    import cv2
    from vdn_minimax_h3_b200.inference.mp4mux import boxes, track_handlers
    from vdn_minimax_h3_b200.inference.vae import AudioDecoderStandIn, VideoDecoderStandIn
    lat = torch.randn(1, 24, 7, 4, 6)
    aud = torch.randn(2, 32, 5)
    dec = VideoDecoderStandIn(24, widths=(16, 16, 8, 8), chunk_frames=5)
    timings = {}
    out = decode_and_save(lat, aud, str(tmp_path / "clip.mp4"), dec, AudioDecoderStandIn(32),
                          timings=timings)
    assert not os.path.exists(str(tmp_path / "clip.partial.mp4"))
    assert timings["frames"] == 22 and timings["decode_s"] > 0
    data = open(out, "rb").read()
    assert track_handlers(data) == [b"vide", b"soun"]
    assert [k for k, _, _ in boxes(data)][-2:] == [b"mdat", b"moov"]
    cap = cv2.VideoCapture(out)
    n = 0
    while True:
        ok, frame = cap.read()
        if not ok:
            break
        assert frame.shape == (64, 96, 3)
        n += 1
    assert n == 22


def _decode_rank(rank, world, port, out_dir, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from vdn_minimax_h3_b200.inference.vae import (AudioDecoderStandIn, VideoDecoderStandIn,
                                                       decode_and_save)
        torch.manual_seed(0)
        lat = torch.randn(1, 24, 7, 4, 6)
        aud = torch.randn(2, 32, 5)
        dec = VideoDecoderStandIn(24, widths=(16, 16, 8, 8), chunk_frames=5)
        timings = {}
        out = decode_and_save(lat, aud, os.path.join(out_dir, "dist.mp4"), dec,
                              AudioDecoderStandIn(32), timings=timings)
        q.put((rank, (out, sorted(timings))))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(240)
def test_decode_and_save_split_over_ranks(tmp_path):
    """Two gloo ranks each decode and encode half of the frames; rank 0 joins the two
    encoded segments: one mp4 with every frame (each within the codec's error of the
    single-process encode) and the soundtrack; the other rank returns None."""
    import socket
    import cv2
    import torch.multiprocessing as mp
    from vdn_minimax_h3_b200.inference.mp4mux import track_handlers
    from vdn_minimax_h3_b200.inference.vae import AudioDecoderStandIn, VideoDecoderStandIn
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_decode_rank, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=200) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    assert res[1] == (None, ["decode_s", "encode_s"]), res
    out, keys = res[0]
    assert keys == ["decode_s", "encode_s", "frames", "mux_s"], res
    data = open(out, "rb").read()
    assert track_handlers(data) == [b"vide", b"soun"]
    torch.manual_seed(0)
    lat = torch.randn(1, 24, 7, 4, 6)
    aud = torch.randn(2, 32, 5)
    single = decode_and_save(lat, aud, str(tmp_path / "single.mp4"),
                             VideoDecoderStandIn(24, widths=(16, 16, 8, 8), chunk_frames=5),
                             AudioDecoderStandIn(32))

    def frames(path):
        cap, got = cv2.VideoCapture(path), []
        while True:
            ok, f = cap.read()
            if not ok:
                return got
            got.append(f.astype("float32"))

    a, b = frames(out), frames(single)
    assert len(a) == len(b) == 22
    for x, y in zip(a, b):
        assert abs(x - y).mean() < 8.0
