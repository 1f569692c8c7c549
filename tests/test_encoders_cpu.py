"""Prompt / keyframe cache encoders (stand-in conditioner and VAE): canvas rules, the
<Picture i> presentation and tags, the cache format that render reads back."""
import json

import numpy as np
import pytest
import torch

from vdn_minimax_h3_b200.inference import encode_keyframes, encode_prompt
from vdn_minimax_h3_b200.inference.encoders import (VIDEO_TAG, TEXT_TAG, StandInConditioner,
                                                    build_presentation, normalize_references,
                                                    put_on_canvas, resolve_canvas_size)
from vdn_minimax_h3_b200.inference.prompt_cache import conditioning_mode, load_prompt

Image = pytest.importorskip("PIL.Image")


def _png(path, w, h, seed):
    rng = np.random.default_rng(seed)
    Image.fromarray(rng.integers(0, 255, (h, w, 3), dtype=np.uint8)).save(path)
    return str(path)


def test_canvas_rules():
    assert resolve_canvas_size(16, 9) == (768, 1344)        # the H3 render canvas
    assert resolve_canvas_size(1920, 1080) == (768, 1344)
    assert resolve_canvas_size(9, 16) == (1344, 768)
    h, w = resolve_canvas_size(4, 3)
    assert h == 768 and w % 32 == 0 and h * w <= 768 * 1344
    assert resolve_canvas_size(1, 1) == (768, 768)


def test_put_on_canvas_and_references():
    a = Image.new("RGB", (1000, 600))
    b = Image.new("RGB", (500, 500))
    out, h, w = put_on_canvas([a, b])
    assert all(im.size == (w, h) for im in out)
    refs = normalize_references([Image.new("RGB", (300, 200))], 768)
    assert refs[0].size == (1152, 768)
    with pytest.raises(ValueError):
        normalize_references([Image.new("RGB", (1000, 200))])


def test_presentation_tags():
    cond = StandInConditioner(width=64)
    im = Image.new("RGB", (112, 56))
    ids, tags = build_presentation(cond, "a cat", [im])
    n_vis = cond.image_tokens(im) + 2
    label = len(cond.tokenize("<Picture 1>: "))
    assert tags[:label] == [TEXT_TAG] * label
    assert tags[label:label + n_vis] == [VIDEO_TAG] * n_vis
    assert tags[label + n_vis:] == [TEXT_TAG] * len(cond.tokenize("a cat"))
    emb = cond.encode(ids, [im])
    assert emb.shape == (len(ids), 64) and emb.dtype == torch.bfloat16


def test_encode_prompt_jsonl(tmp_path):
    rows = tmp_path / "p.jsonl"
    rows.write_text("\n".join(json.dumps({"prompt": f"prompt {i}"}) for i in range(5)))
    out = encode_prompt.main(["--jsonl", str(rows), "--rows", "1", "3", "--out_dir",
                              str(tmp_path), "--name", "x"])
    assert [p.split("/")[-1] for p in out] == ["x_1.pt", "x_3.pt"]
    emb, tags, cond = load_prompt(out[0], "cpu")
    assert emb.shape == (len("prompt 1"), 5120) and cond is None
    assert (tags == TEXT_TAG).all()


@pytest.mark.parametrize("which", [("first",), ("last",), ("first", "last"), ("ref", "ref")])
def test_encode_keyframes_modes(tmp_path, which):
    out = str(tmp_path / "kf.pt")
    if which[0] == "ref":
        argv = ["--refs", _png(tmp_path / "r1.png", 300, 200, 1), _png(tmp_path / "r2.png", 200, 300, 2),
                "--ref_size", "256"]
    else:
        argv = []
        if "first" in which:
            argv += ["--first", _png(tmp_path / "a.png", 640, 360, 3)]
        if "last" in which:
            argv += ["--last", _png(tmp_path / "b.png", 400, 400, 4)]
    encode_keyframes.main(["--prompt", "How the reference pictures align ...", "--out", out] + argv)
    data = torch.load(out, weights_only=True)
    assert conditioning_mode(data["keyframe_anchors"]) == {
        ("first",): "i2va", ("last",): "l2va", ("first", "last"): "fl2va",
        ("ref", "ref"): "ref2va"}[which]
    assert (data["text_token_tags"] == VIDEO_TAG).any()
    for lat in data["condition_latents"]:
        assert lat.dim() == 5 and lat.shape[:3] == (1, 24, 1)
    if which[0] != "ref":
        h, w = data["height"], data["width"]
        assert all(lat.shape[-2:] == (h // 16, w // 16) for lat in data["condition_latents"])
    else:
        assert data["reference_size"] == 256 and (data["height"], data["width"]) == (768, 1344)
    emb, tags, cond = load_prompt(out, "cpu")
    assert cond[0] == tuple(data["keyframe_anchors"]) and emb.shape[0] == tags.shape[0]
