"""The published model component: one flattened modeling file + config.json that point
back at an exploded checkpoint; the flattened class assembles the same model as the
package (same forward), and the flattener refuses what it cannot map."""
import json
import os
import subprocess
import sys

import pytest
import torch

from tests.test_checkpoints import _artifact
from tests.test_model_cpu import _forward_inputs
from vdn_minimax_h3_b200.checkpoints import export_checkpoint_dir
from vdn_minimax_h3_b200.export import component
from vdn_minimax_h3_b200.export.flatten import FlattenError, flatten
from vdn_minimax_h3_b200.inference.render import render_geometry
from vdn_minimax_h3_b200.models.h3 import h3_tiny_config
from vdn_minimax_h3_b200.models.hybrid_transform import set_layout


def test_component_matches_package(tmp_path):
    art, _ = _artifact()
    ckpt = export_checkpoint_dir(art, str(tmp_path / "ckpt"), dtype="keep")
    out_dir, modules = component.export_component(ckpt)
    assert out_dir == os.path.join(ckpt, "diffusers") and len(modules) > 5
    with open(os.path.join(out_dir, "config.json")) as f:
        cfg = json.load(f)
    assert cfg["_class_name"] == "VDNMiniMaxH3Transformer3DModel"
    assert cfg["auto_map"]["AutoModel"] == "modeling_vdn_h3.VDNMiniMaxH3Transformer3DModel"
    assert cfg["vdn"]["adapters"] == ["adapters/default/adapter_model.safetensors"]

    flat = component.load_component_module(out_dir)
    got = flat.VDNMiniMaxH3Transformer3DModel.from_pretrained(out_dir, random_base_seed=5)
    from vdn_minimax_h3_b200.export.modeling import VDNMiniMaxH3Transformer3DModel as Pkg
    want = Pkg.from_pretrained(out_dir, random_base_seed=5)
    sd_a, sd_b = got.state_dict(), want.state_dict()
    assert sd_a.keys() == sd_b.keys()
    assert all(torch.equal(sd_a[k], sd_b[k]) for k in sd_a)

    cfg3 = h3_tiny_config()
    geo = render_geometry(cfg3, 5, latent_h=8, latent_w=8, audio=True, num_latent_frames=5)
    geo.num_audio_latents = 4
    kw, layout = _forward_inputs(cfg3, geo, 6)
    for m in (got, want):
        m.float()
        set_layout(m.transformer, layout)
    with torch.no_grad():
        a = got(**kw)
        b = want(**kw)
    for x, y in zip(a, b):
        torch.testing.assert_close(x, y, rtol=0, atol=0)


def test_flattened_file_imports_standalone(tmp_path):
    """The merged file needs no package: import it in a fresh interpreter that cannot see
    the repository."""
    src, _ = flatten("vdn_minimax_h3_b200.export.modeling")
    path = tmp_path / "modeling_vdn_h3.py"
    path.write_text(src)
    code = ("import sys; sys.path = [p for p in sys.path if 'repo' not in p]; "
            f"sys.path.insert(0, {str(tmp_path)!r}); import modeling_vdn_h3 as m; "
            "assert 'vdn_minimax_h3_b200' not in sys.modules; "
            "print(m.VDNMiniMaxH3Transformer3DModel.__name__)")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       cwd=str(tmp_path), timeout=240)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "VDNMiniMaxH3Transformer3DModel" in r.stdout


def test_index_rewrite(tmp_path):
    base = tmp_path / "base_index.json"
    base.write_text(json.dumps({"_class_name": "Pipe", "transformer": ["diffusers", "X", {}],
                                "vae": ["diffusers", "V", {}]}))
    out = tmp_path / "index.json"
    idx = component.write_index(str(base), str(out), "org/repo", "stage-b/diffusers")
    assert idx["transformer"][2]["subfolder"] == "stage-b/diffusers"
    assert idx["transformer"][2]["type_hint"] == [None, None] and idx["vae"] == ["diffusers", "V", {}]


def test_flatten_refusals(tmp_path, monkeypatch):
    """Module-object imports, top-level imports outside the closure and conflicting
    top-level definitions are refused (a fake package stands in for this one)."""
    from vdn_minimax_h3_b200.export import flatten as fl
    root = tmp_path / "fakepkg"
    root.mkdir()
    (root / "__init__.py").write_text("")
    (root / "a.py").write_text("import fakepkg.b\n")
    (root / "b.py").write_text("X = 1\n")
    (root / "c.py").write_text("X = 2\nfrom fakepkg.b import X as Y\n")
    (root / "d.py").write_text("from fakepkg.b import X\n"
                               "def f():\n    from fakepkg.zzz import q\n    return q\n")
    monkeypatch.syspath_prepend(str(tmp_path))
    monkeypatch.setattr(fl, "PACKAGE", "fakepkg")
    with pytest.raises(FlattenError):
        fl.flatten("fakepkg.a")
    with pytest.raises(FlattenError):
        fl.flatten("fakepkg.c")
    src, mods = fl.flatten("fakepkg.d")        # nested out-of-closure import -> raise
    assert mods == ["fakepkg.b", "fakepkg.d"] and "ImportError" in src
