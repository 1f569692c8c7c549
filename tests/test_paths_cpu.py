"""Repository-relative weight paths and the Hub fallback (downloader injected; no network)."""
import os

import pytest

from vdn_minimax_h3_b200 import paths


def test_relative_absolute_and_legacy(tmp_path):
    assert paths.resolve_repo_path(None) is None
    assert paths.resolve_repo_path(str(tmp_path)) == str(tmp_path)
    assert paths.resolve_repo_path("ckpts/x") == os.path.join(paths.REPO_ROOT, "ckpts/x")
    calls = []

    def fake(repo, patterns):
        calls.append((repo, patterns))
        return str(tmp_path)

    got = paths.resolve_weights("ckpts/converted/stage-b-step-2000", downloader=fake)
    assert got == os.path.join(str(tmp_path), "stage-b-step-2000")
    assert calls == [(paths.HF_WEIGHTS_REPO, ["stage-b-step-2000/**"])]
    # a path outside ckpts/ never goes to the Hub
    assert paths.resolve_weights("elsewhere/w", downloader=fake) == os.path.join(paths.REPO_ROOT, "elsewhere/w")
    assert len(calls) == 1
    assert paths.upstream_snapshot("text_encoder", "processor", downloader=fake) == str(tmp_path)
    assert calls[-1] == (paths.H3_UPSTREAM_REPO, ["text_encoder/**", "processor/**"])


def test_offline_is_an_error(monkeypatch):
    monkeypatch.setenv("HF_HUB_OFFLINE", "1")
    with pytest.raises(FileNotFoundError):
        paths.resolve_weights("ckpts/definitely-not-here")
