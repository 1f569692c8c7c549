"""Repository-relative weight paths with a Hub fallback.

Reference parity: src/paths.py:1-56. A ModelSpec's `base.source`, a config's checkpoint /
base / VAE source and the render defaults are written relative to the repository root
(`ckpts/<name>`), so artifacts carry no machine-specific path. A `ckpts/<name>` directory
that is missing locally is fetched from the weights repository on the Hub (only that
subfolder) and used from the cache; `ckpts/converted/<name>` (the training repository's
spelling) names the same directory; absolute paths pass through. Offline (no
huggingface_hub, or HF_HUB_OFFLINE set) a missing directory is an error that says so.
"""
import os

REPO_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

HF_WEIGHTS_REPO = "OpenVDN/vdn-minimax-h3"     # h3-base/, stage-b-step-2000/, stage-dmd-step-250/
WEIGHTS_PREFIX = "ckpts/"
LEGACY_WEIGHTS_PREFIX = "ckpts/converted/"
H3_BASE = WEIGHTS_PREFIX + "h3-base"
H3_UPSTREAM_REPO = "MiniMaxAI/MiniMax-H3"       # text_encoder/, processor/ (prompt encoding)


def resolve_repo_path(path):
    """Absolute path: unchanged if absolute or None, else joined to the repository root."""
    if path is None or os.path.isabs(path):
        return path
    return os.path.join(REPO_ROOT, path)


def _snapshot(repo, patterns, downloader=None):
    if downloader is not None:
        return downloader(repo, patterns)
    if os.environ.get("HF_HUB_OFFLINE"):
        raise FileNotFoundError(f"{repo} {patterns}: not present locally and HF_HUB_OFFLINE is set")
    try:
        from huggingface_hub import snapshot_download
    except ImportError as exc:   # pragma: no cover - depends on the environment
        raise FileNotFoundError(f"{repo} {patterns}: not present locally and huggingface_hub "
                                "is not installed") from exc
    return snapshot_download(repo, allow_patterns=list(patterns))


def resolve_weights(path, downloader=None):
    """`resolve_repo_path` plus the Hub fallback for a missing `ckpts/<name>`.
    `downloader(repo, patterns) -> local root` replaces the Hub call (tests, mirrors)."""
    if path is not None and path.startswith(LEGACY_WEIGHTS_PREFIX):
        path = WEIGHTS_PREFIX + path[len(LEGACY_WEIGHTS_PREFIX):]
    local = resolve_repo_path(path)
    if local is None or os.path.exists(local):
        return local
    if path.startswith(WEIGHTS_PREFIX):
        name = path[len(WEIGHTS_PREFIX):].strip("/")
        root = _snapshot(HF_WEIGHTS_REPO, [f"{name}/**"], downloader)
        return os.path.join(root, name)
    return local


def upstream_snapshot(*subfolders, downloader=None):
    """The MiniMax-H3 snapshot restricted to `subfolders` (fetched on first use)."""
    return _snapshot(H3_UPSTREAM_REPO, [f"{s}/**" for s in subfolders], downloader)
