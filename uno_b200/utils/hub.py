"""Resolve a model or adapter source to a local directory.

Behaviour of ``nano_vllm_uno/utils/hub.py:19-55``: a local directory is used
as is; anything else is treated as a Hugging Face repository id.  The local
Hugging Face cache (``models--{org}--{name}/snapshots/{commit}``, with
``refs/{revision}`` naming the commit) is searched first, so cached models
resolve without network access; only when the cache has no copy and
``local_files_only`` is false is ``huggingface_hub.snapshot_download`` asked.
"""

from __future__ import annotations

import os
from pathlib import Path
from typing import Sequence

ADAPTER_ALLOW_PATTERNS = ("adapter_config.json", "adapter_model*.safetensors", "adapter_model*.bin")


def hf_cache_root(cache_dir: str | os.PathLike[str] | None = None) -> Path:
    if cache_dir is not None:
        return Path(os.path.expanduser(os.fspath(cache_dir)))
    if os.environ.get("HF_HUB_CACHE"):
        return Path(os.environ["HF_HUB_CACHE"])
    home = os.environ.get("HF_HOME", os.path.join(os.path.expanduser("~"), ".cache", "huggingface"))
    return Path(home) / "hub"


def cached_snapshot(repo_id: str, revision: str | None = None,
                    cache_dir: str | os.PathLike[str] | None = None) -> str | None:
    """The cached snapshot directory of ``repo_id`` at ``revision``, if present."""
    repo = hf_cache_root(cache_dir) / ("models--" + repo_id.replace("/", "--"))
    if not repo.is_dir():
        return None
    rev = revision or "main"
    ref = repo / "refs" / rev
    commit = ref.read_text().strip() if ref.is_file() else rev
    snap = repo / "snapshots" / commit
    return str(snap) if snap.is_dir() else None


def resolve_hf_snapshot(source: str | os.PathLike[str], *, revision: str | None = None,
                        cache_dir: str | os.PathLike[str] | None = None, local_files_only: bool = False,
                        allow_patterns: Sequence[str] | None = None, artifact_name: str = "artifact") -> str:
    """Return a local directory for a path or Hugging Face repository id."""
    source = os.fspath(source)
    expanded = os.path.abspath(os.path.expanduser(source))
    if os.path.isdir(expanded):
        return expanded
    if os.path.exists(expanded):
        raise ValueError(f"{artifact_name} must be a directory: {expanded}")
    hit = cached_snapshot(source, revision, cache_dir)
    if hit is not None:
        return hit
    rev_text = f" at revision {revision!r}" if revision else ""
    if not local_files_only:
        try:
            from huggingface_hub import snapshot_download

            return snapshot_download(repo_id=source, revision=revision,
                                     cache_dir=os.fspath(cache_dir) if cache_dir is not None else None,
                                     allow_patterns=list(allow_patterns) if allow_patterns else None)
        except Exception as exc:
            raise ValueError(f"Could not resolve {artifact_name} {source!r}{rev_text} from a local "
                             "directory, the Hugging Face cache or the Hub.") from exc
    raise ValueError(f"Could not resolve {artifact_name} {source!r}{rev_text} from a local directory "
                     "or the local Hugging Face cache.")
