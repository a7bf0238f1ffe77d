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


# The released Uno Qwen3-8B checkpoint that the training recipe starts from
# (``training/constants.py``, ``training/prefetch_model.py``).
PINNED_MODEL_ID = "s-sahoo/uno-qwen3-8B"
PINNED_MODEL_REVISION = "b8a7577b3223bdcf2b3af0f2fc6e95258b3bbc29"


def main(argv: list[str] | None = None) -> dict:
    """``python -m uno_b200.utils.hub prefetch --cache-dir DIR [--model ID] [--revision REV]``:
    fetch a checkpoint once into a shared cache (a cached copy is reused) and
    print its snapshot directory, so that later jobs can run offline."""
    import argparse
    import json

    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("command", choices=("prefetch",))
    ap.add_argument("--cache-dir", required=True, type=Path)
    ap.add_argument("--model", default=PINNED_MODEL_ID)
    ap.add_argument("--revision")
    ap.add_argument("--local-files-only", action="store_true")
    args = ap.parse_args(argv)
    revision = args.revision or (PINNED_MODEL_REVISION if args.model == PINNED_MODEL_ID else None)
    args.cache_dir.mkdir(parents=True, exist_ok=True)
    path = resolve_hf_snapshot(args.model, revision=revision, cache_dir=args.cache_dir,
                               local_files_only=args.local_files_only, artifact_name="model")
    out = {"model_id": args.model, "revision": revision, "snapshot_path": path}
    print(json.dumps(out, sort_keys=True))
    return out


if __name__ == "__main__":
    main()
