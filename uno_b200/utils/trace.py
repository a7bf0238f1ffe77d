"""Optional NVTX ranges around the engine's stages.

With ``UNO_NVTX=1`` in the environment, the prefill forward, the draft and
verify stages of every Psi-Spec cycle, the tree verification and the
sampling calls are wrapped in named NVTX ranges (``uno/prefill``,
``uno/draft``, ``uno/verify``, ``uno/tree``, ``uno/sample``), so a profiler
timeline (``ncu --nvtx --nvtx-include "uno/verify/"`` or Nsight Systems)
attributes kernels to stages.  Disabled, the ranges cost one dictionary
lookup.  The reference has per-step CUDA-event timing only
(``engine/model_runner.py:428-506``, kept here as ``Config.decode_timing``).
"""

from __future__ import annotations

import contextlib
import os

_ENABLED = os.environ.get("UNO_NVTX", "0") == "1"


@contextlib.contextmanager
def _range(name: str):
    import torch

    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx(name: str):
    """Context manager: an NVTX range ``uno/<name>`` when ``UNO_NVTX=1``, else nothing."""
    return _range("uno/" + name) if _ENABLED else contextlib.nullcontext()
