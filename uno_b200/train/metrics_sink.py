"""Where training metrics go.

Rank 0 appends every optimizer step's metrics to ``OUTPUT_DIR/metrics.jsonl``.
With a W&B mode other than ``disabled`` the same rows also go to a Weights &
Biases run (project, run name, mode and the run's compatibility record as its
config), the reporting the reference gets from the HF Trainer's W&B callback
(``training/train.py:87-92,273-300``).  Online mode needs credentials before
any work starts -- an API key in the environment or a netrc entry for the W&B
host -- the check of ``training/config.py:110-129``; offline mode writes the
run locally for a later ``wandb sync``.
"""

from __future__ import annotations

import json
import netrc
import os
from typing import Any

WANDB_MODES = ("online", "offline", "disabled")


def wandb_host(env=None) -> str:
    env = os.environ if env is None else env
    url = env.get("WANDB_BASE_URL", "https://api.wandb.ai")
    return url.split("://", 1)[-1].split("/", 1)[0]


def wandb_credentials_present(env=None) -> bool:
    env = os.environ if env is None else env
    if env.get("WANDB_API_KEY"):
        return True
    try:
        entry = netrc.netrc(env.get("NETRC")).authenticators(wandb_host(env))
    except (OSError, netrc.NetrcParseError):
        return False
    return bool(entry and entry[2])


def check_wandb(mode: str, env=None) -> None:
    """Fail before training when the requested W&B mode cannot work."""
    if mode not in WANDB_MODES:
        raise ValueError(f"W&B mode must be one of {WANDB_MODES}, got {mode!r}")
    if mode == "disabled":
        return
    try:
        import wandb  # noqa: F401
    except ImportError as exc:
        raise SystemExit(f"--wandb-mode {mode} needs the wandb package; install it or pass --wandb-mode disabled") \
            from exc
    if mode == "online" and not wandb_credentials_present(env):
        raise SystemExit(f"--wandb-mode online found no W&B credentials for {wandb_host(env)} "
                         "(WANDB_API_KEY or a netrc entry from `wandb login`); use offline or disabled instead")


class MetricsSink:
    """``log(metrics)`` per optimizer step on rank 0; ``close()`` once at the end."""

    def __init__(self, out_dir: str, *, rank: int = 0, wandb_mode: str = "disabled", wandb_project: str | None = None,
                 run_name: str | None = None, config: dict[str, Any] | None = None, resume: bool = False):
        self.file = open(os.path.join(out_dir, "metrics.jsonl"), "a", encoding="utf-8") if rank == 0 else None
        self.run = None
        if rank == 0 and wandb_mode != "disabled":
            import wandb

            self.run = wandb.init(project=wandb_project or "uno-training", name=run_name, mode=wandb_mode,
                                  dir=out_dir, config=config or {}, resume="allow" if resume else None)

    def log(self, metrics: dict[str, Any]) -> None:
        if self.file is not None:
            self.file.write(json.dumps(metrics) + "\n")
            self.file.flush()
        if self.run is not None:
            row = {f"train/{k}": v for k, v in metrics.items() if k != "step" and isinstance(v, (int, float))}
            self.run.log(row, step=int(metrics["step"]))

    def close(self) -> None:
        if self.file is not None:
            self.file.close()
            self.file = None
        if self.run is not None:
            self.run.finish()
            self.run = None
