"""``python -m uno_b200.train.make_curriculum fixed|released --output PATH [--epochs E] [--block-size B]``.

``released`` writes the released run's schedule (``released_curriculum``:
block sizes 2, 4, 6, 8, 12, 16 over three epochs).

Writes a one-stage curriculum YAML (``fixed_curriculum``): ``E`` passes over
the recipe's corpus at block size ``B``, for ``python -m uno_b200.train
--curriculum PATH`` or ``CURRICULUM=PATH uno_b200/train/run_slurm.sh``.  An
existing file is kept when it holds the same plan and refused otherwise.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

from uno_b200.train.curriculum import (RECIPE_GLOBAL_BATCH, RECIPE_SEED, RECIPE_SEQUENCE_LENGTH,
                                       RECIPE_STEPS_PER_EPOCH, BlockCurriculumPlan, fixed_curriculum,
                                       released_curriculum, write_curriculum)


def main(argv: list[str] | None = None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("command", choices=("fixed", "released"))
    ap.add_argument("--output", required=True, type=Path)
    ap.add_argument("--epochs", help="passes over the corpus (default: 1 for fixed, 3 for released)")
    ap.add_argument("--block-size", type=int, default=8)
    ap.add_argument("--sequence-length", type=int, default=RECIPE_SEQUENCE_LENGTH)
    ap.add_argument("--global-batch-size", type=int, default=RECIPE_GLOBAL_BATCH)
    ap.add_argument("--steps-per-epoch", type=int, default=RECIPE_STEPS_PER_EPOCH)
    ap.add_argument("--seed", type=int, default=RECIPE_SEED)
    args = ap.parse_args(argv)
    if args.command == "released":
        mapping = released_curriculum(int(args.epochs or 3))
    else:
        mapping = fixed_curriculum(args.epochs or "1", block_size=args.block_size, sequence_length=args.sequence_length,
                                   global_batch_size=args.global_batch_size, steps_per_epoch=args.steps_per_epoch,
                                   seed=args.seed)
    write_curriculum(args.output, mapping)
    plan = BlockCurriculumPlan.from_mapping(mapping)
    out = {"output": str(args.output), "max_steps": plan.max_steps, "sha256": plan.sha256()}
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()
