"""LoRA-only, single-forward Uno trainer.

Training step of ``training/trainer.py:174-308`` on this framework's own
decoder:

1. the curriculum picks the block size for the optimizer step;
2. each micro-batch is laid out as paired noisy/clean copies
   (:mod:`uno_b200.train.layout`) and run through ONE transformer forward
   with the gated LoRA active on the noisy copy only;
3. student = noisy states, teacher = clean states (frozen base, detached);
   loss = ``ce_weight*CE + kl_weight*KL + tv_weight*TV`` per supervised token
   (:func:`uno_b200.train.losses.fused_head_loss`);
4. LoRA gradients are averaged over data-parallel ranks, clipped to
   ``max_grad_norm`` and applied with AdamW -- linear warmup from zero, then
   the constant learning rate of the released recipe (a warmup-stable schedule
   without decay steps), or a cosine decay (``lr_schedule="cosine"``) -- ZeRO-2 style (each rank keeps the moments of one shard), on
   CUDA as one fused reduce-scatter + clip + AdamW + all-gather kernel
   (:class:`uno_b200.train.optim.ShardedLoraAdamW`).

Checkpoints are written only at curriculum stage boundaries
(``checkpoint-{step}/`` with the PEFT adapter, optimizer and RNG state and
``uno_curriculum_state.json``); a resume must come from such a boundary with
the same curriculum hash (``training/trainer.py:104-146``).
"""

from __future__ import annotations

import json
import math
import time
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from uno_b200.train.config import IGNORE_INDEX, UnoObjectiveConfig, write_json_atomic
from uno_b200.train.curriculum import BlockCurriculumPlan
from uno_b200.train.forward import uno_hidden_states
from uno_b200.train.layout import build_uno_batch, shift_labels_for_next_token
from uno_b200.train.lora import TrainableLoRA
from uno_b200.train.losses import fused_head_loss
from uno_b200.train.optim import ShardedLoraAdamW


def lr_at(step: int, base_lr: float, warmup: int, total: int, schedule: str = "constant") -> float:
    """Learning rate of optimizer step ``step`` (0-based).

    ``constant``: ``base * step / warmup`` during the warmup, then ``base``
    (``training/train.py:282-284``: warmup-stable-decay with no decay steps).
    ``cosine``: the same warmup, then a half cosine from ``base`` to 0 at ``total``.
    """
    if warmup > 0 and step < warmup:
        return base_lr * step / warmup
    if schedule == "constant":
        return base_lr
    if schedule != "cosine":
        raise ValueError(f"unknown learning-rate schedule {schedule!r}")
    span = max(1, total - warmup)
    frac = min(1.0, max(0.0, (step - warmup) / span))
    return base_lr * 0.5 * (1.0 + math.cos(math.pi * frac))


class UnoTrainer:
    def __init__(self, model, lora: TrainableLoRA, *, objective: UnoObjectiveConfig,
                 curriculum: BlockCurriculumPlan, mask_token_id: int, lr: float = 1e-4, warmup_steps: int = 0,
                 weight_decay: float = 0.0, max_grad_norm: float = 1.0, output_dir: str | None = None,
                 checkpoint_layers: bool = False, seed: int = 0, process_group=None,
                 base_model_name: str | None = None, loss_chunk: int = 1024, native_gemms: bool = True,
                 fsdp: bool = False, lr_schedule: str = "constant"):
        objective.validate()
        self.model = model
        self.lora = lora
        self.objective = objective
        self.curriculum = curriculum
        self.mask_token_id = int(mask_token_id)
        self.base_lr = float(lr)
        self.warmup = int(warmup_steps)
        if lr_schedule not in ("constant", "cosine"):
            raise ValueError(f"unknown learning-rate schedule {lr_schedule!r}")
        self.lr_schedule = lr_schedule
        self.max_grad_norm = float(max_grad_norm)
        self.output_dir = Path(output_dir) if output_dir else None
        self.checkpoint_layers = bool(checkpoint_layers)
        self.group = process_group
        self.base_model_name = base_model_name
        self.loss_chunk = int(loss_chunk)
        for p in model.parameters():
            p.requires_grad_(False)
        self.device = next(lora.parameters()).device
        self.optimizer = ShardedLoraAdamW(list(lora.parameters()), lr=self.base_lr, betas=(0.9, 0.999), eps=1e-8,
                                          weight_decay=weight_decay, max_grad_norm=self.max_grad_norm,
                                          group=process_group)
        # CUDA: projections (forward and backward) on the tcgen05 GEMMs
        # (with fsdp the frozen projection weights are row-sharded over the ranks and
        # the GEMMs read the peers' rows over NVLink)
        self.native = None
        self.sharded = None
        if self.device.type == "cuda" and native_gemms:
            from uno_b200.train.native import build_projections

            self.native, self.sharded = build_projections(model, lora, group=process_group, fsdp=fsdp)
        self.step = 0
        rank = dist.get_rank(process_group) if (process_group is not None and dist.is_initialized()) else 0
        self.generator = torch.Generator(device=self.device).manual_seed(int(seed) * 1000003 + rank)
        self.last_metrics: dict[str, Any] = {}

    # ---------------------------------------------------------------- step
    def _micro_loss(self, batch: dict[str, torch.Tensor], block_size: int) -> tuple[torch.Tensor, dict]:
        ids = batch["input_ids"].to(self.device)
        labels = batch["labels"].to(self.device)
        positions = batch.get("position_ids")
        positions = (torch.arange(ids.shape[1], device=self.device).expand_as(ids) if positions is None
                     else positions.to(self.device))
        ub = build_uno_batch(ids, labels, positions, block_size=block_size, mask_token_id=self.mask_token_id,
                             generator=self.generator)
        if self.native is not None:
            for proj in self.native:
                for p in proj.values():
                    p.refresh(self.optimizer.step_count)
        vis = ub.attention_mask()
        meta = None
        if self.native is not None:
            from uno_b200.train.attention import AttentionMeta

            meta = AttentionMeta(ub.segment, ub.positions, ub.noisy, ub.block_size, vis=vis)
        hidden = uno_hidden_states(self.model, self.lora, ub.ids, ub.positions, vis, ub.noisy,
                                   self.checkpoint_layers, native=self.native, attn_meta=meta)
        noisy_h, clean_h = ub.gather_regions(hidden)
        H = noisy_h.shape[-1]
        supervised = labels != IGNORE_INDEX
        shifted = shift_labels_for_next_token(labels, positions)
        ce_mask = ub.noised & (shifted != IGNORE_INDEX)
        p_full = torch.ones_like(labels, dtype=torch.float32)
        p_full[ub.noised] = ub.p_mask
        ce_scale = torch.where(ce_mask, 1.0 / p_full, torch.zeros_like(p_full))
        ob = self.objective
        dist_active = ob.kl_weight > 0 or ob.tv_weight > 0
        tokens = int(supervised.sum().item())
        loss = fused_head_loss(
            noisy_h.reshape(-1, H), clean_h.reshape(-1, H), self.model.lm_head.weight,
            dist_mask=(supervised if dist_active else torch.zeros_like(supervised)).reshape(-1),
            ce_mask=(ce_mask if ob.ce_weight > 0 else torch.zeros_like(ce_mask)).reshape(-1),
            ce_target=shifted.reshape(-1), ce_scale=ce_scale.reshape(-1), tv_weight=ob.tv_weight,
            kl_weight=ob.kl_weight, ce_weight=ob.ce_weight, teacher_ce=ob.internal_ce_target == "clean_argmax",
            normalizer=tokens, chunk=self.loss_chunk)
        return loss, {"tokens": tokens, "noised": int(ub.noised.sum().item())}

    def train_step(self, micro_batches: list[dict[str, torch.Tensor]]) -> dict[str, Any]:
        if self.step >= self.curriculum.max_steps:
            raise RuntimeError("training already reached the curriculum's last step")
        t0 = time.perf_counter()
        block = self.curriculum.stage_for_step(self.step).block_size
        self.optimizer.zero_grad()
        total, tokens, noised = 0.0, 0, 0
        for mb in micro_batches:
            loss, info = self._micro_loss(mb, block)
            (loss / len(micro_batches)).backward()
            total += float(loss.detach()) / len(micro_batches)
            tokens += info["tokens"]
            noised += info["noised"]
        lr = lr_at(self.step, self.base_lr, self.warmup, self.curriculum.max_steps, self.lr_schedule)
        self.optimizer.set_lr(lr)
        on_gpu = self.device.type == "cuda"
        if on_gpu:  # the optimizer step holds the exposed communication: gradient reduce-scatter + all-gather
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        grad_norm = self.optimizer.step()  # DP gradient average, clip, AdamW, parameter all-gather
        if on_gpu:
            ev1.record()
        self.step += 1
        metrics = {"step": self.step, "loss": total, "block_size": block, "lr": lr, "grad_norm": grad_norm,
                   "tokens": tokens, "noised_tokens": noised, "seconds": time.perf_counter() - t0,
                   "transformer_forwards": len(micro_batches)}
        if on_gpu:
            ev1.synchronize()
            metrics["optimizer_comm_ms"] = ev0.elapsed_time(ev1)
        self.last_metrics = metrics
        reason = self.curriculum.checkpoint_reasons.get(self.step)
        if reason and self.output_dir is not None:
            self.save_checkpoint(reason)
        return metrics

    def _is_main(self) -> bool:
        return not (self.group is not None and dist.is_initialized() and dist.get_rank(self.group) != 0)

    # ---------------------------------------------------------- checkpoints
    def _rank(self) -> int:
        return dist.get_rank(self.group) if (self.group is not None and dist.is_initialized()) else 0

    def save_checkpoint(self, reason: str) -> Path:
        """Every rank writes its optimizer shard and RNG state; rank 0 the adapter and the boundary record."""
        ckpt = self.output_dir / f"checkpoint-{self.step}"
        ckpt.mkdir(parents=True, exist_ok=True)
        torch.save({"optimizer": self.optimizer.state_dict(), "generator": self.generator.get_state(),
                    "step": self.step}, ckpt / f"trainer_state_rank{self._rank()}.pt")
        if self._is_main():
            self.lora.save(str(ckpt), self.base_model_name)
            write_json_atomic(ckpt / "uno_curriculum_state.json",
                              {"version": 1, "global_step": self.step, "reason": reason,
                               "curriculum_sha256": self.curriculum.sha256()})
        return ckpt

    def resume(self, checkpoint: str | Path) -> None:
        ckpt = Path(checkpoint)
        state_path = ckpt / "uno_curriculum_state.json"
        if not state_path.is_file():
            raise FileNotFoundError("Uno resumes are supported only from curriculum-boundary checkpoints; "
                                    f"missing {state_path}.")
        state = json.loads(state_path.read_text())
        if state.get("curriculum_sha256") != self.curriculum.sha256():
            raise ValueError("Checkpoint curriculum does not match the current curriculum.")
        step = state.get("global_step")
        if step not in self.curriculum.checkpoint_reasons:
            raise ValueError(f"Checkpoint step {step} is not a curriculum boundary.")
        self.lora.load(str(ckpt))
        blob = torch.load(ckpt / f"trainer_state_rank{self._rank()}.pt", map_location=self.device,
                          weights_only=False)
        self.optimizer.load_state_dict(blob["optimizer"])
        self.generator.set_state(blob["generator"].cpu() if hasattr(blob["generator"], "cpu") else blob["generator"])
        self.step = int(blob["step"])
