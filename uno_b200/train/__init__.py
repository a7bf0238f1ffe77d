"""Conditional-LoRA diffusion training (block-diffusion layout, TV/KL/CE
objective, block-size curriculum, boundary checkpoints)."""

from uno_b200.train.config import IGNORE_INDEX, LoraSettings, UnoObjectiveConfig
from uno_b200.train.curriculum import BlockCurriculumPlan, CurriculumStage
from uno_b200.train.layout import UnoBatch, build_uno_batch, shift_labels_for_next_token
from uno_b200.train.lora import TrainableLoRA
from uno_b200.train.trainer import UnoTrainer

__all__ = ["IGNORE_INDEX", "LoraSettings", "UnoObjectiveConfig", "BlockCurriculumPlan", "CurriculumStage",
           "UnoBatch", "build_uno_batch", "shift_labels_for_next_token", "TrainableLoRA", "UnoTrainer"]
