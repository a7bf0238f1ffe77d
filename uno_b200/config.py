"""Engine configuration.

Keyword-compatible with the reference ``Config`` (``nano_vllm_uno/config.py:24-230``),
so ``LLM(model, **kwargs)`` calls written for the reference keep working:
limits (``max_num_batched_tokens``, ``max_num_seqs``, ``max_model_len``,
``gpu_memory_utilization``), parallelism (``tensor_parallel_size``,
``enforce_eager``), paged KV (``kvcache_block_size``), Uno options
(``gated_lora_path``, ``max_diffusion_block_size``, ``cuda_graph_block_sizes``,
``tree_verify_size``, ``tree_candidate_top_k``, ``cuda_graph_batch_sizes``) and
diagnostics (``decode_timing``, ``fail_on_preemption``).

B200-specific additions:

* ``load_format="dummy"`` random-initialises weights on the device instead of
  reading safetensors (used for synthetic benchmarks; no checkpoint needed);
* ``model`` may also be a :class:`ModelConfig` or the name of a preset
  (``"preset:qwen3-8b"``, ``"preset:uno-0.9b"``, ``"preset:tiny-qwen3"``);
* ``device="cpu"`` runs the fp32 PyTorch reference path (the oracle);
* ``attention_backend`` is accepted for compatibility.  Every value runs the
  framework's own sm_100a kernels; ``"fa4"`` keeps the reference's forced
  128-token page size.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass, field

import torch

from uno_b200.utils.hf_compat import ModelConfig, load_model_config

logger = logging.getLogger(__name__)

ATTENTION_BACKENDS = {"fa2", "fa3", "fa4", "native"}


@dataclass
class Config:
    model: str | ModelConfig
    model_revision: str | None = None
    hf_cache_dir: str | None = None
    hf_local_files_only: bool = False
    max_num_batched_tokens: int = 16384
    max_num_seqs: int = 512
    max_model_len: int = 8192
    gpu_memory_utilization: float = 0.9
    tensor_parallel_size: int = 1
    enforce_eager: bool = False
    hf_config: ModelConfig | None = None
    eos: int = -1
    pad: int = -1
    kvcache_block_size: int = 256
    num_kvcache_blocks: int = -1
    fail_on_preemption: bool = False
    attention_backend: str = "native"
    gated_lora_path: str | None = None
    gated_lora_revision: str | None = None
    max_diffusion_block_size: int = 16
    cuda_graph_block_sizes: list[int] | None = None
    tree_verify_size: int | None = None
    tree_candidate_top_k: int = 16
    cuda_graph_batch_sizes: list[int] | None = None
    torch_compile: bool = False
    decode_timing: bool = False
    # --- additions -------------------------------------------------------
    load_format: str = "auto"
    device: str = "cuda"
    seed: int = 0
    dummy_lora_rank: int = 0
    dummy_lora_alpha: float | None = None
    dtype_override: str | None = None
    distributed_init: str = "spawn"  # "spawn" (engine starts ranks) or "env" (torchrun)

    dtype: torch.dtype = field(init=False)
    model_source: str = field(init=False)
    gated_lora_source: str | None = field(init=False, default=None)

    @property
    def gated_lora(self) -> bool:
        return self.gated_lora_path is not None or self.dummy_lora_rank > 0

    def __post_init__(self) -> None:
        from uno_b200.models.presets import resolve_preset

        if isinstance(self.model, ModelConfig):
            self.hf_config = self.model
            self.model_source = f"config:{self.model.model_type}"
            self.model = self.model_source
            if self.load_format == "auto":
                self.load_format = "dummy"
        elif isinstance(self.model, str) and self.model.startswith("preset:"):
            self.hf_config = resolve_preset(self.model[len("preset:"):])
            self.model_source = self.model
            if self.load_format == "auto":
                self.load_format = "dummy"
        else:
            self.model_source = str(self.model)
            path = os.path.expanduser(str(self.model))
            if not os.path.isdir(path):
                from uno_b200.utils.hub import resolve_hf_snapshot

                try:
                    path = resolve_hf_snapshot(self.model, revision=self.model_revision, cache_dir=self.hf_cache_dir,
                                               local_files_only=self.hf_local_files_only, artifact_name="model")
                except ValueError as exc:
                    raise FileNotFoundError(f"Model path does not exist: {path}") from exc
            # Pick the latest ``checkpoint-N`` sub-directory when present
            # (reference ``config.py:91-101``).
            ckpts = [d for d in os.listdir(path) if d.startswith("checkpoint-")
                     and os.path.isdir(os.path.join(path, d))]
            if ckpts:
                path = os.path.join(path, max(ckpts, key=lambda d: int(d.split("-")[1])))
            self.model = path
            if self.hf_config is None:
                self.hf_config = load_model_config(path)
        _ = self.hf_config.family  # validates model_type

        self.attention_backend = str(self.attention_backend).strip().lower()
        if self.attention_backend not in ATTENTION_BACKENDS:
            raise ValueError(
                "attention_backend must be one of "
                f"{sorted(ATTENTION_BACKENDS)}, got {self.attention_backend!r}"
            )
        if self.attention_backend == "fa4" and self.kvcache_block_size == 256:
            self.kvcache_block_size = 128
        if self.kvcache_block_size % 64 != 0 or self.kvcache_block_size <= 0:
            raise ValueError("kvcache_block_size must be a positive multiple of 64")
        if not 1 <= self.tensor_parallel_size <= 8:
            raise ValueError("tensor_parallel_size must be in [1, 8]")
        if not 0 < self.gpu_memory_utilization <= 1:
            raise ValueError("gpu_memory_utilization must be in (0, 1]")
        self.max_diffusion_block_size = int(self.max_diffusion_block_size)
        if self.max_diffusion_block_size < 1:
            raise ValueError("max_diffusion_block_size must be >= 1")
        self.tree_candidate_top_k = int(self.tree_candidate_top_k)
        if self.tree_candidate_top_k < 1:
            raise ValueError("tree_candidate_top_k must be >= 1")
        if self.tree_verify_size is not None:
            self.tree_verify_size = int(self.tree_verify_size)
            if self.tree_verify_size < 1:
                raise ValueError("tree_verify_size must include at least the root")
            if self.tree_candidate_top_k == 1:
                # A K=1 tree is the linear verifier in tree notation
                # (reference ``config.py:124-133``).
                if self.tree_verify_size != self.max_diffusion_block_size:
                    raise ValueError(
                        "tree_candidate_top_k=1 selects the linear fast path; "
                        "tree_verify_size must equal max_diffusion_block_size"
                    )
                self.tree_verify_size = None
        self.cuda_graph_block_sizes = (
            list(range(1, self.max_diffusion_block_size + 1))
            if self.cuda_graph_block_sizes is None
            else sorted({int(s) for s in self.cuda_graph_block_sizes})
        )
        if not self.cuda_graph_block_sizes or self.cuda_graph_block_sizes[0] < 1:
            raise ValueError("cuda_graph_block_sizes must contain positive sizes")
        if self.cuda_graph_block_sizes[-1] > self.max_diffusion_block_size:
            raise ValueError(
                "cuda_graph_block_sizes cannot exceed "
                f"max_diffusion_block_size={self.max_diffusion_block_size}"
            )
        if self.cuda_graph_batch_sizes is not None:
            self.cuda_graph_batch_sizes = sorted({int(b) for b in self.cuda_graph_batch_sizes})
            if not self.cuda_graph_batch_sizes or self.cuda_graph_batch_sizes[0] < 1:
                raise ValueError("cuda_graph_batch_sizes must contain positive sizes")
            if self.cuda_graph_batch_sizes[-1] > self.max_num_seqs:
                raise ValueError(
                    f"cuda_graph_batch_sizes cannot exceed max_num_seqs={self.max_num_seqs}"
                )
        if self.torch_compile:
            # Hand-fused sm_100a kernels replace the reference's optional
            # Inductor pass; the flag is accepted so old call sites still run.
            logger.warning("torch_compile is ignored: the hot path is hand-written kernels")
            self.torch_compile = False
        if self.load_format not in {"auto", "dummy", "safetensors"}:
            raise ValueError("load_format must be 'auto', 'dummy' or 'safetensors'")
        if self.gated_lora_path is not None:
            self.gated_lora_source = self.gated_lora_path
            if not os.path.isdir(self.gated_lora_path):
                from uno_b200.utils.hub import ADAPTER_ALLOW_PATTERNS, resolve_hf_snapshot

                try:
                    self.gated_lora_path = resolve_hf_snapshot(
                        self.gated_lora_path, revision=self.gated_lora_revision, cache_dir=self.hf_cache_dir,
                        local_files_only=self.hf_local_files_only, allow_patterns=ADAPTER_ALLOW_PATTERNS,
                        artifact_name="gated LoRA adapter")
                except ValueError as exc:
                    raise FileNotFoundError(f"gated LoRA adapter not found: {self.gated_lora_path}") from exc
        if self.device not in {"cuda", "cpu"}:
            raise ValueError("device must be 'cuda' or 'cpu'")
        if self.device == "cpu" or os.environ.get("NANO_VLLM_FORCE_FLOAT32", "0") == "1":
            self.dtype = torch.float32
        else:
            name = self.dtype_override or self.hf_config.dtype_name
            dtype = getattr(torch, name, None)
            if dtype is None or dtype == torch.float32:
                dtype = torch.bfloat16  # fp32 checkpoints are served in bf16
            if dtype not in (torch.bfloat16, torch.float16):
                raise TypeError(f"Unsupported model dtype: {dtype!r}")
            if dtype == torch.float16:
                dtype = torch.bfloat16  # the sm_100a kernels are bf16
            self.dtype = dtype
        if self.max_model_len > self.hf_config.max_position_embeddings:
            self.hf_config.max_position_embeddings = self.max_model_len
        if self.max_num_batched_tokens < 1:
            raise ValueError("max_num_batched_tokens must be >= 1")
        if self.distributed_init not in {"spawn", "env"}:
            raise ValueError("distributed_init must be 'spawn' or 'env'")
