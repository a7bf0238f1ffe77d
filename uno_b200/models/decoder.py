"""Dense decoder-only transformer shared by the Qwen3 and Llama/K2 families.

Layer structure (reference ``models/qwen3.py:19-246`` and ``models/xllm.py:26-338``):
pre-norm residual blocks ``add+RMSNorm -> QKV -> [QK-norm] -> RoPE -> paged
attention -> o_proj -> add+RMSNorm -> gate_up -> SiLU*up -> down``, a final
norm and an (optionally tied) vocab-parallel LM head.  Every op goes through
``uno_b200.ops`` so the same module runs the sm_100a kernels on GPU and the
fp32 reference on CPU.  On GPU the QKV projection, QK-norm, RoPE and the
paged K/V store are one kernel; gate_up and SiLU*up are one kernel.
"""

from __future__ import annotations

import torch
from torch import nn

from uno_b200 import ops
from uno_b200.layers.linear import MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear
from uno_b200.layers.meta import ForwardMeta, Mode
from uno_b200.layers.rotary import cos_sin_cache
from uno_b200.parallel.state import divide, tp_rank, tp_size
from uno_b200.utils.hf_compat import ModelConfig


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-6, n_groups: int = 1):
        super().__init__()
        if hidden_size % n_groups:
            raise ValueError(f"hidden_size={hidden_size} must be divisible by n_groups={n_groups}")
        self.eps = float(eps)
        self.n_groups = int(n_groups)
        self.weight = nn.Parameter(torch.ones(hidden_size), requires_grad=False)
        # the model's last norm: its rows leave the fused tensor-parallel path
        self.final = False

    def forward(self, x, residual=None):
        if residual is None:
            if self.final:
                return ops.rms_norm_first(x, self.weight, self.eps, self.n_groups, final=True)[0]
            return ops.rms_norm(x, self.weight, self.eps, self.n_groups)
        return ops.add_rms_norm(x, residual, self.weight, self.eps, self.n_groups, final=self.final)

    def first(self, x):
        """Normalise the start of the residual stream: returns (normed, residual)."""
        return ops.rms_norm_first(x, self.weight, self.eps, self.n_groups, final=self.final)


class VocabParallelEmbedding(nn.Module):
    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        self.tp_rank, self.tp_size = tp_rank(), tp_size()
        self.num_embeddings = num_embeddings
        self.per_partition = divide(num_embeddings, self.tp_size)
        self.vocab_start = self.per_partition * self.tp_rank
        self.weight = nn.Parameter(torch.empty(self.per_partition, embedding_dim), requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param, loaded, *args):
        param.data.copy_(loaded.narrow(0, self.tp_rank * self.per_partition, self.per_partition))

    def forward(self, ids):
        return ops.embedding(ids, self.weight, self.vocab_start)


class ParallelLMHead(VocabParallelEmbedding):
    """Vocab-parallel output projection; returns this rank's logit shard."""

    def forward(self, x):
        return ops.lm_head(x, self.weight)


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        tp = tp_size()
        self.total_heads = cfg.num_attention_heads
        self.total_kv_heads = cfg.num_key_value_heads
        self.num_heads = divide(cfg.num_attention_heads, tp)
        self.num_kv_heads = divide(cfg.num_key_value_heads, tp)
        self.head_dim = cfg.head_dim
        self.scale = self.head_dim ** -0.5
        self.eps = cfg.rms_norm_eps
        self.qkv_proj = QKVParallelLinear(cfg.hidden_size, self.head_dim, self.total_heads,
                                          self.total_kv_heads, bias=cfg.attention_bias)
        self.o_proj = RowParallelLinear(self.total_heads * self.head_dim, cfg.hidden_size, bias=False)
        self.qk_norm = bool(cfg.query_key_norm)
        if self.qk_norm:
            self.q_norm = RMSNorm(self.head_dim, cfg.rms_norm_eps)
            self.k_norm = RMSNorm(self.head_dim, cfg.rms_norm_eps)
        # Per-layer views into the engine-owned paged cache.
        self.k_cache = torch.empty(0)
        self.v_cache = torch.empty(0)

    def forward(self, x, meta: ForwardMeta, cos_sin):
        q = ops.qkv_rope_store(
            x, self.qkv_proj, meta.lora_mask, meta.positions, cos_sin,
            self.q_norm.weight if self.qk_norm else None,
            self.k_norm.weight if self.qk_norm else None,
            self.eps, self.num_heads, self.num_kv_heads, self.head_dim,
            self.k_cache, self.v_cache, meta.slot_mapping,
        )
        o = ops.attention(q, self.k_cache, self.v_cache, meta, self.scale)
        return ops.linear(o, self.o_proj, meta.lora_mask)


class MLP(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        if cfg.hidden_act != "silu":
            raise ValueError(f"Unsupported activation: {cfg.hidden_act}. Only silu is supported.")
        self.gate_up_proj = MergedColumnParallelLinear(cfg.hidden_size, [cfg.intermediate_size] * 2)
        self.down_proj = RowParallelLinear(cfg.intermediate_size, cfg.hidden_size)

    def forward(self, x, meta: ForwardMeta):
        act = ops.gate_up_silu(x, self.gate_up_proj, meta.lora_mask)
        return ops.linear(act, self.down_proj, meta.lora_mask)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        if getattr(cfg, "num_experts", 0):
            raise NotImplementedError("only dense checkpoints are supported")
        if cfg.extra.get("attention_gate_func") is not None:
            raise NotImplementedError("attention gating is not supported")
        if cfg.extra.get("use_sliding_window", False):
            raise NotImplementedError("sliding-window attention is not supported")
        groups = int(cfg.layernorm_num_groups or 1)
        self.self_attn = Attention(cfg)
        self.mlp = MLP(cfg)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, groups)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, groups)

    def forward(self, x, residual, meta, cos_sin):
        if residual is None:
            x, residual = self.input_layernorm.first(x)
        else:
            x, residual = self.input_layernorm(x, residual)
        x = self.self_attn(x, meta, cos_sin)
        x, residual = self.post_attention_layernorm(x, residual)
        return self.mlp(x, meta), residual


class DecoderModel(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.embed_tokens = VocabParallelEmbedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(cfg) for _ in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, int(cfg.layernorm_num_groups or 1))
        self.norm.final = True

    def forward(self, input_ids, meta, cos_sin):
        x = self.embed_tokens(input_ids)
        residual = None
        for layer in self.layers:
            x, residual = layer(x, residual, meta, cos_sin)
        x, _ = self.norm(x, residual)
        return x


class DecoderForCausalLM(nn.Module):
    packed_modules_mapping = {
        "q_proj": ("qkv_proj", "q"),
        "k_proj": ("qkv_proj", "k"),
        "v_proj": ("qkv_proj", "v"),
        "gate_proj": ("gate_up_proj", 0),
        "up_proj": ("gate_up_proj", 1),
    }

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.config = cfg
        self.model = DecoderModel(cfg)
        self.lm_head = ParallelLMHead(cfg.vocab_size, cfg.hidden_size)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        self.register_buffer(
            "cos_sin_cache",
            cos_sin_cache(cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta, cfg.rope_scaling,
                          device=self.lm_head.weight.device),
            persistent=False,
        )

    @property
    def attention_layers(self) -> list[Attention]:
        return [layer.self_attn for layer in self.model.layers]

    def forward(self, input_ids, meta: ForwardMeta):
        return self.model(input_ids, meta, self.cos_sin_cache)

    def compute_logits(self, hidden, meta: ForwardMeta | None = None):
        if meta is not None and meta.mode is Mode.PREFILL and meta.logits_indices is not None:
            hidden = hidden.index_select(0, meta.logits_indices)
        return self.lm_head(hidden)


class Qwen3ForCausalLM(DecoderForCausalLM):
    """Qwen3 / SDAR checkpoints (QK-norm when ``attention_bias`` is false)."""


class XllmForCausalLM(DecoderForCausalLM):
    """Llama-style XLLM / K2 checkpoints (grouped RMSNorm, optional QK-norm, YaRN)."""


def build_model(cfg: ModelConfig) -> DecoderForCausalLM:
    if cfg.family == "qwen3":
        return Qwen3ForCausalLM(cfg)
    return XllmForCausalLM(cfg)
