"""Tensor-parallel linear layers with gated (row-masked) LoRA slices.

Sharding follows the Megatron rules of the reference
(``nano_vllm_uno/layers/linear.py:70-499``) so HF checkpoints load identically:

* ``ColumnParallelLinear`` splits the output dimension; ``QKVParallelLinear``
  splits q/k/v by heads; ``MergedColumnParallelLinear`` splits gate and up
  separately; ``RowParallelLinear`` splits the input dimension and sums the
  partial products across ranks.
* A LoRA slice ``(A [r, K], B [n, r], scale, out_start)`` adds
  ``scale * (mask * (x A^T)) B^T`` to output columns ``[out_start, out_start+n)``
  for rows whose gate mask is 1 (noisy draft rows).  Column-parallel layers
  shard ``B`` by rows; row-parallel layers shard ``A`` by columns and reduce
  the rank-``r`` hidden across ranks (``nano_vllm_uno/utils/lora.py:103-118``).

For the sm_100a path, :meth:`LinearBase.pack_lora` concatenates every slice's
``A`` into ``lora_a_cat [R, K]`` (R padded to a multiple of 64) and scatters the
``B`` matrices into a block-structured ``lora_b_cat [N, R]`` so one extra GEMM
column block produces all hidden activations and one small GEMM applies all
``B`` projections.
"""

from __future__ import annotations

import torch
from torch import nn

from uno_b200.parallel.state import divide, tp_rank, tp_size


class LoRASlice:
    __slots__ = ("A", "B", "scaling", "out_start", "out_end")

    def __init__(self, A: torch.Tensor, B: torch.Tensor, scaling: float, out_start: int):
        self.A = A.contiguous()
        self.B = B.contiguous()
        self.scaling = float(scaling)
        self.out_start = int(out_start)
        self.out_end = int(out_start + B.shape[0])


class LinearBase(nn.Module):
    # tp_dim: 0 = output split (column parallel), 1 = input split (row parallel)
    tp_dim: int | None = None

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        super().__init__()
        self.tp_rank = tp_rank()
        self.tp_size = tp_size()
        self.input_size = input_size
        self.output_size = output_size
        self.weight = nn.Parameter(torch.empty(output_size, input_size), requires_grad=False)
        self.weight.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.empty(output_size), requires_grad=False)
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)
        self.lora_slices: list[LoRASlice] = []
        self.lora_a_cat: torch.Tensor | None = None
        self.lora_b_cat: torch.Tensor | None = None
        self.lora_rank_total = 0
        self.lora_scaling = 0.0
        # Optional sm_100a-specific packed weight (set by ``prepare_device_weights``).
        self.device_weight: torch.Tensor | None = None

    def weight_loader(self, param: nn.Parameter, loaded: torch.Tensor, *args) -> None:
        param.data.copy_(loaded)

    @property
    def has_lora(self) -> bool:
        return bool(self.lora_slices)

    def add_lora_slice(self, A: torch.Tensor, B: torch.Tensor, scaling: float, output_start: int = 0) -> None:
        dev, dt = self.weight.device, self.weight.dtype
        self.lora_slices.append(LoRASlice(A.to(dev, dt), B.to(dev, dt), scaling, output_start))
        self.lora_a_cat = None

    def pack_lora(self, align: int = 64) -> None:
        """Build ``lora_a_cat``/``lora_b_cat`` for the fused device path."""
        if not self.lora_slices:
            return
        scales = {s.scaling for s in self.lora_slices}
        if len(scales) != 1:
            raise ValueError("all LoRA slices of one layer must share a scaling")
        total = sum(s.A.shape[0] for s in self.lora_slices)
        padded = -(-total // align) * align
        K = self.lora_slices[0].A.shape[1]
        dev, dt = self.weight.device, self.weight.dtype
        a_cat = torch.zeros(padded, K, device=dev, dtype=dt)
        b_cat = torch.zeros(self.output_size, padded, device=dev, dtype=dt)
        off = 0
        for s in sorted(self.lora_slices, key=lambda s: s.out_start):
            r = s.A.shape[0]
            a_cat[off:off + r] = s.A
            b_cat[s.out_start:s.out_end, off:off + r] = s.B
            off += r
        self.lora_a_cat = a_cat.contiguous()
        self.lora_b_cat = b_cat.contiguous()
        self.lora_rank_total = padded
        self.lora_scaling = scales.pop()


class ReplicatedLinear(LinearBase):
    pass


class ColumnParallelLinear(LinearBase):
    tp_dim = 0

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        super().__init__(input_size, divide(output_size, tp_size()), bias)

    def weight_loader(self, param, loaded, *args):
        shard = param.data.shape[0]
        param.data.copy_(loaded.narrow(0, self.tp_rank * shard, shard))


class MergedColumnParallelLinear(ColumnParallelLinear):
    def __init__(self, input_size: int, output_sizes: list[int], bias: bool = False):
        self.output_sizes = list(output_sizes)
        super().__init__(input_size, sum(output_sizes), bias)

    def shard_offset(self, shard_id: int) -> int:
        return sum(self.output_sizes[:shard_id]) // self.tp_size

    def weight_loader(self, param, loaded, shard_id: int = 0):
        offset = self.shard_offset(shard_id)
        size = self.output_sizes[shard_id] // self.tp_size
        dst = param.data.narrow(0, offset, size)
        dst.copy_(loaded.chunk(self.tp_size, 0)[self.tp_rank])


class QKVParallelLinear(ColumnParallelLinear):
    def __init__(self, hidden_size: int, head_size: int, total_num_heads: int,
                 total_num_kv_heads: int | None = None, bias: bool = False):
        total_num_kv_heads = total_num_kv_heads or total_num_heads
        tp = tp_size()
        self.head_size = head_size
        self.num_heads = divide(total_num_heads, tp)
        self.num_kv_heads = divide(total_num_kv_heads, tp)
        out = (total_num_heads + 2 * total_num_kv_heads) * head_size
        super().__init__(hidden_size, out, bias)

    def shard_offset(self, shard_id: str) -> int:
        return {
            "q": 0,
            "k": self.num_heads * self.head_size,
            "v": (self.num_heads + self.num_kv_heads) * self.head_size,
        }[shard_id]

    def weight_loader(self, param, loaded, shard_id: str = "q"):
        size = (self.num_heads if shard_id == "q" else self.num_kv_heads) * self.head_size
        dst = param.data.narrow(0, self.shard_offset(shard_id), size)
        dst.copy_(loaded.chunk(self.tp_size, 0)[self.tp_rank])


class RowParallelLinear(LinearBase):
    tp_dim = 1

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        super().__init__(divide(input_size, tp_size()), output_size, bias)

    def weight_loader(self, param, loaded, *args):
        if param.data.dim() == 1:  # bias is replicated; only rank 0 adds it
            param.data.copy_(loaded)
            return
        shard = param.data.shape[1]
        param.data.copy_(loaded.narrow(1, self.tp_rank * shard, shard))
