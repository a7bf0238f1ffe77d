"""Per-rank model execution: weights, paged KV cache, staging, forwards, graphs.

Responsibilities of the reference ``ModelRunner`` (``nano_vllm_uno/engine/model_runner.py:52-946``):
build the model, load base weights and the gated-LoRA adapter, size and
allocate the paged KV cache, stage prefill / block / tree forwards, compact
accepted tree K/V and capture decode CUDA graphs.  Rank 0 drives; other TP
ranks execute the same calls (the engine forwards each call over a gloo
control-plane group).  Every rank computes identical sampling decisions from
identical (all-gathered) logits with the same counter-keyed RNG, so no decision
broadcast is needed.

KV cache layout: one tensor ``[layers, 2, pages, kv_heads, page, head_dim]``;
a (page, head) tile is contiguous, which is what the attention kernels stream.
"""

from __future__ import annotations

import logging
import os
import time

import numpy as np
import torch

from uno_b200.engine.decoder import TwoPassDecoder
from uno_b200.engine.draft_tree import tree_kv_moves
from uno_b200.engine.sampling import Sampler, VocabShard
from uno_b200.engine.sequence import Sequence
from uno_b200.engine.workspace import DecodeWorkspace, slots_for
from uno_b200.layers.meta import ForwardMeta, Mode, ancestor_masks, causal_suffix_masks
from uno_b200.models.decoder import build_model
from uno_b200.parallel import state as tp
from uno_b200.sampling_params import SamplingParams
from uno_b200.utils.loader import dummy_init, load_model
from uno_b200.utils.lora import dummy_lora, load_lora_adapter
from uno_b200.utils.trace import nvtx

logger = logging.getLogger(__name__)


def sglang_batch_ladder(max_bs: int) -> list[int]:
    """Capture ladder 1-8, 10-32 step 2, 40-64 step 4, 72-256 step 8, then 16."""
    sizes = list(range(1, 9)) + list(range(10, 33, 2)) + list(range(40, 65, 4)) + list(range(72, 257, 8))
    sizes += list(range(272, max(272, max_bs) + 16, 16))
    out = sorted({s for s in sizes if s <= max_bs})
    if not out or out[-1] != max_bs:
        out.append(max_bs)
    return out


class ModelRunner:
    def __init__(self, config, rank: int = 0, control=None):
        self.config = config
        self.rank = rank
        self.control = control
        self.tp_comm = None
        self.world_size = config.tensor_parallel_size
        self.page = config.kvcache_block_size
        cfg = config.hf_config
        self.device = torch.device(config.device if config.device == "cpu" else f"cuda:{torch.cuda.current_device()}")
        self.dtype = config.dtype
        self.cuda_graph_hits = 0
        self.cuda_graph_misses = 0
        self.cuda_graph_memory: dict[str, int] = {}
        self._timing_events: list[dict] = []
        self._timing_step = 0
        self.graphs: dict[tuple, object] = {}

        prev_dtype = torch.get_default_dtype()
        torch.set_default_dtype(self.dtype)
        try:
            with torch.device(self.device):
                self.model = build_model(cfg)
        finally:
            torch.set_default_dtype(prev_dtype)
        self.model.eval()
        t0 = time.perf_counter()
        if config.load_format == "dummy":
            dummy_init(self.model, seed=config.seed)
        else:
            load_model(self.model, config.model)
        if config.gated_lora_path is not None:
            load_lora_adapter(self.model, config.gated_lora_path)
        elif config.dummy_lora_rank > 0:
            dummy_lora(self.model, config.dummy_lora_rank, config.dummy_lora_alpha, seed=config.seed + 1)
        logger.info("weights ready in %.1fs", time.perf_counter() - t0)
        if self.device.type == "cuda":
            from uno_b200.ops import cuda as cuda_ops

            cuda_ops.prepare_model(self.model)
            if self.world_size > 1 and os.environ.get("UNO_TP_COMM", "fused") != "nccl":
                # Row-parallel outputs travel over NVLink peer memory with the
                # reduction fused into residual-add + RMSNorm (no NCCL all-reduce).
                from uno_b200.parallel.symm import FusedTPComm

                max_q = max(config.max_diffusion_block_size, config.tree_verify_size or 0)
                max_tokens = max(config.max_num_batched_tokens, config.max_num_seqs * max_q)
                self.tp_comm = FusedTPComm(rank, self.world_size, control.group if control is not None else None,
                                           max_tokens, cfg.hidden_size, self.device,
                                           max_logit_rows=config.max_num_seqs * max(max_q, 1))
                cuda_ops.set_tp_comm(self.tp_comm)

        shard = None
        head = self.model.lm_head
        if (self.tp_comm is not None and os.environ.get("UNO_VOCAB_PARALLEL", "1") != "0"
                and head.per_partition % 8 == 0 and head.vocab_start % 8 == 0):
            # logits stay vocab-sharded: sampling and verify exchange per-row partials over NVLink
            shard = VocabShard(head.vocab_start, cfg.vocab_size, tp.all_gather_last_dim)
        self.vocab_parallel = shard is not None
        self.sampler = Sampler(config.seed, shard)
        self.allocate_kv_cache()
        max_q = max(config.max_diffusion_block_size, config.tree_verify_size or 0)
        max_pages = -(-(config.max_model_len + max_q) // self.page) + 1
        self.workspace = DecodeWorkspace(config.max_num_seqs, max_q, max_pages, self.device, self.page)
        self.decoder = TwoPassDecoder(
            run_block=self.run_block,
            eos_token_id=config.eos,
            pad_token_id=config.pad,
            vocab_size=cfg.vocab_size,
            device=self.device,
            sampler=self.sampler,
            gated_lora=config.gated_lora,
            run_tree=self.run_tree if config.tree_verify_size is not None else None,
            compact_tree_kv=self.compact_tree_kv if config.tree_verify_size is not None else None,
            tree_verify_size=config.tree_verify_size,
            tree_candidate_top_k=config.tree_candidate_top_k,
            noise_seed=config.seed + 17,
        )
        if self.device.type == "cuda" and not config.enforce_eager:
            self.capture_cudagraphs()

    # ------------------------------------------------------------- KV cache
    def kv_bytes_per_page(self) -> int:
        cfg = self.config.hf_config
        kvh = cfg.num_key_value_heads // self.world_size
        return 2 * cfg.num_hidden_layers * self.page * kvh * cfg.head_dim * torch.tensor([], dtype=self.dtype).element_size()

    def allocate_kv_cache(self) -> None:
        config, cfg = self.config, self.config.hf_config
        per_page = self.kv_bytes_per_page()
        if config.num_kvcache_blocks <= 0:
            if self.device.type == "cuda":
                torch.cuda.synchronize()
                free, total = torch.cuda.mem_get_info()
                # Keep headroom for activations, logits and graph pools.
                reserve = self._activation_reserve_bytes()
                budget = int(total * config.gpu_memory_utilization - (total - free) - reserve)
                config.num_kvcache_blocks = budget // per_page
            else:
                pages_per_seq = -(-(config.max_model_len + config.max_diffusion_block_size) // self.page) + 1
                config.num_kvcache_blocks = min(config.max_num_seqs, 16) * pages_per_seq
            if config.num_kvcache_blocks <= 0:
                raise RuntimeError(
                    "Insufficient GPU memory for KV cache allocation "
                    f"({per_page / 1e6:.2f} MB per page); increase gpu_memory_utilization"
                )
            if self.world_size > 1:
                # Rank 0 schedules pages for every rank: all caches must hold the
                # same page count, so agree on the smallest one.
                import torch.distributed as dist

                n = torch.tensor([config.num_kvcache_blocks], device=self.device)
                dist.all_reduce(n, op=dist.ReduceOp.MIN)
                config.num_kvcache_blocks = int(n.item())
        kvh = cfg.num_key_value_heads // self.world_size
        self.kv_cache = torch.zeros(
            cfg.num_hidden_layers, 2, config.num_kvcache_blocks, kvh, self.page, cfg.head_dim,
            dtype=self.dtype, device=self.device,
        )
        for i, attn in enumerate(self.model.attention_layers):
            attn.k_cache = self.kv_cache[i, 0]
            attn.v_cache = self.kv_cache[i, 1]

    def _activation_reserve_bytes(self) -> int:
        config, cfg = self.config, self.config.hf_config
        max_q = max(config.max_diffusion_block_size, config.tree_verify_size or 0)
        T = max(config.max_num_seqs * max_q, min(config.max_num_batched_tokens, 16384))
        vocab_local = cfg.vocab_size // self.world_size
        inter = cfg.intermediate_size // self.world_size
        per_token = 2 * (vocab_local * 3 + cfg.hidden_size * 8 + inter * 4 + cfg.vocab_size * 2)
        return int(T * per_token) + (2 << 30)

    # ------------------------------------------------------------ forwards
    def _logits_full(self, logits: torch.Tensor) -> torch.Tensor:
        """Gather vocab shards so every rank holds the full logits row (kept sharded when
        sampling is vocab-parallel)."""
        if self.vocab_parallel:
            return logits
        return tp.all_gather_last_dim(logits)

    @torch.inference_mode()
    def run_prefill(self, seqs: list[Sequence], sp: SamplingParams) -> list[list[int]]:
        ids, pos, slots, cu_q, cu_k = [], [], [], [0], [0]
        max_pages = max(len(s.block_table) for s in seqs)
        tables = np.full((len(seqs), max_pages), -1, dtype=np.int32)
        for i, seq in enumerate(seqs):
            start, n = seq.num_cached_tokens, len(seq)
            ids.extend(seq.token_ids[start:])
            pos.append(np.arange(start, n, dtype=np.int64))
            slots.append(slots_for(seq.block_table, start, n - start, self.page))
            cu_q.append(cu_q[-1] + n - start)
            cu_k.append(cu_k[-1] + n)
            tables[i, : len(seq.block_table)] = seq.block_table
        dev = self.device
        meta = ForwardMeta(
            mode=Mode.PREFILL,
            positions=torch.from_numpy(np.concatenate(pos)).to(dev),
            slot_mapping=torch.from_numpy(np.concatenate(slots)).to(dev),
            block_tables=torch.from_numpy(tables).to(dev),
            cu_seqlens_q=torch.tensor(cu_q, dtype=torch.int32, device=dev),
            cu_seqlens_k=torch.tensor(cu_k, dtype=torch.int32, device=dev),
            max_seqlen_q=max(b - a for a, b in zip(cu_q, cu_q[1:])),
            max_seqlen_k=max(b - a for a, b in zip(cu_k, cu_k[1:])),
            logits_indices=torch.tensor(cu_q[1:], dtype=torch.int64, device=dev) - 1,
        )
        input_ids = torch.tensor(ids, dtype=torch.int64, device=dev)
        with nvtx("prefill"):
            hidden = self.model(input_ids, meta)
            logits = self._logits_full(self.model.compute_logits(hidden, meta))
        self.last_prefill_logits = logits  # last-position logits of the latest prefill (diagnostics)
        tokens, _ = self.sampler.sample(logits, sp)
        out = tokens.tolist()
        for seq, t in zip(seqs, out):
            seq.extend_tokens([int(t)])
            seq.num_cached_tokens = len(seq) - 1
        return [[int(t)] for t in out]

    def _stage_common(self, seqs, Q: int):
        ws = self.workspace
        B = len(seqs)
        if B > ws.max_seqs or Q > ws.max_q:
            raise ValueError(f"decode shape B={B}, Q={Q} exceeds workspace ({ws.max_seqs}, {ws.max_q})")
        ws.h_tables[:B].fill(-1)
        starts = np.empty(B, dtype=np.int64)
        for b, seq in enumerate(seqs):
            start = seq.num_cached_tokens
            if not 0 <= start <= len(seq):
                raise ValueError(f"invalid KV frontier {start} for length {len(seq)}")
            need = -(-(start + Q) // self.page)
            if len(seq.block_table) < need:
                raise RuntimeError(
                    "Scheduler did not reserve enough KV blocks for block forward: "
                    f"seq_id={seq.seq_id}, blocks={len(seq.block_table)}, required={need}"
                )
            if len(seq.block_table) > ws.max_pages:
                raise RuntimeError("sequence exceeds max_model_len page budget")
            ws.h_tables[b, : len(seq.block_table)] = seq.block_table
            starts[b] = start
        ws.h_prefix[:B] = starts
        return B, starts

    def stage_block(self, seqs, tokens: torch.Tensor, lora: bool):
        ws = self.workspace
        B, L = tokens.shape
        _, starts = self._stage_common(seqs, L)
        T = B * L
        pos = starts[:, None] + np.arange(L, dtype=np.int64)[None, :]
        ws.h_pos[:T] = pos.reshape(-1)
        tables = ws.h_tables[:B].astype(np.int64)
        pages = np.take_along_axis(tables, pos // self.page, axis=1)
        ws.h_slot[:T] = (pages * self.page + pos % self.page).reshape(-1)
        ws.h_mask[:T] = np.tile(causal_suffix_masks(L).numpy(), B)
        if lora:
            m = np.ones((B, L), dtype=np.float32)
            m[:, 0] = 0.0
            ws.h_lora[:T] = m.reshape(-1)
        ws.upload(lora, T)
        ws.input_ids[:T].copy_(tokens.reshape(-1))
        return B, L, starts

    @torch.inference_mode()
    def run_block(self, seqs, tokens: torch.Tensor, lora: bool = False) -> torch.Tensor:
        B, L, starts = self.stage_block(seqs, tokens, lora)
        logits = self._execute(Mode.BLOCK, B, L, lora)
        for seq, s in zip(seqs, starts):
            seq.num_cached_tokens = int(s) + L
        return logits.view(B, L, -1)

    def _execute(self, mode: Mode, B: int, Q: int, lora: bool) -> torch.Tensor:
        ws = self.workspace
        t0 = None
        if self.config.decode_timing and self.device.type == "cuda":
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record()
        key = self._graph_key(mode, B, Q, lora)
        if key is not None:
            graph, out = self.graphs[key]
            self._pad_rows(B, key[1], Q)
            graph.replay()
            self.cuda_graph_hits += 1
            logits = out[: B * Q]
        else:
            meta = ws.meta(mode, B, Q, lora)
            hidden = self.model(ws.input_ids[: B * Q], meta)
            logits = self.model.compute_logits(hidden, meta)
            self.cuda_graph_misses += 1
        logits = self._logits_full(logits)
        if t0 is not None:
            t1 = torch.cuda.Event(enable_timing=True)
            t1.record()
            self._timing_events.append({"start": t0, "end": t1, "step_index": self._timing_step,
                                        "batch_size": B, "block_len": Q, "cuda_graph_hit": key is not None})
        return logits

    # -------------------------------------------------------------- trees
    @torch.inference_mode()
    def run_tree(self, seqs, tokens, depths, parents) -> torch.Tensor:
        ws = self.workspace
        B, Q = tokens.shape
        _, starts = self._stage_common(seqs, Q)
        T = B * Q
        logical = starts[:, None] + np.arange(Q, dtype=np.int64)[None, :]
        tables = ws.h_tables[:B].astype(np.int64)
        pages = np.take_along_axis(tables, logical // self.page, axis=1)
        ws.h_slot[:T] = (pages * self.page + logical % self.page).reshape(-1)
        if self.device.type == "cuda":
            # positions (prefix + depth) and ancestor masks stay on the device: no host round trip
            ws.upload(False, T)
            from uno_b200.ops import cuda as cuda_ops

            cuda_ops.tree_meta(parents, depths, ws.prefix_lens[:B], ws.suffix_mask_flat[:T], ws.positions[:T])
        else:
            d = depths.cpu().numpy()
            ws.h_pos[:T] = (starts[:, None] + d).reshape(-1)
            ws.h_mask[:T] = ancestor_masks(parents.cpu()).numpy().reshape(-1)
            ws.upload(False, T)
        ws.input_ids[:T].copy_(tokens.reshape(-1))
        logits = self._execute(Mode.TREE, B, Q, False)
        for seq, s in zip(seqs, starts):
            seq.num_cached_tokens = int(s) + Q
        return logits.view(B, Q, -1)

    @torch.inference_mode()
    def compact_tree_kv(self, seqs, accepted_nodes, cache_lengths, tree_size: int) -> None:
        prefix = torch.tensor([s.num_cached_tokens - tree_size for s in seqs], dtype=torch.int64,
                              device=accepted_nodes.device)
        if bool((prefix < 0).any()):
            raise RuntimeError("invalid tree KV frontier")
        src, dst = tree_kv_moves(accepted_nodes, cache_lengths, prefix)
        tables = self.workspace.block_tables[: len(seqs)].to(torch.int64)
        if self.device.type == "cuda":
            from uno_b200.ops import cuda

            cuda.copy_tree_kv(self.kv_cache, tables, src, dst, self.page)
            return
        for b in range(len(seqs)):
            for j in range(src.shape[1]):
                s, t = int(src[b, j]), int(dst[b, j])
                if s < 0:
                    continue
                sp_, so = int(tables[b, s // self.page]), s % self.page
                dp_, do = int(tables[b, t // self.page]), t % self.page
                self.kv_cache[:, :, dp_, :, do, :] = self.kv_cache[:, :, sp_, :, so, :].clone()

    # ------------------------------------------------------------ graphs
    def _graph_batch_sizes(self) -> list[int]:
        if self.config.cuda_graph_batch_sizes is not None:
            return list(self.config.cuda_graph_batch_sizes)
        return sglang_batch_ladder(self.config.max_num_seqs)

    def _graph_key(self, mode, B, Q, lora):
        if not self.graphs:
            return None
        for bs in self._graph_batch_sizes():
            if bs >= B:
                key = (mode, bs, Q, lora)
                return key if key in self.graphs else None
        return None

    def _pad_rows(self, B: int, Bp: int, Q: int) -> None:
        """Neutralise rows B..Bp of a padded graph batch (no KV store)."""
        if Bp == B:
            return
        ws = self.workspace
        ws.slot_mapping[B * Q: Bp * Q].fill_(-1)
        ws.prefix_lens[B:Bp].zero_()
        ws.block_tables[B:Bp].zero_()
        ws.suffix_mask_flat[B * Q: Bp * Q].copy_(causal_suffix_masks(Q, self.device).repeat(Bp - B))

    @torch.inference_mode()
    def capture_cudagraphs(self) -> None:
        ws = self.workspace
        sizes = self._graph_batch_sizes()
        shapes = []
        for L in self.config.cuda_graph_block_sizes:
            shapes.append((Mode.BLOCK, L, False))
            if self.config.gated_lora and L > 1:
                shapes.append((Mode.BLOCK, L, True))
        if self.config.tree_verify_size is not None:
            shapes.append((Mode.TREE, self.config.tree_verify_size, False))
        from uno_b200.ops import cuda as cuda_ops

        cfg = self.config.hf_config
        cuda_ops.reserve_attention_scratch(self.device, ws.max_tokens,
                                           cfg.num_attention_heads // self.world_size, 16,
                                           max(1, cfg.num_key_value_heads // self.world_size))
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        pool = torch.cuda.graph_pool_handle()
        # Make all rows harmless during capture (no KV writes, zero prefixes).
        ws.slot_mapping.fill_(-1)
        ws.prefix_lens.zero_()
        ws.block_tables.zero_()
        ws.lora_mask.zero_()
        for mode, Q, lora in shapes:
            ws.suffix_mask_flat.copy_(causal_suffix_masks(Q, self.device).repeat(ws.max_tokens // Q + 1)[: ws.max_tokens])
            for bs in reversed(sizes):
                if bs * Q > ws.max_tokens:
                    continue
                meta = ws.meta(mode, bs, Q, lora)
                ids = ws.input_ids[: bs * Q]
                # warm-up run outside capture (allocations, lazy init)
                self.model.compute_logits(self.model(ids, meta), meta)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=pool):
                    out = self.model.compute_logits(self.model(ids, meta), meta)
                self.graphs[(mode, bs, Q, lora)] = (g, out)
        torch.cuda.synchronize()
        self.cuda_graph_memory = {
            "device_footprint_bytes": max(0, int(free0 - torch.cuda.mem_get_info()[0])),
            "num_graphs": len(self.graphs),
        }
        logger.info("captured %d CUDA graphs", len(self.graphs))

    def release_graphs(self) -> None:
        self.graphs.clear()

    # ------------------------------------------------------------ entry
    def reseed(self, seed: int) -> None:
        """Restart the sampler and noise streams (identically on every rank)."""
        self.sampler.reseed(seed)
        self.decoder.noise_gen.manual_seed(int(seed) + 17)

    def run(self, seqs: list[Sequence], is_prefill: bool, sp: SamplingParams) -> list[list[int]]:
        if is_prefill:
            return self.run_prefill(seqs, sp)
        self._timing_step += 1
        return self.decoder.run_cycle(seqs, sp)

    # ------------------------------------------------------------ bench hooks
    def timer_start(self) -> None:
        """Barrier + synchronise, then record a start event on this rank."""
        if self.world_size > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()
        self._t0 = torch.cuda.Event(enable_timing=True)
        self._t0.record()

    def timer_stop(self) -> float:
        """Elapsed device ms since ``timer_start``, max over TP ranks."""
        t1 = torch.cuda.Event(enable_timing=True)
        t1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([self._t0.elapsed_time(t1)], device=self.device)
        if self.world_size > 1:
            import torch.distributed as dist

            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            dist.barrier()
        return float(ms.item())

    def reset_decode_timing(self) -> None:
        self._timing_step = 0
        self._timing_events.clear()

    def get_decode_timing(self) -> dict:
        if not self.config.decode_timing:
            return {"enabled": False, "forward_records": []}
        if self.device.type == "cuda":
            torch.cuda.synchronize()
        recs = []
        for ev in self._timing_events:
            r = {k: v for k, v in ev.items() if k not in ("start", "end")}
            r["gpu_ms"] = ev["start"].elapsed_time(ev["end"])
            recs.append(r)
        return {"enabled": True, "forward_records": recs}

    def exit(self) -> None:
        self.release_graphs()
        if self.device.type == "cuda":
            torch.cuda.synchronize()
            if self.tp_comm is not None:
                from uno_b200.ops import cuda as cuda_ops

                cuda_ops.set_tp_comm(None)
                if self.control is not None:
                    import torch.distributed as dist

                    dist.barrier(group=self.control.group)  # no peer still reads our workspace
                self.tp_comm.close()
                self.tp_comm = None
