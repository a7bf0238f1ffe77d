"""Host-side engine pieces: block manager, prefix cache, scheduler, noise, trees."""

import numpy as np
import pytest
import torch

from uno_b200.engine.block_manager import BlockManager
from uno_b200.engine.draft_tree import build_tree_from_candidates, tree_kv_moves, walk_tree
from uno_b200.engine.noise import build_draft_batch, deterministic_noise, noise_bounds
from uno_b200.engine.scheduler import Scheduler
from uno_b200.engine.sequence import Sequence, SequenceStatus
from uno_b200.layers.meta import ancestor_masks, causal_suffix_masks
from uno_b200.sampling_params import SamplingParams


class _Cfg:
    def __init__(self, blocks=32, page=4, max_seqs=8, max_tokens=64, tree=None, fail=False):
        self.max_num_seqs = max_seqs
        self.max_num_batched_tokens = max_tokens
        self.eos = 0
        self.fail_on_preemption = fail
        self.tree_verify_size = tree
        self.num_kvcache_blocks = blocks
        self.kvcache_block_size = page


@pytest.fixture(autouse=True)
def _page4():
    old = Sequence.block_size
    Sequence.block_size = 4
    yield
    Sequence.block_size = old


def test_sequence_rollback_bounds():
    s = Sequence([1, 2, 3])
    s.num_cached_tokens = 3
    s.extend_tokens([4, 5])
    with pytest.raises(ValueError):
        s.rollback_kv_to(5)  # above current frontier
    with pytest.raises(ValueError):
        s.rollback_kv_to(1)  # below len - 1
    s.num_cached_tokens = 5
    s.rollback_kv_to(4)
    assert s.num_cached_tokens == 4


def test_run_command_roundtrip_through_the_channel():
    """A packed ``run`` command rebuilds the follower's view of every sequence."""
    from uno_b200.engine.control import CommandChannel, RunDecoder, RunEncoder, TokenTail
    from uno_b200.sampling_params import SamplingParams

    a = Sequence([5, 6, 7, 8, 9], max_completion_tokens=7)
    a.block_table = [3, 1]
    a.num_cached_tokens = 4
    b = Sequence(list(range(1, 300)))
    b.block_table = [0, 2, 4]
    b.num_cached_tokens = 298
    sp = SamplingParams(temperature=1.0, max_tokens=8, diffusion_block_size=4, mask_token_id=90,
                        noise_mode="deterministic_uniform")
    ch = CommandChannel(None, 0, 1, size=1 << 16)
    try:
        enc, dec = RunEncoder(), RunDecoder()
        for prefill in (True, False, False):
            n = enc.encode(ch.begin_write(), [a, b], prefill, sp)
            seqs, is_prefill, sp2 = dec.decode(bytes(ch.payload[:n]))
            assert is_prefill == prefill and sp2 == sp
            for src, got in zip((a, b), seqs):
                assert (got.seq_id, len(got), got.last_token, got.num_cached_tokens, got.block_table,
                        got.num_prompt_tokens, got.max_completion_tokens) == \
                       (src.seq_id, len(src), src.last_token, src.num_cached_tokens, src.block_table,
                        src.num_prompt_tokens, src.max_completion_tokens)
                assert got.noise_seed == src.noise_seed is not None  # deterministic noise needs the prompt hash
                if prefill:
                    assert got.token_ids == src.token_ids
                else:
                    assert isinstance(got.token_ids, TokenTail)
        tail = TokenTail(3, 7)
        tail.extend([8, 9])
        assert len(tail) == 5 and tail[-1] == 9
    finally:
        ch.close()


def test_prefix_cache_hit_and_reactivation():
    bm = BlockManager(16, 4)
    a = Sequence(list(range(1, 11)))  # 10 tokens: 2 full pages + 2
    assert bm.plan_prefix_cache_and_check_capacity(a) == 0
    bm.allocate(a, 0)
    a.num_cached_tokens = 9
    bm.publish_computed_prefix_blocks(a)
    b = Sequence(list(range(1, 11)) + [99])
    assert bm.plan_prefix_cache_and_check_capacity(b) == 2
    bm.allocate(b, 2)
    assert b.block_table[:2] == a.block_table[:2]
    assert bm.blocks[a.block_table[0]].ref_count == 2
    bm.deallocate(a)
    bm.deallocate(b)
    # Pages are free but still hashed: a third request re-activates them.
    c = Sequence(list(range(1, 10)) + [7, 7])
    hits = bm.plan_prefix_cache_and_check_capacity(c)
    assert hits == 2
    bm.allocate(c, hits)
    assert c.num_cached_tokens == 8


def test_uncached_last_token_not_shared():
    bm = BlockManager(8, 4)
    a = Sequence([1, 2, 3, 4])
    bm.allocate(a, 0)
    a.num_cached_tokens = 4
    bm.publish_computed_prefix_blocks(a)
    b = Sequence([1, 2, 3, 4])
    # all 4 tokens would be cached but the last token must stay uncached
    assert bm.plan_prefix_cache_and_check_capacity(b) == 0


def test_scheduler_prefill_then_decode_and_preempt():
    cfg = _Cfg(blocks=6, page=4, max_seqs=4, max_tokens=64)
    sch = Scheduler(cfg)
    sp = SamplingParams(diffusion_block_size=4, mask_token_id=50)
    seqs = [Sequence([1] * 6), Sequence([2] * 6)]
    for s in seqs:
        sch.add(s)
    batch, prefill = sch.schedule(sp)
    assert prefill and len(batch) == 2
    for s in batch:
        s.extend_tokens([3])
        s.num_cached_tokens = len(s) - 1
    batch, prefill = sch.schedule(sp)
    assert not prefill
    # 6 pages total; each seq of 7 tokens + 4 reserve needs 3 pages -> both fit
    assert len(batch) == 2 and sch.num_preemptions == 0
    for s in batch:
        s.extend_tokens([5] * 4)
        s.num_cached_tokens = len(s) - 1
    batch, _ = sch.schedule(sp)
    # 11 tokens + 4 reserve = 4 pages each: one request must be preempted
    assert sch.num_preemptions >= 1
    assert seqs[1].status is SequenceStatus.WAITING


def test_scheduler_fail_on_preemption():
    cfg = _Cfg(blocks=3, page=4, fail=True)
    sch = Scheduler(cfg)
    sp = SamplingParams(diffusion_block_size=4, mask_token_id=50)
    a, b = Sequence([1] * 4), Sequence([2] * 4)
    sch.add(a)
    sch.add(b)
    sch.schedule(sp)
    for s in (a, b):
        s.extend_tokens([1])
        s.num_cached_tokens = len(s) - 1
    with pytest.raises(RuntimeError, match="preemption disabled"):
        sch.schedule(sp)


def test_prefill_budget_is_unchunked():
    sch = Scheduler(_Cfg(blocks=64, max_tokens=8))
    sch.add(Sequence([1] * 9))
    with pytest.raises(ValueError, match="non-chunked"):
        sch.schedule(SamplingParams())


def test_noise_modes():
    sp = SamplingParams(diffusion_block_size=4, mask_token_id=100, noise_mode="random_uniform")
    seqs = [Sequence([5, 6]), Sequence([7])]
    g = torch.Generator().manual_seed(0)
    d = build_draft_batch(seqs, 4, sp, vocab_size=1000, generator=g)
    assert d.shape == (2, 4) and list(d[:, 0]) == [6, 7]
    assert ((d[:, 1:] >= 1) & (d[:, 1:] < 100)).all()
    spm = SamplingParams(diffusion_block_size=4, mask_token_id=100, noise_mode="mask")
    assert (build_draft_batch(seqs, 4, spm, vocab_size=1000)[:, 1:] == 100).all()
    spd = SamplingParams(diffusion_block_size=4, mask_token_id=100, noise_mode="deterministic_uniform", noise_salt=3)
    a = deterministic_noise(seqs[0], 3, 1, 100, 6, spd)
    b = deterministic_noise(seqs[0], 3, 1, 100, 6, spd)
    assert a == b and all(1 <= t < 100 for t in a)
    assert noise_bounds(sp, 50) == (1, 50)


def test_tree_builder_best_first_and_order():
    toks = [[10, 11], [20, 21], [30, 31]]
    lps = [[-0.1, -1.0], [-0.2, -2.0], [-0.3, -3.0]]
    t = build_tree_from_candidates(1, toks, lps, 5)
    assert t.num_nodes == 5
    assert t.token_ids[0] == 1 and t.parent_indices[0] == -1
    for i, p in enumerate(t.parent_indices[1:], start=1):
        assert p < i and t.depths[i] == t.depths[p] + 1
    # best chain first: 10 -> 20 -> 30
    assert list(t.token_ids[1:4]) == [10, 20, 30]


def test_walk_tree_follows_targets():
    tokens = torch.tensor([[1, 10, 11, 20]])
    parents = torch.tensor([[-1, 0, 0, 1]])
    targets = torch.tensor([[10, 20, 0, 42]])
    committed, acc, lens = walk_tree(tokens, parents, targets, max_depth=3, pad_token_id=0)
    assert lens.tolist() == [4]
    assert committed[0, :4].tolist() == [1, 10, 20, 42]
    assert acc[0, :3].tolist() == [0, 1, 3]
    src, dst = tree_kv_moves(acc, lens - 1, torch.tensor([100]))
    assert src[0, :3].tolist() == [100, 101, 103] and dst[0, :3].tolist() == [100, 101, 102]


def test_masks():
    m = causal_suffix_masks(3)
    assert m.tolist() == [1, 3, 7]
    par = torch.tensor([[-1, 0, 0, 1]])
    am = ancestor_masks(par)
    assert am.tolist() == [[1, 3, 5, 11]]
    assert causal_suffix_masks(64)[-1].item() == -1


def test_command_channel_size_from_environment():
    import pytest

    from uno_b200.engine.control import CommandChannel, channel_bytes

    assert channel_bytes({}) == 64 << 20
    assert channel_bytes({"INFERENCE_ENGINE_SHM_SIZE": str(1 << 20)}) == 1 << 20
    with pytest.raises(ValueError):
        channel_bytes({"INFERENCE_ENGINE_SHM_SIZE": "12"})
    ch = CommandChannel(None, 0, 1, size=8192)
    try:
        assert ch.capacity >= 8192
        with pytest.raises(ValueError, match="INFERENCE_ENGINE_SHM_SIZE"):
            ch.commit(ch.capacity + 1)
    finally:
        ch.close()
