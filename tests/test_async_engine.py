"""AsyncLLMEngine: concurrent submission, results equal to the synchronous
engine, and the failure paths (fatal step error, shutdown, cancellation)."""

import concurrent.futures
import threading
import time

import pytest

from uno_b200 import SamplingParams
from uno_b200.engine.async_engine import AsyncLLMEngine, GenerationResult


class FakeEngine:
    """Minimal engine: each request finishes after `steps` steps."""

    def __init__(self, steps=2, fail_at=None):
        self.steps, self.fail_at = steps, fail_at
        self.live: dict[int, list] = {}
        self.next_id = 0
        self.nsteps = 0
        self.exited = threading.Event()

    def add_request(self, prompt, sp, max_tokens=None):
        if prompt == "bad":
            raise ValueError("bad prompt")
        sid = self.next_id
        self.next_id += 1
        self.live[sid] = [list(prompt) if not isinstance(prompt, str) else [len(prompt)], 0, max_tokens]
        return sid

    def is_finished(self):
        return not self.live

    def step(self):
        self.nsteps += 1
        if self.fail_at is not None and self.nsteps >= self.fail_at:
            raise RuntimeError("device lost")
        done = []
        for sid, st in list(self.live.items()):
            st[1] += 1
            if st[1] >= self.steps:
                done.append((sid, st[0] + [7] * (st[2] or 1), {"forwards": 2 * st[1], "accepts": st[1]}))
                del self.live[sid]
        return done, len(done)

    def finalize_output(self, token_ids, stats, sp):
        return {"text": " ".join(map(str, token_ids)), "token_ids": token_ids, "stats": stats}

    def exit(self):
        self.exited.set()


def sp():
    return SamplingParams(temperature=0.0, max_tokens=4, diffusion_block_size=4, mask_token_id=4095)


def test_concurrent_submit_resolves_every_future():
    eng = AsyncLLMEngine(FakeEngine(steps=3), sp())
    eng.start()
    futs = []

    def worker(base):
        for i in range(5):
            futs.append(eng.submit([base + i], request_id=f"r{base + i}", max_tokens=2))

    threads = [threading.Thread(target=worker, args=(100 * t,)) for t in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    results = [f.result(timeout=10) for f in futs]
    assert len(results) == 20 and all(isinstance(r, GenerationResult) for r in results)
    for r in results:
        assert r.token_ids[0] == int(r.request_id[1:]) and r.token_ids[1:] == [7, 7]
    eng.shutdown()
    assert not eng.is_running


def test_bad_request_fails_alone():
    eng = AsyncLLMEngine(FakeEngine(), sp())
    eng.start()
    bad = eng.submit("bad")
    good = eng.submit([1, 2])
    with pytest.raises(ValueError):
        bad.result(timeout=10)
    assert good.result(timeout=10).token_ids[:2] == [1, 2]
    assert eng.is_running
    eng.shutdown()


def test_fatal_step_error_fails_pending_and_rejects_new():
    fake = FakeEngine(steps=100, fail_at=3)
    eng = AsyncLLMEngine(fake, sp())
    eng.start()
    futs = [eng.submit([i]) for i in range(3)]
    for f in futs:
        with pytest.raises(RuntimeError, match="device lost"):
            f.result(timeout=10)
    deadline = time.time() + 5
    while eng.is_running and time.time() < deadline:
        time.sleep(0.01)
    assert isinstance(eng.fatal_error, RuntimeError)
    with pytest.raises(RuntimeError, match="failed"):
        eng.submit([9])
    assert fake.exited.wait(5)


def test_shutdown_fails_unfinished_and_releases_engine():
    fake = FakeEngine(steps=10 ** 9)
    eng = AsyncLLMEngine(fake, sp())
    eng.start()
    fut = eng.submit([1])
    time.sleep(0.05)
    eng.shutdown(timeout=10)
    with pytest.raises(RuntimeError, match="shut down before this request finished"):
        fut.result(timeout=5)
    assert fake.exited.is_set()
    with pytest.raises(RuntimeError, match="not running"):
        eng.submit([2])


def test_cancelled_request_is_not_admitted():
    fake = FakeEngine(steps=1)
    eng = AsyncLLMEngine(fake, sp())
    eng.start()
    with eng._cv:  # hold the loop off while the request is cancelled
        fut = eng.submit([5])
        assert fut.cancel()
    time.sleep(0.05)
    assert fake.next_id == 0
    eng.shutdown()


def test_real_engine_matches_synchronous_generate():
    """Greedy decoding through the async front end equals LLM.generate (tiny CPU model)."""
    from uno_b200 import LLM

    kw = dict(device="cpu", max_num_seqs=8, max_model_len=256, kvcache_block_size=64, dummy_lora_rank=8,
              dummy_lora_alpha=16, max_diffusion_block_size=4)
    prompts = [[3, 14, 15, 92, 65], [35, 89, 79, 32, 38, 46], [26, 43]]
    params = SamplingParams(temperature=0.0, max_tokens=12, diffusion_block_size=4, mask_token_id=4095,
                            ignore_eos=True)
    ref_llm = LLM("preset:tiny-qwen3", **kw)
    ref = [o["token_ids"] for o in ref_llm.generate(prompts, params, use_tqdm=False)]
    ref_llm.exit()
    eng = AsyncLLMEngine(LLM("preset:tiny-qwen3", **kw), params)
    eng.start()
    futs = [eng.submit(p) for p in prompts]
    got = [f.result(timeout=120).token_ids for f in futs]
    eng.shutdown()
    assert got == ref
