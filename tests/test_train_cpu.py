"""Conditional-LoRA diffusion training on CPU (BASELINE config 1 training step)."""

import json
import os

import pytest
import torch

from uno_b200.train import (IGNORE_INDEX, BlockCurriculumPlan, LoraSettings, TrainableLoRA, UnoObjectiveConfig,
                            UnoTrainer, build_uno_batch, shift_labels_for_next_token)
from uno_b200.train.layout import visibility
from uno_b200.train.losses import fused_head_loss, reference_losses


# ------------------------------------------------------------------ layout
def test_layout_places_noisy_then_clean_per_packed_sequence():
    ids = torch.tensor([[10, 11, 12, 13, 20, 21]])
    labels = torch.tensor([[IGNORE_INDEX, 11, 12, 13, 20, 21]])
    pos = torch.tensor([[0, 1, 2, 3, 0, 1]])  # two packed sequences of 4 and 2 tokens
    ub = build_uno_batch(ids, labels, pos, block_size=2, mask_token_id=100, generator=torch.Generator().manual_seed(0))
    # layout: [noisy(seq0) 4][clean(seq0) 4][noisy(seq1) 2][clean(seq1) 2]
    assert ub.noisy.tolist() == [[True] * 4 + [False] * 4 + [True] * 2 + [False] * 2]
    assert ub.positions.tolist() == [[0, 1, 2, 3, 0, 1, 2, 3, 0, 1, 0, 1]]
    assert ub.ids[0, 4:8].tolist() == [10, 11, 12, 13] and ub.ids[0, 10:].tolist() == [20, 21]
    # unsupervised tokens are never noised; noise ids lie in [1, mask)
    assert not bool(ub.noised[0, 0])
    noisy_ids = ub.ids[0, ub.noisy_index[0]]
    assert bool(((noisy_ids == ids[0]) | ub.noised[0]).all())
    assert bool(((noisy_ids >= 1) & (noisy_ids < 100) | ~ub.noised[0]).all())
    assert ub.p_mask.numel() == int(ub.noised.sum())
    hidden = torch.arange(12.0)[None, :, None]
    n, c = ub.gather_regions(hidden)
    assert n[0, :, 0].tolist() == [0, 1, 2, 3, 8, 9] and c[0, :, 0].tolist() == [4, 5, 6, 7, 10, 11]


def test_visibility_rules():
    seg = torch.tensor([[0] * 8])
    pos = torch.tensor([[0, 1, 2, 3, 0, 1, 2, 3]])
    noisy = torch.tensor([[True] * 4 + [False] * 4])
    vis = visibility(seg, pos, noisy, block_size=2)[0]
    # noisy token at position 2 (block 1): noisy 2,3 of its block; clean positions 0,1 only
    assert vis[2].tolist() == [False, False, True, True, True, True, False, False]
    # noisy token at position 0: only its own block's noisy tokens
    assert vis[0].tolist() == [True, True, False, False, False, False, False, False]
    # clean token at position 2: clean 0..2
    assert vis[6].tolist() == [False, False, False, False, True, True, True, False]
    # packed sequences never see each other
    seg2 = torch.tensor([[0, 0, 1, 1]])
    vis2 = visibility(seg2, torch.tensor([[0, 1, 0, 1]]), torch.tensor([[False] * 4]), 2)[0]
    assert not bool(vis2[2, 0]) and not bool(vis2[3, 1])


def test_shift_labels_masks_packed_boundaries():
    labels = torch.tensor([[1, 2, 3, 4, 5]])
    pos = torch.tensor([[0, 1, 2, 0, 1]])
    assert shift_labels_for_next_token(labels, pos).tolist() == [[2, 3, IGNORE_INDEX, 5, IGNORE_INDEX]]


# ------------------------------------------------------------------ losses
@pytest.mark.parametrize("weights,teacher_ce", [((1.0, 0.0, 0.0), True), ((0.0, 1.0, 0.0), True),
                                                ((0.3, 0.5, 0.7), True), ((0.0, 0.0, 1.0), False)])
def test_fused_head_loss_matches_autograd(weights, teacher_ce):
    torch.manual_seed(0)
    N, H, V = 23, 16, 97
    W = torch.randn(V, H)
    sh = torch.randn(N, H, requires_grad=True)
    th = torch.randn(N, H)
    dist_mask = torch.rand(N) < 0.8
    ce_mask = dist_mask & (torch.rand(N) < 0.6)
    p = torch.rand(N) * 0.9 + 0.1
    tgt = torch.randint(0, V, (N,))
    tv_w, kl_w, ce_w = weights
    count = int(dist_mask.sum())
    loss = fused_head_loss(sh, th, W, dist_mask=dist_mask, ce_mask=ce_mask, ce_target=tgt, ce_scale=1 / p,
                           tv_weight=tv_w, kl_weight=kl_w, ce_weight=ce_w, teacher_ce=teacher_ce,
                           normalizer=count, chunk=7)
    loss.backward()
    g_fused = sh.grad.clone()
    sh2 = sh.detach().clone().requires_grad_(True)
    s, t = sh2 @ W.t(), th @ W.t()
    tv, kl = reference_losses(s[dist_mask], t[dist_mask], count)
    y = t.argmax(-1) if teacher_ce else tgt
    ce = (torch.nn.functional.cross_entropy(s[ce_mask], y[ce_mask], reduction="none") / p[ce_mask]).sum() / count
    ref = tv_w * tv + kl_w * kl + ce_w * ce
    ref.backward()
    assert torch.allclose(loss, ref, rtol=1e-4, atol=1e-5)
    assert torch.allclose(g_fused, sh2.grad, rtol=1e-3, atol=1e-5)


# -------------------------------------------------------------- training
def _tiny_setup(rank=8, seed=0):
    from uno_b200.models.decoder import build_model
    from uno_b200.models.presets import resolve_preset
    from uno_b200.utils.loader import dummy_init

    cfg = resolve_preset("tiny-qwen3")
    model = build_model(cfg)
    dummy_init(model, seed=seed)
    lora = TrainableLoRA(cfg, LoraSettings(rank=rank, alpha=16), seed=seed)
    return cfg, model, lora


def _batch(B=2, S=128, vocab=4096, seed=0):
    from uno_b200.train.data import synthetic_batches

    return next(synthetic_batches(B, S, vocab, seed=seed))


def test_config1_training_step_updates_lora_only():
    cfg, model, lora = _tiny_setup()
    base_before = {k: v.clone() for k, v in model.state_dict().items()}
    plan = BlockCurriculumPlan.fixed([4], 3, 128, 2)
    tr = UnoTrainer(model, lora, objective=UnoObjectiveConfig(ce_weight=0.5, kl_weight=0.5, tv_weight=1.0),
                    curriculum=plan, mask_token_id=cfg.mask_token_id, lr=1e-2)
    m = tr.train_step([_batch()])
    assert m["step"] == 1 and m["block_size"] == 4 and m["tokens"] == 256 and m["noised_tokens"] > 0
    assert torch.isfinite(torch.tensor(m["loss"])) and m["grad_norm"] > 0
    assert any(float(b.detach().abs().sum()) > 0 for b in lora.B.values())  # B starts at zero
    for k, v in model.state_dict().items():
        assert torch.equal(v, base_before[k]), k


def test_training_reduces_loss_on_a_fixed_batch():
    cfg, model, lora = _tiny_setup(seed=1)
    plan = BlockCurriculumPlan.fixed([4], 12, 64, 2)
    tr = UnoTrainer(model, lora, objective=UnoObjectiveConfig(), curriculum=plan, mask_token_id=cfg.mask_token_id,
                    lr=3e-3, seed=5)
    batch = _batch(2, 64, seed=3)
    losses = []
    for _ in range(12):
        tr.generator.manual_seed(123)  # same noise every step
        losses.append(tr.train_step([batch])["loss"])
    assert losses[-1] < 0.7 * losses[0]


def test_curriculum_checkpoint_and_resume(tmp_path):
    cfg, model, lora = _tiny_setup()
    plan = BlockCurriculumPlan.fixed([2, 4], 1, 32, 1)
    obj = UnoObjectiveConfig()
    tr = UnoTrainer(model, lora, objective=obj, curriculum=plan, mask_token_id=cfg.mask_token_id, lr=1e-2,
                    output_dir=str(tmp_path))
    b = _batch(1, 32)
    assert tr.train_step([b])["block_size"] == 2
    ckpt = tmp_path / "checkpoint-1"
    state = json.loads((ckpt / "uno_curriculum_state.json").read_text())
    assert state["reason"] == "completed_block_size_2" and state["curriculum_sha256"] == plan.sha256()
    assert (ckpt / "adapter_config.json").is_file()
    # resume into a fresh trainer: same LoRA, continues at stage 2
    _, model2, lora2 = _tiny_setup(seed=9)
    tr2 = UnoTrainer(model2, lora2, objective=obj, curriculum=plan, mask_token_id=cfg.mask_token_id, lr=1e-2)
    tr2.resume(ckpt)
    assert tr2.step == 1
    for k in lora.A:
        assert torch.equal(lora.A[k], lora2.A[k]) and torch.equal(lora.B[k], lora2.B[k])
    assert tr2.curriculum.stage_for_step(tr2.step).block_size == 4
    other = BlockCurriculumPlan.fixed([2, 8], 1, 32, 1)
    tr3 = UnoTrainer(model2, lora2, objective=obj, curriculum=other, mask_token_id=cfg.mask_token_id)
    with pytest.raises(ValueError, match="curriculum"):
        tr3.resume(ckpt)


def test_trained_adapter_serves_in_the_inference_engine(tmp_path):
    from uno_b200 import LLM, SamplingParams

    cfg, model, lora = _tiny_setup()
    plan = BlockCurriculumPlan.fixed([4], 1, 32, 1)
    UnoTrainer(model, lora, objective=UnoObjectiveConfig(), curriculum=plan, mask_token_id=cfg.mask_token_id,
               lr=1e-2).train_step([_batch(1, 32)])
    path = str(tmp_path / "adapter")
    lora.save(path, "preset:tiny-qwen3")
    llm = LLM("preset:tiny-qwen3", device="cpu", max_num_seqs=2, max_model_len=128, kvcache_block_size=64,
              gated_lora_path=path, max_diffusion_block_size=4)
    out = llm.generate([[5, 6, 7]], SamplingParams(temperature=0.0, max_tokens=8, diffusion_block_size=4,
                                                   mask_token_id=cfg.mask_token_id, ignore_eos=True),
                       use_tqdm=False)
    llm.exit()
    assert len(out[0]["token_ids"]) >= 8


def test_curriculum_yaml_rules(tmp_path):
    y = tmp_path / "c.yaml"
    y.write_text("tokens_per_step: 64\nsequence_length: 32\nglobal_batch_size: 2\nseed: 1\n"
                 "stages:\n  - block_size: 2\n    tokens: 128\n  - block_size: 4\n    tokens: 200\n")
    plan = BlockCurriculumPlan.from_yaml(y)
    assert [(s.block_size, s.start_step, s.end_step) for s in plan.stages] == [(2, 0, 2), (4, 2, 5)]
    assert plan.stage_for_step(1).block_size == 2 and plan.stage_for_step(2).block_size == 4
    assert plan.checkpoint_reasons == {2: "completed_block_size_2", 5: "completed_block_size_4"}
    y.write_text("tokens_per_step: 64\nsequence_length: 32\nglobal_batch_size: 2\nseed: 1\n"
                 "stages:\n  - block_size: 4\n    tokens: 128\n  - block_size: 2\n    tokens: 200\n")
    with pytest.raises(ValueError, match="increasing"):
        BlockCurriculumPlan.from_yaml(y)


def _dp_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg, model, lora = _tiny_setup()
    plan = BlockCurriculumPlan.fixed([4], 2, 32, 2)
    tr = UnoTrainer(model, lora, objective=UnoObjectiveConfig(), curriculum=plan, mask_token_id=cfg.mask_token_id,
                    lr=1e-2, process_group=dist.group.WORLD, seed=3)
    tr.train_step([_batch(1, 32, seed=rank)])  # different data per rank
    torch.save({k: v.detach().clone() for k, v in lora.state_dict().items()}, os.path.join(out, f"r{rank}.pt"))
    dist.destroy_process_group()


def test_data_parallel_ranks_stay_in_sync(tmp_path):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_dp_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    a, b = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)


def test_training_cli_stops_and_resumes_at_a_stage_boundary(tmp_path, capsys):
    from uno_b200.train.__main__ import main

    out = str(tmp_path / "run")
    common = ["--model", "preset:tiny-qwen3", "--output-dir", out, "--device", "cpu", "--block-sizes", "4,8",
              "--steps-per-stage", "2", "--seq-len", "32", "--global-batch", "2", "--micro-batch", "1",
              "--lora-rank", "8"]
    first = main(common + ["--max-steps", "2"])
    assert [m["step"] for m in first] == [1, 2]
    assert os.path.isfile(os.path.join(out, "checkpoint-2", "uno_curriculum_state.json"))
    rest = main(common + ["--resume", os.path.join(out, "checkpoint-2")])
    assert [m["step"] for m in rest] == [3, 4] and all(m["block_size"] == 8 for m in rest)
    assert os.path.isfile(os.path.join(out, "final_adapter", "adapter_model.safetensors"))
    # a different objective does not match the run manifest
    with pytest.raises(ValueError, match="does not match"):
        main(common + ["--resume", os.path.join(out, "checkpoint-2"), "--kl-weight", "1.0"])


# ---------------------------------------------------------- sharded AdamW
def _adamw_ref(init, grads_per_rank, steps, lr, wd, clip):
    """torch.optim.AdamW on rank-averaged, globally clipped gradients."""
    params = [torch.nn.Parameter(t.clone()) for t in init]
    opt = torch.optim.AdamW(params, lr=lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=wd)
    for s in range(steps):
        for i, p in enumerate(params):
            p.grad = sum(g[s][i] for g in grads_per_rank) / len(grads_per_rank)
        torch.nn.utils.clip_grad_norm_(params, clip)
        opt.step()
    return [p.detach() for p in params]


def _grads(rank, steps, shapes):
    g = torch.Generator().manual_seed(100 + rank)
    return [[torch.randn(*sh, generator=g) * (3.0 if s == 0 else 0.01) for sh in shapes] for s in range(steps)]


def _adamw_worker(rank, world, port, box):
    import torch.distributed as dist

    from uno_b200.train.optim import ShardedLoraAdamW

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    shapes = [(3, 5), (7,), (2, 2, 3)]
    init = [torch.linspace(-1, 1, int(torch.tensor(sh).prod())).view(*sh) for sh in shapes]
    params = [torch.nn.Parameter(t.clone()) for t in init]
    opt = ShardedLoraAdamW(params, lr=0.05, weight_decay=0.1, max_grad_norm=1.0, group=dist.group.WORLD)
    grads = _grads(rank, 3, shapes)
    norms = []
    for s in range(3):
        opt.zero_grad()
        for p, g in zip(params, grads[s]):
            p.grad += g  # accumulate like autograd does into the flat buffer view
        norms.append(opt.step())
    box.put((rank, [p.detach().clone() for p in params], norms))
    dist.destroy_process_group()


def test_sharded_adamw_matches_torch_adamw_two_ranks():
    import multiprocessing as mp
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")  # forked children of a process with torch threads can deadlock
    box = ctx.Queue()
    procs = [ctx.Process(target=_adamw_worker, args=(r, 2, port, box)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict((r, (ps, ns)) for r, ps, ns in (box.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(30)
    shapes = [(3, 5), (7,), (2, 2, 3)]
    init = [torch.linspace(-1, 1, int(torch.tensor(sh).prod())).view(*sh) for sh in shapes]
    want = _adamw_ref(init, [_grads(r, 3, shapes) for r in range(2)], 3, 0.05, 0.1, 1.0)
    for r in range(2):
        for got, ref in zip(out[r][0], want):
            torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-6)
    assert out[0][1] == out[1][1] and out[0][1][0] > 1.0  # the first step is clipped


def _dp_trainer_worker(rank, port, box):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    cfg, model, lora = _tiny_setup(seed=4)  # same initial weights on every rank
    plan = BlockCurriculumPlan.fixed([4], 3, 64, 2)
    tr = UnoTrainer(model, lora, objective=UnoObjectiveConfig(), curriculum=plan, mask_token_id=cfg.mask_token_id,
                    lr=1e-2, seed=9, process_group=dist.group.WORLD)
    metrics = [tr.train_step([_batch(1, 64, seed=rank * 10 + s)]) for s in range(2)]  # different data per rank
    flat = torch.cat([p.detach().reshape(-1) for p in lora.parameters()])
    box.put((rank, flat, [m["grad_norm"] for m in metrics]))
    dist.destroy_process_group()


def test_data_parallel_training_keeps_ranks_in_sync():
    """Two gloo ranks on different data: the ZeRO-2 step leaves identical LoRA parameters on both."""
    import multiprocessing as mp
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")  # forked children of a process with torch threads can deadlock
    box = ctx.Queue()
    procs = [ctx.Process(target=_dp_trainer_worker, args=(r, port, box)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict((r, (flat, norms)) for r, flat, norms in (box.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(30)
    assert torch.equal(out[0][0], out[1][0])
    assert out[0][1] == out[1][1]  # the global gradient norm is the same on both ranks
    assert float(out[0][0].abs().sum()) > 0


def _dp_resume_worker(rank, port, out_dir, box):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    plan = BlockCurriculumPlan.fixed([4, 8], 2, 64, 2)  # boundary checkpoint after step 2

    def trainer(output_dir):
        cfg, model, lora = _tiny_setup(seed=4)
        return UnoTrainer(model, lora, objective=UnoObjectiveConfig(), curriculum=plan,
                          mask_token_id=cfg.mask_token_id, lr=1e-2, seed=9, process_group=dist.group.WORLD,
                          output_dir=output_dir), lora

    def batches(steps):
        return [[_batch(1, 64, seed=rank * 10 + s)] for s in steps]

    tr, lora = trainer(None)  # uninterrupted: 4 steps
    for b in batches(range(4)):
        tr.train_step(b)
    straight = torch.cat([p.detach().reshape(-1) for p in lora.parameters()])
    tr1, _ = trainer(out_dir)  # 2 steps, checkpoint at the stage boundary
    for b in batches(range(2)):
        tr1.train_step(b)
    dist.barrier()
    tr2, lora2 = trainer(None)  # fresh process state, resume, 2 more steps
    tr2.resume(f"{out_dir}/checkpoint-2")
    for b in batches(range(2, 4)):
        tr2.train_step(b)
    resumed = torch.cat([p.detach().reshape(-1) for p in lora2.parameters()])
    box.put((rank, torch.equal(straight, resumed), float((straight - resumed).abs().max())))
    dist.destroy_process_group()


def test_data_parallel_resume_from_boundary_matches_uninterrupted(tmp_path):
    """Per-rank optimizer shards + RNG state in the boundary checkpoint: resuming reproduces the run."""
    import multiprocessing as mp
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")  # forked children of a process with torch threads can deadlock
    box = ctx.Queue()
    procs = [ctx.Process(target=_dp_resume_worker, args=(r, port, str(tmp_path), box)) for r in range(2)]
    for p in procs:
        p.start()
    out = [box.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(30)
    assert (tmp_path / "checkpoint-2" / "trainer_state_rank1.pt").is_file()
    assert all(same for _, same, _ in out), out


def test_openthoughts_encoding_budget_alignment_and_hash(tmp_path):
    import json

    from uno_b200.train.prepare import corpus_hash, encode_conversation, prepare, split_budget

    class Tok:  # one token per character; pad id 0
        pad_token_id = 0

        def encode(self, text, add_special_tokens=False):
            return [1 + (ord(c) % 200) for c in text]

    assert split_budget(10, 10, 100) == (10, 10)
    assert split_budget(10, 80, 100) == (10, 80)       # prompt under half: the answer gets the rest
    assert split_budget(80, 80, 100) == (50, 50)       # proportional split
    conv = [{"from": "human", "value": "hi"}, {"from": "gpt", "value": "yo"}]
    enc = encode_conversation(conv, Tok(), cutoff=4096, align=3)
    n_src = len("<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n")
    assert enc["labels"][:n_src] == [-100] * n_src and len(enc["input_ids"]) % 3 == 0
    assert enc["labels"][n_src:n_src + len("<think>\n")] == Tok().encode("<think>\n")   # empty think block added
    long = [{"from": "human", "value": "q" * 5000}, {"from": "gpt", "value": "a" * 5000}]
    assert len(encode_conversation(long, Tok(), cutoff=4096, align=3)["input_ids"]) <= 4095
    h1 = corpus_hash([enc])
    assert h1["row_count"] == 1 and h1["supervised_token_count"] == sum(t != -100 for t in enc["labels"])
    src = tmp_path / "src.jsonl"
    src.write_text("\n".join(json.dumps({"conversations": conv}) for _ in range(3)) + "\n")
    man = prepare(str(src), tmp_path / "out", Tok())
    assert man["hash"]["row_count"] == 3
    prepare(str(src), tmp_path / "again", Tok(), verify_against=tmp_path / "out")   # same corpus verifies
    many = tmp_path / "many.jsonl"
    many.write_text("".join(json.dumps({"conversations": [{"from": "human", "value": f"q{i}" * (i + 1)},
                                                           {"from": "gpt", "value": f"a{i}"}]}) + "\n"
                            for i in range(7)))
    one = prepare(str(many), tmp_path / "p1", Tok())
    two = prepare(str(many), tmp_path / "p2", Tok(), num_proc=2, writer_batch_size=2)
    assert one["hash"] == two["hash"] and one["hash"]["row_count"] == 7
    assert (tmp_path / "p1" / "rows.jsonl").read_text() == (tmp_path / "p2" / "rows.jsonl").read_text()


def test_fixed_curriculum_builder(tmp_path):
    import pytest

    from uno_b200.train.curriculum import BlockCurriculumPlan, fixed_curriculum, write_curriculum
    from uno_b200.train.make_curriculum import main as make_curriculum

    m = fixed_curriculum("0.5")  # 0.5 x 9375 = 4687.5 steps, rounded half up
    plan = BlockCurriculumPlan.from_mapping(m)
    assert plan.max_steps == 4688 and [s.block_size for s in plan.stages] == [8]
    assert m["tokens_per_step"] == 4096 * 128 and m["total_tokens"] == 4688 * 4096 * 128
    assert m["requested_epochs"] == "0.5" and m["resolved_epochs"].startswith("0.50005")
    with pytest.raises(ValueError):
        fixed_curriculum("0")
    with pytest.raises(ValueError):
        fixed_curriculum("nan")
    out = tmp_path / "c" / "b16.yaml"
    got = make_curriculum(["fixed", "--output", str(out), "--epochs", "2", "--block-size", "16",
                           "--steps-per-epoch", "10", "--global-batch-size", "4", "--sequence-length", "64"])
    loaded = BlockCurriculumPlan.from_yaml(out)
    assert got["max_steps"] == loaded.max_steps == 20 and loaded.stages[0].block_size == 16
    assert got["sha256"] == loaded.sha256()
    write_curriculum(out, fixed_curriculum("2", block_size=16, steps_per_epoch=10, global_batch_size=4,
                                           sequence_length=64))  # the same plan: kept
    with pytest.raises(FileExistsError):
        write_curriculum(out, fixed_curriculum("3", block_size=16, steps_per_epoch=10, global_batch_size=4,
                                               sequence_length=64))


def test_training_cli_accepts_the_reference_option_names(tmp_path):
    """``training/train.py`` spellings and a DeepSpeed config drive the same trainer."""
    import json

    from uno_b200.train.__main__ import main

    ds = tmp_path / "zero2.json"
    ds.write_text(json.dumps({"zero_optimization": {"stage": 2}, "gradient_clipping": 0.5,
                              "train_micro_batch_size_per_gpu": "auto", "gradient_accumulation_steps": "auto"}))
    out = tmp_path / "run"
    hist = main(["--model", "preset:tiny-qwen3", "--output-dir", str(out), "--device", "cpu", "--block-sizes", "4",
                 "--steps-per-stage", "2", "--seq-len", "32", "--lora-rank", "8", "--learning-rate", "2e-4",
                 "--per-device-batch-size", "1", "--gradient-accumulation-steps", "2", "--dataset-path", "synthetic",
                 "--tv-gamma", "1.0", "--kl-beta", "0.5", "--ce-alpha", "0.1", "--run-name", "ref-names",
                 "--logging-steps", "5", "--deepspeed", str(ds), "--wandb-mode", "offline", "--local_rank", "0"])
    assert [m["step"] for m in hist] == [1, 2]
    logged = [json.loads(x) for x in (out / "metrics.jsonl").read_text().splitlines()]
    assert [m["step"] for m in logged] == [1, 2]
    manifest = json.loads(next(out.glob("*manifest*.json")).read_text())
    assert manifest["run_name"] == "ref-names"
    assert manifest["deepspeed_config"]["applied"] == {"max_grad_norm": 0.5, "zero_stage": 2}
    obj = manifest["compatibility"]["objective"]
    assert (obj["tv_weight"], obj["kl_weight"], obj["ce_weight"]) == (1.0, 0.5, 0.1)
    with pytest.raises(SystemExit, match="dropout"):
        main(["--model", "preset:tiny-qwen3", "--output-dir", str(tmp_path / "r2"), "--device", "cpu",
              "--lora-dropout", "0.05"])


def test_released_curriculum_schedule(tmp_path):
    """Six half-epoch stages over three epochs: 28,125 steps, 14.7456 B tokens, 4,688 / 4,687 alternating."""
    from uno_b200.train.curriculum import BlockCurriculumPlan, released_curriculum
    from uno_b200.train.make_curriculum import main as make_curriculum

    plan = BlockCurriculumPlan.from_mapping(released_curriculum())
    assert plan.max_steps == 28125 and plan.total_tokens == 14_745_600_000
    assert [s.block_size for s in plan.stages] == [2, 4, 6, 8, 12, 16]
    assert [s.end_step - s.start_step for s in plan.stages] == [4688, 4687] * 3
    assert plan.stage_for_step(4687).block_size == 2 and plan.stage_for_step(4688).block_size == 4
    out = make_curriculum(["released", "--output", str(tmp_path / "released.yaml")])
    assert out["max_steps"] == 28125 and BlockCurriculumPlan.from_yaml(tmp_path / "released.yaml").sha256() == \
        plan.sha256()


def test_learning_rate_schedules():
    import pytest

    from uno_b200.train.trainer import lr_at

    # warmup from zero, then constant (the released recipe's warmup-stable schedule without decay)
    assert [lr_at(s, 1.0, 4, 100) for s in range(6)] == [0.0, 0.25, 0.5, 0.75, 1.0, 1.0]
    assert lr_at(99, 1.0, 4, 100) == 1.0
    assert lr_at(4, 1.0, 4, 100, "cosine") == 1.0 and lr_at(100, 1.0, 4, 100, "cosine") == pytest.approx(0.0)
    with pytest.raises(ValueError):
        lr_at(10, 1.0, 4, 100, "linear")


def test_training_data_from_prepared_directories(tmp_path):
    """``--data DIR`` works for rows.jsonl directories and for ``datasets`` directories saved by the
    reference preparer, and the run manifest fingerprints the directory's files."""
    import json

    from datasets import Dataset

    from uno_b200.train.data import data_manifest, load_jsonl

    rows = [{"input_ids": [5, 6, 7], "labels": [-100, 6, 7]}, {"input_ids": [8, 9, 10], "labels": [8, 9, 10]}]
    mine = tmp_path / "mine"
    mine.mkdir()
    (mine / "rows.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    (mine / "uno_dataset_manifest.json").write_text(json.dumps({"hash": {"content_sha256": "abc"}}))
    theirs = tmp_path / "theirs"
    Dataset.from_list(rows).save_to_disk(str(theirs))
    assert load_jsonl(mine) == rows and load_jsonl(theirs) == rows
    m = data_manifest([mine])
    assert m["corpus_hash"] == {"content_sha256": "abc"} and {f["path"] for f in m["files"]} >= {"rows.jsonl"}
    assert data_manifest([theirs])["files"]


def test_prepared_rows_are_padded_one_per_sequence(tmp_path):
    import json

    import pytest

    from uno_b200.train.__main__ import main
    from uno_b200.train.data import pad_rows

    rows = [{"input_ids": [5, 6, 7], "labels": [-100, 6, 7]}, {"input_ids": [8, 9], "labels": [8, 9]}]
    seqs = pad_rows(rows, 4, pad_id=0)
    assert [s["input_ids"].tolist() for s in seqs] == [[5, 6, 7, 0], [8, 9, 0, 0]]
    assert [s["labels"].tolist() for s in seqs] == [[-100, 6, 7, -100], [8, 9, -100, -100]]
    with pytest.raises(ValueError, match="sequence length"):
        pad_rows(rows, 2)
    data = tmp_path / "rows.jsonl"
    data.write_text("".join(json.dumps({"input_ids": [7 + i % 50] * 40, "labels": [7 + i % 50] * 40}) + "\n"
                            for i in range(8)))
    hist = main(["--model", "preset:tiny-qwen3", "--output-dir", str(tmp_path / "run"), "--device", "cpu",
                 "--data", str(data), "--block-sizes", "4", "--steps-per-stage", "2", "--seq-len", "64",
                 "--global-batch", "2", "--lora-rank", "8"])
    assert [m["step"] for m in hist] == [1, 2] and all(m["tokens"] > 0 for m in hist)
    man = json.loads((tmp_path / "run" / "uno_training_manifest.json").read_text())
    assert man["compatibility"]["data"]["collation"] == "pad"


def test_wandb_reporting_and_credential_check(tmp_path, monkeypatch):
    import json
    import sys
    import types

    import pytest

    from uno_b200.train.__main__ import main
    from uno_b200.train.metrics_sink import check_wandb, wandb_credentials_present

    calls = []

    class Run:
        def log(self, row, step):
            calls.append(("log", step, sorted(row)))

        def finish(self):
            calls.append(("finish",))

    fake = types.ModuleType("wandb")
    fake.init = lambda **kw: calls.append(("init", kw["project"], kw["mode"], kw["name"])) or Run()
    monkeypatch.setitem(sys.modules, "wandb", fake)
    env = {"NETRC": str(tmp_path / "no-netrc")}
    assert not wandb_credentials_present(env)
    with pytest.raises(SystemExit, match="credentials"):
        check_wandb("online", env)
    (tmp_path / "netrc").write_text("machine api.wandb.ai login user password k3y\n")
    assert wandb_credentials_present({"NETRC": str(tmp_path / "netrc")})
    assert wandb_credentials_present({"WANDB_API_KEY": "x", **env})
    monkeypatch.delitem(sys.modules, "wandb")
    monkeypatch.setattr("builtins.__import__", _refuse_wandb(__import__))
    with pytest.raises(SystemExit, match="wandb package"):
        check_wandb("offline", env)
    monkeypatch.undo()
    monkeypatch.setitem(sys.modules, "wandb", fake)
    out = tmp_path / "run"
    main(["--model", "preset:tiny-qwen3", "--output-dir", str(out), "--device", "cpu", "--block-sizes", "4",
          "--steps-per-stage", "2", "--seq-len", "32", "--global-batch", "2", "--lora-rank", "8",
          "--wandb-mode", "offline", "--wandb-project", "p", "--run-name", "r1"])
    assert calls[0] == ("init", "p", "offline", "r1") and calls[-1] == ("finish",)
    assert [c[1] for c in calls if c[0] == "log"] == [1, 2]
    assert "train/loss" in calls[1][2]
    man = json.loads((out / "uno_training_manifest.json").read_text())
    assert man["wandb"] == {"project": "p", "mode": "offline"}


def _refuse_wandb(real_import):
    def guarded(name, *args, **kwargs):
        if name == "wandb":
            raise ImportError("no wandb")
        return real_import(name, *args, **kwargs)
    return guarded


def test_slurm_launcher_dry_run(tmp_path):
    import os
    import subprocess

    script = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "uno_b200", "train",
                          "run_slurm.sh")
    env = {k: v for k, v in os.environ.items() if not k.startswith(("SLURM_", "WANDB_", "UNO_"))}
    env.update(MODEL="preset:tiny-qwen3", DATA="synthetic", OUTPUT_ROOT=str(tmp_path), RUN_NAME="r1", DRY_RUN="1")
    sub = subprocess.run(["bash", script], env=env, capture_output=True, text=True, timeout=60)
    assert sub.returncode == 0, sub.stderr
    assert sub.stdout.startswith("sbatch ") and "--nodes=2" in sub.stdout and "--job-name=r1" in sub.stdout
    env.update(UNO_NODE_WORKER="1", SLURM_NNODES="2", SLURM_PROCID="1", MASTER_ADDR="127.0.0.1", MASTER_PORT="29500",
               WANDB_MODE="disabled", SLURM_TMPDIR=str(tmp_path))
    sub = subprocess.run(["bash", script], env=env, capture_output=True, text=True, timeout=60)
    assert sub.returncode == 0, sub.stderr
    cmd = sub.stdout.strip().splitlines()[-1].split()
    assert cmd[1:3] == ["-m", "torch.distributed.run"] and "--node-rank=1" in cmd and "--nproc-per-node=8" in cmd
    for flag, value in (("--global-batch", "128"), ("--seq-len", "4096"), ("--lr", "1e-5"), ("--warmup-steps", "562"),
                        ("--curriculum", "released"), ("--run-name", "r1"), ("--wandb-mode", "disabled"),
                        ("--lora-rank", "128")):
        assert cmd[cmd.index(flag) + 1] == value, flag


def test_training_recipe_dry_run_uses_the_released_settings():
    import os
    import subprocess

    from uno_b200.train.__main__ import build_parser

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = {k: v for k, v in os.environ.items() if not k.startswith(("SLURM_", "NODES", "CURRICULUM", "LORA_", "LR"))}
    env.update(DRY_RUN="1", RUN_NAME="r")
    out = subprocess.run(["bash", os.path.join(root, "examples", "uno_qwen3_8B", "run_train.sh"), "--max-steps", "2"],
                         env=env, capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    cmd = out.stdout.split()
    args = build_parser().parse_args(cmd[cmd.index("uno_b200.train") + 1:])
    assert (args.lora_rank, args.lora_alpha, args.lr, args.warmup_steps, args.global_batch, args.curriculum) == \
        (128, 2048, 1e-5, 562, 128, "released")
    assert args.max_steps == 2 and args.fsdp
