"""Evaluation stack on CPU: parsers, graders, protocol guard, runner with resume, pull suite."""

import json
import multiprocessing as mp
import os
import socket
import threading

import pytest

from uno_b200.eval import benchmarks, graders, parsers


def test_registry_and_aliases():
    assert len(benchmarks.list_benchmarks()) == 13
    assert benchmarks.get_benchmark("AA-LCR").task == "aa_lcr"
    assert benchmarks.get_benchmark("gpqa-diamond").temperature == 0.6
    with pytest.raises(KeyError, match="Unknown benchmark"):
        benchmarks.get_benchmark("nope")


def test_parsers():
    assert parsers.last_boxed(r"so \boxed{\frac{1}{2}} then \boxed{x^{2}+1}") == "x^{2}+1"
    assert parsers.last_boxed("no box") is None
    assert parsers.extract_mc_answer("<think>maybe A</think>The answer is (C).") == "C"
    assert parsers.extract_mc_answer(r"... \boxed{B}") == "B"
    assert parsers.extract_mc_answer(r"... \boxed{\text{B}}") is None  # the protocol reads bare boxed letters only
    assert parsers.extract_mc_answer("<answer>(2)</answer>") == "B" and parsers.extract_mc_answer("Final answer: **E**") == "E"
    assert parsers.extract_mc_answer("<think>x</think>\nB. because") == "B"
    assert parsers.extract_mc_answer("Reasoning...\nD") == "D"
    code = "text\n```python\ndef f(x):\n    return x + 1\n```\nmore"
    assert parsers.extract_code(code) == "def f(x):\n    return x + 1\n"
    with pytest.raises(ValueError):
        parsers.parse_generation("nope", "x")


@pytest.mark.parametrize("pred,truth,ok", [
    (r"\frac{1}{2}", "0.5", True), ("1,000", "1000", True), (r"\dfrac{\sqrt{2}}{2}", r"\frac{\sqrt{2}}{2}", True),
    ("x = 3", "3", True), ("2\\pi", "6.283185307", True), ("7", "8", False), ("", "1", False),
])
def test_math_equivalence(pred, truth, ok):
    assert graders.math_equal(pred, truth) is ok


def test_grade_math_and_mc():
    assert graders.grade_math(r"<think>hmm</think> result \boxed{42}", 42)["correct"]
    assert graders.grade_multiple_choice("b", "B")["correct"]
    assert not graders.grade_multiple_choice(None, "B")["correct"]


def test_code_sandbox():
    ok = graders.grade_code("def add(a, b):\n    return a + b", {"test_list": ["assert add(1, 2) == 3"]})
    bad = graders.grade_code("def add(a, b):\n    return a - b", {"test_list": ["assert add(1, 2) == 3"]})
    he = graders.grade_code("def inc(x):\n    return x + 1", {"prompt": "", "entry_point": "inc",
                                                            "test": "def check(f):\n    assert f(1) == 2"})
    slow = graders.run_code_sandboxed("while True:\n    pass\n", timeout=1.0)
    env = graders.run_code_sandboxed("import os, sys\nsys.exit(0 if 'HF_TOKEN' not in os.environ else 1)\n")
    assert ok["correct"] and not bad["correct"] and he["correct"]
    assert slow["status"] == "timeout" and env["passed"]


def test_llm_judge_with_fake_transport():
    seen = {}

    def transport(payload):
        seen.update(payload)
        return "CORRECT"

    res = graders.grade_with_judge("q?", "a", "<think>x</think>final", model="judge-1", transport=transport)
    assert res["correct"] and seen["model"] == "judge-1" and "final" in seen["messages"][0]["content"]


# ------------------------------------------------------------- runner
def _chat_model_dir(tmp_path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    from uno_b200.utils.hf_compat import model_config_from_dict, save_model_config

    words = ["<unk>", "<eos>", "system", "user", "assistant", ":", "what", "is", "two", "plus", "three", "\n"]
    words += [f"w{i}" for i in range(100)]
    tok = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="<unk>", eos_token="<eos>")
    fast.chat_template = ("{% for m in messages %}{{ m['role'] }} : {{ m['content'] }} {% endfor %}"
                          "{% if add_generation_prompt %}assistant : {% endif %}")
    d = tmp_path / "model"
    fast.save_pretrained(str(d))
    save_model_config(model_config_from_dict(dict(
        model_type="qwen3", vocab_size=4096, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=32, eos_token_id=1, mask_token_id=4095,
        torch_dtype="float32")), str(d))
    return d


def _dataset(tmp_path):
    p = tmp_path / "toy.jsonl"
    rows = [{"id": "q1", "chat_input": [{"role": "user", "content": "what is two plus three"}], "answer": "5"},
            {"id": "q2", "chat_input": [{"role": "user", "content": "what is two"}], "answer": "2"}]
    p.write_text("".join(json.dumps(r) + "\n" for r in rows))
    return p


def test_eval_runner_generates_resumes_and_scores(tmp_path):
    from uno_b200.eval.run import main

    model = _chat_model_dir(tmp_path)
    data = _dataset(tmp_path)
    out = tmp_path / "toy-generations.jsonl"
    common = ["--model", str(model), "--data", str(data), "--output", str(out), "--device", "cpu",
              "--load-format", "dummy", "--num-samples", "2", "--max-tokens", "12", "--max-model-len", "128",
              "--diffusion-block-size", "4", "--temperature", "1.0", "--seed", "0"]
    s1 = main(common)
    rows = [json.loads(x) for x in out.read_text().splitlines()]
    assert s1["generated"] == 4 and len(rows) == 4
    assert [(r["id"], r["sample"]) for r in rows] == [("q1", 0), ("q1", 1), ("q2", 0), ("q2", 1)]
    assert s1["decoder_tokens_per_sequence_forward"] > 0 and s1["scores"]["rows"] == 4
    assert (tmp_path / "scores.json").is_file() and (tmp_path / "grades.jsonl").is_file()
    s2 = main(common)  # resume: nothing left to generate
    assert s2["generated"] == 0 and s2["resumed"] == 4 and len(out.read_text().splitlines()) == 4


def test_protocol_overrides_need_an_arm(tmp_path):
    from uno_b200.eval.run import main

    model = _chat_model_dir(tmp_path)
    data = _dataset(tmp_path)
    args = ["--benchmark", "math500", "--model", str(model), "--data", str(data), "--device", "cpu",
            "--load-format", "dummy", "--output", str(tmp_path / "m.jsonl"), "--no-grade"]
    with pytest.raises(ValueError, match="protocol-arm"):
        main(args)  # the toy file is not the pinned math500 artifact
    s = main(args + ["--protocol-arm", "toy", "--skip-row-count-check", "--max-tokens", "4",
                     "--max-model-len", "128", "--diffusion-block-size", "4"])
    assert set(s["overrides"]) >= {"data", "max_tokens", "max_model_len"} and s["protocol_arm"] == "toy"


# ---------------------------------------------------------- pull suite
def _fake_generate(jobs):
    return [f"gen {j['id']} {j['sample']}" for j in jobs]


def _worker(port, manifest, box):
    from uno_b200.eval.pull_suite import run_worker

    try:
        box.put(("ok", run_worker(("127.0.0.1", port), b"k", manifest, _fake_generate, batch=3,
                                  connect_deadline=30)))
    except Exception as exc:  # report to the parent
        box.put(("err", repr(exc)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_pull_suite_distributes_resumes_and_guards_manifest(tmp_path):
    from uno_b200.eval.pull_suite import completed_keys, run_coordinator

    ctx = mp.get_context("spawn")  # forked children of a process with torch threads can deadlock
    manifest = {"model": "toy", "protocol": "p1"}
    jobs = [{"benchmark": "toy", "id": f"q{i}", "sample": s, "ground_truth": str(i)} for i in range(7) for s in (0, 1)]
    results = tmp_path / "results.jsonl"
    # two jobs finished in an earlier, interrupted run
    results.write_text("".join(json.dumps({**jobs[k], "generation": "old"}) + "\n" for k in (0, 5)))
    port = _port()
    box = ctx.Queue()
    summary = {}

    def coord():
        summary.update(run_coordinator(jobs, results, manifest, ("127.0.0.1", port), b"k", num_workers=2,
                                       timeout=60))

    t = threading.Thread(target=coord)
    t.start()
    workers = [ctx.Process(target=_worker, args=(port, manifest, box)) for _ in range(2)]
    for w in workers:
        w.start()
    for w in workers:
        w.join(60)
    t.join(60)
    outcomes = [box.get(timeout=5) for _ in workers]
    assert all(o[0] == "ok" for o in outcomes), outcomes
    assert summary["resumed"] == 2 and summary["completed"] == 12
    assert sum(o[1] for o in outcomes) == 12
    lines = [json.loads(x) for x in results.read_text().splitlines()]
    assert len(lines) == 14 and len(completed_keys(results)) == 14

    # a worker with a different manifest is refused
    port2 = _port()
    seen = {}

    def coord2():
        try:
            run_coordinator(jobs[:1], tmp_path / "r2.jsonl", manifest, ("127.0.0.1", port2), b"k", num_workers=1,
                            timeout=8)
        except TimeoutError as exc:  # its only worker was refused, so the job never finishes
            seen["timeout"] = str(exc)

    t2 = threading.Thread(target=coord2)
    t2.start()
    bad = ctx.Process(target=_worker, args=(port2, {"model": "other"}, box))
    bad.start()
    bad.join(30)
    kind, msg = box.get(timeout=5)
    assert kind == "err" and "manifest mismatch" in msg
    t2.join(30)
    assert "1 jobs unfinished" in seen.get("timeout", "")


# ------------------------------------------------------------------ ifeval
@pytest.mark.parametrize("iid,kwargs,good,bad", [
    ("keywords:existence", {"keywords": ["apple", "pie"]}, "An apple Pie.", "An apple."),
    ("keywords:frequency", {"keyword": "cat", "frequency": 2, "relation": "at least"}, "cat CAT", "cat"),
    ("keywords:forbidden_words", {"forbidden_words": ["bad"]}, "badge is fine", "that is bad"),
    ("keywords:letter_frequency", {"letter": "z", "let_frequency": 3, "let_relation": "less than"}, "zz", "zzz"),
    ("language:response_language", {"language": "ru"}, "Привет, как дела?", "Hello there"),
    ("language:response_language", {"language": "de"}, "Das ist nicht der Weg und die Zeit",
     "The way and the time of it"),
    ("length_constraints:number_sentences", {"num_sentences": 3, "relation": "less than"}, "One. Two.",
     "One. Two. Three."),
    ("length_constraints:number_paragraphs", {"num_paragraphs": 2}, "first\n***\nsecond", "only one"),
    ("length_constraints:number_words", {"num_words": 5, "relation": "at least"}, "one two three four five",
     "one two"),
    ("length_constraints:nth_paragraph_first_word",
     {"num_paragraphs": 2, "nth_paragraph": 2, "first_word": "then"}, "First.\n\nThen, more.", "First.\n\nNo."),
    ("detectable_content:number_placeholders", {"num_placeholders": 2}, "[name] at [address]", "[name]"),
    ("detectable_content:postscript", {"postscript_marker": "P.S."}, "Body.\nP.S. hi", "Body only."),
    ("detectable_format:number_bullet_lists", {"num_bullets": 2}, "* a\n* b", "* a\n* b\n* c"),
    ("detectable_format:constrained_response", {}, "My answer is yes.", "Yes."),
    ("detectable_format:number_highlighted_sections", {"num_highlights": 2}, "*one* and *two*", "*one*"),
    ("detectable_format:multiple_sections", {"section_spliter": "Section", "num_sections": 2},
     "Section 1\na\nSection 2\nb", "Section 1\na"),
    ("detectable_format:json_format", {}, '```json\n{"a": 1}\n```', "{a: 1}"),
    ("detectable_format:title", {}, "<<My Title>>\ntext", "no title"),
    ("combination:two_responses", {}, "first answer\n******\nsecond answer", "one answer"),
    ("combination:repeat_prompt", {"prompt_to_repeat": "Say hi"}, "Say hi. Hi!", "Hi!"),
    ("startend:end_checker", {"end_phrase": "Is there anything else?"}, "Done. Is there anything else?", "Done."),
    ("change_case:capital_word_frequency", {"capital_frequency": 2, "capital_relation": "at least"},
     "THIS is VERY good", "This is good"),
    ("change_case:english_capital", {}, "THIS IS ALL CAPS AND THE END", "This is not"),
    ("change_case:english_lowercase", {}, "this is all lower and the end", "This is not"),
    ("punctuation:no_comma", {}, "no commas here", "one, two"),
    ("startend:quotation", {}, '"quoted"', "not quoted"),
])
def test_ifeval_checkers(iid, kwargs, good, bad):
    from uno_b200.eval.ifeval import check

    assert check(iid, good, kwargs) and not check(iid, bad, kwargs)


def test_ifeval_grade_strict_loose_and_scoring(tmp_path):
    from uno_b200.eval.ifeval import grade_ifeval
    from uno_b200.eval.score import grade_row

    truth = {"instruction_id_list": ["punctuation:no_comma", "startend:end_checker"],
             "kwargs": [{}, {"end_phrase": "bye"}]}
    # the trailing sign-off line breaks strict end_checker; loose drops the last line
    gen = "<think>plan, then answer</think>hello there\nbye\n**thanks**"
    g = grade_ifeval(gen, truth)
    assert g["strict_inst_follow"] == [True, False] and not g["strict_prompt_follow"]
    assert g["loose_inst_follow"] == [True, True] and g["loose_prompt_follow"] and g["correct"] is False
    row = {"generation": "hello bye", "ground_truth": truth}
    assert grade_row(row, None, task="ifeval", parser="passthrough")["correct"] is True


def test_lcb_grader_stdin_functional_and_failures():
    import json

    from uno_b200.eval.lcb import extract_python_code, pass_at_k, score_lcb

    assert extract_python_code("text\n```python\nprint(1)\n```\nmore ```py\nprint(2)\n```") == "print(2)"
    assert extract_python_code("no fences") == "no fences"
    stdin = json.dumps([{"input": "3 4\n", "output": "7\n", "testtype": "stdin"},
                        {"input": "1.5 2\n", "output": "3.50\n", "testtype": "stdin"}])
    func = json.dumps([{"input": "[1,2]\n3", "output": "[1, 2, 3]", "testtype": "functional", "method_name": "f"}])
    rows = [
        {"ground_truth": stdin, "generations": [
            "```python\na, b = map(float, input().split())\nr = a + b\nprint(int(r) if r == int(r) else r)\n```",
            "print(5)",                                    # wrong answer
            "```python\nwhile True:\n    pass\n```",       # time limit
            "```python\nraise ValueError()\n```"]},        # runtime error
        {"ground_truth": func, "generation": "class Solution:\n    def f(self, a, b):\n        return tuple(a + [b])\n"},
    ]
    graded, summary = score_lcb(rows, timeout=2, workers=4)
    assert graded[0]["correct"] == [True, False, False, False]
    assert graded[0]["test_results"][1:] == [[-2], [-3], [-4]]
    assert graded[1]["correct"] == [True]
    assert summary["num_correct"] == 2 and abs(summary["pass@1"] - (0.25 + 1.0) / 2) < 1e-9
    assert pass_at_k(5, 0, 1) == 0.0 and pass_at_k(5, 5, 5) == 1.0 and abs(pass_at_k(4, 1, 1) - 0.25) < 1e-12


def test_lcr_grader_parses_json_grade():
    from uno_b200.eval.graders import grade_lcr

    seen = []

    def judge(payload):
        seen.append(payload)
        text = " ".join(m["content"] for m in payload["messages"])
        return 'Reasoning... {"GRADE": "CORRECT"}' if "Paris" in text.split("STUDENT ANSWER:")[-1] else "{}"

    assert grade_lcr("Capital of France?", "<think>hmm</think>Paris", "Paris", transport=judge, model="m")["correct"]
    assert not grade_lcr("Capital of France?", "Lyon", "Lyon is wrong", transport=lambda p: "INCORRECT",
                         model="m")["correct"]
    assert seen[0]["model"] == "m" and seen[0]["messages"][0]["role"] == "system"


def test_prepare_installs_pinned_artifact_and_rejects_mismatch(tmp_path, monkeypatch):
    import hashlib

    from uno_b200.eval import benchmarks as B
    from uno_b200.eval.prepare import prepare_benchmark_data

    body = "".join('{"row": %d, "ground_truth": "1"}\n' % i for i in range(30)).encode()
    sha = hashlib.sha256(body).hexdigest()
    cfg = B.BENCHMARKS["aime24"]
    monkeypatch.setitem(B.BENCHMARKS, "aime24", type(cfg)(**{**cfg.__dict__, "data_sha256": sha}))
    src = tmp_path / "src"
    (src / "aime-2024").mkdir(parents=True)
    (src / "aime-2024" / "aime-2024.jsonl").write_bytes(body)     # repository-shaped bundle
    out = prepare_benchmark_data("aime-24", output_dir=tmp_path / "out", source_dir=src)
    assert out.read_bytes() == body
    assert prepare_benchmark_data("aime24", output_dir=tmp_path / "out") == out   # re-validated, not rebuilt
    (src / "aime24.jsonl").write_bytes(body.replace(b'"1"', b'"2"'))              # flat bundle wins, wrong bytes
    with pytest.raises(ValueError, match="sha256"):
        prepare_benchmark_data("aime24", output_dir=tmp_path / "o2", source_dir=src)


def test_prepare_builders_render_protocol_prompts():
    import base64
    import json
    import pickle
    import zlib

    from uno_b200.eval.prepare import build_gpqa, build_lcb, build_mbpp, decode_lcb_tests, gpqa_order

    row = {"Question": "What is 2+2?", "Correct Answer": "4", "Incorrect Answer 1": "3",
           "Incorrect Answer 2": "5", "Incorrect Answer 3": "22"}
    rec = build_gpqa([row])[0]
    order = gpqa_order(row["Question"])
    assert sorted(order) == [0, 1, 2, 3] and order == gpqa_order(row["Question"])
    assert rec["ground_truth"] == "ABCD"[order.index(0)]
    assert f"{rec['ground_truth']}) 4" in rec["completion_input"]
    shots = [{"task_id": t, "text": f"task {t}", "test_list": [f"assert f{t}()"], "code": f"def f{t}(): return 1"}
             for t in (2, 3, 4)]
    mb = build_mbpp([{"task_id": 11, "text": "do it", "test_list": ["assert g()"]}], shots)[0]
    assert mb["completion_input"].count("[DONE]") == 3 and mb["completion_input"].endswith("assert g()\n[BEGIN]\n")
    tests = [{"input": "1\n", "output": "1\n", "testtype": "stdin"}]
    packed = base64.b64encode(zlib.compress(pickle.dumps(json.dumps(tests)))).decode()
    assert decode_lcb_tests(packed) == tests
    evil = base64.b64encode(zlib.compress(pickle.dumps(OSError("x")))).decode()
    with pytest.raises(pickle.UnpicklingError):
        decode_lcb_tests(evil)
    lcb = build_lcb([{"question_content": "Sum.", "public_test_cases": json.dumps(tests),
                      "private_test_cases": packed, "metadata": json.dumps({"func_name": "f"}), "starter_code": "x"}])[0]
    assert len(json.loads(lcb["ground_truth"])) == 2 and json.loads(lcb["ground_truth"])[0]["method_name"] == "f"
    assert lcb["chat_input"][0]["role"] == "system" and "```python\nx\n```" in lcb["chat_input"][1]["content"]


def test_pull_suite_jobs_manifest_and_scoring(tmp_path):
    """``jobs`` expands a registered benchmark with the canonical prompt rendering and budgets;
    ``score`` splits the results per benchmark and grades them."""
    from uno_b200.eval.benchmarks import get_benchmark
    from uno_b200.eval.pull_suite import build_jobs, score_results, suite_sampling
    from uno_b200.utils.hf_compat import load_model_config, load_tokenizer

    model = _chat_model_dir(tmp_path)
    tok = load_tokenizer(str(model), load_model_config(str(model)))
    root = tmp_path / "data"
    root.mkdir()
    bench = get_benchmark("gsm8k")
    (root / bench.data_path.name).write_text(_dataset(tmp_path).read_text())
    jobs, entries = build_jobs(["gsm8k"], tok, data_root=root, context_length=64, reserve=8)
    assert len(jobs) == 2 * bench.num_samples
    assert {(j["id"], j["sample"]) for j in jobs} == {("q1", 0), ("q1", 1), ("q2", 0), ("q2", 1)}
    assert all(j["max_tokens"] == 64 - len(j["prompt_ids"]) - 8 for j in jobs)
    assert entries[0]["rows"] == 2 and entries[0]["num_samples"] == bench.num_samples
    assert suite_sampling(entries) == {"temperature": 1.0, "top_p": 0.95, "top_k": None}
    assert suite_sampling(entries, {"top_p": 0.5})["top_p"] == 0.5
    # a prompt longer than the context gets no job
    short, e2 = build_jobs(["gsm8k"], tok, data_root=root, context_length=12, reserve=8)
    assert short == [] and e2[0]["skipped_no_budget"] == 2
    results = tmp_path / "results.jsonl"
    results.write_text("".join(json.dumps({"benchmark": "gsm8k", "id": j["id"], "sample": j["sample"],
                                           "generation": "so \\boxed{5}", "ground_truth": j["ground_truth"]}) + "\n"
                               for j in jobs))
    summary = score_results(results, {"benchmarks": entries}, tmp_path / "run")
    assert summary["gsm8k"]["rows"] == 4 and summary["gsm8k"]["accuracy"] == 0.5  # q1 (5) right, q2 (2) wrong
    assert (tmp_path / "run" / "gsm8k" / "scores.json").is_file()


def test_suite_launchers_dry_run(tmp_path):
    """The suite and Slurm launchers print their commands under DRY_RUN=1 and run nothing."""
    import subprocess

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    base = dict(os.environ, DRY_RUN="1", MODEL="preset:tiny-qwen3", RESULTS_ROOT=str(tmp_path / "results"))

    def run(script, **env):
        out = subprocess.run(["bash", os.path.join(root, "uno_b200", "eval", script)], env={**base, **env},
                             capture_output=True, text=True, timeout=120)
        assert out.returncode == 0, out.stderr
        return out.stdout.splitlines()

    lines = run("run_suite.sh", BENCHMARKS="gsm8k math500")
    assert len(lines) == 2 and lines[0].startswith("run:") and "BENCHMARKS=gsm8k" in lines[0]
    lines = run("submit_suite.sh", BENCHMARKS="gsm8k aime25", SBATCH_ARGS="--partition=p1")
    assert len(lines) == 2 and all("sbatch" in ln and "--partition=p1" in ln for ln in lines)
    lines = run("submit_pull_suite.sh", BENCHMARKS="ifeval")
    assert len(lines) == 1 and "run_pull_suite_slurm.sh" in lines[0] and "BENCHMARKS=ifeval" in lines[0]
    lines = run("run_pull_suite_slurm.sh", BENCHMARKS="gsm8k", SLURM_JOB_ID="77", SLURM_NNODES="2",
                SLURM_NTASKS="16", TOP_P="0.9")
    roles = [ln.split(":", 1)[0] for ln in lines]
    assert roles == ["jobs", "coord", "worker", "score"]
    assert "--top-p 0.9" in lines[0] and "--num-workers 16" in lines[1] and "--ntasks=16" in lines[2]
    assert not (tmp_path / "results").exists()  # a dry run writes nothing


def test_eval_runner_grades_judge_benchmarks_through_an_endpoint(tmp_path):
    """``--judge-base-url`` / ``--judge-model`` reach the grader: an OpenAI-compatible stub judge
    on 127.0.0.1 sees the benchmark's judge request and its verdict lands in the scores."""
    from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

    from uno_b200.eval.run import main

    seen = []

    class Judge(BaseHTTPRequestHandler):
        def do_POST(self):  # noqa: N802 - http.server API
            body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
            seen.append((self.path, body["model"], self.headers.get("Authorization"), body))
            reply = json.dumps({"choices": [{"message": {"content": "extracted_final_answer: 5\ncorrect: yes"}}]}
                               ).encode()
            self.send_response(200)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(reply)))
            self.end_headers()
            self.wfile.write(reply)

        def log_message(self, *args):
            pass

    server = ThreadingHTTPServer(("127.0.0.1", 0), Judge)
    threading.Thread(target=server.serve_forever, daemon=True).start()
    try:
        model = _chat_model_dir(tmp_path)
        data = _dataset(tmp_path)
        s = main(["--benchmark", "hle", "--model", str(model), "--data", str(data), "--device", "cpu",
                  "--load-format", "dummy", "--output", str(tmp_path / "hle.jsonl"), "--protocol-arm", "toy",
                  "--skip-row-count-check", "--num-samples", "1", "--max-tokens", "4", "--max-model-len", "128",
                  "--diffusion-block-size", "4", "--seed", "0",
                  "--judge-base-url", f"http://127.0.0.1:{server.server_port}", "--judge-model", "stub-judge",
                  "--judge-api-key", "k1", "--judge-temperature", "0.3", "--judge-max-tokens", "77",
                  "--judge-reasoning-effort", "low", "--judge-max-concurrency", "2", "--save-token-ids",
                  "--no-progress", "--grades", str(tmp_path / "g.jsonl"), "--scores", str(tmp_path / "s.json")])
    finally:
        server.shutdown()
    assert s["scores"]["graded"] == 2 and s["scores"]["num_correct"] == 2
    assert s["scores"]["fixed_denominator"] == 2158  # HLE's question count: the toy rows are 2 of them
    assert seen and all(p == "/v1/chat/completions" and m == "stub-judge" and a == "Bearer k1"
                        for p, m, a, _ in seen)
    assert all(b["temperature"] == 0.3 and b["max_tokens"] == 77 and b["reasoning_effort"] == "low"
               for *_, b in seen)
    rows = [json.loads(x) for x in (tmp_path / "hle.jsonl").read_text().splitlines()]
    assert all(len(r["token_ids"]) == r["token_count"] for r in rows)
    assert (tmp_path / "g.jsonl").is_file() and json.loads((tmp_path / "s.json").read_text())["graded"] == 2


def test_score_cli_grades_a_generations_file(tmp_path):
    from uno_b200.eval.score import main

    gen = tmp_path / "gens.jsonl"
    gen.write_text("".join(json.dumps(r) + "\n" for r in (
        {"id": "a", "sample": 0, "generation": "thus \\boxed{12}", "ground_truth": "12"},
        {"id": "a", "sample": 1, "generation": "thus \\boxed{13}", "ground_truth": "12"},
        {"id": "b", "sample": 0, "generation": "\\boxed{\\frac{1}{2}}", "ground_truth": "0.5"})))
    scores = main(["--generations", str(gen), "--task", "math", "--grader-num-processes", "2",
                   "--scores", str(tmp_path / "sc.json")])
    assert scores["rows"] == 3 and abs(scores["accuracy"] - 2 / 3) < 1e-9
    assert scores["question_accuracy"] == 0.75  # a: 1/2, b: 1/1
    assert (tmp_path / "grades.jsonl").is_file() and json.loads((tmp_path / "sc.json").read_text())["rows"] == 3


def test_reference_parser_names():
    from uno_b200.eval.parsers import parse_generation

    assert parse_generation("gpqa_answer", "<think>A or B or C?</think>\nThe answer is **(C)**") == "C"
    assert parse_generation("gpqa_answer", "ANSWER: b") == "B"
    assert parse_generation("gpqa_answer", "so \\boxed{D}") == "D"
    assert parse_generation("gpqa_answer", "I pick **B**") == "B"
    assert parse_generation("gpqa_answer", "no letter here") == "?" and parse_generation("gpqa_answer", "") == "?"
    assert parse_generation("mmlu_pro_answer", "The answer is (J).") == "J"
    assert parse_generation("mmlu_pro_answer", "reasoning\nE.\n") == "E"
    assert parse_generation("mmlu_pro_answer", "Answer: (G)") == "G"
    chan = ("<|channel|>analysis<|message|>thinking<|channel|>final<|message|>"
            "```python\ndef f(x):\n    return x\nprint(f(2))\n```<|end|>")
    assert parse_generation("lcb_code", chan) == "def f(x):\n    return x"
    assert parse_generation("lcb_code", "import sys\n\ndef main():\n    pass\n\nmain()\nprose") == \
        "import sys\n\ndef main():\n    pass"
    assert parse_generation("lcb_code", "just words") is None
    assert parse_generation("identity", " x ") == " x " and parse_generation("noop", None) is None
    assert parse_generation("multiple_choice_answer", "The answer is B") == "B"
    assert parse_generation("humaneval", "```python\nx = 1\n```") == "x = 1\n"


def test_choice_parser_routes_to_multiple_choice_grading():
    from uno_b200.eval.score import grade_row

    row = {"generation": "<think>hmm</think> ANSWER: C", "ground_truth": "C"}
    assert grade_row(row, None, task="gpqa_diamond", parser="gpqa_answer")["correct"] is True
    assert grade_row({**row, "ground_truth": "A"}, None, task="gpqa_diamond", parser="gpqa_answer")["correct"] is False


def test_judge_protocols_hle_omniscience_lcr(tmp_path):
    """Per-benchmark judge prompts and verdicts; HLE letter questions skip the judge; the
    AA-Omniscience scores are its accuracy, non-hallucination rate and index over 600 questions."""
    from uno_b200.eval.graders import judge_messages, parse_verdict
    from uno_b200.eval.score import score_file

    assert parse_verdict("hle", "<think>x</think>extracted_final_answer: 7\ncorrect: yes\nconfidence: 90") == 1
    assert parse_verdict("hle", "correct: no") == 0
    assert [parse_verdict("aa_omniscience", r) for r in ("A", "B", "C", "D", "")] == [1, -1, 0, 0, 0]
    assert parse_verdict("aa_lcr", '{"answer": {"GRADE": "correct"}}') == 1 and parse_verdict("aa_lcr", "INCORRECT") == 0
    msgs = judge_messages("aa_lcr", "docs...\n=== QUESTION ===\nWho?\n\nAnswer:", "Ann", "Ann")
    assert msgs[0]["role"] == "system" and "QUESTION: Who?\n" in msgs[1]["content"]
    assert "[correct_answer]: 42" in judge_messages("hle", "q", 42, "r")[0]["content"]

    data = tmp_path / "omni.jsonl"
    data.write_text("".join(json.dumps({"id": f"o{i}", "completion_input": f"question {i}", "ground_truth": "x"}) + "\n"
                            for i in range(4)))
    gens = tmp_path / "gens.jsonl"
    gens.write_text("".join(json.dumps({"id": f"o{i}", "sample": 0, "generation": f"g{i}", "ground_truth": "x"}) + "\n"
                            for i in range(4)))
    verdicts = {"question 0": "A", "question 1": "B", "question 2": "C", "question 3": "A"}

    def judge(payload):
        text = payload["messages"][-1]["content"]
        return next(v for q, v in verdicts.items() if f"Question: {q}\n" in text)

    scores = score_file(gens, benchmark="omniscience", data=data, judge=judge, judge_model="j")
    assert scores["num_correct"] == 2 and scores["num_incorrect"] == 1
    assert scores["omniscience_index"] == (2 - 1) / 600 and scores["non_hallucination_rate"] == 1 - 1 / 600

    hle = tmp_path / "hle.jsonl"
    hle.write_text(json.dumps({"id": "h", "completion_input": "pick", "ground_truth": "C",
                               "answer_type": "multipleChoice"}) + "\n")
    hg = tmp_path / "hg.jsonl"
    hg.write_text(json.dumps({"id": "h", "sample": 0, "generation": "The answer is C", "ground_truth": "C"}) + "\n")
    assert score_file(hg, benchmark="hle", data=hle, judge=None)["num_correct"] == 1  # graded without a judge


def test_protocol_math_grading():
    from uno_b200.eval import math_grading
    from uno_b200.eval.graders import grade_math

    if not math_grading.available():
        pytest.skip("math_verify is not installed")
    for gen, truth, ok in (("so \\boxed{12}", "12", True), ("thus \\boxed{\\frac{1}{2}}", "0.5", True),
                           ("\\boxed{\\dfrac{3}{4}}", "\\frac{3}{4}", True), ("The answer is 42.", "42", True),
                           ("#### 1,234", "1234", True), ("<think>\\boxed{9}</think> so 9", "9", True),
                           ("\\boxed{5 cm}", "5", True), ("\\boxed{13}", "12", False), ("The answer is 7", "8", False)):
        assert grade_math(gen, truth)["correct"] is ok, (gen, truth)
    assert math_grading.normalise_answer("\\left( 1{,}000 \\right)") == "(1000)"


def test_protocol_code_grading_on_prepared_records(tmp_path):
    """HumanEval and MBPP rows in the prepared format (tests in ground_truth, the prompt in
    completion_input) grade through score_file with the protocol's program assembly."""
    from uno_b200.eval.code_grading import extract_mbpp_code
    from uno_b200.eval.score import score_file

    prompt = 'def inc(x):\n    """Add one."""\n'
    he = tmp_path / "he.jsonl"
    he.write_text(json.dumps({"id": "h0", "completion_input": prompt,
                              "ground_truth": {"test": "def check(candidate):\n    assert candidate(2) == 3\n",
                                               "entry_point": "inc"}}) + "\n")
    gens = ["    return x + 1\n",                                   # body only
            "def inc(y):\n    return y + 1\n",                      # whole function, renamed parameter
            "<think>easy</think>\n```python\ndef inc(x):\n    return x + 1\n```",  # fenced after reasoning
            "    return x\n"]                                        # wrong
    hg = tmp_path / "hg.jsonl"
    hg.write_text("".join(json.dumps({"id": "h0", "sample": i, "generation": g}) + "\n" for i, g in enumerate(gens)))
    he_scores = score_file(hg, benchmark="humaneval", data=he, grades_out=tmp_path / "hgr.jsonl")
    grades = [json.loads(x)["correct"] for x in (tmp_path / "hgr.jsonl").read_text().splitlines()]
    assert grades == [True, True, True, False] and he_scores["accuracy"] == 0.75

    tests = "assert add(1, 2) == 3"
    assert extract_mbpp_code("```python\ndef helper():\n    pass\n```\n```python\ndef add(a, b):\n    return a + b\n```",
                             tests).startswith("def add")
    mb = tmp_path / "mb.jsonl"
    mb.write_text(json.dumps({"id": "m0", "completion_input": "task", "ground_truth": tests}) + "\n")
    mg = tmp_path / "mg.jsonl"
    mg.write_text("".join(json.dumps({"id": "m0", "sample": i, "generation": g}) + "\n" for i, g in enumerate(
        ["Here:\n```python\ndef add(a, b):\n    return a + b\n```\n[DONE]", "[BEGIN]\ndef add(a, b):\n    return a - b\n[DONE]"])))
    assert score_file(mg, benchmark="mbpp", data=mb)["accuracy"] == 0.5


def test_scorer_reads_reference_runner_rows(tmp_path):
    """Rows written by the reference runner (record:sampleN ids, source_row / sample_index, or a
    generations list) grade like this framework's own rows."""
    from uno_b200.eval.score import score_file

    gens = tmp_path / "ref.jsonl"
    gens.write_text("".join(json.dumps(r) + "\n" for r in (
        {"id": "q1:sample0", "source_row": "q1", "sample_index": 0, "generation": "\\boxed{5}", "ground_truth": "5"},
        {"id": "q1:sample1", "source_row": "q1", "sample_index": 1, "generation": "\\boxed{6}", "ground_truth": "5"},
        {"source_row": "q2", "generations": ["\\boxed{2}", "\\boxed{2}"], "ground_truth": "2"})))
    scores = score_file(gens, task="math", grades_out=tmp_path / "g.jsonl")
    assert scores["rows"] == 4 and scores["accuracy"] == 0.75 and scores["question_accuracy"] == 0.75
    ids = [(json.loads(x)["id"], json.loads(x)["sample"]) for x in (tmp_path / "g.jsonl").read_text().splitlines()]
    assert ids == [("q1", 0), ("q1", 1), ("q2", 0), ("q2", 1)]


def test_grouped_pass_at_k():
    from uno_b200.eval.score import grouped_summary, pass_at_k

    assert pass_at_k(5, 0, 1) == 0.0 and pass_at_k(5, 5, 1) == 1.0 and abs(pass_at_k(5, 1, 1) - 0.2) < 1e-12
    assert abs(pass_at_k(5, 1, 5) - 1.0) < 1e-12 and pass_at_k(2, 1, 5) == 1.0  # k capped at n
    s = grouped_summary({"a": [True, False, False, False, False], "b": [False] * 5})
    assert s["num_problems"] == 2 and s["max_samples_per_problem"] == 5
    assert abs(s["pass_at_1"] - 0.1) < 1e-12 and s["pass_at_5"] == 0.5 and "pass_at_10" not in s


def test_fixed_denominator_counts_missing_generations(tmp_path):
    from uno_b200.eval.score import score_file

    gens = tmp_path / "gpqa.jsonl"  # 2 of GPQA-Diamond's 198 x 5 generations, both right
    gens.write_text("".join(json.dumps({"id": f"g{i}", "sample": 0, "generation": "ANSWER: A", "ground_truth": "A"})
                            + "\n" for i in range(2)))
    scores = score_file(gens, benchmark="gpqa_diamond")
    assert scores["fixed_denominator"] == 198 * 5 and scores["accuracy"] == 2 / 990
    summary = tmp_path / "summary.json"
    summary.write_text(json.dumps({"num_samples_per_problem": 1}))
    assert score_file(gens, benchmark="gpqa_diamond", summary=summary)["fixed_denominator"] == 198


def test_pull_suite_settings_from_env_and_canonical_guard(tmp_path):
    import pytest

    from uno_b200.eval.benchmarks import get_benchmark
    from uno_b200.eval.pull_suite import apply_env, build_parser, resolve_suite, worker_settings, \
        write_suite_summary

    def parse(argv, env):
        args = build_parser().parse_args(["jobs", *argv])
        apply_env(args, env)
        return args

    bench = get_benchmark("gsm8k")
    args = parse([], {"NANO_MODEL": "m", "NANO_BENCHMARKS": "gsm8k", "NANO_SAVE_TOKEN_IDS": "1",
                      "NANO_STOP_TOKEN_IDS": "5,6", "NANO_DIFFUSION_BLOCK_SIZE": "8"})
    assert args.model == "m" and args.benchmark == ["gsm8k"] and args.save_token_ids and args.stop_token_ids == [5, 6]
    assert args.diffusion_block_size == 8 and args.tree_candidate_top_k == 16
    assert resolve_suite(args) == {}
    assert (args.num_samples, args.context_length, args.top_p) == (bench.num_samples, bench.max_model_len,
                                                                    bench.top_p)
    assert args.max_num_batched_tokens == bench.max_model_len
    # the command line wins over the environment; a departure needs a protocol arm
    args = parse(["--top-p", "0.5"], {"NANO_BENCHMARKS": "gsm8k", "NANO_TOP_P": "0.7"})
    assert args.top_p == 0.5
    with pytest.raises(SystemExit, match="protocol-arm"):
        resolve_suite(args)
    args = parse(["--top-p", "0.5", "--limit", "3"], {"NANO_BENCHMARKS": "gsm8k", "NANO_PROTOCOL_ARM": "arm-a"})
    assert set(resolve_suite(args)) == {"top_p", "limit"}
    with pytest.raises(SystemExit, match="one benchmark"):
        resolve_suite(parse([], {"NANO_BENCHMARKS": "gsm8k,math500"}))
    args = parse([], {"NANO_BENCHMARKS": "gsm8k math500", "NANO_PROTOCOL_ARM": "uniform"})
    assert resolve_suite(args) == {} and args.max_num_seqs == 64

    manifest = {"model": "m", "diffusion_block_size": 8, "sampling": {"temperature": 0.6, "top_p": 0.95, "top_k": 20},
                "request": {"mask_token_id": 9, "stop_token_ids": [5], "noise_mode": "random_uniform",
                            "noise_salt": None, "ignore_eos": False},
                "engine": {"max_num_seqs": 32, "max_model_len": 4096, "tree_verify_size": None,
                           "cuda_graph_block_sizes": [1, 8]}, "benchmarks": [{"name": "gsm8k"}]}
    sp, kw = worker_settings(manifest, build_parser().parse_args(["worker", "--device", "cpu"]))
    assert (sp.temperature, sp.top_k, sp.mask_token_id, sp.stop_token_ids, sp.diffusion_block_size) == \
        (0.6, 20, 9, [5], 8)
    assert kw["max_num_seqs"] == 32 and kw["max_model_len"] == 4096 and "tree_verify_size" not in kw
    assert kw["device"] == "cpu" and kw["max_diffusion_block_size"] == 8

    path = tmp_path / "suite_summary.json"
    a = write_suite_summary(path, manifest, 4, {"num_generations": 10, "output_tokens": 4000, "elapsed_seconds": 2.0})
    assert a["invocation_output_tokens_per_second_per_gpu"] == 500.0
    b = write_suite_summary(path, manifest, 4, {"num_generations": 0, "output_tokens": 0, "elapsed_seconds": 1.0})
    assert b["generation_invocation_output_tokens_per_second"] == 2000.0 and b["benchmarks"] == ["gsm8k"]
    assert len(json.loads(path.read_text())["invocations"]) == 2


def test_pull_suite_jobs_role_writes_engine_and_request_settings(tmp_path, monkeypatch):
    from uno_b200.eval.benchmarks import get_benchmark
    from uno_b200.eval.pull_suite import main

    model = _chat_model_dir(tmp_path)
    root = tmp_path / "data"
    root.mkdir()
    (root / get_benchmark("gsm8k").data_path.name).write_text(_dataset(tmp_path).read_text())
    monkeypatch.setenv("NANO_RESULTS_ROOT", str(tmp_path / "results"))
    monkeypatch.setenv("NANO_RUN_NAME", "r1")
    monkeypatch.setenv("NANO_BENCHMARKS", "gsm8k")
    monkeypatch.setenv("NANO_MODEL", str(model))
    monkeypatch.setenv("NANO_DATA_ROOT", str(root))
    monkeypatch.setenv("NANO_SAVE_TOKEN_IDS", "true")
    main(["jobs", "--stop-token-ids", "3"])
    run = tmp_path / "results" / "r1"
    man = json.loads((run / "run_manifest.json").read_text())
    assert man["engine"]["max_model_len"] == get_benchmark("gsm8k").max_model_len
    assert man["request"]["stop_token_ids"] == [3] and man["protocol_arm"] is None and man["overrides"] == {}
    jobs = [json.loads(x) for x in (run / "jobs.jsonl").read_text().splitlines()]
    assert jobs and all(j["save_token_ids"] for j in jobs)


def test_eval_runner_replica_default():
    from types import SimpleNamespace

    from uno_b200.eval.run import build_parser, default_replicas

    args = build_parser().parse_args(["--model", "m", "--repetitions", "2"])
    assert args.num_samples == 2 and args.data_parallel_size is None
    assert default_replicas(SimpleNamespace(data_parallel_size=None, device="cpu", tensor_parallel_size=1)) == 1
    assert default_replicas(SimpleNamespace(data_parallel_size=3, device="cuda", tensor_parallel_size=1)) == 3


def test_model_eval_recipes_take_the_benchmark_positionally(tmp_path):
    import subprocess

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = {k: v for k, v in os.environ.items() if k not in ("MODEL", "BENCHMARKS", "DP")}
    env.update(DRY_RUN="1", RESULTS_ROOT=str(tmp_path), RUN_NAME="r", DATA_PARALLEL_SIZE="2")
    for recipe, model in (("uno_qwen3_8B", "s-sahoo/uno-qwen3-8B"), ("uno_8B", "IFM/K2-Horizon-7B"),
                          ("uno_1B", "IFM/K2-Horizon-0.9B")):
        out = subprocess.run(["bash", os.path.join(root, "examples", recipe, "run_eval.sh"), "gsm8k",
                              "--protocol-arm", "a"], env=env, capture_output=True, text=True, timeout=60)
        assert out.returncode == 0, out.stderr
        lines = out.stdout.strip().splitlines()
        assert lines[0].split()[-1] == "gsm8k" and len(lines) == 2, lines
        run = lines[1].split()
        assert run[run.index("--benchmark") + 1] == "gsm8k" and run[run.index("--model") + 1] == model
        assert run[run.index("--data-parallel-size") + 1] == "2" and run[-2:] == ["--protocol-arm", "a"]
    assert not any(tmp_path.iterdir())  # a dry run writes nothing
