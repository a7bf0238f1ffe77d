"""generation / inference applications, hub resolution and token-id rules (CPU)."""

import json
import os

import pytest

from uno_b200.utils.hf_compat import model_config_from_dict, save_model_config


def _tiny_cfg(**kw):
    base = dict(model_type="qwen3", vocab_size=4096, hidden_size=256, intermediate_size=768, num_hidden_layers=2,
                num_attention_heads=4, num_key_value_heads=2, head_dim=64, eos_token_id=7, mask_token_id=4095,
                torch_dtype="float32")
    base.update(kw)
    return model_config_from_dict(base)


def test_inference_cli_runs_end_to_end_on_cpu(capsys):
    from uno_b200.inference import main

    res = main(["--model", "preset:tiny-qwen3", "--device", "cpu", "--prompt-ids", "5,6,7,8,9",
                "--prompt-ids", "11,12,13", "--max-tokens", "16", "--max-model-len", "256",
                "--diffusion-block-size", "4", "--no-progress", "--temperature", "1.0"])
    out = capsys.readouterr().out  # the engine's exit line precedes the JSON document
    printed = json.loads(out[out.index("{"):])
    assert printed["generations"] == res["generations"] and len(res["generations"]) == 2
    assert res["total_output_tokens"] > 0 and res["output_tokens_per_second"] > 0
    # TPF: at least one committed token per two-forward cycle
    assert res["decoder_tokens_per_sequence_forward"] >= 0.5


def _chat_tokenizer(tmp_path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    words = ["<unk>", "<eos>", "system", "user", "assistant", ":", "be", "brief", "hi", "there", "\n"]
    tok = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="<unk>", eos_token="<eos>")
    fast.chat_template = ("{% for m in messages %}{{ m['role'] }} : {{ m['content'] }} {% endfor %}"
                          "{% if add_generation_prompt %}assistant : {% endif %}")
    return fast


def test_format_chat_prompt_merges_instruction(tmp_path):
    from uno_b200.generation import format_chat_prompt

    tok = _chat_tokenizer(tmp_path)
    ids, text, msgs = format_chat_prompt(tok, [{"role": "user", "content": "hi there"}], "be brief")
    assert msgs[0] == {"role": "system", "content": "be brief"}
    assert text == "system : be brief user : hi there assistant : "
    assert ids == tok.encode(text, add_special_tokens=False)
    # an existing system message gets the instruction prepended once
    _, _, msgs2 = format_chat_prompt(tok, [{"role": "system", "content": "hi"}, {"role": "user", "content": "hi"}],
                                     "be brief")
    assert msgs2[0]["content"] == "be brief\n\nhi"
    with pytest.raises(ValueError, match="chat_template"):
        from uno_b200.utils.hf_compat import TokenIdTokenizer

        format_chat_prompt(TokenIdTokenizer(10), [{"role": "user", "content": "x"}])


def test_resolve_model_sources_bundle(tmp_path):
    from uno_b200.generation import resolve_model_sources

    bundle = tmp_path / "bundle"
    (bundle / "adapter").mkdir(parents=True)
    (bundle / "adapter" / "adapter_config.json").write_text("{}")
    model, adapter = resolve_model_sources(str(bundle), None, gated_lora_subfolder="adapter")
    assert model == str(bundle) and adapter == str(bundle / "adapter")
    assert resolve_model_sources("m", "a") == ("m", "a")
    with pytest.raises(ValueError, match="only one"):
        resolve_model_sources(str(bundle), "x", gated_lora_subfolder="adapter")
    with pytest.raises(ValueError, match="invalid"):
        resolve_model_sources(str(bundle), None, gated_lora_subfolder="missing")


def test_hub_resolves_local_dirs_and_the_offline_cache(tmp_path):
    from uno_b200.utils.hub import resolve_hf_snapshot

    assert resolve_hf_snapshot(str(tmp_path)) == str(tmp_path)
    cache = tmp_path / "hub"
    repo = cache / "models--org--tiny"
    (repo / "snapshots" / "abc123").mkdir(parents=True)
    (repo / "snapshots" / "def456").mkdir(parents=True)
    (repo / "refs").mkdir()
    (repo / "refs" / "main").write_text("abc123\n")
    assert resolve_hf_snapshot("org/tiny", cache_dir=cache, local_files_only=True).endswith("abc123")
    assert resolve_hf_snapshot("org/tiny", revision="def456", cache_dir=cache,
                               local_files_only=True).endswith("def456")
    with pytest.raises(ValueError, match="local Hugging Face cache"):
        resolve_hf_snapshot("org/absent", cache_dir=cache, local_files_only=True)


def test_config_resolves_a_cached_repo_id(tmp_path):
    from uno_b200.config import Config

    snap = tmp_path / "hub" / "models--org--tiny" / "snapshots" / "c0ffee"
    snap.mkdir(parents=True)
    (tmp_path / "hub" / "models--org--tiny" / "refs").mkdir()
    (tmp_path / "hub" / "models--org--tiny" / "refs" / "main").write_text("c0ffee")
    save_model_config(_tiny_cfg(), str(snap))
    cfg = Config("org/tiny", device="cpu", load_format="dummy", hf_cache_dir=str(tmp_path / "hub"),
                 hf_local_files_only=True)
    assert cfg.model == str(snap) and cfg.hf_config.vocab_size == 4096


def test_model_token_ids_rules(tmp_path):
    from uno_b200.utils.hf_compat import TokenIdTokenizer
    from uno_b200.utils.model_tokens import resolve_model_token_ids

    d = tmp_path / "m"
    save_model_config(_tiny_cfg(), str(d))
    (d / "generation_config.json").write_text(json.dumps({"eos_token_id": [9, 7]}))
    tok = TokenIdTokenizer(4096, eos_token_id=3)
    mask, stops, vocab = resolve_model_token_ids(str(d), tok)
    assert (mask, stops, vocab) == (4095, [9, 7, 3], 4096)
    assert resolve_model_token_ids(str(d), tok, mask_token_id=17, stop_token_ids=[5, 5, 6])[:2] == (17, [5, 6])
    with pytest.raises(ValueError, match="outside model vocabulary"):
        resolve_model_token_ids(str(d), tok, stop_token_ids=[5000])
    # K2 / XLLM checkpoints with uniform noise may use the id one past the vocabulary
    k2 = tmp_path / "k2"
    save_model_config(_tiny_cfg(model_type="xllm", mask_token_id=None), str(k2))
    assert resolve_model_token_ids(str(k2), tok, noise_mode="random_uniform")[0] == 4096
    with pytest.raises(ValueError, match="mask token"):
        resolve_model_token_ids(str(k2), tok, noise_mode="mask")


def test_hub_prefetch_reuses_the_cache(tmp_path):
    from uno_b200.utils.hub import PINNED_MODEL_ID, PINNED_MODEL_REVISION, main

    repo = tmp_path / ("models--" + PINNED_MODEL_ID.replace("/", "--"))
    snap = repo / "snapshots" / PINNED_MODEL_REVISION
    snap.mkdir(parents=True)
    (snap / "config.json").write_text("{}")
    out = main(["prefetch", "--cache-dir", str(tmp_path), "--local-files-only"])
    assert out["snapshot_path"] == str(snap) and out["revision"] == PINNED_MODEL_REVISION
    (repo / "refs").mkdir()
    (repo / "refs" / "v1").write_text(PINNED_MODEL_REVISION)
    assert main(["prefetch", "--cache-dir", str(tmp_path), "--revision", "v1", "--local-files-only"])[
        "snapshot_path"] == str(snap)
