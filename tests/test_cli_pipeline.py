"""prepare -> precompute -> qa CLIs end to end on the CPU plumbing model."""
import json

import torch

from sparsecache_b200 import data, precompute, qa
from sparsecache_b200.metrics import answer_em, answer_f1, clean_short_answer, normalize_answer
from sparsecache_b200.models.checkpoint import load_oracle, random_checkpoint
from sparsecache_b200.modeling import baseline_generate, cacheblend_generate, direct_reuse_generate
from sparsecache_b200.prompting import tokenize_case
from sparsecache_b200.store import compose_cache, load_manifest
from sparsecache_b200.tokenizer import ByteTokenizer


def _hotpot_jsonl(path):
    passages = "".join(f"Passage {i}:\nTitle {i}\nBody text number {i} about topic {i % 3}.\n" for i in range(1, 11))
    row = {"_id": "q1", "dataset": "hotpotqa", "input": "Which topic?", "answers": ["topic 1"], "context": passages}
    path.write_text(json.dumps(row) + "\n")


def test_adapters_and_metrics(tmp_path):
    _hotpot_jsonl(tmp_path / "h.jsonl")
    case = data.load_hotpotqa_case(tmp_path / "h.jsonl", index=0, max_chunks=10)
    assert len(case.chunks) == 10 and case.chunks[0].title == "Title 1"
    assert case.chunks[2].text.startswith("Body text number 3")
    mus = {"id": "m1", "question": "q?", "answer": "Paris", "answer_aliases": ["paris", "Paris"],
           "paragraphs": [{"idx": i, "title": f"t{i}", "paragraph_text": f"p{i}", "is_supporting": i == 2}
                          for i in range(12)]}
    (tmp_path / "m.jsonl").write_text(json.dumps(mus) + "\n")
    mc = data.load_musique_case(tmp_path / "m.jsonl", index=0, max_chunks=10)
    assert len(mc.chunks) == 10 and mc.chunks[2].supporting and mc.answers == ("Paris", "paris")
    assert normalize_answer("The  Eiffel, Tower!") == "eiffel tower"
    assert answer_em("the eiffel tower", ["Eiffel Tower"]) == 1.0
    assert abs(answer_f1("eiffel", ["Eiffel Tower"]) - 2 / 3) < 1e-9
    assert clean_short_answer("Answer: Paris<|eot_id|>\nmore") == "Paris"


def test_cli_end_to_end(tmp_path):
    model_dir = random_checkpoint(tmp_path / "model", "tiny", seed=0, std=0.05)
    _hotpot_jsonl(tmp_path / "h.jsonl")
    data.main(["--dataset", "hotpotqa", "--input", str(tmp_path / "h.jsonl"), "--output", str(tmp_path / "case.json")])
    precompute.main(["--case", str(tmp_path / "case.json"), "--model", str(model_dir), "--output-dir",
                     str(tmp_path / "cache"), "--device", "cpu", "--dtype", "float32"])
    manifest = json.loads((tmp_path / "cache" / "manifest.json").read_text())
    assert manifest["format"] == "sparsecache.chunk-kv.v1" and len(manifest["chunks"]) == 10
    assert all(c["source_start"] == manifest["system"]["tokens"] for c in manifest["chunks"])
    qa.main(["--manifest", str(tmp_path / "cache" / "manifest.json"), "--output", str(tmp_path / "qa.json"),
             "--modes", "baseline", "direct", "cacheblend", "--device", "cpu", "--max-new-tokens", "6",
             "--recompute-ratio", "1.0"])
    out = json.loads((tmp_path / "qa.json").read_text())
    by_mode = {r["mode"]: r for r in out["results"]}
    assert set(by_mode) == {"baseline", "direct", "cacheblend"}
    # ratio 1.0 reproduces the full-prefill answer
    assert by_mode["cacheblend"]["token_ids"] == by_mode["baseline"]["token_ids"]
    assert out["relocated_tokens"] > 0


def test_public_api_oracle(tmp_path):
    model_dir = random_checkpoint(tmp_path / "model", "tiny", seed=1, std=0.05)
    model = load_oracle(model_dir)
    tok = ByteTokenizer(1024)
    _hotpot_jsonl(tmp_path / "h.jsonl")
    case = data.load_hotpotqa_case(tmp_path / "h.jsonl", index=0, max_chunks=10)
    prompt = tokenize_case(tok, case)
    full = prompt.full_ids
    S, D = len(prompt.system_ids), len(prompt.document_ids)
    _, cache = model.prefill(full[: S + D])
    base = baseline_generate(model, full_ids=full, max_new_tokens=5, eos_token_ids={2})
    direct = direct_reuse_generate(model, prefix_cache=cache, suffix_ids=prompt.suffix_ids, max_new_tokens=5,
                                   eos_token_ids={2})
    blend = cacheblend_generate(model, full_ids=full, prefix_cache=cache, system_tokens=S,
                                suffix_tokens=len(prompt.suffix_ids), check_layer=1, recompute_ratio=0.15,
                                max_new_tokens=5, eos_token_ids={2})
    # with the exact full-prompt cache, direct reuse equals the baseline
    assert direct.token_ids == base.token_ids
    assert blend.metadata["document_tokens"] == D
    assert blend.metadata["document_tokens_selected"] == max(1, -(-D * 15 // 100))
    assert base.as_dict()["metadata"]["full_prefill"] is True
