"""Teacher formats (v3 + v5 chained manifests) written and re-read with hash
checks, memory views, windows, the SparseKVDrafter training loop, its
evaluators and checkpoint format, and the corpus builder (behaviours of the
reference's test_train_sparse_kv_drafter.py, test_extract_sparse_kv_teacher.py,
test_eval_sparse_kv_boundaries.py and test_build_sparse_kv_draft_corpus.py)."""
import json

import pytest
import torch

from sparsecache_b200.models.sparse_kv_draft import SparseKVDraftConfig, SparseKVDrafter
from sparsecache_b200.training import corpus, sparse_drafter
from sparsecache_b200.training.teacher import (TeacherSample, load_teacher_dataset, select_memory,
                                               training_window_inputs, write_teacher_dataset)

L, H, D, HT, V = 2, 2, 4, 16, 40


def _sample(i, T=200, t=6, g=None):
    gen = torch.Generator().manual_seed(i)
    ids = torch.randint(0, V, (t + 1,), generator=gen)
    return TeacherSample(i, T, {
        "memory_keys": torch.randn(L, H, T, D, generator=gen), "memory_values": torch.randn(L, H, T, D, generator=gen),
        "seed_hidden": torch.randn(2, HT, generator=gen), "input_ids": ids[:-1].clone(), "labels": ids[1:].clone(),
        "teacher_topk_ids": torch.randint(0, V, (t, 4), generator=gen), "teacher_topk_logprobs": torch.randn(t, 4),
        "teacher_hidden": torch.randn(t, HT, generator=gen), "priority_page_scores": torch.rand(-(-T // 64)),
        "query_cos": torch.randn(t, D, generator=gen), "query_sin": torch.randn(t, D, generator=gen),
        "prompt_ids": torch.randint(0, V, (T,), generator=gen, dtype=torch.int32),
        "continuation_seed_hidden": torch.randn(t, 2, HT, generator=gen)}, g)


def test_teacher_roundtrip_v3_v5_and_hash_check(tmp_path):
    samples = [_sample(i, g=f"ds{i % 2}") for i in range(3)]
    kw = dict(target_fingerprint="fp", kv_layers=(0, 1), seed_layers=(0, 1), head_dim=D, kv_heads=H,
              target_hidden_size=HT, vocab_size=V)
    m5 = write_teacher_dataset(samples, tmp_path / "t", with_boundaries=True, **kw)
    man, loaded = load_teacher_dataset(m5)
    assert man["format"].endswith(".v5") and set(loaded) == {0, 1, 2}
    s = loaded[1]
    assert torch.equal(s.tensors["memory_keys"], samples[1].tensors["memory_keys"])
    assert "initial_input_ids" in s.tensors and s.source_group == "ds1"
    ids, seed, cos, sin, labels, _, _ = training_window_inputs(s, "cpu", offset=2, window_tokens=3)
    assert ids.shape == (1, 3) and torch.equal(seed[0], samples[1].tensors["continuation_seed_hidden"][1])
    k, v, frac, n = select_memory(s, page_size=64, requested_fraction=0.5, seed=0, device="cpu")
    assert k.shape[2] == n and 0 < frac <= 1
    (tmp_path / "t" / "sample_00001.safetensors").write_bytes(b"corrupt")
    with pytest.raises(Exception):
        load_teacher_dataset(tmp_path / "t" / "manifest.json")


def test_sparse_drafter_training_eval_and_checkpoint(tmp_path):
    torch.manual_seed(0)
    cfg = SparseKVDraftConfig(target_hidden_size=HT, draft_hidden_size=8, head_dim=D, num_draft_heads=2,
                              num_memory_heads=H, num_memory_layers=L, num_seed_layers=2, mlp_ratio=2)
    model = SparseKVDrafter(cfg)
    model.bind_target_weights(torch.randn(V, HT), torch.randn(V, HT))
    train = [_sample(i, g=f"ds{i % 2}") for i in range(4)]
    hist = sparse_drafter.train_sparse_drafter(model, train, fractions=(0.2, 0.5), steps=8, device="cpu",
                                               log_every=4, lr=1e-2, window_tokens=3)
    assert len(hist) == 2 and all(torch.isfinite(torch.tensor(h["loss"])) for h in hist)
    res = sparse_drafter.five_cell_ablation(model, train[:2], (0.5,), device="cpu", max_proposal_tokens=4)
    assert set(res) == {"exact", "zero_memory", "shuffled_memory", "zero_seed", "zero_memory_zero_seed"}
    assert 0 <= res["exact"][0]["mean_accepted_prefix"] <= 4
    b = sparse_drafter.evaluate_boundaries(model, train[:2], (0.5,), device="cpu", window_tokens=3,
                                           maximum_windows_per_sample=2)
    assert b[0]["overall"]["windows"] == 4 and set(b[0]["by_source_group"]) == {"ds0", "ds1"}
    assert sparse_drafter.select_offsets(10, 3) == (1, 4, 7)
    p = tmp_path / "drafter.pt"
    sparse_drafter.save_checkpoint(model, p, target_model="m", target_fingerprint="fp", completed_steps=8)
    m2, ck = sparse_drafter.load_checkpoint(p, target_fingerprint="fp")
    assert ck["completed_steps"] == 8 and all("target_" not in k for k in ck["state_dict"])
    with pytest.raises(ValueError):
        sparse_drafter.load_checkpoint(p, target_fingerprint="other")


def test_corpus_builder(tmp_path):
    root = tmp_path / "packs"
    for ds in ("a", "b"):
        d = root / ds
        d.mkdir(parents=True)
        (d / "requests.jsonl").write_text("".join(json.dumps({"prompt": [0] * (5 + i)}) + "\n" for i in range(10)))
        (d / "metadata.jsonl").write_text("".join(json.dumps({"i": i}) + "\n" for i in range(10)))
        (d / "manifest.json").write_text(json.dumps({"dataset": ds}))
    reqs, meta, man = corpus.build_corpus(root, ("a", "b"), 3)
    assert [r["source_dataset"] for r in reqs] == ["a", "b"] * 3
    assert man["source_manifests"]["a"]["selected_source_indices"] == [1, 5, 8]
    corpus.write_corpus(tmp_path / "out", reqs, meta, man)
    assert json.loads((tmp_path / "out" / "manifest.json").read_text())["format"].endswith("corpus.v1")


def test_training_clis_end_to_end_on_cpu(tmp_path):
    """train-eagle (with snapshot + resume) and train-drafter over a written teacher dataset."""
    from sparsecache_b200.training import cli

    samples = [_sample(i, g=f"ds{i % 2}") for i in range(6)]
    man = write_teacher_dataset(samples, tmp_path / "teacher", target_fingerprint="fp", kv_layers=(0, 1),
                                seed_layers=(0, 1), head_dim=D, kv_heads=H, target_hidden_size=HT, vocab_size=V,
                                with_boundaries=True)
    g = torch.Generator().manual_seed(3)
    torch.save({"embed": torch.randn(V, HT, generator=g), "lm_head": torch.randn(V, HT, generator=g)},
               tmp_path / "target.pt")
    (tmp_path / "eagle.json").write_text(json.dumps(dict(
        target_hidden_size=HT, hidden_size=16, intermediate_size=32, head_dim=D, num_attention_heads=4,
        num_key_value_heads=2, num_memory_heads=H, num_memory_layers=L, num_seed_layers=2, target_vocab_size=V,
        draft_vocab_size=24)))
    common = ["--teacher-manifest", str(man), "--device", "cpu", "--target-model", "tiny",
              "--target-embedding", str(tmp_path / "target.pt"), "--eval-modulus", "3", "--log-every", "1"]
    out = tmp_path / "eagle"
    s = cli.main(["train-eagle", *common, "--output-dir", str(out), "--drafter-config", str(tmp_path / "eagle.json"),
                  "--steps", "3", "--save-every", "2", "--global-batch", "2", "--adapter-scale-init", "0"])
    assert s["completed_steps"] == 3 and s["train_samples"] == 4 and s["eval_samples"] == 2
    assert (out / "adapter.pt").exists() and (out / "adapter_step000002.pt").exists()
    assert set(s["evaluation"]) == {"exact", "disabled"} and len(s["history"]) == 2
    s2 = cli.main(["train-eagle", *common, "--output-dir", str(tmp_path / "eagle2"), "--drafter-config",
                   str(tmp_path / "eagle.json"), "--steps", "2", "--global-batch", "2",
                   "--resume-adapter", str(out / "adapter.pt")])
    assert s2["resumed_from_step"] == 3 and s2["completed_steps"] == 5
    d = cli.main(["train-drafter", *common, "--output-dir", str(tmp_path / "drafter"), "--steps", "4",
                  "--draft-hidden-size", "8", "--mlp-ratio", "2", "--visibility-fractions", "0.5",
                  "--training-window-tokens", "3", "--max-eval-tokens", "3"])
    assert (tmp_path / "drafter" / "checkpoint.pt").exists() and "exact" in d["ablation"]
    ev_common = ["--checkpoint", str(tmp_path / "drafter" / "checkpoint.pt"), "--teacher-manifest", str(man),
                 "--device", "cpu", "--target-embedding", str(tmp_path / "target.pt"), "--eval-indices", "0,3",
                 "--visibility-fractions", "0.5,1.0"]
    ev = cli.main(["eval-drafter", *ev_common, "--output", str(tmp_path / "eval.json"), "--max-eval-tokens", "3"])
    assert ev["eval_indices"] == [0, 3] and set(ev["cells"]) == {"exact", "zero_memory", "shuffled_memory",
                                                                 "zero_seed", "zero_memory_zero_seed"}
    assert len(ev["cells"]["exact"]) == 2 and (tmp_path / "eval.json").exists()
    bd = cli.main(["eval-boundaries", *ev_common, "--output", str(tmp_path / "bd.json"), "--window-tokens", "2",
                   "--max-windows-per-sample", "2"])
    row = bd["memory_modes"]["exact"][0]
    assert row["overall"]["windows"] == 4 and set(row["by_source_group"]) == {"ds0", "ds1"}
    assert cli.split_indices({0, 1, 2, 3}, train="0-2", evaluate=None, eval_modulus=0, eval_remainder=0) == ([0, 1, 2], [3])
    with pytest.raises(ValueError):
        cli.split_indices({0, 1}, train="0-1", evaluate="1", eval_modulus=0, eval_remainder=0)


def test_teacher_extraction_and_extension_clis_on_cpu(tmp_path):
    """extract-teacher (v3) then extend-teacher (v5 chained to it) from a model directory on the CPU oracle,
    re-read through the trainer's loader; the extender refuses a changed corpus."""
    from sparsecache_b200.models.checkpoint import load_oracle, random_checkpoint
    from sparsecache_b200.training import cli
    from sparsecache_b200.training.teacher import prompt_sha256

    model_dir = random_checkpoint(tmp_path / "model", "tiny", seed=1, std=0.05)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(4, 1024, (n,), generator=g).tolist() for n in (70, 130, 90)]
    corpus = tmp_path / "requests.jsonl"
    corpus.write_text("".join(json.dumps({"prompt": p, "source_dataset": f"ds{i}", "source_index": i}) + "\n"
                              for i, p in enumerate(prompts)))
    m3 = cli.main(["extract-teacher", "--model", str(model_dir), "--requests-jsonl", str(corpus),
                   "--output-dir", str(tmp_path / "t3"), "--request-indices", "0,2", "--continuation-tokens", "4",
                   "--kv-layers", "0,1", "--seed-layers", "0,1", "--teacher-topk", "8", "--device", "cpu"])
    assert m3["format"].endswith(".v3") and [r["request_index"] for r in m3["samples"]] == [0, 2]
    assert m3["samples"][1]["prompt_sha256"] == prompt_sha256(prompts[2])
    _, loaded = load_teacher_dataset(tmp_path / "t3" / "manifest.json")
    s = loaded[2].tensors
    oracle = load_oracle(model_dir)
    _, cache = oracle.prefill(prompts[2])
    assert s["memory_keys"].shape == (2, 2, 90, 64) and s["priority_page_scores"].shape == (2,)
    assert torch.allclose(s["memory_keys"][1].float(), cache[1][0][0], atol=2e-2, rtol=2e-2)
    assert torch.allclose(s["priority_page_scores"].sum(), torch.tensor(1.0), atol=1e-4)
    n = s["labels"].numel()
    assert 1 <= n <= 4 and torch.equal(s["labels"][:-1], s["input_ids"][1:])
    assert torch.equal(s["teacher_topk_ids"][:, 0], s["labels"])
    m5 = cli.main(["extend-teacher", "--base-manifest", str(tmp_path / "t3" / "manifest.json"),
                   "--output-dir", str(tmp_path / "t5"), "--continuation-tokens", "7", "--teacher-topk", "8",
                   "--device", "cpu"])
    assert m5["format"].endswith(".v5") and m5["kv_layers"] == [0, 1]
    man, loaded5 = load_teacher_dataset(tmp_path / "t5" / "manifest.json")
    t = loaded5[2].tensors
    assert torch.equal(t["memory_keys"], s["memory_keys"]) and t["continuation_seed_hidden"].shape[1:] == (2, 256)
    assert torch.equal(t["input_ids"][:n], s["input_ids"]) and torch.equal(t["initial_labels"], s["labels"])
    # the seed layer's hidden at continuation token j is its output at that row of one oracle pass
    full = torch.tensor(prompts[2] + t["input_ids"].tolist())
    hid, _ = oracle.forward_tokens(full, torch.arange(full.numel()))
    assert torch.allclose(t["teacher_hidden"][-1].float(), oracle.norm(hid[0, -1]), atol=3e-2, rtol=3e-2)
    corpus.write_text(corpus.read_text() + "\n")
    with pytest.raises(ValueError, match="corpus hash"):
        cli.main(["extend-teacher", "--base-manifest", str(tmp_path / "t3" / "manifest.json"),
                  "--output-dir", str(tmp_path / "t5b"), "--device", "cpu"])


def test_teacher_request_rows_are_exact_and_bounded(tmp_path):
    from sparsecache_b200.training import cli

    path = tmp_path / "r.jsonl"
    path.write_text("".join(json.dumps(r) + "\n" for r in (
        {"prompt": [5, 6, 7], "source_dataset": "a", "source_index": 3}, {"prompt": [1] * 9},
        {"prompt": [1, "x"]}, {"prompt": [8, 9]})))
    rows = cli.load_request_rows(path, [3, 0], 8)
    assert [r["request_index"] for r in rows] == [0, 3] and rows[0]["source_index"] == 3
    with pytest.raises(ValueError, match="cap"):
        cli.load_request_rows(path, [1], 8)
    with pytest.raises(ValueError, match="invalid prompt"):
        cli.load_request_rows(path, [2], 8)
    with pytest.raises(ValueError, match="missing"):
        cli.load_request_rows(path, [0, 7], 8)
    assert cli.parse_layer_list("8,20,31", name="KV layers") == (8, 20, 31)
    for bad in ("", "1,1", "-1"):
        with pytest.raises(ValueError):
            cli.parse_layer_list(bad, name="KV layers")
