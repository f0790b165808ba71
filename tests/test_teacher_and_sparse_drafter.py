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
    assert cli.split_indices({0, 1, 2, 3}, train="0-2", evaluate=None, eval_modulus=0, eval_remainder=0) == ([0, 1, 2], [3])
    with pytest.raises(ValueError):
        cli.split_indices({0, 1}, train="0-1", evaluate="1", eval_modulus=0, eval_remainder=0)
