"""Semantic feasibility runners (reuse and P/D modes) on the CPU oracle: slot-map views, teacher-forced
stage metrics and commit chains, in the reference's result layout (behaviours of the reference's
test_progressive_kv_feasibility.py / test_pd_progressive_kv_feasibility.py)."""
import json

import torch

from sparsecache_b200.pipelines import feasibility as fz


def _dataset(path, n=3):
    g = torch.Generator().manual_seed(0)
    words = ["alpha", "beta", "gamma", "delta", "river", "city", "born", "year", "museum", "king"]
    rows = []
    for i in range(n):
        paras = []
        for j in range(3):
            text = " ".join(words[int(k)] for k in torch.randint(0, len(words), (12,), generator=g))
            paras.append({"idx": j, "title": f"T{j}", "paragraph_text": text, "is_supporting": j == i % 3})
        rows.append({"id": f"q{i}", "question": f"Where was {words[i]} born?", "answer": words[i],
                     "answer_aliases": [], "question_decomposition": [{}] * (2 + i % 2), "paragraphs": paras})
    path.write_text("".join(json.dumps(r) + "\n" for r in rows))
    return rows


def test_stratified_sample_keeps_hop_mix():
    rows = [{"question_decomposition": [{}] * (2 + (i % 3 == 0))} for i in range(30)]
    idx = fz.stratified_indices(rows, 9, seed=1)
    assert len(set(idx)) == 9 and sum(len(rows[i]["question_decomposition"]) == 3 for i in idx) == 3
    assert idx == fz.stratified_indices(rows, 9, seed=1)
    assert fz.parse_windows("1,2,inf") == [1, 2, None]


def test_level_metrics_agreement_and_survival():
    from sparsecache_b200.serving.progressive import Document

    docs = [Document((1,) * 4, supporting=True), Document((2,) * 6, supporting=False)]
    rows = [{"predictions": p, "mean_target_logprob": -1.0, "mean_top1_margin": 0.5, "forward_ms": 0.0}
            for p in ([1, 9, 3, 4], [1, 2, 8, 4], [1, 2, 3, 4])]
    lv = fz.level_metrics(rows, [1, 2, 3, 4], [{0}, {0}, {0, 1}], docs, [0.3, 0.5, 1.0])
    assert lv[0]["final_top1_agreement"] == 0.75 and lv[0]["adjacent_top1_agreement"] is None
    assert lv[1]["adjacent_top1_agreement"] == 0.5
    assert lv[0]["strict_final_survival"] == 0.5 and lv[2]["strict_final_survival"] == 1.0
    assert lv[0]["supporting_token_coverage"] == 1.0 and lv[0]["actual_document_fraction"] == 0.4


def test_feasibility_runners_end_to_end(tmp_path):
    from sparsecache_b200.models.checkpoint import random_checkpoint

    model_dir = random_checkpoint(tmp_path / "model", "tiny", seed=4, std=0.05)
    _dataset(tmp_path / "musique.jsonl")
    common = ["--model", str(model_dir), "--dataset", str(tmp_path / "musique.jsonl"), "--sample-count", "2",
              "--stage-fractions", "0.34,1.0", "--schedules", "sequential,oracle", "--commit-windows", "1,inf",
              "--draft-tokens", "3", "--max-new-tokens", "6", "--device", "cpu", "--dtype", "float32"]
    fz.main(["reuse", *common, "--output", str(tmp_path / "reuse.jsonl")])
    rows = [json.loads(x) for x in (tmp_path / "reuse.jsonl").read_text().splitlines()]
    assert len(rows) == 2
    r = rows[0]
    assert set(r["schedules"]) == {"sequential", "oracle"} and r["protocol"]["commit_windows"] == [1, "inf"]
    lv = r["schedules"]["oracle"]["levels"]
    assert lv[-1]["final_top1_agreement"] == 1.0 and lv[-1]["strict_final_survival"] == 1.0
    assert r["schedules"]["oracle"]["levels"][0]["supporting_token_coverage"] == 1.0
    assert r["fullreuse"]["teacher_self_top1_agreement"] == 1.0
    inf = r["schedules"]["sequential"]["chains"]["inf"]
    assert inf["lossless_gate_pass"] and inf["token_match_fullreuse"]  # one final full-view verifier
    assert len(r["fullreuse"]["token_ids"]) <= 6 and "fullcontext_cache" in r
    fz.main(["pd", *common, "--seed-tokens", "1", "--output", str(tmp_path / "pd.jsonl")])
    p = json.loads((tmp_path / "pd.jsonl").read_text().splitlines()[0])
    assert p["pd_target"]["seed_token_ids"] == p["prefill_side"]["token_ids"][:1]
    # a full view of the contiguous cache decodes the prefill side's own answer
    assert p["pd_target"]["token_match_prefill_side"]
    for sched in p["schedules"].values():
        assert sched["chains"]["inf"]["lossless_gate_pass"]
        assert 0 < sched["levels"][0]["actual_total_kv_fraction"] < 1 == sched["levels"][-1]["actual_total_kv_fraction"]


def test_feasibility_aggregation_of_both_modes(tmp_path):
    from sparsecache_b200.models.checkpoint import random_checkpoint

    model_dir = random_checkpoint(tmp_path / "model", "tiny", seed=5, std=0.05)
    _dataset(tmp_path / "musique.jsonl", n=4)
    common = ["--model", str(model_dir), "--dataset", str(tmp_path / "musique.jsonl"), "--sample-count", "4",
              "--stage-fractions", "0.5,1.0", "--schedules", "uniform", "--commit-windows", "inf",
              "--draft-tokens", "2", "--max-new-tokens", "4", "--device", "cpu", "--dtype", "float32"]
    for mode in ("reuse", "pd"):
        fz.main([mode, *common, "--offset", "0", "--count", "2", "--output", str(tmp_path / f"{mode}0.jsonl")])
        fz.main([mode, *common, "--offset", "2", "--count", "2", "--output", str(tmp_path / f"{mode}1.jsonl")])
        out = fz.aggregate_main([str(tmp_path / f"{mode}0.jsonl"), str(tmp_path / f"{mode}1.jsonl"),
                                 "--output", str(tmp_path / f"{mode}.json")])
        s = out["summary"]
        assert s["mode"] == mode and s["cases"] == 4 and sum(s["hop_counts"].values()) == 4
        chain = s["schedules"]["uniform"]["chains"]["inf"]
        timing = chain["optimistic_timing_by_bandwidth_gib_s"]
        assert set(timing) == {"1", "3", "6", "12", "25", "50"} and timing["1"]["speedup"] > 0
        assert s["schedules"]["uniform"]["levels"][-1]["final_top1_agreement"] == 1.0
        if mode == "pd":
            assert chain["lossless_gate_pass"] == 1.0 and "mean_required_total_kv_fraction" in chain
        else:
            assert "f1_vs_fullcontext_cache" in chain and "fullcontext_correct_to_fullreuse_wrong" in s["base"]["fullreuse"]
    import pytest
    with pytest.raises(ValueError, match="duplicate"):
        fz.aggregate_main([str(tmp_path / "pd0.jsonl"), str(tmp_path / "pd0.jsonl"), "--output", str(tmp_path / "x.json")])
