"""LongBench metrics/packs, RULER normalisation/packs and chunk priorities
(behaviours of the reference's test_longbench_metrics.py,
test_longbench_pd_pack.py, test_build_ruler_pd_pack.py and
test_ruler_chunk_priorities.py)."""
import json

import pytest

from sparsecache_b200.evaluation import longbench, priorities, ruler


def test_qa_and_rouge_metrics():
    name, em, score = longbench.score_prediction("2wikimqa", "The Eiffel Tower", ["Eiffel Tower"])
    assert (name, em, score) == ("qa_f1", 1.0, 1.0)
    name, _, score = longbench.score_prediction("qmsum", "alpha beta gamma", ["alpha gamma"])
    assert name == "rouge_l_f1" and score == pytest.approx(0.8, abs=1e-7)


def test_retrieval_count_code_classification_and_choice():
    assert longbench.score_prediction("passage_retrieval_en", "Paragraph 7", ["Paragraph 7"])[1:] == (1.0, 1.0)
    assert longbench.score_prediction("passage_count", "There are 12.", ["12"])[2] == 1.0
    assert longbench.score_prediction("lcc", "value = item", ["value = item"])[2] == 1.0
    assert longbench.score_prediction("lcc", "# comment\nx = 1", ["x = 1"])[2] == 1.0
    name, _, s = longbench.score_prediction("trec", "Location\nextra", ["Location"], ["Location", "Person"])
    assert name == "classification_accuracy" and s == 1.0
    name, em, s = longbench.score_prediction("longbench_v2", "After checking, The correct answer is (C)", ["C"])
    assert (name, em, s) == ("choice_accuracy", 1.0, 1.0)
    assert longbench.lcs_length("a b c d".split(), "b d".split()) == 2


def test_chunk_alignment_trims_the_middle_or_pads():
    prompt, cap, removed, pad = longbench.align_context_to_chunk([1] * 10, list(range(1000)), [2] * 6,
                                                                  max_prompt_tokens=600, chunk_tokens=256)
    assert len(prompt) == 512 and cap == 1000 - 584 and removed == 584 - 496 and pad == 0
    assert prompt[10] == 0 and prompt[-7] == 999  # head and tail of the context survive
    prompt, _, _, pad = longbench.align_context_to_chunk([1] * 10, [5] * 20, [2] * 6, max_prompt_tokens=600,
                                                         chunk_tokens=256, padding_token_id=9)
    assert len(prompt) == 256 and pad == 256 - 36 and prompt[30] == 9


class _Tok:
    name_or_path = "fake"

    def __init__(self):
        self.kwargs = None

    def apply_chat_template(self, messages, **kw):
        self.kwargs = kw
        return "PRE " + " | ".join(m["content"] for m in messages) + " SUF"

    @staticmethod
    def encode(text, add_special_tokens=False):
        return list(text.encode())


def test_longbench_request_row():
    tok = _Tok()
    row = {"input": "who?", "context": "x" * 3000, "answers": ["me"]}
    req = longbench.build_longbench_request(tok, "hotpotqa", row, max_prompt_tokens=2048, chunk_tokens=256,
                                            disable_thinking=True)
    assert len(req["prompt"]) % 256 == 0 and len(req["prompt"]) <= 2048
    assert req["max_tokens"] == 32 and tok.kwargs["enable_thinking"] is False


def test_ruler_parse_placements_and_render():
    prompt = ("x " + ruler.CONTEXT_START + "Document 1:\nAlpha\nbody a\n\nDocument 2:\nBeta\nbody b\n\n"
              "Document 3:\nGamma\nbody c" + ruler.CONTEXT_END + "Q?<|eot_id|>")
    docs = ruler.parse_documents(prompt)
    assert [d["title"] for d in docs] == ["Alpha", "Beta", "Gamma"]
    for d, s in zip(docs, (False, True, False)):
        d["supporting"] = s
    orders = ruler.placement_orders(docs)
    assert orders["evidence_first"] == [1, 0, 2] and orders["evidence_last"] == [0, 2, 1]
    assert sorted(orders["evidence_uniform"]) == [0, 1, 2]
    tok = _Tok()
    row = {"question": "Q?", "placements": orders, "documents": docs}
    prefix, rendered, suffix = ruler.render_parts(tok, row, "evidence_first", disable_thinking=True)
    assert prefix and suffix and rendered[0]["supporting"] and rendered[0]["source_document_index"] == 1
    assert tok.kwargs["enable_thinking"] is False


def test_ruler_fit_documents_exact_budget():
    docs = [{"token_ids": list(range(50)), "supporting": True}, {"token_ids": list(range(30)), "supporting": False},
            {"token_ids": list(range(20)), "supporting": False}]
    fitted, total, mode = ruler.fit_documents(docs, 70)
    assert mode == "trim_distractors" and sum(map(len, fitted)) == 70 and len(fitted[0]) == 50
    fitted, _, mode = ruler.fit_documents(docs, 160)
    assert mode == "repeat_distractors" and sum(map(len, fitted)) == 160 and len(fitted[0]) == 50
    with pytest.raises(ValueError):
        ruler.fit_documents(docs, 51)


def test_ruler_pack_files(tmp_path):
    tok = _Tok()
    docs = [{"title": "A", "text": "alpha " * 40, "supporting": True}, {"title": "B", "text": "beta " * 90,
                                                                         "supporting": False}]
    row = {"id": "r0", "question": "Q?", "answers": ["a"], "documents": docs,
           "placements": ruler.placement_orders(docs)}
    src = tmp_path / "qa2.jsonl"
    src.write_text(json.dumps(row) + "\n")
    man = ruler.build_pack(tok, src, "evidence_last", 1024, tmp_path / "pack")
    req = json.loads((tmp_path / "pack" / "requests.jsonl").read_text())
    meta = json.loads((tmp_path / "pack" / "metadata.jsonl").read_text())
    assert len(req["prompt"]) == 1024 and man["requests"] == 1
    assert meta["document_spans"][-1]["supporting"] is True


def test_bm25_and_oracle_prioritise_relevant_chunks():
    documents = [{"text": "irrelevant apples", "supporting": False},
                 {"text": "Scott Derrickson nationality", "supporting": True}]
    common = dict(request_id="row-1", question="What is Scott Derrickson nationality?", documents=documents,
                  spans=[{"start_token": 256, "end_token": 512}, {"start_token": 512, "end_token": 768}],
                  total_chunks=6, chunk_tokens=256, protected_prefix_chunks=1, protected_suffix_chunks=1, seed=7)
    for mode in ("bm25", "oracle"):
        order = priorities.priority_for_mode(mode, **common)
        assert set(order[:2]) == {0, 5} and order.index(2) < order.index(1) and sorted(order) == list(range(6))
    assert priorities.bm25_scores(common["question"], [d["text"] for d in documents])[1] > 0


def test_random_priority_stable_and_protected_first():
    common = dict(request_id="row-9", question="q", documents=[{"text": "d", "supporting": False}],
                  spans=[{"start_token": 256, "end_token": 1024}], total_chunks=8, chunk_tokens=256,
                  protected_prefix_chunks=1, protected_suffix_chunks=2, seed=42)
    a = priorities.priority_for_mode("random", **common)
    assert a == priorities.priority_for_mode("random", **common) and set(a[:3]) == {0, 6, 7}
    assert priorities.uniform_order(9)[:3] == [0, 8, 4]


def test_spans_from_prompt_markers():
    class T:
        @staticmethod
        def encode(text, add_special_tokens=False):
            return list(text.encode())

    source = {"placements": {"original": [1, 0]},
              "documents": [{"text": "zero", "supporting": False}, {"text": "one", "supporting": True}]}
    prompt = list("prefix Document 1:\none Document 2:\nzero suffix".encode())
    spans, docs = priorities.document_spans_from_prompt_markers(T(), prompt, source, "original", 7)
    assert spans[0]["supporting"] is True and spans[0]["end_token"] == spans[1]["start_token"]
    assert [d["text"] for d in docs] == ["one", "zero"]
    cov = priorities.coverage_curve([1, 0], [{"start_token": 0, "end_token": 4, "supporting": True}], 4)
    assert cov == [0.0, 1.0]


def test_pack_audits_matrix_coverage_and_quality(tmp_path):
    import hashlib

    from sparsecache_b200.evaluation import audits

    d = tmp_path / "hotpotqa"
    d.mkdir()
    (d / "requests.jsonl").write_text("".join(json.dumps({"prompt": [1] * 512}) + "\n" for _ in range(3)))
    (d / "metadata.jsonl").write_text("".join(json.dumps({"request_index": i, "dataset": "hotpotqa",
                                                          "answers": ["paris"]}) + "\n" for i in range(3)))
    h = lambda p: hashlib.sha256(p.read_bytes()).hexdigest()  # noqa: E731
    (d / "manifest.json").write_text(json.dumps({"dataset": "hotpotqa", "chunk_tokens": 256,
                                                 "requests_sha256": h(d / "requests.jsonl"),
                                                 "metadata_sha256": h(d / "metadata.jsonl")}))
    assert audits.audit_pack(d, expected_dataset="hotpotqa")["rows"] == 3
    m = audits.audit_dataset_matrix(tmp_path, ["hotpotqa", "musique"])
    assert m["status"] == "failed" and "hotpotqa" in m["cells"] and m["failures"][0].startswith("musique")
    cov = audits.priority_coverage([2, 0, 1], [{"start_token": 512, "end_token": 768, "supporting": True}], 256)
    assert cov["0.5"] == 1.0
    q = audits.quality_audit([{"request_index": 0, "token_ids": [1, 2]}],
                             [{"request_index": 0, "dataset": "hotpotqa", "answers": ["Paris"]}],
                             decode=lambda ids: "paris")
    assert q["overall"] == 1.0


def test_pd_pipeline_auto_draft_and_aggregate():
    from sparsecache_b200.pipelines.pd import aggregate, auto_draft_tokens

    g, wire = auto_draft_tokens(prompt_tokens=16384, first_stage_tokens=4096, bytes_per_token=131072,
                                transport_gbps=100.0, tpot_ms=3.5, max_draft_tokens=7)
    assert wire == pytest.approx(12288 * 131072 * 8 / 1e8) and g == 7
    g, _ = auto_draft_tokens(prompt_tokens=1000, first_stage_tokens=990, bytes_per_token=131072,
                             transport_gbps=100.0, tpot_ms=3.5, max_draft_tokens=7)
    assert g == 1
    rows = [{"tokens_equal": True, "full_target": {"response_ms": 100.0, "first_ready_ms": 40.0},
             "chain": {"response_ms": 90.0, "first_ready_ms": 30.0, "accepted": 3}}]
    agg = aggregate(rows)
    assert agg["token_equality_rate"] == 1.0 and agg["response_gain_ms"]["mean"] == 10.0


def _pd_row(i, *, target_ms, pipe_ms, fixed_ms, graft_batches, fixed_batch, acc, fixed_acc, match=True):
    def pipe(batches, accepted, ms):
        trace = [{"stage": s, "drafted": len(b), "draft_token_ids": b} for s, b in enumerate(batches)]
        trace.append({"stage": 3, "verified": True, "accepted_pending": accepted,
                      "rejected_pending": sum(map(len, batches)) - accepted, "drafted": 0})
        return {"response_ms": ms, "first_committed_ms": ms / 2, "terminated_stage": len(batches) - 1,
                "trace": trace, "draft_prefill_ms": 0.0, "draft_decode_ms": 2.0,
                "visible_fraction_per_draft": [0.25] * len(batches[0]) + [0.5] * sum(map(len, batches[1:])),
                "transfer": {"stage_wire_ms": [1.0, 2.0, 3.0], "total_h2d_ms": 0.5, "stage_wire_wait_ms": [0.1]}}

    graft = pipe(graft_batches, acc, pipe_ms)
    fixed = pipe([fixed_batch], fixed_acc, fixed_ms)
    return {"dataset_index": i, "protocol": {"schedules": ["query"], "commit_windows": ["inf"],
                                             "transport_gbps": 50.0, "draft_tokens": 6},
            "schedules": {"query": {"full_target": {"response_ms": target_ms, "decode_ms": 5.0, "seed_forward_ms": 0.0,
                                                    "transfer": {"total_h2d_ms": 1.0}},
                                    "chains": {"inf": {"configured_draft_tokens": 6, "timing_token_match_target": match,
                                                       "pipeline": graft, "paired_fixed_control": fixed}}}}}


def test_pd_run_summary_and_graft_triggers():
    from sparsecache_b200.pipelines.analysis import analyze_graft_triggers, paired_delta, summarize_run

    rows = [_pd_row(0, target_ms=30.0, pipe_ms=20.0, fixed_ms=24.0, graft_batches=[[1, 2], [3, 4]],
                    fixed_batch=[1, 2, 9, 9, 9, 9], acc=3, fixed_acc=2),
            _pd_row(1, target_ms=40.0, pipe_ms=35.0, fixed_ms=33.0, graft_batches=[[5, 6], [7, 8, 1]],
                    fixed_batch=[5, 6, 7, 8, 1, 0], acc=2, fixed_acc=2)]
    s = summarize_run(rows)
    assert s["cases"] == 2 and s["latency"]["saved_vs_full_target_ms"]["mean"] == 7.5
    assert s["drafts"]["accepted_at_final_verifier"]["mean"] == 2.5 and s["drafts"]["proposed"]["max"] == 5
    assert s["terminated_stage_counts"] == {"2": 2}
    assert s["residual_wire_ms"]["mean"] == 5.0
    pf = s["paired_fixed_control"]
    assert pf["latency_saved_by_method_ms"]["mean"] == 1.0 and pf["accepted_token_delta_method_minus_fixed"]["positive"] == 1
    t = analyze_graft_triggers(rows)
    assert t["cases"] == 2 and t["triggers"]["margin_trigger"] is None
    by = {c["dataset_index"]: c for c in t["rows"]}
    # request 0: the second batch differs from the fixed proposals -> instability fires, gain 1
    assert by[0]["s2_first_token_instability"] and by[0]["acceptance_gain"] == 1
    # request 1: the graft proposals equal the fixed ones -> no trigger, no gain
    assert not by[1]["s2_batch_instability"] and by[1]["acceptance_gain"] == 0
    trig = t["triggers"]["s2_batch_instability"]
    assert trig["triggered"] == 1 and trig["true_positive"] == 1 and trig["missed_positive"] == 0
    assert paired_delta([3, 1], [1, 1])["positive"] == 1


def test_pd_link_helpers(tmp_path):
    from sparsecache_b200.pipelines.pd import (common_prefix_length, parse_bandwidths, target_kv_bytes_per_token,
                                               transfer_ms)

    assert parse_bandwidths("100,25,50") == (25.0, 50.0, 100.0)
    assert common_prefix_length([1, 2, 3], [1, 2, 9]) == 2
    for bad in ("25,25", "0"):
        with pytest.raises(ValueError):
            parse_bandwidths(bad)
    (tmp_path / "config.json").write_text(json.dumps({"num_hidden_layers": 32, "num_attention_heads": 32,
                                                      "num_key_value_heads": 8, "hidden_size": 4096}))
    assert target_kv_bytes_per_token(tmp_path) == 131072
    assert transfer_ms(8_000_000_000, 100.0) == pytest.approx(640.0)


def test_pd_rows_feed_validator_summary_and_aggregate():
    from types import SimpleNamespace

    from sparsecache_b200.pipelines.analysis import summarize_run
    from sparsecache_b200.pipelines.pd import aggregate, build_result_row
    from sparsecache_b200.serving.live.validate import validate_latency_cell
    from sparsecache_b200.serving.progressive import ChainResult

    proto = {"schedules": ["query"], "commit_windows": ["inf"], "transport_gbps": 50.0, "draft_tokens": 4,
             "fixed_token_horizon": True, "paired_measurement": True, "require_exclusive_gpu": True,
             "initial_gpu_used_bytes": 0}
    rows = []
    for i in range(4):
        req = SimpleNamespace(prompt_tokens=100, prefix=[1] * 4, suffix=[2] * 6, documents=[[3] * 45, [4] * 45])
        toks = (7, 8, 9, 10)
        trace = ({"stage": 0, "drafted": 2, "draft_token_ids": [8, 9]},
                 {"stage": 1, "verified": True, "accepted_pending": 2, "rejected_pending": 0, "drafted": 0})
        chain = ChainResult(toks, (8, 9), 2, 5.0, 20.0, 1, (0.5, 0.5),
                            {"total_h2d_ms": 1.0, "stage_wire_ms": [2.0, 3.0], "stage_wire_wait_ms": [0.5]},
                            trace, 4.0, 1)
        out = {"full_target": {"tokens": list(toks), "first_ready_ms": 10.0, "response_ms": 30.0,
                               "seed_forward_ms": 0.0, "decode_ms": 20.0, "transfer": {"total_h2d_ms": 1.0}},
               "chain": chain, "fixed": chain}
        arms = ["full_target", "chain", "fixed"] if i % 2 == 0 else ["fixed", "chain", "full_target"]
        rows.append(build_result_row(i, req, "query", [0, 1], [{0}, {0, 1}], out, arms=arms, gamma=4,
                                     residual=None, bytes_per_token=128, prefill_ms=3.0, protocol=proto))
    v = validate_latency_cell(rows, expected_count=4, max_unattributed_ms=100.0)
    assert v["passed"], v
    import tempfile
    from pathlib import Path

    from sparsecache_b200.serving.live import validate as validate_mod

    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "rows.jsonl"
        path.write_text("".join(json.dumps(r) + "\n" for r in rows))
        assert validate_mod.main(["latency-cell", str(path), "--expected", "4"]) == 0
        assert validate_mod.main(["latency-cell", str(path), "--expected", "5"]) == 1
    s = summarize_run(rows)
    assert s["latency"]["saved_vs_full_target_ms"]["mean"] == 10.0 and s["paired_fixed_control"] is not None
    agg = aggregate(rows)
    assert agg["token_equality_rate"] == 1.0 and agg["response_gain_ms"]["mean"] == 10.0


def test_question_attention_document_scores_match_direct_attention():
    import torch

    from sparsecache_b200.config import get_model_config
    from sparsecache_b200.pipelines.pd import question_attention_document_scores
    from sparsecache_b200.rope import apply_rope, rope_cos_sin

    cfg = get_model_config("tiny")
    g = torch.Generator().manual_seed(0)
    T, d, D, H, Hkv = 40, cfg.d_model, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    ln1 = torch.ones(d, dtype=torch.bfloat16)
    w = (torch.randn(cfg.qkv_rows, d, generator=g) * 0.05).to(torch.bfloat16)
    keys = torch.randn(Hkv, T, D, generator=g).to(torch.bfloat16)
    x = torch.randn(3, d, generator=g).to(torch.bfloat16)
    pos = torch.arange(T - 3, T)
    ranges = [(0, 10), (10, 25), (25, 37)]
    got = question_attention_document_scores(cfg, {0: x}, {0: (ln1, w)}, {0: keys}, pos, T, ranges)
    # direct: per head and row softmax over the keys of its kv head, mean over heads and rows
    xn = (x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + cfg.rms_eps)).to(torch.bfloat16) * ln1
    q = (xn.float() @ w[: cfg.q_size].float().t()).view(3, H, D).transpose(0, 1)
    cos, sin = rope_cos_sin(cfg, pos)
    q = apply_rope(q, cos, sin, sequence_dim=1)
    tok = torch.zeros(T)
    for hh in range(H):
        s = (q[hh] @ keys[hh // (H // Hkv)].float().t()) / D ** 0.5
        tok += s.softmax(-1).sum(0)
    tok /= H * 3
    want = [float(tok[b:e].sum()) for b, e in ranges]
    assert max(abs(a - b) for a, b in zip(got, want)) < 1e-5
    assert sum(got) < 1.0 + 1e-5  # the rest of the mass sits on prefix / question tokens


def _ruler_raw(tmp_path, n=3, length=2048):
    """A HotpotQA source list and RULER qa_2 rows built from it (two supporting titles per row)."""
    import random as _r

    rng = _r.Random(0)
    words = "river city king museum year born league album river tower".split()
    source, rows = [], []
    for i in range(n):
        titles = [f"Title{i}_{j}" for j in range(5)]
        source.append({"question": f"Which city is {i}?", "supporting_facts": [[titles[1], 0], [titles[3], 0]]})
        body = "\n\n".join(f"Document {j + 1}:\n{t}\n" + " ".join(rng.choice(words) for _ in range(60))
                           for j, t in enumerate(titles))
        prompt = ("<|begin_of_text|>sys " + ruler.CONTEXT_START + body + ruler.CONTEXT_END + source[-1]["question"]
                  + "<|eot_id|>")
        rows.append({"index": i, "input": prompt, "outputs": [f"city{i}"], "length": 900})
    (tmp_path / "hotpot.json").write_text(json.dumps(source))
    d = tmp_path / "raw" / str(length) / "qa_2"
    d.mkdir(parents=True)
    (d / "validation.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))


def test_evaluation_clis_end_to_end(tmp_path):
    """normalize -> RULER pack -> priority sidecars -> coverage -> audits, LongBench pack -> audit -> quality."""
    from sparsecache_b200.evaluation import cli
    from sparsecache_b200.models.checkpoint import random_checkpoint

    model = random_checkpoint(tmp_path / "model", "tiny", seed=0)
    _ruler_raw(tmp_path)
    norm = cli.main(["normalize-ruler", "--source-hotpot", str(tmp_path / "hotpot.json"), "--input-root",
                     str(tmp_path / "raw"), "--output-root", str(tmp_path / "norm"), "--lengths", "2048"])
    assert norm["2048"]["rows"] == 3 and norm["2048"]["supporting_document_counts"] == [2]
    pack = tmp_path / "packs" / "2048" / "original"
    man = cli.main(["ruler-pack", "--dataset", str(tmp_path / "norm" / "qa2_2048.jsonl"), "--placement", "original",
                    "--tokenizer", str(model), "--prompt-tokens", "2048", "--output-dir", str(pack)])
    assert man["requests"] == 3 and man["prompt_tokens"] == 2048
    audit = cli.main(["priorities", "--pack-dir", str(pack), "--output-dir", str(tmp_path / "sched"),
                      "--chunk-tokens", "128", "--protected-prefix-tokens", "128", "--protected-suffix-tokens", "128"])
    assert audit["status"] == "passed" and audit["coordinate_reconstruction_modes"] == {"pack_metadata_spans": 3}
    oracle = [json.loads(x) for x in (tmp_path / "sched" / "priority_oracle.jsonl").read_text().splitlines()]
    assert all(sorted(r["priority_chunks"]) == list(range(16)) for r in oracle)
    cov = cli.main(["priority-coverage", "--schedule-root", str(tmp_path / "sched"), "--output",
                    str(tmp_path / "cov.json"), "--fractions", "0.25,0.5", "--selection-requests", "2"])
    o, s = cov["modes"]["oracle"]["0.5"]["all"], cov["modes"]["sequential"]["0.5"]["all"]
    assert o["mean_support_chunk_recall"] >= s["mean_support_chunk_recall"] and o["requests"] == 3
    assert cov["modes"]["oracle"]["0.25"]["confirmation"]["requests"] == 1
    ar = cli.main(["audit-ruler", "--root", str(tmp_path / "packs"), "--output", str(tmp_path / "ar.json"),
                   "--lengths", "2048", "--placements", "original", "--requests-per-cell", "3"])
    assert ar["status"] == "passed"
    ar2 = cli.main(["audit-ruler", "--root", str(tmp_path / "packs"), "--output", str(tmp_path / "ar2.json"),
                    "--lengths", "2048", "--placements", "original,evidence_last", "--requests-per-cell", "3"])
    assert ar2["status"] == "failed" and ar2["failures"][0].startswith("2048/evidence_last")
    # LongBench pack, audit and the token-id quality scorer
    rows = [{"_id": f"h{i}", "input": f"Who is {i}?", "context": "Passage text. " * (40 + 30 * i),
             "answers": [f"answer {i}"]} for i in range(3)]
    (tmp_path / "hotpotqa.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    lb = cli.main(["longbench-pack", "--dataset", str(tmp_path / "hotpotqa.jsonl"), "--dataset-name", "hotpotqa",
                   "--tokenizer", str(model), "--output-dir", str(tmp_path / "lb" / "hotpotqa"),
                   "--max-prompt-tokens", "1024", "--chunk-tokens", "256", "--fixed-output-tokens", "8"])
    assert lb["requests"] == 3 and lb["prompt_tokens"]["max"] <= 1024
    assert cli.main(["audit-packs", "--root", str(tmp_path / "lb"), "--datasets", "hotpotqa", "--output",
                     str(tmp_path / "ap.json")])["status"] == "passed"
    from sparsecache_b200.tokenizer import ByteTokenizer

    tok = ByteTokenizer(1024)
    (tmp_path / "run").mkdir()
    (tmp_path / "run" / "results.jsonl").write_text("".join(
        json.dumps({"request_index": i, "token_ids": tok.encode(t, add_special_tokens=False)}) + "\n"
        for i, t in enumerate(["answer 0", "wrong", "answer 2"])))
    q = cli.main(["quality", "--result-dir", str(tmp_path / "run"), "--metadata-jsonl",
                  str(tmp_path / "lb" / "hotpotqa" / "metadata.jsonl"), "--model", str(model),
                  "--bootstrap-samples", "200"])
    assert abs(q["overall"] - 2 / 3) < 1e-9 and q["requests"] == 3


def test_live_requests_and_scheduling_queue(tmp_path):
    """Fixed-length live requests (supports whole, distractors trimmed) and the paired scheduling queue that
    pins every priority sidecar; an edited sidecar is refused."""
    from sparsecache_b200.evaluation import cli
    from sparsecache_b200.models.checkpoint import random_checkpoint
    from sparsecache_b200.serving.live import queue as q
    from sparsecache_b200.serving.live import requests as lr

    model = random_checkpoint(tmp_path / "model", "tiny", seed=0)
    _ruler_raw(tmp_path, n=4)
    cli.main(["normalize-ruler", "--source-hotpot", str(tmp_path / "hotpot.json"), "--input-root",
              str(tmp_path / "raw"), "--output-root", str(tmp_path / "norm"), "--lengths", "2048"])
    norm = tmp_path / "norm" / "qa2_2048.jsonl"
    s = lr.main(["--dataset", str(norm), "--tokenizer", str(model), "--output", str(tmp_path / "live.jsonl"),
                 "--prompt-tokens", "2048", "--num-requests", "3"])
    reqs = [json.loads(x) for x in (tmp_path / "live.jsonl").read_text().splitlines()]
    assert s["requests"] == 3 and all(len(r["prompt"]) == 2048 and r["ignore_eos"] for r in reqs)
    with pytest.raises(ValueError, match="fit exactly"):  # no row is long enough to be trimmed to 4096
        lr.main(["--dataset", str(norm), "--tokenizer", str(model), "--output", str(tmp_path / "x.jsonl"),
                 "--prompt-tokens", "4096", "--num-requests", "1"])
    pack = tmp_path / "pack"
    cli.main(["ruler-pack", "--dataset", str(norm), "--placement", "original", "--tokenizer", str(model),
              "--prompt-tokens", "2048", "--output-dir", str(pack)])
    cli.main(["priorities", "--pack-dir", str(pack), "--output-dir", str(tmp_path / "sched"), "--chunk-tokens", "128",
              "--protected-prefix-tokens", "128", "--protected-suffix-tokens", "128"])
    assert q.main(["scheduling", "--pack-dir", str(pack), "--schedule-dir", str(tmp_path / "sched"), "--run-root",
                   str(tmp_path / "runs"), "--output", str(tmp_path / "queue.json"), "--selection-requests", "2",
                   "--confirmation-requests", "2", "--warmup-requests", "0", "--tranche-fraction", "0.25",
                   "--start-fraction", "0.25"]) == 0
    queue = json.loads((tmp_path / "queue.json").read_text())
    assert len(queue["jobs"]) == 4 and queue["jobs"][0]["retrieve_fractions"] == [0.25, 0.5, 0.75, 1.0]
    job, _ = q.load_job(tmp_path / "queue.json", queue["jobs"][2]["job_id"])
    assert job["status"].startswith("blocked") and job["request_offset"] == 2
    assert set(job["priority_sidecars"]) == set(q.SCHEDULING_MODES)
    q.validate_pack_hashes(job)
    (tmp_path / "sched" / "priority_bm25.jsonl").write_text("{}\n")
    with pytest.raises(ValueError, match="bm25"):
        q.validate_pack_hashes(job)
    with pytest.raises(ValueError):
        q.fraction_schedule(0.3)


def test_pd_requests_from_packs(tmp_path):
    """P/D pipeline inputs from a RULER pack (document spans, supporting flags) and a LongBench pack
    (context pages between the recorded prefix and suffix)."""
    from sparsecache_b200.evaluation import cli
    from sparsecache_b200.models.checkpoint import random_checkpoint
    from sparsecache_b200.pipelines.pd import requests_from_pack

    model = random_checkpoint(tmp_path / "model", "tiny", seed=0)
    _ruler_raw(tmp_path, n=3)
    cli.main(["normalize-ruler", "--source-hotpot", str(tmp_path / "hotpot.json"), "--input-root",
              str(tmp_path / "raw"), "--output-root", str(tmp_path / "norm"), "--lengths", "2048"])
    pack = tmp_path / "pack"
    cli.main(["ruler-pack", "--dataset", str(tmp_path / "norm" / "qa2_2048.jsonl"), "--placement", "evidence_last",
              "--tokenizer", str(model), "--prompt-tokens", "2048", "--output-dir", str(pack)])
    rows = requests_from_pack(pack, offset=1, limit=5)
    assert [r.index for r, _ in rows] == [1, 2]
    r, flags = rows[0]
    prompt = json.loads((pack / "requests.jsonl").read_text().splitlines()[1])["prompt"]
    assert list(r.prompt) == prompt and len(r.documents) == 5 and flags == [False, False, False, True, True]
    lb_rows = [{"_id": "h0", "input": "Who?", "context": "Passage text. " * 120, "answers": ["x"]}]
    (tmp_path / "hotpotqa.jsonl").write_text(json.dumps(lb_rows[0]) + "\n")
    cli.main(["longbench-pack", "--dataset", str(tmp_path / "hotpotqa.jsonl"), "--dataset-name", "hotpotqa",
              "--tokenizer", str(model), "--output-dir", str(tmp_path / "lb"), "--max-prompt-tokens", "2048"])
    (r, flags), = requests_from_pack(tmp_path / "lb", page_tokens=256)
    meta = json.loads((tmp_path / "lb" / "metadata.jsonl").read_text())
    assert len(r.prefix) == meta["prefix_tokens"] and len(r.suffix) == meta["suffix_tokens"]
    assert all(len(d) == 256 for d in r.documents[:-1]) and 0 < len(r.documents[-1]) <= 256
    assert flags == [None] * len(r.documents) and r.prompt_tokens % 256 == 0


def test_matrix_queue_separates_selection_from_confirmation(tmp_path):
    from sparsecache_b200.pipelines import matrix_queue as mq

    matrix = {"datasets": [{"name": "qmsum", "path": "d/qmsum.jsonl", "available": 200},
                           {"name": "hotpotqa", "path": "d/hotpotqa.jsonl", "available": 200}],
              "models": [{"name": "Llama-3.1-8B-Instruct", "path": "m/llama"}, {"name": "Qwen3-8B", "path": "m/qwen"}],
              "selection_split": {"progressive_focus_cells": {"transport_gbps": [25, 50], "draft_tokens": [16],
                                                              "arrival_bundles": [4, 8]}},
              "controlled_context": {"paths": {"16000": "r/qa2_16384.jsonl"}, "evidence_placement": ["first", "last"],
                                     "requests_per_cell": 200, "primary_model_max_prompt_tokens": 131040},
              "longbench_v2": {"path": "d/lb2.json", "available": 503, "llama31_8b_max_context_tokens": 120000}}
    (tmp_path / "m.json").write_text(json.dumps(matrix))
    q = mq.main(["--matrix", str(tmp_path / "m.json"), "--run-root", str(tmp_path / "runs"),
                 "--output", str(tmp_path / "q.json")])
    assert q["counts"] == {"ready": 10, "measurement_integrity": 1, "continuous_policy_selection": 8,
                           "sparse_kernel_mechanism": 1, "confirmation_templates": 7}
    sel = [j for j in q["ready_jobs"] if j["phase"] == "continuous_policy_selection"]
    assert sel[0]["id"] == "select_llama_31_8b_instruct_qmsum_n30_bw25_g16_b4"
    cmd = sel[1]["command"]
    assert cmd[cmd.index("--stage-fractions") + 1] == mq.fractions_for_bundles(0.02, 8)
    assert "--paired-fixed-control" in cmd and cmd[cmd.index("--pack") + 1].endswith("qmsum_n30")
    assert mq.fractions_for_bundles(0.02, 4).split(",")[-1] == "1.000000"
    gate = q["ready_jobs"][0]
    assert gate["validator"][3] == "latency-cell" and "--paired-fixed-control" not in gate["command"]
    assert q["confirmation_policy"]["status"].startswith("blocked")
    assert {t["ruler_placement"] for t in q["confirmation_policy"]["templates"] if "ruler_placement" in t} == {
        "evidence_first", "evidence_last"}


def test_pd_source_aggregation_pairs_arms_and_models_the_link():
    from sparsecache_b200.pipelines import pd_source as ps

    dense = [{"request_index": i, "prompt_tokens": 8192, "prompt_sha256": f"h{i}", "seed_token_id": 5,
              "elapsed_ms": 100.0 + i} for i in range(4)]
    eagle = [{"request_index": i, "prompt_tokens": 8192, "prompt_sha256": f"h{i}", "seed_token_id": 5 + (i == 3),
              "proposal_ready_ms": 104.0 + 3 * i, "proposal_token_ids": [1, 2, 3, 4],
              "first_proposal_accepted_prefix": i} for i in range(4)]
    out = ps.aggregate_source(dense, eagle, bandwidths=(25.0, 1e6), kv_bytes_per_token=131072,
                              bootstrap_samples=200)
    assert out["samples"] == 4 and out["seed_match_fraction"] == 0.75
    assert out["source_extra_ms"]["min"] == 4.0 and out["source_extra_ms"]["max"] == 10.0
    # 8192 tokens x 128 KiB at 25 Gbit/s = 343.6 ms of transfer: every proposal is ready first
    slow = out["bandwidths"]["25"]
    assert slow["proposal_ready_before_full_kv_fraction"] == 1.0
    assert abs(slow["full_target_kv_transfer_ms"]["mean"] - 8192 * 131072 * 8 / 25e6) < 1e-6
    assert out["bandwidths"]["1e+06"]["proposal_ready_before_full_kv_fraction"] == 0.0
    assert ps.accepted_prefix([1, 2, 9], [1, 2, 3]) == 2
    eagle[0]["prompt_sha256"] = "other"
    with pytest.raises(ValueError, match="hashes"):
        ps.aggregate_source(dense, eagle, bandwidths=(25.0,), kv_bytes_per_token=1)
    with pytest.raises(ValueError, match="different requests"):
        ps.aggregate_source(dense, eagle[:3], bandwidths=(25.0,), kv_bytes_per_token=1)


def test_reuse_pipeline_dataset_requests_and_scoring(tmp_path):
    """MuSiQue rows become prefix / one document per paragraph / question requests with texts and supporting
    flags for the schedules; arms are scored against the gold answers."""
    from sparsecache_b200.config import get_model_config
    from sparsecache_b200.pipelines import reuse

    rows = [{"id": f"q{i}", "question": f"Where is {i}?", "answer": f"place {i}", "answer_aliases": ["p"],
             "question_decomposition": [{}] * 2,
             "paragraphs": [{"title": f"T{j}", "paragraph_text": f"text {i} {j}", "is_supporting": j == 1}
                            for j in range(3)]} for i in range(4)]
    (tmp_path / "m.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    cfg = get_model_config("tiny")
    reqs, meta = reuse.dataset_requests(tmp_path / "m.jsonl", cfg, sample_count=3, seed=0, limit=2)
    assert len(reqs) == 2 and len(reqs[0].documents) == 3 and meta[0]["supporting"] == [False, True, False]
    r, m = reqs[0], meta[0]
    assert meta[0]["decode"](list(r.documents[1])).endswith(m["texts"][1].split("\n")[-1])
    prep = reuse.prepare_request(r, schedule="oracle", fractions=(0.34, 1.0), question=m["question"],
                                 texts=m["texts"], supporting=m["supporting"])
    assert prep.ranking[0] == 1  # the supporting paragraph first
    from sparsecache_b200.tokenizer import ByteTokenizer

    tok = ByteTokenizer(cfg.vocab)
    row = {"arms": {"full": {"tokens": tok.encode("place 7", add_special_tokens=False) + [2, 50]},
                    "cacheblend": {"tokens": tok.encode("nowhere", add_special_tokens=False)}}}
    reuse.score_row(row, {**m, "golds": ["place 7"]}, {2})
    assert row["arms"]["full"]["em"] == 1.0 and row["arms"]["cacheblend"]["f1"] == 0.0


def test_pd_rows_scored_with_the_pack_metric():
    from sparsecache_b200.pipelines.pd import score_pack_row

    row = {"schedules": {"query": {"full_target": {"timing_token_ids": [1, 2]},
                                   "chains": {"inf": {"timing_token_ids": [3],
                                                      "paired_fixed_control": {"timing_token_ids": [1, 2]}}}}}}
    text = {(1, 2): "Paris", (3,): "Rome"}
    score_pack_row(row, {"dataset": "hotpotqa", "answers": ["Paris"]}, lambda ids: text[tuple(ids)])
    cell = row["schedules"]["query"]
    assert cell["full_target"]["score"] == 1.0 and cell["full_target"]["metric"] == "qa_f1"
    assert cell["chains"]["inf"]["score"] == 0.0 and cell["chains"]["inf"]["paired_fixed_control"]["score"] == 1.0


def test_reuse_aggregate_command_over_shards(tmp_path):
    from sparsecache_b200.pipelines import reuse

    def row(i, same):
        full = [5, 6, 7]
        return {"request_index": i, "prompt_tokens": 100, "document_tokens": 80,
                "arms": {"full": {"tokens": full, "ttft_ms": 20.0, "e2e_ms": 50.0, "em": 1.0, "f1": 1.0},
                         "cacheblend": {"tokens": full if same else [5, 9, 7], "ttft_ms": 8.0, "e2e_ms": 40.0,
                                        "em": float(same), "f1": float(same)}}}

    (tmp_path / "a.jsonl").write_text(json.dumps({"protocol": {"model": "m"}}) + "\n"
                                      + "".join(json.dumps(row(i, i % 2 == 0)) + "\n" for i in range(4)))
    (tmp_path / "b.jsonl").write_text("".join(json.dumps(row(i, True)) + "\n" for i in range(4, 6)))
    out = reuse.aggregate_main([str(tmp_path / "a.jsonl"), str(tmp_path / "b.jsonl"), "--output",
                                str(tmp_path / "agg.json"), "--bootstrap-samples", "100"])
    cb = out["summary"]["arms"]["cacheblend"]
    assert out["summary"]["requests"] == 6 and out["protocol"] == {"model": "m"}
    assert abs(cb["token_equal_rate"] - 4 / 6) < 1e-9 and abs(cb["em"] - 4 / 6) < 1e-9
    assert cb["ttft_gain_vs_reference_ms"]["mean"] == 12.0
    with pytest.raises(ValueError, match="duplicate"):
        reuse.aggregate_main([str(tmp_path / "b.jsonl"), str(tmp_path / "b.jsonl"), "--output", str(tmp_path / "x")])
