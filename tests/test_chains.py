"""Progressive commit-window and graft chains on a deterministic CPU stage model:
every chain's output equals full-KV greedy decoding (the exactness gate of the
reference's progressive chains), with the trace invariants of each stage."""
import pytest

from sparsecache_b200.serving.chains import ToyStageModel, progressive_commit_chain, progressive_graft_chain


@pytest.mark.parametrize("window", [1, 2, None])
@pytest.mark.parametrize("seed", range(6))
def test_commit_chain_is_exact(window, seed):
    m = ToyStageModel(n_stages=4, flip_rate=0.5, seed=seed)
    want = m.final_decode([], 24)
    out = progressive_commit_chain(m, commit_window=window, draft_tokens=6, max_new_tokens=24)
    assert len(out.tokens) == 24
    if window is None:  # only the full-KV verifier commits: exact
        assert out.tokens == want and out.ignored_committed_flips == 0
    else:  # a finite window freezes tokens that survived W noisy verifications
        first_bad = next((i for i, (a, b) in enumerate(zip(out.tokens, want)) if a != b), 24)
        assert first_bad == 24 or out.trace[-1]["committed_before"] > first_bad
    for row in out.trace:
        assert row["accepted_pending"] + row["rejected_pending"] == (row["pending_before"] if row["verified"] else 0)
        assert row["committed_after"] >= row["committed_before"]
    assert out.trace[0]["drafted"] == 6 and not out.trace[0]["verified"]


def test_commit_chain_stops_at_eos():
    m = ToyStageModel(n_stages=3, flip_rate=0.0, seed=1)
    full = m.final_decode([], 30)
    eos = {full[4]}
    out = progressive_commit_chain(m, commit_window=1, draft_tokens=8, max_new_tokens=30, eos_ids=eos)
    assert out.tokens == full[:full.index(full[4]) + 1]


def test_graft_chain_is_exact_and_verifies_once():
    for seed in range(5):
        m = ToyStageModel(n_stages=4, flip_rate=0.4, seed=seed)
        out = progressive_graft_chain(m, draft_tokens_per_stage=3, max_new_tokens=20)
        assert out.tokens == m.final_decode([], 20) and out.verifications == 1


def test_reuse_pipeline_helpers():
    from sparsecache_b200.pipelines.reuse import aggregate, expand_documents, prepare_request
    from sparsecache_b200.synthetic import RAGRequest

    docs = expand_documents([[1, 2, 3], [4, 5]], target_tokens=20, prefix_tokens=2)
    assert sum(map(len, docs)) + 2 >= 20 and docs[0][:3] == [1, 2, 3]
    req = RAGRequest(0, (9, 9), ((1, 2, 3, 4), (5, 6), (7, 8, 9, 10, 11, 12)), (13,))
    prep = prepare_request(req, schedule="sequential", fractions=(0.3, 0.7, 1.0))
    assert prep.ranking == [0, 1, 2] and prep.selected_sets[-1] == {0, 1, 2}
    assert all(a <= b for a, b in zip(prep.selected_sets, prep.selected_sets[1:]))
    rows = [{"request_index": i, "arms": {"full": {"tokens": [1, 2, 3], "ttft_ms": 10.0, "e2e_ms": 20.0},
                                          "progressive": {"tokens": [1, 2, 4], "ttft_ms": 5.0, "e2e_ms": 18.0}}}
            for i in range(3)]
    agg = aggregate(rows, bootstrap_samples=100)
    assert agg["arms"]["progressive"]["token_equal_rate"] == 0.0
    assert agg["arms"]["progressive"]["mean_agreeing_prefix"] == 2.0
    assert agg["arms"]["progressive"]["ttft_gain_vs_reference_ms"]["mean"] == 5.0


def test_layer_subset_patterns(tmp_path):
    import json
    from pathlib import Path

    import pytest

    from sparsecache_b200.pipelines.screens import load_patterns, sandwich_layers, standard_patterns, uniform_layers

    assert uniform_layers(32, 8) == [0, 4, 9, 13, 18, 22, 27, 31]
    assert sandwich_layers(32, 8) == [0, 1, 2, 3, 28, 29, 30, 31]
    assert len(uniform_layers(32, 24)) == 24 and uniform_layers(80, 16)[-1] == 79
    root = Path(__file__).resolve().parents[1] / "configs"
    pats = load_patterns(root / "layer_subset_patterns_llama31_8b.json", 32)
    assert pats["uniform16"] == uniform_layers(32, 16) and set(pats) == {p["id"] for p in standard_patterns(32)["patterns"]}
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps({"schema_version": 1, "patterns": [{"id": "x", "layer_indices": [3, 1]}]}))
    with pytest.raises(ValueError):
        load_patterns(bad, 32)


def test_crossover_queue_is_fail_closed(tmp_path):
    import json

    import pytest

    from sparsecache_b200.pipelines.screens import build_crossover_queue, run_crossover_job

    q = build_crossover_queue(model="llama3-8b", contexts=[8192, 32768], fractions=[0.05, 0.2],
                              run_root=str(tmp_path / "runs"))
    qp = tmp_path / "queue.json"
    qp.write_text(json.dumps(q))
    calls = []

    def runner(cmd, out):
        calls.append(cmd)
        out.write_text("{}")
        return 0

    rec = run_crossover_job(qp, "crossover_llama3-8b_ctx8192", gate=lambda: {"passed": True}, runner=runner)
    assert rec["exit_code"] == 0 and calls[0][:3] == ["python", "-m", "sparsecache_b200.pipelines.screens"]
    assert (tmp_path / "runs" / "crossover_llama3-8b_ctx8192" / "run_record.json").exists()
    with pytest.raises(RuntimeError):  # GPUs busy
        run_crossover_job(qp, "crossover_llama3-8b_ctx32768", gate=lambda: {"passed": False}, runner=runner)
    q["jobs"][1]["command"].append("--extra")  # edited after registration
    qp.write_text(json.dumps(q))
    with pytest.raises(ValueError):
        run_crossover_job(qp, "crossover_llama3-8b_ctx32768", gate=lambda: {"passed": True}, runner=runner)
    assert len(calls) == 1


def test_crossover_schedule_and_aggregate():
    import pytest

    from sparsecache_b200.pipelines.screens import (aggregate_crossover, balanced_fraction_schedule,
                                                    measurement_seed_token, parse_fractions)

    fr = parse_fractions("1,.1,.02")
    sched = balanced_fraction_schedule(fr, 4)
    assert len(sched) == 12
    for r in range(4):
        assert {f for rr, _, f in sched if rr == r} == set(fr)
    assert [x[2] for x in sched[:3]] != [x[2] for x in sched[3:6]]
    with pytest.raises(ValueError, match="include"):
        parse_fractions(".02,.1")
    assert measurement_seed_token(128256, 0) == 1024 and measurement_seed_token(128256, 1) == 1025
    rows = [{"context_tokens": 1024, "requested_fraction": f, "visible_fraction": f, "repeat": r,
             "draft_step_ms": 8.0 if f == 0.1 else (13.0 if f == 0.5 else 12.0)}
            for r in range(3) for f in (0.1, 0.5, 1.0)]
    agg = aggregate_crossover(rows)["1024"]
    assert agg["crossover_fraction"] == 0.1 and agg["fractions"]["0.1"]["speedup_vs_full_mean"] == 1.5
    with pytest.raises(ValueError, match="incomplete"):
        aggregate_crossover(rows[:-1])


def test_tp_shared_buffers_carry_guard_bands(monkeypatch, tmp_path):
    """Peer-mapped buffers sit between guard bands; an overrun into a band is reported
    (host logic with a fake extension and one gloo rank)."""
    import torch
    import torch.distributed as dist

    from sparsecache_b200 import ops
    from sparsecache_b200.parallel import tp

    class FakeExt:
        def shared_empty(self, nbytes, device):
            return torch.zeros(nbytes, dtype=torch.uint8), b"handle"

        def shared_open(self, handle):  # pragma: no cover - one rank opens nothing
            raise AssertionError

    monkeypatch.setattr(ops, "ext", lambda: FakeExt())
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    dist.init_process_group("gloo", init_method=f"file://{tmp_path / 'store'}", rank=0, world_size=1)
    try:
        g = tp.TPGroup()
        buf, ptrs = g.shared(100)
        buf2, _ = g.shared(64)
        assert buf.numel() == 100 and ptrs == [buf.data_ptr()] and buf.data_ptr() % 16 == 0
        buf.fill_(7)
        buf2.fill_(9)
        assert g.check_canaries() == []
        g._guards[1][0][tp.CANARY_BYTES + 64] = 0  # one byte past the second buffer
        assert g.check_canaries() == [1]
    finally:
        dist.destroy_process_group()


def test_speculative_loop_host_logic():
    """speculative_generate with a fake verifier (the greedy sequence is known) and a drafter
    that is right for the first k drafts: the output is the greedy sequence and the accepted
    counts / positions follow the accept-longest-prefix rule."""
    from types import SimpleNamespace

    import torch

    from sparsecache_b200.models.engine import _Workspace
    from sparsecache_b200.parallel.tp_draft import speculative_generate

    truth = [(7 * i + 3) % 50 for i in range(40)]  # token at position T + i
    T = 100

    class Eng:
        MAX_ROWS = 8

        def __init__(self):
            self.ws = _Workspace("cpu")
            self.bufs = {"log": torch.zeros(64, dtype=torch.int32), "tok": torch.zeros(8, dtype=torch.int32)}

        def _decode_buffers(self, *a):
            return self.bufs

    calls = []

    class TPE:
        engine = Eng()
        seed_layers = (0, 1, 2)
        full_cfg = SimpleNamespace(d_model=4)

        def verify(self, slot, rows, position, use_graph=True):
            rows = rows.tolist()
            calls.append((position, rows))
            assert rows[0] == truth[position - T]  # row 0 is the token at ``position``
            out = torch.tensor([truth[position - T + 1 + i] for i in range(len(rows))], dtype=torch.int32)
            self.engine.bufs["tok"][:len(rows)] = out
            return out

        def check_status(self):
            pass

    class Drafter:
        gamma = 4

        def __init__(self, right):
            self.right = right

        def propose(self, slot, first, seed_row, position, use_graph=True):
            assert int(first[0]) == truth[position - T]
            d = [truth[position - T + 1 + i] for i in range(4)]
            for i in range(self.right, 4):
                d[i] = (d[i] + 1) % 50
            return torch.tensor(d, dtype=torch.int32)

    tpe = TPE()
    tpe.engine.bufs["log"][0] = truth[0]
    for right in (0, 2, 4):
        calls.clear()
        out = speculative_generate(tpe, Drafter(right), None, prompt_tokens=T, max_new=20)
        assert out["tokens"] == truth[:20]
        assert all(a == right for a in out["accepted"][:-1])
        # every verify after the first starts right after the previously committed tokens
        assert [p for p, _ in calls][:3] == [T, T + 1, T + 2 + right]


def test_page_view_sink_recent_and_budget():
    from sparsecache_b200.pipelines.screens import page_view

    T = 32768
    v = page_view(T, 0.05)
    idx = v.tolist()
    assert idx == sorted(set(idx)) and idx[-1] == T - 1
    assert set(range(64)) <= set(idx) and set(range(T - 512, T)) <= set(idx)  # sink and recent always visible
    assert abs(len(idx) / T - 0.05) < 0.01
    small = page_view(T, 0.001)  # the budget never drops below sink + recent
    assert len(small) >= 64 + 512
