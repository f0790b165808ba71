"""Live 1P1D harness on the CPU: resource gate, proxy request rules, the
whole proxy -> prefill -> store-completion -> decode chain in process with
the toy worker, the paired client, validity-gated aggregation, the
input-trace audit, queue registration and the launcher's process control
(behaviours of the reference's test_progressive_pd_proxy.py,
test_progressive_pd_resource_gate.py, test_aggregate_progressive_pd_live.py,
test_verify_progressive_pd_input_trace.py, test_progressive_pd_live_queue.py
and test_run_progressive_pd_live_job.py)."""
import asyncio
import json
import time
import os
import sys

import httpx
import pytest

from sparsecache_b200.serving.live import aggregate, client, gate, launcher, proxy, queue, trace
from sparsecache_b200.serving.live.worker import TelemetrySink, ToyWorker, make_app

GPU_QUERY = ("0, GPU-a, NVIDIA B200, 12, 183359, 0, P8, 31, 140.5\n"
             "1, GPU-b, NVIDIA B200, 120000, 183359, 99, P0, 72, 950.0\n")
PROC_QUERY = "GPU-b, 1234, python, 119000\n"


def test_resource_gate():
    cmds = []

    def runner(cmd):
        cmds.append(cmd)
        return GPU_QUERY if cmd[1].startswith("--query-gpu=") else PROC_QUERY

    states = gate.inspect_gpus(command_runner=runner)
    assert len(cmds) == 2 and not states[0].compute_processes
    assert states[1].compute_processes[0]["pid"] == 1234
    ok = gate.evaluate_exclusivity(states, (0,), max_used_memory_mib=1024, max_utilization_pct=5)
    bad = gate.evaluate_exclusivity(states, (1,), max_used_memory_mib=1024, max_utilization_pct=5)
    assert ok["status"] == "passed" and bad["status"] == "failed"
    assert {f["reason"] for f in bad["failures"]} == {"compute_processes_present", "memory_used_above_threshold",
                                                       "utilization_above_threshold"}
    assert gate.parse_compute_query("No running processes found") == {}
    assert gate.parse_compute_query("GPU-b, 7, x, [N/A]\n") == {"GPU-b": [
        {"pid": 7, "process_name": "x", "used_gpu_memory_mib": None}]}
    with pytest.raises(ValueError, match="unexpected nvidia-smi GPU row"):
        gate.parse_gpu_query("0, GPU-a\n")
    with pytest.raises(ValueError, match="no GPUs"):
        gate.parse_gpu_query("")
    with pytest.raises(ValueError, match="non-empty unique"):
        gate.evaluate_exclusivity(states, (0, 0), max_used_memory_mib=1024, max_utilization_pct=5)
    with pytest.raises(ValueError, match="do not exist"):
        gate.evaluate_exclusivity(states, (0, 5), max_used_memory_mib=1024, max_utilization_pct=5)
    # the thresholds are inclusive limits: exactly at the limit passes
    edge = gate.evaluate_exclusivity(states, (0,), max_used_memory_mib=12, max_utilization_pct=0)
    assert edge["status"] == "passed" and edge["requested_gpus"] == [0]


def test_runtime_monitor_finds_foreign_processes():
    """The runtime watch ignores the run's own service tree and reports the first
    compute process outside it (or a GPU that vanished)."""
    parents = {500: 400, 400: 300, 300: 1, 900: 1}
    procs = {"text": ""}

    def runner(cmd):
        return GPU_QUERY if cmd[1].startswith("--query-gpu=") else procs["text"]

    mon = gate.ExclusivityMonitor([0, 1], service_roots=[300], command_runner=runner, parent_of=parents.get)
    assert mon.check() is None
    procs["text"] = "GPU-a, 500, python, 100\n"  # grandchild of the service root: owned
    assert mon.check() is None
    procs["text"] = "GPU-a, 500, python, 100\nGPU-b, 900, intruder, 2000\n"
    found = mon.check()
    assert found["reason"] == "foreign_compute_process" and found["pid"] == 900 and found["gpu"] == 1
    gone = gate.ExclusivityMonitor([3], service_roots=[300], command_runner=runner, parent_of=parents.get)
    assert gone.check()["reason"] == "gpu_disappeared"
    # the daemon thread reports once and stops
    hits = []
    mon2 = gate.ExclusivityMonitor([1], service_roots=[300], command_runner=runner, parent_of=parents.get,
                                   interval_s=0.01)
    mon2.start(hits.append)
    deadline = time.time() + 5
    while not hits and time.time() < deadline:
        time.sleep(0.01)
    mon2.stop()
    assert len(hits) == 1 and hits[0]["pid"] == 900 and mon2.finding == hits[0]
    assert gate.parent_pid(os.getpid()) == os.getppid()


def test_launcher_stops_the_cell_on_interference(tmp_path):
    """A foreign compute process during the run stops every launched process
    group and fails the run with the monitor's finding."""
    pack = tmp_path / "pack"
    pack.mkdir()
    (pack / "requests.jsonl").write_text('{"prompt": [1]}\n')
    (pack / "metadata.jsonl").write_text('{}\n')
    job = queue.build_job(job_id="j", phase="p", status="s", pack_dir=pack, run_dir=tmp_path / "run", requests=1,
                          request_offset=0, warmups=0, bandwidth_gbps=25)
    spec = [{"name": "svc", "argv": [sys.executable, "-c", "import time; time.sleep(60)"], "env": {}}]
    intruder = {"on": False}

    def runner(cmd):
        if cmd[1].startswith("--query-gpu="):
            return GPU_QUERY
        return "GPU-a, 424242, intruder, 10\n" if intruder["on"] else ""

    def make_monitor(pids):
        return gate.ExclusivityMonitor([0], pids, command_runner=runner, parent_of=lambda p: 1, interval_s=0.02)

    def client():
        intruder["on"] = True
        deadline = time.time() + 5
        while time.time() < deadline:  # the cell keeps running until the monitor stops it
            time.sleep(0.02)
        return {"requests": 1}

    t0 = time.time()
    man = launcher.execute(job, tmp_path / "run", spec=spec, monitor=make_monitor, run_client=client)
    assert man["status"] == "failed" and "interference" in man["error"] and "424242" in man["error"]
    assert man["runtime_monitor"]["finding"]["reason"] == "foreign_compute_process"
    assert time.time() - t0 < 30


CFG = proxy.ProxyConfig()


def test_proxy_request_rules():
    req = {"model": "m", "prompt": [1, 2], "max_tokens": 32, "temperature": 0, "stream": True,
           "sparsecache_mode": "progressive", "sparsecache_priority_chunks": [3, 0, 2, 1]}
    pre, dec, mode = proxy.prepare_requests(req, CFG, 123)
    assert mode == "progressive" and pre["max_tokens"] == 1 and pre["stream"] is False
    assert pre["return_token_ids"] is True and dec["max_tokens"] == 32 and dec["stream"] is True
    assert dec["kv_transfer_params"]["progressive_sparse_draft"] == {
        "seed_token_id": 123, "max_draft_tokens": 8, "start_fraction": 0.05, "visibility_mode": "continuous"}
    assert dec["kv_transfer_params"]["progressive_priority_chunks"] == [3, 0, 2, 1]
    assert not any(k.startswith("sparsecache_") for k in list(pre) + list(dec))
    _, dec, _ = proxy.prepare_requests({**req, "sparsecache_mode": "baseline"}, CFG, 123)
    assert dec["kv_transfer_params"] == {"producer_seed_token_id": 123, "require_full_remote_kv": True}
    for bad in ({"temperature": 0.7}, {"sparsecache_max_draft_tokens": 0}, {"sparsecache_start_fraction": 1.0},
                {"sparsecache_priority_chunks": [1, 1]}, {"sparsecache_mode": "x"},
                {"kv_transfer_params": {"require_full_remote_kv": False}}):
        with pytest.raises(ValueError):
            proxy.prepare_requests({**req, **bad}, CFG, 1)
    assert proxy.prefill_fingerprint("/v1/completions", pre) != proxy.prefill_fingerprint("/v1/chat/completions", pre)
    assert proxy.extract_seed_token({"choices": [{"token_ids": [7]}]}) == 7
    with pytest.raises(RuntimeError):
        proxy.extract_seed_token({"choices": []})


def _stack(tmp_path):
    sink = TelemetrySink(tmp_path / "telemetry")
    worker = ToyWorker(telemetry=sink)
    holder = {}
    p_app = make_app(worker, "prefill", notify=lambda rid: holder["proxy"].notify(rid))
    d_app = make_app(worker, "decode")
    apps = {CFG.prefiller_url: p_app, CFG.decoder_url: d_app}
    px = proxy.Proxy(CFG, client_factory=lambda url: httpx.AsyncClient(transport=httpx.ASGITransport(app=apps[url]),
                                                                      base_url=url))
    holder["proxy"] = px
    return px, sink


def test_full_chain_paired_run_aggregate_and_trace(tmp_path):
    px, sink = _stack(tmp_path)
    reqs = [{"model": "toy", "prompt": list(range(1 + i, 40 + i)), "max_tokens": 12, "temperature": 0}
            for i in range(4)]

    async def go():
        async with httpx.AsyncClient(transport=httpx.ASGITransport(app=px.app), base_url="http://proxy") as c:
            return await client.run_benchmark(c, "/v1/completions", reqs, ("baseline", "fixed_s1", "continuous"),
                                              warmup=1, output=tmp_path / "results.jsonl", run_id="t")

    records, summ = asyncio.run(go())
    assert summ["pairs"] == 4
    assert summ["comparisons"]["baseline_vs_continuous"]["token_equality_rate"] == 1.0
    r0 = records[0]
    assert r0["prefill_group"] and isinstance(r0["seed_token_id"], int) and len(r0["token_ids"]) == 12
    reused = [r["prefill_reused"] for r in records if r["request_index"] == 0]
    assert sorted(reused) == [False, True, True]  # one producer prefill per paired execution
    meta = [{"request_index": i, "dataset": "hotpotqa", "answers": ["x"]} for i in range(4)]
    summary, rows = aggregate.aggregate_live_run(
        records, meta, sink.records["scheduler"], sink.records["link"], attention_rows=sink.records["attention"],
        arms=("baseline", "fixed_s1", "continuous"),
        expected_requests=4, fixed_output_tokens=12, bootstrap_samples=200, seed=0, protected_chunks=1)
    failed = {k: v for k, v in summary["gates"].items() if not v["passed"]}
    # the warm-up execution's scheduler/link records belong to other proxy ids; all gates hold
    assert not failed, failed
    aggregate.write_artifacts(tmp_path / "agg", summary, rows)
    assert (tmp_path / "agg" / "paper_table.csv").exists()
    # the same run through the aggregator's command line
    for name, recs in (("meta", meta), ("sched", sink.records["scheduler"]), ("link", sink.records["link"]),
                       ("attn", sink.records["attention"])):
        (tmp_path / f"{name}.jsonl").write_text("".join(json.dumps(r) + "\n" for r in recs))
    rc = aggregate.main(["--results", str(tmp_path / "results.jsonl"), "--metadata", str(tmp_path / "meta.jsonl"),
                         "--scheduler-trace", str(tmp_path / "sched.jsonl"), "--link-trace",
                         str(tmp_path / "link.jsonl"), "--attention-trace", str(tmp_path / "attn.jsonl"),
                         "--expected-requests", "4", "--fixed-output-tokens", "12",
                         "--bootstrap-samples", "200", "--protected-chunks", "1", "--output-dir",
                         str(tmp_path / "agg_cli")])
    assert rc == 0 and (tmp_path / "agg_cli" / "summary.md").exists()
    # input-trace audit of every progressive request
    n_prog = len(sink.records["scheduler"])
    rep = trace.verify_input_trace(sink.records["scheduler"], sink.records["input_trace"], expected_requests=n_prog)
    assert rep["status"] == "passed" and rep["verify_forwards"] == n_prog


def test_prefill_group_reused_for_another_prompt_is_refused(tmp_path):
    px, _ = _stack(tmp_path)

    async def go():
        async with httpx.AsyncClient(transport=httpx.ASGITransport(app=px.app), base_url="http://proxy") as c:
            base = {"model": "toy", "max_tokens": 2, "temperature": 0, "sparsecache_prefill_group": "g"}
            r1 = await c.post("/v1/completions", json={**base, "prompt": [1, 2, 3]})
            r2 = await c.post("/v1/completions", json={**base, "prompt": [4, 5, 6]})
            r3 = await c.post("/v1/completions", json={**base, "prompt": [1, 2, 3], "temperature": 0.5})
            return r1, r2, r3

    r1, r2, r3 = asyncio.run(go())
    assert r1.status_code == 200 and r1.headers["x-sparsecache-prefill-reused"] == "false"
    assert r2.status_code == 409 and r3.status_code == 400
    assert "store_wait;dur=" in r1.headers["server-timing"]


def test_aggregate_gates_catch_protocol_violations(tmp_path):
    base = {"source_request_index": 0, "warmup": False, "header_ms": 1.0, "ttft_ms": 2.0, "decode_ttft_ms": 1.0,
            "completion_ms": 5.0, "decode_completion_ms": 4.0, "token_arrival_ms": [2.0, 1.0], "token_ids": [1, 2],
            "text": "", "prefill_group": "g", "prefill_reused": False, "seed_token_id": 1}
    results = [{**base, "request_index": 0, "arm": "baseline", "runtime_mode": "baseline", "proxy_request_id": "a"},
               {**base, "request_index": 0, "arm": "continuous", "runtime_mode": "progressive",
                "proxy_request_id": "b", "token_ids": [1, 3], "prefill_reused": False}]
    summary, _ = aggregate.aggregate_live_run(results, [{"request_index": 0, "answers": ["a"]}], [], [],
                                              arms=("baseline", "continuous"), expected_requests=1,
                                              bootstrap_samples=50)
    g = summary["gates"]
    assert not g["request_protocol"]["passed"]  # non-monotonic arrivals
    assert not g["single_paired_prefill"]["passed"]  # two fresh prefills
    assert not g["exact_greedy_output_equivalence"]["passed"]
    assert not g["one_scheduler_transition_per_method"]["passed"] and summary["status"] == "failed_gates"
    assert aggregate.percentile([1, 2, 3, 4], 0.5) == 2.5


def test_trace_audit_rejects_wrong_inputs():
    sch = [{"request_id": "r", "seed_token_id": 5, "draft_token_ids": [6, 7], "draft_tokens": 2,
            "max_draft_tokens": 2, "started_at_ns": 0, "last_draft_at_ns": 20, "full_arrival_at_ns": 30,
            "verify_started_at_ns": 40, "verify_completed_at_ns": 60}]
    good = [{"request_id": "r", "recorded_at_ns": 10, "input_token_ids": [5], "positions": [9],
             "num_scheduled_tokens": 1},
            {"request_id": "r", "recorded_at_ns": 20, "input_token_ids": [6], "positions": [10],
             "num_scheduled_tokens": 1},
            {"request_id": "r", "recorded_at_ns": 50, "input_token_ids": [5, 6, 7], "positions": [9, 10, 11],
             "num_scheduled_tokens": 3}]
    assert trace.verify_input_trace(sch, good, expected_requests=1)["status"] == "passed"
    bad = [dict(r) for r in good]
    bad[2] = {**bad[2], "positions": [10, 11, 12]}
    with pytest.raises(ValueError, match="rewind"):
        trace.verify_input_trace(sch, bad, expected_requests=1)
    bad = [dict(r) for r in good]
    bad[1] = {**bad[1], "input_token_ids": [8]}
    with pytest.raises(ValueError, match="sparse chain"):
        trace.verify_input_trace(sch, bad, expected_requests=1)


def test_queue_registration_and_hash_checks(tmp_path):
    pack = tmp_path / "pack"
    pack.mkdir()
    (pack / "requests.jsonl").write_text("".join(json.dumps({"prompt": [i]}) + "\n" for i in range(10)))
    (pack / "metadata.jsonl").write_text("".join(json.dumps({"i": i}) + "\n" for i in range(10)))
    q = queue.build_queue([{"name": "ruler16k", "pack_dir": str(pack)}], tmp_path / "runs", bandwidths=(25, 100),
                          core_requests=6, confirmation_requests=4, warmup_requests=1, max_draft_tokens=8)
    assert len(q["jobs"]) == 4
    qp = tmp_path / "queue.json"
    qp.write_text(json.dumps(q))
    job, _ = queue.load_job(qp, "confirm_ruler16k_bw25_n4_offset6")
    assert job["request_offset"] == 6 and queue.validate_pack_hashes(job)
    (tmp_path / "packs.json").write_text(json.dumps([{"name": "ruler16k", "pack_dir": str(pack)}]))
    assert queue.main(["--packs", str(tmp_path / "packs.json"), "--run-root", str(tmp_path / "runs"),
                       "--bandwidths", "25,100", "--core-requests", "6", "--confirmation-requests", "4",
                       "--warmup-requests", "1", "--output", str(tmp_path / "q2.json")]) == 0
    assert json.loads((tmp_path / "q2.json").read_text())["jobs_sha256"] == q["jobs_sha256"]
    (pack / "metadata.jsonl").write_text("changed\n")
    with pytest.raises(ValueError):
        queue.validate_pack_hashes(job)
    with pytest.raises(ValueError):
        queue.build_queue([{"name": "x", "pack_dir": str(pack)}], tmp_path, bandwidths=(1,), core_requests=20,
                          confirmation_requests=1, warmup_requests=0, max_draft_tokens=1)


def test_launcher_process_control_and_fail_closed(tmp_path):
    mp = launcher.spawn("sleeper", [sys.executable, "-c", "import time; time.sleep(60)"], tmp_path)
    assert mp.popen.poll() is None
    launcher.stop([mp], timeout_s=5)
    assert mp.popen.poll() is not None
    crash = launcher.spawn("crash", [sys.executable, "-c", "raise SystemExit(3)"], tmp_path)
    crash.popen.wait()
    with pytest.raises(RuntimeError, match="exited"):
        launcher.fatal_startup([crash])
    pack = tmp_path / "pack"
    pack.mkdir()
    (pack / "requests.jsonl").write_text('{"prompt": [1]}\n')
    (pack / "metadata.jsonl").write_text('{}\n')
    job = queue.build_job(job_id="j", phase="p", status="s", pack_dir=pack, run_dir=tmp_path / "run", requests=1,
                          request_offset=0, warmups=0, bandwidth_gbps=25)
    man = launcher.execute(job, tmp_path / "run", gate=lambda: {"status": "failed"})
    assert man["status"] == "failed" and "gate" in man["error"]
    assert (tmp_path / "run" / "run_manifest.json").exists()


def test_scheduling_benchmark_shares_one_prefill(tmp_path):
    from sparsecache_b200.evaluation.priorities import priority_for_mode
    from sparsecache_b200.serving.live import validate

    px, _ = _stack(tmp_path)
    reqs = [{"model": "toy", "prompt": list(range(3 + i, 600 + i)), "max_tokens": 6, "temperature": 0}
            for i in range(2)]
    pri = {s: {i: priority_for_mode(s, request_id=str(i), question="q", documents=[{"text": "a", "supporting": True}],
                                    spans=[{"start_token": 0, "end_token": 256}], total_chunks=3, chunk_tokens=256,
                                    protected_prefix_chunks=1, protected_suffix_chunks=1, seed=0)
               for i in range(2)} for s in validate.SCHEDULES}

    async def go():
        async with httpx.AsyncClient(transport=httpx.ASGITransport(app=px.app), base_url="http://proxy") as c:
            return await validate.run_scheduling_benchmark(c, "/v1/completions", reqs, pri)

    recs = asyncio.run(go())
    assert len(recs) == 2 * 5 * 2
    agg = validate.aggregate_scheduling(recs, expected_requests=2, bootstrap_samples=50)
    assert agg["status"] == "passed", agg["gates"]
    assert sum(r["prefill_reused"] is False for r in recs) == 2


def test_latency_cell_validator():
    from sparsecache_b200.serving.live.validate import validate_latency_cell

    def row(i, order):
        return {"dataset_index": i, "protocol": {"fixed_token_horizon": True, "paired_measurement": True,
                                                 "require_exclusive_gpu": True, "initial_gpu_used_bytes": 0},
                "schedules": {"uniform": {"full_target": {"timing_token_ids": [1, 2]},
                                          "chains": {"inf": {"measurement_order": order, "timing_token_ids": [1, 2],
                                                             "pipeline": {"response_ms": 50.0, "verify_ms": 10.0,
                                                                          "final_decode_ms": 30.0}}}}}}

    ok = validate_latency_cell([row(0, "full_target_then_pipeline"), row(1, "pipeline_then_full_target")],
                               expected_count=2)
    assert ok["passed"], ok["failures"]
    bad = validate_latency_cell([row(0, "full_target_then_pipeline"), row(0, "full_target_then_pipeline"),
                                 row(2, "full_target_then_pipeline")], expected_count=2, max_unattributed_ms=5.0)
    assert not bad["passed"] and len(bad["failures"]) >= 3


def test_proposal_trace_is_atomic_and_first_writer_wins(tmp_path):
    import json

    import torch

    from sparsecache_b200.serving.live.trace import publish_proposal_trace

    dest = tmp_path / "proposal.json"
    rec = publish_proposal_trace(dest, method="eagle3", proposal_started_at_ns=1,
                                 seed_token_ids=torch.tensor([17], dtype=torch.int32),
                                 draft_token_ids=torch.tensor([[18, 19, 20]], dtype=torch.int32))
    stored = json.loads(dest.read_text())
    assert rec == stored and stored["state"] == "ready" and stored["seed_token_id"] == 17
    assert stored["draft_token_ids"] == [18, 19, 20] and stored["created_at_ns"] >= stored["proposal_started_at_ns"]
    assert not list(tmp_path.glob("*.tmp"))
    assert publish_proposal_trace(dest, method="eagle3", proposal_started_at_ns=2, seed_token_ids=[99],
                                  draft_token_ids=[[100]]) is None
    assert json.loads(dest.read_text()) == stored
    other = tmp_path / "other.json"
    assert publish_proposal_trace(other, method="eagle", proposal_started_at_ns=1, seed_token_ids=[1],
                                  draft_token_ids=[[2]]) is None and not other.exists()


def test_scheduling_cli_sidecar_parsing_and_source_rows(tmp_path):
    """``--priority-sidecar MODE=PATH`` needs two or more unique modes and a row for every source request."""
    with pytest.raises(ValueError):
        client.parse_sidecars(["uniform=a.jsonl"])
    with pytest.raises(ValueError):
        client.parse_sidecars(["uniform=a.jsonl", "uniform=b.jsonl"])
    assert set(client.parse_sidecars(["uniform=a", "bm25=b"])) == {"uniform", "bm25"}
    (tmp_path / "r.jsonl").write_text("".join(json.dumps({"model": "toy", "prompt": [1, 2, 3]}) + "\n"
                                              for _ in range(3)))
    for mode in ("uniform", "bm25"):
        (tmp_path / f"{mode}.jsonl").write_text("".join(
            json.dumps({"request_index": i, "priority_chunks": [0, 1]}) + "\n" for i in range(2)))
    with pytest.raises(ValueError, match="no source request 2"):
        client.main(["--requests-jsonl", str(tmp_path / "r.jsonl"), "--output-jsonl", str(tmp_path / "o.jsonl"),
                     "--num-requests", "2", "--request-offset", "1", "--priority-sidecar",
                     f"uniform={tmp_path / 'uniform.jsonl'}", "--priority-sidecar", f"bm25={tmp_path / 'bm25.jsonl'}"])


def test_pd_pipeline_exclusive_gpu_check(monkeypatch):
    """``pipelines.pd --require-exclusive-gpu`` maps CUDA_VISIBLE_DEVICES to the physical GPU and fails closed."""
    from sparsecache_b200.pipelines.pd import exclusive_gpu_or_exit

    def runner(cmd):
        return GPU_QUERY if cmd[1].startswith("--query-gpu=") else PROC_QUERY

    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "0")
    assert exclusive_gpu_or_exit(command_runner=runner)["status"] == "passed"
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "1,0")
    with pytest.raises(SystemExit, match="GPU 1 is not exclusive"):
        exclusive_gpu_or_exit(command_runner=runner)


class _FakeEngine:
    """Host stand-in of the engine calls ``EngineWorker`` makes (greedy rule of the toy worker).

    A row with input token t at position q predicts (31 t + 7 q + S) % V, where S sums the prompt
    tokens the row can see: the whole prompt, or the visible ones of a sparse view (so sparse
    drafts can differ from the verifier while verified rows equal greedy decoding).
    """

    MAX_ROWS = 8
    V = 1000

    def __init__(self):
        import torch
        from types import SimpleNamespace

        self.torch = torch
        self.device = torch.device("cpu")
        self.cfg = SimpleNamespace(n_layers=2, n_kv_heads=2, head_dim=8)
        self.w = SimpleNamespace(embed=None)
        self.ext = SimpleNamespace(embedding=lambda ids, table, h: None)
        self.prompt = []
        self.b = {k: torch.zeros(64, dtype=torch.int64) for k in ("ids", "tok", "log")}
        self.b["h"] = torch.zeros(1)
        self.b["gen"] = torch.zeros(1, dtype=torch.int64)
        self.pos = 0

    def new_slot(self, capacity):
        from types import SimpleNamespace

        return SimpleNamespace(capacity=capacity)

    def _rule(self, t, q, s):
        return (31 * int(t) + 7 * int(q) + s) % self.V

    def prefill(self, ids, slot):
        self.prompt = [int(x) for x in ids.tolist()]
        return self.torch.zeros(len(self.prompt), 1)

    def first_token(self, h, position, max_new):
        tok = (sum(self.prompt) * 13 + len(self.prompt)) % self.V
        self.b["tok"][0] = tok
        self.b["log"][0] = tok
        self.b["gen"][0] = 1
        self.b["ids"][0] = tok
        self.pos = position
        return self.b

    def _decode_buffers(self, n=0):
        return self.b

    def set_decode_state(self, *, position, slot=None, n_virtual=None):
        self.pos = position

    def decode(self, slot, n_steps, *, max_new, use_graph=True):
        s = sum(self.prompt)
        tok = int(self.b["ids"][0])
        for _ in range(n_steps):
            tok = self._rule(tok, self.pos, s)
            self.b["log"][int(self.b["gen"][0])] = tok
            self.b["gen"][0] += 1
            self.b["ids"][0] = tok
            self.pos += 1

    def generated_tokens(self, n):
        return self.b["log"][:n]

    def verify(self, slot, tokens, *, position, slot_start=None, view=None, n_visible=None, sparse=False):
        assert not sparse or view is not None  # the split sized for the view applies to views only
        T = len(self.prompt)
        if view is None:
            s = sum(self.prompt)
        else:
            keys = [int(i) for i in view[:n_visible + len(tokens)].tolist()]
            # the engine attends view[0 : n_visible + M]: the new rows' own slots come last
            assert keys[n_visible:] == list(range(slot_start, slot_start + len(tokens))), keys[n_visible:]
            s = sum(self.prompt[i] for i in keys[:n_visible] if i < T)
        return self.torch.tensor([self._rule(t, position + j, s) for j, t in enumerate(tokens.tolist())])


def test_engine_worker_progressive_chain_on_a_host_engine(tmp_path):
    """EngineWorker's draft / verify / continue logic and telemetry pass the aggregator's gates and the
    input-trace audit, and its progressive arms stream the baseline's tokens."""
    from sparsecache_b200.serving.live.worker import EngineWorker

    sink = TelemetrySink(tmp_path / "telemetry")
    worker = EngineWorker(_FakeEngine(), capacity=4096, telemetry=sink)
    cfg = proxy.ProxyConfig(max_draft_tokens=6)
    holder = {}
    apps = {cfg.prefiller_url: make_app(worker, "prefill", notify=lambda rid: holder["proxy"].notify(rid)),
            cfg.decoder_url: make_app(worker, "decode")}
    px = proxy.Proxy(cfg, client_factory=lambda url: httpx.AsyncClient(transport=httpx.ASGITransport(app=apps[url]),
                                                                      base_url=url))
    holder["proxy"] = px
    reqs = [{"model": "m", "prompt": [(37 * j + 11 * i) % 900 + 1 for j in range(600 + 150 * i)], "max_tokens": 12,
             "temperature": 0} for i in range(3)]
    arms = ("baseline", "fixed_s1", "continuous")

    async def go():
        async with httpx.AsyncClient(transport=httpx.ASGITransport(app=px.app), base_url="http://proxy") as c:
            return await client.run_benchmark(c, "/v1/completions", reqs, arms, warmup=1,
                                              output=tmp_path / "results.jsonl", run_id="fake")

    records, summ = asyncio.run(go())
    assert summ["pairs"] == 3
    assert all(v["token_equality_rate"] == 1.0 for v in summ["comparisons"].values())
    meta = [{"request_index": i, "dataset": "hotpotqa", "answers": ["x"]} for i in range(3)]
    summary, rows = aggregate.aggregate_live_run(
        records, meta, sink.records["scheduler"], sink.records["link"], arms=arms, expected_requests=3,
        fixed_output_tokens=12, bootstrap_samples=200, seed=0, protected_chunks=1,
        attention_rows=sink.records["attention"])
    failed = {k: v for k, v in summary["gates"].items() if not v["passed"]}
    assert not failed, failed
    for row in rows:  # continuous views grow over the steps, the fixed first stage does not
        assert row["arms"]["continuous"]["attention"]["distinct_visible_fractions"] > 1
        assert row["arms"]["fixed_s1"]["attention"]["distinct_visible_fractions"] == 1
    sched = sink.records["scheduler"]
    assert {s["visibility_mode"] for s in sched} == {"fixed_s1", "continuous"}
    assert all(s["draft_tokens"] == 6 for s in sched)
    assert any(s["accepted_tokens"] < 6 for s in sched)  # sparse views do change some drafts
    rep = trace.verify_input_trace(sched, sink.records["input_trace"], expected_requests=len(sched))
    assert rep["status"] == "passed" and rep["verify_forwards"] == len(sched)


def test_sparse_attention_gate_rejects_bad_views():
    sched = {"request_id": "r", "draft_tokens": 3}

    def rec(step, frac, ranges, vis, mode="continuous", rid="r"):
        return {"request_id": rid, "visibility_mode": mode, "decode_step": step, "visible_fraction": frac,
                "visible_token_ranges": ranges, "visible_pages": vis, "candidate_pages": 4}

    good = [rec(0, 0.25, [[0, 256]], 1), rec(1, 0.5, [[0, 512]], 2), rec(2, 0.75, [[0, 768]], 3)]
    summ, errs = aggregate.sparse_attention_summary(good, sched, "continuous")
    assert not errs and summ["sparse_steps"] == 3 and summ["distinct_visible_fractions"] == 3
    shrink = [good[0], rec(1, 0.25, [[256, 512]], 1), good[2]]
    assert any("shrank" in e for e in aggregate.sparse_attention_summary(shrink, sched, "continuous")[1])
    fixed = [rec(0, 0.25, [[0, 256]], 1, "fixed_s1"), rec(1, 0.5, [[0, 512]], 2, "fixed_s1"),
             rec(2, 0.25, [[0, 256]], 1, "fixed_s1")]
    assert any("fixed" in e for e in aggregate.sparse_attention_summary(fixed, sched, "fixed_s1")[1])
    missing = good[:2]
    assert any("cover" in e for e in aggregate.sparse_attention_summary(missing, sched, "continuous")[1])
    other = [rec(0, 0.25, [[0, 256]], 1, rid="x")] + good[1:]
    assert any("another request" in e for e in aggregate.sparse_attention_summary(other, sched, "continuous")[1])
    disagree = good + [rec(1, 0.75, [[0, 768]], 3)]
    assert any("disagree" in e for e in aggregate.sparse_attention_summary(disagree, sched, "continuous")[1])


def test_visibility_snapshot_and_stage_chunks():
    from sparsecache_b200.serving.live.worker import stage_chunks, visibility_snapshot

    snap = visibility_snapshot(700, [0, 2, 1], 2, 256)  # chunks 0 and 2 of [0,256) [256,512) [512,700)
    assert snap["visible_token_ranges"] == [[0, 256], [512, 700]]
    assert snap["visible_pages"] == 2 and snap["candidate_pages"] == 3
    assert abs(snap["visible_fraction"] - (256 + 188) / 700) < 1e-12
    merged = visibility_snapshot(700, [1, 0], 2, 256)  # adjacent chunks merge into one range
    assert merged["visible_token_ranges"] == [[0, 512]]
    assert visibility_snapshot(700, [5, 0], 2, 256)["visible_pages"] == 1  # out-of-range chunk ids are ignored
    assert [stage_chunks("fixed_s1", 0.05, 4, i) for i in range(5)] == [1] * 5
    assert [stage_chunks("continuous", 0.05, 4, i) for i in range(5)] == [1, 2, 3, 4, 4]
    assert stage_chunks("continuous", 0.6, 4, 0) == 3
