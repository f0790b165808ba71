"""Live 1P1D harness with this package's engine behind both worker roles (one GPU, in process):
the proxy -> prefill -> store-completion -> decode chain, the paired client over the baseline and
the two progressive arms, the validity-gated aggregation and the input-trace audit, as the CPU
test runs them with the toy worker.  Progressive arms draft over sparse prompt views, verify once
over the full prompt and must stream exactly the baseline's greedy tokens."""
import asyncio

import httpx
import pytest

pytestmark = pytest.mark.gpu


def test_live_chain_with_engine_workers(tmp_path, cuda_device):
    from sparsecache_b200.config import get_model_config
    from sparsecache_b200.models.engine import B200Engine
    from sparsecache_b200.models.llama import LlamaOracle
    from sparsecache_b200.serving.live import aggregate, client, proxy, trace
    from sparsecache_b200.serving.live.worker import EngineWorker, TelemetrySink, make_app

    cfg = get_model_config("tiny128")
    engine = B200Engine.from_oracle(LlamaOracle.random_init(cfg, seed=11, std=0.05), cuda_device,
                                    max_positions=4096)
    sink = TelemetrySink(tmp_path / "telemetry")
    worker = EngineWorker(engine, capacity=2048, telemetry=sink)
    pcfg = proxy.ProxyConfig(max_draft_tokens=6)
    holder = {}
    apps = {pcfg.prefiller_url: make_app(worker, "prefill", notify=lambda rid: holder["proxy"].notify(rid)),
            pcfg.decoder_url: make_app(worker, "decode")}
    px = proxy.Proxy(pcfg, client_factory=lambda url: httpx.AsyncClient(transport=httpx.ASGITransport(app=apps[url]),
                                                                       base_url=url))
    holder["proxy"] = px
    # 3-4 chunks of 256 tokens per prompt; ids above the special range
    reqs = [{"model": "m", "prompt": [5 + (37 * j + 11 * i) % 4000 for j in range(600 + 150 * i)],
             "max_tokens": 12, "temperature": 0} for i in range(3)]
    arms = ("baseline", "fixed_s1", "continuous")

    async def go():
        async with httpx.AsyncClient(transport=httpx.ASGITransport(app=px.app), base_url="http://proxy") as c:
            return await client.run_benchmark(c, "/v1/completions", reqs, arms, warmup=1,
                                              output=tmp_path / "results.jsonl", run_id="engine")

    records, summ = asyncio.run(go())
    assert summ["pairs"] == 3
    for k, v in summ["comparisons"].items():
        assert v["token_equality_rate"] == 1.0, (k, v)
    meta = [{"request_index": i, "dataset": "hotpotqa", "answers": ["x"]} for i in range(3)]
    summary, _ = aggregate.aggregate_live_run(
        records, meta, sink.records["scheduler"], sink.records["link"], arms=arms, expected_requests=3,
        fixed_output_tokens=12, bootstrap_samples=200, seed=0, protected_chunks=1,
        attention_rows=sink.records["attention"])
    failed = {k: v for k, v in summary["gates"].items() if not v["passed"]}
    assert not failed, failed
    # every progressive request: gamma single-token sparse forwards, then one verifier batch
    sched = sink.records["scheduler"]
    assert all(s["draft_tokens"] == 6 and 0 <= s["accepted_tokens"] <= 6 for s in sched)
    rep = trace.verify_input_trace(sched, sink.records["input_trace"], expected_requests=len(sched))
    assert rep["status"] == "passed" and rep["verify_forwards"] == len(sched)
