"""Paired live benchmark client for the 1P1D proxy.

Parity with the reference's experiments/benchmark_progressive_pd_live.py:
arms ``baseline`` / ``fixed_s1`` / ``continuous`` (at least two, unique), an
execution plan of warm-up rows followed by measured rows, per request one
prefill group shared by every arm (the proxy prefills once), arm order
rotated per request, streamed responses with per-token arrival times, and a
summary with paired comparisons (token equality, decode-completion and
decode-TTFT gains; positive favours the right arm) (:15-354).
"""
from __future__ import annotations

import argparse
import asyncio
import json
import math
import statistics
import time
import uuid
from pathlib import Path
from typing import Any, Sequence

VALID_ARMS = ("baseline", "fixed_s1", "continuous")


def parse_arms(raw: str) -> tuple[str, ...]:
    arms = tuple(a.strip() for a in raw.split(",") if a.strip())
    if len(arms) < 2 or len(arms) != len(set(arms)):
        raise argparse.ArgumentTypeError("arms must contain at least two unique values")
    bad = [a for a in arms if a not in VALID_ARMS]
    if bad:
        raise argparse.ArgumentTypeError(f"unknown benchmark arms: {bad}")
    return arms


def read_priority_rows(path: Path) -> dict[int, list[int]]:
    out: dict[int, list[int]] = {}
    for n, line in enumerate(Path(path).read_text(encoding="utf-8").splitlines(), start=1):
        if not line.strip():
            continue
        row = json.loads(line)
        i, pr = row.get("request_index"), row.get("priority_chunks")
        if not isinstance(i, int) or isinstance(i, bool) or i < 0 or i in out:
            raise ValueError(f"{path}:{n} has invalid request_index")
        if (not isinstance(pr, list) or not pr or any(not isinstance(c, int) or isinstance(c, bool) or c < 0
                                                       for c in pr) or len(pr) != len(set(pr))):
            raise ValueError(f"{path}:{n} has invalid priority_chunks")
        if sorted(pr) != list(range(len(pr))):
            raise ValueError(f"{path}:{n} priority is not a full permutation")
        out[i] = pr
    if not out:
        raise ValueError(f"no priority rows in {path}")
    return out


def read_requests(path: Path, limit: int, offset: int = 0, priorities: dict[int, list[int]] | None = None):
    rows = []
    for i, line in enumerate(Path(path).read_text(encoding="utf-8").splitlines()):
        if i < offset or not line.strip():
            continue
        req = json.loads(line)
        if not isinstance(req, dict):
            raise TypeError("each JSONL row must be an OpenAI request object")
        if priorities is not None:
            if i not in priorities:
                raise ValueError(f"priority sidecar has no row {i}")
            req["sparsecache_priority_chunks"] = priorities[i]
        req.update(stream=True, return_token_ids=True, temperature=0)
        rows.append(req)
        if len(rows) == limit:
            break
    if len(rows) < limit:
        raise ValueError(f"requested {limit} rows but {path} contains {len(rows)}")
    return rows


def execution_plan(requests: Sequence[dict], warmup: int, source_offset: int = 0):
    """[(measured index or None for warm-up, source row, request)]."""
    if not requests:
        raise ValueError("execution plan requires at least one request")
    warm = [(None, source_offset + i % len(requests), requests[i % len(requests)]) for i in range(warmup)]
    return warm + [(i, source_offset + i, r) for i, r in enumerate(requests)]


def rotated_arms(arms: Sequence[str], index: int) -> list[str]:
    k = index % len(arms)
    return list(arms[k:]) + list(arms[:k])


def _tokens_and_text(payload: dict) -> tuple[list[int], str]:
    ch = (payload.get("choices") or [{}])[0]
    return [int(t) for t in ch.get("token_ids") or []], str(ch.get("text") or (ch.get("delta") or {}).get("content")
                                                             or "")


async def run_one(client, endpoint: str, payload: dict, arm: str, prefill_group: str) -> dict[str, Any]:
    req = dict(payload)
    req.update(stream=True, return_token_ids=True)  # this client measures streamed token arrivals
    req["sparsecache_prefill_group"] = prefill_group
    if arm == "baseline":
        req["sparsecache_mode"] = "baseline"
    else:
        req["sparsecache_mode"] = "progressive"
        req["sparsecache_visibility_mode"] = arm
    t0 = time.perf_counter()
    header_at = first_at = None
    toks: list[int] = []
    arrivals: list[float] = []
    text: list[str] = []
    async with client.stream("POST", endpoint, json=req) as resp:
        header_at = time.perf_counter()
        resp.raise_for_status()
        hdr = {k.lower(): v for k, v in resp.headers.items()}
        async for line in resp.aiter_lines():
            if not line.startswith("data: ") or line[6:] == "[DONE]":
                continue
            new, tx = _tokens_and_text(json.loads(line[6:]))
            at = time.perf_counter()
            if first_at is None and (new or tx):
                first_at = at
            toks += new
            arrivals += [(at - t0) * 1000.0] * len(new)
            text.append(tx)
    done = time.perf_counter()
    if first_at is None:
        raise RuntimeError("stream completed without a visible output token")
    seed, reused = hdr.get("x-sparsecache-seed-token", ""), hdr.get("x-sparsecache-prefill-reused", "")
    if not seed.isdecimal() or reused not in ("true", "false"):
        raise RuntimeError("proxy did not return paired-prefill telemetry headers")
    return {"arm": arm, "runtime_mode": hdr.get("x-sparsecache-mode", ""), "header_ms": (header_at - t0) * 1e3,
            "ttft_ms": (first_at - t0) * 1e3, "decode_ttft_ms": (first_at - header_at) * 1e3,
            "completion_ms": (done - t0) * 1e3, "decode_completion_ms": (done - header_at) * 1e3,
            "token_ids": toks, "token_arrival_ms": arrivals, "text": "".join(text),
            "server_timing": hdr.get("server-timing", ""), "proxy_request_id": hdr.get("x-sparsecache-request-id", ""),
            "prefill_group": hdr.get("x-sparsecache-prefill-group", ""), "prefill_reused": reused == "true",
            "seed_token_id": int(seed)}


def percentile_nearest_rank(values: Sequence[float], q: float) -> float:
    if not values:
        return math.nan
    v = sorted(values)
    return v[min(len(v) - 1, math.ceil(q * len(v)) - 1)]


def comparison(pairs: Sequence[dict[str, dict]], left: str, right: str) -> dict[str, Any]:
    comp = [p[left]["decode_completion_ms"] - p[right]["decode_completion_ms"] for p in pairs]
    ttft = [p[left]["decode_ttft_ms"] - p[right]["decode_ttft_ms"] for p in pairs]
    eq = [p[left]["token_ids"] == p[right]["token_ids"] for p in pairs]

    def dist(x):
        return {"mean": statistics.fmean(x) if x else math.nan, "p05": percentile_nearest_rank(x, 0.05),
                "p50": percentile_nearest_rank(x, 0.5), "p95": percentile_nearest_rank(x, 0.95)}

    return {"left": left, "right": right, "gain_definition": "left latency minus right latency; positive favors right",
            "token_equality_rate": statistics.fmean(eq) if eq else math.nan,
            "right_faster_completion": sum(d > 0 for d in comp), "decode_completion_gain_ms": dist(comp),
            "decode_ttft_gain_ms": dist(ttft)}


def summary(records: Sequence[dict], arms: Sequence[str]) -> dict[str, Any]:
    pairs: dict[int, dict[str, dict]] = {}
    for r in records:
        pairs.setdefault(r["request_index"], {})[r["arm"]] = r
    full = [p for p in pairs.values() if all(a in p for a in arms)]
    comps = {}
    if "baseline" in arms:
        comps.update({f"baseline_vs_{a}": comparison(full, "baseline", a) for a in arms if a != "baseline"})
    if "fixed_s1" in arms and "continuous" in arms:
        comps["fixed_s1_vs_continuous"] = comparison(full, "fixed_s1", "continuous")
    return {"arms": list(arms), "pairs": len(full), "comparisons": comps}


async def run_benchmark(client, endpoint: str, requests: Sequence[dict], arms: Sequence[str], *, warmup: int,
                        output: Path | None = None, source_offset: int = 0, run_id: str | None = None):
    """Run the plan; returns (measured records, summary).  Records stream to ``output`` as JSONL."""
    run_id = run_id or uuid.uuid4().hex[:8]
    records = []
    sink = open(output, "w", encoding="utf-8") if output else None
    try:
        for n, (index, source, req) in enumerate(execution_plan(requests, warmup, source_offset)):
            group = f"{run_id}:{'w' if index is None else 'm'}:{n}"
            for arm in rotated_arms(arms, n):
                rec = await run_one(client, endpoint, req, arm, group)
                rec.update(request_index=index, source_request_index=source, warmup=index is None)
                if index is not None:
                    records.append(rec)
                    if sink:
                        sink.write(json.dumps(rec) + "\n")
    finally:
        if sink:
            sink.close()
    return records, summary(records, arms)


def parse_sidecars(values: Sequence[str]) -> dict[str, Path]:
    """``MODE=PATH`` values -> {mode: path}; at least two unique modes."""
    out: dict[str, Path] = {}
    for v in values:
        mode, sep, path = v.partition("=")
        mode, path = mode.strip(), path.strip()
        if not sep or not mode or not path or mode in out:
            raise ValueError("priority sidecars must be unique non-empty MODE=PATH values")
        out[mode] = Path(path)
    if len(out) < 2:
        raise ValueError("a scheduling run needs at least two modes")
    return out


def main(argv=None) -> None:
    """Paired arms over a request file; with ``--priority-sidecar MODE=PATH`` (two or more) every request
    runs under every schedule x arm on one shared prefill (reference:
    experiments/benchmark_progressive_pd_scheduling_live.py)."""
    import httpx

    p = argparse.ArgumentParser()
    p.add_argument("--url", default="http://127.0.0.1:8000")
    p.add_argument("--endpoint", choices=("/v1/completions", "/v1/chat/completions"), default="/v1/completions")
    p.add_argument("--requests-jsonl", type=Path, required=True)
    p.add_argument("--output-jsonl", type=Path, required=True)
    p.add_argument("--num-requests", type=int, default=100)
    p.add_argument("--request-offset", type=int, default=0)
    p.add_argument("--warmup-requests", type=int, default=4)
    p.add_argument("--fixed-output-tokens", type=int)
    p.add_argument("--priority-jsonl", type=Path)
    p.add_argument("--arms", type=parse_arms, default=None)
    p.add_argument("--priority-sidecar", action="append", default=[], metavar="MODE=PATH")
    a = p.parse_args(argv)
    if a.priority_sidecar:
        return _scheduling_main(a)
    a.arms = a.arms or ("baseline", "continuous")
    pri = read_priority_rows(a.priority_jsonl) if a.priority_jsonl else None
    reqs = read_requests(a.requests_jsonl, a.num_requests, a.request_offset, pri)
    if a.fixed_output_tokens:
        for r in reqs:
            r["max_tokens"] = a.fixed_output_tokens
            r["ignore_eos"] = True

    async def go():
        async with httpx.AsyncClient(base_url=a.url, timeout=None, trust_env=False) as c:
            return await run_benchmark(c, a.endpoint, reqs, a.arms, warmup=a.warmup_requests,
                                       output=a.output_jsonl, source_offset=a.request_offset)

    _, summ = asyncio.run(go())
    print(json.dumps(summ, indent=2))



def _scheduling_main(a) -> dict:
    import httpx

    from .validate import run_scheduling_benchmark

    if a.output_jsonl.exists():
        raise FileExistsError(f"refusing to overwrite {a.output_jsonl}")
    arms = a.arms or ("fixed_s1", "continuous")
    sidecars = parse_sidecars(a.priority_sidecar)
    rows = {m: read_priority_rows(path) for m, path in sidecars.items()}
    reqs = read_requests(a.requests_jsonl, a.num_requests, a.request_offset)
    horizon = a.fixed_output_tokens or 32
    for r in reqs:
        r["max_tokens"], r["ignore_eos"] = horizon, True
    local = {}
    for m, by_source in rows.items():
        missing = [a.request_offset + i for i in range(len(reqs)) if a.request_offset + i not in by_source]
        if missing:
            raise ValueError(f"{m} sidecar has no source request {missing[0]}")
        local[m] = {i: by_source[a.request_offset + i] for i in range(len(reqs))}

    async def go():
        async with httpx.AsyncClient(base_url=a.url, timeout=None, trust_env=False) as c:
            return await run_scheduling_benchmark(c, a.endpoint, reqs, local, arms=arms, schedules=tuple(sidecars),
                                                  run_id=uuid.uuid4().hex[:8])

    recs = asyncio.run(go())
    a.output_jsonl.parent.mkdir(parents=True, exist_ok=True)
    with open(a.output_jsonl, "w", encoding="utf-8") as f:
        for r in recs:
            r["source_request_index"] = a.request_offset + r["request_index"]
            f.write(json.dumps(r) + "\n")
    summ = {"schema_version": 1, "status": "raw live measurements; aggregation gates not yet applied",
            "modes": list(sidecars), "arms": list(arms), "requests": len(reqs), "request_offset": a.request_offset,
            "fixed_output_tokens": horizon, "measured_records": len(recs),
            "expected_records": len(reqs) * len(sidecars) * len(arms),
            "priority_sidecars": {m: str(pth) for m, pth in sidecars.items()},
            "prefill_pairing": "one exact producer prefill per request, reused by every schedule x arm"}
    a.output_jsonl.with_suffix(".summary.json").write_text(json.dumps(summ, indent=2) + "\n")
    print(json.dumps(summ, indent=2))
    return summ


if __name__ == "__main__":
    main()
