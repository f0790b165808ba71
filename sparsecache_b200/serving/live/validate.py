"""Latency-cell validation and the schedule x arm live benchmark.

``validate_latency_cell`` (reference: experiments/validate_pd_latency_cell.py:20-117): a P/D
latency cell is valid when it has the expected number of unique requests, its protocol block
asserts a fixed token horizon, paired measurement, an exclusive GPU (and little memory in use at
start), the baseline and the method produced timing sequences of the same length, the time of
each request that no measured phase accounts for stays under a threshold, and the two
measurement orders (baseline first / method first) are balanced within one.

``run_scheduling_benchmark`` / ``aggregate_scheduling`` (reference:
experiments/benchmark_progressive_pd_scheduling_live.py:32-171,
experiments/aggregate_progressive_pd_scheduling_live.py:79-306): every source request is run
under each chunk-priority schedule (sequential, uniform, random, bm25, oracle) and each
progressive arm (fixed_s1, continuous), all sharing ONE producer prefill per request; the
aggregate checks that every (request, schedule, arm) cell exists, that all cells of a request
share one prefill and one seed, and that greedy outputs agree across schedules, then compares
schedules by decode completion and TTFT.
"""
from __future__ import annotations

import statistics
from collections import Counter
from typing import Any, Sequence

from .aggregate import describe, gate
from .client import run_one

SCHEDULES = ("sequential", "uniform", "random", "bm25", "oracle")


def unattributed_ms(pipeline: dict) -> float:
    """Wall time of one request not covered by any measured phase (lower bound)."""
    accounted = sum(float(pipeline.get(k, 0.0)) for k in ("draft_prefill_ms", "draft_decode_ms", "final_prefill_ms",
                                                          "final_correction_ms", "final_decode_ms", "verify_ms"))
    transfer = pipeline.get("transfer", {})
    accounted += float(transfer.get("total_h2d_ms", 0.0)) + sum(transfer.get("stage_wire_wait_ms", []))
    return max(0.0, float(pipeline["response_ms"]) - accounted)


def validate_latency_cell(rows: Sequence[dict], *, expected_count: int, max_unattributed_ms: float = 100.0,
                          max_initial_gpu_bytes: int = 1 << 30) -> dict[str, Any]:
    failures: list[str] = []
    if len(rows) != expected_count:
        failures.append(f"expected {expected_count} rows, observed {len(rows)}")
    idx = [r["dataset_index"] for r in rows]
    if len(idx) != len(set(idx)):
        failures.append("dataset indices are not unique")
    if not rows:
        raise ValueError("no rows")
    proto = rows[0]["protocol"]
    for key in ("fixed_token_horizon", "paired_measurement", "require_exclusive_gpu"):
        if not proto.get(key, False):
            failures.append(f"protocol field {key} is not true")
    if proto.get("initial_gpu_used_bytes", 1 << 62) > max_initial_gpu_bytes:
        failures.append("selected GPU was not exclusive at process start")
    mismatched, noisy, orders = [], [], Counter()
    for r in rows:
        for sname, sched in r["schedules"].items():
            target = sched["full_target"]
            for window, chain in sched["chains"].items():
                key = (r["dataset_index"], sname, window)
                orders[chain.get("measurement_order", "missing")] += 1
                if len(target["timing_token_ids"]) != len(chain["timing_token_ids"]):
                    mismatched.append(key)
                u = unattributed_ms(chain["pipeline"])
                if u > max_unattributed_ms:
                    noisy.append((*key, u))
    if mismatched:
        failures.append(f"{len(mismatched)} baseline/method timing-length mismatches")
    if noisy:
        failures.append(f"{len(noisy)} requests exceed the unattributed-wall threshold")
    if abs(orders["full_target_then_pipeline"] - orders["pipeline_then_full_target"]) > 1:
        failures.append(f"measurement order is unbalanced: {dict(orders)}")
    return {"passed": not failures, "rows": len(rows), "failures": failures, "noisy": noisy[:20],
            "orders": dict(orders)}


async def run_scheduling_benchmark(client, endpoint: str, requests: Sequence[dict],
                                   priorities: dict[str, dict[int, list[int]]], *, arms=("fixed_s1", "continuous"),
                                   schedules: Sequence[str] = SCHEDULES, run_id: str = "sched") -> list[dict]:
    """Every request x schedule x arm, one shared producer prefill per request."""
    out = []
    for i, req in enumerate(requests):
        group = f"{run_id}:{i}"
        for k, sname in enumerate(schedules):
            payload = dict(req)
            payload["sparsecache_priority_chunks"] = priorities[sname][i]
            for arm in (arms if k % 2 == 0 else tuple(reversed(arms))):  # alternate arm order
                rec = await run_one(client, endpoint, payload, arm, group)
                rec.update(request_index=i, schedule=sname, warmup=False)
                out.append(rec)
    return out


def aggregate_scheduling(records: Sequence[dict], *, schedules: Sequence[str] = SCHEDULES,
                         arms: Sequence[str] = ("fixed_s1", "continuous"), expected_requests: int,
                         bootstrap_samples: int = 2000, seed: int = 0) -> dict[str, Any]:
    cells: dict[int, dict[tuple[str, str], dict]] = {}
    errors = []
    for r in records:
        key = (r["schedule"], r["arm"])
        c = cells.setdefault(r["request_index"], {})
        if key in c:
            errors.append(f"duplicate cell {r['request_index']}/{key}")
        c[key] = r
    want = {(s, a) for s in schedules for a in arms}
    complete = set(cells) == set(range(expected_requests)) and all(set(c) == want for c in cells.values())
    prefill_errors, output_errors = [], []
    for i, c in cells.items():
        if len({r["prefill_group"] for r in c.values()}) != 1 or len({r["seed_token_id"] for r in c.values()}) != 1:
            prefill_errors.append(f"{i}: cells do not share one prefill and seed")
        if sum(r["prefill_reused"] is False for r in c.values()) != 1:
            prefill_errors.append(f"{i}: expected exactly one producer prefill")
        if len({tuple(r["token_ids"]) for r in c.values()}) != 1:
            output_errors.append(f"{i}: greedy outputs differ across schedules/arms")
    gates = {"complete_schedule_matrix": gate(complete and not errors, errors=errors),
             "single_shared_prefill": gate(not prefill_errors, errors=prefill_errors),
             "exact_output_across_schedules": gate(not output_errors, errors=output_errors)}
    gates["overall"] = gate(all(g["passed"] for g in gates.values()))
    by_cell = {}
    for s in schedules:
        for a in arms:
            rows = [c[(s, a)] for c in cells.values() if (s, a) in c]
            if rows:
                by_cell[f"{s}/{a}"] = {
                    "decode_completion_ms": describe([r["decode_completion_ms"] for r in rows],
                                                     bootstrap_samples=bootstrap_samples, seed=seed),
                    "decode_ttft_ms": statistics.fmean(r["decode_ttft_ms"] for r in rows)}
    return {"status": "passed" if gates["overall"]["passed"] else "failed_gates", "gates": gates, "cells": by_cell}


def main(argv=None) -> int:
    """``latency-cell ROWS.jsonl --expected N`` or ``scheduling RECORDS.jsonl --expected-requests N``.

    Counterparts of the reference's experiments/validate_pd_latency_cell.py and
    aggregate_progressive_pd_scheduling_live.py CLIs; exit code 1 on a failed check.
    """
    import argparse
    import json
    from pathlib import Path

    from .trace import load_jsonl

    p = argparse.ArgumentParser()
    sub = p.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("latency-cell")
    c.add_argument("rows", type=Path)
    c.add_argument("--expected", type=int, required=True)
    c.add_argument("--max-unattributed-ms", type=float, default=100.0)
    c.add_argument("--max-initial-gpu-bytes", type=int, default=1 << 30)
    s = sub.add_parser("scheduling")
    s.add_argument("records", type=Path)
    s.add_argument("--expected-requests", type=int, required=True)
    s.add_argument("--schedules", default=",".join(SCHEDULES))
    s.add_argument("--arms", default="fixed_s1,continuous")
    s.add_argument("--bootstrap-samples", type=int, default=2000)
    for q in (c, s):
        q.add_argument("--output", type=Path, default=None)
    a = p.parse_args(argv)
    if a.cmd == "latency-cell":
        rows = [r for r in load_jsonl(a.rows) if "schedules" in r]
        out = validate_latency_cell(rows, expected_count=a.expected, max_unattributed_ms=a.max_unattributed_ms,
                                    max_initial_gpu_bytes=a.max_initial_gpu_bytes)
        ok = out["passed"]
    else:
        out = aggregate_scheduling(load_jsonl(a.records), schedules=a.schedules.split(","), arms=a.arms.split(","),
                                   expected_requests=a.expected_requests, bootstrap_samples=a.bootstrap_samples)
        ok = out["status"] == "passed"
    text = json.dumps(out, indent=2, default=str)
    if a.output is not None:
        a.output.write_text(text + "\n")
    print(text)
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
