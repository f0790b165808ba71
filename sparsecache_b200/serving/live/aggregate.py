"""Aggregation of a live paired run: validity gates, latency model, paired bootstrap.

Parity with the reference's experiments/aggregate_progressive_pd_live.py:
linear-interpolated percentiles and a seeded bootstrap of the mean
(:101-138); per-request validation of token-arrival telemetry (:507-524);
the request latency model that predicts a method's decode-completion gain
from independently observed terms, accepted tokens x mean target step
minus verification time minus the draft span not hidden behind the residual
wire time (:527-602); paired comparisons with bootstrap CIs (:605-685); and
the validity gates of a run (:688-1130):
  complete_paired_matrix, request_protocol, single_paired_prefill,
  fixed_output_horizon, one_scheduler_transition_per_method,
  scheduler_transition_invariants, request_attributed_sparse_attention
  (the per-step sparse-view records of every progressive request, :416-504),
  fair_controlled_link,
  protected_anchor_arrival, request_scoped_priority_schedule,
  latency_model_telemetry, exact_greedy_output_equivalence, overall.
Quality is scored with the LongBench metrics of the request's dataset.
Outputs: ``summary.json``, ``summary.md``, ``paper_table.csv``,
``paired_rows.jsonl``.
"""
from __future__ import annotations

import csv
import json
import math
import random
import statistics
from itertools import pairwise
from pathlib import Path
from typing import Any, Sequence

from ...evaluation.longbench import score_prediction
from .client import VALID_ARMS

STATE_ORDER = ("WAIT_ANCHOR", "DRAFT_WHILE_LOADING", "READY_TO_VERIFY", "TARGET_DECODING", "FINISHED")


def percentile(values: Sequence[float], q: float) -> float:
    if not values:
        return math.nan
    v = sorted(float(x) for x in values)
    pos = q * (len(v) - 1)
    lo, hi = math.floor(pos), math.ceil(pos)
    return v[lo] if lo == hi else v[lo] * (1 - (pos - lo)) + v[hi] * (pos - lo)


def bootstrap_mean_ci(values: Sequence[float], *, samples: int, seed: int) -> list[float]:
    if not values:
        return [math.nan, math.nan]
    rng = random.Random(seed)
    est = [statistics.fmean(rng.choices(values, k=len(values))) for _ in range(samples)]
    return [percentile(est, 0.025), percentile(est, 0.975)]


def describe(values: Sequence[float], *, bootstrap_samples: int, seed: int) -> dict[str, Any]:
    x = [float(v) for v in values]
    return {"mean": statistics.fmean(x), "mean_bootstrap_ci95": bootstrap_mean_ci(x, samples=bootstrap_samples,
                                                                                   seed=seed),
            "p50": percentile(x, 0.5), "p95": percentile(x, 0.95), "p99": percentile(x, 0.99), "min": min(x),
            "max": max(x)}


def gate(passed: bool, **details) -> dict[str, Any]:
    return {"passed": bool(passed), **details}


def validate_token_arrivals(result: dict) -> list[str]:
    arr, toks = result.get("token_arrival_ms"), result.get("token_ids")
    if not isinstance(arr, list) or not isinstance(toks, list):
        return ["token arrival telemetry is not a list"]
    if len(arr) != len(toks):
        return ["token arrival telemetry does not cover returned token IDs"]
    if any(not isinstance(a, (int, float)) or isinstance(a, bool) or not math.isfinite(a) or a < 0 for a in arr):
        return ["token arrival telemetry contains an invalid timestamp"]
    if arr != sorted(arr):
        return ["token arrival telemetry is not monotonic"]
    return []


def request_latency_model(baseline: dict, method: dict) -> tuple[dict | None, list[str]]:
    """Predicted vs observed decode-completion gain of one method request."""
    sch, link = method.get("scheduler"), method.get("link")
    if not isinstance(sch, dict) or not isinstance(link, dict):
        return None, ["latency model requires scheduler and link telemetry"]
    steps = [b - a for a, b in pairwise(baseline.get("token_arrival_ms") or []) if b > a]
    if not steps:
        return None, ["latency model has no positive baseline decode intervals"]
    done, started = sch.get("draft_completed_at_ns"), sch.get("started_at_ns")
    verify_ns, accepted = sch.get("verify_ns"), sch.get("accepted_tokens")
    if (not isinstance(done, list) or not all(isinstance(v, int) for v in done) or not isinstance(started, int)
            or not isinstance(verify_ns, (int, float)) or not isinstance(accepted, int)):
        return None, ["latency model scheduler timing fields are incomplete"]
    step = statistics.fmean(steps)
    span = (done[-1] - started) / 1e6 if done else 0.0
    wire = float(link.get("residual_modeled_wire_ms", math.nan))
    verify = float(verify_ns) / 1e6
    if not all(math.isfinite(v) and v >= 0 for v in (step, span, wire, verify)):
        return None, ["latency model contains an invalid duration"]
    value = accepted * step
    exposed = max(0.0, span - wire)
    predicted = value - verify - exposed
    observed = float(baseline["decode_completion_ms"]) - float(method["decode_completion_ms"])
    err = observed - predicted
    return {"target_step_ms": step, "accepted_tokens": float(accepted), "accepted_decode_value_ms": value,
            "verify_ms": verify, "sparse_draft_span_ms": span, "residual_modeled_wire_ms": wire,
            "exposed_draft_ms": exposed, "predicted_gain_ms": predicted, "observed_gain_ms": observed,
            "prediction_error_ms": err, "absolute_prediction_error_ms": abs(err),
            "gain_sign_matches": float((predicted > 0) == (observed > 0))}, []


def pair_comparison(pairs: Sequence[dict], left: str, right: str, *, bootstrap_samples: int, seed: int) -> dict:
    L = [p["arms"][left] for p in pairs]
    R = [p["arms"][right] for p in pairs]
    comp = [a["decode_completion_ms"] - b["decode_completion_ms"] for a, b in zip(L, R)]
    ttft = [a["decode_ttft_ms"] - b["decode_ttft_ms"] for a, b in zip(L, R)]
    qual = [b["quality_score"] - a["quality_score"] for a, b in zip(L, R)]
    speed = [a["decode_completion_ms"] / max(b["decode_completion_ms"], 1e-9) for a, b in zip(L, R)]
    out = {"left": left, "right": right, "latency_gain_definition": "left minus right; positive favors right",
           "token_equality_rate": statistics.fmean([a["token_ids"] == b["token_ids"] for a, b in zip(L, R)]),
           "decode_completion_gain_ms": describe(comp, bootstrap_samples=bootstrap_samples, seed=seed),
           "decode_ttft_gain_ms": describe(ttft, bootstrap_samples=bootstrap_samples, seed=seed + 1),
           "decode_completion_speedup": describe(speed, bootstrap_samples=bootstrap_samples, seed=seed + 2),
           "quality_score_delta": describe(qual, bootstrap_samples=bootstrap_samples, seed=seed + 3),
           "right_faster_completion": sum(c > 0 for c in comp), "right_faster_ttft": sum(t > 0 for t in ttft)}
    if left == "baseline":
        models = [p.get("latency_models", {}).get(right) for p in pairs]
        models = [m for m in models if m]
        if models:
            out["latency_model"] = {k: describe([m[k] for m in models], bootstrap_samples=bootstrap_samples,
                                                seed=seed + 10 + i) for i, k in enumerate(sorted(models[0]))}
    return out


def _scheduler_errors(s: dict, result: dict) -> list[str]:
    errs = []
    tr = s.get("transitions")
    if not isinstance(tr, list) or tr != [x for x in STATE_ORDER if x in tr] or tr[-1:] != ["FINISHED"]:
        errs.append("scheduler transitions are not an ordered path ending in FINISHED")
    d, a = s.get("draft_tokens"), s.get("accepted_tokens")
    if not isinstance(d, int) or not isinstance(a, int) or not 0 <= a <= d:
        errs.append("accepted tokens must lie in [0, draft tokens]")
    if s.get("visibility_mode") != result["arm"]:
        errs.append("scheduler visibility mode differs from the arm")
    if s.get("seed_token_id") is not None and s.get("seed_token_id") != result.get("seed_token_id"):
        errs.append("scheduler seed differs from the producer seed")
    return errs


def sparse_attention_summary(rows: Sequence[dict], scheduler: dict, arm: str) -> tuple[dict, list[str]]:
    """Check and summarise the sparse-view records of one progressive request.

    Every draft step 0 .. draft_tokens-1 has records (one per layer, or one
    covering ``layers`` layers) carrying the request's id, the arm as
    visibility mode, the visible fraction, the exact visible token ranges and
    visible / candidate page counts; the records of a step agree.  A
    ``continuous`` view never shrinks (fraction, pages, token ranges); a
    ``fixed_s1`` view keeps one partial snapshot.
    """
    errs: list[str] = []
    if any(r.get("request_id") != scheduler.get("request_id") for r in rows):
        errs.append("sparse-attention record of another request")
    if any(r.get("visibility_mode") != arm for r in rows):
        errs.append("sparse-attention visibility mode differs from the arm")
    by_step: dict[int, list[dict]] = {}
    for r in rows:
        st = r.get("decode_step")
        if not isinstance(st, int) or isinstance(st, bool) or st < 0:
            errs.append("invalid sparse-attention decode step")
            continue
        by_step.setdefault(st, []).append(r)
    n_draft = scheduler.get("draft_tokens")
    if not isinstance(n_draft, int) or set(by_step) != set(range(n_draft)):
        errs.append("sparse-attention steps do not cover the scheduler's draft tokens exactly")
    steps, prev, partial = [], None, set()
    for st in sorted(by_step):
        snaps = {(float(r.get("visible_fraction", -1.0)), json.dumps(r.get("visible_token_ranges")),
                  r.get("candidate_pages"), r.get("visible_pages")) for r in by_step[st]}
        if len(snaps) != 1:
            errs.append(f"step {st}: records disagree on the view")
        frac, ranges_json, cand, vis = next(iter(snaps))
        ranges = json.loads(ranges_json) if ranges_json != "null" else None
        if not isinstance(cand, int) or not isinstance(vis, int) or cand <= 0 or not 0 <= vis <= cand:
            errs.append(f"step {st}: invalid page counts")
            continue
        if not 0.0 < frac <= 1.0:
            errs.append(f"step {st}: visible fraction outside (0, 1]")
        if not isinstance(ranges, list) or any(not isinstance(x, list) or len(x) != 2 or not x[0] < x[1]
                                               for x in ranges):
            errs.append(f"step {st}: invalid visible token ranges")
            continue
        tokens = {t for lo, hi in ranges for t in range(int(lo), int(hi))}
        if arm == "continuous" and prev is not None:
            if frac < prev[0] or vis < prev[1] or not prev[2] <= tokens:
                errs.append(f"step {st}: the continuous view shrank")
        if arm == "fixed_s1" and frac < 1.0:
            partial.add((frac, ranges_json, vis))
        prev = (frac, vis, tokens)
        steps.append({"decode_step": st, "records": len(by_step[st]), "visible_fraction": frac,
                      "visible_pages": vis, "candidate_pages": cand})
    if len(partial) > 1:
        errs.append("the fixed first-stage view changed between steps")
    sparse = sum(x["visible_pages"] < x["candidate_pages"] for x in steps)
    return {"steps": len(steps), "sparse_steps": sparse, "sparse_step_rate": sparse / len(steps) if steps else 0.0,
            "distinct_visible_fractions": len({x["visible_fraction"] for x in steps}),
            "first_visible_fraction": steps[0]["visible_fraction"] if steps else None,
            "last_visible_fraction": steps[-1]["visible_fraction"] if steps else None}, errs


def aggregate_live_run(results: Sequence[dict], metadata: Sequence[dict], scheduler_rows: Sequence[dict],
                       link_rows: Sequence[dict], *, arms: Sequence[str], expected_requests: int,
                       fixed_output_tokens: int | None = None, bootstrap_samples: int = 10000, seed: int = 0,
                       priority_rows: Sequence[dict] | None = None, protected_chunks: int = 0,
                       enforce_paired_prefill: bool = True, attention_rows: Sequence[dict] = ()):
    """(summary with gates, paired rows) of one live run.

    ``attention_rows`` are the workers' request-attributed sparse-view records;
    a progressive request without them fails ``request_attributed_sparse_attention``.
    """
    arms = tuple(arms)
    if expected_requests <= 0 or bootstrap_samples <= 0:
        raise ValueError("expected requests and bootstrap samples must be positive")
    if len(arms) < 2 or len(arms) != len(set(arms)) or any(a not in VALID_ARMS for a in arms):
        raise ValueError(f"invalid arms: {arms}")
    meta = {}
    for m in metadata:
        i = m.get("request_index")
        if not isinstance(i, int) or i in meta:
            raise ValueError("metadata request indices must be unique integers")
        meta[i] = m
    priorities = {int(r["request_index"]): list(r["priority_chunks"]) for r in (priority_rows or [])}
    matrix: dict[int, dict[str, dict]] = {}
    proxy_ids, raw_errors = set(), []
    for r in results:
        i, src, arm = r.get("request_index"), r.get("source_request_index"), r.get("arm")
        if not isinstance(i, int) or i < 0:
            raise ValueError("result request_index must be a non-negative integer")
        if src not in meta:
            raise ValueError("result source_request_index has no metadata row")
        if arm not in arms:
            raise ValueError(f"unexpected result arm: {arm}")
        pair = matrix.setdefault(i, {})
        if arm in pair:
            raise ValueError(f"duplicate result for request {i}/{arm}")
        raw_errors += [f"{i}/{arm}: {e}" for e in validate_token_arrivals(r)]
        pid = r.get("proxy_request_id")
        if not isinstance(pid, str) or not pid:
            raw_errors.append(f"missing proxy request ID for {i}/{arm}")
        elif pid in proxy_ids:
            raw_errors.append(f"duplicate proxy request ID {pid}")
        proxy_ids.add(pid)
        if r.get("warmup") is not False:
            raw_errors.append(f"warmup record leaked into results for {i}/{arm}")
        if r.get("runtime_mode") != ("baseline" if arm == "baseline" else "progressive"):
            raw_errors.append(f"runtime mode mismatch for {i}/{arm}")
        pair[arm] = dict(r)
    complete = set(matrix) == set(range(expected_requests)) and all(set(p) == set(arms) for p in matrix.values())
    sched_by = {}
    for s in scheduler_rows:
        sched_by.setdefault(str(s.get("request_id", "")), []).append(s)
    link_by = {}
    for ln in link_rows:
        link_by.setdefault(str(ln.get("request_id", "")), []).append(ln)
    attn_by: dict[str, list[dict]] = {}
    for at in attention_rows:
        attn_by.setdefault(str(at.get("request_id", "")), []).append(at)
    attn_errors, with_attention = [], 0
    prefill_errors, sched_errors, link_errors, anchor_errors, priority_errors, model_errors = [], [], [], [], [], []
    horizon_errors, one_sched, method_records = [], 0, 0
    groups_seen: set[str] = set()
    rows = []
    for i in sorted(matrix):
        pair = matrix[i]
        srcs = {r["source_request_index"] for r in pair.values()}
        if len(srcs) != 1:
            raw_errors.append(f"arms do not share metadata for request {i}")
            continue
        m = meta[next(iter(srcs))]
        if enforce_paired_prefill:
            groups = {r.get("prefill_group") for r in pair.values()}
            seeds = {r.get("seed_token_id") for r in pair.values()}
            fresh = sum(r.get("prefill_reused") is False for r in pair.values())
            if len(groups) != 1 or not next(iter(groups)):
                prefill_errors.append(f"{i}: arms do not share one prefill group")
            elif next(iter(groups)) in groups_seen:
                prefill_errors.append(f"{i}: prefill group was reused across executions")
            else:
                groups_seen.add(next(iter(groups)))
            if len(seeds) != 1:
                prefill_errors.append(f"{i}: arms do not share one producer seed")
            if fresh != 1:
                prefill_errors.append(f"{i}: expected one producer prefill, got {fresh}")
        enriched = {}
        for arm, r in pair.items():
            name, em, q = score_prediction(str(m.get("dataset", "hotpotqa")), str(r.get("text", "")),
                                           list(m.get("answers", [""])), m.get("all_classes"))
            e = {**r, "metric_name": name, "exact_match": em, "quality_score": q}
            if fixed_output_tokens is not None and len(r["token_ids"]) != fixed_output_tokens:
                horizon_errors.append(f"{i}/{arm}: {len(r['token_ids'])} tokens != {fixed_output_tokens}")
            links = link_by.get(r.get("proxy_request_id", ""), [])
            if len(links) != 1:
                link_errors.append(f"{i}/{arm}: expected one request-attributed link trace, got {len(links)}")
                e["link"] = None
            else:
                e["link"] = links[0]
                first = (links[0].get("bundles") or [{}])[0].get("chunks", [])
                need = set(range(protected_chunks))
                if protected_chunks and not need <= set(first):
                    anchor_errors.append(f"{i}/{arm}: first bundle misses protected anchor chunks")
            if arm != "baseline":
                method_records += 1
                sch = sched_by.get(r.get("proxy_request_id", ""), [])
                if len(sch) == 1:
                    one_sched += 1
                    e["scheduler"] = sch[0]
                    sched_errors += [f"{i}/{arm}: {x}" for x in _scheduler_errors(sch[0], r)]
                    attn = attn_by.get(str(sch[0].get("request_id", "")), [])
                    if attn:
                        with_attention += 1
                        e["attention"], errs = sparse_attention_summary(attn, sch[0], arm)
                        attn_errors += [f"{i}/{arm}: {x}" for x in errs]
                    else:
                        e["attention"] = None
                        attn_errors.append(f"{i}/{arm}: no request-attributed sparse-attention records")
                    if i in priorities and sch[0].get("priority_chunks") != priorities[i]:
                        priority_errors.append(f"{i}/{arm}: scheduler priority differs from the sidecar")
                else:
                    e["scheduler"] = None
            enriched[arm] = e
        row = {"request_index": i, "source_request_index": m.get("request_index"), "arms": enriched,
               "latency_models": {}}
        if "baseline" in enriched:
            for arm in arms:
                if arm != "baseline" and arm in enriched:
                    model, errs = request_latency_model(enriched["baseline"], enriched[arm])
                    model_errors += [f"{i}/{arm}: {x}" for x in errs]
                    if model:
                        row["latency_models"][arm] = model
        rows.append(row)
    equal = all(len({tuple(r["token_ids"]) for r in p["arms"].values()}) == 1 for p in rows)
    gates = {
        "complete_paired_matrix": gate(complete, requests=len(matrix), expected=expected_requests),
        "request_protocol": gate(not raw_errors, errors=raw_errors),
        "single_paired_prefill": gate(not prefill_errors, errors=prefill_errors),
        "fixed_output_horizon": gate(not horizon_errors, errors=horizon_errors),
        "one_scheduler_transition_per_method": gate(one_sched == method_records, records=method_records,
                                                    with_one_scheduler=one_sched),
        "scheduler_transition_invariants": gate(not sched_errors, errors=sched_errors),
        "request_attributed_sparse_attention": gate(with_attention == method_records and not attn_errors,
                                                    records=method_records, with_attention=with_attention,
                                                    errors=attn_errors),
        "fair_controlled_link": gate(not link_errors, errors=link_errors),
        "protected_anchor_arrival": gate(not anchor_errors, errors=anchor_errors),
        "request_scoped_priority_schedule": gate(not priority_errors, errors=priority_errors),
        "latency_model_telemetry": gate(not model_errors, errors=model_errors),
        "exact_greedy_output_equivalence": gate(equal),
    }
    gates["overall"] = gate(all(g["passed"] for g in gates.values()))
    comps = {}
    full = [p for p in rows if all(a in p["arms"] for a in arms)]
    if full:
        if "baseline" in arms:
            comps.update({f"baseline_vs_{a}": pair_comparison(full, "baseline", a, bootstrap_samples=bootstrap_samples,
                                                              seed=seed) for a in arms if a != "baseline"})
        if "fixed_s1" in arms and "continuous" in arms:
            comps["fixed_s1_vs_continuous"] = pair_comparison(full, "fixed_s1", "continuous",
                                                              bootstrap_samples=bootstrap_samples, seed=seed + 100)
    per_arm = {a: {"decode_completion_ms": describe([p["arms"][a]["decode_completion_ms"] for p in full],
                                                    bootstrap_samples=bootstrap_samples, seed=seed + 200),
                   "ttft_ms": describe([p["arms"][a]["ttft_ms"] for p in full], bootstrap_samples=bootstrap_samples,
                                       seed=seed + 300),
                   "quality_score": statistics.fmean(p["arms"][a]["quality_score"] for p in full)}
               for a in arms} if full else {}
    summary = {"status": "passed" if gates["overall"]["passed"] else "failed_gates", "arms": list(arms),
               "requests": len(rows), "gates": gates, "per_arm": per_arm, "comparisons": comps}
    return summary, rows


def write_artifacts(out_dir: Path, summary: dict, rows: Sequence[dict]) -> None:
    out_dir.mkdir(parents=True, exist_ok=True)
    (out_dir / "summary.json").write_text(json.dumps(summary, indent=2, sort_keys=True) + "\n")
    with open(out_dir / "paired_rows.jsonl", "w") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")
    lines = [f"# Live run: {summary['status']}", "", "| gate | passed |", "|---|---|"]
    lines += [f"| {k} | {v['passed']} |" for k, v in summary["gates"].items()]
    lines += ["", "| arm | completion p50 ms | ttft p50 ms | quality |", "|---|---|---|---|"]
    for a, d in summary.get("per_arm", {}).items():
        lines.append(f"| {a} | {d['decode_completion_ms']['p50']:.2f} | {d['ttft_ms']['p50']:.2f} | "
                     f"{d['quality_score']:.4f} |")
    (out_dir / "summary.md").write_text("\n".join(lines) + "\n")
    with open(out_dir / "paper_table.csv", "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["comparison", "token_equality_rate", "completion_gain_mean_ms", "ci_low", "ci_high",
                    "ttft_gain_mean_ms"])
        for k, c in summary.get("comparisons", {}).items():
            g = c["decode_completion_gain_ms"]
            w.writerow([k, c["token_equality_rate"], g["mean"], *g["mean_bootstrap_ci95"],
                        c["decode_ttft_gain_ms"]["mean"]])


def main(argv=None) -> int:
    """Aggregate one live run directory (results / metadata / scheduler / link / attention JSONL) into gated artifacts.

    Counterpart of the reference's experiments/aggregate_progressive_pd_live.py CLI;
    exits 1 when a validity gate fails (the artifacts are written either way).
    """
    import argparse

    from .trace import load_jsonl

    p = argparse.ArgumentParser()
    p.add_argument("--results", type=Path, required=True)
    p.add_argument("--metadata", type=Path, required=True)
    p.add_argument("--scheduler-trace", type=Path, required=True)
    p.add_argument("--link-trace", type=Path, required=True)
    p.add_argument("--attention-trace", type=Path, required=True,
                   help="workers' sparse-view records (attention.jsonl)")
    p.add_argument("--arms", default="baseline,fixed_s1,continuous")
    p.add_argument("--expected-requests", type=int, required=True)
    p.add_argument("--fixed-output-tokens", type=int, default=None)
    p.add_argument("--bootstrap-samples", type=int, default=10000)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--priority-jsonl", type=Path, default=None)
    p.add_argument("--protected-chunks", type=int, default=0)
    p.add_argument("--output-dir", type=Path, required=True)
    a = p.parse_args(argv)
    summary, rows = aggregate_live_run(
        load_jsonl(a.results), load_jsonl(a.metadata), load_jsonl(a.scheduler_trace), load_jsonl(a.link_trace),
        arms=a.arms.split(","), expected_requests=a.expected_requests, fixed_output_tokens=a.fixed_output_tokens,
        bootstrap_samples=a.bootstrap_samples, seed=a.seed,
        priority_rows=load_jsonl(a.priority_jsonl) if a.priority_jsonl else None,
        protected_chunks=a.protected_chunks, attention_rows=load_jsonl(a.attention_trace))
    write_artifacts(a.output_dir, summary, rows)
    print(json.dumps({"status": summary["status"], "output_dir": str(a.output_dir)}))
    return 0 if summary["status"] == "passed" else 1


if __name__ == "__main__":
    raise SystemExit(main())
