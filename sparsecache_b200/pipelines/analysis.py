"""Analyses of P/D pipeline result rows: matched-bandwidth run summary and graft-trigger study.

Both read rows in the layout ``pipelines.pd`` writes (the reference pipeline's
layout): ``protocol`` + ``schedules[name].{full_target, chains[window]}`` with
``chains[window].pipeline.trace`` and an optional ``paired_fixed_control``.

  * ``summarize_run`` (reference: experiments/aggregate_pd_sparse_draft_sweep.py):
    full-target vs pipeline latency (paired), configured / proposed / accepted
    drafts (acceptance counted at the last, full-KV verifier only: summing
    intermediate verifiers would count a tentative prefix several times),
    the stage at which drafting stopped, the residual wire time after the
    first tranche, unattributed time of both arms, the KV fraction visible
    to the proposals, and the paired comparison with the fixed first-stage
    control when it was run.
  * ``analyze_graft_triggers`` (reference: experiments/analyze_pd_graft_triggers.py):
    for each request, the acceptance gain and latency saved by the growing
    ("graft") view over the fixed first-stage view, and how well three
    online triggers would have picked the requests where grafting helps:
    the first proposals' top-1 margins above a threshold (when the rows
    carry ``draft_top1_margins``), a changed first token of the second
    proposal batch, and a changed second batch.  Idealised: the cost of
    probing is not charged.
"""
from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path
from typing import Any, Iterable, Sequence


def describe(values: Iterable[float]) -> dict[str, Any] | None:
    x = sorted(float(v) for v in values)
    if not x:
        return None
    q = lambda p: x[min(len(x) - 1, int(p * len(x)))]  # noqa: E731
    return {"n": len(x), "mean": statistics.fmean(x), "p50": q(0.5), "p90": q(0.9), "p99": q(0.99),
            "min": x[0], "max": x[-1]}


def paired_delta(a: Iterable[float], b: Iterable[float]) -> dict[str, Any] | None:
    """Distribution of a_i - b_i plus how often it is positive / negative."""
    d = [float(x) - float(y) for x, y in zip(a, b)]
    if not d:
        return None
    out = describe(d)
    out.update(positive=sum(v > 0 for v in d), negative=sum(v < 0 for v in d), zero=sum(v == 0 for v in d))
    return out


def _mean(values) -> float | None:
    values = list(values)
    return statistics.fmean(values) if values else None


def _cells(rows: Sequence[dict]) -> list[tuple[dict, dict, dict]]:
    """(full_target, chain cell, pipeline) of every row at the protocol's first schedule / window."""
    out = []
    for r in rows:
        proto = r["protocol"]
        sched = r["schedules"][proto["schedules"][0]]
        chain = sched["chains"][str(proto["commit_windows"][0])]
        out.append((sched["full_target"], chain, chain["pipeline"]))
    return out


def _final_accepted(pipe: dict) -> int:
    verified = [t for t in pipe["trace"] if t.get("verified")]
    return verified[-1]["accepted_pending"] if verified else 0


def _proposed(pipe: dict) -> int:
    return sum(t.get("drafted", 0) for t in pipe["trace"])


def _unattributed(item: dict, keys: Sequence[str]) -> float:
    tr = item.get("transfer", {})
    used = sum(float(item.get(k, 0.0) or 0.0) for k in keys)
    used += float(tr.get("total_h2d_ms", 0.0)) + sum(tr.get("stage_wire_wait_ms", []) or [])
    return max(0.0, float(item["response_ms"]) - used)


def summarize_run(rows: Sequence[dict]) -> dict[str, Any]:
    if not rows:
        raise ValueError("no rows")
    cells = _cells(rows)
    targets = [t for t, _, _ in cells]
    pipes = [p for _, _, p in cells]
    target_ms = [t["response_ms"] for t in targets]
    pipe_ms = [p["response_ms"] for p in pipes]
    accepted = [_final_accepted(p) for p in pipes]
    proposed = [_proposed(p) for p in pipes]
    intermediate = [sum(t["accepted_pending"] for t in [s for s in p["trace"] if s.get("verified")][:-1])
                    for p in pipes]
    terminated: dict[str, int] = {}
    for p in pipes:
        k = str(int(p.get("terminated_stage", 0)) + 1)
        terminated[k] = terminated.get(k, 0) + 1
    protocol = rows[0]["protocol"]
    out: dict[str, Any] = {
        "transport_gbps": protocol.get("transport_gbps"),
        "cases": len(rows),
        "latency": {
            "full_target_ms": describe(target_ms),
            "pipeline_ms": describe(pipe_ms),
            "saved_vs_full_target_ms": paired_delta(target_ms, pipe_ms),
            "speedup_ratio_of_means": _mean(target_ms) / _mean(pipe_ms),
            "full_target_first_decode_token_ms": describe(t["response_ms"] - t.get("decode_ms", 0.0)
                                                          for t in targets),
            "pipeline_first_committed_ms": describe(p["first_committed_ms"] for p in pipes
                                                    if p.get("first_committed_ms") is not None),
        },
        "drafts": {
            "configured": describe(c.get("configured_draft_tokens", protocol.get("draft_tokens", 0))
                                   for _, c, _ in cells),
            "proposed": describe(proposed),
            "accepted_at_final_verifier": describe(accepted),
            "accepted_fraction": describe(a / max(1, n) for a, n in zip(accepted, proposed)),
            "intermediate_accepted_checks": describe(intermediate),
        },
        "terminated_stage_counts": dict(sorted(terminated.items())),
        "timing_token_match_target_rate": _mean(bool(c.get("timing_token_match_target")) for _, c, _ in cells),
        "sparse_draft_ms": describe(p.get("draft_prefill_ms", 0.0) + p.get("draft_decode_ms", 0.0) for p in pipes),
        "residual_wire_ms": describe(sum((p.get("transfer", {}).get("stage_wire_ms") or [0.0])[1:]) for p in pipes),
        "unattributed_ms": {
            "full_target": describe(_unattributed(t, ("seed_forward_ms", "decode_ms")) for t in targets),
            "pipeline": describe(_unattributed(p, ("draft_prefill_ms", "draft_decode_ms", "final_prefill_ms",
                                                   "final_correction_ms", "final_decode_ms", "verify_ms"))
                                 for p in pipes),
        },
    }
    fracs = [p.get("visible_fraction_per_draft") for p in pipes]
    if all(f is not None for f in fracs):
        out["proposal_visibility"] = {
            "mean_visible_kv_fraction_per_request": describe(_mean(f) or 0.0 for f in fracs),
            "last_proposal_visible_kv_fraction": describe(f[-1] for f in fracs if f),
            "proposal_fraction_after_first_stage": describe(
                _mean(v > f[0] for v in f) or 0.0 for f in fracs if f),
        }
    fixed = [c.get("paired_fixed_control") for _, c, _ in cells]
    if fixed and all(f is not None for f in fixed):
        f_acc = [_final_accepted(f) for f in fixed]
        f_prop = [_proposed(f) for f in fixed]
        out["paired_fixed_control"] = {
            "latency_saved_by_method_ms": paired_delta((f["response_ms"] for f in fixed), pipe_ms),
            "accepted_token_delta_method_minus_fixed": paired_delta(accepted, f_acc),
            "proposal_token_delta_method_minus_fixed": paired_delta(proposed, f_prop),
            "accepted_fraction_delta_method_minus_fixed": paired_delta(
                (a / max(1, n) for a, n in zip(accepted, proposed)),
                (a / max(1, n) for a, n in zip(f_acc, f_prop))),
            "fixed_response_ms": describe(f["response_ms"] for f in fixed),
            "fixed_sparse_draft_ms": describe(f.get("draft_prefill_ms", 0.0) + f.get("draft_decode_ms", 0.0)
                                              for f in fixed),
        }
    return out


def _draft_batches(pipe: dict) -> list[list[int]]:
    return [list(t["draft_token_ids"]) for t in pipe["trace"] if t.get("drafted", 0) > 0]


def analyze_graft_triggers(rows: Sequence[dict], *, margin_threshold: float = 6.0) -> dict[str, Any]:
    """Graft (growing view) vs fixed first-stage view per request, and three trigger policies."""
    cases, skipped = [], []
    for r, (_, chain, graft) in zip(rows, _cells(rows)):
        fixed = chain.get("paired_fixed_control")
        if fixed is None:
            raise ValueError("rows were written without the paired fixed control")
        fixed_batches = _draft_batches(fixed)
        fixed_tokens = [t for b in fixed_batches for t in b]
        batches = _draft_batches(graft)
        if len(batches) < 2 or len(fixed_tokens) < 4:
            skipped.append(r.get("dataset_index"))
            continue
        first, second = batches[0], batches[1]
        prefix_changed = first != fixed_tokens[:len(first)]
        s2 = len(first)
        margins = graft["trace"][0].get("draft_top1_margins")
        cases.append({
            "dataset_index": r.get("dataset_index"),
            "acceptance_gain": _final_accepted(graft) - _final_accepted(fixed),
            "latency_saved_ms": float(fixed["response_ms"]) - float(graft["response_ms"]),
            "margin_trigger": None if not margins else min(margins) >= margin_threshold,
            "s2_first_token_instability": prefix_changed or (s2 >= len(fixed_tokens)
                                                             or second[0] != fixed_tokens[s2]),
            "s2_batch_instability": prefix_changed or second != fixed_tokens[s2:s2 + len(second)],
        })

    def trigger_summary(key: str) -> dict[str, Any] | None:
        if any(c[key] is None for c in cases):
            return None  # rows without margin telemetry
        hit = [c for c in cases if c[key]]
        return {"triggered": len(hit),
                "true_positive": sum(c["acceptance_gain"] > 0 for c in hit),
                "false_positive": sum(c["acceptance_gain"] <= 0 for c in hit),
                "missed_positive": sum(c["acceptance_gain"] > 0 and not c[key] for c in cases),
                "latency_positive_when_triggered": sum(c["latency_saved_ms"] > 0 for c in hit),
                "idealized_policy_latency_saved_ms": describe(c["latency_saved_ms"] if c[key] else 0.0
                                                              for c in cases),
                "probe_cost_charged": False}

    return {"cases": len(cases), "skipped": skipped, "margin_threshold": margin_threshold,
            "unconditional_graft": {"latency_saved_ms": describe(c["latency_saved_ms"] for c in cases),
                                    "acceptance_gain": describe(c["acceptance_gain"] for c in cases)},
            "triggers": {k: trigger_summary(k) for k in ("margin_trigger", "s2_first_token_instability",
                                                          "s2_batch_instability")},
            "rows": cases}


def load_rows(path: str | Path) -> list[dict]:
    return [json.loads(line) for line in Path(path).read_text().splitlines()
            if line.strip() and "schedules" in json.loads(line)]


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("kind", choices=("run", "triggers"))
    p.add_argument("inputs", nargs="+")
    p.add_argument("--margin-threshold", type=float, default=6.0)
    p.add_argument("--output", type=Path, default=None)
    a = p.parse_args(argv)
    if a.kind == "run":
        out = {str(Path(x)): summarize_run(load_rows(x)) for x in a.inputs}
    else:
        out = {str(Path(x)): analyze_graft_triggers(load_rows(x), margin_threshold=a.margin_threshold)
               for x in a.inputs}
    text = json.dumps(out, indent=2)
    if a.output is not None:
        a.output.parent.mkdir(parents=True, exist_ok=True)
        a.output.write_text(text + "\n")
    print(text)


if __name__ == "__main__":
    main()
