"""Fail-closed audits of request packs, dataset matrices and priority coverage, and the
quality audit of generated token ids.

Parity with the reference's experiments/audit_pd_request_packs.py and audit_ruler_pd_packs.py
(manifest identity, request/metadata hashes, contiguous request indices, chunk-aligned prompt
lengths), audit_iclr_dataset_matrix.py (every dataset x length cell present and passing),
analyze_ruler_priority_coverage.py (supporting-evidence coverage after each arrived chunk of a
priority order) and evaluate_eagle3_quality.py (decode token ids, join them with the pack
metadata and score with the LongBench metrics).
"""
from __future__ import annotations

import hashlib
import json
import statistics
from pathlib import Path
from typing import Any, Callable, Sequence

from .longbench import score_prediction
from .priorities import coverage_curve


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _jsonl(path: Path) -> list[dict]:
    return [json.loads(x) for x in Path(path).read_text(encoding="utf-8").splitlines() if x.strip()]


def audit_pack(pack_dir: Path, *, expected_dataset: str | None = None, chunk_tokens: int | None = None) -> dict:
    """Hash, identity, row-count, index and chunk-alignment checks of one pack; raises on failure."""
    pack_dir = Path(pack_dir)
    man = json.loads((pack_dir / "manifest.json").read_text(encoding="utf-8"))
    if expected_dataset is not None and man.get("dataset") != expected_dataset:
        raise ValueError(f"dataset mismatch in {pack_dir}")
    for name in ("requests", "metadata"):
        want = man.get(f"{name}_sha256")
        if want is not None and _sha256(pack_dir / f"{name}.jsonl") != want:
            raise ValueError(f"{name} hash mismatch in {pack_dir}")
    reqs, meta = _jsonl(pack_dir / "requests.jsonl"), _jsonl(pack_dir / "metadata.jsonl")
    if len(reqs) != len(meta):
        raise ValueError(f"request/metadata row count mismatch in {pack_dir}")
    chunk = chunk_tokens or man.get("chunk_tokens")
    lengths = []
    for i, (r, m) in enumerate(zip(reqs, meta)):
        if m.get("request_index", i) != i:
            raise ValueError(f"non-contiguous request index in {pack_dir}")
        toks = r.get("prompt")
        if not isinstance(toks, list) or not toks:
            raise ValueError(f"row {i} of {pack_dir} has no token prompt")
        if chunk and len(toks) % int(chunk):
            raise ValueError(f"row {i} of {pack_dir} is not chunk aligned")
        lengths.append(len(toks))
    return {"pack": str(pack_dir), "dataset": man.get("dataset"), "rows": len(reqs),
            "mean_prompt_tokens": statistics.fmean(lengths), "max_prompt_tokens": max(lengths), "status": "passed"}


def audit_dataset_matrix(root: Path, datasets: Sequence[str], lengths: Sequence[int] | None = None,
                         **kw) -> dict[str, Any]:
    """Every dataset (x length) pack under ``root`` passes ``audit_pack``."""
    cells, failures = {}, []
    for ds in datasets:
        for length in (lengths or [None]):
            d = Path(root) / ds / (str(length) if length is not None else "")
            key = f"{ds}/{length}" if length is not None else ds
            try:
                cells[key] = audit_pack(d, expected_dataset=ds, **kw)
            except (OSError, ValueError) as exc:
                failures.append(f"{key}: {exc}")
    return {"status": "passed" if not failures else "failed", "cells": cells, "failures": failures}


def priority_coverage(order: Sequence[int], spans: Sequence[dict], chunk_tokens: int,
                      fractions: Sequence[float] = (0.05, 0.1, 0.2, 0.5)) -> dict[str, float]:
    """Evidence coverage once the first fraction of the chunks (in priority order) has arrived."""
    curve = coverage_curve(order, spans, chunk_tokens)
    return {f"{f:g}": curve[max(0, min(len(curve) - 1, int(f * len(curve)) - 1))] for f in fractions}


def quality_audit(records: Sequence[dict], metadata: Sequence[dict], decode: Callable[[list[int]], str]) -> dict:
    """Score generated token ids against the pack metadata (per dataset and overall)."""
    by_index = {m.get("request_index", i): m for i, m in enumerate(metadata)}
    per_ds: dict[str, list[float]] = {}
    rows = []
    for r in records:
        m = by_index[r["request_index"]]
        text = decode(list(r["token_ids"]))
        name, em, score = score_prediction(m["dataset"], text, m.get("answers", []), m.get("all_classes"))
        per_ds.setdefault(m["dataset"], []).append(score)
        rows.append({"request_index": r["request_index"], "dataset": m["dataset"], "metric": name, "em": em,
                     "score": score})
    return {"overall": statistics.fmean(x["score"] for x in rows) if rows else None,
            "per_dataset": {k: statistics.fmean(v) for k, v in per_ds.items()}, "rows": rows}


def _percentile_rank(values: Sequence[int], q: float) -> float:
    import math

    if not values:
        return 0.0
    xs = sorted(values)
    return float(xs[min(len(xs) - 1, math.ceil(q * len(xs)) - 1)])


def _coverage_summary(rows: Sequence[dict]) -> dict[str, Any]:
    if not rows:
        raise ValueError("cannot summarise an empty coverage split")
    return {"requests": len(rows),
            "any_support_chunk_rate": statistics.fmean(float(r["selected_support_chunks"] > 0) for r in rows),
            "all_support_chunks_rate": statistics.fmean(float(r["support_chunk_recall"] == 1.0) for r in rows),
            "mean_support_chunk_recall": statistics.fmean(r["support_chunk_recall"] for r in rows),
            "all_support_documents_touched_rate": statistics.fmean(float(r["support_document_recall"] == 1.0)
                                                                  for r in rows),
            "mean_support_document_recall": statistics.fmean(r["support_document_recall"] for r in rows),
            "all_support_chunks_rank_p50": _percentile_rank([r["all_support_chunks_rank"] for r in rows], 0.5),
            "all_support_chunks_rank_p95": _percentile_rank([r["all_support_chunks_rank"] for r in rows], 0.95)}


def analyze_priority_coverage(schedule_root: Path, *, fractions: Sequence[float],
                              selection_requests: int) -> dict[str, Any]:
    """Evidence coverage of every priority mode at chunk budgets, split into selection / confirmation rows.

    Reference: experiments/analyze_ruler_priority_coverage.py.  For each
    fraction f the first ceil(f * chunks) chunks of the order are "arrived":
    supporting-chunk recall, supporting-document touch rate and the rank at
    which the last supporting chunk arrives.
    """
    import math

    if not fractions or len(set(fractions)) != len(fractions) or any(not 0 < f <= 1 for f in fractions):
        raise ValueError("fractions must be unique and lie in (0, 1]")
    root = Path(schedule_root)
    audit = json.loads((root / "audit.json").read_text(encoding="utf-8"))
    if audit.get("status") != "passed":
        raise ValueError("the priority schedule audit has not passed")
    n = int(audit["requests"])
    if not 0 < selection_requests < n:
        raise ValueError("the selection split must leave a non-empty confirmation split")
    chunk = int(audit["chunk_tokens"])
    total = int(audit["prompt_tokens"]) // chunk
    spans = _jsonl(root / "document_spans.jsonl")
    if len(spans) != n:
        raise ValueError("document span row count differs from the audit")
    modes = {}
    for mode in audit["modes"]:
        prio = _jsonl(root / f"priority_{mode}.jsonl")
        if len(prio) != n:
            raise ValueError("priority row count differs from the audit")
        per_fraction = {}
        for f in fractions:
            budget = math.ceil(total * f)
            rows = []
            for i, (srow, prow) in enumerate(zip(spans, prio)):
                if int(srow.get("request_index", -1)) != i or int(prow.get("request_index", -1)) != i:
                    raise ValueError("request order differs across scheduling files")
                order = prow.get("priority_chunks")
                if not isinstance(order, list) or sorted(order) != list(range(total)):
                    raise ValueError("priority row is not a complete permutation")
                docs = [set(range(int(s["start_token"]) // chunk, math.ceil(int(s["end_token"]) / chunk)))
                        for s in srow["document_spans"] if s.get("supporting") is True]
                if not docs:
                    raise ValueError("request has no supporting document span")
                support = set().union(*docs)
                rank = {c: k + 1 for k, c in enumerate(order)}
                chosen = set(order[:budget])
                rows.append({"request_index": i, "support_chunks": len(support),
                             "selected_support_chunks": len(chosen & support),
                             "support_chunk_recall": len(chosen & support) / len(support),
                             "support_document_recall": sum(bool(chosen & d) for d in docs) / len(docs),
                             "all_support_chunks_rank": max(rank[c] for c in support)})
            per_fraction[str(f)] = {"fraction": f, "budget_chunks": budget, "budget_tokens": budget * chunk,
                                    "all": _coverage_summary(rows),
                                    "selection": _coverage_summary(rows[:selection_requests]),
                                    "confirmation": _coverage_summary(rows[selection_requests:])}
        modes[mode] = per_fraction
    return {"schema_version": 1, "status": "passed", "schedule_root": str(root), "requests": n,
            "selection_rows": [0, selection_requests], "confirmation_rows": [selection_requests, n],
            "prompt_tokens": int(audit["prompt_tokens"]), "chunk_tokens": chunk, "total_chunks": total,
            "fractions": list(fractions), "modes": modes}
