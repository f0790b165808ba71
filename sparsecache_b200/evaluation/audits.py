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
