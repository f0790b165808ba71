"""Request-level chunk priority orders (the P/D transfer schedule sidecars).

Parity with the reference's experiments/build_ruler_chunk_priorities.py:
uniform bisection order (:56-71), per-request BM25 with k1 = 1.2, b = 0.75
(:77-104), protected-first reordering (:107-117), chunk scores from document
spans (:120-132), prompt-marker span recovery (:145-182) and the five modes
sequential / uniform / random (hashed seed) / bm25 / oracle (:185-235).
Every order returned is a complete permutation of the chunk indices with the
protected prefix and suffix chunks first.  ``build_priority_sidecars`` writes a
pack's per-mode sidecars, its document spans and the passing audit (:236-400).
"""
from __future__ import annotations

import hashlib
import json
import math
import random
import re
from collections import Counter
from pathlib import Path
from typing import Any, Sequence

MODES = ("sequential", "uniform", "random", "bm25", "oracle")
_TERM = re.compile(r"[a-z0-9]+")


def uniform_order(total: int) -> list[int]:
    """0, last, then midpoints of every interval, breadth first."""
    if total < 3:
        return list(range(total))
    order = [0, total - 1]
    level = [(0, total - 1)]
    while level:
        nxt = []
        for lo, hi in level:
            if hi - lo <= 1:
                continue
            mid = (lo + hi) // 2
            order.append(mid)
            nxt += [(lo, mid), (mid, hi)]
        level = nxt
    return order


def terms(text: str) -> list[str]:
    return _TERM.findall(text.lower())


def bm25_scores(question: str, documents: Sequence[str], *, k1: float = 1.2, b: float = 0.75) -> list[float]:
    """Per-request BM25 of each document against the question (query-term counts weighted)."""
    toks = [terms(d) for d in documents]
    q = Counter(terms(question))
    n = len(toks)
    avg = sum(map(len, toks)) / max(n, 1)
    df = Counter(t for d in toks for t in set(d))
    out = []
    for d in toks:
        tf = Counter(d)
        s = 0.0
        for term, qf in q.items():
            f = tf[term]
            if f:
                idf = math.log(1.0 + (n - df[term] + 0.5) / (df[term] + 0.5))
                s += qf * idf * f * (k1 + 1.0) / (f + k1 * (1.0 - b + b * len(d) / max(avg, 1.0)))
        out.append(s)
    return out


def protected_first(order: Sequence[int], total: int, prefix_chunks: int, suffix_chunks: int) -> list[int]:
    keep = set(range(min(prefix_chunks, total))) | set(range(max(0, total - suffix_chunks), total))
    return [c for c in order if c in keep] + [c for c in order if c not in keep]


def chunk_scores(spans: Sequence[dict], document_scores: Sequence[float], total: int, chunk_tokens: int):
    """Each chunk takes the best score of any document overlapping it (-inf if none)."""
    out = [-math.inf] * total
    for span, s in zip(spans, document_scores, strict=True):
        for c in range(int(span["start_token"]) // chunk_tokens,
                       min(-(-int(span["end_token"]) // chunk_tokens), total)):
            out[c] = max(out[c], s)
    return out


def find_subsequence(values: Sequence[int], pattern: Sequence[int], start: int) -> int:
    if not pattern:
        raise ValueError("marker token sequence must be non-empty")
    pattern = list(pattern)
    for i in range(start, len(values) - len(pattern) + 1):
        if list(values[i:i + len(pattern)]) == pattern:
            return i
    raise ValueError(f"prompt does not contain expected marker after token {start}")


def document_spans_from_prompt_markers(tokenizer, prompt: Sequence[int], source: dict, placement: str,
                                       protected_suffix_tokens: int):
    """Recover displayed document token spans from the "Document i:" markers of a built prompt."""
    order = source["placements"][placement]
    starts, cursor = [], 0
    for shown in range(1, len(order) + 1):
        marker = tokenizer.encode(f"Document {shown}:\n", add_special_tokens=False)
        cursor = find_subsequence(prompt, marker, cursor)
        starts.append(cursor)
        cursor += len(marker)
    last_end = len(prompt) - protected_suffix_tokens
    if not starts or last_end <= starts[0]:
        raise ValueError("protected suffix leaves no schedulable document tokens")
    spans, docs = [], []
    for i, src in enumerate(order):
        d = source["documents"][src]
        raw_end = starts[i + 1] if i + 1 < len(starts) else len(prompt)
        spans.append({"source_document_index": src, "start_token": min(starts[i], last_end),
                      "end_token": min(raw_end, last_end), "supporting": bool(d["supporting"])})
        docs.append(d)
    return spans, docs


def priority_for_mode(mode: str, *, request_id: str, question: str, documents: Sequence[dict],
                      spans: Sequence[dict], total_chunks: int, chunk_tokens: int, protected_prefix_chunks: int,
                      protected_suffix_chunks: int, seed: int) -> list[int]:
    uni = uniform_order(total_chunks)
    if mode == "sequential":
        order = list(range(total_chunks))
    elif mode == "uniform":
        order = uni
    elif mode == "random":
        order = list(range(total_chunks))
        digest = hashlib.sha256(f"{seed}:{request_id}".encode()).digest()
        random.Random(int.from_bytes(digest[:8], "big")).shuffle(order)
    elif mode in ("bm25", "oracle"):
        ds = (bm25_scores(question, [str(d["text"]) for d in documents]) if mode == "bm25"
              else [float(bool(d["supporting"])) for d in documents])
        cs = chunk_scores(spans, ds, total_chunks, chunk_tokens)
        rank = {c: r for r, c in enumerate(uni)}
        order = sorted(range(total_chunks), key=lambda c: (-cs[c], rank[c]))
    else:
        raise ValueError(f"unsupported priority mode: {mode}")
    out = protected_first(order, total_chunks, protected_prefix_chunks, protected_suffix_chunks)
    if sorted(out) != list(range(total_chunks)):
        raise AssertionError("chunk priority is not a complete permutation")
    return out


def coverage_curve(order: Sequence[int], spans: Sequence[dict[str, Any]], chunk_tokens: int) -> list[float]:
    """Fraction of supporting-document tokens visible after each chunk of ``order`` arrives."""
    support = set()
    for s in spans:
        if s["supporting"]:
            support.update(range(int(s["start_token"]), int(s["end_token"])))
    if not support:
        return [1.0] * len(order)
    seen, out = 0, []
    for c in order:
        seen += sum(1 for t in range(c * chunk_tokens, (c + 1) * chunk_tokens) if t in support)
        out.append(seen / len(support))
    return out


def _read_jsonl(path) -> list[dict]:
    rows = [json.loads(x) for x in Path(path).read_text(encoding="utf-8").splitlines() if x.strip()]
    if not rows:
        raise ValueError(f"{path} contains no rows")
    return rows


def build_priority_sidecars(pack_dir, output_dir, *, modes: Sequence[str] = MODES, chunk_tokens: int = 256,
                            protected_prefix_tokens: int = 256, protected_suffix_tokens: int = 512,
                            seed: int = 20260827, tokenizer=None) -> dict[str, Any]:
    """Write ``priority_<mode>.jsonl`` sidecars, ``document_spans.jsonl`` and ``audit.json`` for a RULER pack.

    Reference: experiments/build_ruler_chunk_priorities.py:236-400.  Document
    spans come from the pack metadata when the pack builder recorded them
    (``pack_metadata_spans``); otherwise they are recovered from the
    "Document i:" markers of the immutable prompt ids (``exact_token_marker_scan``,
    which needs ``tokenizer``).  Every row of every mode is a full permutation of
    the prompt's chunks with the protected prefix / suffix chunks first.
    """
    from .audits import _sha256

    modes = tuple(modes)
    if not modes or len(set(modes)) != len(modes) or any(m not in MODES for m in modes):
        raise ValueError(f"modes must be unique values from {MODES}")
    if min(chunk_tokens, protected_prefix_tokens, protected_suffix_tokens) <= 0:
        raise ValueError("chunk and protected token counts must be positive")
    pack_dir, output_dir = Path(pack_dir), Path(output_dir)
    if output_dir.exists():
        raise FileExistsError(f"refusing to overwrite {output_dir}")
    manifest = json.loads((pack_dir / "manifest.json").read_text(encoding="utf-8"))
    if manifest.get("dataset") != "ruler_qa2":
        raise ValueError("chunk scheduling needs a RULER qa_2 pack")
    prompt_tokens = int(manifest["prompt_tokens"])
    if prompt_tokens % chunk_tokens:
        raise ValueError("the prompt length must hold whole scheduling chunks")
    sources = _read_jsonl(manifest["source"])
    req_path, meta_path = pack_dir / "requests.jsonl", pack_dir / "metadata.jsonl"
    requests, metadata = _read_jsonl(req_path), _read_jsonl(meta_path)
    if len(requests) != len(metadata):
        raise ValueError("request and metadata row counts differ")
    total = prompt_tokens // chunk_tokens
    pre, suf = math.ceil(protected_prefix_tokens / chunk_tokens), math.ceil(protected_suffix_tokens / chunk_tokens)
    out_rows: dict[str, list[dict]] = {m: [] for m in modes}
    span_rows, recon = [], Counter()
    for index, (req, meta) in enumerate(zip(requests, metadata)):
        source = sources[int(meta["source_index"])]
        rid = str(meta.get("id", source.get("id", index)))
        if meta.get("document_spans"):
            spans = [dict(s) for s in meta["document_spans"]]
            docs = [source["documents"][int(s["source_document_index"])] for s in spans]
            how = "pack_metadata_spans"
        else:
            if tokenizer is None:
                raise ValueError("the pack has no document spans; a tokenizer is needed to recover them")
            spans, docs = document_spans_from_prompt_markers(tokenizer, req["prompt"], source, manifest["placement"],
                                                             protected_suffix_tokens)
            how = "exact_token_marker_scan"
        recon[how] += 1
        span_rows.append({"request_index": index, "id": rid, "prefix_tokens": int(spans[0]["start_token"]),
                          "suffix_tokens": len(req["prompt"]) - int(spans[-1]["end_token"]),
                          "coordinate_reconstruction": how, "document_spans": spans})
        for mode in modes:
            out_rows[mode].append({"request_index": index, "id": rid, "mode": mode, "priority_chunks": priority_for_mode(
                mode, request_id=rid, question=str(source["question"]), documents=docs, spans=spans,
                total_chunks=total, chunk_tokens=chunk_tokens, protected_prefix_chunks=pre,
                protected_suffix_chunks=suf, seed=seed)})
    output_dir.mkdir(parents=True)
    spans_path = output_dir / "document_spans.jsonl"
    spans_path.write_text("".join(json.dumps(r, ensure_ascii=False) + "\n" for r in span_rows), encoding="utf-8")
    hashes = {}
    for mode, rows in out_rows.items():
        path = output_dir / f"priority_{mode}.jsonl"
        path.write_text("".join(json.dumps(r) + "\n" for r in rows), encoding="utf-8")
        hashes[mode] = _sha256(path)
    audit = {"schema_version": 1, "status": "passed", "pack_dir": str(pack_dir), "requests": len(requests),
             "prompt_tokens": prompt_tokens, "chunk_tokens": chunk_tokens,
             "protected_prefix_tokens": protected_prefix_tokens, "protected_suffix_tokens": protected_suffix_tokens,
             "modes": list(modes), "online_modes": [m for m in modes if m != "oracle"],
             "analysis_upper_bound_modes": [m for m in modes if m == "oracle"],
             "coordinate_reconstruction_modes": dict(recon), "requests_sha256": _sha256(req_path),
             "metadata_sha256": _sha256(meta_path), "document_spans_sha256": _sha256(spans_path),
             "priority_sha256": hashes}
    (output_dir / "audit.json").write_text(json.dumps(audit, indent=2) + "\n", encoding="utf-8")
    return audit
