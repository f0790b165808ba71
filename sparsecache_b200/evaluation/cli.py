"""Command lines of the evaluation data pipeline.

    python -m sparsecache_b200.evaluation.cli normalize-ruler --source-hotpot H.json --input-root R --output-root N
    python -m sparsecache_b200.evaluation.cli ruler-pack --dataset N/qa2_65536.jsonl --placement original \\
        --tokenizer M --prompt-tokens 65536 --output-dir P
    python -m sparsecache_b200.evaluation.cli longbench-pack --dataset qmsum.jsonl --dataset-name qmsum \\
        --tokenizer M --output-dir P
    python -m sparsecache_b200.evaluation.cli priorities --pack-dir P --output-dir S
    python -m sparsecache_b200.evaluation.cli audit-packs --root PACKS --datasets qmsum,hotpotqa --output A.json
    python -m sparsecache_b200.evaluation.cli audit-ruler --root PACKS --lengths 16384,65536 --output A.json
    python -m sparsecache_b200.evaluation.cli priority-coverage --schedule-root S --output C.json
    python -m sparsecache_b200.evaluation.cli quality --result-dir RUN --metadata-jsonl P/metadata.jsonl \\
        --model M --output Q.json

Counterparts of the reference's experiments/normalize_ruler_qa2.py,
build_ruler_pd_pack.py, build_longbench_pd_pack.py,
build_ruler_chunk_priorities.py, audit_pd_request_packs.py,
audit_ruler_pd_packs.py / audit_iclr_dataset_matrix.py,
analyze_ruler_priority_coverage.py and evaluate_eagle3_quality.py, with the
same flag names.  ``--tokenizer`` / ``--model`` name a model directory: its
Hugging Face tokenizer when it ships one, else the byte-level tokenizer of
this package (random-init models).  Every writer refuses to overwrite.
"""
from __future__ import annotations

import argparse
import json
import random
from pathlib import Path
from typing import Any

LONGBENCH_DATASETS = ("2wikimqa", "hotpotqa", "musique", "qasper", "multifieldqa_en", "narrativeqa", "qmsum",
                      "gov_report", "multi_news", "passage_retrieval_en", "passage_count", "lcc", "repobench-p")
RULER_PLACEMENTS = ("original", "evidence_first", "evidence_uniform", "evidence_last", "adversarial_split")


def _tokenizer(path: str):
    from ..tokenizer import load_tokenizer

    root = Path(path)
    vocab, eos = 128256, (2,)
    if (root / "config.json").exists():
        cfg = json.loads((root / "config.json").read_text())
        vocab = int(cfg.get("vocab", cfg.get("vocab_size", vocab)))
        eos = tuple(cfg.get("eos_token_ids", ())) or eos
    return load_tokenizer(root, vocab, eos=eos)


def _ints(text: str) -> list[int]:
    return [int(x) for x in text.split(",") if x.strip()]


def _write(path: Path | None, payload: dict) -> None:
    text = json.dumps(payload, indent=2, ensure_ascii=False)
    if path is not None:
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(text + "\n", encoding="utf-8")
    print(text)


def _bootstrap_ci(values, samples: int, seed: int):
    if not values:
        return None
    rng = random.Random(seed)
    n = len(values)
    est = sorted(sum(values[rng.randrange(n)] for _ in range(n)) / n for _ in range(samples))
    return [est[int(0.025 * samples)], est[min(samples - 1, int(0.975 * samples))]]


def cmd_quality(a) -> dict[str, Any]:
    """Score a run's generated token ids against pack metadata (reference: evaluate_eagle3_quality.py:103-242)."""
    from .audits import quality_audit

    tok = _tokenizer(a.model)
    metadata = [json.loads(x) for x in a.metadata_jsonl.read_text(encoding="utf-8").splitlines() if x.strip()]
    records = []
    for path in sorted(a.result_dir.glob("*.jsonl")):
        for line in path.read_text(encoding="utf-8").splitlines():
            if not line.strip():
                continue
            row = json.loads(line)
            if "request_index" in row and "token_ids" in row:
                records.append({"request_index": int(row["request_index"]), "token_ids": row["token_ids"]})
    if not records:
        raise ValueError(f"no result rows with request_index and token_ids under {a.result_dir}")
    seen = [r["request_index"] for r in records]
    if len(seen) != len(set(seen)):
        raise ValueError("duplicate request indices across result files")
    out = quality_audit(records, metadata, lambda ids: tok.decode(ids, skip_special_tokens=True))
    scores = [r["score"] for r in out["rows"]]
    out["overall_bootstrap_ci95"] = _bootstrap_ci(scores, a.bootstrap_samples, a.seed)
    out["requests"] = len(records)
    _write(a.output, out)
    return out


def main(argv=None) -> dict[str, Any]:
    from . import audits, longbench, priorities, ruler

    p = argparse.ArgumentParser()
    sub = p.add_subparsers(dest="cmd", required=True)
    n = sub.add_parser("normalize-ruler")
    n.add_argument("--source-hotpot", type=Path, required=True)
    n.add_argument("--input-root", type=Path, required=True)
    n.add_argument("--output-root", type=Path, required=True)
    n.add_argument("--lengths", default="16384,32768,65536,131072")
    r = sub.add_parser("ruler-pack")
    r.add_argument("--dataset", type=Path, required=True)
    r.add_argument("--placement", required=True, choices=RULER_PLACEMENTS)
    r.add_argument("--tokenizer", required=True)
    r.add_argument("--served-model-name", default="sparsecache-llama31-8b")
    r.add_argument("--prompt-tokens", type=int, required=True)
    r.add_argument("--output-tokens", type=int, default=32)
    r.add_argument("--num-requests", type=int)
    r.add_argument("--output-dir", type=Path, required=True)
    r.add_argument("--disable-thinking", action="store_true")
    lb = sub.add_parser("longbench-pack")
    lb.add_argument("--dataset", type=Path, required=True)
    lb.add_argument("--dataset-name", required=True)
    lb.add_argument("--format", choices=("longbench", "longbench_v2"), default="longbench")
    lb.add_argument("--tokenizer", required=True)
    lb.add_argument("--served-model-name", default="sparsecache-llama31-8b")
    lb.add_argument("--output-dir", type=Path, required=True)
    lb.add_argument("--num-requests", type=int)
    lb.add_argument("--max-prompt-tokens", type=int, default=32768)
    lb.add_argument("--chunk-tokens", type=int, default=256)
    lb.add_argument("--fixed-output-tokens", type=int)
    lb.add_argument("--disable-thinking", action="store_true")
    pr = sub.add_parser("priorities")
    pr.add_argument("--pack-dir", type=Path, required=True)
    pr.add_argument("--output-dir", type=Path, required=True)
    pr.add_argument("--modes", default=",".join(priorities.MODES))
    pr.add_argument("--chunk-tokens", type=int, default=256)
    pr.add_argument("--protected-prefix-tokens", type=int, default=256)
    pr.add_argument("--protected-suffix-tokens", type=int, default=512)
    pr.add_argument("--seed", type=int, default=20260827)
    pr.add_argument("--tokenizer", default=None, help="only for packs without recorded document spans")
    ap = sub.add_parser("audit-packs")
    ap.add_argument("--root", type=Path, required=True)
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--datasets", default=",".join(LONGBENCH_DATASETS))
    ar = sub.add_parser("audit-ruler")
    ar.add_argument("--root", type=Path, required=True)
    ar.add_argument("--output", type=Path, required=True)
    ar.add_argument("--lengths", default="16384,32768,65536,131072")
    ar.add_argument("--placements", default=",".join(RULER_PLACEMENTS))
    ar.add_argument("--requests-per-cell", type=int, default=200)
    pc = sub.add_parser("priority-coverage")
    pc.add_argument("--schedule-root", type=Path, required=True)
    pc.add_argument("--output", type=Path, required=True)
    pc.add_argument("--fractions", default="0.02,0.05,0.10,0.20")
    pc.add_argument("--selection-requests", type=int, default=100)
    q = sub.add_parser("quality")
    q.add_argument("--result-dir", type=Path, required=True)
    q.add_argument("--metadata-jsonl", type=Path, required=True)
    q.add_argument("--model", required=True)
    q.add_argument("--output", type=Path)
    q.add_argument("--bootstrap-samples", type=int, default=10_000)
    q.add_argument("--seed", type=int, default=20260827)
    a = p.parse_args(argv)

    if a.cmd == "normalize-ruler":
        out = ruler.normalize_tree(a.source_hotpot, a.input_root, a.output_root, _ints(a.lengths))
        _write(None, out)
        return out
    if a.cmd == "ruler-pack":
        tok = _tokenizer(a.tokenizer)
        out = ruler.build_pack(tok, a.dataset, a.placement, a.prompt_tokens, a.output_dir,
                               output_tokens=a.output_tokens, num_requests=a.num_requests,
                               disable_thinking=a.disable_thinking, model_name=a.served_model_name)
        _write(None, out)
        return out
    if a.cmd == "longbench-pack":
        tok = _tokenizer(a.tokenizer)
        out = longbench.build_longbench_pack(tok, a.dataset, a.dataset_name, a.output_dir, fmt=a.format,
                                             served_model_name=a.served_model_name, num_requests=a.num_requests,
                                             max_prompt_tokens=a.max_prompt_tokens, chunk_tokens=a.chunk_tokens,
                                             fixed_output_tokens=a.fixed_output_tokens,
                                             disable_thinking=a.disable_thinking, tokenizer_name=str(a.tokenizer))
        _write(None, out)
        return out
    if a.cmd == "priorities":
        tok = _tokenizer(a.tokenizer) if a.tokenizer else None
        out = priorities.build_priority_sidecars(
            a.pack_dir, a.output_dir, modes=[m for m in a.modes.split(",") if m], chunk_tokens=a.chunk_tokens,
            protected_prefix_tokens=a.protected_prefix_tokens, protected_suffix_tokens=a.protected_suffix_tokens,
            seed=a.seed, tokenizer=tok)
        _write(None, out)
        return out
    if a.cmd == "audit-packs":
        out = audits.audit_dataset_matrix(a.root, [d for d in a.datasets.split(",") if d])
        _write(a.output, out)
        return out
    if a.cmd == "audit-ruler":
        cells, failures = {}, []
        for length in _ints(a.lengths):
            for placement in [x for x in a.placements.split(",") if x]:
                key = f"{length}/{placement}"
                d = a.root / str(length) / placement
                try:
                    cell = audits.audit_pack(d, expected_dataset="ruler_qa2")
                    man = json.loads((d / "manifest.json").read_text())
                    if int(man["prompt_tokens"]) != length or man["placement"] != placement:
                        raise ValueError("manifest length / placement differ from the cell")
                    if cell["rows"] != a.requests_per_cell:
                        raise ValueError(f"{cell['rows']} rows, expected {a.requests_per_cell}")
                    if cell["max_prompt_tokens"] != length or cell["mean_prompt_tokens"] != length:
                        raise ValueError("a prompt is not of the exact cell length")
                    cells[key] = cell
                except (OSError, ValueError, KeyError) as exc:
                    failures.append(f"{key}: {exc}")
        out = {"status": "passed" if not failures else "failed", "cells": cells, "failures": failures}
        _write(a.output, out)
        return out
    if a.cmd == "priority-coverage":
        out = audits.analyze_priority_coverage(a.schedule_root, fractions=[float(x) for x in a.fractions.split(",")],
                                               selection_requests=a.selection_requests)
        _write(a.output, out)
        return out
    return cmd_quality(a)


if __name__ == "__main__":
    main()
