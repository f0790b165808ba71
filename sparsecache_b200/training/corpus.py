"""Drafter-training corpus: length-stratified, task-interleaved request selection.

Parity with the reference's experiments/build_sparse_kv_draft_corpus.py:
per dataset pack, ``samples_per_dataset`` requests are taken at evenly spaced
ranks of the prompt-length order (:33-53); the corpus interleaves datasets
round-robin by length stratum, records each row's source, and writes
``requests.jsonl``, ``metadata.jsonl`` and a manifest
(``sparsecache.sparse-kv-draft-corpus.v1``) with the source hashes (:55-115).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import time
from pathlib import Path
from typing import Any, Sequence

CORPUS_FORMAT = "sparsecache.sparse-kv-draft-corpus.v1"


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def load_jsonl(path: Path) -> list[dict[str, Any]]:
    rows = []
    for n, line in enumerate(Path(path).read_text(encoding="utf-8").splitlines(), start=1):
        if line.strip():
            row = json.loads(line)
            if not isinstance(row, dict):
                raise ValueError(f"{path}:{n} is not an object")
            rows.append(row)
    return rows


def length_stratified_indices(requests: Sequence[dict], count: int) -> list[int]:
    """Indices at the centres of ``count`` equal strata of the prompt-length order."""
    if count <= 0 or count > len(requests):
        raise ValueError("sample count is outside the request range")
    ranked = sorted(range(len(requests)), key=lambda i: (len(requests[i]["prompt"]), i))
    out = [ranked[min(len(ranked) - 1, int((k + 0.5) * len(ranked) / count))] for k in range(count)]
    if len(out) != len(set(out)):
        raise RuntimeError("stratified selection produced duplicate indices")
    return out


def build_corpus(pack_root: Path, datasets: Sequence[str], samples_per_dataset: int):
    if not datasets or len(datasets) != len(set(datasets)):
        raise ValueError("datasets must be non-empty and unique")
    chosen, sources = {}, {}
    for ds in datasets:
        d = Path(pack_root) / ds
        reqs, meta = load_jsonl(d / "requests.jsonl"), load_jsonl(d / "metadata.jsonl")
        if len(reqs) != len(meta):
            raise ValueError(f"{ds} request and metadata counts differ")
        man = json.loads((d / "manifest.json").read_text(encoding="utf-8"))
        if man.get("dataset") != ds:
            raise ValueError(f"{ds} manifest identity differs")
        idx = length_stratified_indices(reqs, samples_per_dataset)
        chosen[ds] = [(i, reqs[i], meta[i]) for i in idx]
        sources[ds] = {"manifest": str((d / "manifest.json").resolve()),
                       "requests_sha256": sha256_file(d / "requests.jsonl"),
                       "metadata_sha256": sha256_file(d / "metadata.jsonl"), "selected_source_indices": idx}
    requests, metadata = [], []
    for rank in range(samples_per_dataset):
        for ds in datasets:
            src, req, meta = chosen[ds][rank]
            requests.append({**req, "source_dataset": ds, "source_index": src})
            metadata.append({**meta, "corpus_index": len(metadata), "source_dataset": ds, "source_index": src})
    manifest = {"schema_version": 1, "format": CORPUS_FORMAT, "created_at_ns": time.time_ns(),
                "pack_root": str(Path(pack_root).resolve()), "datasets": list(datasets),
                "samples_per_dataset": samples_per_dataset, "requests": len(requests),
                "interleave": "round_robin_by_length_stratum", "source_manifests": sources}
    return requests, metadata, manifest


def write_corpus(out_dir: Path, requests, metadata, manifest) -> None:
    out_dir = Path(out_dir)
    if out_dir.exists():
        raise FileExistsError(f"refusing to overwrite {out_dir}")
    out_dir.mkdir(parents=True)
    for name, rows in (("requests.jsonl", requests), ("metadata.jsonl", metadata)):
        with open(out_dir / name, "w", encoding="utf-8") as f:
            for r in rows:
                f.write(json.dumps(r, separators=(",", ":")) + "\n")
    manifest = {**manifest, "requests_sha256": sha256_file(out_dir / "requests.jsonl"),
                "metadata_sha256": sha256_file(out_dir / "metadata.jsonl")}
    (out_dir / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n")


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--pack-root", required=True, type=Path)
    p.add_argument("--output-dir", required=True, type=Path)
    p.add_argument("--datasets", default="qmsum,musique,qasper,multi_news,hotpotqa,narrativeqa")
    p.add_argument("--samples-per-dataset", type=int, default=100)
    a = p.parse_args(argv)
    reqs, meta, man = build_corpus(a.pack_root, tuple(x for x in a.datasets.split(",") if x), a.samples_per_dataset)
    write_corpus(a.output_dir, reqs, meta, man)
    print(json.dumps({"requests": len(reqs), "datasets": man["datasets"]}))


if __name__ == "__main__":
    main()
