"""Preregistered live-job queues (selection and confirmation splits).

Parity with the reference's queue builders (experiments/build_progressive_pd_live_queue.py:108-450 and its
siblings for scheduling and crossover jobs): a queue is a JSON document of
jobs, each pinning the pack it reads by sha256 (requests and metadata), the
request window (offset, count: core/selection requests first, confirmation
requests after them, never overlapping), warm-ups, arms, the controlled link
bandwidth, the draft horizon, the fixed output horizon and the protected
anchor sizes.  Confirmation jobs start blocked until the core gate passes
and the method is frozen.  The queue itself carries a sha256 over its jobs.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Any, Sequence

ARMS = ("baseline", "fixed_s1", "continuous")


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def canonical_sha256(obj: Any) -> str:
    return hashlib.sha256(json.dumps(obj, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def build_job(*, job_id: str, phase: str, status: str, pack_dir: Path, run_dir: Path, requests: int,
              request_offset: int, warmups: int, bandwidth_gbps: int, arms: Sequence[str] = ARMS,
              fixed_output_tokens: int = 32, max_draft_tokens: int = 8, model: dict | None = None,
              protected_prefix_tokens: int = 256, protected_suffix_tokens: int = 512,
              priority_jsonl: Path | None = None) -> dict[str, Any]:
    pack_dir = Path(pack_dir)
    rq, md = pack_dir / "requests.jsonl", pack_dir / "metadata.jsonl"
    n_rows = sum(1 for line in rq.read_text().splitlines() if line.strip())
    if request_offset + requests > n_rows:
        raise ValueError(f"{job_id}: window [{request_offset}, {request_offset + requests}) exceeds {n_rows} rows")
    job = {"job_id": job_id, "phase": phase, "status": status, "pack_dir": str(pack_dir), "run_dir": str(run_dir),
           "requests_jsonl": str(rq), "requests_sha256": sha256_file(rq), "metadata_jsonl": str(md),
           "metadata_sha256": sha256_file(md), "requests": requests, "request_offset": request_offset,
           "warmup_requests": warmups, "arms": list(arms), "bandwidth_gbps": bandwidth_gbps,
           "fixed_output_tokens": fixed_output_tokens, "max_draft_tokens": max_draft_tokens,
           "protected_prefix_tokens": protected_prefix_tokens, "protected_suffix_tokens": protected_suffix_tokens,
           "model": model or {}}
    if priority_jsonl is not None:
        job["priority_jsonl"] = str(priority_jsonl)
        job["priority_sha256"] = sha256_file(Path(priority_jsonl))
    return job


def build_queue(packs: Sequence[dict], run_root: Path, *, bandwidths: Sequence[int], core_requests: int,
                confirmation_requests: int, warmup_requests: int, max_draft_tokens: int,
                model: dict | None = None) -> dict[str, Any]:
    """``packs``: [{"name", "pack_dir", "core": bool}] -> queue with core and confirmation jobs."""
    if not bandwidths or len(set(bandwidths)) != len(bandwidths) or any(b <= 0 for b in bandwidths):
        raise ValueError("bandwidths must be a non-empty unique list of positive values")
    if min(core_requests, confirmation_requests, max_draft_tokens) <= 0 or warmup_requests < 0:
        raise ValueError("request and draft counts must be positive")
    jobs = []
    for pack in packs:
        for bw in bandwidths:
            if pack.get("core", True):
                jid = f"core_{pack['name']}_bw{bw}_n{core_requests}"
                jobs.append(build_job(job_id=jid, phase="core_mechanism", status="ready_when_gpus_are_exclusive",
                                      pack_dir=Path(pack["pack_dir"]), run_dir=Path(run_root) / jid,
                                      requests=core_requests, request_offset=0, warmups=warmup_requests,
                                      bandwidth_gbps=bw, max_draft_tokens=max_draft_tokens, model=model))
            jid = f"confirm_{pack['name']}_bw{bw}_n{confirmation_requests}_offset{core_requests}"
            jobs.append(build_job(job_id=jid, phase="controlled_confirmation",
                                  status="blocked_on_core_gate_and_method_freeze", pack_dir=Path(pack["pack_dir"]),
                                  run_dir=Path(run_root) / jid, requests=confirmation_requests,
                                  request_offset=core_requests, warmups=warmup_requests, bandwidth_gbps=bw,
                                  max_draft_tokens=max_draft_tokens, model=model))
    ids = [j["job_id"] for j in jobs]
    if len(ids) != len(set(ids)):
        raise ValueError("duplicate job ids")
    return {"format": "sparsecache.live-job-queue.v1", "jobs": jobs, "jobs_sha256": canonical_sha256(jobs)}


def load_job(queue_path: Path, job_id: str) -> tuple[dict, str]:
    queue = json.loads(Path(queue_path).read_text())
    if canonical_sha256(queue["jobs"]) != queue.get("jobs_sha256"):
        raise ValueError("queue jobs were edited after registration")
    for job in queue["jobs"]:
        if job["job_id"] == job_id:
            return job, queue["jobs_sha256"]
    raise KeyError(job_id)


def validate_pack_hashes(job: dict) -> dict[str, str]:
    """Refuse a job whose pack files changed since the queue was built."""
    got = {"requests": sha256_file(Path(job["requests_jsonl"])), "metadata": sha256_file(Path(job["metadata_jsonl"]))}
    if got["requests"] != job["requests_sha256"] or got["metadata"] != job["metadata_sha256"]:
        raise ValueError(f"pack hashes of {job['job_id']} differ from the registered queue")
    if "priority_jsonl" in job and sha256_file(Path(job["priority_jsonl"])) != job["priority_sha256"]:
        raise ValueError(f"priority sidecar of {job['job_id']} differs from the registered queue")
    return got


def main(argv=None) -> int:
    """Build a preregistered live-job queue from a packs JSON (``[{"name", "pack_dir", "core"}]``)."""
    import argparse

    p = argparse.ArgumentParser()
    p.add_argument("--packs", type=Path, required=True)
    p.add_argument("--run-root", type=Path, required=True)
    p.add_argument("--bandwidths", default="25,50")
    p.add_argument("--core-requests", type=int, default=64)
    p.add_argument("--confirmation-requests", type=int, default=192)
    p.add_argument("--warmup-requests", type=int, default=2)
    p.add_argument("--max-draft-tokens", type=int, default=8)
    p.add_argument("--output", type=Path, required=True)
    a = p.parse_args(argv)
    queue = build_queue(json.loads(a.packs.read_text()), a.run_root,
                        bandwidths=[int(x) for x in a.bandwidths.split(",")], core_requests=a.core_requests,
                        confirmation_requests=a.confirmation_requests, warmup_requests=a.warmup_requests,
                        max_draft_tokens=a.max_draft_tokens)
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(queue, indent=2) + "\n")
    print(json.dumps({"jobs": len(queue["jobs"]), "jobs_sha256": queue["jobs_sha256"]}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
