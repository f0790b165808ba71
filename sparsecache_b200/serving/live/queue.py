"""Preregistered live-job queues (selection and confirmation splits).

Parity with the reference's queue builders (experiments/build_progressive_pd_live_queue.py:108-450 and its
siblings for scheduling and crossover jobs): a queue is a JSON document of
jobs, each pinning the pack it reads by sha256 (requests and metadata), the
request window (offset, count: core/selection requests first, confirmation
requests after them, never overlapping), warm-ups, arms, the controlled link
bandwidth, the draft horizon, the fixed output horizon and the protected
anchor sizes.  Confirmation jobs start blocked until the core gate passes
and the method is frozen.  The queue itself carries a sha256 over its jobs.
``build_scheduling_queue`` (experiments/build_progressive_pd_scheduling_queue.py)
adds the paired scheduling jobs, each pinning all five priority sidecars.
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


SCHEDULING_MODES = ("sequential", "uniform", "random", "bm25", "oracle")
SCHEDULING_ARMS = ("fixed_s1", "continuous")


def fraction_schedule(tranche_fraction: float) -> list[float]:
    """Cumulative arrival fractions of equal tranches; the fraction must split (0, 1] evenly."""
    steps = round(1.0 / tranche_fraction)
    if not 0.0 < tranche_fraction < 1.0 or steps < 2 or abs(tranche_fraction * steps - 1.0) > 1e-9:
        raise ValueError("the tranche fraction must split (0, 1] into equal steps")
    return [k / steps for k in range(1, steps + 1)]


def build_scheduling_queue(pack_dir: Path, schedule_dir: Path, run_root: Path, *, bandwidths: Sequence[int],
                           selection_requests: int, confirmation_requests: int, warmup_requests: int,
                           max_draft_tokens: int, start_fraction: float = 0.05, tranche_fraction: float = 0.05,
                           modes: Sequence[str] = SCHEDULING_MODES, model: dict | None = None,
                           protected_prefix_tokens: int = 256, protected_suffix_tokens: int = 512) -> dict[str, Any]:
    """Paired scheduling jobs: every priority mode x {fixed_s1, continuous} on one shared prefill per request.

    Reference: experiments/build_progressive_pd_scheduling_queue.py.  The
    sidecar audit of ``schedule_dir`` must have passed with exactly ``modes``
    over as many requests as the pack holds; selection rows come first,
    confirmation rows after them (blocked until the selection freeze).  Each
    job pins every sidecar by sha256 next to the pack hashes.
    """
    if not bandwidths or len(set(bandwidths)) != len(bandwidths) or any(b <= 0 for b in bandwidths):
        raise ValueError("bandwidths must be a non-empty unique list of positive values")
    if min(selection_requests, confirmation_requests, max_draft_tokens) <= 0 or warmup_requests < 0:
        raise ValueError("request and draft counts must be positive")
    fractions = fraction_schedule(tranche_fraction)
    ratio = start_fraction / tranche_fraction
    if not 0.0 < start_fraction < 1.0 or abs(ratio - round(ratio)) > 1e-9:
        raise ValueError("the start fraction must be a whole number of tranches")
    schedule_dir = Path(schedule_dir)
    audit = json.loads((schedule_dir / "audit.json").read_text())
    if audit.get("status") != "passed" or tuple(audit.get("modes", ())) != tuple(modes):
        raise ValueError("the scheduling audit must pass with exactly the requested modes")
    if selection_requests + confirmation_requests > int(audit["requests"]):
        raise ValueError("selection and confirmation rows exceed the pack")
    manifest = json.loads((Path(pack_dir) / "manifest.json").read_text())
    if int(manifest["requests"]) != int(audit["requests"]):
        raise ValueError("schedule and pack request counts differ")
    sidecars = {m: schedule_dir / f"priority_{m}.jsonl" for m in modes}
    missing = [str(p) for p in sidecars.values() if not p.is_file()]
    if missing:
        raise FileNotFoundError(f"missing priority sidecars: {missing}")
    pinned = {m: {"path": str(p), "sha256": sha256_file(p)} for m, p in sidecars.items()}
    for m, pin in pinned.items():
        if audit.get("priority_sha256", {}).get(m) not in (None, pin["sha256"]):
            raise ValueError(f"sidecar {m} differs from its audit")
    suffix = "" if abs(tranche_fraction - 0.05) < 1e-12 else f"_tranche{round(tranche_fraction * 10_000)}bp"
    jobs = []
    for phase, status, n, offset in (("scheduling_selection", "ready_when_gpus_are_exclusive", selection_requests, 0),
                                     ("scheduling_confirmation", "blocked_on_scheduling_selection_freeze",
                                      confirmation_requests, selection_requests)):
        for bw in bandwidths:
            jid = f"{phase}_bw{bw}_n{n}_offset{offset}{suffix}"
            job = build_job(job_id=jid, phase=phase, status=status, pack_dir=Path(pack_dir),
                            run_dir=Path(run_root) / jid, requests=n, request_offset=offset, warmups=warmup_requests,
                            bandwidth_gbps=bw, arms=SCHEDULING_ARMS, max_draft_tokens=max_draft_tokens, model=model,
                            protected_prefix_tokens=protected_prefix_tokens,
                            protected_suffix_tokens=protected_suffix_tokens)
            job.update(schedule_modes=list(modes), priority_sidecars=pinned, start_fraction=start_fraction,
                       retrieve_fractions=fractions, chunk_tokens=int(audit["chunk_tokens"]),
                       schedule_audit_sha256=sha256_file(schedule_dir / "audit.json"))
            jobs.append(job)
    return {"format": "sparsecache.live-scheduling-queue.v1", "jobs": jobs, "jobs_sha256": canonical_sha256(jobs)}


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
    for mode, pin in job.get("priority_sidecars", {}).items():
        if sha256_file(Path(pin["path"])) != pin["sha256"]:
            raise ValueError(f"{mode} priority sidecar of {job['job_id']} differs from the registered queue")
    return got


def scheduling_main(argv=None) -> int:
    import argparse

    p = argparse.ArgumentParser(prog="queue scheduling")
    p.add_argument("--pack-dir", type=Path, required=True)
    p.add_argument("--schedule-dir", type=Path, required=True)
    p.add_argument("--run-root", type=Path, required=True)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--bandwidths", default="25,50")
    p.add_argument("--selection-requests", type=int, default=100)
    p.add_argument("--confirmation-requests", type=int, default=100)
    p.add_argument("--warmup-requests", type=int, default=4)
    p.add_argument("--max-draft-tokens", type=int, default=8)
    p.add_argument("--start-fraction", type=float, default=0.05)
    p.add_argument("--tranche-fraction", type=float, default=0.05)
    a = p.parse_args(argv)
    queue = build_scheduling_queue(a.pack_dir, a.schedule_dir, a.run_root,
                                   bandwidths=[int(x) for x in a.bandwidths.split(",")],
                                   selection_requests=a.selection_requests,
                                   confirmation_requests=a.confirmation_requests,
                                   warmup_requests=a.warmup_requests, max_draft_tokens=a.max_draft_tokens,
                                   start_fraction=a.start_fraction, tranche_fraction=a.tranche_fraction)
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(queue, indent=2) + "\n")
    print(json.dumps({"jobs": len(queue["jobs"]), "jobs_sha256": queue["jobs_sha256"]}))
    return 0


def main(argv=None) -> int:
    """Build a preregistered live-job queue from a packs JSON (``[{"name", "pack_dir", "core"}]``);
    ``scheduling ...`` builds the paired scheduling queue instead."""
    import argparse
    import sys

    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "scheduling":
        return scheduling_main(argv[1:])
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
