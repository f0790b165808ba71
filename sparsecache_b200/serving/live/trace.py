"""Fail-closed audit of the inputs a progressive request actually consumed.

Parity with the reference's experiments/verify_progressive_pd_input_trace.py:
joins the scheduler trace (seed, sparse drafts, the full-KV verification
interval) with the worker input trace (token ids and positions of every
small forward) by request id, and proves, per request, that
  * the sparse chain was exactly γ single-token forwards consuming
    [seed, d0, .., d_{γ-2}] at contiguous positions,
  * the scheduler timestamps are monotonic (start <= last draft <= full
    arrival <= verify start <= verify end), and
  * one verifier batch rewound to the seed's position and consumed
    [seed, d0, .., d_{γ-1}] at contiguous positions.
Any violation raises ``ValueError`` (:60-239).
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Any, Sequence


def publish_proposal_trace(destination: str | Path, *, method: str, proposal_started_at_ns: int,
                           seed_token_ids, draft_token_ids, methods: Sequence[str] = ("eagle3",)) -> dict | None:
    """Write one drafter proposal record atomically; the first writer wins.

    The record (state "ready", seed token, draft token ids, start and
    creation timestamps in ns) is written to a temporary file and linked into
    place with ``os.link``, which fails if the destination exists, so a later
    proposal for the same destination is dropped (returns None) and readers
    never see a partial file.  Methods outside ``methods`` publish nothing.
    Counterpart of the proposal trace the reference's EAGLE-3 screens read
    (tests/test_eagle_proposal_trace.py).
    """
    import os
    import tempfile
    import time

    if method not in methods:
        return None
    dest = Path(destination)
    if dest.exists():
        return None

    def ids(x) -> list[int]:
        return [int(v) for v in (x.reshape(-1).tolist() if hasattr(x, "reshape") else x)]

    seed = ids(seed_token_ids)
    payload = {"state": "ready", "method": method, "proposal_started_at_ns": int(proposal_started_at_ns),
               "created_at_ns": max(time.time_ns(), int(proposal_started_at_ns)),
               "seed_token_id": seed[-1] if seed else None, "draft_token_ids": ids(draft_token_ids)}
    dest.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=dest.parent, prefix=dest.name, suffix=".tmp")
    try:
        with os.fdopen(fd, "w") as f:
            json.dump(payload, f)
        try:
            os.link(tmp, dest)
        except FileExistsError:
            return None
    finally:
        os.unlink(tmp)
    return payload


def load_jsonl(path: Path) -> list[dict[str, Any]]:
    if not Path(path).is_file():
        raise FileNotFoundError(path)
    rows = []
    for n, line in enumerate(Path(path).read_text(encoding="utf-8").splitlines(), start=1):
        if line.strip():
            v = json.loads(line)
            if not isinstance(v, dict):
                raise ValueError(f"{path}:{n} is not a JSON object")
            rows.append(v)
    if not rows:
        raise ValueError(f"{path} contains no records")
    return rows


def _ints(rec: dict, key: str) -> list[int]:
    v = rec.get(key)
    if not isinstance(v, list) or any(not isinstance(x, int) or isinstance(x, bool) for x in v):
        raise ValueError(f"{key} must be a list of integers")
    return v


def _int(rec: dict, key: str) -> int:
    v = rec.get(key)
    if not isinstance(v, int) or isinstance(v, bool):
        raise ValueError(f"{key} must be an integer")
    return v


def _contiguous(v: Sequence[int]) -> bool:
    return all(b == a + 1 for a, b in zip(v, v[1:]))


def verify_input_trace(scheduler: Sequence[dict], inputs: Sequence[dict], *, expected_requests: int) -> dict:
    if expected_requests <= 0:
        raise ValueError("expected_requests must be positive")
    if len(scheduler) != expected_requests:
        raise ValueError(f"scheduler request count mismatch: {len(scheduler)} != {expected_requests}")
    by_req: dict[str, list[dict]] = {}
    for r in inputs:
        rid = r.get("request_id")
        if not isinstance(rid, str) or not rid:
            raise ValueError("input trace contains an invalid request_id")
        _int(r, "recorded_at_ns")
        n = _int(r, "num_scheduled_tokens")
        if n <= 0 or len(_ints(r, "input_token_ids")) != n or len(_ints(r, "positions")) != n:
            raise ValueError(f"input trace shape mismatch for {rid}")
        by_req.setdefault(rid, []).append(r)
    for v in by_req.values():
        v.sort(key=lambda r: r["recorded_at_ns"])
    seen, reports, n_sparse, n_verify = set(), [], 0, 0
    for s in scheduler:
        rid = s.get("request_id")
        if not isinstance(rid, str) or not rid:
            raise ValueError("scheduler trace contains an invalid request_id")
        if rid in seen:
            raise ValueError(f"duplicate scheduler request_id: {rid}")
        seen.add(rid)
        seed = _int(s, "seed_token_id")
        drafts = _ints(s, "draft_token_ids")
        g = _int(s, "draft_tokens")
        if not drafts or len(drafts) != g:
            raise ValueError(f"incomplete draft sequence for {rid}")
        if g != _int(s, "max_draft_tokens"):
            raise ValueError(f"draft did not reach its fixed horizon for {rid}")
        t = [_int(s, k) for k in ("started_at_ns", "last_draft_at_ns", "full_arrival_at_ns", "verify_started_at_ns",
                                  "verify_completed_at_ns")]
        if t != sorted(t):
            raise ValueError(f"non-monotonic scheduler timestamps for {rid}")
        recs = by_req.get(rid, [])
        sparse = [r for r in recs if t[0] <= r["recorded_at_ns"] <= t[1]]
        verify = [r for r in recs if t[3] <= r["recorded_at_ns"] <= t[4]]
        if len(sparse) != g:
            raise ValueError(f"sparse forward count mismatch for {rid}: {len(sparse)} != {g}")
        if any(len(r["input_token_ids"]) != 1 for r in sparse):
            raise ValueError(f"sparse forward was not single-token for {rid}")
        toks = [r["input_token_ids"][0] for r in sparse]
        pos = [r["positions"][0] for r in sparse]
        if toks != [seed, *drafts[:-1]]:
            raise ValueError(f"sparse chain consumed unexpected tokens for {rid}")
        if not _contiguous(pos):
            raise ValueError(f"sparse chain positions are not contiguous for {rid}")
        if len(verify) != 1:
            raise ValueError(f"expected one verifier batch for {rid}, got {len(verify)}")
        v = verify[0]
        if v["input_token_ids"] != [seed, *drafts]:
            raise ValueError(f"verifier consumed unexpected tokens for {rid}")
        if v["positions"][0] != pos[0] or not _contiguous(v["positions"]):
            raise ValueError(f"verifier did not rewind to the seed position for {rid}")
        n_sparse += len(sparse)
        n_verify += 1
        reports.append({"request_id": rid, "draft_tokens": g, "seed_position": pos[0],
                        "verify_tokens": len(v["input_token_ids"])})
    return {"status": "passed", "requests": len(reports), "sparse_forwards": n_sparse, "verify_forwards": n_verify,
            "per_request": reports}


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--scheduler-stats-jsonl", type=Path, required=True)
    p.add_argument("--input-stats-jsonl", type=Path, required=True)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--expected-requests", type=int, required=True)
    a = p.parse_args(argv)
    rep = verify_input_trace(load_jsonl(a.scheduler_stats_jsonl), load_jsonl(a.input_stats_jsonl),
                             expected_requests=a.expected_requests)
    a.output.write_text(json.dumps(rep, indent=2) + "\n", encoding="utf-8")
    print(json.dumps({k: rep[k] for k in ("status", "requests", "sparse_forwards", "verify_forwards")}))


if __name__ == "__main__":
    main()
