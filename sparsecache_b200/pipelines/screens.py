"""Compute-only draft screens on the engine: layer-sparse / layer-subset drafts and the
sparse-page draft crossover.

Counterparts of the reference's vLLM compute screens
(experiments/benchmark_layer_sparse_draft.py, benchmark_layer_subset_draft.py,
benchmark_sparse_draft_crossover.py, benchmark_eagle3_draft.py): instead of out-of-tree vLLM
backends, the drafts run on this package's engine.
  * ``layer_draft_screen``: greedy drafts computed with a subset of the target's layers (the
    first N, or a frozen pattern; skipped layers are identity) against the full model's greedy
    continuation: accepted prefix and per-token draft time (CUDA graph per subset).
  * layer patterns: uniform and sandwich subsets (``standard_patterns``) or a
    schema-1 pattern file (configs/layer_subset_patterns_*.json, the layout
    of the reference's configs/layer_subset_patterns_llama32.json);
  * ``sparse_page_crossover``: per-token cost of a draft step whose attention reads a page view
    (64 sink + 512 recent + evenly spaced 64-token pages up to the visible fraction) against a
    full-context step, over fractions and context lengths: where sparse drafting stops paying.
    The draft step sizes its attention split for the view's keys (``verify(..., sparse=True)``);
    each row also times the same view with the split sized for the whole cache (the verifier's
    geometry), which shows what that sizing is worth.
The EAGLE drafter's screen is ``training.drafter_trainer.evaluate_drafter``.
"""
from __future__ import annotations

import json
from typing import Any, Sequence

import torch

from ..models.sparse_kv_draft import accepted_prefix_length, sink_recent_topk_indices


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


@torch.inference_mode()
def layer_draft_screen(engine, prompt: Sequence[int], patterns: dict[str, Sequence[int]], *,
                       draft_tokens: int = 8) -> list[dict[str, Any]]:
    dev = engine.device
    T = len(prompt)
    slot = engine.new_slot(T + draft_tokens + 64)
    ids = torch.tensor(list(prompt), dtype=torch.int32, device=dev)
    h = engine.prefill(ids, slot)
    last = h[T - 1:T].clone()

    def run(layers):
        engine.first_token(last, position=T, max_new=draft_tokens)
        engine.decode(slot, 1, max_new=draft_tokens, layers=layers)  # capture / warm
        engine.first_token(last, position=T, max_new=draft_tokens)
        a, b = _events()
        a.record()
        engine.decode(slot, draft_tokens - 1, max_new=draft_tokens, layers=layers)
        b.record()
        b.synchronize()
        return engine.generated_tokens(draft_tokens).tolist(), a.elapsed_time(b) / max(1, draft_tokens - 1)

    ref, full_ms = run(None)
    out = [{"pattern": "full", "layers": engine.cfg.n_layers, "accepted_prefix": draft_tokens - 1,
            "ms_per_token": full_ms, "relative_cost": 1.0}]
    for name, layers in patterns.items():
        toks, ms = run(tuple(int(x) for x in layers))
        out.append({"pattern": name, "layers": len(layers),
                    "accepted_prefix": accepted_prefix_length(toks[1:], ref[1:]), "ms_per_token": ms,
                    "relative_cost": ms / full_ms})
    return out


def uniform_layers(n_layers: int, k: int) -> list[int]:
    """k layer indices spread evenly over [0, n_layers - 1] (both ends included)."""
    if not 1 <= k <= n_layers:
        raise ValueError("pattern size outside the model")
    if k == 1:
        return [0]
    return sorted({int(i * (n_layers - 1) / (k - 1) + 0.5) for i in range(k)})


def sandwich_layers(n_layers: int, k: int) -> list[int]:
    """The first k/2 and the last k/2 layers."""
    if k % 2 or not 2 <= k <= n_layers:
        raise ValueError("sandwich patterns take an even size within the model")
    return list(range(k // 2)) + list(range(n_layers - k // 2, n_layers))


def standard_patterns(n_layers: int, sizes=(8, 16, 24)) -> dict:
    """Pattern file content (schema 1): uniform and sandwich subsets of each size."""
    pats = []
    for k in sizes:
        if k >= n_layers:
            continue
        pats.append({"id": f"uniform{k}", "layer_indices": uniform_layers(n_layers, k),
                     "description": f"{k} layers spread evenly over the network"})
        pats.append({"id": f"sandwich{k}", "layer_indices": sandwich_layers(n_layers, k),
                     "description": f"first {k // 2} and last {k // 2} layers"})
    return {"schema_version": 1, "n_layers": n_layers, "patterns": pats}


def load_patterns(path, n_layers: int) -> dict[str, list[int]]:
    """{id: layer indices} of a schema-1 pattern file; indices are checked against the model."""
    data = json.loads(open(path).read())
    if data.get("schema_version") != 1:
        raise ValueError("unsupported layer-pattern schema")
    out = {}
    for p in data["patterns"]:
        idx = [int(i) for i in p["layer_indices"]]
        if idx != sorted(set(idx)) or not idx or idx[0] < 0 or idx[-1] >= n_layers:
            raise ValueError(f"pattern {p['id']}: indices must be sorted, unique and inside the model")
        out[p["id"]] = idx
    return out


def page_view(T: int, fraction: float, *, page: int = 64, sink: int = 64, recent: int = 512) -> torch.Tensor:
    """Sorted visible token indices of a sink + recent + evenly spaced pages view."""
    budget = max(sink + recent, int(T * fraction))
    return sink_recent_topk_indices(T, None, sink=sink, recent=recent, chunk=page, budget=budget)


@torch.inference_mode()
def sparse_page_crossover(engine, context_lengths: Sequence[int], fractions: Sequence[float], *,
                          reps: int = 20, seed: int = 0) -> list[dict[str, Any]]:
    dev = engine.device
    g = torch.Generator().manual_seed(seed)
    rows = []
    for T in context_lengths:
        slot = engine.new_slot(T + 64)
        ids = torch.randint(0, engine.cfg.vocab, (T,), generator=g, dtype=torch.int32).to(dev)
        engine.prefill(ids, slot)
        tok = torch.tensor([1], dtype=torch.int32)
        view = torch.zeros(slot.capacity, dtype=torch.int32, device=dev)

        def step(n_vis=None, sparse=False):
            if n_vis is None:
                engine.verify(slot, tok, position=T)
            else:
                engine.verify(slot, tok, position=T, slot_start=T, view=view, n_visible=n_vis, sparse=sparse)

        def timed(fn):
            for _ in range(3):
                fn()
            a, b = _events()
            a.record()
            for _ in range(reps):
                fn()
            b.record()
            b.synchronize()
            return a.elapsed_time(b) / reps

        full_ms = timed(step)
        for f in fractions:
            idx = page_view(T, f)
            view[: idx.numel()].copy_(idx.to(torch.int32))
            view[idx.numel()] = T  # the draft row's own slot follows the visible keys
            ms = timed(lambda: step(idx.numel(), sparse=True))
            # the same view with the attention split sized for the whole cache (the verifier's geometry)
            ms_cap = timed(lambda: step(idx.numel()))
            rows.append({"context_tokens": T, "visible_fraction": idx.numel() / T, "requested_fraction": f,
                         "draft_step_ms": ms, "draft_step_capacity_split_ms": ms_cap, "full_step_ms": full_ms,
                         "speedup": full_ms / ms})
    return rows


def parse_fractions(text: str) -> tuple[float, ...]:
    """Comma-separated visible fractions in (0, 1]; the full view (1.0) must be among them."""
    vals = tuple(float(x) for x in text.split(",") if x.strip())
    if not vals or any(not 0.0 < v <= 1.0 for v in vals) or len(set(vals)) != len(vals):
        raise ValueError("fractions must be unique values in (0, 1]")
    if 1.0 not in vals:
        raise ValueError("the fractions must include the full view 1.0 (the paired reference)")
    return vals


def balanced_fraction_schedule(fractions: Sequence[float], repeats: int) -> list[tuple[int, int, float]]:
    """(repeat, order index, fraction): every repeat measures every fraction once, the order
    rotated by one position per repeat so no fraction always runs first (warm-state bias)."""
    n = len(fractions)
    return [(r, i, fractions[(i + r) % n]) for r in range(repeats) for i in range(n)]


def measurement_seed_token(vocab: int, repeat: int) -> int:
    """A fixed ordinary-text seed token per repeat (clear of the low special ids)."""
    return (1024 + repeat) % vocab


def aggregate_crossover(rows: Sequence[dict]) -> dict[str, Any]:
    """Per context length: draft-step time per visible fraction, speedup over the full view
    paired by repeat, and the crossover (the largest fraction still faster than full).

    Fails closed: every repeat must have measured every fraction of the context.
    """
    import statistics

    out = {}
    for T in sorted({r["context_tokens"] for r in rows}):
        sub = [r for r in rows if r["context_tokens"] == T]
        fracs = sorted({r["requested_fraction"] for r in sub})
        reps = sorted({r.get("repeat", 0) for r in sub})
        cell = {(r.get("repeat", 0), r["requested_fraction"]): r for r in sub}
        missing = [(rp, f) for rp in reps for f in fracs if (rp, f) not in cell]
        if missing:
            raise ValueError(f"context {T}: incomplete fraction x repeat matrix, missing {missing[:4]}")
        if 1.0 not in fracs:
            raise ValueError(f"context {T}: no full-view reference")
        per = {}
        for f in fracs:
            ms = [cell[(rp, f)]["draft_step_ms"] for rp in reps]
            sp = [cell[(rp, 1.0)]["draft_step_ms"] / cell[(rp, f)]["draft_step_ms"] for rp in reps]
            per[str(f)] = {"draft_step_ms_mean": statistics.fmean(ms), "speedup_vs_full_mean": statistics.fmean(sp),
                           "speedup_vs_full_min": min(sp),
                           "visible_fraction": statistics.fmean(cell[(rp, f)]["visible_fraction"] for rp in reps)}
        faster = [f for f in fracs if f < 1.0 and per[str(f)]["speedup_vs_full_min"] > 1.0]
        out[str(T)] = {"repeats": len(reps), "fractions": per,
                       "crossover_fraction": max(faster) if faster else None}
    return out


def main(argv=None) -> None:
    import argparse

    from ..config import get_model_config
    from ..models.engine import B200Engine

    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--prompt-tokens", type=int, default=4096)
    p.add_argument("--draft-tokens", type=int, default=8)
    p.add_argument("--contexts", default="8192,32768")
    p.add_argument("--fractions", default="0.05,0.1,0.2,0.5")
    p.add_argument("--patterns", default=None, help="schema-1 layer-pattern JSON (default: generated)")
    p.add_argument("--repeats", type=int, default=3, help="crossover repeats, fraction order rotated per repeat")
    a = p.parse_args(argv)
    cfg = get_model_config(a.model)
    ctxs = [int(x) for x in a.contexts.split(",")]
    eng = B200Engine.random(cfg, seed=0, device="cuda", max_positions=max(ctxs + [a.prompt_tokens]) + 256)
    L = cfg.n_layers
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab, (a.prompt_tokens,), generator=g).tolist()
    patterns = {f"first_{n}": list(range(n)) for n in (L // 4, L // 2, 3 * L // 4)}
    patterns["every_other"] = list(range(0, L, 2))
    if a.patterns:
        patterns.update(load_patterns(a.patterns, L))
    else:
        patterns.update({p["id"]: p["layer_indices"] for p in standard_patterns(L)["patterns"]})
    vals = [float(x) for x in a.fractions.split(",") if x.strip()]
    fractions = list(parse_fractions(",".join(map(str, vals + ([] if 1.0 in vals else [1.0])))))
    cross = []
    for T in ctxs:
        for rep in range(a.repeats):
            order = [f for r, _, f in balanced_fraction_schedule(fractions, a.repeats) if r == rep]
            for i, row in enumerate(sparse_page_crossover(eng, [T], order, seed=rep)):
                row.update(repeat=rep, order_index=i)
                cross.append(row)
    print(json.dumps({"layer_draft": layer_draft_screen(eng, prompt, patterns, draft_tokens=a.draft_tokens),
                      "sparse_page_crossover": cross, "crossover_summary": aggregate_crossover(cross)}, indent=1))


if __name__ == "__main__":
    main()


# --------------------------------------------------------------------------
# Frozen crossover jobs (reference: experiments/build_sparse_draft_crossover_queue.py,
# experiments/run_sparse_draft_crossover_job.py): a queue pins each job's exact
# command, the queue carries a sha256 over its jobs, and the runner refuses a
# job that is not "ready", an edited queue, or GPUs that are not exclusive,
# then runs the frozen command and writes a run record next to its output.
# --------------------------------------------------------------------------
CROSSOVER_QUEUE_FORMAT = "sparsecache.crossover-job-queue.v1"


def build_crossover_queue(*, model: str, contexts: Sequence[int], fractions: Sequence[float], run_root: str,
                          prompt_tokens: int = 4096, draft_tokens: int = 8, patterns: str | None = None) -> dict:
    from ..serving.live.queue import canonical_sha256

    jobs = []
    for T in contexts:
        job_id = f"crossover_{model}_ctx{T}"
        out_dir = f"{run_root}/{job_id}"
        cmd = ["python", "-m", "sparsecache_b200.pipelines.screens", "--model", model, "--contexts", str(T),
               "--fractions", ",".join(str(f) for f in fractions), "--prompt-tokens", str(prompt_tokens),
               "--draft-tokens", str(draft_tokens)]
        if patterns:
            cmd += ["--patterns", patterns]
        jobs.append({"id": job_id, "status": "ready", "command": cmd, "output_dir": out_dir,
                     "context_tokens": T, "fractions": list(fractions)})
    if len({j["id"] for j in jobs}) != len(jobs):
        raise ValueError("duplicate job ids")
    return {"format": CROSSOVER_QUEUE_FORMAT, "jobs": jobs, "jobs_sha256": canonical_sha256(jobs)}


def run_crossover_job(queue_path, job_id: str, *, gpus: Sequence[int] = (0,), gate=None, runner=None,
                      max_used_memory_mib: float = 1024.0) -> dict:
    """Run one frozen job fail-closed; returns (and writes) its run record."""
    import hashlib
    import subprocess
    import time
    from pathlib import Path

    from ..serving.live.queue import canonical_sha256

    queue_path = Path(queue_path)
    raw = queue_path.read_bytes()
    queue = json.loads(raw)
    if queue.get("format") != CROSSOVER_QUEUE_FORMAT:
        raise ValueError("not a crossover job queue")
    if canonical_sha256(queue["jobs"]) != queue.get("jobs_sha256"):
        raise ValueError("queue jobs were edited after registration")
    matches = [j for j in queue["jobs"] if j["id"] == job_id]
    if len(matches) != 1:
        raise ValueError(f"expected exactly one job named {job_id!r}")
    job = matches[0]
    if job["status"] != "ready":
        raise ValueError(f"job is not executable: {job['status']!r}")
    if gate is None:
        from ..serving.live.gate import evaluate_exclusivity, inspect_gpus

        def gate():
            v = evaluate_exclusivity(inspect_gpus(), list(gpus), max_used_memory_mib=max_used_memory_mib,
                                     max_utilization_pct=5.0)
            return {**v, "passed": v["status"] == "passed"}
    verdict = gate()
    if not verdict.get("passed", False):
        raise RuntimeError(f"GPUs are not exclusive: {verdict}")
    out_dir = Path(job["output_dir"])
    out_dir.mkdir(parents=True, exist_ok=True)
    result_path = out_dir / "result.json"
    t0 = time.time()
    if runner is None:
        with open(result_path, "w") as f:
            rc = subprocess.run(job["command"], stdout=f, check=False).returncode
    else:
        rc = runner(job["command"], result_path)
    record = {"job_id": job_id, "queue_sha256": hashlib.sha256(raw).hexdigest(),
              "jobs_sha256": queue["jobs_sha256"], "command": job["command"], "exit_code": int(rc),
              "wall_s": time.time() - t0, "gate": verdict, "result": str(result_path)}
    (out_dir / "run_record.json").write_text(json.dumps(record, indent=2) + "\n")
    if rc != 0:
        raise RuntimeError(f"{job_id} exited with {rc}")
    return record
