"""When does a producer-side EAGLE proposal become transferable (token-only P/D handoff)?

    python -m sparsecache_b200.pipelines.pd_source --model llama3-8b --workload pd_long --requests 32 \\
        --horizon 4 --bandwidths 25,50,100 --output-dir runs/pd_source

Counterpart of the reference's experiments/benchmark_eagle3_pd_source.py
(worker :131-251, aggregation :253-362), on this package's engine instead of
vLLM.  For every request, on the prefill GPU:

  * dense arm: prefill + LM head of the prompt, timed with CUDA events up to
    the first exact token (the seed);
  * EAGLE arm: the same prefill with feature hooks on the seed layers, the
    seed, then ``horizon`` greedy proposals of the sparse-KV EAGLE drafter
    reading a sink + recent + evenly spaced chunk view of the prompt's K/V at
    its memory layers, timed up to the proposal tokens on the device.

The proposal is audited against the target's own greedy continuation (its
accepted prefix).  ``aggregate_source`` pairs the arms by request and, for
each link rate, compares the extra source time of the proposal with the
transfer window of the whole prompt's K/V: the proposal is useful to a
decode side that receives tokens first when it is ready before the K/V.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import random
import statistics
from pathlib import Path
from typing import Any, Sequence

import torch

from .pd import parse_bandwidths, transfer_ms


def describe(values: Sequence[float]) -> dict[str, Any] | None:
    x = sorted(float(v) for v in values)
    if not x:
        return None
    q = lambda p: x[min(len(x) - 1, int(p * len(x)))]  # noqa: E731
    return {"n": len(x), "mean": statistics.fmean(x), "p50": q(0.5), "p90": q(0.9), "p99": q(0.99),
            "min": x[0], "max": x[-1]}


def bootstrap_mean_ci(values: Sequence[float], *, samples: int = 10000, seed: int = 0):
    if not values:
        return None
    rng = random.Random(seed)
    n = len(values)
    est = sorted(sum(values[rng.randrange(n)] for _ in range(n)) / n for _ in range(samples))
    return [est[int(0.025 * samples)], est[min(samples - 1, int(0.975 * samples))]]


def prompt_sha256(prompt: Sequence[int]) -> str:
    return hashlib.sha256(json.dumps([int(t) for t in prompt], separators=(",", ":")).encode()).hexdigest()


def accepted_prefix(proposal: Sequence[int], target: Sequence[int]) -> int:
    n = 0
    for a, b in zip(proposal, target):
        if a != b:
            break
        n += 1
    return n


def aggregate_source(dense: Sequence[dict], eagle: Sequence[dict], *, bandwidths: Sequence[float],
                     kv_bytes_per_token: int, bootstrap_samples: int = 10000, seed: int = 0) -> dict[str, Any]:
    """Pair the arms by request and model the proposal's lead over the K/V transfer per link rate."""
    d_by = {int(r["request_index"]): r for r in dense}
    e_by = {int(r["request_index"]): r for r in eagle}
    if len(d_by) != len(dense) or len(e_by) != len(eagle):
        raise ValueError("duplicate request indices in an arm")
    if set(d_by) != set(e_by):
        raise ValueError("the dense and EAGLE arms cover different requests")
    paired = []
    for i in sorted(d_by):
        d, e = d_by[i], e_by[i]
        if d["prompt_sha256"] != e["prompt_sha256"]:
            raise ValueError(f"request {i}: paired prompt hashes differ")
        paired.append({"request_index": i, "prompt_tokens": int(e["prompt_tokens"]),
                       "dense_seed_ready_ms": float(d["elapsed_ms"]),
                       "eagle_proposal_ready_ms": float(e["proposal_ready_ms"]),
                       "source_extra_ms": float(e["proposal_ready_ms"]) - float(d["elapsed_ms"]),
                       "first_proposal_accepted_prefix": int(e["first_proposal_accepted_prefix"]),
                       "seed_match": int(d["seed_token_id"]) == int(e["seed_token_id"]),
                       "proposal_token_ids": list(e["proposal_token_ids"])})
    if not paired:
        raise ValueError("no paired requests")
    extra = [p["source_extra_ms"] for p in paired]
    per_bw = {}
    for bw in bandwidths:
        windows = [transfer_ms(p["prompt_tokens"] * kv_bytes_per_token, bw) for p in paired]
        slack = [w - x for w, x in zip(windows, extra)]
        per_bw[f"{bw:g}"] = {"bandwidth_gbps": bw, "full_target_kv_transfer_ms": describe(windows),
                             "proposal_ready_before_full_kv_fraction": sum(s >= 0 for s in slack) / len(slack),
                             "remaining_overlap_slack_ms": describe(slack)}
    return {"schema_version": 1, "samples": len(paired),
            "scope": "producer prefill plus the first drafter proposal; no transport or decode-side replay",
            "target_kv_bytes_per_prompt_token": kv_bytes_per_token,
            "seed_match_fraction": sum(p["seed_match"] for p in paired) / len(paired),
            "source_extra_ms": {**describe(extra),
                                "bootstrap_95pct_ci": bootstrap_mean_ci(extra, samples=bootstrap_samples, seed=seed)},
            "first_proposal_accepted_prefix": describe([p["first_proposal_accepted_prefix"] for p in paired]),
            "bandwidths": per_bw, "paired": paired}


@torch.no_grad()
def source_worker(engine, drafter, requests, *, horizon: int, memory_layers: Sequence[int],
                  seed_layers: Sequence[int], view_budget: int = 2048, warmup: int = 1):
    """(dense rows, EAGLE rows) of ``requests`` (``RAGRequest``-like: ``index``, ``prompt``); GPU."""
    from ..models.sparse_kv_draft import sink_recent_topk_indices
    from ..rope import rope_cos_sin

    cfg, dev = engine.cfg, engine.device
    dense, eagle = [], []
    for k, req in enumerate(list(requests[:warmup]) + list(requests)):
        record = k >= warmup
        prompt = [int(t) for t in req.prompt]
        T = len(prompt)
        ids = torch.tensor(prompt, dtype=torch.int32, device=dev)
        # dense arm: prompt -> first exact token
        slot = engine.new_slot(T + horizon + 64)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record()
        h = engine.prefill(ids, slot)
        b = engine.first_token(h[T - 1:T], position=T, max_new=horizon + 1)
        e1.record()
        torch.cuda.synchronize(dev)
        seed = int(b["tok"][0].item())
        engine.decode(slot, horizon, max_new=horizon + 1)
        target = engine.generated_tokens(horizon + 1)[1:].tolist()
        if record:
            dense.append({"request_index": int(req.index), "prompt_tokens": T, "prompt_sha256": prompt_sha256(prompt),
                          "seed_token_id": seed, "elapsed_ms": e0.elapsed_time(e1)})
        # EAGLE arm: the same prefill with seed-layer hooks, the seed, then the proposal
        slot2 = engine.new_slot(T + horizon + 64)
        captured: dict[int, torch.Tensor] = {}

        def hook(layer: int, hh: torch.Tensor) -> None:
            if layer - 1 in seed_layers:
                captured[layer - 1] = hh[T - 1].clone()

        view = sink_recent_topk_indices(T, None, budget=view_budget).to(dev)
        cos, sin = rope_cos_sin(cfg, torch.arange(T, T + horizon), device=dev, dtype=torch.bfloat16)
        stage = torch.tensor([[min(1.0, view.numel() / T), float(torch.log2(torch.tensor(T + 1.0)) / 17.0)]],
                             device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record()
        h = engine.prefill(ids, slot2, layer_hook=hook)
        if cfg.n_layers - 1 in seed_layers:
            captured[cfg.n_layers - 1] = h[T - 1].clone()
        b = engine.first_token(h[T - 1:T], position=T, max_new=1)
        mk = torch.stack([slot2.k(l).index_select(1, view) for l in memory_layers])
        mv = torch.stack([slot2.v(l).index_select(1, view) for l in memory_layers])
        seeds = torch.stack([captured[l] for l in seed_layers]).unsqueeze(0).to(drafter.fc.weight.dtype)
        first = b["tok"][:1].view(1, 1).long()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            proposal = drafter.propose(first, seeds, mk, mv, cos, sin, stage, n_tokens=horizon)
        e1.record()
        torch.cuda.synchronize(dev)
        prop = proposal[0].tolist()
        if record:
            eagle.append({"request_index": int(req.index), "prompt_tokens": T, "prompt_sha256": prompt_sha256(prompt),
                          "seed_token_id": int(b["tok"][0].item()), "proposal_ready_ms": e0.elapsed_time(e1),
                          "proposal_token_ids": prop, "first_proposal_accepted_prefix": accepted_prefix(prop, target)})
        del slot, slot2
    return dense, eagle


def main(argv=None) -> dict[str, Any]:
    from ..config import get_model_config
    from ..models.engine import B200Engine
    from ..models.sparse_kv_eagle import SparseKVEagleConfig
    from ..synthetic import make_requests
    from ..training.drafter_trainer import load_adapter_checkpoint, prepare_for_training, random_eagle_drafter

    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--workload", default="pd_long")
    p.add_argument("--requests", type=int, default=32)
    p.add_argument("--request-offset", type=int, default=0)
    p.add_argument("--horizon", type=int, default=4)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--bandwidths", default="25,50,100")
    p.add_argument("--memory-layers", default="8,16,24")
    p.add_argument("--seed-layers", default="2,16,29")
    p.add_argument("--drafter-config", default=None, help="SparseKVEagleConfig JSON (default: 8B width)")
    p.add_argument("--adapter", default=None, help="trained adapter checkpoint (default: random init)")
    p.add_argument("--bootstrap-samples", type=int, default=10000)
    p.add_argument("--output-dir", type=Path, required=True)
    a = p.parse_args(argv)
    cfg = get_model_config(a.model)
    engine = B200Engine.random(cfg, seed=0, device="cuda", max_positions=65536)
    ecfg = (SparseKVEagleConfig.from_dict(json.loads(Path(a.drafter_config).read_text())) if a.drafter_config
            else SparseKVEagleConfig())
    drafter = random_eagle_drafter(ecfg, seed=0)
    if a.adapter:
        load_adapter_checkpoint(drafter, a.adapter)
    drafter.freeze_eagle()
    drafter = prepare_for_training(drafter, torch.device("cuda")).eval()  # bf16 trunk, fp32 adapter
    drafter.bind_target_embedding(engine.w.embed)
    reqs = make_requests(a.workload, cfg)[a.request_offset:a.request_offset + a.requests]
    dense, eagle = source_worker(engine, drafter, reqs, horizon=a.horizon,
                                 memory_layers=[int(x) for x in a.memory_layers.split(",")],
                                 seed_layers=[int(x) for x in a.seed_layers.split(",")], warmup=a.warmup)
    out = aggregate_source(dense, eagle, bandwidths=parse_bandwidths(a.bandwidths),
                           kv_bytes_per_token=cfg.n_layers * 2 * cfg.n_kv_heads * cfg.head_dim * 2,
                           bootstrap_samples=a.bootstrap_samples)
    out.update(model=a.model, workload=a.workload, horizon=a.horizon, drafter="adapter" if a.adapter else "random")
    a.output_dir.mkdir(parents=True, exist_ok=True)
    for name, rows in (("dense", dense), ("eagle", eagle), ("paired", out["paired"])):
        (a.output_dir / f"{name}.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    (a.output_dir / "summary.json").write_text(json.dumps({k: v for k, v in out.items() if k != "paired"},
                                                          indent=2) + "\n")
    print(json.dumps({k: v for k, v in out.items() if k != "paired"}, indent=2))
    return out


if __name__ == "__main__":
    main()
