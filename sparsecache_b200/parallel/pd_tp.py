"""Prefill/decode disaggregation between two tensor-parallel groups (TPn -> TPn).

    torchrun --nproc-per-node 8 -m sparsecache_b200.parallel.pd_tp --tp 4 --mode push

Ranks [0, tp) form the prefill group, ranks [tp, 2 tp) the decode group; both
hold the same column/row-parallel shards (rank index i of either group owns
kv heads [i * kv/tp, (i + 1) * kv/tp)).  Decode rank tp + i allocates its
serving slots and flag blocks with CUDA IPC handles; prefill rank i maps
them (plain peer mapping, no multicast object).  Per request:

  prefill group  fused TP prefill (all-gather -> QKV GEMM, GEMM ->
                 reduce-scatter, peer-memory flags); rank i's QKV epilogue
                 stores every rotated K/V row of its kv heads into decode
                 rank tp + i's slot as well as its own cache, and releases
                 that layer's flag right after the GEMM, while its attention
                 and MLP run.  After the LM head the owner of the last row
                 hands the token to the group; every prefill rank then writes
                 it into its partner's seed word and releases the seed flag.
  decode group   each rank waits (bounded, on the device) for its partner's
                 last layer flag and seed flag, then the group runs the TP
                 greedy decode (GEMV + fused all-reduce, one CUDA graph per
                 step).

The K/V of a layer therefore crosses NVLink while later layers are being
prefilled; the exposed transfer is what remains between the prefill group's
end and the decode group's readiness.  The seed token is the last thing to
exist (it needs the final layer), so nothing on the decode side can start
before it: at NVLink rate every layer's K/V has landed by then, and the
draft-while-loading path of the reference (sparse drafting over the pages
already received, one verifier at the end) is the host-wire path
(``serving.progressive``), where transfer is slower than prefill.

Control (``--mode nccl``): the prefill group prefills without push, then each
prefill rank sends its kv heads' prompt K/V layer by layer and the seed with
NCCL send/recv to its partner.

Open-loop serving (``--arrival-rate``): seeded Poisson arrivals; the prefill
group starts request i at max(arrival, its previous end) into decode slot
i mod n_slots once the decode group released it (bounded device wait on a
free flag in the prefill rank's memory), so request i+1's prefill and push
overlap request i's decode.

Reference behaviour: the reference's 1P1D handoff goes through an LMCache CPU
store over a paced TCP wire (docs/RUN_PROGRESSIVE_PD_LIVE.md:3-23;
experiments/pd_progressive_kv_pipeline.py:187-456); here both sides are TP
groups and the transport is device-initiated NVLink stores.

Timing: TTFT and the exposed transfer use the host monotonic clock (one
machine, the same clock in every process) between barrier-aligned starts and
each decode rank's device-synchronised readiness, max over ranks; TPOT uses
CUDA events on the decode ranks, max over ranks.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import random
import statistics
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from ..config import get_model_config
from ..synthetic import make_requests
from .pd import PDChannel, wait_ready
from .tp import TPEngine, TPGroup
from .tp_bench import random_shard


class TPPD:
    """One rank's view of a TPn -> TPn prefill/decode deployment."""

    def __init__(self, cfg, tp: int, *, capacity: int, n_slots: int = 1, push: bool = True, seed: int = 0) -> None:
        world, rank = dist.get_world_size(), dist.get_rank()
        if world != 2 * tp:
            raise ValueError(f"TP{tp} -> TP{tp} needs {2 * tp} ranks, got {world}")
        self.tp, self.cfg = tp, cfg
        self.role = "prefill" if rank < tp else "decode"
        self.index = rank % tp
        self.partner = rank + tp if self.role == "prefill" else rank - tp
        # every rank creates every group in the same order
        groups = [dist.new_group(list(range(tp))), dist.new_group(list(range(tp, 2 * tp)))]
        pairs = [dist.new_group([i, i + tp]) for i in range(tp)]
        self.tp_group = groups[0 if self.role == "prefill" else 1]
        self.pair_group = pairs[self.index]
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.group = TPGroup(self.tp_group)
        weights = random_shard(cfg, self.index, tp, seed, dev)
        self.capacity = capacity
        self.tpe = TPEngine(cfg, weights, self.group, max_rows=(capacity + tp * 128) // tp,
                            max_positions=capacity + 1024)
        self.push = push
        self.ch = None
        self.nccl_slot = None
        if push:
            self.ch = PDChannel(self.tpe.engine, role=self.role, capacity=capacity, prefill_rank=self.index,
                                decode_rank=self.index + tp, group=self.pair_group, n_slots=n_slots)
        else:
            self.nccl_slot = self.tpe.new_slot(capacity)

    @property
    def n_layers(self) -> int:
        return self.cfg.n_layers

    # ------------------------------------------------------------ prefill
    def prefill(self, ids: torch.Tensor, max_new: int, index: int = 0) -> torch.Tensor:
        """Prefill group: TP prefill (with the fused push in push mode) and the first token."""
        T = ids.numel()
        tpe = self.tpe
        if self.push:
            ch = self.ch
            push = ch.push_target(index)
            x, rows, _ = tpe.prefill(ids, ch.slot, push=push)
            tok = tpe.first_token(x, rows, T, max_new=max_new)
            L = self.n_layers
            tpe.ext.peer_signal(push.flag(L), 0, None, tok)
            tpe.ext.peer_signal(push.flag(L + 1), push.epoch, ch.stamps[0:1])
            return tok
        x, rows, _ = tpe.prefill(ids, self.nccl_slot)
        return tpe.first_token(x, rows, T, max_new=max_new)

    def send_kv(self, T: int, tok: torch.Tensor) -> None:
        """Control path, prefill side: every layer's local prompt K/V, then the seed, with NCCL."""
        for layer in range(self.n_layers):
            dist.send(self.nccl_slot.data[layer, :, :, :T].contiguous(), self.partner)
        dist.send(tok.clone(), self.partner)

    # ------------------------------------------------------------- decode
    def wait(self, index: int = 0, timeout_s: float = 60.0) -> None:
        """Decode side, push mode: bounded device wait for the partner's last layer and seed."""
        wait_ready(self.ch, index, timeout_s)

    def recv_kv(self, T: int) -> torch.Tensor:
        """Control path, decode side: receive every layer's local prompt K/V and the seed."""
        lc = self.tpe.lcfg
        buf = torch.empty(2, lc.n_kv_heads, T, lc.head_dim, dtype=torch.bfloat16, device=self.device)
        for layer in range(self.n_layers):
            dist.recv(buf, self.partner)
            self.nccl_slot.data[layer, :, :, :T].copy_(buf)
        seed = torch.empty(1, dtype=torch.int32, device=self.device)
        dist.recv(seed, self.partner)
        return seed

    def decode(self, T: int, max_new: int, index: int = 0, seed: torch.Tensor | None = None) -> None:
        """Decode group: greedy TP decode from the received K/V and seed token."""
        if self.push:
            slot = self.ch.slots[index]
            seed = self.ch.slot_flags(index)[self.n_layers:self.n_layers + 1]
        else:
            slot = self.nccl_slot
        self.tpe.seed_decode(seed, T, max_new=max_new)
        self.tpe.decode(slot, max_new - 1)

    def tokens(self, n: int) -> list[int]:
        return self.tpe.engine.generated_tokens(n).tolist()

    def check(self) -> None:
        self.tpe.check_status()
        if self.ch is not None and int(self.ch.status.item()) != 0:
            raise RuntimeError(f"a bounded peer-flag wait timed out (status {int(self.ch.status.item())})")

    def close(self) -> None:
        self.tpe.engine.release_graphs()
        dist.barrier()
        if self.ch is not None:
            self.ch.close()
        self.tpe.close()


def _max_over_ranks(values: list[float], dev) -> list[float]:
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run_closed_loop(args) -> dict | None:
    """One request at a time: TTFT, TPOT and exposed transfer per request (max over ranks)."""
    tp = args.tp
    cfg = get_model_config(args.model)
    if args.layers:
        cfg = cfg.with_layers(args.layers)
    requests = make_requests("pd_long", cfg)
    need = args.warmup + args.steps
    served = [requests[i % len(requests)] for i in range(need)]
    capacity = max(r.prompt_tokens for r in served) + args.new_tokens + tp * 128 + 64
    dep = TPPD(cfg, tp, capacity=capacity, push=args.mode == "push")
    dev = dep.device
    rows = []
    for i, req in enumerate(served):
        ids = torch.tensor(req.prompt, dtype=torch.int32, device=dev)
        T = req.prompt_tokens
        if dep.ch is not None:
            dep.ch.epoch = i + 1
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.monotonic()
        prefill_end = ready = 0.0
        tpot = 0.0
        if dep.role == "prefill":
            tok = dep.prefill(ids, args.new_tokens)
            torch.cuda.synchronize()
            prefill_end = time.monotonic() - t0
            if not dep.push:
                dep.send_kv(T, tok)
                torch.cuda.synchronize()
        else:
            seed = None
            if dep.push:
                dep.wait()
            else:
                seed = dep.recv_kv(T)
            torch.cuda.synchronize()
            ready = time.monotonic() - t0
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record()
            dep.decode(T, args.new_tokens, seed=seed)
            b.record()
            b.synchronize()
            tpot = a.elapsed_time(b) / max(1, args.new_tokens - 1)
        dep.check()
        # prefill ranks contribute their end, decode ranks their readiness and TPOT (max over all ranks)
        prefill_end, ready, tpot = _max_over_ranks([prefill_end, ready, tpot], dev)
        if i >= args.warmup:
            rows.append({"prompt_tokens": T, "ttft_ms": ready * 1e3, "prefill_ms": prefill_end * 1e3,
                         "exposed_ms": max(0.0, ready - prefill_end) * 1e3, "tpot_ms": tpot})
    last = dep.tokens(args.new_tokens)[:8] if dep.role == "decode" else None
    gathered = [None] * dist.get_world_size()
    dist.all_gather_object(gathered, last)
    dep.close()
    if dist.get_rank() != 0:
        return None
    out = {"mode": args.mode, "layout": f"TP{tp} prefill -> TP{tp} decode", "model": cfg.name,
           "layers": cfg.n_layers, "new_tokens": args.new_tokens, "requests": len(rows),
           "mean_prompt_tokens": statistics.fmean(r["prompt_tokens"] for r in rows),
           "decode_tokens_rank0_of_group": gathered[tp]}
    for key in ("ttft_ms", "prefill_ms", "exposed_ms", "tpot_ms"):
        xs = sorted(r[key] for r in rows)
        out[key.replace("_ms", "_p50_ms")] = statistics.median(xs)
        out[key.replace("_ms", "_p99_ms")] = xs[min(len(xs) - 1, int(round(0.99 * (len(xs) - 1))))]
    # NVLink bytes of the push per request (all ranks): every layer's K and V of the padded prompt
    kv_bytes = [2 * cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 2 * r["prompt_tokens"] for r in rows]
    out["kv_bytes_mean"] = statistics.fmean(kv_bytes)
    out["rows"] = rows
    return out


def run_poisson(args) -> dict | None:
    """Open-loop Poisson arrivals on the TP pair of groups (push mode, n_slots decode slots)."""
    tp = args.tp
    cfg = get_model_config(args.model)
    if args.layers:
        cfg = cfg.with_layers(args.layers)
    requests = make_requests("pd_long", cfg)
    n = args.warmup + args.steps
    served = [requests[i % len(requests)] for i in range(n)]
    capacity = max(r.prompt_tokens for r in served) + args.new_tokens + tp * 128 + 64
    dep = TPPD(cfg, tp, capacity=capacity, n_slots=args.slots, push=True)
    dev, ch, ext = dep.device, dep.ch, dep.tpe.ext
    rng = random.Random(args.seed)
    arrivals, t = [], 0.0
    for i in range(n):
        arrivals.append(t)
        t += rng.expovariate(args.arrival_rate) if i >= args.warmup else 1.0
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.monotonic()
    rec = []
    for i, req in enumerate(served):
        s = i % args.slots
        ch.epoch = i + 1
        T = req.prompt_tokens
        if dep.role == "prefill":
            wait = arrivals[i] - (time.monotonic() - t0)
            if wait > 0:
                time.sleep(wait)
            start = time.monotonic() - t0
            if i >= args.slots:  # the decode partner has released the slot's previous request
                ext.wait_flag(ch.free, s, i + 1 - args.slots, int(60e9), ch.status)
            dep.prefill(torch.tensor(req.prompt, dtype=torch.int32, device=dev), args.new_tokens, index=s)
            torch.cuda.synchronize()
            rec.append({"start": start, "prefill_end": time.monotonic() - t0})
        else:
            dep.wait(s)
            torch.cuda.synchronize()
            ready = time.monotonic() - t0
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record()
            dep.decode(T, args.new_tokens, index=s)
            b.record()
            ext.peer_signal(ch.free_base + 4 * s, i + 1)
            b.synchronize()
            rec.append({"ready": ready, "tpot_ms": a.elapsed_time(b) / max(1, args.new_tokens - 1)})
    dep.check()
    gathered = [None] * dist.get_world_size()
    dist.all_gather_object(gathered, (dep.role, rec))
    dep.close()
    if dist.get_rank() != 0:
        return None
    pre = [r for role, r in gathered if role == "prefill"]
    dec = [r for role, r in gathered if role == "decode"]
    rows = []
    for i in range(args.warmup, n):
        ready = max(d[i]["ready"] for d in dec)
        pend = max(p[i]["prefill_end"] for p in pre)
        start = max(p[i]["start"] for p in pre)
        rows.append({"ttft_ms": (ready - arrivals[i]) * 1e3, "tpot_ms": max(d[i]["tpot_ms"] for d in dec),
                     "prefill_ms": (pend - start) * 1e3, "prefill_queue_ms": (start - arrivals[i]) * 1e3,
                     "decoder_queue_ms": max(0.0, ready - pend) * 1e3, "prompt_tokens": served[i].prompt_tokens})

    def pct(key, q):
        v = sorted(x[key] for x in rows)
        return v[min(len(v) - 1, int(round(q * (len(v) - 1))))]

    return {"mode": "push_poisson", "layout": f"TP{tp} prefill -> TP{tp} decode", "arrival_rate": args.arrival_rate,
            "slots": args.slots, "model": cfg.name, "layers": cfg.n_layers, "new_tokens": args.new_tokens,
            "requests": len(rows), "mean_prompt_tokens": statistics.fmean(r["prompt_tokens"] for r in rows),
            **{f"{k}_p{int(q * 100)}": pct(k, q) for k in ("ttft_ms", "tpot_ms", "prefill_ms", "prefill_queue_ms",
                                                                 "decoder_queue_ms") for q in (0.5, 0.99)}}


def parse_modes(mode: str, arrival_rate: float) -> list[str]:
    """The arms of one run: ``push`` / ``nccl`` (closed loop) and ``poisson`` (open loop), in order.

    A lone ``push`` with an arrival rate means Poisson arrivals only (the
    single-mode form of the command line).
    """
    modes = [m.strip() for m in mode.split(",") if m.strip()]
    if not modes or any(m not in ("push", "nccl", "poisson") for m in modes):
        raise ValueError(f"--mode: expected push, nccl or poisson (comma list), got {mode!r}")
    if len(set(modes)) != len(modes):
        raise ValueError(f"--mode: an arm is listed twice in {mode!r}")
    if modes == ["push"] and arrival_rate > 0:
        modes = ["poisson"]
    if "poisson" in modes and arrival_rate <= 0:
        raise ValueError("--mode poisson needs --arrival-rate > 0")
    return modes


def main() -> None:
    p = argparse.ArgumentParser(description="TPn prefill -> TPn decode with the fused NVLink KV push")
    p.add_argument("--tp", type=int, default=4)
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--mode", default="push",
                   help="push | nccl | poisson, or a comma list run back to back in one process group "
                        "(e.g. push,nccl,poisson); poisson serves open-loop arrivals at --arrival-rate")
    p.add_argument("--steps", type=int, default=6)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--new-tokens", type=int, default=128)
    p.add_argument("--arrival-rate", type=float, default=0.0,
                   help="requests/s of the poisson mode; > 0 with a single --mode push serves only Poisson arrivals")
    p.add_argument("--slots", type=int, default=2, help="decode slots (Poisson mode)")
    p.add_argument("--seed", type=int, default=0)
    args = p.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    try:
        modes = parse_modes(args.mode, args.arrival_rate)
    except ValueError as exc:
        raise SystemExit(str(exc)) from None
    try:
        for i, mode in enumerate(modes):
            if i:  # the previous arm's engines, peer mappings and cached blocks are gone before the next
                gc.collect()
                torch.cuda.synchronize()
                torch.cuda.empty_cache()
                dist.barrier()
            run = argparse.Namespace(**{**vars(args), "mode": "push" if mode == "poisson" else mode})
            out = run_poisson(run) if mode == "poisson" else run_closed_loop(run)
            if out is not None:
                print(json.dumps(out), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
