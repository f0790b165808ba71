"""Prefill/decode disaggregation across GPUs with the KV push fused into prefill.

One process per GPU.  The decode rank allocates its serving slot and a small
flag array with ``shared_empty`` (cudaMalloc + CUDA IPC handle); the prefill
rank maps both with ``shared_open`` (plain peer mapping over NVLink, no
multicast object).  Per request (epoch e):

  prefill rank   prefill with ``push``: the QKV GEMM epilogue of every layer
                 stores each rotated K/V row into its own cache AND into the
                 decode slot; right after each layer's GEMM a signal kernel
                 releases flags[layer] = e (system-scope fence + st.release),
                 while the prefill GPU continues with the layer's attention and
                 MLP; after the LM head the seed token is written to
                 flags[L] and flags[L + 1] = e is released.
  decode rank    a bounded device-side wait on flags[L - 1] (every layer, in
                 stream order) and flags[L + 1]; the seed token is read on the
                 device and greedy decode runs from its CUDA graph.

Exposed transfer = time between the prefill rank finishing its prompt and the
decode rank having every layer's K/V + the seed.  The control path
(``mode="nccl"``) prefills without push and then sends the whole prompt KV
with NCCL send/recv per layer (the baseline to beat).

Reference behaviour: the reference's 1P1D handoff goes through an
out-of-tree LMCache CPU store over ZMQ/TCP with a paced wire
(docs/RUN_PROGRESSIVE_PD_LIVE.md:3-23, 56-116); here the transport is
device-initiated NVLink stores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from .. import ops
from ..config import get_model_config
from ..models.engine import B200Engine, KVSlot, PushTarget
from ..synthetic import make_requests

FLAG_SLOTS = 8


class PDChannel:
    """Decode-side slots + flags shared with the prefill rank over CUDA IPC.

    ``n_slots`` decode slots let the prefill rank push request i+1 while the
    decode rank still decodes request i.  Slot s has its own flag block
    (``n_layers`` layer flags, the seed token, the completion flag); the
    prefill rank owns ``free`` flags (one per slot) that the decode rank
    releases when it is done with a slot, and waits on them (bounded) before
    pushing into a slot again.
    """

    def __init__(self, engine: B200Engine, *, role: str, capacity: int, prefill_rank: int, decode_rank: int,
                 group=None, n_slots: int = 1) -> None:
        self.engine = engine
        self.role = role
        self.capacity = capacity
        self.n_slots = n_slots
        cfg = engine.cfg
        self.n_layers = cfg.n_layers
        self.flag_stride = cfg.n_layers + FLAG_SLOTS
        ext = ops.ext()
        dev = engine.device.index
        self.slot_bytes = KVSlot.nbytes_for(cfg, capacity)
        self.status = torch.zeros(1, dtype=torch.int32, device=engine.device)
        self.stamps = torch.zeros(4, dtype=torch.int64, device=engine.device)
        handles = None
        if role == "decode":
            buf, h_slot = ext.shared_empty(self.slot_bytes * n_slots, dev)
            flags, h_flags = ext.shared_empty(4 * self.flag_stride * n_slots, dev)
            self._buffers = (buf, flags)
            self.slots = [KVSlot.from_buffer(cfg, capacity, buf[i * self.slot_bytes:(i + 1) * self.slot_bytes])
                          for i in range(n_slots)]
            self.slot = self.slots[0]
            self.all_flags = flags.view(torch.int32)
            self.flags = self.all_flags[: self.flag_stride]
            handles = (h_slot, h_flags)
        else:
            free, h_free = ext.shared_empty(4 * max(n_slots, 4), dev)
            self._free = free
            self.free = free.view(torch.int32)
            handles = (h_free,)
        gathered = [None] * dist.get_world_size(group)
        dist.all_gather_object(gathered, handles, group=group)
        self.epoch = 0

        def peer(rank):
            return gathered[dist.get_group_rank(group, rank) if group is not None else rank]

        if role == "prefill":
            h_slot, h_flags = peer(decode_rank)
            self.base = ext.shared_open(h_slot)
            self.flag_base = ext.shared_open(h_flags)
            self.slot = engine.new_slot(capacity)
        else:
            (h_free,) = peer(prefill_rank)
            self.free_base = ext.shared_open(h_free)

    def push_target(self, index: int = 0) -> PushTarget:
        cfg = self.engine.cfg
        return PushTarget(self.base + index * self.slot_bytes, self.capacity,
                          self.flag_base + 4 * self.flag_stride * index, self.epoch, cfg.n_layers,
                          cfg.n_kv_heads * self.capacity * cfg.head_dim)

    def slot_flags(self, index: int) -> torch.Tensor:
        return self.all_flags[index * self.flag_stride:(index + 1) * self.flag_stride]

    def close(self) -> None:
        ext = ops.ext()
        if self.role == "prefill":
            ext.shared_close(self.base)
            ext.shared_close(self.flag_base)
        else:
            ext.shared_close(self.free_base)


def prefill_request(ch: PDChannel, ids: torch.Tensor, max_new: int, index: int = 0) -> None:
    """Prefill side: prefill with the fused push into decode slot ``index``, then publish the seed token."""
    eng = ch.engine
    ext = eng.ext
    T = ids.numel()
    push = ch.push_target(index)
    h = eng.prefill(ids, ch.slot, push=push)
    b = eng.first_token(h[T - 1:T], position=T, max_new=max_new)
    L = ch.n_layers
    ext.peer_signal(push.flag(L), 0, None, b["tok"][0:1])
    ext.peer_signal(push.flag(L + 1), push.epoch, ch.stamps[0:1])


def wait_ready(ch: PDChannel, index: int = 0, timeout_s: float = 20.0) -> None:
    """Decode side: bounded device wait for every layer of slot ``index`` and its seed."""
    ext, L, flags = ch.engine.ext, ch.n_layers, ch.slot_flags(index)
    ext.wait_flag(flags, L - 1, ch.epoch, int(timeout_s * 1e9), ch.status, ch.stamps[0:1])
    ext.wait_flag(flags, L + 1, ch.epoch, int(timeout_s * 1e9), ch.status, ch.stamps[1:2])


def decode_ready(ch: PDChannel, T: int, max_new: int, index: int = 0) -> None:
    """Decode side, after ``wait_ready``: greedy decode from the pushed KV and seed."""
    eng, L = ch.engine, ch.n_layers
    flags = ch.slot_flags(index)
    b = eng._decode_buffers(max_new)
    eng.ext.embedding(flags[L:L + 1], eng.w.embed, b["h"][:1])
    b["log"][0:1].copy_(flags[L:L + 1])
    b["gen"].fill_(1)
    b["counter"].zero_()
    eng.set_decode_state(position=T)
    eng.decode(ch.slots[index], max_new - 1, max_new=max_new)


def decode_request(ch: PDChannel, T: int, max_new: int, timeout_s: float = 20.0, index: int = 0) -> None:
    """Decode side: wait (bounded) for every layer and the seed, then greedy decode."""
    wait_ready(ch, index, timeout_s)
    decode_ready(ch, T, max_new, index)


def nccl_prefill_request(eng: B200Engine, slot: KVSlot, ids: torch.Tensor, max_new: int, peer: int) -> torch.Tensor:
    """Control path: prefill locally, then send every layer's K/V and the seed with NCCL."""
    T = ids.numel()
    h = eng.prefill(ids, slot)
    b = eng.first_token(h[T - 1:T], position=T, max_new=max_new)
    for layer in range(eng.cfg.n_layers):
        dist.send(slot.data[layer, :, :, :T].contiguous(), peer)
    dist.send(b["tok"][0:1].clone(), peer)
    return b["tok"]


def nccl_decode_request(eng: B200Engine, slot: KVSlot, T: int, max_new: int, peer: int) -> None:
    cfg = eng.cfg
    buf = torch.empty(2, cfg.n_kv_heads, T, cfg.head_dim, dtype=torch.bfloat16, device=eng.device)
    for layer in range(cfg.n_layers):
        dist.recv(buf, peer)
        slot.data[layer, :, :, :T].copy_(buf)
    tok = torch.empty(1, dtype=torch.int32, device=eng.device)
    dist.recv(tok, peer)
    b = eng._decode_buffers(max_new)
    eng.ext.embedding(tok, eng.w.embed, b["h"][:1])
    b["log"][0:1].copy_(tok)
    b["gen"].fill_(1)
    eng.set_decode_state(position=T)
    eng.decode(slot, max_new - 1, max_new=max_new)


def build_engine(args, dev) -> B200Engine:
    """The serving engine of a rank: a model directory's weights, else the seeded random-init preset."""
    if getattr(args, "model_dir", None):
        from ..models.checkpoint import load_oracle

        return B200Engine.from_oracle(load_oracle(args.model_dir, dtype=torch.bfloat16), dev, max_positions=65536)
    cfg = get_model_config(args.model)
    if args.layers:
        cfg = cfg.with_layers(args.layers)
    return B200Engine.random(cfg, seed=0, device=dev, max_positions=65536)


def run(args) -> dict | None:
    rank, world = dist.get_rank(), dist.get_world_size()
    if world % 2:
        raise ValueError("prefill/decode needs an even number of ranks (pairs)")
    pairs = world // 2
    role = "prefill" if rank < pairs else "decode"
    peer = rank + pairs if role == "prefill" else rank - pairs
    dev = torch.device("cuda", torch.cuda.current_device())
    engine = build_engine(args, dev)
    cfg = engine.cfg
    requests = make_requests("pd_long", cfg)
    mine = [r for r in requests if r.index % pairs == rank % pairs]
    need = args.warmup + args.steps
    served = [mine[i % len(mine)] for i in range(need)]
    capacity = max(r.prompt_tokens for r in served) + args.new_tokens + 64
    # one channel per prefill/decode pair: a 2-rank group
    groups = [dist.new_group([p, p + pairs]) for p in range(pairs)]
    group = groups[rank % pairs]
    ch = PDChannel(engine, role=role, capacity=capacity, prefill_rank=rank % pairs, decode_rank=rank % pairs + pairs,
                   group=group) if args.mode == "push" else None
    nccl_slot = engine.new_slot(capacity) if args.mode == "nccl" else None
    ttft, tpot, exposed = [], [], []
    for i, req in enumerate(served):
        ids = torch.tensor(req.prompt, dtype=torch.int32, device=dev)
        T = req.prompt_tokens
        if ch is not None:
            ch.epoch += 1
        dist.barrier(group=group)
        torch.cuda.synchronize()
        t0 = time.monotonic()
        if role == "prefill":
            if args.mode == "push":
                prefill_request(ch, ids, args.new_tokens)
                torch.cuda.synchronize()
                t_prefill_end = time.monotonic() - t0
            else:
                # the prompt is done (seed token ready) before any byte is sent
                h = engine.prefill(ids, nccl_slot)
                b = engine.first_token(h[T - 1:T], position=T, max_new=args.new_tokens)
                torch.cuda.synchronize()
                t_prefill_end = time.monotonic() - t0
                for layer in range(cfg.n_layers):
                    dist.send(nccl_slot.data[layer, :, :, :T].contiguous(), peer)
                dist.send(b["tok"][0:1].clone(), peer)
                torch.cuda.synchronize()
            rec = torch.tensor([t_prefill_end], dtype=torch.float64, device=dev)
            dist.send(rec, peer)
        else:
            first = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start = torch.cuda.Event(enable_timing=True)
            start.record()
            L = cfg.n_layers
            ext = engine.ext
            b = engine._decode_buffers(args.new_tokens)
            if args.mode == "push":
                ext.wait_flag(ch.flags, L - 1, ch.epoch, int(20e9), ch.status, ch.stamps[0:1])
                ext.wait_flag(ch.flags, L + 1, ch.epoch, int(20e9), ch.status, ch.stamps[1:2])
                seed, slot = ch.flags[L:L + 1], ch.slot
            else:
                buf = torch.empty(2, cfg.n_kv_heads, T, cfg.head_dim, dtype=torch.bfloat16, device=dev)
                for layer in range(L):
                    dist.recv(buf, peer)
                    nccl_slot.data[layer, :, :, :T].copy_(buf)
                seed = torch.empty(1, dtype=torch.int32, device=dev)
                dist.recv(seed, peer)
                slot = nccl_slot
            first.record()
            first.synchronize()
            t_ready = time.monotonic() - t0
            if args.mode == "push" and int(ch.status.item()) != 0:
                raise RuntimeError("decode rank timed out waiting for the pushed KV")
            ext.embedding(seed, engine.w.embed, b["h"][:1])
            b["log"][0:1].copy_(seed)
            b["gen"].fill_(1)
            engine.set_decode_state(position=T)
            engine.decode(slot, args.new_tokens - 1, max_new=args.new_tokens)
            end.record()
            end.synchronize()
            rec = torch.empty(1, dtype=torch.float64, device=dev)
            dist.recv(rec, peer)
            t_prefill_end = float(rec.item())
            if i >= args.warmup:
                ttft.append(t_ready * 1000)
                exposed.append(max(0.0, (t_ready - t_prefill_end) * 1000))
                tpot.append(first.elapsed_time(end) / max(1, args.new_tokens - 1))
    if ch is not None:
        dist.barrier(group=group)
        ch.close()
    stats = None
    if role == "decode":
        last_tokens = engine.generated_tokens(args.new_tokens)[:8].tolist()
        stats = {"ttft_ms": ttft, "tpot_ms": tpot, "exposed_ms": exposed, "last_tokens": last_tokens,
                 "prompt_tokens": [r.prompt_tokens for r in served[args.warmup:]]}
    gathered = [None] * world
    dist.all_gather_object(gathered, stats)
    if rank != 0:
        return None
    dec = [g for g in gathered if g is not None]
    flat = lambda key: [x for g in dec for x in g[key] if x is not None]  # noqa: E731
    out = {"mode": args.mode, "pairs": pairs, "model": cfg.name, "layers": cfg.n_layers,
           "new_tokens": args.new_tokens, "requests": args.steps * pairs,
           "last_tokens": dec[0]["last_tokens"], "prompt_tokens": dec[0]["prompt_tokens"]}
    for key in ("ttft_ms", "tpot_ms", "exposed_ms"):
        xs = flat(key)
        if xs:
            out[key.replace("_ms", "_p50_ms")] = statistics.median(xs)
            out[key.replace("_ms", "_max_ms")] = max(xs)
    return out


def serve_poisson(args) -> dict | None:
    """Open-loop serving of Poisson arrivals on prefill/decode pairs.

    Each pair draws seeded exponential inter-arrival gaps at ``arrival_rate``
    requests/s.  The prefill rank starts request i at max(arrival_i, its
    previous prefill end), waits (bounded, on the device) until decode slot
    i mod n_slots is free again, and prefills with the fused push into that
    slot.  The decode rank decodes the requests in order; after each it
    releases the slot's free flag in the prefill rank's memory.  So a
    request's prefill and its KV transfer overlap the previous request's
    decode.  Per request: TTFT = decode-side readiness of KV + seed minus the
    arrival time; TPOT from CUDA events around the decode; the decoder queue =
    readiness minus the prefill rank's prefill end (the pushed KV is complete
    when the prefill ends; the closed-loop mode measures the exposed
    transfer itself).  Host monotonic clock, one machine.
    """
    import random

    rank, world = dist.get_rank(), dist.get_world_size()
    if world % 2:
        raise ValueError("prefill/decode needs an even number of ranks (pairs)")
    pairs = world // 2
    role = "prefill" if rank < pairs else "decode"
    pair = rank % pairs
    dev = torch.device("cuda", torch.cuda.current_device())
    engine = build_engine(args, dev)
    cfg = engine.cfg
    mine = [r for r in make_requests("pd_long", cfg) if r.index % pairs == pair]
    n = args.warmup + args.steps
    served = [mine[i % len(mine)] for i in range(n)]
    capacity = max(r.prompt_tokens for r in served) + args.new_tokens + 64
    groups = [dist.new_group([p, p + pairs]) for p in range(pairs)]
    group = groups[pair]
    ch = PDChannel(engine, role=role, capacity=capacity, prefill_rank=pair, decode_rank=pair + pairs, group=group,
                   n_slots=args.slots)
    rng = random.Random(args.seed * 1000 + pair)
    arrivals, t = [], 0.0
    for i in range(n):
        arrivals.append(t)
        t += rng.expovariate(args.arrival_rate) if i >= args.warmup else 0.5
    ext = engine.ext
    timeout_ns = int(60e9)
    dist.barrier(group=group)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    rec: list[dict] = []
    for i, req in enumerate(served):
        s = i % args.slots
        ch.epoch = i + 1
        T = req.prompt_tokens
        if role == "prefill":
            wait = arrivals[i] - (time.monotonic() - t0)
            if wait > 0:
                time.sleep(wait)
            t_start = time.monotonic() - t0
            if i >= args.slots:  # the decode rank has finished the slot's previous request
                ext.wait_flag(ch.free, s, i + 1 - args.slots, timeout_ns, ch.status)
            prefill_request(ch, torch.tensor(req.prompt, dtype=torch.int32, device=dev), args.new_tokens, index=s)
            torch.cuda.synchronize()
            rec.append({"i": i, "start": t_start, "prefill_end": time.monotonic() - t0})
        else:
            wait_ready(ch, s, timeout_s=60.0)
            torch.cuda.synchronize()
            t_ready = time.monotonic() - t0
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record()
            decode_ready(ch, T, args.new_tokens, index=s)
            b.record()
            ext.peer_signal(ch.free_base + 4 * s, i + 1)
            b.synchronize()
            rec.append({"i": i, "ready": t_ready, "arrival": arrivals[i], "prompt_tokens": T,
                        "tpot_ms": a.elapsed_time(b) / max(1, args.new_tokens - 1)})
    torch.cuda.synchronize()
    if int(ch.status.item()) != 0:
        raise RuntimeError("a bounded peer-flag wait timed out")
    gathered = [None] * world
    dist.all_gather_object(gathered, (role, pair, rec))
    dist.barrier()
    ch.close()
    if rank != 0:
        return None
    pre = {(p, r["i"]): r for role_, p, rr in gathered if role_ == "prefill" for r in rr}
    rows = []
    for role_, p, rr in gathered:
        if role_ != "decode":
            continue
        for r in rr:
            if r["i"] < args.warmup:
                continue
            pr = pre[(p, r["i"])]
            rows.append({"ttft_ms": (r["ready"] - r["arrival"]) * 1e3, "tpot_ms": r["tpot_ms"],
                         # KV + seed are complete on the decode GPU at prefill end (the push is fused
                         # into the prefill); what remains is the wait for the decoder to be free
                         "decoder_queue_ms": max(0.0, (r["ready"] - pr["prefill_end"]) * 1e3),
                         "prefill_queue_ms": (pr["start"] - r["arrival"]) * 1e3,
                         "prefill_ms": (pr["prefill_end"] - pr["start"]) * 1e3, "prompt_tokens": r["prompt_tokens"]})

    def pct(key, q):
        v = sorted(x[key] for x in rows)
        return v[min(len(v) - 1, int(round(q * (len(v) - 1))))] if v else None

    return {"mode": "push_poisson", "pairs": pairs, "arrival_rate_per_pair": args.arrival_rate, "slots": args.slots,
            "model": cfg.name, "layers": cfg.n_layers, "new_tokens": args.new_tokens, "requests": len(rows),
            **{f"{k}_p{int(q * 100)}": pct(k, q) for k in ("ttft_ms", "tpot_ms", "prefill_ms", "prefill_queue_ms",
                                                                 "decoder_queue_ms")
               for q in (0.5, 0.99)},
            "mean_prompt_tokens": statistics.fmean(r["prompt_tokens"] for r in rows) if rows else None}


def main() -> None:
    p = argparse.ArgumentParser(description="Prefill/decode disaggregation with the fused NVLink KV push")
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--model-dir", default=None, help="model directory (HF Llama / Mistral or this package's)")
    p.add_argument("--mode", choices=("push", "nccl"), default="push")
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--new-tokens", type=int, default=128)
    p.add_argument("--arrival-rate", type=float, default=0.0,
                   help="requests/s per pair; > 0 serves open-loop Poisson arrivals")
    p.add_argument("--slots", type=int, default=2, help="decode slots per pair (Poisson mode)")
    p.add_argument("--seed", type=int, default=0)
    args = p.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    try:
        out = serve_poisson(args) if args.arrival_rate > 0 else run(args)
        if out is not None:
            print(json.dumps(out), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
