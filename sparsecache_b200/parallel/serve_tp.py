"""Tensor-parallel RAG serving: CacheBlend reuse + sparse-KV speculative decoding (70B TP8).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m sparsecache_b200.parallel.serve_tp \\
        --model llama3-70b --requests 8 --new-tokens 128

Per rank (one process per GPU, TP group = the whole world):
  * producer: every unique document is prefilled alone at positions 0..n-1
    by the fused TP prefill; each rank stores the K/V of its own kv heads in
    a deduplicated HBM store (the reference's independent-document producer,
    experiments/reuse_cacheblend_pipeline.py:347-405, sharded by head);
  * consumer: the composer re-rotates and concatenates the local blocks
    (layers from the check layer up), ``TPEngine.cacheblend`` recomputes the
    check layer over every row and the top ``ratio`` deviating document rows
    above it (reuse_cacheblend_pipeline.py:580-660), the last active row's
    LM head gives the first token;
  * decode: greedy CUDA-graph steps with all-reduce-fused GEMVs, or
    speculative decoding with the TP sparse-KV EAGLE drafter (gamma-token
    proposals over sink + recent + top-chunk target KV, verified in one
    batched target step).

Reported (rank 0, one JSON line; device time, max over ranks): TTFT p50/p99
of CacheBlend vs full prefill, TPOT and decode tokens/s for greedy and
speculative decoding, mean accepted drafts, and batched greedy decode
(B sequences per step on the skinny tensor-core GEMMs and one attention
launch for all sequences, B <= 32).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
from datetime import timedelta

import torch
import torch.distributed as dist

from ..config import CacheBlendConfig, get_model_config
from ..models.sparse_kv_draft import sink_recent_topk_indices
from ..models.sparse_kv_eagle import SparseKVEagleConfig
from ..store import DocumentKVStore
from ..synthetic import make_requests
from .tp import TPEngine, TPGroup
from .tp_draft import TPDraftWeights, TPEagleDrafter, speculative_generate


def memory_layers_for(n_layers: int) -> tuple[int, int, int]:
    """Low / mid / high target layers whose KV the drafter reads."""
    return (n_layers // 4, n_layers // 2, (3 * n_layers) // 4)


def drafter_config_for(cfg, draft_vocab: int = 32000) -> SparseKVEagleConfig:
    """One-layer EAGLE drafter of the target's width."""
    return SparseKVEagleConfig(target_hidden_size=cfg.d_model, hidden_size=cfg.d_model,
                               intermediate_size=cfg.ffn, head_dim=cfg.head_dim,
                               num_attention_heads=cfg.n_heads, num_key_value_heads=cfg.n_kv_heads,
                               num_memory_heads=cfg.n_kv_heads, num_memory_layers=3, num_seed_layers=3,
                               target_vocab_size=cfg.vocab, draft_vocab_size=min(draft_vocab, cfg.vocab),
                               rms_norm_eps=cfg.rms_eps)


class TPRAGServer:
    """Batch-1 RAG serving over one TP group (every rank calls every method in the same order)."""

    def __init__(self, tpe: TPEngine, *, capacity: int, blend: CacheBlendConfig | None = None,
                 drafter: TPEagleDrafter | None = None, sink: int = 64, recent: int = 512, chunk: int = 64,
                 budget: int = 2048, document_capacity: int | None = None) -> None:
        self.tpe = tpe
        self.blend = blend or CacheBlendConfig()
        self.drafter = drafter
        self.slot = tpe.new_slot(capacity)
        self.store = DocumentKVStore(tpe.lcfg, tier="hbm", device=tpe.engine.device)
        # producer slot: one document at a time (padded to the TP row multiple)
        doc_cap = tpe.max_rows * tpe.tp if document_capacity is None else \
            -(-int(document_capacity) // (tpe.tp * 128)) * tpe.tp * 128
        self._scratch = tpe.new_slot(doc_cap)
        self.view_args = dict(sink=sink, recent=recent, chunk=chunk, budget=budget)

    # ---------------------------------------------------------- producer
    def encode_local(self, tokens) -> torch.Tensor:
        """TP prefill of one document at positions 0..n-1; this rank's kv heads [L, 2, Hkv/tp, n, D]."""
        n = len(tokens)
        ids = torch.tensor(list(tokens), dtype=torch.int32).to(self.tpe.engine.device)
        self.tpe.prefill(ids, self._scratch)
        return self._scratch.data[:, :, :, :n].clone()

    def produce(self, requests) -> dict:
        return self.store.produce(self.encode_local, [d for r in requests for d in r.documents])

    # ------------------------------------------------------------ serve
    def prefill_request(self, request, *, mode: str = "cacheblend", max_new: int = 128) -> dict:
        """Prompt -> first token (device state for decode).  Returns host metadata."""
        tpe, eng = self.tpe, self.tpe.engine
        T = request.prompt_tokens
        ids = torch.tensor(request.prompt, dtype=torch.int32).to(eng.device, non_blocking=True)
        if mode == "cacheblend":
            blocks = [self.store[d].kv for d in request.documents]
            eng.compose(self.slot, blocks, first_slot=len(request.prefix), layer_begin=self.blend.check_layer)
            x, rows, A, meta = tpe.cacheblend(ids, self.slot, prefix_tokens=len(request.prefix),
                                              suffix_tokens=len(request.suffix), blend=self.blend)
            tpe.first_token(x, rows, T, max_new=max_new, last_row=A - 1)
            return {"active_rows": A, "active": meta["active"]}
        x, rows, _ = tpe.prefill(ids, self.slot)
        tpe.first_token(x, rows, T, max_new=max_new)
        return {"active_rows": T, "active": None}

    def memory_view(self, T: int, active: torch.Tensor | None) -> torch.Tensor:
        """Sink + recent + top 64-token chunks: chunks ranked by CacheBlend recomputed rows (else evenly)."""
        a = self.view_args
        n_chunks = (T + a["chunk"] - 1) // a["chunk"]
        if active is not None:
            scores = torch.bincount((active.long() // a["chunk"]).clamp_max(n_chunks - 1), minlength=n_chunks)
            scores = scores.float().cpu()
        else:
            scores = None
        return sink_recent_topk_indices(T, scores, sink=a["sink"], recent=a["recent"], chunk=a["chunk"],
                                        budget=a["budget"]).to(torch.int32).to(self.tpe.engine.device)

    def decode(self, request, meta: dict, *, max_new: int, speculative: bool) -> dict:
        T = request.prompt_tokens
        if speculative:
            if self.drafter is None:
                raise ValueError("no drafter")
            self.drafter.set_request(self.memory_view(T, meta["active"]), T, max_new=max_new)
            return speculative_generate(self.tpe, self.drafter, self.slot, prompt_tokens=T, max_new=max_new)
        self.tpe.decode(self.slot, max_new - 1)
        return {"tokens": self.tpe.engine.generated_tokens(max_new).tolist(), "accepted": []}


def _max_over_ranks(x: float) -> float:
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _pct(xs, q):
    xs = sorted(xs)
    return xs[min(len(xs) - 1, int(q * len(xs)))]


def main(argv=None) -> None:
    from .tp_bench import random_shard

    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama3-70b")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--workload", default="llama70b_rag")
    p.add_argument("--requests", type=int, default=8)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--new-tokens", type=int, default=128)
    p.add_argument("--gamma", type=int, default=4)
    p.add_argument("--ratio", type=float, default=0.15)
    p.add_argument("--check-layer", type=int, default=1)
    p.add_argument("--no-spec", action="store_true")
    p.add_argument("--batches", default="8,32", help="batched greedy decode sizes (<= 32 sequences)")
    p.add_argument("--model-dir", default=None,
                   help="model directory (HF Llama or this package's): each rank reads only its shard")
    a = p.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    try:
        group = TPGroup()
        tp, rank = group.size, group.rank
        shard = None
        if a.model_dir:
            from ..models.checkpoint import checkpoint_shard

            cfg, shard = checkpoint_shard(a.model_dir, rank, tp, dev)
        else:
            cfg = get_model_config(a.model)
            if a.layers:
                cfg = cfg.with_layers(a.layers)
        reqs = make_requests(a.workload, cfg)[: a.warmup + a.requests]
        T_max = max(r.prompt_tokens for r in reqs)
        doc_max = max(len(d) for r in reqs for d in r.documents)
        rows = (max(T_max, doc_max) + tp * 128) // tp + 128
        weights = shard if shard is not None else random_shard(cfg, rank, tp, 0, dev)
        tpe = TPEngine(cfg, weights, group, max_rows=rows,
                       max_positions=T_max + a.new_tokens + tp * 128 + 1024)
        dcfg = drafter_config_for(cfg)
        drafter = None
        if not a.no_spec:
            drafter = TPEagleDrafter(tpe, dcfg, TPDraftWeights.random(dcfg, rank, tp, 1, dev),
                                     memory_layers=memory_layers_for(cfg.n_layers), gamma=a.gamma,
                                     view_capacity=4096 + a.new_tokens)
        server = TPRAGServer(tpe, capacity=T_max + a.new_tokens + tp * 128 + 64,
                             blend=CacheBlendConfig(check_layer=a.check_layer, recompute_ratio=a.ratio),
                             drafter=drafter, document_capacity=doc_max)
        prod = server.produce(reqs)
        torch.cuda.synchronize()
        res = {"ttft_blend": [], "ttft_full": [], "tpot_greedy": [], "tpot_spec": [], "accepted": [],
               "active_rows": [], "prompt_tokens": [], "spec_equals_greedy": []}
        for i, r in enumerate(reqs):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            row = {}
            for mode in ("full", "cacheblend"):
                dist.barrier()
                torch.cuda.synchronize()
                ev[0].record()
                meta = server.prefill_request(r, mode=mode, max_new=a.new_tokens)
                ev[1].record()
                torch.cuda.synchronize()
                row[mode] = _max_over_ranks(ev[0].elapsed_time(ev[1]))
            # greedy decode from the CacheBlend state
            dist.barrier()
            ev[0].record()
            out_g = server.decode(r, meta, max_new=a.new_tokens, speculative=False)
            ev[1].record()
            torch.cuda.synchronize()
            tg = _max_over_ranks(ev[0].elapsed_time(ev[1]))
            ts, out_s = None, None
            if drafter is not None:
                server.prefill_request(r, mode="cacheblend", max_new=a.new_tokens)
                dist.barrier()
                torch.cuda.synchronize()
                ev[0].record()
                out_s = server.decode(r, meta, max_new=a.new_tokens, speculative=True)
                ev[1].record()
                torch.cuda.synchronize()
                ts = _max_over_ranks(ev[0].elapsed_time(ev[1]))
            tpe.check_status()
            if i < a.warmup:
                continue
            res["ttft_full"].append(row["full"])
            res["ttft_blend"].append(row["cacheblend"])
            res["tpot_greedy"].append(tg / (a.new_tokens - 1))
            res["active_rows"].append(meta["active_rows"])
            res["prompt_tokens"].append(r.prompt_tokens)
            if ts is not None:
                res["tpot_spec"].append(ts / (a.new_tokens - 1))
                res["accepted"].append(out_s["mean_accepted"])
                diff = next((k for k, (x, y) in enumerate(zip(out_s["tokens"], out_g["tokens"])) if x != y), None)
                res["spec_equals_greedy"].append(diff)
        # batched greedy decode: B requests prefilled (CacheBlend) into one batch of slots
        batch_out = {}
        cap = T_max + a.new_tokens + tp * 128 + 64
        for B in [int(x) for x in a.batches.split(",") if x.strip()]:
            if B > tpe.MAX_BATCH:
                continue
            bslots = tpe.batch_slots(B, cap)
            firsts, positions = [], []
            own_slot = server.slot
            # B sequences, the requests taken in turn (each its own slot and CacheBlend prefill)
            for r, sl in zip([reqs[k % len(reqs)] for k in range(B)], bslots):
                server.slot = sl
                server.prefill_request(r, mode="cacheblend", max_new=a.new_tokens)
                firsts.append(int(tpe.engine.generated_tokens(1)[0]))
                positions.append(r.prompt_tokens)
            server.slot = own_slot
            tpe.start_batch(bslots, firsts, positions, max_new=a.new_tokens)
            tpe.decode_batch(bslots, 2)  # capture + warm
            tpe.start_batch(bslots, firsts, positions, max_new=a.new_tokens)
            dist.barrier()
            torch.cuda.synchronize()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            ev[0].record()
            tpe.decode_batch(bslots, a.new_tokens - 1)
            ev[1].record()
            torch.cuda.synchronize()
            ms = _max_over_ranks(ev[0].elapsed_time(ev[1])) / (a.new_tokens - 1)
            tpe.check_status()
            batch_out[str(B)] = {"step_ms": ms, "decode_tokens_per_s": B * 1e3 / ms}
            del bslots
            tpe.engine.release_graphs()
        tpe.engine.release_graphs()
        if drafter is not None:
            drafter._graph = None
        dist.barrier()
        if rank == 0:
            out = {"model": cfg.name, "layers": cfg.n_layers, "tp": tp, "batch": 1, "requests": a.requests,
                   "new_tokens": a.new_tokens, "recompute_ratio": a.ratio, "check_layer": a.check_layer,
                   "producer": {k: v for k, v in prod.items() if isinstance(v, (int, float))},
                   "prompt_tokens_mean": statistics.fmean(res["prompt_tokens"]),
                   "active_rows_mean": statistics.fmean(res["active_rows"]),
                   "ttft_cacheblend_ms": {"p50": _pct(res["ttft_blend"], 0.5), "p99": _pct(res["ttft_blend"], 0.99)},
                   "ttft_full_prefill_ms": {"p50": _pct(res["ttft_full"], 0.5), "p99": _pct(res["ttft_full"], 0.99)},
                   "tpot_greedy_ms": statistics.fmean(res["tpot_greedy"]),
                   "decode_tokens_per_s_greedy": 1e3 / statistics.fmean(res["tpot_greedy"]),
                   "batched_greedy_decode": batch_out}
            if res["tpot_spec"]:
                out.update(tpot_spec_ms=statistics.fmean(res["tpot_spec"]),
                           decode_tokens_per_s_spec=1e3 / statistics.fmean(res["tpot_spec"]),
                           gamma=a.gamma, mean_accepted_drafts=statistics.fmean(res["accepted"]),
                           # the verifier runs on the tensor-core skinny GEMM, the greedy decode on
                           # the GEMV: both greedy, equal up to rounding ties (first differing index)
                           spec_first_difference_vs_decode_path=res["spec_equals_greedy"],
                           drafter="random-init one-layer EAGLE of the target width (acceptance is not meaningful)")
            print(json.dumps(out), flush=True)
        dist.barrier()
        tpe.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
