"""Small, self-contained serving case for kernel profiling and phase timing.

    python -m sparsecache_b200.utils.profile_case --model llama3-8b --new-tokens 4

Builds a random-init engine, produces the documents of ``--requests``
synthetic requests, serves them ``--warmup`` times, then serves one request
inside an NVTX range named ``profile`` (so ``ncu --nvtx --nvtx-include
profile/`` captures only that request) and prints CUDA-event timings.
The device working set is the model plus one request's cache.
"""
from __future__ import annotations

import argparse
import json

import torch

from ..config import CacheBlendConfig, get_model_config
from ..models.engine import B200Engine
from ..serving.server import RAGServer
from ..store import DocumentKVStore
from ..synthetic import make_requests


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--mode", default="cacheblend", choices=("cacheblend", "full", "direct"))
    p.add_argument("--requests", type=int, default=1)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--new-tokens", type=int, default=24)
    p.add_argument("--ratio", type=float, default=0.15)
    p.add_argument("--batch", type=int, default=0, help="> 0: profile serve_batch of this many requests")
    args = p.parse_args()
    cfg = get_model_config(args.model)
    if args.layers:
        cfg = cfg.with_layers(args.layers)
    dev = torch.device("cuda:0")
    engine = B200Engine.random(cfg, seed=0, device=dev)
    requests = make_requests("llama8b_rag", cfg)[: max(args.requests, args.batch)]
    store = DocumentKVStore(cfg, tier="hbm", device=dev)
    blend = CacheBlendConfig(recompute_ratio=args.ratio, max_new_tokens=args.new_tokens)
    server = RAGServer(engine, store, capacity=max(r.prompt_tokens for r in requests) + args.new_tokens + 64,
                       blend=blend)
    server.produce(requests)
    if args.batch > 0:
        batch = requests[: args.batch]
        for _ in range(args.warmup):
            server.serve_batch(batch)
        torch.cuda.synchronize()
        launches = engine.ext.launches
        torch.cuda.nvtx.range_push("profile")
        res = server.serve_batch(batch)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        print(json.dumps({"mode": "batch", "batch": args.batch, "batch_ms": res.response_ms,
                          "decode_step_ms": res.decode_step_ms, "first_tokens_ms": res.metadata["first_tokens_ms"],
                          "launches": engine.ext.launches - launches}))
        return
    for _ in range(args.warmup):
        server.serve(requests[0], mode=args.mode, sync=True)
    torch.cuda.synchronize()
    launches = engine.ext.launches
    torch.cuda.nvtx.range_push("profile")
    res = server.serve(requests[0], mode=args.mode, sync=True)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(json.dumps({"mode": args.mode, "prompt_tokens": requests[0].prompt_tokens, "ttft_ms": res.ttft_ms,
                      "response_ms": res.response_ms,
                      "tpot_ms": res.decode_ms / max(1, args.new_tokens - 1),
                      "launches": engine.ext.launches - launches, "tokens": list(res.token_ids)}))


if __name__ == "__main__":
    main()
