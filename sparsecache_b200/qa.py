"""``sparsecache-qa``: compose a manifest's cache and answer with baseline / direct / CacheBlend.

Reference src/sparsecache/qa.py:20-160: the manifest fingerprint must match
the model directory, the composed cache is built once (chunk keys relocated
to their target positions), every requested mode is run and scored with
EM / F1, and a results JSON is written.
"""
from __future__ import annotations

import argparse
import gc
import json
from pathlib import Path
from time import perf_counter

import torch

from .metrics import answer_em, answer_f1, clean_short_answer
from .modeling import baseline_generate, cacheblend_generate, direct_reuse_generate
from .models.checkpoint import load_config, load_oracle
from .store import cache_bytes, compose_cache, load_manifest, model_fingerprint
from .tokenizer import load_tokenizer


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(description="Run paired QA modes over a composed chunk cache")
    parser.add_argument("--manifest", required=True)
    parser.add_argument("--output", required=True)
    parser.add_argument("--modes", nargs="+", choices=("baseline", "direct", "cacheblend"),
                        default=("direct", "cacheblend"))
    parser.add_argument("--device", default="cuda:0")
    parser.add_argument("--max-new-tokens", type=int, default=16)
    parser.add_argument("--check-layer", type=int, default=1)
    parser.add_argument("--recompute-ratio", type=float, default=0.15)
    parser.add_argument("--deviation-metric", default="key",
                        choices=("value", "key", "kv", "value_l1", "key_l1", "kv_l1"))
    parser.add_argument("--keep-prefix", action="store_true",
                        help="treat the system prefix as mandatory active rows (strict protocol)")
    args = parser.parse_args(argv)
    if args.max_new_tokens < 1:
        parser.error("max-new-tokens must be positive")
    manifest = load_manifest(args.manifest)
    model_path = manifest["model"]["path"]
    if model_fingerprint(model_path) != manifest["model"]["fingerprint"]:
        raise RuntimeError("model files do not match the cache manifest")
    cfg = load_config(model_path)
    tokenizer = load_tokenizer(model_path, cfg.vocab, cfg.n_special, cfg.eos_token_ids)
    if args.device.startswith("cuda"):
        from .models.engine import B200Engine

        model = B200Engine.from_oracle(load_oracle(model_path), args.device)
    else:
        model = load_oracle(model_path, dtype=torch.float32)
    t0 = perf_counter()
    prefix_cache, layout = compose_cache(cfg, manifest)
    compose_ms = (perf_counter() - t0) * 1000
    system_ids = tuple(int(x) for x in manifest["system"]["token_ids"])
    document_ids = tuple(int(t) for c in manifest["chunks"] for t in c["token_ids"])
    suffix_ids = tuple(int(x) for x in manifest["online_suffix"]["token_ids"])
    full_ids = system_ids + document_ids + suffix_ids
    eos = set(cfg.eos_token_ids)
    case = manifest["case"]
    rows = []
    for mode in args.modes:
        if mode == "baseline":
            result = baseline_generate(model, full_ids=full_ids, max_new_tokens=args.max_new_tokens,
                                       eos_token_ids=eos)
        elif mode == "direct":
            result = direct_reuse_generate(model, prefix_cache=prefix_cache, suffix_ids=suffix_ids,
                                           max_new_tokens=args.max_new_tokens, eos_token_ids=eos)
        else:
            result = cacheblend_generate(
                model, full_ids=full_ids, prefix_cache=prefix_cache, system_tokens=layout["system_tokens"],
                suffix_tokens=len(suffix_ids), check_layer=args.check_layer,
                recompute_ratio=args.recompute_ratio, max_new_tokens=args.max_new_tokens, eos_token_ids=eos,
                deviation_metric=args.deviation_metric, keep_prefix=args.keep_prefix)
        text = clean_short_answer(tokenizer.decode(result.token_ids, skip_special_tokens=False))
        row = {"mode": mode, "question": case["question"], "gold_answers": case["answers"], "answer": text,
               "token_ids": list(result.token_ids), "em": answer_em(text, case["answers"]),
               "f1": answer_f1(text, case["answers"]), "prefill_ms": result.prefill_ms,
               "decode_ms": result.decode_ms, "metadata": result.metadata}
        rows.append(row)
        print(json.dumps({"event": "qa", **row}, ensure_ascii=False, default=str), flush=True)
        gc.collect()
    out = {"manifest": str(Path(args.manifest).resolve()), "model": model_path, "case_id": case["case_id"],
           "chunks": len(manifest["chunks"]), "system_tokens": layout["system_tokens"],
           "document_tokens": layout["document_tokens"], "suffix_tokens": len(suffix_ids),
           "relocated_tokens": layout["relocated_tokens"], "prefix_kv_bytes": cache_bytes(prefix_cache),
           "compose_ms": compose_ms, "results": rows}
    path = Path(args.output)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(out, ensure_ascii=False, indent=2, default=str) + "\n", encoding="utf-8")
    print(json.dumps({"event": "complete", "output": str(path)}), flush=True)


if __name__ == "__main__":
    main()
