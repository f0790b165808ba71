"""``sparsecache-precompute``: write the system cache and one KV file per chunk.

Legacy S-conditioned producer (reference src/sparsecache/precompute.py:20-154):
the system prompt is prefilled once; every chunk is prefilled as
system + chunk and only the chunk's KV is kept (``source_start`` = system
length).  Output: ``system.safetensors``, ``chunk_NN.safetensors`` and a
``sparsecache.chunk-kv.v1`` manifest.  ``--producer independent`` instead
prefills every chunk alone at positions 0.. (``source_start`` 0), the
query-agnostic protocol of the reuse pipeline.

``--model`` is a model directory (config.json + model.safetensors);
``--device cpu`` runs the PyTorch oracle, ``cuda:N`` the sm_100a engine.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path
from time import perf_counter

import torch

from .data import load_prepared_case
from .models.checkpoint import load_config, load_oracle
from .prompting import tokenize_case
from .store import MANIFEST_FORMAT, model_fingerprint, save_cache
from .tokenizer import load_tokenizer


def _encoder(model_dir: str, device: str, dtype: torch.dtype):
    """Return prefill(ids) -> legacy cache [(k [1,H,T,D], v)] on CPU."""
    if device.startswith("cuda"):
        from .models.engine import B200Engine, KVSlot

        oracle = load_oracle(model_dir, dtype=torch.float32)
        engine = B200Engine.from_oracle(oracle, device)
        del oracle

        def prefill(ids):
            slot = KVSlot(engine.cfg, len(ids), engine.device)
            engine.prefill(torch.tensor(ids, dtype=torch.int32, device=engine.device), slot)
            kv = slot.data.cpu()
            return tuple((kv[i, 0].unsqueeze(0), kv[i, 1].unsqueeze(0)) for i in range(kv.shape[0]))

        return prefill
    model = load_oracle(model_dir, dtype=dtype)

    def prefill(ids):
        _, cache = model.prefill(ids)
        return tuple((k.to(torch.bfloat16), v.to(torch.bfloat16)) for k, v in cache)

    return prefill


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(description="Precompute reusable chunk KV caches")
    parser.add_argument("--case", required=True)
    parser.add_argument("--model", required=True)
    parser.add_argument("--output-dir", required=True)
    parser.add_argument("--device", default="cuda:0")
    parser.add_argument("--dtype", choices=("bfloat16", "float16", "float32"), default="bfloat16")
    parser.add_argument("--producer", choices=("system-conditioned", "independent"), default="system-conditioned")
    parser.add_argument("--expected-chunks", type=int, default=10)
    parser.add_argument("--overwrite", action="store_true")
    args = parser.parse_args(argv)
    out_dir = Path(args.output_dir)
    manifest_path = out_dir / "manifest.json"
    if manifest_path.exists() and not args.overwrite:
        raise FileExistsError(f"{manifest_path} already exists; pass --overwrite to replace it")
    out_dir.mkdir(parents=True, exist_ok=True)
    cfg = load_config(args.model)
    case = load_prepared_case(args.case)
    tokenizer = load_tokenizer(args.model, cfg.vocab, cfg.n_special, cfg.eos_token_ids)
    prompt = tokenize_case(tokenizer, case)
    if args.expected_chunks and len(prompt.chunks) != args.expected_chunks:
        raise ValueError(f"the producer expects {args.expected_chunks} chunks, got {len(prompt.chunks)}")
    prefill = _encoder(args.model, args.device, getattr(torch, args.dtype))
    started = perf_counter()
    S = len(prompt.system_ids)
    system_cache = prefill(prompt.system_ids)
    system_bytes = save_cache(out_dir / "system.safetensors", system_cache)
    rows = []
    for index, (chunk_id, title, ids) in enumerate(prompt.chunks):
        t0 = perf_counter()
        if args.producer == "system-conditioned":
            cache = prefill(prompt.system_ids + ids)
            cache = tuple((k[:, :, S:].contiguous(), v[:, :, S:].contiguous()) for k, v in cache)
            source_start = S
        else:
            cache = prefill(ids)
            source_start = 0
        name = f"chunk_{index:02d}.safetensors"
        nbytes = save_cache(out_dir / name, cache)
        rows.append({"chunk_id": chunk_id, "title": title, "file": name, "source_start": source_start,
                     "tokens": len(ids), "token_ids": list(ids), "kv_bytes": nbytes,
                     "producer_ms": (perf_counter() - t0) * 1000})
        print(json.dumps({"event": "chunk_saved", "index": index, "title": title, "tokens": len(ids),
                          "kv_bytes": nbytes}, ensure_ascii=False), flush=True)
    manifest = {
        "format": MANIFEST_FORMAT,
        "producer": "independent-system-conditioned" if args.producer == "system-conditioned" else "independent-local",
        "model": {"path": str(Path(args.model).resolve()), "fingerprint": model_fingerprint(args.model),
                  "dtype": args.dtype, "layers": cfg.n_layers, "attention_heads": cfg.n_heads,
                  "kv_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim},
        "case": case.as_dict(),
        "system": {"file": "system.safetensors", "tokens": S, "token_ids": list(prompt.system_ids),
                   "kv_bytes": system_bytes},
        "chunks": rows,
        "online_suffix": {"tokens": len(prompt.suffix_ids), "token_ids": list(prompt.suffix_ids)},
        "full_prompt_tokens": len(prompt.full_ids),
        "document_tokens": len(prompt.document_ids),
        "total_kv_bytes": system_bytes + sum(r["kv_bytes"] for r in rows),
        "producer_wall_ms": (perf_counter() - started) * 1000,
    }
    manifest_path.write_text(json.dumps(manifest, ensure_ascii=False, indent=2) + "\n", encoding="utf-8")
    print(json.dumps({"event": "complete", "manifest": str(manifest_path)}), flush=True)


if __name__ == "__main__":
    main()
