"""``sparsecache-qa``: answer one prepared case from its chunk caches, mode by mode.

Inputs are a ``sparsecache.chunk-kv.v1`` manifest (written by
``sparsecache-precompute``) and the model directory it names.  The chunk
caches are composed once (keys moved to their positions in the full prompt);
then every requested mode answers the question:

  baseline    full prefill of the whole prompt
  direct      the composed cache reused as-is, only the question suffix prefilled
  cacheblend  selective recompute against the composed cache

Each answer is cleaned and scored (EM / token F1 against the case's gold
answers) and a results JSON is written.  The manifest's model fingerprint
must match the model directory.  The field names of the printed events and
of the results file follow the reference's consumer
(src/sparsecache/qa.py:20-160) so downstream scripts read either.

On ``--device cuda:N`` the modes run on the sm_100a engine; on ``cpu`` on the
fp32 PyTorch oracle.
"""
from __future__ import annotations

import argparse
import gc
import json
from dataclasses import dataclass
from pathlib import Path
from time import perf_counter
from typing import Any, Callable

import torch

from .metrics import answer_em, answer_f1, clean_short_answer
from .modeling import GenerationResult, baseline_generate, cacheblend_generate, direct_reuse_generate
from .models.checkpoint import load_config, load_oracle
from .store import cache_bytes, compose_cache, load_manifest, model_fingerprint
from .tokenizer import load_tokenizer

MODES = ("baseline", "direct", "cacheblend")


@dataclass
class ComposedCase:
    """A manifest's prompt segments and its composed prefix cache."""

    manifest_path: Path
    manifest: dict[str, Any]
    config: Any
    prefix_cache: Any
    layout: dict[str, Any]
    compose_ms: float

    @classmethod
    def open(cls, manifest_path: str | Path) -> "ComposedCase":
        manifest = load_manifest(manifest_path)
        model = manifest["model"]
        if model_fingerprint(model["path"]) != model["fingerprint"]:
            raise RuntimeError("model files do not match the cache manifest")
        cfg = load_config(model["path"])
        t0 = perf_counter()
        prefix_cache, layout = compose_cache(cfg, manifest)
        return cls(Path(manifest_path), manifest, cfg, prefix_cache, layout, (perf_counter() - t0) * 1000)

    @property
    def model_path(self) -> str:
        return self.manifest["model"]["path"]

    @property
    def case(self) -> dict[str, Any]:
        return self.manifest["case"]

    def _ids(self, segment: dict) -> tuple[int, ...]:
        return tuple(int(t) for t in segment["token_ids"])

    @property
    def system_ids(self) -> tuple[int, ...]:
        return self._ids(self.manifest["system"])

    @property
    def suffix_ids(self) -> tuple[int, ...]:
        return self._ids(self.manifest["online_suffix"])

    @property
    def full_ids(self) -> tuple[int, ...]:
        docs = tuple(t for c in self.manifest["chunks"] for t in self._ids(c))
        return self.system_ids + docs + self.suffix_ids


def load_model(case: ComposedCase, device: str):
    """The sm_100a engine on a CUDA device, the fp32 oracle otherwise."""
    oracle = load_oracle(case.model_path, dtype=torch.float32)
    if device.startswith("cuda"):
        from .models.engine import B200Engine

        return B200Engine.from_oracle(oracle, device)
    return oracle


def mode_runners(args: argparse.Namespace) -> dict[str, Callable[[Any, ComposedCase, set], GenerationResult]]:
    n = args.max_new_tokens
    return {
        "baseline": lambda m, c, eos: baseline_generate(m, full_ids=c.full_ids, max_new_tokens=n, eos_token_ids=eos),
        "direct": lambda m, c, eos: direct_reuse_generate(m, prefix_cache=c.prefix_cache, suffix_ids=c.suffix_ids,
                                                          max_new_tokens=n, eos_token_ids=eos),
        "cacheblend": lambda m, c, eos: cacheblend_generate(
            m, full_ids=c.full_ids, prefix_cache=c.prefix_cache, system_tokens=c.layout["system_tokens"],
            suffix_tokens=len(c.suffix_ids), check_layer=args.check_layer, recompute_ratio=args.recompute_ratio,
            max_new_tokens=n, eos_token_ids=eos, deviation_metric=args.deviation_metric,
            keep_prefix=args.keep_prefix),
    }


def scored_row(mode: str, result: GenerationResult, case: dict[str, Any], tokenizer) -> dict[str, Any]:
    answer = clean_short_answer(tokenizer.decode(result.token_ids, skip_special_tokens=False))
    gold = case["answers"]
    return {"mode": mode, "question": case["question"], "gold_answers": gold, "answer": answer,
            "token_ids": list(result.token_ids), "em": answer_em(answer, gold), "f1": answer_f1(answer, gold),
            "prefill_ms": result.prefill_ms, "decode_ms": result.decode_ms, "metadata": result.metadata}


def run(args: argparse.Namespace) -> dict[str, Any]:
    composed = ComposedCase.open(args.manifest)
    cfg = composed.config
    tokenizer = load_tokenizer(composed.model_path, cfg.vocab, cfg.n_special, cfg.eos_token_ids)
    model = load_model(composed, args.device)
    runners = mode_runners(args)
    eos = set(cfg.eos_token_ids)
    rows = []
    for mode in args.modes:
        row = scored_row(mode, runners[mode](model, composed, eos), composed.case, tokenizer)
        rows.append(row)
        print(json.dumps({"event": "qa", **row}, ensure_ascii=False, default=str), flush=True)
        gc.collect()
    layout = composed.layout
    return {"manifest": str(composed.manifest_path.resolve()), "model": composed.model_path,
            "case_id": composed.case["case_id"], "chunks": len(composed.manifest["chunks"]),
            "system_tokens": layout["system_tokens"], "document_tokens": layout["document_tokens"],
            "suffix_tokens": len(composed.suffix_ids), "relocated_tokens": layout["relocated_tokens"],
            "prefix_kv_bytes": cache_bytes(composed.prefix_cache), "compose_ms": composed.compose_ms,
            "results": rows}


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(description="Answer a prepared case from its chunk caches")
    parser.add_argument("--manifest", required=True)
    parser.add_argument("--output", required=True)
    parser.add_argument("--modes", nargs="+", choices=MODES, default=("direct", "cacheblend"))
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
    report = run(args)
    target = Path(args.output)
    target.parent.mkdir(parents=True, exist_ok=True)
    target.write_text(json.dumps(report, ensure_ascii=False, indent=2, default=str) + "\n", encoding="utf-8")
    print(json.dumps({"event": "complete", "output": str(target)}), flush=True)


if __name__ == "__main__":
    main()
