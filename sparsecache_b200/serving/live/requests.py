"""Fixed-length token-id requests for the live P/D gate.

Counterpart of the reference's experiments/build_progressive_pd_live_requests.py:
every request is a streaming completion of exactly ``prompt_tokens`` prompt
ids built from a normalised RULER qa_2 row: the chat prompt rendered around
the documents in the chosen placement, every supporting document kept whole
and the distractors trimmed proportionally (at least one token each) to fill
the budget exactly.  Rows too short to fill the budget, or whose evidence
alone overflows it, are skipped and counted.  Output is fixed-horizon
(``ignore_eos``) so every arm decodes the same number of tokens.

    python -m sparsecache_b200.serving.live.requests --dataset N/qa2_16384.jsonl --tokenizer M \\
        --output live/requests.jsonl --prompt-tokens 8192 --num-requests 104
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Any, Sequence

from ...evaluation.ruler import allocate_trim_lengths, render_parts


def live_prompt(tokenizer, row: dict[str, Any], placement: str, prompt_tokens: int) -> list[int] | None:
    """Exactly ``prompt_tokens`` ids for ``row``, or None when the row cannot fill the budget by trimming."""
    prefix, docs, suffix = render_parts(tokenizer, row, placement)
    budget = prompt_tokens - len(prefix) - len(suffix)
    if budget <= 0:
        raise ValueError("the prompt target leaves no room for documents")
    if sum(len(d["token_ids"]) for d in docs) < budget:
        return None
    try:
        lengths = allocate_trim_lengths(docs, budget)
    except ValueError:
        return None
    prompt = list(prefix) + [t for d, k in zip(docs, lengths) for t in d["token_ids"][:k]] + list(suffix)
    if len(prompt) != prompt_tokens:
        raise AssertionError("the built prompt is not of the requested length")
    return prompt


def build_live_requests(tokenizer, rows: Sequence[dict], *, placement: str, prompt_tokens: int, max_tokens: int,
                        num_requests: int, served_model_name: str) -> tuple[list[dict], int]:
    """(requests, rows skipped) in dataset order until ``num_requests`` fit."""
    if prompt_tokens <= 0 or prompt_tokens % 256:
        raise ValueError("prompt_tokens must be a positive multiple of 256")
    if max_tokens <= 0 or num_requests <= 0:
        raise ValueError("request and output counts must be positive")
    out, skipped = [], 0
    for row in rows:
        prompt = live_prompt(tokenizer, row, placement, prompt_tokens)
        if prompt is None:
            skipped += 1
            continue
        out.append({"model": served_model_name, "prompt": prompt, "max_tokens": max_tokens, "temperature": 0,
                    "ignore_eos": True, "stream": True, "return_token_ids": True})
        if len(out) == num_requests:
            break
    if len(out) < num_requests:
        raise ValueError(f"only {len(out)} rows fit exactly; {num_requests} requested")
    return out, skipped


def main(argv=None) -> dict[str, Any]:
    from ...evaluation.cli import _tokenizer

    p = argparse.ArgumentParser()
    p.add_argument("--dataset", type=Path, required=True)
    p.add_argument("--tokenizer", required=True)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--served-model-name", default="sparsecache-llama31-8b")
    p.add_argument("--placement", default="evidence_first")
    p.add_argument("--prompt-tokens", type=int, default=8192)
    p.add_argument("--max-tokens", type=int, default=32)
    p.add_argument("--num-requests", type=int, default=104)
    a = p.parse_args(argv)
    if a.output.exists():
        raise FileExistsError(f"refusing to overwrite {a.output}")
    rows = [json.loads(x) for x in a.dataset.read_text(encoding="utf-8").splitlines() if x.strip()]
    reqs, skipped = build_live_requests(_tokenizer(a.tokenizer), rows, placement=a.placement,
                                        prompt_tokens=a.prompt_tokens, max_tokens=a.max_tokens,
                                        num_requests=a.num_requests, served_model_name=a.served_model_name)
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text("".join(json.dumps(r) + "\n" for r in reqs), encoding="utf-8")
    summary = {"output": str(a.output), "requests": len(reqs), "skipped_short_or_infeasible": skipped,
               "prompt_tokens": a.prompt_tokens, "placement": a.placement}
    print(json.dumps(summary, indent=2))
    return summary


if __name__ == "__main__":
    main()
