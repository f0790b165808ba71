"""Seeded synthetic RAG workloads (no datasets are downloaded).

Each request is a system prefix, an ordered list of documents and a question
suffix, all as token ids drawn uniformly from the non-special vocabulary.
A fixed number (or fraction) of document slots are exact repeats of earlier
documents, which the deduplicating store turns into cache hits.

Workloads:
  * ``tiny_plumbing``  8 samples x 10 docs, lengths ~U[60, 180], 20% of slots
                       repeated, system 16, question ~U[10, 30];
  * ``llama8b_rag``    150 samples x 10 docs = 1,500 uses of 1,255 unique
                       sequences (245 exact repeats), lengths ~N(160, 50)
                       clipped to [40, 400], system 32, question ~U[12, 40];
  * ``long_rag``       10 docs summing to a log-uniform total (8k-32k or
                       4k-16k tokens), for the P/D and 70B serving cases.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass, field

from .config import ModelConfig


@dataclass(frozen=True)
class RAGRequest:
    index: int
    prefix: tuple[int, ...]
    documents: tuple[tuple[int, ...], ...]
    suffix: tuple[int, ...]

    @property
    def document_tokens(self) -> int:
        return sum(len(d) for d in self.documents)

    @property
    def prompt(self) -> tuple[int, ...]:
        out = self.prefix
        for d in self.documents:
            out += d
        return out + self.suffix

    @property
    def prompt_tokens(self) -> int:
        return len(self.prefix) + self.document_tokens + len(self.suffix)

    def document_ranges(self) -> list[tuple[int, int]]:
        cursor = len(self.prefix)
        out = []
        for d in self.documents:
            out.append((cursor, cursor + len(d)))
            cursor += len(d)
        return out


@dataclass(frozen=True)
class WorkloadSpec:
    n_samples: int
    docs_per_sample: int
    doc_len: tuple[str, float, float, int, int]  # (dist, a, b, lo, hi)
    system_tokens: int
    question: tuple[int, int]
    repeat_uses: int | None = None      # exact number of repeated slots
    repeat_fraction: float | None = None
    total_tokens: tuple[int, int] | None = None  # log-uniform total doc tokens
    seed: int = 0
    extra: dict = field(default_factory=dict)


WORKLOADS = {
    "tiny_plumbing": WorkloadSpec(8, 10, ("uniform", 60, 180, 60, 180), 16, (10, 30), repeat_fraction=0.2),
    "llama8b_rag": WorkloadSpec(150, 10, ("normal", 160, 50, 40, 400), 32, (12, 40), repeat_uses=245),
    "pd_long": WorkloadSpec(64, 10, ("share", 0, 0, 1, 1 << 30), 32, (12, 40), repeat_fraction=0.3,
                            total_tokens=(8192, 32768)),
    "llama70b_rag": WorkloadSpec(64, 10, ("share", 0, 0, 1, 1 << 30), 32, (12, 40), repeat_fraction=0.16,
                                 total_tokens=(4096, 16384)),
}


def token_range(config: ModelConfig) -> tuple[int, int]:
    """[low, high) of ids treated as ordinary text tokens."""
    high = config.vocab
    if config.vocab == 128256:  # Llama 3: ids >= 128000 are special
        high = 128000
    return config.n_special, high


def make_requests(spec: WorkloadSpec | str, config: ModelConfig, *, seed: int | None = None) -> list[RAGRequest]:
    if isinstance(spec, str):
        spec = WORKLOADS[spec]
    rng = random.Random(spec.seed if seed is None else seed)
    lo, hi = token_range(config)

    def ids(n: int) -> tuple[int, ...]:
        return tuple(rng.randrange(lo, hi) for _ in range(n))

    def doc_length() -> int:
        dist, a, b, mn, mx = spec.doc_len
        if dist == "uniform":
            n = rng.randint(int(a), int(b))
        else:
            n = int(round(rng.gauss(a, b)))
        return max(mn, min(mx, n))

    n_slots = spec.n_samples * spec.docs_per_sample
    n_repeats = spec.repeat_uses
    if n_repeats is None:
        n_repeats = int(round((spec.repeat_fraction or 0.0) * n_slots))
    repeats = set(rng.sample(range(1, n_slots), min(n_repeats, n_slots - 1)))
    unique: list[tuple[int, ...]] = []
    requests = []
    slot = 0
    for index in range(spec.n_samples):
        lengths = None
        if spec.total_tokens is not None:
            lo_t, hi_t = spec.total_tokens
            total = int(round(math.exp(rng.uniform(math.log(lo_t), math.log(hi_t)))))
            weights = [rng.uniform(0.5, 1.5) for _ in range(spec.docs_per_sample)]
            scale = total / sum(weights)
            lengths = [max(1, int(w * scale)) for w in weights]
            lengths[-1] += total - sum(lengths)
        docs = []
        for j in range(spec.docs_per_sample):
            if slot in repeats and unique:
                docs.append(unique[rng.randrange(len(unique))])
            else:
                doc = ids(lengths[j] if lengths else doc_length())
                unique.append(doc)
                docs.append(doc)
            slot += 1
        qlen = rng.randint(*spec.question)
        requests.append(RAGRequest(index, ids(spec.system_tokens), tuple(docs), ids(qlen)))
    return requests


def workload_summary(requests: list[RAGRequest]) -> dict:
    uses = [d for r in requests for d in r.documents]
    return {
        "requests": len(requests),
        "document_uses": len(uses),
        "unique_documents": len(set(uses)),
        "repeated_uses": len(uses) - len(set(uses)),
        "mean_prompt_tokens": sum(r.prompt_tokens for r in requests) / max(1, len(requests)),
        "mean_document_tokens": sum(r.document_tokens for r in requests) / max(1, len(requests)),
    }
