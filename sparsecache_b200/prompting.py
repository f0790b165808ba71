"""Stable prompt assembly for independently precomputed document chunks.

The chat template is rendered once with a placeholder where the documents go;
the text before it becomes the system ids, the text after it the online
question suffix, and every chunk is tokenised on its own so its boundaries
(and therefore its reusable KV) are stable across requests
(reference src/sparsecache/prompting.py).
"""
from __future__ import annotations

from dataclasses import dataclass

from .data import QACase

PLACEHOLDER = "<|SPARSECACHE_DOCUMENTS|>"
SYSTEM_INSTRUCTION = (
    "You are a careful question-answering assistant. Answer the user's question "
    "using the supplied documents. Return only the exact short answer without "
    "explanation."
)


@dataclass(frozen=True)
class TokenizedPrompt:
    system_ids: tuple[int, ...]
    chunks: tuple[tuple[str, str, tuple[int, ...]], ...]
    suffix_ids: tuple[int, ...]

    @property
    def document_ids(self) -> tuple[int, ...]:
        return tuple(t for _, _, ids in self.chunks for t in ids)

    @property
    def full_ids(self) -> tuple[int, ...]:
        return self.system_ids + self.document_ids + self.suffix_ids


def tokenize_case(tokenizer, case: QACase) -> TokenizedPrompt:
    user = (
        f"<DOCUMENTS>\n{PLACEHOLDER}\n</DOCUMENTS>\n\n"
        f"Question: {case.question.strip()}\n"
        "Return only the exact short answer without explanation."
    )
    rendered = tokenizer.apply_chat_template(
        [{"role": "system", "content": SYSTEM_INSTRUCTION}, {"role": "user", "content": user}],
        tokenize=False,
        add_generation_prompt=True,
    )
    pivot = rendered.index(PLACEHOLDER)
    system_ids = tokenizer.encode(rendered[:pivot], add_special_tokens=True)
    suffix_ids = tokenizer.encode(rendered[pivot + len(PLACEHOLDER):], add_special_tokens=False)
    chunks = []
    for i, chunk in enumerate(case.chunks, 1):
        text = f"Document {i}: {chunk.title}\n{chunk.text.strip()}\n"
        ids = tokenizer.encode(text, add_special_tokens=False)
        chunks.append((chunk.chunk_id, chunk.title, tuple(int(x) for x in ids)))
    return TokenizedPrompt(
        system_ids=tuple(int(x) for x in system_ids),
        chunks=tuple(chunks),
        suffix_ids=tuple(int(x) for x in suffix_ids),
    )
