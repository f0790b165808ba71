"""Prompt assembly that keeps every document chunk's tokens independent.

A chunk's cached KV can only be reused if the chunk tokenises to the same ids
wherever it appears.  So the chat template is rendered ONCE per question with
a placeholder where the documents go, and the prompt is cut into three kinds
of segment that are tokenised separately:

  head    template text before the placeholder (system message, BOS added)
  chunks  "Document {k}: {title}\\n{text}\\n" for k = 1.. (no special tokens)
  tail    template text after the placeholder (question + generation prompt)

The template strings, the placeholder and the chunk text format are the
reference's (src/sparsecache/prompting.py) on purpose: the same case must
give the same token ids in either implementation, or caches produced by one
would not serve the other.
"""
from __future__ import annotations

from dataclasses import dataclass
from itertools import accumulate, chain

from .data import DocumentChunk, QACase

PLACEHOLDER = "<|SPARSECACHE_DOCUMENTS|>"
SYSTEM_INSTRUCTION = (
    "You are a careful question-answering assistant. Answer the user's question "
    "using the supplied documents. Return only the exact short answer without "
    "explanation."
)
USER_TEMPLATE = (
    "<DOCUMENTS>\n{placeholder}\n</DOCUMENTS>\n\n"
    "Question: {question}\n"
    "Return only the exact short answer without explanation."
)
CHUNK_TEMPLATE = "Document {position}: {title}\n{text}\n"


@dataclass(frozen=True)
class TokenizedPrompt:
    """Segment token ids; ``chunks`` holds (chunk_id, title, ids) per document."""

    system_ids: tuple[int, ...]
    chunks: tuple[tuple[str, str, tuple[int, ...]], ...]
    suffix_ids: tuple[int, ...]

    @property
    def document_ids(self) -> tuple[int, ...]:
        return tuple(chain.from_iterable(ids for _, _, ids in self.chunks))

    @property
    def full_ids(self) -> tuple[int, ...]:
        return self.system_ids + self.document_ids + self.suffix_ids

    def chunk_spans(self) -> list[tuple[int, int]]:
        """[start, end) of every chunk in the full prompt (its target positions)."""
        ends = list(accumulate((len(ids) for _, _, ids in self.chunks), initial=len(self.system_ids)))
        return list(zip(ends[:-1], ends[1:]))


class PromptAssembler:
    """Render-once, tokenise-per-segment prompt builder for one tokenizer."""

    def __init__(self, tokenizer) -> None:
        self.tok = tokenizer

    def frame(self, question: str) -> tuple[str, str]:
        """(head text, tail text) around the placeholder for ``question``."""
        messages = [
            {"role": "system", "content": SYSTEM_INSTRUCTION},
            {"role": "user", "content": USER_TEMPLATE.format(placeholder=PLACEHOLDER, question=question.strip())},
        ]
        rendered = self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)
        head, sep, tail = rendered.partition(PLACEHOLDER)
        if not sep:
            raise ValueError("the chat template dropped the document placeholder")
        return head, tail

    def encode(self, text: str, *, special: bool) -> tuple[int, ...]:
        return tuple(int(t) for t in self.tok.encode(text, add_special_tokens=special))

    def chunk_ids(self, position: int, chunk: DocumentChunk) -> tuple[int, ...]:
        return self.encode(CHUNK_TEMPLATE.format(position=position, title=chunk.title, text=chunk.text.strip()),
                           special=False)

    def assemble(self, case: QACase) -> TokenizedPrompt:
        head, tail = self.frame(case.question)
        docs = tuple((c.chunk_id, c.title, self.chunk_ids(k, c)) for k, c in enumerate(case.chunks, 1))
        return TokenizedPrompt(self.encode(head, special=True), docs, self.encode(tail, special=False))


def tokenize_case(tokenizer, case: QACase) -> TokenizedPrompt:
    """Token ids of ``case`` as system / per-chunk / suffix segments."""
    return PromptAssembler(tokenizer).assemble(case)
