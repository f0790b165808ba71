"""Tokenizer loading for the CLIs.

A model directory may carry an HF tokenizer (tokenizer.json /
tokenizer_config.json), which is loaded with ``local_files_only``.  Without one
(random-init models, tests) a deterministic byte-level tokenizer with a small
Llama-3-style chat template is used, so the CLI pipeline runs end to end with
no downloads.
"""
from __future__ import annotations

from pathlib import Path


class ByteTokenizer:
    """UTF-8 bytes shifted past ``n_special`` reserved ids; ids wrap into the vocab."""

    def __init__(self, vocab: int, n_special: int = 4, bos_token_id: int = 1, eos_token_id: int = 2) -> None:
        if vocab < n_special + 256:
            raise ValueError("vocabulary too small for a byte tokenizer")
        self.vocab = vocab
        self.n_special = n_special
        self.bos_token_id = bos_token_id
        self.eos_token_id = eos_token_id

    def encode(self, text: str, add_special_tokens: bool = True) -> list[int]:
        ids = [self.n_special + b for b in text.encode("utf-8")]
        return ([self.bos_token_id] if add_special_tokens else []) + ids

    def decode(self, ids, skip_special_tokens: bool = False) -> str:
        out = bytearray()
        for i in ids:
            i = int(i)
            if self.n_special <= i < self.n_special + 256:
                out.append(i - self.n_special)
            elif not skip_special_tokens and i == self.eos_token_id:
                out.extend(b"<|eot_id|>")
        return out.decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, tokenize: bool = False, add_generation_prompt: bool = True):
        parts = []
        for m in messages:
            parts.append(f"<|start_header_id|>{m['role']}<|end_header_id|>\n\n{m['content']}<|eot_id|>")
        if add_generation_prompt:
            parts.append("<|start_header_id|>assistant<|end_header_id|>\n\n")
        text = "".join(parts)
        return self.encode(text) if tokenize else text


def load_tokenizer(model_dir: str | Path, vocab: int, n_special: int = 4, eos: tuple[int, ...] = (2,)):
    root = Path(model_dir)
    if (root / "tokenizer.json").exists() or (root / "tokenizer_config.json").exists():
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(str(root), local_files_only=True)
    return ByteTokenizer(vocab, n_special=max(n_special, 4), eos_token_id=eos[0] if eos else 2)
