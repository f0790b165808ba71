"""Short-answer metrics (SQuAD-style normalisation, EM, token F1, answer cleaning).

Reference: src/sparsecache/metrics.py.
"""
from __future__ import annotations

import re
import string
from collections import Counter

_PUNCT = set(string.punctuation)
_TERMINATORS = ("<|eot_id|>", "<|end_of_text|>", "<|im_end|>", "<|endoftext|>")


def normalize_answer(text: str) -> str:
    """Lower-case, drop punctuation and English articles, collapse whitespace."""
    text = "".join(ch for ch in text.lower() if ch not in _PUNCT)
    text = re.sub(r"\b(a|an|the)\b", " ", text)
    return " ".join(text.split())


def answer_em(prediction: str, golds) -> float:
    pred = normalize_answer(prediction)
    return float(any(pred == normalize_answer(g) for g in golds))


def _f1(prediction: str, gold: str) -> float:
    p = normalize_answer(prediction).split()
    g = normalize_answer(gold).split()
    if not p or not g:
        return float(p == g)
    common = sum((Counter(p) & Counter(g)).values())
    if common == 0:
        return 0.0
    precision, recall = common / len(p), common / len(g)
    return 2 * precision * recall / (precision + recall)


def answer_f1(prediction: str, golds) -> float:
    return max((_f1(prediction, g) for g in golds), default=0.0)


def clean_short_answer(text: str) -> str:
    """Strip chat terminators; keep the first non-empty line without an 'Answer:' label."""
    for marker in _TERMINATORS:
        text = text.replace(marker, "")
    lines = [line.strip() for line in text.strip().splitlines() if line.strip()]
    if not lines:
        return ""
    answer = re.sub(r"^(?:final\s+answer|answer)\s*:\s*", "", lines[0], flags=re.IGNORECASE)
    return answer.strip().strip('"').strip()
