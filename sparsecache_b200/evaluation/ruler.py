"""RULER qa_2 normalisation and exact-length P/D packs.

Parity with the reference's experiments/normalize_ruler_qa2.py (document
parsing, evidence tagging and the five placements :20-129) and
experiments/build_ruler_pd_pack.py (chat rendering with a documents
placeholder, exact-budget fitting that trims or repeats distractors only
:39-164).  A pack is ``requests.jsonl`` (prompt ids, max_tokens) plus
``metadata.jsonl`` (answers, fit mode, supporting-document spans) plus a
``manifest.json`` with the source hash.
"""
from __future__ import annotations

import hashlib
import json
import math
import re
from pathlib import Path
from typing import Any, Sequence

DOCUMENT_PATTERN = re.compile(r"(?:^|\n\n)Document (\d+):\n")
CONTEXT_START = "The following are given documents.\n\n"
CONTEXT_END = ("\n\nAnswer the question based on the given documents. Only give me the answer and do not output any "
               "other words.\n\nQuestion: ")
PLACEMENTS = ("original", "evidence_first", "evidence_uniform", "evidence_last", "adversarial_split")


def parse_documents(prompt: str) -> list[dict[str, str]]:
    """Documents (title = first line, text) of a generated RULER qa_2 prompt."""
    start = prompt.index(CONTEXT_START) + len(CONTEXT_START)
    body = prompt[start:prompt.index(CONTEXT_END, start)]
    marks = list(DOCUMENT_PATTERN.finditer(body))
    docs = []
    for i, m in enumerate(marks):
        end = marks[i + 1].start() if i + 1 < len(marks) else len(body)
        text = body[m.end():end].strip()
        docs.append({"title": text.splitlines()[0].strip(), "text": text})
    return docs


def uniform_order(supporting: Sequence[int], other: Sequence[int], total: int) -> list[int]:
    """Distractors in order with supporting documents spread evenly between them."""
    out = list(other)
    for i, doc in enumerate(supporting):
        out.insert(min(round((i + 1) * (total - 1) / (len(supporting) + 1)), len(out)), doc)
    return out


def placement_orders(documents: Sequence[dict]) -> dict[str, list[int]]:
    sup = [i for i, d in enumerate(documents) if d["supporting"]]
    oth = [i for i, d in enumerate(documents) if not d["supporting"]]
    adversarial = [sup[0], *oth, *sup[1:]] if len(sup) > 1 else [*oth, *sup]
    return {"original": list(range(len(documents))), "evidence_first": [*sup, *oth],
            "evidence_uniform": uniform_order(sup, oth, len(documents)), "evidence_last": [*oth, *sup],
            "adversarial_split": adversarial}


def normalize_row(row: dict, source_row: dict, length: int) -> dict[str, Any]:
    """One RULER qa_2 row with evidence flags (checked against HotpotQA supporting facts)."""
    docs = parse_documents(row["input"])
    titles = {f[0] for f in source_row["supporting_facts"]}
    for d in docs:
        d["supporting"] = d["title"] in titles
    found = {d["title"] for d in docs if d["supporting"]}
    if found != titles:
        raise ValueError(f"row {row['index']} evidence mismatch: {found} != {titles}")
    q0 = row["input"].index(CONTEXT_END) + len(CONTEXT_END)
    question = row["input"][q0:row["input"].index("<|eot_id|>", q0)].strip()
    if question != source_row["question"].strip():
        raise ValueError(f"row {row['index']} question mismatch")
    return {"id": f"ruler_qa2_{length}_{row['index']}", "index": row["index"], "dataset": "ruler_qa2",
            "target_length": length, "source_length_tokens": row["length"], "question": question,
            "answers": list(row["outputs"]), "documents": docs, "placements": placement_orders(docs)}


# ------------------------------------------------------------------ packing
def render_parts(tokenizer, row: dict, placement: str, *, disable_thinking: bool = False):
    """(prefix ids, per-document {token_ids, supporting, source_document_index}, suffix ids)."""
    ph = "{DOCUMENTS}"
    user = ("Answer the question based on the given documents. Only give me the answer and do not output any other "
            f"words.\n\nThe following are given documents.\n\n{ph}\n\nAnswer the question based on the given "
            "documents. Only give me the answer and do not output any other words.\n\nQuestion: "
            f"{row['question']}")
    kwargs = {"enable_thinking": False} if disable_thinking else {}
    text = tokenizer.apply_chat_template([{"role": "system", "content": "You are a helpful assistant"},
                                          {"role": "user", "content": user}], tokenize=False,
                                         add_generation_prompt=True, **kwargs)
    pivot = text.index(ph)
    prefix = tokenizer.encode(text[:pivot], add_special_tokens=False)
    suffix = tokenizer.encode(text[pivot + len(ph):], add_special_tokens=False)
    if placement not in row.get("placements", {}):
        raise ValueError(f"row does not define placement {placement}")
    order = row["placements"][placement]
    docs = []
    for shown, src in enumerate(order, start=1):
        d = row["documents"][src]
        sep = "\n\n" if shown < len(order) else ""
        docs.append({"token_ids": tokenizer.encode(f"Document {shown}:\n{d['text']}{sep}", add_special_tokens=False),
                     "supporting": bool(d["supporting"]), "source_document_index": src})
    return prefix, docs, suffix


def _largest_remainder(base: list[int], exact: dict[int, float], budget: int) -> list[int]:
    out = list(base)
    for i, x in exact.items():
        out[i] += math.floor(x)
    rem = budget - sum(out)
    for i in sorted(exact, key=lambda i: (-(exact[i] - math.floor(exact[i])), i))[:rem]:
        out[i] += 1
    return out


def allocate_trim_lengths(documents: Sequence[dict], budget: int) -> list[int]:
    """Shrink distractors (keeping >= 1 token each) proportionally to fit ``budget``; evidence untouched."""
    n = [len(d["token_ids"]) for d in documents]
    dis = [i for i, d in enumerate(documents) if not d["supporting"]]
    sup_tokens = sum(n[i] for i, d in enumerate(documents) if d["supporting"])
    room = budget - sup_tokens
    if room < len(dis):
        raise ValueError("budget cannot preserve supporting documents and distractors")
    removable = sum(n[i] - 1 for i in dis)
    extra = room - len(dis)
    if extra > removable:
        raise ValueError("trim allocation exceeds original document tokens")
    base = [1 if i in set(dis) else n[i] for i in range(len(n))]
    return _largest_remainder(base, {i: extra * (n[i] - 1) / removable for i in dis}, budget)


def allocate_expand_lengths(documents: Sequence[dict], budget: int) -> list[int]:
    """Grow distractors proportionally (by repetition) to fill ``budget``."""
    n = [len(d["token_ids"]) for d in documents]
    dis = [i for i, d in enumerate(documents) if not d["supporting"]]
    if not dis:
        raise ValueError("cannot expand a row without distractor documents")
    deficit = budget - sum(n)
    total = sum(n[i] for i in dis)
    return _largest_remainder(n, {i: deficit * n[i] / total for i in dis}, budget)


def fit_documents(documents: Sequence[dict], budget: int):
    """(fitted token lists summing to exactly ``budget``, original total, mode)."""
    total = sum(len(d["token_ids"]) for d in documents)
    if total > budget:
        lengths, mode = allocate_trim_lengths(documents, budget), "trim_distractors"
    elif total < budget:
        lengths, mode = allocate_expand_lengths(documents, budget), "repeat_distractors"
    else:
        lengths, mode = [len(d["token_ids"]) for d in documents], "unchanged"
    fitted = []
    for d, k in zip(documents, lengths):
        t = d["token_ids"]
        fitted.append(t[:k] if k <= len(t) else (t * -(-k // len(t)))[:k])
    if sum(map(len, fitted)) != budget:
        raise AssertionError("fitted documents do not fill the exact budget")
    return fitted, total, mode


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def build_pack(tokenizer, dataset_path: Path, placement: str, prompt_tokens: int, output_dir: Path, *,
               output_tokens: int = 32, num_requests: int | None = None, disable_thinking: bool = False,
               model_name: str = "sparsecache-llama31-8b") -> dict[str, Any]:
    """Write an exact-length pack from a normalised RULER JSONL; returns the manifest."""
    if prompt_tokens <= 0 or prompt_tokens % 256:
        raise ValueError("prompt_tokens must be a positive multiple of 256")
    if output_dir.exists():
        raise FileExistsError(f"refusing to overwrite {output_dir}")
    output_dir.mkdir(parents=True)
    modes: dict[str, int] = {}
    n = 0
    with open(dataset_path, encoding="utf-8") as src, open(output_dir / "requests.jsonl", "w") as rq, \
            open(output_dir / "metadata.jsonl", "w") as md:
        for index, line in enumerate(src):
            if num_requests is not None and n >= num_requests:
                break
            row = json.loads(line)
            prefix, docs, suffix = render_parts(tokenizer, row, placement, disable_thinking=disable_thinking)
            fitted, original, mode = fit_documents(docs, prompt_tokens - len(prefix) - len(suffix))
            prompt = prefix + [t for d in fitted for t in d] + suffix
            spans, at = [], len(prefix)
            for d, f in zip(docs, fitted):
                spans.append({"source_document_index": d["source_document_index"], "start_token": at,
                              "end_token": at + len(f), "supporting": d["supporting"]})
                at += len(f)
            rq.write(json.dumps({"model": model_name, "prompt": prompt, "max_tokens": output_tokens,
                                 "temperature": 0.0}) + "\n")
            md.write(json.dumps({"source_index": index, "id": row.get("id"), "answers": row["answers"],
                                 "fit_mode": mode, "original_document_tokens": original,
                                 "prefix_tokens": len(prefix), "suffix_tokens": len(suffix),
                                 "document_spans": spans}) + "\n")
            modes[mode] = modes.get(mode, 0) + 1
            n += 1
    manifest = {"dataset": "ruler_qa2", "source": str(Path(dataset_path).resolve()),
                "source_sha256": sha256_file(Path(dataset_path)), "placement": placement,
                "prompt_tokens": prompt_tokens, "output_tokens": output_tokens, "requests": n, "fit_modes": modes,
                "thinking_mode": "disabled" if disable_thinking else "default",
                "tokenizer": getattr(tokenizer, "name_or_path", "")}
    (output_dir / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n")
    return manifest


def normalize_tree(source_hotpot: Path, input_root: Path, output_root: Path,
                   lengths: Sequence[int]) -> dict[str, Any]:
    """Normalise ``<input_root>/<length>/qa_2/validation.jsonl`` for every length -> ``qa2_<length>.jsonl``.

    Reference: experiments/normalize_ruler_qa2.py:68-125.  ``source_hotpot`` is
    the HotpotQA JSON list the RULER rows index into (evidence titles and
    questions are checked against it).  Returns and writes ``audit.json``.
    """
    source = json.loads(Path(source_hotpot).read_text(encoding="utf-8"))
    output_root = Path(output_root)
    output_root.mkdir(parents=True, exist_ok=True)
    audit = {}
    for length in lengths:
        src = Path(input_root) / str(length) / "qa_2" / "validation.jsonl"
        rows = [json.loads(x) for x in src.read_text(encoding="utf-8").splitlines() if x.strip()]
        out = [normalize_row(r, source[r["index"]], int(length)) for r in rows]
        dst = output_root / f"qa2_{length}.jsonl"
        dst.write_text("".join(json.dumps(r, ensure_ascii=False) + "\n" for r in out), encoding="utf-8")
        audit[str(length)] = {"input": str(src.resolve()), "output": str(dst.resolve()), "rows": len(out),
                              "mean_documents": sum(len(r["documents"]) for r in out) / max(1, len(out)),
                              "supporting_document_counts": sorted({sum(d["supporting"] for d in r["documents"])
                                                                    for r in out}),
                              "placements": sorted(out[0]["placements"]) if out else []}
    (output_root / "audit.json").write_text(json.dumps(audit, indent=2) + "\n", encoding="utf-8")
    return audit
