"""Dataset adapters and the ``sparsecache-prepare`` CLI.

Normalises one QA record into a ``QACase`` with an ordered list of
independently reusable document chunks (reference src/sparsecache/data.py):
  * HotpotQA-E / LongBench JSONL: the ``context`` field is split on lines of
    the form ``Passage N:``; the first line of a passage is its title;
  * official MuSiQue JSONL: ``paragraphs`` with ``idx``, ``title``,
    ``paragraph_text`` and ``is_supporting``; gold answers are ``answer`` plus
    ``answer_aliases``.
"""
from __future__ import annotations

import argparse
import json
import re
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any


@dataclass(frozen=True)
class DocumentChunk:
    chunk_id: str
    title: str
    text: str
    supporting: bool | None = None


@dataclass(frozen=True)
class QACase:
    case_id: str
    source: str
    question: str
    answers: tuple[str, ...]
    chunks: tuple[DocumentChunk, ...]

    def as_dict(self) -> dict[str, Any]:
        out = asdict(self)
        out["answers"] = list(self.answers)
        out["chunks"] = [asdict(c) for c in self.chunks]
        return out


def load_prepared_case(path: str | Path) -> QACase:
    row = json.loads(Path(path).read_text(encoding="utf-8"))
    return QACase(
        case_id=str(row["case_id"]),
        source=str(row["source"]),
        question=str(row["question"]),
        answers=tuple(str(a) for a in row["answers"]),
        chunks=tuple(DocumentChunk(**c) for c in row["chunks"]),
    )


def _jsonl_row(path: str | Path, index: int) -> dict[str, Any]:
    with Path(path).open(encoding="utf-8") as handle:
        for i, line in enumerate(handle):
            if i == index:
                return json.loads(line)
    raise ValueError(f"dataset does not contain row {index}")


_PASSAGE = re.compile(r"(?=^Passage \d+:\n)", flags=re.M)


def split_passages(context: str) -> list[str]:
    parts = [p for p in _PASSAGE.split(context.strip()) if p.strip()]
    return parts or [context]


def load_hotpotqa_case(path: str | Path, *, index: int, max_chunks: int) -> QACase:
    row = _jsonl_row(path, index)
    chunks = []
    for i, passage in enumerate(split_passages(str(row["context"]))[:max_chunks]):
        lines = passage.strip().splitlines()
        if lines and re.fullmatch(r"Passage \d+:", lines[0]):
            lines = lines[1:]
        title = lines[0].strip() if lines else f"Passage {i + 1}"
        text = "\n".join(lines[1:]).strip() if len(lines) > 1 else title
        chunks.append(DocumentChunk(chunk_id=f"passage-{i + 1:02d}", title=title, text=text))
    return QACase(
        case_id=str(row.get("_id", index)),
        source=str(row.get("dataset", "hotpotqa")),
        question=str(row["input"]),
        answers=tuple(str(a) for a in row.get("answers", [])),
        chunks=tuple(chunks),
    )


def load_musique_case(path: str | Path, *, index: int, max_chunks: int) -> QACase:
    row = _jsonl_row(path, index)
    chunks = tuple(
        DocumentChunk(
            chunk_id=f"paragraph-{int(p['idx']):02d}",
            title=str(p["title"]),
            text=str(p["paragraph_text"]),
            supporting=bool(p.get("is_supporting", False)),
        )
        for p in row["paragraphs"][:max_chunks]
    )
    answers: list[str] = [str(row["answer"])] if row.get("answer") else []
    answers.extend(str(a) for a in row.get("answer_aliases", []) if a not in answers)
    return QACase(
        case_id=str(row.get("id", index)),
        source="musique",
        question=str(row["question"]),
        answers=tuple(answers),
        chunks=chunks,
    )


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(description="Prepare one normalised ten-chunk QA case")
    parser.add_argument("--dataset", choices=("hotpotqa", "musique"), required=True)
    parser.add_argument("--input", required=True)
    parser.add_argument("--output", required=True)
    parser.add_argument("--index", type=int, default=0)
    parser.add_argument("--max-chunks", type=int, default=10)
    args = parser.parse_args(argv)
    if args.index < 0 or args.max_chunks < 1:
        parser.error("index must be non-negative and max-chunks positive")
    loader = load_hotpotqa_case if args.dataset == "hotpotqa" else load_musique_case
    case = loader(args.input, index=args.index, max_chunks=args.max_chunks)
    if len(case.chunks) != args.max_chunks:
        raise ValueError(f"requested {args.max_chunks} chunks but case contains {len(case.chunks)}")
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(case.as_dict(), ensure_ascii=False, indent=2) + "\n", encoding="utf-8")
    print(json.dumps({"event": "prepared", "output": str(out), "case_id": case.case_id,
                      "chunks": len(case.chunks)}, ensure_ascii=False))


if __name__ == "__main__":
    main()
