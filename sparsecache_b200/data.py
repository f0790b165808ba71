"""Dataset readers and the ``sparsecache-prepare`` command.

A prepared case is one question with its gold answers and an ordered list of
document chunks, each of which is prefilled and cached on its own.  Two
source formats are read (behaviour of the reference's
src/sparsecache/data.py, whose prepared-case JSON and chunk ids this module
keeps so that caches and manifests stay interchangeable):

* passage-context rows (HotpotQA-E / LongBench JSONL): the ``context``
  string holds ``Passage N:`` header lines; each header opens a passage
  whose first line is its title and whose remaining lines are its text;
  chunk ids are ``passage-01`` ...;
* MuSiQue rows: a ``paragraphs`` list with ``idx``, ``title``,
  ``paragraph_text`` and ``is_supporting``; gold answers are ``answer``
  followed by the ``answer_aliases`` not already listed; chunk ids are
  ``paragraph-<idx>``.
"""
from __future__ import annotations

import argparse
import itertools
import json
import re
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Callable, Iterator


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
        """The prepared-case JSON object (lists, not tuples)."""
        return {"case_id": self.case_id, "source": self.source, "question": self.question,
                "answers": list(self.answers), "chunks": [asdict(c) for c in self.chunks]}

    @classmethod
    def from_dict(cls, obj: dict[str, Any]) -> "QACase":
        return cls(case_id=str(obj["case_id"]), source=str(obj["source"]), question=str(obj["question"]),
                   answers=tuple(map(str, obj["answers"])),
                   chunks=tuple(DocumentChunk(**c) for c in obj["chunks"]))


def load_prepared_case(path: str | Path) -> QACase:
    return QACase.from_dict(json.loads(Path(path).read_text(encoding="utf-8")))


def read_jsonl_row(path: str | Path, index: int) -> dict[str, Any]:
    """Row ``index`` (0-based) of a JSONL file, reading no further than it."""
    with Path(path).open(encoding="utf-8") as lines:
        hit = next(itertools.islice(lines, index, None), None)
    if hit is None:
        raise ValueError(f"dataset does not contain row {index}")
    return json.loads(hit)


_HEADER = re.compile(r"Passage \d+:")


def split_passages(context: str) -> list[str]:
    """Cut a passage-context string into passages.

    A line ``Passage N:`` that is followed by another line starts a new
    passage (the header stays at the head of its passage); text before the
    first header is a passage of its own; with no non-blank passage at all the
    whole context is returned as one.
    """
    lines = context.strip().split("\n")
    groups: list[list[str]] = [[]]
    for pos, line in enumerate(lines):
        if _HEADER.fullmatch(line) and pos + 1 < len(lines) and groups[-1]:
            groups.append([])
        groups[-1].append(line)
    passages = ["\n".join(g) for g in groups]
    kept = [p for p in passages if p.strip()]
    return kept or [context]


def passage_chunk(position: int, passage: str) -> DocumentChunk:
    """Chunk ``position`` (1-based) from one passage: header dropped, first line the title."""
    lines = passage.strip().splitlines()
    if lines and _HEADER.fullmatch(lines[0]):
        lines = lines[1:]
    if not lines:
        title, text = f"Passage {position}", f"Passage {position}"
    else:
        title = lines[0].strip()
        text = "\n".join(lines[1:]).strip() if len(lines) > 1 else title
    return DocumentChunk(chunk_id=f"passage-{position:02d}", title=title, text=text)


def _passage_rows(row: dict[str, Any], index: int, max_chunks: int) -> QACase:
    parts = split_passages(str(row["context"]))[:max_chunks]
    return QACase(
        case_id=str(row.get("_id", index)),
        source=str(row.get("dataset", "hotpotqa")),
        question=str(row["input"]),
        answers=tuple(map(str, row.get("answers", []))),
        chunks=tuple(passage_chunk(k, part) for k, part in enumerate(parts, 1)),
    )


def _musique_answers(row: dict[str, Any]) -> tuple[str, ...]:
    ordered: dict[str, None] = {}
    if row.get("answer"):
        ordered[str(row["answer"])] = None
    for alias in row.get("answer_aliases", []):
        ordered.setdefault(str(alias), None)
    return tuple(ordered)


def _musique_rows(row: dict[str, Any], index: int, max_chunks: int) -> QACase:
    paragraphs = row["paragraphs"][:max_chunks]
    return QACase(
        case_id=str(row.get("id", index)),
        source="musique",
        question=str(row["question"]),
        answers=_musique_answers(row),
        chunks=tuple(DocumentChunk(chunk_id=f"paragraph-{int(p['idx']):02d}", title=str(p["title"]),
                                   text=str(p["paragraph_text"]), supporting=bool(p.get("is_supporting", False)))
                     for p in paragraphs),
    )


# dataset name -> reader of one parsed JSONL row
READERS: dict[str, Callable[[dict[str, Any], int, int], QACase]] = {
    "hotpotqa": _passage_rows,
    "musique": _musique_rows,
}


def load_case(dataset: str, path: str | Path, *, index: int, max_chunks: int) -> QACase:
    if dataset not in READERS:
        raise ValueError(f"unknown dataset {dataset!r}; known: {sorted(READERS)}")
    return READERS[dataset](read_jsonl_row(path, index), index, max_chunks)


def load_hotpotqa_case(path: str | Path, *, index: int, max_chunks: int) -> QACase:
    return load_case("hotpotqa", path, index=index, max_chunks=max_chunks)


def load_musique_case(path: str | Path, *, index: int, max_chunks: int) -> QACase:
    return load_case("musique", path, index=index, max_chunks=max_chunks)


def iter_cases(dataset: str, path: str | Path, *, max_chunks: int, start: int = 0,
               count: int | None = None) -> Iterator[QACase]:
    """Cases of a JSONL file in order (for batch preparation), one row per case."""
    with Path(path).open(encoding="utf-8") as lines:
        rows = itertools.islice(lines, start, None if count is None else start + count)
        for offset, line in enumerate(rows):
            yield READERS[dataset](json.loads(line), start + offset, max_chunks)


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(description="Prepare one normalised multi-chunk QA case")
    parser.add_argument("--dataset", choices=tuple(READERS), required=True)
    parser.add_argument("--input", required=True)
    parser.add_argument("--output", required=True)
    parser.add_argument("--index", type=int, default=0)
    parser.add_argument("--max-chunks", type=int, default=10)
    args = parser.parse_args(argv)
    if args.index < 0 or args.max_chunks < 1:
        parser.error("index must be non-negative and max-chunks positive")
    case = load_case(args.dataset, args.input, index=args.index, max_chunks=args.max_chunks)
    if len(case.chunks) != args.max_chunks:
        raise ValueError(f"requested {args.max_chunks} chunks but case contains {len(case.chunks)}")
    target = Path(args.output)
    target.parent.mkdir(parents=True, exist_ok=True)
    target.write_text(json.dumps(case.as_dict(), ensure_ascii=False, indent=2) + "\n", encoding="utf-8")
    event = {"event": "prepared", "output": str(target), "case_id": case.case_id, "chunks": len(case.chunks)}
    print(json.dumps(event, ensure_ascii=False))


if __name__ == "__main__":
    main()
