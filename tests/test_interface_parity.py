"""Interfaces that must stay identical to the reference's, pinned two ways.

* Golden values (always run): fixed inputs give the same chunk split, chunk
  ids, token ids and gate verdicts as recorded here.
* Side by side with the reference's own code when it is installed under
  baseline/_ref (skipped otherwise): the dataset readers and the prompt
  assembly give identical results on seeded random inputs.
"""
import json
import os
import random
import sys

import pytest

from sparsecache_b200 import data, prompting
from sparsecache_b200.tokenizer import ByteTokenizer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def _reference():
    if not os.path.isfile(os.path.join(REF, "sparsecache", "data.py")):
        pytest.skip("the reference is not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import sparsecache.data as ref_data
    import sparsecache.prompting as ref_prompting

    return ref_data, ref_prompting


def _random_context(rng: random.Random) -> str:
    parts = []
    if rng.random() < 0.2:
        parts.append("preamble line\nmore preamble")
    for k in range(1, rng.randint(0, 12)):
        body = "\n".join(f"line {k}.{i} " + "x" * rng.randint(0, 5) for i in range(rng.randint(0, 3)))
        header = f"Passage {k}:" if rng.random() < 0.9 else f"Passage {k}: inline"
        parts.append(f"{header}\nTitle {k}\n{body}".rstrip("\n") if rng.random() < 0.8 else header)
    sep = "\n" if rng.random() < 0.7 else "\n\n"
    return (" " if rng.random() < 0.3 else "") + sep.join(parts) + ("\n" if rng.random() < 0.5 else "")


def test_golden_split_and_chunk_ids(tmp_path):
    ctx = "Passage 1:\nAlpha\nfirst body\nsecond line\nPassage 2:\nBeta\nPassage 3:\nGamma\ntext\nPassage 4:"
    parts = data.split_passages(ctx)
    assert len(parts) == 3 and parts[2].endswith("Passage 4:")
    row = {"_id": "x", "input": "q", "answers": ["a"], "context": ctx}
    (tmp_path / "h.jsonl").write_text("{}\n" + json.dumps(row) + "\n")
    case = data.load_hotpotqa_case(tmp_path / "h.jsonl", index=1, max_chunks=10)
    assert [(c.chunk_id, c.title, c.text) for c in case.chunks] == [
        ("passage-01", "Alpha", "first body\nsecond line"), ("passage-02", "Beta", "Beta"),
        ("passage-03", "Gamma", "text\nPassage 4:")]
    assert case.source == "hotpotqa" and case.case_id == "x"
    with pytest.raises(ValueError, match="row 5"):
        data.load_hotpotqa_case(tmp_path / "h.jsonl", index=5, max_chunks=10)


def test_golden_prompt_ids():
    tok = ByteTokenizer(1024)
    case = data.QACase("c", "s", " Who?  ", ("a",), (data.DocumentChunk("p1", "T1", " body one "),
                                                     data.DocumentChunk("p2", "T2", "two")))
    p = prompting.tokenize_case(tok, case)
    assert p.full_ids == p.system_ids + p.document_ids + p.suffix_ids
    assert [c[0] for c in p.chunks] == ["p1", "p2"]
    assert tok.decode(p.chunks[0][2]) == "Document 1: T1\nbody one\n"
    spans = p.chunk_spans()
    assert spans[0][0] == len(p.system_ids) and spans[-1][1] == len(p.system_ids) + len(p.document_ids)
    assert "Question: Who?\n" in tok.decode(p.suffix_ids)


def test_readers_match_reference(tmp_path):
    ref_data, _ = _reference()
    rng = random.Random(1234)
    for trial in range(300):
        ctx = _random_context(rng)
        assert data.split_passages(ctx) == ref_data._split_hotpot_passages(ctx) or \
            [p.strip() for p in data.split_passages(ctx)] == [p.strip() for p in ref_data._split_hotpot_passages(ctx)]
        row = {"_id": f"id{trial}", "dataset": "hotpotqa", "input": "q?", "answers": ["x"], "context": ctx}
        (tmp_path / "h.jsonl").write_text(json.dumps(row) + "\n")
        ours = data.load_hotpotqa_case(tmp_path / "h.jsonl", index=0, max_chunks=7)
        theirs = ref_data.load_hotpotqa_case(tmp_path / "h.jsonl", index=0, max_chunks=7)
        assert ours.as_dict() == theirs.as_dict(), ctx
    for trial in range(50):
        n = rng.randint(1, 14)
        aliases = [rng.choice(["A", "a", "B", "A "]) for _ in range(rng.randint(0, 4))]
        row = {"id": f"m{trial}", "question": "q", "answer": rng.choice(["A", "", "B"]), "answer_aliases": aliases,
               "paragraphs": [{"idx": i, "title": f"t{i}", "paragraph_text": f"p{i}",
                               "is_supporting": rng.random() < 0.3} for i in range(n)]}
        (tmp_path / "m.jsonl").write_text(json.dumps(row) + "\n")
        ours = data.load_musique_case(tmp_path / "m.jsonl", index=0, max_chunks=10)
        theirs = ref_data.load_musique_case(tmp_path / "m.jsonl", index=0, max_chunks=10)
        assert ours.as_dict() == theirs.as_dict()


def test_prompt_ids_match_reference():
    ref_data, ref_prompting = _reference()
    tok = ByteTokenizer(1024)
    rng = random.Random(7)
    for trial in range(40):
        chunks = [data.DocumentChunk(f"c{i}", f"Title {i}", " " * rng.randint(0, 2) + "text " * rng.randint(1, 9))
                  for i in range(rng.randint(1, 10))]
        case = data.QACase(f"k{trial}", "s", "  question %d ?  " % trial, ("a",), tuple(chunks))
        ref_case = ref_data.QACase(case.case_id, case.source, case.question, case.answers,
                                   tuple(ref_data.DocumentChunk(c.chunk_id, c.title, c.text) for c in chunks))
        ours = prompting.tokenize_case(tok, case)
        theirs = ref_prompting.tokenize_case(tok, ref_case)
        assert ours.system_ids == theirs.system_ids
        assert ours.chunks == theirs.chunks
        assert ours.suffix_ids == theirs.suffix_ids
        assert ours.full_ids == theirs.full_ids
