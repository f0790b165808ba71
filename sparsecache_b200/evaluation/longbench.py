"""LongBench / LongBench-v2 prompts, output caps, metrics and P/D pack building.

Parity with the reference's experiments/longbench_metrics.py (dataset ->
metric map :26-37; QA F1, ROUGE-L via LCS, retrieval / count accuracy, code
edit similarity, classification, LongBench-v2 choice :40-194),
experiments/longbench_prompts.py (the public LongBench templates and
generation limits :4-124) and experiments/build_longbench_pd_pack.py
(chunk-aligned middle truncation / padding :48-93, rendering :95-153).

The templates below are LongBench's published prompts, reproduced verbatim
(typos included) because scores are only comparable with the exact prompt.
All metrics are dependency-free and return values in [0, 1].
"""
from __future__ import annotations

import difflib
import math
import re
import string
from collections import Counter
from typing import Any, Sequence

QA_DATASETS = frozenset({"narrativeqa", "qasper", "multifieldqa_en", "hotpotqa", "2wikimqa", "musique", "triviaqa"})
ROUGE_DATASETS = frozenset({"gov_report", "qmsum", "multi_news", "samsum"})
CLASSIFICATION_DATASETS = frozenset({"trec", "lsht"})
CODE_DATASETS = frozenset({"lcc", "repobench-p"})
FIRST_LINE_DATASETS = frozenset({"trec", "triviaqa", "samsum", "lsht"})

_PASSAGES_QA = ("Answer the question based on the given passages. Only give me the answer and do not output any other "
                "words.\n\nThe following are given passages.\n{context}\n\nAnswer the question based on the given "
                "passages. Only give me the answer and do not output any other words.\n\nQuestion: {input}\nAnswer:")

LONG_BENCH_PROMPTS = {
    "narrativeqa": ("You are given a story, which can be either a novel or a movie script, and a question. Answer the "
                    "question asconcisely as you can, using a single phrase if possible. Do not provide any "
                    "explanation.\n\nStory: {context}\n\nNow, answer the question based on the story asconcisely as "
                    "you can, using a single phrase if possible. Do not provide any explanation.\n\nQuestion: "
                    "{input}\n\nAnswer:"),
    "qasper": ("You are given a scientific article and a question. Answer the question as concisely as you can, using "
               "a single phrase or sentence if possible. If the question cannot be answered based on the information "
               "in the article, write \"unanswerable\". If the question is a yes/no question, answer \"yes\", "
               "\"no\", or \"unanswerable\". Do not provide any explanation.\n\nArticle: {context}\n\n Answer the "
               "question based on the above article as concisely as you can, using a single phrase or sentence if "
               "possible. If the question cannot be answered based on the information in the article, write "
               "\"unanswerable\". If the question is a yes/no question, answer \"yes\", \"no\", or "
               "\"unanswerable\". Do not provide any explanation.\n\nQuestion: {input}\n\nAnswer:"),
    "multifieldqa_en": ("Read the following text and answer briefly.\n\n{context}\n\nNow, answer the following "
                        "question based on the above text, only give me the answer and do not output any other "
                        "words.\n\nQuestion: {input}\nAnswer:"),
    "hotpotqa": _PASSAGES_QA,
    "2wikimqa": _PASSAGES_QA,
    "musique": _PASSAGES_QA,
    "gov_report": ("You are given a report by a government agency. Write a one-page summary of the report.\n\n"
                   "Report:\n{context}\n\nNow, write a one-page summary of the report.\n\nSummary:"),
    "qmsum": ("You are given a meeting transcript and a query containing a question or instruction. Answer the query "
              "in one or more sentences.\n\nTranscript:\n{context}\n\nNow, answer the query based on the above "
              "meeting transcript in one or more sentences.\n\nQuery: {input}\nAnswer:"),
    "multi_news": ("You are given several news passages. Write a one-page summary of all news. \n\nNews:\n{context}"
                   "\n\nNow, write a one-page summary of all the news.\n\nSummary:"),
    "passage_count": ("There are some paragraphs below sourced from Wikipedia. Some of them may be duplicates. Please "
                      "carefully read these paragraphs and determine how many unique paragraphs there are after "
                      "removing duplicates. In other words, how many non-repeating paragraphs are there in total?"
                      "\n\n{context}\n\nPlease enter the final count of unique paragraphs after removing duplicates. "
                      "The output format should only contain the number, such as 1, 2, 3, and so on.\n\nThe final "
                      "answer is: "),
    "passage_retrieval_en": ("Here are 30 paragraphs from Wikipedia, along with an abstract. Please determine which "
                             "paragraph the abstract is from.\n\n{context}\n\nThe following is an abstract.\n\n"
                             "{input}\n\nPlease enter the number of the paragraph that the abstract is from. The "
                             "answer format must be like \"Paragraph 1\", \"Paragraph 2\", etc.\n\nThe answer is: "),
    "lcc": "Please complete the code given below. \n{context}Next line of code:\n",
    "repobench-p": "Please complete the code given below. \n{context}{input}Next line of code:\n",
}

LONG_BENCH_MAX_NEW_TOKENS = {
    "narrativeqa": 128, "qasper": 128, "multifieldqa_en": 64, "hotpotqa": 32, "2wikimqa": 32, "musique": 32,
    "gov_report": 512, "qmsum": 512, "multi_news": 512, "passage_count": 32, "passage_retrieval_en": 32,
    "lcc": 64, "repobench-p": 64,
}

LONG_BENCH_V2_PROMPT = (
    "Please read the following text and answer the question below.\n\n<text>\n{context}\n</text>\n\n"
    "What is the correct answer to this question: {question}\nChoices:\n(A) {choice_A}\n(B) {choice_B}\n"
    "(C) {choice_C}\n(D) {choice_D}\n\nFormat your response as follows: \"The correct answer is (insert answer "
    "here)\".")
LONG_BENCH_V2_MAX_NEW_TOKENS = 128


# -------------------------------------------------------------------- metrics
def normalize_answer(text: str) -> str:
    """Lower-case, drop punctuation and articles, collapse whitespace."""
    text = "".join(ch for ch in text.lower() if ch not in string.punctuation)
    text = re.sub(r"\b(a|an|the)\b", " ", text)
    return " ".join(text.split())


def exact_match(prediction: str, expected: str) -> float:
    return float(normalize_answer(prediction) == normalize_answer(expected))


def qa_f1(prediction: str, expected: str) -> float:
    pred, gold = normalize_answer(prediction).split(), normalize_answer(expected).split()
    same = sum((Counter(pred) & Counter(gold)).values())
    if same == 0:
        return 0.0
    p, r = same / len(pred), same / len(gold)
    return 2 * p * r / (p + r)


def lcs_length(a: Sequence[str], b: Sequence[str]) -> int:
    """Longest common subsequence length, O(len(a) * len(b)) time, O(min) memory."""
    if len(a) < len(b):
        a, b = b, a
    row = [0] * (len(b) + 1)
    for x in a:
        prev_diag = 0
        for j, y in enumerate(b, start=1):
            keep = row[j]
            row[j] = prev_diag + 1 if x == y else max(row[j], row[j - 1])
            prev_diag = keep
    return row[-1]


def rouge_l_f1(prediction: str, expected: str) -> float:
    pred, gold = prediction.lower().split(), expected.lower().split()
    if not pred or not gold:
        return 0.0
    lcs = lcs_length(pred, gold)
    if lcs == 0:
        return 0.0
    p, r = lcs / len(pred), lcs / len(gold)
    return 2 * p * r / (p + r)


def retrieval_accuracy(prediction: str, expected: str) -> float:
    want = re.findall(r"Paragraph (\d+)", expected)
    got = re.findall(r"\d+", prediction)
    if not want or not got:
        return 0.0
    return sum(g == want[0] for g in got) / len(got)


def count_accuracy(prediction: str, expected: str) -> float:
    got = re.findall(r"\d+", prediction)
    return sum(g == str(expected) for g in got) / len(got) if got else 0.0


def code_similarity(prediction: str, expected: str) -> float:
    """Edit similarity of the first non-comment line against the reference line."""
    line = next((ln for ln in prediction.lstrip("\n").split("\n")
                 if "`" not in ln and "#" not in ln and "//" not in ln), "")
    return difflib.SequenceMatcher(None, line, expected).ratio()


def classification_accuracy(prediction: str, expected: str, all_classes: Sequence[str] | None) -> float:
    hits = [c for c in (all_classes or []) if c in prediction and not (c in expected and c != expected)]
    return 1.0 / len(hits) if expected in hits else 0.0


def longbench_v2_choice(prediction: str) -> str:
    text = prediction.replace("*", "")
    for pat in (r"The correct answer is \(([A-D])\)", r"The correct answer is ([A-D])"):
        m = re.search(pat, text, flags=re.IGNORECASE)
        if m:
            return m.group(1).upper()
    return ""


def metric_for(dataset: str) -> str:
    if dataset == "longbench_v2":
        return "choice_accuracy"
    if dataset in ROUGE_DATASETS:
        return "rouge_l_f1"
    if dataset == "passage_retrieval_en":
        return "retrieval_accuracy"
    if dataset == "passage_count":
        return "count_accuracy"
    if dataset in CODE_DATASETS:
        return "code_similarity"
    if dataset in CLASSIFICATION_DATASETS:
        return "classification_accuracy"
    return "qa_f1"


def score_prediction(dataset: str, prediction: str, expected_answers: Sequence[str],
                     all_classes: Sequence[str] | None = None) -> tuple[str, float, float]:
    """(metric name, normalised exact match, task score) for one prediction."""
    if dataset in FIRST_LINE_DATASETS:
        prediction = prediction.lstrip("\n").split("\n")[0]
    name = metric_for(dataset)
    if name == "choice_accuracy":
        choice = longbench_v2_choice(prediction)
        s = max((float(choice == str(a).upper()) for a in expected_answers), default=0.0)
        return name, s, s
    scorer = {
        "qa_f1": qa_f1,
        "rouge_l_f1": rouge_l_f1,
        "retrieval_accuracy": retrieval_accuracy,
        "count_accuracy": count_accuracy,
        "code_similarity": code_similarity,
        "classification_accuracy": lambda p, e: classification_accuracy(p, e, all_classes),
    }[name]
    em = max((exact_match(prediction, a) for a in expected_answers), default=0.0)
    return name, em, max((scorer(prediction, a) for a in expected_answers), default=0.0)


# --------------------------------------------------------------- pack building
def middle_truncate(tokens: list[int], length: int) -> list[int]:
    """Keep the first ceil(length/2) and the last floor(length/2) tokens."""
    if len(tokens) <= length:
        return tokens
    head = math.ceil(length / 2)
    tail = length - head
    return tokens[:head] + (tokens[-tail:] if tail else [])


def align_context_to_chunk(prefix: list[int], context: list[int], suffix: list[int], *, max_prompt_tokens: int,
                           chunk_tokens: int, padding_token_id: int = 198):
    """Trim only the context (middle first) so the prompt is a whole number of chunks.

    Returns (prompt, tokens removed by the length cap, tokens removed for
    alignment, padding added).  Padding is used only when alignment would
    remove the entire context.
    """
    fixed = len(prefix) + len(suffix)
    if fixed >= max_prompt_tokens:
        raise ValueError("prompt scaffolding leaves no context budget")
    keep = min(len(context), max_prompt_tokens - fixed)
    cap_removed = len(context) - keep
    ctx = middle_truncate(context, keep)
    total = fixed + len(ctx)
    aligned_ctx = total - total % chunk_tokens - fixed
    if aligned_ctx <= 0:
        padded = -(-total // chunk_tokens) * chunk_tokens
        if padded > max_prompt_tokens:
            raise ValueError("short prompt cannot be padded within the model limit")
        pad = padded - total
        return prefix + ctx + [padding_token_id] * pad + suffix, cap_removed, 0, pad
    removed = len(ctx) - aligned_ctx
    prompt = prefix + middle_truncate(ctx, aligned_ctx) + suffix
    assert len(prompt) % chunk_tokens == 0
    return prompt, cap_removed, removed, 0


def render_longbench(tokenizer, dataset: str, row: dict[str, Any], *, disable_thinking: bool = False):
    """Chat-rendered prompt with a context placeholder -> (rendered text, placeholder)."""
    placeholder = "{CONTEXT}"
    kwargs = {"enable_thinking": False} if disable_thinking else {}
    if dataset == "longbench_v2":
        body = LONG_BENCH_V2_PROMPT.format(context=placeholder, question=row["question"],
                                           **{f"choice_{c}": row[f"choice_{c}"] for c in "ABCD"})
    else:
        if dataset not in LONG_BENCH_PROMPTS:
            raise ValueError(f"no official LongBench prompt for {dataset}")
        body = LONG_BENCH_PROMPTS[dataset].format(context=placeholder, input=row.get("input", ""))
        if dataset in CODE_DATASETS:  # code completion is not chat-wrapped
            return body, placeholder
    return tokenizer.apply_chat_template([{"role": "user", "content": body}], tokenize=False,
                                         add_generation_prompt=True, **kwargs), placeholder


def encode_parts(tokenizer, rendered: str, placeholder: str, context: str):
    pivot = rendered.index(placeholder)
    return (tokenizer.encode(rendered[:pivot], add_special_tokens=False),
            tokenizer.encode(context, add_special_tokens=False),
            tokenizer.encode(rendered[pivot + len(placeholder):], add_special_tokens=False))


def build_longbench_request(tokenizer, dataset: str, row: dict[str, Any], *, max_prompt_tokens: int,
                            chunk_tokens: int = 256, disable_thinking: bool = False,
                            padding_token_id: int = 198) -> dict[str, Any]:
    """One P/D request row: chunk-aligned prompt ids plus its scoring metadata."""
    rendered, ph = render_longbench(tokenizer, dataset, row, disable_thinking=disable_thinking)
    prefix, ctx, suffix = encode_parts(tokenizer, rendered, ph, str(row["context"]))
    prompt, cap_removed, align_removed, pad = align_context_to_chunk(
        prefix, ctx, suffix, max_prompt_tokens=max_prompt_tokens, chunk_tokens=chunk_tokens,
        padding_token_id=padding_token_id)
    cap = LONG_BENCH_V2_MAX_NEW_TOKENS if dataset == "longbench_v2" else LONG_BENCH_MAX_NEW_TOKENS.get(dataset, 32)
    answers = row.get("answers") or [row.get("answer", "")]
    return {"prompt": prompt, "max_tokens": cap, "dataset": dataset, "answers": list(answers),
            "all_classes": row.get("all_classes"), "cap_removed_tokens": cap_removed,
            "alignment_removed_tokens": align_removed, "padding_tokens": pad, "prefix_tokens": len(prefix),
            "suffix_tokens": len(suffix)}


def iter_dataset_rows(path):
    """Rows of a JSON list or a JSONL file (objects only)."""
    import json
    from pathlib import Path

    path = Path(path)
    if path.suffix == ".json":
        rows = json.loads(path.read_text(encoding="utf-8"))
        if not isinstance(rows, list):
            raise TypeError("a JSON dataset must hold a list of request objects")
    else:
        rows = (json.loads(x) for x in path.read_text(encoding="utf-8").splitlines() if x.strip())
    for row in rows:
        if not isinstance(row, dict):
            raise TypeError("dataset rows must be objects")
        yield row


def build_longbench_pack(tokenizer, dataset_path, dataset: str, output_dir, *, fmt: str = "longbench",
                         served_model_name: str = "sparsecache-llama31-8b", num_requests: int | None = None,
                         max_prompt_tokens: int = 32768, chunk_tokens: int = 256,
                         fixed_output_tokens: int | None = None, disable_thinking: bool = False,
                         tokenizer_name: str = "") -> dict[str, Any]:
    """Write a chunk-aligned LongBench / LongBench-v2 P/D pack; returns its manifest.

    Reference: experiments/build_longbench_pd_pack.py:182-344.  The context is
    middle-truncated to the length cap and then down to whole transfer chunks;
    one newline token pads a prompt only when aligning would remove the whole
    context.  ``requests.jsonl`` holds completion requests (prompt ids),
    ``metadata.jsonl`` the scoring fields, ``manifest.json`` the hashes.
    """
    import json
    from pathlib import Path

    from .audits import _sha256

    if chunk_tokens <= 0 or max_prompt_tokens <= 0 or max_prompt_tokens % chunk_tokens:
        raise ValueError("max_prompt_tokens must be a positive multiple of chunk_tokens")
    if num_requests is not None and num_requests <= 0:
        raise ValueError("num_requests must be positive")
    if fixed_output_tokens is not None and fixed_output_tokens <= 0:
        raise ValueError("fixed_output_tokens must be positive")
    if fmt not in ("longbench", "longbench_v2"):
        raise ValueError(f"unknown pack format {fmt}")
    output_dir = Path(output_dir)
    if output_dir.exists():
        raise FileExistsError(f"refusing to overwrite {output_dir}")
    newline = tokenizer.encode("\n", add_special_tokens=False)
    if len(newline) != 1:
        raise ValueError("the tokenizer must encode a newline as one alignment token")
    output_dir.mkdir(parents=True)
    req_path, meta_path = output_dir / "requests.jsonl", output_dir / "metadata.jsonl"
    lengths, cap_rm, align_rm, pads = [], [], [], []
    name = "longbench_v2" if fmt == "longbench_v2" else dataset
    with req_path.open("w", encoding="utf-8") as rq, meta_path.open("w", encoding="utf-8") as md:
        for source_index, row in enumerate(iter_dataset_rows(dataset_path)):
            r = build_longbench_request(tokenizer, name, row, max_prompt_tokens=max_prompt_tokens,
                                        chunk_tokens=chunk_tokens, disable_thinking=disable_thinking,
                                        padding_token_id=int(newline[0]))
            out_tokens = fixed_output_tokens or r["max_tokens"]
            rq.write(json.dumps({"model": served_model_name, "prompt": r["prompt"], "max_tokens": out_tokens,
                                 "temperature": 0, "ignore_eos": fixed_output_tokens is not None,
                                 "stream": True, "return_token_ids": True}) + "\n")
            answers = r["answers"] if fmt == "longbench" else (
                list(row["answer"]) if isinstance(row.get("answer"), list) else [str(row.get("answer", ""))])
            md.write(json.dumps({"request_index": len(lengths), "source_index": source_index,
                                 "id": str(row.get("_id", row.get("id", source_index))), "dataset": dataset,
                                 "format": fmt, "answers": answers, "all_classes": row.get("all_classes"),
                                 "prompt_tokens": len(r["prompt"]),
                                 "cap_removed_context_tokens": r["cap_removed_tokens"],
                                 "alignment_removed_context_tokens": r["alignment_removed_tokens"],
                                 "alignment_added_newline_tokens": r["padding_tokens"],
                                 "prefix_tokens": r["prefix_tokens"], "suffix_tokens": r["suffix_tokens"],
                                 "output_tokens": out_tokens,
                                 "fixed_output_horizon": fixed_output_tokens is not None},
                                ensure_ascii=False) + "\n")
            lengths.append(len(r["prompt"]))
            cap_rm.append(r["cap_removed_tokens"])
            align_rm.append(r["alignment_removed_tokens"])
            pads.append(r["padding_tokens"])
            if num_requests is not None and len(lengths) == num_requests:
                break
    if not lengths:
        raise ValueError("the dataset produced no requests")
    if num_requests is not None and len(lengths) != num_requests:
        raise ValueError(f"the dataset produced {len(lengths)} requests, expected {num_requests}")
    n = len(lengths)
    manifest = {"schema_version": 1, "status": "deterministic P/D request pack; no experiment result",
                "dataset": dataset, "format": fmt, "source": str(Path(dataset_path).resolve()),
                "tokenizer": tokenizer_name, "served_model_name": served_model_name, "prompt_mode": "official_chat",
                "thinking_mode": "disabled" if disable_thinking else "template_default",
                "context_truncation": "middle",
                "transport_alignment": "context trimmed down to whole chunks; padded only when trimming would "
                                       "remove the whole context",
                "alignment_padding_token_id": int(newline[0]), "chunk_tokens": chunk_tokens,
                "max_prompt_tokens": max_prompt_tokens, "fixed_output_tokens": fixed_output_tokens, "requests": n,
                "prompt_tokens": {"min": min(lengths), "max": max(lengths), "mean": sum(lengths) / n},
                "alignment_removed_context_tokens": {"max": max(align_rm), "mean": sum(align_rm) / n},
                "alignment_added_newline_tokens": {"max": max(pads), "mean": sum(pads) / n,
                                                   "affected_requests": sum(x > 0 for x in pads)},
                "cap_removed_context_tokens": {"max": max(cap_rm), "mean": sum(cap_rm) / n},
                "requests_sha256": _sha256(req_path), "metadata_sha256": _sha256(meta_path)}
    (output_dir / "manifest.json").write_text(json.dumps(manifest, indent=2, ensure_ascii=False) + "\n",
                                              encoding="utf-8")
    return manifest
