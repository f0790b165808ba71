"""Semantic feasibility runners: progressive KV visibility over one whole cache.

Two pre-experiments that ask whether a model that sees only part of the
document KV can draft tokens the full-KV model keeps, before any transfer or
timing machinery is involved:

``reuse`` mode (reference: experiments/progressive_kv_feasibility.py:1802-2079)
    The prefix and every document are encoded independently (keys relocated
    to their prompt positions); stage s sees the prefix plus the documents of
    the schedule's cumulative stage set, and the question suffix is prefilled
    after the view each time (with the generated history).  Controls: full
    prefill, a contiguous cache of prefix + documents, and full independent
    reuse (the exactness target of the chains).

``pd`` mode (reference: experiments/pd_progressive_kv_feasibility.py:94-371)
    One contiguous prefill of the whole prompt; stage s sees the prefix, the
    question suffix (the mandatory P/D anchor) and the stage's documents; the
    first ``seed_tokens`` tokens of the prefill side's greedy answer seed the
    decode side.  With an unbounded commit window the chain's output is
    audited against the full-KV target and a replay is charged when near-tied
    logits made them differ.

Command lines::

    python -m sparsecache_b200.pipelines.feasibility reuse --model M --dataset musique.jsonl --output r.jsonl
    python -m sparsecache_b200.pipelines.feasibility pd --model M --dataset musique.jsonl --output p.jsonl
    python -m sparsecache_b200.pipelines.feasibility aggregate r*.jsonl --output summary.json

``aggregate`` (reference: experiments/aggregate_progressive_kv.py,
experiments/aggregate_pd_progressive_kv.py) joins shards (duplicate dataset
indices are refused) and summarises either mode: baseline means, paired F1
diagnostics with bootstrap intervals, per-stage metrics, chain summaries,
the overlap-free latency model per link bandwidth and per-hop F1.

For every schedule (``serving.progressive.SCHEDULES``) each stage gets a
teacher-forced pass along the full-view target (top-1 agreement with the
final view and with the previous stage, strict survival of a position through
every later stage, mean target log-prob, mean top-1 margin: ``level_metrics``)
and ``serving.chains.progressive_commit_chain`` runs for every commit window.

B200 design: a stage's view is a slot map, the int32 indices of its visible
cache rows, and the view's past is the gather of those rows at their original
positions, the form the engine's paged attention reads; no [1, T] mask is
built and no invisible row enters the attention.  These runners measure
semantics, so they run on the plain-PyTorch oracle model (CPU or GPU); the
timed P/D and reuse pipelines run on the engine.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import random
import statistics
import time
from collections import defaultdict
from pathlib import Path
from typing import Any, Sequence

import torch

from ..metrics import answer_em, answer_f1, clean_short_answer, normalize_answer
from ..serving.chains import ChainPayload, progressive_commit_chain
from ..serving.progressive import (Document, encode_contiguous_cache, encode_independent_cache,
                                   pd_visibility_mask, prefix_visibility_mask, ranked_document_indices,
                                   stage_document_sets, visible_slot_map)

SYSTEM_PROMPT = ("You are a careful question-answering assistant. Answer the user's question using the "
                 "supplied documents. Return only the exact short answer without explanation.")


def _sync(device) -> None:
    if torch.device(device).type == "cuda":
        torch.cuda.synchronize(device)


def timed(device, fn):
    """(fn(), elapsed ms) with the device synchronised on both sides."""
    _sync(device)
    t = time.perf_counter()
    out = fn()
    _sync(device)
    return out, (time.perf_counter() - t) * 1e3


# ---------------------------------------------------------------- views
class ViewModel:
    """The oracle model over one base cache; views are slot maps of visible base rows.

    ``base_length`` is the width of the base cache; tokens run after a view
    (anchor ids, then history) take positions ``base_length, base_length+1, ...``
    whatever the view, as in the reference (static global positions).
    """

    def __init__(self, model, base_cache, base_length: int) -> None:
        self.model, self.cache, self.base_length = model, base_cache, int(base_length)
        self.device = model.device
        self._key: tuple | None = None
        self._past = None

    def _view(self, view: torch.Tensor):
        key = tuple(view.tolist())
        if key != self._key:
            idx = view.to(device=self.device, dtype=torch.long)
            self._past = tuple((k.index_select(2, idx), v.index_select(2, idx)) for k, v in self.cache)
            self._key = key
        return self._past, view.to(device=self.device, dtype=torch.long)

    @torch.no_grad()
    def _run(self, view, ids: Sequence[int], start: int, past=None, past_positions=None):
        if past is None:
            past, past_positions = self._view(view)
        ids_t = torch.tensor(list(ids), dtype=torch.long, device=self.device)
        pos = torch.arange(start, start + len(ids), device=self.device)
        hidden, cache = self.model.forward_tokens(ids_t, pos, past=past, past_positions=past_positions)
        return self.model.logits(hidden[0]).float(), cache, torch.cat((past_positions, pos))

    def continue_from_view(self, view, anchor_ids: Sequence[int], existing_ids: Sequence[int], *,
                           additional_tokens: int, eos_ids=frozenset(), return_margins: bool = False):
        """Prefill anchor + existing after the view, then greedy decode (reference feasibility:499-613)."""
        inputs = list(anchor_ids) + list(existing_ids)
        (logits, cache, kpos), prefill_ms = timed(self.device, lambda: self._run(view, inputs, self.base_length))
        generated, margins, decode_ms = [], [], 0.0
        last = logits[-1]
        position = self.base_length + len(inputs)
        for step in range(additional_tokens):
            if return_margins:
                top2 = last.topk(2).values
                margins.append(float(top2[0] - top2[1]))
            token = int(last.argmax())
            generated.append(token)
            if token in eos_ids or step + 1 == additional_tokens:
                break
            (lg, cache, kpos), ms = timed(self.device, lambda: self._run(
                None, [token], position, past=cache, past_positions=kpos))
            decode_ms += ms
            last = lg[-1]
            position += 1
        if return_margins:
            return generated, prefill_ms, decode_ms, margins
        return generated, prefill_ms, decode_ms

    def teacher_predictions(self, view, anchor_ids: Sequence[int], target_ids: Sequence[int]) -> dict[str, Any]:
        """One teacher-forced pass of anchor + target (reference feasibility:617-683)."""
        inputs = list(anchor_ids) + list(target_ids)
        (logits, _, _), ms = timed(self.device, lambda: self._run(view, inputs, self.base_length))
        start = len(anchor_ids) - 1
        scores = logits[start:start + len(target_ids)]
        lp = scores.log_softmax(-1)
        tgt = torch.tensor(list(target_ids), dtype=torch.long, device=scores.device)
        target_lp = lp.gather(1, tgt.unsqueeze(1)).squeeze(1).tolist()
        top2 = scores.topk(2, dim=-1).values
        margins = (top2[:, 0] - top2[:, 1]).tolist()
        return {"predictions": scores.argmax(-1).tolist(), "target_log_probs": target_lp, "top1_margins": margins,
                "mean_target_logprob": statistics.fmean(target_lp) if target_lp else 0.0,
                "mean_top1_margin": statistics.fmean(margins) if margins else 0.0, "forward_ms": ms}


class ViewStageModel:
    """``serving.chains.StageModel`` over a ViewModel: stage s = views[s], prompt = view + anchor ids."""

    def __init__(self, vm: ViewModel, views: Sequence[torch.Tensor], anchor_ids: Sequence[int],
                 eos_ids=frozenset()) -> None:
        self.vm, self.views, self.anchor, self.eos = vm, list(views), list(anchor_ids), set(eos_ids)
        self.n_stages = len(self.views)

    def verify(self, stage: int, sequence: Sequence[int]) -> list[int]:
        (logits, _, _) = self.vm._run(self.views[stage], self.anchor + list(sequence), self.vm.base_length)
        return logits[len(self.anchor) - 1:].argmax(-1).tolist()

    def draft(self, stage: int, sequence: Sequence[int], n: int) -> list[int]:
        if n <= 0:
            return []
        out, _, _ = self.vm.continue_from_view(self.views[stage], self.anchor, sequence, additional_tokens=n,
                                               eos_ids=self.eos)
        return out

    def final_decode(self, sequence: Sequence[int], n: int) -> list[int]:
        return self.draft(self.n_stages - 1, sequence, n)


# ---------------------------------------------------------------- metrics
def level_metrics(teacher_rows: Sequence[dict], target_ids: Sequence[int], stage_sets: Sequence[set[int]],
                  documents: Sequence[Document], fractions: Sequence[float]) -> list[dict[str, Any]]:
    """Per stage: agreement with the final view and the previous stage, strict survival, support coverage.

    Reference: experiments/progressive_kv_feasibility.py:1744-1799.
    """
    final = teacher_rows[-1]["predictions"]
    doc_tokens = sum(len(d.token_ids) for d in documents)
    support_tokens = sum(len(d.token_ids) for d in documents if d.supporting)

    def agree(a, b):
        pairs = list(zip(a, b))
        return statistics.fmean(x == y for x, y in pairs) if pairs else 1.0

    rows = []
    for s, (teacher, chosen, frac) in enumerate(zip(teacher_rows, stage_sets, fractions)):
        preds = teacher["predictions"]
        survival = [all(later["predictions"][p] == final[p] for later in teacher_rows[s:])
                    for p in range(len(target_ids))]
        rows.append({
            "stage": s, "configured_fraction": frac,
            "actual_document_fraction": sum(len(documents[i].token_ids) for i in chosen) / max(1, doc_tokens),
            "supporting_token_coverage": sum(len(documents[i].token_ids) for i in chosen if documents[i].supporting)
            / max(1, support_tokens),
            "adjacent_top1_agreement": None if s == 0 else agree(teacher_rows[s - 1]["predictions"], preds),
            "final_top1_agreement": agree(preds, final),
            "strict_final_survival": statistics.fmean(survival) if survival else 1.0,
            "mean_target_logprob": teacher["mean_target_logprob"],
            "mean_top1_margin": teacher["mean_top1_margin"],
            "teacher_forward_ms": teacher["forward_ms"]})
    return rows


def chain_record(payload: ChainPayload) -> dict[str, Any]:
    """A chain's result fields; ``draft_and_refresh_ms`` is all its model time except verification."""
    return {"trace": payload.trace, "draft_ms": payload.draft_ms, "verify_ms": payload.verify_ms,
            "final_decode_ms": payload.final_decode_ms,
            "draft_and_refresh_ms": payload.draft_ms + payload.final_decode_ms,
            "ignored_committed_flips": payload.ignored_committed_flips,
            "committed_token_checks": payload.committed_checks,
            "ignored_committed_flip_rate": payload.ignored_committed_flips / max(1, payload.committed_checks),
            "verifications": payload.verifications, "terminated_stage": payload.terminated_stage,
            "first_draft_batch_ms": payload.first_draft_ms, "first_committed_ms": payload.first_committed_ms}


def answer_scores(text: str, golds: Sequence[str]) -> tuple[float, float]:
    answer = clean_short_answer(text)
    return answer_em(answer, golds), answer_f1(answer, golds)


# ---------------------------------------------------------------- data
def stratified_indices(rows: Sequence[dict], count: int, seed: int) -> list[int]:
    """A seeded sample keeping the dataset's hop-count mix (largest-remainder quotas).

    Reference: experiments/progressive_kv_feasibility.py:136-161.
    """
    if count > len(rows):
        raise ValueError("sample count exceeds the dataset size")
    groups: dict[int, list[int]] = defaultdict(list)
    for i, row in enumerate(rows):
        groups[len(row.get("question_decomposition", []))].append(i)
    exact = {h: count * len(ix) / len(rows) for h, ix in groups.items()}
    quota = {h: min(len(groups[h]), math.floor(v)) for h, v in exact.items()}
    left = count - sum(quota.values())
    for h in sorted(groups, key=lambda h: exact[h] - quota[h], reverse=True):
        if left == 0:
            break
        if quota[h] < len(groups[h]):
            quota[h] += 1
            left -= 1
    rng = random.Random(seed)
    chosen = []
    for h, ix in sorted(groups.items()):
        ix = list(ix)
        rng.shuffle(ix)
        chosen += ix[:quota[h]]
    rng.shuffle(chosen)
    if len(chosen) != count:
        raise RuntimeError("could not build the stratified sample")
    return chosen


def tokenize_prompt(tokenizer, row: dict, answer_word_limit: int):
    """(prefix ids, documents with prompt spans, suffix ids) of a MuSiQue-style row.

    The chat template is rendered once around a placeholder; each paragraph is
    tokenised alone (reference: experiments/progressive_kv_feasibility.py:164-207).
    """
    placeholder = "{DOCUMENTS}"
    user = (f"<DOCUMENTS>\n{placeholder}\n</DOCUMENTS>\n\nQuestion: {row['question'].strip()}\n"
            f"Return only the exact short answer without explanation. Answer within {answer_word_limit} words.")
    rendered = tokenizer.apply_chat_template([{"role": "system", "content": SYSTEM_PROMPT},
                                              {"role": "user", "content": user}],
                                             tokenize=False, add_generation_prompt=True)
    pivot = rendered.index(placeholder)
    prefix = tuple(tokenizer.encode(rendered[:pivot], add_special_tokens=False))
    suffix = tuple(tokenizer.encode(rendered[pivot + len(placeholder):], add_special_tokens=False))
    docs, cursor = [], len(prefix)
    for p in row["paragraphs"]:
        title, text = p.get("title", "").strip(), p["paragraph_text"].strip()
        ids = tuple(tokenizer.encode(f"\n\nDocument:\n{title}\n{text}", add_special_tokens=False))
        docs.append(Document(ids, text=f"{title}\n{text}", supporting=bool(p.get("is_supporting", False)),
                             start=cursor, end=cursor + len(ids)))
        cursor += len(ids)
    return prefix, tuple(docs), suffix


# ---------------------------------------------------------------- runners
def full_prefill_generate(model, prompt: Sequence[int], *, max_new_tokens: int, eos_ids, device):
    """Greedy answer of one causal prefill: (ids, prefill ms, decode ms)."""
    vm = ViewModel(model, tuple(), 0)
    ids = torch.tensor(list(prompt), dtype=torch.long, device=model.device)
    (hidden, cache), prefill_ms = timed(device, lambda: model.forward_tokens(ids, torch.arange(len(prompt))))
    out, decode_ms = [], 0.0
    logits = model.logits(hidden[0, -1:]).float()[-1]
    kpos = torch.arange(len(prompt), device=model.device)
    for step in range(max_new_tokens):
        token = int(logits.argmax())
        out.append(token)
        if token in eos_ids or step + 1 == max_new_tokens:
            break
        (lg, cache, kpos), ms = timed(device, lambda: vm._run(None, [token], len(prompt) + step, past=cache,
                                                               past_positions=kpos))
        decode_ms += ms
        logits = lg[-1]
    return out, prefill_ms, decode_ms


def _schedules(vm: ViewModel, *, mode: str, row: dict, dataset_index: int, documents, prefix, suffix, anchor,
               target_tail, final_teacher, args, tokenizer, golds, eos_ids, reference_ids, replay_ms: float):
    out = {}
    for schedule in args.schedules:
        ranking = ranked_document_indices(schedule, question=row["question"], documents=documents,
                                          random_seed=args.seed + dataset_index)
        sets = stage_document_sets(ranking, documents, args.stage_fractions)
        if mode == "pd":
            masks = [pd_visibility_mask(len(prefix), documents, len(suffix), s) for s in sets]
        else:
            masks = [prefix_visibility_mask(len(prefix), documents, s) for s in sets]
        views = [visible_slot_map(m) for m in masks]
        teachers = [final_teacher if i == len(views) - 1 else vm.teacher_predictions(v, anchor, target_tail)
                    for i, v in enumerate(views)]
        stage_model = ViewStageModel(vm, views, anchor, eos_ids)
        # P/D: the seed tokens already count against the answer budget
        max_new = args.max_new_tokens - (len(anchor) if mode == "pd" else 0)
        chains = {}
        for window in args.commit_windows:
            payload = progressive_commit_chain(stage_model, commit_window=window, draft_tokens=args.draft_tokens,
                                               max_new_tokens=max_new, eos_ids=eos_ids)
            chain = chain_record(payload)
            tail = list(payload.tokens)
            if mode == "pd" and window is None:
                chain["pre_exact_replay_token_match"] = tail == list(target_tail)
                chain["exact_replay_required"] = float(tail != list(target_tail))
                chain["exact_replay_ms"] = replay_ms if tail != list(target_tail) else 0.0
                chain["draft_and_refresh_ms"] += chain["exact_replay_ms"]
                if tail != list(target_tail):
                    tail = list(target_tail)
            ids = (list(anchor) if mode == "pd" else []) + tail
            text = tokenizer.decode(ids, skip_special_tokens=True)
            ref_text = tokenizer.decode(reference_ids, skip_special_tokens=True)
            chain["answer"] = clean_short_answer(text)
            chain["em"], chain["f1"] = answer_scores(text, golds)
            key = "pd_target" if mode == "pd" else "fullreuse"
            chain[f"token_match_{key}"] = ids == list(reference_ids)
            chain[f"raw_match_{key}"] = text == ref_text
            chain[f"normalized_match_{key}"] = normalize_answer(text) == normalize_answer(ref_text)
            if window is None:
                chain["lossless_gate_pass"] = chain[f"token_match_{key}"]
            chains["inf" if window is None else str(window)] = chain
        levels = level_metrics(teachers, target_tail, sets, documents, args.stage_fractions)
        if mode == "pd":
            prompt_tokens = len(prefix) + len(suffix) + sum(len(d.token_ids) for d in documents)
            for level, chosen in zip(levels, sets):
                level["actual_total_kv_fraction"] = (len(prefix) + len(suffix) + sum(
                    len(documents[i].token_ids) for i in chosen)) / prompt_tokens
        out[schedule] = {"ranking": ranking, "levels": levels, "chains": chains}
    return out


def _bf16_kv_bytes(cache) -> int:
    return sum(k.numel() + v.numel() for k, v in cache) * 2


def evaluate_example(model, tokenizer, row: dict, dataset_index: int, args, *, mode: str) -> dict[str, Any]:
    device = model.device
    prefix, documents, suffix = tokenize_prompt(tokenizer, row, args.answer_word_limit)
    doc_ids = tuple(t for d in documents for t in d.token_ids)
    full_prompt = tuple(prefix) + doc_ids + tuple(suffix)
    eos_ids = set(args.eos_ids)
    golds = [row["answer"], *row.get("answer_aliases", [])]
    head = {"dataset_index": dataset_index, "id": row.get("id"),
            "hop_count": len(row.get("question_decomposition", [])), "question": row["question"],
            "gold_answers": golds, "document_count": len(documents), "document_tokens": len(doc_ids),
            "supporting_document_count": sum(bool(d.supporting) for d in documents),
            "supporting_document_tokens": sum(len(d.token_ids) for d in documents if d.supporting)}
    decode = lambda ids: tokenizer.decode(ids, skip_special_tokens=True)  # noqa: E731
    p_ids, p_prefill_ms, p_decode_ms = full_prefill_generate(model, full_prompt, max_new_tokens=args.max_new_tokens,
                                                            eos_ids=eos_ids, device=device)
    p_text = decode(p_ids)
    if mode == "pd":
        cache, producer_ms = timed(device, lambda: encode_contiguous_cache(model, full_prompt))
        vm = ViewModel(model, cache, len(full_prompt))
        full_view = visible_slot_map(pd_visibility_mask(len(prefix), documents, len(suffix), set(range(len(documents)))))
        seed_ids = list(p_ids[:args.seed_tokens])
        tail, seed_ms, dec_ms = vm.continue_from_view(full_view, seed_ids, (), eos_ids=eos_ids,
                                                      additional_tokens=args.max_new_tokens - len(seed_ids))
        target_ids = seed_ids + list(tail)
        final_teacher = vm.teacher_predictions(full_view, seed_ids, tail)
        t_text = decode(target_ids)
        agreement = statistics.fmean(p == g for p, g in zip(final_teacher["predictions"], tail)) if tail else 1.0
        schedules = _schedules(vm, mode=mode, row=row, dataset_index=dataset_index, documents=documents,
                               prefix=prefix, suffix=suffix, anchor=seed_ids, target_tail=tail,
                               final_teacher=final_teacher, args=args, tokenizer=tokenizer, golds=golds,
                               eos_ids=eos_ids, reference_ids=target_ids, replay_ms=seed_ms + dec_ms)
        em, f1 = answer_scores(p_text, golds)
        tem, tf1 = answer_scores(t_text, golds)
        out = {**head, "prompt_tokens": len(full_prompt), "anchor_tokens": len(prefix) + len(suffix),
               "logical_bf16_kv_bytes": _bf16_kv_bytes(cache),
               "prefill_side": {"answer": clean_short_answer(p_text), "token_ids": p_ids, "em": em, "f1": f1,
                                "prefill_ms": p_prefill_ms, "decode_ms": p_decode_ms,
                                "cache_producer_ms": producer_ms},
               "pd_target": {"answer": clean_short_answer(t_text), "token_ids": target_ids,
                             "seed_token_ids": seed_ids, "em": tem, "f1": tf1, "seed_forward_ms": seed_ms,
                             "decode_ms": dec_ms, "token_match_prefill_side": target_ids == p_ids,
                             "normalized_match_prefill_side": normalize_answer(t_text) == normalize_answer(p_text),
                             "teacher_self_top1_agreement": agreement},
               "schedules": schedules}
    else:
        contiguous = encode_contiguous_cache(model, tuple(prefix) + doc_ids)
        cvm = ViewModel(model, contiguous, len(prefix) + len(doc_ids))
        c_ids, c_ms, c_dec = cvm.continue_from_view(torch.arange(len(prefix) + len(doc_ids), dtype=torch.int32),
                                                    suffix, (), additional_tokens=args.max_new_tokens,
                                                    eos_ids=eos_ids)
        c_text = decode(c_ids)
        del contiguous, cvm
        cache, producer_ms = timed(device, lambda: encode_independent_cache(model, prefix, documents))
        vm = ViewModel(model, cache, len(prefix) + len(doc_ids))
        full_view = visible_slot_map(prefix_visibility_mask(len(prefix), documents, set(range(len(documents)))))
        r_ids, r_ms, r_dec = vm.continue_from_view(full_view, suffix, (), additional_tokens=args.max_new_tokens,
                                                   eos_ids=eos_ids)
        final_teacher = vm.teacher_predictions(full_view, suffix, r_ids)
        r_text = decode(r_ids)
        agreement = statistics.fmean(p == g for p, g in zip(final_teacher["predictions"], r_ids)) if r_ids else 1.0
        schedules = _schedules(vm, mode=mode, row=row, dataset_index=dataset_index, documents=documents,
                               prefix=prefix, suffix=suffix, anchor=list(suffix), target_tail=r_ids,
                               final_teacher=final_teacher, args=args, tokenizer=tokenizer, golds=golds,
                               eos_ids=eos_ids, reference_ids=r_ids, replay_ms=0.0)
        pem, pf1 = answer_scores(p_text, golds)
        rem, rf1 = answer_scores(r_text, golds)
        cem, cf1 = answer_scores(c_text, golds)
        out = {**head, "logical_bf16_kv_bytes": _bf16_kv_bytes(cache),
               "producer_ms": producer_ms,
               "fullprefill": {"answer": clean_short_answer(p_text), "token_ids": p_ids, "em": pem, "f1": pf1,
                               "prefill_ms": p_prefill_ms, "decode_ms": p_decode_ms},
               "fullreuse": {"answer": clean_short_answer(r_text), "token_ids": r_ids, "em": rem, "f1": rf1,
                             "prefill_ms": r_ms, "decode_ms": r_dec, "teacher_self_top1_agreement": agreement,
                             "raw_match_fullprefill": r_ids == p_ids,
                             "normalized_match_fullprefill": normalize_answer(r_text) == normalize_answer(p_text),
                             "raw_match_fullcontext_cache": r_ids == c_ids,
                             "normalized_match_fullcontext_cache": normalize_answer(r_text) == normalize_answer(c_text)},
               "fullcontext_cache": {"answer": clean_short_answer(c_text), "token_ids": c_ids, "em": cem, "f1": cf1,
                                     "prefill_ms": c_ms, "decode_ms": c_dec,
                                     "token_match_one_shot_fullprefill": c_ids == p_ids,
                                     "normalized_match_one_shot_fullprefill":
                                         normalize_answer(c_text) == normalize_answer(p_text)},
               "schedules": schedules}
    del cache, vm
    gc.collect()
    return out


# ---------------------------------------------------------------- aggregation
BANDWIDTHS_GIB_S = (1, 3, 6, 12, 25, 50)


def _mean(items, key):
    values = [float(x[key]) for x in items if x.get(key) is not None]
    return statistics.fmean(values) if values else None


def bootstrap_mean_ci(values: Sequence[float], *, samples: int = 10000, seed: int = 20260825):
    """Percentile 95% interval of the mean under resampling with replacement."""
    if not values:
        return None
    rng = random.Random(seed)
    n = len(values)
    est = sorted(sum(values[rng.randrange(n)] for _ in range(n)) / n for _ in range(samples))
    return [est[int(samples * 0.025)], est[int(samples * 0.975)]]


def paired_diagnostics(left: Sequence[float], right: Sequence[float]) -> dict[str, Any]:
    d = [a - b for a, b in zip(left, right)]
    tol = 1e-12
    return {"mean_delta": statistics.fmean(d) if d else None, "mean_delta_bootstrap_ci95": bootstrap_mean_ci(d),
            "wins": sum(x > tol for x in d), "ties": sum(abs(x) <= tol for x in d), "losses": sum(x < -tol for x in d)}


def ci95(values: Sequence[float]):
    return 1.96 * statistics.stdev(values) / len(values) ** 0.5 if len(values) >= 2 else None


def optimistic_timing(rows: Sequence[dict], schedule: str, window: str, *, mode: str) -> dict[str, Any]:
    """Idealised latency per link bandwidth (GiB/s): the whole KV then the target's compute, against
    the first tranche then max(rest of the KV the chain needed, the chain's compute), all overlap free.

    Reference: experiments/aggregate_progressive_kv.py:56-90 and aggregate_pd_progressive_kv.py:17-51.
    """
    frac_key = "actual_total_kv_fraction" if mode == "pd" else "actual_document_fraction"
    out = {}
    for bw in BANDWIDTHS_GIB_S:
        base, prog = [], []
        for row in rows:
            gib = row["logical_bf16_kv_bytes"] / 2 ** 30
            target = row["pd_target"] if mode == "pd" else row["fullreuse"]
            compute = (target["seed_forward_ms"] if mode == "pd" else target["prefill_ms"]) + target["decode_ms"]
            chain = row["schedules"][schedule]["chains"][window]
            levels = row["schedules"][schedule]["levels"]
            first = levels[0][frac_key]
            needed = levels[int(chain["terminated_stage"])][frac_key]
            base.append(gib / bw * 1e3 + compute)
            prog.append(gib * first / bw * 1e3 + max(gib * (needed - first) / bw * 1e3,
                                                     chain["draft_and_refresh_ms"] + chain["verify_ms"]))
        b, q = statistics.fmean(base), statistics.fmean(prog)
        out[str(bw)] = {"baseline_ms": b, "optimistic_progressive_ms": q, "speedup": b / q}
    return out


def summarize(rows: Sequence[dict]) -> dict[str, Any]:
    """Means, paired F1 diagnostics, per-stage metrics, chain summaries and per-hop F1 of runner rows."""
    if not rows:
        raise ValueError("no result rows")
    mode = "pd" if "pd_target" in rows[0] else "reuse"
    target_key = "pd_target" if mode == "pd" else "fullreuse"
    if mode == "pd":
        base = {"prefill_side": {k: _mean([r["prefill_side"] for r in rows], k)
                                 for k in ("em", "f1", "prefill_ms", "decode_ms", "cache_producer_ms")},
                "pd_target": {k: _mean([r["pd_target"] for r in rows], k)
                              for k in ("em", "f1", "seed_forward_ms", "decode_ms", "token_match_prefill_side",
                                        "normalized_match_prefill_side", "teacher_self_top1_agreement")}}
    else:
        base = {name: {k: _mean([r[name] for r in rows], k) for k in ("em", "f1", "prefill_ms", "decode_ms")}
                for name in ("fullprefill", "fullcontext_cache", "fullreuse")}
        fr = [r["fullreuse"] for r in rows]
        for k in ("raw_match_fullprefill", "normalized_match_fullprefill", "raw_match_fullcontext_cache",
                  "normalized_match_fullcontext_cache", "teacher_self_top1_agreement"):
            base["fullreuse"][k] = _mean(fr, k)
        fc = [r["fullcontext_cache"] for r in rows]
        for k in ("token_match_one_shot_fullprefill", "normalized_match_one_shot_fullprefill"):
            base["fullcontext_cache"][k] = _mean(fc, k)
        base["fullcontext_cache"]["f1_vs_one_shot_fullprefill"] = paired_diagnostics(
            [r["fullcontext_cache"]["f1"] for r in rows], [r["fullprefill"]["f1"] for r in rows])
        base["fullreuse"]["f1_vs_fullcontext_cache"] = paired_diagnostics(
            [r["fullreuse"]["f1"] for r in rows], [r["fullcontext_cache"]["f1"] for r in rows])
        correct = [r for r in rows if r["fullcontext_cache"]["em"] == 1]
        lost = sum(r["fullreuse"]["em"] == 0 for r in correct)
        base["fullreuse"]["fullcontext_correct_to_fullreuse_wrong"] = {
            "count": lost, "denominator": len(correct), "rate": lost / len(correct) if correct else None}
    level_keys = ("configured_fraction", "actual_document_fraction", "actual_total_kv_fraction",
                  "supporting_token_coverage", "adjacent_top1_agreement", "final_top1_agreement",
                  "strict_final_survival", "mean_target_logprob", "mean_top1_margin", "teacher_forward_ms")
    chain_keys = ("em", "f1", f"token_match_{target_key}", f"raw_match_{target_key}",
                  f"normalized_match_{target_key}", "draft_and_refresh_ms", "verify_ms",
                  "ignored_committed_flip_rate", "terminated_stage")
    schedules = {}
    for sched in rows[0]["schedules"]:
        n_levels = len(rows[0]["schedules"][sched]["levels"])
        levels = []
        for i in range(n_levels):
            vals = [r["schedules"][sched]["levels"][i] for r in rows]
            levels.append({k: _mean(vals, k) for k in level_keys if k in vals[0]})
        chains = {}
        for window in rows[0]["schedules"][sched]["chains"]:
            vals = [r["schedules"][sched]["chains"][window] for r in rows]
            f1 = [v["f1"] for v in vals]
            c = {k: _mean(vals, k) for k in chain_keys}
            c["f1_ci95"] = ci95(f1)
            c[f"f1_vs_{target_key}"] = paired_diagnostics(f1, [r[target_key]["f1"] for r in rows])
            if mode == "reuse":
                c["f1_vs_fullcontext_cache"] = paired_diagnostics(f1, [r["fullcontext_cache"]["f1"] for r in rows])
                c["fullreuse_correct_to_chain_wrong"] = sum(r["fullreuse"]["em"] == 1 and v["em"] == 0
                                                            for r, v in zip(rows, vals))
                c["fullreuse_wrong_to_chain_correct"] = sum(r["fullreuse"]["em"] == 0 and v["em"] == 1
                                                            for r, v in zip(rows, vals))
            elif window == "inf":
                c["pre_exact_replay_token_match"] = _mean(vals, "pre_exact_replay_token_match")
                c["exact_replay_rate"] = _mean(vals, "exact_replay_required")
                c["exact_replay_ms"] = _mean(vals, "exact_replay_ms")
                c["lossless_gate_pass"] = _mean(vals, "lossless_gate_pass")
            needed = [r["schedules"][sched]["levels"][int(v["terminated_stage"])] for r, v in zip(rows, vals)]
            c["mean_required_document_fraction"] = _mean(needed, "actual_document_fraction")
            if mode == "pd":
                c["mean_required_total_kv_fraction"] = _mean(needed, "actual_total_kv_fraction")
            c["optimistic_timing_by_bandwidth_gib_s"] = optimistic_timing(rows, sched, window, mode=mode)
            chains[window] = c
        schedules[sched] = {"levels": levels, "chains": chains}
    groups: dict[int, list[dict]] = defaultdict(list)
    for r in rows:
        groups[r["hop_count"]].append(r)
    by_hop = {}
    for hop, g in sorted(groups.items()):
        entry = {"cases": len(g), f"{target_key}_f1": _mean([r[target_key] for r in g], "f1"),
                 "chains": {s: {w: _mean([r["schedules"][s]["chains"][w] for r in g], "f1")
                                for w in g[0]["schedules"][s]["chains"]} for s in g[0]["schedules"]}}
        if mode == "reuse":
            entry["fullprefill_f1"] = _mean([r["fullprefill"] for r in g], "f1")
        by_hop[str(hop)] = entry
    out = {"mode": mode, "cases": len(rows), "hop_counts": {str(h): len(g) for h, g in sorted(groups.items())},
           "mean_document_tokens": _mean(rows, "document_tokens"),
           "mean_supporting_document_tokens": _mean(rows, "supporting_document_tokens"),
           "mean_logical_bf16_kv_mib": _mean(rows, "logical_bf16_kv_bytes") / 2 ** 20,
           "base": base, "schedules": schedules, "by_hop": by_hop}
    if mode == "pd":
        out.update(mean_prompt_tokens=_mean(rows, "prompt_tokens"), mean_anchor_tokens=_mean(rows, "anchor_tokens"))
    return out


def aggregate_main(argv=None) -> dict[str, Any]:
    p = argparse.ArgumentParser(prog="feasibility aggregate")
    p.add_argument("inputs", nargs="+")
    p.add_argument("--output", required=True)
    a = p.parse_args(argv)
    rows = []
    for name in a.inputs:
        rows += [json.loads(x) for x in Path(name).read_text(encoding="utf-8").splitlines() if x.strip()]
    if not rows:
        raise ValueError("no result rows found")
    idx = [r["dataset_index"] for r in rows]
    if len(idx) != len(set(idx)):
        raise ValueError("duplicate dataset indices across shards")
    payload = {"protocol": rows[0]["protocol"], "source_files": [str(Path(x).resolve()) for x in a.inputs],
               "summary": summarize(rows), "rows": rows}
    out = Path(a.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(payload, ensure_ascii=False, indent=2) + "\n")
    print(json.dumps(payload["summary"], ensure_ascii=False, indent=2))
    return payload


def parse_windows(text: str) -> list[int | None]:
    """``"1,2,inf"`` -> [1, 2, None] (None = commit only at the final stage)."""
    out = []
    for part in text.split(","):
        part = part.strip()
        if part:
            out.append(None if part in ("inf", "none") else int(part))
    return out


def main(argv=None) -> None:
    import sys

    from ..models.checkpoint import load_oracle
    from ..tokenizer import load_tokenizer

    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "aggregate":
        aggregate_main(argv[1:])
        return
    p = argparse.ArgumentParser()
    p.add_argument("mode", choices=("reuse", "pd"))
    p.add_argument("--model", required=True, help="model directory (config.json + model.safetensors)")
    p.add_argument("--dataset", required=True, help="MuSiQue-style JSONL (question, answer, paragraphs)")
    p.add_argument("--output", required=True)
    p.add_argument("--sample-count", type=int, default=100)
    p.add_argument("--offset", type=int, default=0)
    p.add_argument("--count", type=int, default=None)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--stage-fractions", default="0.25,0.5,0.75,1.0")
    p.add_argument("--schedules", default="sequential,uniform,query,oracle,random")
    p.add_argument("--commit-windows", default="1,2,inf")
    p.add_argument("--draft-tokens", type=int, default=4)
    p.add_argument("--max-new-tokens", type=int, default=16)
    p.add_argument("--seed-tokens", type=int, default=1)
    p.add_argument("--answer-word-limit", type=int, default=5)
    p.add_argument("--device", default="cuda")
    p.add_argument("--dtype", choices=("bfloat16", "float32"), default="bfloat16")
    p.add_argument("--overwrite", action="store_true")
    a = p.parse_args(argv)
    a.stage_fractions = [float(x) for x in a.stage_fractions.split(",")]
    if a.stage_fractions[-1] != 1.0 or any(x >= y for x, y in zip(a.stage_fractions, a.stage_fractions[1:])):
        raise ValueError("stage fractions must increase and end at 1.0")
    a.schedules = [s for s in a.schedules.split(",") if s]
    a.commit_windows = parse_windows(a.commit_windows)
    out_path = Path(a.output)
    if out_path.exists() and not a.overwrite:
        raise FileExistsError(f"{out_path} exists; pass --overwrite")
    out_path.parent.mkdir(parents=True, exist_ok=True)
    rows = [json.loads(x) for x in Path(a.dataset).read_text(encoding="utf-8").splitlines() if x.strip()]
    chosen = stratified_indices(rows, a.sample_count, a.seed)
    count = a.count if a.count is not None else len(chosen) - a.offset
    if a.offset < 0 or a.offset + count > len(chosen):
        raise ValueError("invalid sample shard")
    model = load_oracle(a.model, dtype=getattr(torch, a.dtype), device=a.device)
    cfg = model.config
    a.eos_ids = tuple(cfg.eos_token_ids)
    tokenizer = load_tokenizer(a.model, cfg.vocab, cfg.n_special, cfg.eos_token_ids)
    protocol = {"experiment": "progressive-kv-feasibility" if a.mode == "reuse" else "pd-progressive-full-context-kv",
                "model": str(Path(a.model).resolve()), "dataset": str(Path(a.dataset).resolve()),
                "sample_count": a.sample_count, "sample_seed": a.seed, "shard_offset": a.offset,
                "shard_count": count, "stage_fractions": a.stage_fractions, "schedules": a.schedules,
                "commit_windows": ["inf" if w is None else w for w in a.commit_windows],
                "draft_tokens": a.draft_tokens, "decoding": "greedy", "static_global_positions": True,
                "representation_refresh": "all generated token identities",
                "cache_source": ("single contiguous full-prompt prefill" if a.mode == "pd"
                                 else "independent documents, keys relocated"),
                "view": "slot map of visible cache rows"}
    if a.mode == "pd":
        protocol.update(seed_tokens_from_prefill_side=a.seed_tokens,
                        mandatory_first_stream="system/chat prefix plus query KV",
                        progressive_stream="document token regions")
    with out_path.open("w", encoding="utf-8") as f:
        for k, index in enumerate(chosen[a.offset:a.offset + count]):
            result = evaluate_example(model, tokenizer, rows[index], index, a, mode=a.mode)
            result["protocol"] = protocol
            f.write(json.dumps(result, ensure_ascii=False) + "\n")
            f.flush()
            print(json.dumps({"event": "example_complete", "local": k + 1, "count": count,
                              "dataset_index": index, "hop_count": result["hop_count"]}), flush=True)
    print(json.dumps({"event": "complete", "output": str(out_path)}), flush=True)


if __name__ == "__main__":
    main()
