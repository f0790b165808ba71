"""CacheBlend reuse pipeline: one-shot and progressive repair, paired driver, aggregation.

Parity with the reference's experiments/reuse_cacheblend_pipeline.py:
  * ``expand_documents`` (:239-273): proportional document repetition up to a
    token target, for scale sweeps (timing only);
  * ``prepare_request`` (:276-319): rank documents by a schedule (BM25 over
    the question by default), lay them out in ranked order, and compute the
    cumulative staged document sets of the stage fractions;
  * ``run_progressive_cacheblend`` (:896-1141): documents arrive in stages;
    every stage is a CacheBlend repair of the cache with only that stage's
    documents present (absent documents are zero placeholders); stage 0
    drafts, later stages verify + commit with a commit window of 1, the final
    stage commits and corrects, then decoding continues on the full repair;
  * ``evaluate_request`` / ``main`` (:1144-1334): paired measurement of full
    prefill, one-shot CacheBlend and progressive CacheBlend per request after
    a warm-up, written as JSONL with a protocol block;
  * ``aggregate`` (experiments/aggregate_reuse_cacheblend_pipeline.py:46-229):
    token agreement with full prefill, TTFT and end-to-end latency
    distributions, paired bootstrap of the latency differences.
The documents' K/V blocks wait in pinned host memory (``--store-tier
pinned``, the reference's CPU tier): the one-shot arm composes them over PCIe
inside the request, and the progressive arm stages each stage's new
documents H2D on a copy stream (``serving.doc_stager``), overlapped with the
previous stage's work or serially, and compares the two.  The stage model
runs this package's engine (composer, CacheBlend kernels, batched verifier).
"""
from __future__ import annotations

import argparse
import json
import math
import statistics
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Sequence

import torch

from ..config import DEVIATION_METRICS
from ..serving.chains import progressive_commit_chain
from ..serving.progressive import Document, ranked_document_indices, stage_document_sets
from ..synthetic import RAGRequest


def expand_documents(documents: Sequence[Sequence[int]], target_tokens: int, prefix_tokens: int = 0):
    """Repeat documents proportionally until the prompt reaches ``target_tokens`` (timing sweeps)."""
    docs = [list(d) for d in documents]
    have = prefix_tokens + sum(map(len, docs))
    if have >= target_tokens or not docs:
        return docs
    factor = target_tokens / max(1, have - prefix_tokens)
    out = []
    for d in docs:
        reps = max(1, math.floor(factor))
        out.append(d * reps)
    i = 0
    while prefix_tokens + sum(map(len, out)) < target_tokens:
        out[i % len(out)] += docs[i % len(docs)]
        i += 1
    return out


@dataclass
class PreparedRequest:
    request: RAGRequest
    ranking: list[int]
    selected_sets: list[set[int]]
    stage_fractions: tuple[float, ...]


def prepare_request(request: RAGRequest, *, question: str = "", schedule: str = "query",
                    fractions: Sequence[float] = (0.25, 0.5, 1.0), seed: int = 0,
                    texts: Sequence[str] | None = None,
                    supporting: Sequence[bool | None] | None = None) -> PreparedRequest:
    """Rank the request's documents, re-lay them in ranked order, stage them cumulatively."""
    docs = [Document(tuple(d), texts[i] if texts else " ".join(map(str, d[:64])),
                     supporting=supporting[i] if supporting else None)
            for i, d in enumerate(request.documents)]
    ranking = ranked_document_indices(schedule, question=question or " ".join(map(str, request.suffix)),
                                      documents=docs, random_seed=seed)
    laid = RAGRequest(request.index, request.prefix, tuple(request.documents[i] for i in ranking), request.suffix)
    ranked_docs = [Document(tuple(d)) for d in laid.documents]
    sets = stage_document_sets(list(range(len(ranking))), ranked_docs, fractions)
    return PreparedRequest(laid, ranking, sets, tuple(fractions))


class EngineStageModel:
    """Stage s = CacheBlend repair of the prompt that holds only the documents arrived by stage s.

    The stage prompt is prefix + ranked documents[:count_s] + question suffix,
    with the suffix (and every appended token) at its FINAL global position,
    so drafts made at an early stage line up with the full prompt; the
    documents' K/V come from the ``PinnedDocumentStager`` arena (HBM) after
    the stage's copy event.  ``verify``/``draft``/``final_decode`` append the
    given token sequence with the batched verifier (8 rows a pass) behind the
    stage's repaired prompt, through an identity slot map so the appended
    rows sit right after the stage's slots while their RoPE positions are
    global (reference cacheblend_repair with final_prompt_tokens,
    experiments/reuse_cacheblend_pipeline.py:512-706).
    """

    def __init__(self, server, prepared: PreparedRequest, *, stager, overlap: bool = True) -> None:
        self.server, self.eng = server, server.engine
        self.req = prepared.request
        self.sets = prepared.selected_sets
        self.n_stages = len(self.sets)
        self.stager = stager
        self.overlap = overlap
        self.T = self.req.prompt_tokens
        self.slot = server.slot
        dev = self.eng.device
        self.view = torch.arange(self.slot.capacity, dtype=torch.int32, device=dev)
        self._stage = None
        self._first = None
        self._len = 0
        self._appended: list[int] = []
        self.repairs = 0

    def _stage_prompt(self, stage: int):
        req = self.req
        count = len(self.sets[stage])
        docs = req.documents[:count]
        body = tuple(req.prefix) + tuple(t for d in docs for t in d)
        ids = body + tuple(req.suffix)
        S = len(req.suffix)
        gpos = list(range(len(body))) + list(range(self.T - S, self.T))
        dev = self.eng.device
        return (torch.tensor(ids, dtype=torch.int32, device=dev), torch.tensor(gpos, dtype=torch.int32, device=dev),
                len(ids))

    def _repair(self, stage: int) -> None:
        if self._stage == stage:
            return
        eng, req = self.eng, self.req
        blend = self.server.blend
        self.stager.arrive(stage, overlap=self.overlap)
        ids, gpos, n = self._stage_prompt(stage)
        eng.compose(self.slot, self.stager.blocks(stage), first_slot=len(req.prefix), layer_begin=blend.check_layer)
        h_a, A, _ = eng.cacheblend(ids, self.slot, prefix_tokens=len(req.prefix), suffix_tokens=len(req.suffix),
                                   blend=blend, global_positions=gpos)
        b = eng.first_token(h_a[A - 1:A], position=self.T, max_new=1)
        self._first = int(b["tok"][0].item())
        self._stage, self._len, self._appended = stage, n, []
        self.repairs += 1

    def _append(self, seq: Sequence[int]) -> list[int]:
        """Predictions after each appended token (rows beyond the cached common prefix)."""
        common = 0
        while common < min(len(seq), len(self._appended)) and seq[common] == self._appended[common]:
            common += 1
        preds = []
        self._appended = self._appended[:common]
        for k in range(common, len(seq), 8):
            chunk = list(seq[k:k + 8])
            out = self.eng.verify(self.slot, torch.tensor(chunk, dtype=torch.int32, device=self.eng.device),
                                  position=self.T + k, slot_start=self._len + k, view=self.view,
                                  n_visible=self._len + k)
            preds += out.cpu().tolist()
            self._appended += chunk
        return preds

    def _preds_all(self, seq: Sequence[int]) -> list[int]:
        self._appended = []  # recompute the whole tail (verifier state is positional)
        return [self._first] + self._append(seq)

    def verify(self, stage: int, sequence: Sequence[int]) -> list[int]:
        self._repair(stage)
        return self._preds_all(sequence)

    def draft(self, stage: int, sequence: Sequence[int], n: int) -> list[int]:
        self._repair(stage)
        nxt = self._preds_all(sequence)[-1]
        out, seq = [], list(sequence)
        for _ in range(n):
            out.append(nxt)
            seq.append(nxt)
            nxt = self._append(seq)[-1]
        return out

    def final_decode(self, sequence: Sequence[int], n: int) -> list[int]:
        return self.draft(self.n_stages - 1, sequence, n)


def host_blocks(server, request: RAGRequest, pinned_store=None) -> list[torch.Tensor]:
    """Pinned host copies of the request's document blocks (the reuse pipeline's CPU tier)."""
    out = []
    for d in request.documents:
        if pinned_store is not None and d in pinned_store:
            out.append(pinned_store[d].kv)
            continue
        block = server.store[d].kv
        out.append(block if block.device.type == "cpu" and block.is_pinned() else block.cpu().pin_memory())
    return out


def run_progressive_cacheblend(server, prepared: PreparedRequest, blocks_host, *, draft_tokens: int,
                               max_new_tokens: int, eos_ids=frozenset(), overlap: bool = True) -> dict[str, Any]:
    """One progressive run with the documents staged from pinned host memory (overlapped or serial)."""
    from ..serving.doc_stager import PinnedDocumentStager

    eng = server.engine
    torch.cuda.synchronize(eng.device)
    t0 = time.perf_counter()
    stager = PinnedDocumentStager(blocks_host, prepared.selected_sets, device=eng.device,
                                  layer_begin=server.blend.check_layer)
    model = EngineStageModel(server, prepared, stager=stager, overlap=overlap)
    out = progressive_commit_chain(model, commit_window=1, draft_tokens=draft_tokens, max_new_tokens=max_new_tokens,
                                   eos_ids=set(eos_ids))
    torch.cuda.synchronize(eng.device)
    response_ms = (time.perf_counter() - t0) * 1e3
    return {"tokens": out.tokens, "response_ms": response_ms,
            "first_draft_ms": out.first_draft_ms, "first_committed_ms": out.first_committed_ms,
            "verify_ms": out.verify_ms, "draft_ms": out.draft_ms, "final_decode_ms": out.final_decode_ms,
            "ignored_committed_flips": out.ignored_committed_flips, "stages": model.n_stages,
            "repairs": model.repairs, "trace": out.trace, "transfer": stager.finish(), "overlap": overlap}


def evaluate_request(server, prepared: PreparedRequest, *, max_new_tokens: int, draft_tokens: int = 8,
                     modes: Sequence[str] = ("full", "cacheblend", "progressive"), pinned_store=None,
                     serial: bool = True) -> dict[str, Any]:
    """Paired arms of one request: device-timed TTFT and end-to-end latency per arm.

    The progressive arm stages its documents from pinned host memory on a
    copy stream; with ``serial`` it runs a second time with each stage's copy
    started only when the stage begins, and the row records both response
    times and whether the two produced the same tokens (they must).
    """
    req = prepared.request
    row: dict[str, Any] = {"request_index": req.index, "prompt_tokens": req.prompt_tokens,
                           "document_tokens": req.document_tokens, "arms": {}}
    for mode in modes:
        if mode == "progressive":
            blocks = host_blocks(server, req, pinned_store)
            res = run_progressive_cacheblend(server, prepared, blocks, draft_tokens=draft_tokens,
                                             max_new_tokens=max_new_tokens, eos_ids=server.eos, overlap=True)
            arm = {"tokens": res["tokens"], "ttft_ms": res["first_committed_ms"],
                   "first_draft_ms": res["first_draft_ms"], "e2e_ms": res["response_ms"],
                   "ignored_committed_flips": res["ignored_committed_flips"], "transfer": res["transfer"]}
            if serial:
                ser = run_progressive_cacheblend(server, prepared, blocks, draft_tokens=draft_tokens,
                                                 max_new_tokens=max_new_tokens, eos_ids=server.eos, overlap=False)
                arm.update(serial_response_ms=ser["response_ms"],
                           serial_pipeline_token_match=ser["tokens"] == res["tokens"],
                           serial_transfer=ser["transfer"])
            row["arms"][mode] = arm
        elif mode == "cacheblend" and pinned_store is not None:
            # one-shot CacheBlend from the pinned tier: the composer reads the
            # host blocks over PCIe inside the timed request
            r = server.serve(req, mode=mode, store=pinned_store, max_new_tokens=max_new_tokens, sync=True)
            row["arms"][mode] = {"tokens": list(r.token_ids), "ttft_ms": r.ttft_ms, "e2e_ms": r.response_ms,
                                 "store_tier": "pinned"}
        else:
            r = server.serve(req, mode=mode, max_new_tokens=max_new_tokens, sync=True)
            row["arms"][mode] = {"tokens": list(r.token_ids), "ttft_ms": r.ttft_ms, "e2e_ms": r.response_ms}
    return row


# ------------------------------------------------------------------ aggregate
def _pct(v, q):
    v = sorted(v)
    if not v:
        return math.nan
    pos = q * (len(v) - 1)
    lo, hi = math.floor(pos), math.ceil(pos)
    return v[lo] + (v[hi] - v[lo]) * (pos - lo)


def _boot(values, samples=10000, seed=0):
    import random

    if not values:
        return [math.nan, math.nan]
    rng = random.Random(seed)
    est = sorted(statistics.fmean(rng.choices(values, k=len(values))) for _ in range(samples))
    return [_pct(est, 0.025), _pct(est, 0.975)]


def aggregate(rows: Sequence[dict], *, reference: str = "full", bootstrap_samples: int = 10000) -> dict[str, Any]:
    """Token agreement with the reference arm, latency distributions, paired bootstrap of differences."""
    arms = sorted({a for r in rows for a in r["arms"]})
    out: dict[str, Any] = {"requests": len(rows), "reference_arm": reference, "arms": {}}
    for a in arms:
        rr = [r for r in rows if a in r["arms"] and reference in r["arms"]]
        ttft = [r["arms"][a]["ttft_ms"] for r in rr if r["arms"][a]["ttft_ms"] is not None]
        e2e = [r["arms"][a]["e2e_ms"] for r in rr]
        agree = [r["arms"][a]["tokens"] == r["arms"][reference]["tokens"] for r in rr]
        prefix = [next((i for i, (x, y) in enumerate(zip(r["arms"][a]["tokens"], r["arms"][reference]["tokens"]))
                        if x != y), len(r["arms"][a]["tokens"])) for r in rr]
        d_ttft = [r["arms"][reference]["ttft_ms"] - r["arms"][a]["ttft_ms"] for r in rr
                  if r["arms"][a]["ttft_ms"] is not None]
        out["arms"][a] = {
            "token_equal_rate": statistics.fmean(agree) if agree else math.nan,
            "mean_agreeing_prefix": statistics.fmean(prefix) if prefix else math.nan,
            "ttft_ms": {"p50": _pct(ttft, 0.5), "p99": _pct(ttft, 0.99), "mean": statistics.fmean(ttft) if ttft
                        else math.nan},
            "e2e_ms": {"p50": _pct(e2e, 0.5), "p99": _pct(e2e, 0.99)},
            "ttft_gain_vs_reference_ms": {"mean": statistics.fmean(d_ttft) if d_ttft else math.nan,
                                          "ci95": _boot(d_ttft, bootstrap_samples)},
        }
        serial = [r["arms"][a] for r in rr if "serial_response_ms" in r["arms"][a]]
        if serial:  # overlapped vs serial staging of the progressive arm
            gains = [x["serial_response_ms"] - x["e2e_ms"] for x in serial]
            out["arms"][a]["serial_staging"] = {
                "serial_e2e_ms": {"p50": _pct([x["serial_response_ms"] for x in serial], 0.5)},
                "overlap_gain_ms": {"mean": statistics.fmean(gains), "ci95": _boot(gains, bootstrap_samples)},
                "token_match_rate": statistics.fmean(bool(x["serial_pipeline_token_match"]) for x in serial),
                "h2d_ms_mean": statistics.fmean(x["transfer"]["total_h2d_ms"] for x in serial)}
        scored = [r["arms"][a] for r in rr if "f1" in r["arms"][a]]
        if scored:  # dataset runs: short-answer quality
            out["arms"][a].update(em=statistics.fmean(x["em"] for x in scored),
                                  f1=statistics.fmean(x["f1"] for x in scored))
    return out


def blend_config_from_args(a) -> "CacheBlendConfig":
    """CacheBlendConfig of the runner flags (single check layer, or the gradual schedule)."""
    from ..config import CacheBlendConfig

    common = dict(deviation_metric=a.deviation_metric, max_new_tokens=a.max_new_tokens,
                  target_average_recompute_ratio=a.target_average_recompute_ratio)
    if a.blend_check_layers or a.recompute_ratios:
        if not (a.blend_check_layers and a.recompute_ratios):
            raise SystemExit("--blend-check-layers and --recompute-ratios go together")
        layers = tuple(int(x) for x in a.blend_check_layers.split(","))
        ratios = tuple(float(x) for x in a.recompute_ratios.split(","))
        return CacheBlendConfig(check_layers=layers, recompute_ratios=ratios, **common)
    return CacheBlendConfig(check_layer=a.check_layer, recompute_ratio=a.recompute_ratio, **common)


def dataset_requests(path: Path, cfg, *, model_dir=None, sample_count: int | None = None, seed: int = 0,
                     answer_word_limit: int = 5, limit: int | None = None) -> tuple[list[RAGRequest], list[dict]]:
    """Requests (prefix, one document per paragraph, question suffix) of a MuSiQue-style JSONL.

    Rows are a hop-stratified seeded sample (``sample_count``; all rows when
    None); the prompt is rendered with the model directory's tokenizer (the
    byte tokenizer of this package for random-init presets).  The metadata
    keeps the question, the paragraph texts and supporting flags (for the
    query and oracle schedules), the gold answers and a decoder.
    """
    from ..tokenizer import ByteTokenizer, load_tokenizer
    from .feasibility import stratified_indices, tokenize_prompt

    rows = [json.loads(x) for x in Path(path).read_text(encoding="utf-8").splitlines() if x.strip()]
    order = stratified_indices(rows, sample_count, seed) if sample_count else list(range(len(rows)))
    if limit is not None:
        order = order[:limit]
    if model_dir is not None:
        tok = load_tokenizer(model_dir, cfg.vocab, max(cfg.n_special, 4), cfg.eos_token_ids)
    else:
        tok = ByteTokenizer(cfg.vocab, n_special=max(cfg.n_special, 4),
                            eos_token_id=cfg.eos_token_ids[0] if cfg.eos_token_ids else 2)
    reqs, meta = [], []
    for index in order:
        row = rows[index]
        prefix, docs, suffix = tokenize_prompt(tok, row, answer_word_limit)
        reqs.append(RAGRequest(index, tuple(prefix), tuple(tuple(d.token_ids) for d in docs), tuple(suffix)))
        meta.append({"question": row["question"], "texts": [d.text for d in docs],
                     "supporting": [bool(d.supporting) for d in docs],
                     "golds": [row["answer"], *row.get("answer_aliases", [])],
                     "decode": lambda ids, _t=tok: _t.decode(ids, skip_special_tokens=True)})
    return reqs, meta


def score_row(row: dict[str, Any], meta: dict, eos_ids) -> None:
    """Short-answer EM / F1 of every arm's tokens against the row's gold answers (in place)."""
    from ..metrics import answer_em, answer_f1, clean_short_answer

    row["gold_answers"] = meta["golds"]
    for arm in row["arms"].values():
        toks = [t for t in arm["tokens"]]
        for k, t in enumerate(toks):
            if t in eos_ids:
                toks = toks[:k]
                break
        ans = clean_short_answer(meta["decode"](toks))
        arm.update(answer=ans, em=answer_em(ans, meta["golds"]), f1=answer_f1(ans, meta["golds"]))


def aggregate_main(argv=None) -> dict[str, Any]:
    """Aggregate run files (reference: experiments/aggregate_reuse_cacheblend_pipeline.py:46-229).

    Protocol lines are skipped; a request index seen twice across shards is refused.
    """
    p = argparse.ArgumentParser(prog="reuse aggregate")
    p.add_argument("inputs", nargs="+", type=Path)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--reference-arm", default="full")
    p.add_argument("--bootstrap-samples", type=int, default=10000)
    a = p.parse_args(argv)
    rows, protocols = [], []
    for path in a.inputs:
        for line in path.read_text(encoding="utf-8").splitlines():
            if not line.strip():
                continue
            obj = json.loads(line)
            (protocols if "protocol" in obj else rows).append(obj.get("protocol", obj))
    if not rows:
        raise ValueError("no result rows found")
    idx = [r["request_index"] for r in rows]
    if len(idx) != len(set(idx)):
        raise ValueError("duplicate request indices across shards")
    out = {"protocol": protocols[0] if protocols else None, "source_files": [str(x.resolve()) for x in a.inputs],
           "summary": aggregate(rows, reference=a.reference_arm, bootstrap_samples=a.bootstrap_samples)}
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(out, indent=2, default=float) + "\n")
    print(json.dumps(out["summary"], indent=2, default=float))
    return out


def main(argv=None) -> None:
    from ..config import get_model_config
    from ..models.engine import B200Engine
    from ..serving.server import RAGServer
    from ..store import DocumentKVStore
    from ..synthetic import make_requests

    import sys

    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "aggregate":
        aggregate_main(argv[1:])
        return
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--workload", default="llama8b_rag")
    p.add_argument("--requests", type=int, default=16)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--max-new-tokens", type=int, default=24)
    p.add_argument("--draft-tokens", type=int, default=8)
    p.add_argument("--fractions", default="0.25,0.5,1.0")
    p.add_argument("--schedule", default="query")
    p.add_argument("--recompute-ratio", type=float, default=0.15)
    p.add_argument("--check-layer", "--blend-check-layer", dest="check_layer", type=int, default=1)
    p.add_argument("--blend-check-layers", default=None, help="gradual filtering: ascending check layers, e.g. 0,1,2")
    p.add_argument("--recompute-ratios", default=None, help="retained document ratio at each check layer")
    p.add_argument("--target-average-recompute-ratio", type=float, default=None,
                   help="fail unless the layer-average document ratio is within 0.002 of this")
    p.add_argument("--deviation-metric", default="value", choices=DEVIATION_METRICS)
    p.add_argument("--dataset", type=Path, default=None,
                   help="MuSiQue-style JSONL (question, answer, paragraphs) instead of --workload")
    p.add_argument("--sample-count", type=int, default=None, help="stratified sample size of --dataset")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--answer-word-limit", type=int, default=5)
    p.add_argument("--model-dir", type=Path, default=None,
                   help="model directory (HF Llama / Mistral or this package's) instead of random-init --model")
    p.add_argument("--store-tier", choices=("pinned", "hbm"), default="pinned",
                   help="where reused document KV waits: pinned host memory (the reference's CPU tier; the "
                        "one-shot arm composes from it over PCIe, the progressive arm stages it on a copy "
                        "stream) or HBM")
    p.add_argument("--no-serial", action="store_true", help="skip the serial-staging rerun of the progressive arm")
    p.add_argument("--output", type=Path, required=True)
    a = p.parse_args(argv)
    blend = blend_config_from_args(a)
    if a.model_dir is not None:
        from ..models.checkpoint import load_config, load_oracle

        blend.check_target(load_config(a.model_dir).n_layers)  # fail before any work when the target is missed
        eng = B200Engine.from_oracle(load_oracle(a.model_dir, dtype=torch.bfloat16), "cuda")
        cfg, a.model = eng.cfg, str(a.model_dir)
    else:
        cfg = get_model_config(a.model)
        blend.check_target(cfg.n_layers)
        eng = B200Engine.random(cfg, seed=0, device="cuda")
    meta: list[dict] = []
    if a.dataset is not None:
        reqs, meta = dataset_requests(a.dataset, cfg, model_dir=a.model_dir, sample_count=a.sample_count,
                                      seed=a.seed, answer_word_limit=a.answer_word_limit,
                                      limit=a.requests + a.warmup)
        a.workload = str(a.dataset)
    else:
        reqs = make_requests(a.workload, cfg)[: a.requests + a.warmup]
    store = DocumentKVStore(cfg, tier="hbm", device=eng.device)
    server = RAGServer(eng, store, capacity=max(r.prompt_tokens for r in reqs) + a.max_new_tokens + 64,
                       blend=blend)
    server.produce(reqs)
    pinned = None
    if a.store_tier == "pinned":
        # the reference's CPU tier: every document block in pinned host memory
        pinned = DocumentKVStore(cfg, tier="pinned")
        for r in reqs:
            for d in r.documents:
                if d not in pinned:
                    pinned.put(d, store[d].kv)
    fractions = tuple(float(x) for x in a.fractions.split(","))
    rows = []
    with open(a.output, "w") as f:
        f.write(json.dumps({"protocol": {"model": a.model, "workload": a.workload, "fractions": fractions,
                                         "schedule": a.schedule, "recompute_ratio": a.recompute_ratio,
                                         "check_layer": a.check_layer, "draft_tokens": a.draft_tokens,
                                         "blend_schedule": [list(x) for x in blend.schedule],
                                         "layer_document_trace": blend.layer_document_trace(cfg.n_layers),
                                         "layer_document_mean": blend.check_target(cfg.n_layers),
                                         "deviation_metric": blend.deviation_metric,
                                         "max_new_tokens": a.max_new_tokens, "commit_window": 1,
                                         "store_tier": a.store_tier, "serial_staging": not a.no_serial}}) + "\n")
        for i, r in enumerate(reqs):
            m = meta[i] if meta else {}
            prep = prepare_request(r, schedule=a.schedule, fractions=fractions, seed=i,
                                   question=m.get("question", ""), texts=m.get("texts"),
                                   supporting=m.get("supporting"))
            row = evaluate_request(server, prep, max_new_tokens=a.max_new_tokens, draft_tokens=a.draft_tokens,
                                   pinned_store=pinned, serial=not a.no_serial)
            if m:
                score_row(row, m, server.eos)
            if i >= a.warmup:
                rows.append(row)
                f.write(json.dumps(row) + "\n")
    print(json.dumps(aggregate(rows), indent=2))


if __name__ == "__main__":
    main()
