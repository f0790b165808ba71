"""Progressive P/D pipeline driver: full-target transfer vs draft-while-loading, paired per request.

Parity with the reference's experiments/pd_progressive_kv_pipeline.py:
  * ``auto_draft_tokens`` (:1363-1381): the draft horizon of a request is the
    number of target decode steps that fit in the residual wire window (the
    bytes still in flight after the first tranche, at the controlled link
    rate, times a utilisation factor), capped by the configured horizon;
  * ``run_full_target`` (:1066-1117): every tranche lands, then the target
    decodes greedily from the full KV;
  * ``run_chain`` (:1120-1243): the continuous draft-while-loading chain with
    one final verifier (``serving.progressive.continuous_graft_chain``);
  * ``requests_from_pack``: requests of a RULER pack (document spans) or a
    LongBench pack (context pages) for ``main --pack``;
  * ``evaluate_request`` / ``main`` (:1246-1699): rank documents by a schedule,
    stage them into tranches (anchor = prefix + first ranked documents +
    suffix), run both arms in alternating order on the same staged request,
    check the greedy outputs are identical, and write JSONL rows with the
    transfer, draft and verification breakdown.
  * ``aggregate`` (experiments/aggregate_pd_progressive_kv_pipeline.py):
    token equality, accepted drafts, TTFT/response distributions, paired gains.
Result rows follow the reference's layout (pd_progressive_kv_pipeline.py:1560-1700):
``schedules[name] = {ranking, stage_document_counts, full_target, chains}``,
``chains[window] = {timing_token_ids, pipeline: {response_ms, first_committed_ms,
terminated_stage, trace, ...}, paired_fixed_control, measurement_order}`` and a
``protocol`` block, so ``pipelines.analysis`` and the latency-cell validator read them.
The transport is the pinned-host tranche stager with an optional paced link
(``TrancheStager``); the prefill producer is this package's engine.
"""
from __future__ import annotations

import argparse
import json
import math
import statistics
import time
from pathlib import Path
from typing import Any, Sequence

import torch

from ..serving.progressive import (Document, TrancheStager, continuous_graft_chain, ranked_document_indices,
                                   stage_document_sets)


def parse_bandwidths(text: str) -> tuple[float, ...]:
    """Comma-separated link rates in Gbit/s: positive, unique, returned ascending."""
    vals = [float(x) for x in text.split(",") if x.strip()]
    if not vals or any(v <= 0 for v in vals) or len(set(vals)) != len(vals):
        raise ValueError("bandwidths must be unique positive values")
    return tuple(sorted(vals))


def common_prefix_length(a: Sequence[int], b: Sequence[int]) -> int:
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


def target_kv_bytes_per_token(model_dir: str | Path) -> int:
    """bf16 K+V bytes per token of an HF Llama-style config.json (all layers)."""
    cfg = json.loads((Path(model_dir) / "config.json").read_text())
    head_dim = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
    kv = cfg.get("num_key_value_heads", cfg["num_attention_heads"])
    return int(cfg["num_hidden_layers"] * 2 * kv * head_dim * 2)


def transfer_ms(nbytes: float, gbps: float) -> float:
    """Wire time of ``nbytes`` at ``gbps`` Gbit/s."""
    return nbytes * 8 / (gbps * 1e6)


def question_attention_document_scores(cfg, layer_inputs: dict, layer_weights: dict, layer_keys: dict,
                                       positions: torch.Tensor, n_tokens: int,
                                       document_ranges: Sequence[tuple[int, int]]) -> list[float]:
    """Producer-side attention mass of the question on every document (the ``p_attention`` schedule).

    For each scored layer: the question rows' residual inputs ``layer_inputs[l]``
    [q, d] are RMS-normalised with the layer's input norm, projected to query
    heads (``layer_weights[l] = (ln1, w_qkv)``), rotated at ``positions``;
    softmax(q K^T / sqrt(D)) over the prompt keys ``layer_keys[l]`` [H_kv, T, D]
    (query heads of a GQA group share a key head) is averaged over heads and
    question rows and summed over each document's token range; the scores are
    averaged over layers (reference: pd_progressive_kv_pipeline.py:117-141).
    """
    from ..rope import apply_rope, rope_cos_sin

    D, H = cfg.head_dim, cfg.n_heads
    cos, sin = rope_cos_sin(cfg, positions.cpu(), device=next(iter(layer_inputs.values())).device)
    queries, keys = [], []
    for l, x in layer_inputs.items():
        ln1, w_qkv = layer_weights[l]
        xf = x.float()
        xn = (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + cfg.rms_eps)).to(torch.bfloat16) * ln1
        q = (xn.float() @ w_qkv[: cfg.q_size].float().t()).view(-1, H, D).transpose(0, 1)  # [H, q, D]
        queries.append(apply_rope(q, cos, sin, sequence_dim=1).transpose(0, 1).contiguous())  # [q, H, D]
        keys.append(layer_keys[l])
    tok = token_attention_scores(torch.stack(queries), keys, n_tokens)
    return [float(tok[b:e].sum()) for b, e in document_ranges]


def token_attention_scores(q: torch.Tensor, keys: Sequence[torch.Tensor], n_tokens: int) -> torch.Tensor:
    """Mean over layers, query rows and heads of softmax(q K^T / sqrt(D)) per prompt token (K11).

    ``q`` [L, R, H, D] fp32 (RoPE applied), ``keys[l]`` [H_kv, >= n_tokens, D].
    On the GPU this is the sm_100a page-score kernel; CPU tensors (the fp32
    oracle path) use the same formula in PyTorch.
    """
    D = q.shape[-1]
    if q.is_cuda:
        from .. import ops

        return ops.ext().page_token_scores(q.float().contiguous(), [k.contiguous() for k in keys], n_tokens,
                                           D ** -0.5)
    L, R, H, _ = q.shape
    out = torch.zeros(n_tokens, dtype=torch.float32)
    for l in range(L):
        k = keys[l][:, :n_tokens].float()
        g = H // k.shape[0]
        logits = torch.einsum("rhd,htd->rht", q[l].float(), k.repeat_interleave(g, dim=0)) * D ** -0.5
        out += logits.softmax(-1).mean(dim=(0, 1))
    return out / L


def auto_draft_tokens(*, prompt_tokens: int, first_stage_tokens: int, bytes_per_token: float, transport_gbps: float,
                      tpot_ms: float, max_draft_tokens: int, utilization: float = 1.0) -> tuple[int, float]:
    """(draft horizon, residual wire ms) of one request."""
    if tpot_ms <= 0 or not 0 < utilization <= 1 or transport_gbps <= 0:
        raise ValueError("invalid auto-draft parameters")
    residual_ms = (prompt_tokens - first_stage_tokens) * bytes_per_token * 8 / (transport_gbps * 1e6)
    return max(1, min(max_draft_tokens, math.floor(residual_ms * utilization / tpot_ms))), residual_ms


def run_full_target(engine, stager: TrancheStager, *, seed_token: int, prompt_tokens: int, max_new_tokens: int,
                    clock=time.perf_counter) -> dict[str, Any]:
    """Baseline arm: wait for every tranche, then greedy decode from the full KV."""
    t0 = clock()
    for i in range(len(stager.stages)):
        stager.launch(i)
    for i in range(len(stager.stages)):
        stager.wait_on_compute_stream(i)
    b = engine._decode_buffers(max_new_tokens)
    b["ids"][:1].fill_(int(seed_token))
    engine.ext.embedding(b["ids"][:1], engine.w.embed, b["h"][:1])
    b["log"][0:1].fill_(int(seed_token))
    b["gen"].fill_(1)
    b["counter"].zero_()
    engine.set_decode_state(position=prompt_tokens)
    torch.cuda.current_stream(engine.device).synchronize()
    ready = (clock() - t0) * 1e3
    engine.decode(stager.slot, max_new_tokens - 1, max_new=max_new_tokens)
    tokens = engine.generated_tokens(max_new_tokens).tolist()
    torch.cuda.current_stream(engine.device).synchronize()
    response = (clock() - t0) * 1e3
    return {"tokens": tokens, "first_ready_ms": ready, "response_ms": response, "seed_forward_ms": 0.0,
            "decode_ms": response - ready, "transfer": stager.finish()}


def _schedule_cells(rows: Sequence[dict]):
    """(full_target, chain) pairs of every row (first schedule and commit window of the protocol)."""
    for r in rows:
        if "schedules" not in r:  # compact rows: {"full_target": ..., "chain": ...}
            yield r["full_target"], r["chain"], r.get("tokens_equal")
            continue
        proto = r["protocol"]
        sched = r["schedules"][proto["schedules"][0]]
        chain = sched["chains"][str(proto["commit_windows"][0])]
        pipe = dict(chain["pipeline"])
        pipe.setdefault("first_ready_ms", pipe.get("first_committed_ms"))
        yield sched["full_target"], pipe, chain.get("timing_token_match_target")


def aggregate(rows: Sequence[dict]) -> dict[str, Any]:
    """Token equality, accepted drafts, response / first-ready distributions and paired gains."""
    def stats(x):
        x = sorted(v for v in x if v is not None)
        if not x:
            return None
        return {"mean": statistics.fmean(x), "p50": x[len(x) // 2], "p99": x[min(len(x) - 1, int(0.99 * len(x)))]}

    cells = list(_schedule_cells(rows))
    return {"requests": len(cells),
            "token_equality_rate": statistics.fmean(bool(e) for _, _, e in cells) if cells else None,
            "accepted_draft_tokens": stats([c["accepted"] for _, c, _ in cells]),
            "full_target_response_ms": stats([t["response_ms"] for t, _, _ in cells]),
            "chain_response_ms": stats([c["response_ms"] for _, c, _ in cells]),
            "full_target_first_ready_ms": stats([t.get("first_ready_ms") for t, _, _ in cells]),
            "chain_first_ready_ms": stats([c.get("first_ready_ms") for _, c, _ in cells]),
            "response_gain_ms": stats([t["response_ms"] - c["response_ms"] for t, c, _ in cells])}


def build_result_row(index: int, request, schedule: str, ranking, sets, out: dict, *, arms: Sequence[str],
                     gamma: int, residual: float | None, bytes_per_token: int, prefill_ms: float,
                     protocol: dict, window: str = "inf") -> dict[str, Any]:
    """One request's result row in the reference layout from the arms' results.

    ``out`` maps "full_target" (``run_full_target``'s dict), "chain" and
    optionally "fixed" (``ChainResult``) to their results; ``arms`` is the
    order they ran in.
    """
    target = dict(out["full_target"])
    target_ids = target.pop("tokens")

    def chain_cell(res, configured):
        return {"timing_token_ids": list(res.token_ids), "configured_draft_tokens": configured,
                "timing_token_match_target": list(res.token_ids) == target_ids,
                "speedup_vs_full_target": target["response_ms"] / res.response_ms, **res.pipeline_record()}

    pipe = out["chain"]
    order = ("full_target_then_pipeline" if list(arms).index("full_target") < list(arms).index("chain")
             else "pipeline_then_full_target")
    chains = {window: {
        "timing_token_ids": list(pipe.token_ids), "configured_draft_tokens": gamma,
        "estimated_residual_wire_ms": residual,
        "timing_token_match_target": list(pipe.token_ids) == target_ids,
        "pipeline": pipe.pipeline_record(),
        "pipeline_speedup_vs_full_target": target["response_ms"] / pipe.response_ms,
        "paired_fixed_control": chain_cell(out["fixed"], gamma) if "fixed" in out else None,
        "measurement_order": order, "arm_order": "->".join(arms)}}
    T = request.prompt_tokens
    return {"dataset_index": index, "prompt_tokens": T, "anchor_tokens": len(request.prefix) + len(request.suffix),
            "document_tokens": sum(len(d) for d in request.documents), "document_pages": len(request.documents),
            "logical_bf16_kv_bytes": T * bytes_per_token, "producer": {"prefill_ms": prefill_ms},
            "schedules": {schedule: {"ranking": list(ranking), "stage_document_counts": [len(x) for x in sets],
                                     "full_target": {"timing_token_ids": target_ids, **target},
                                     "chains": chains}},
            "protocol": protocol}


def requests_from_pack(pack_dir: str | Path, *, page_tokens: int = 256, offset: int = 0,
                       limit: int | None = None) -> list[tuple[Any, list[bool | None]]]:
    """(request, supporting flag per document) of the rows of a P/D pack.

    A RULER pack records the document spans of every prompt: each span is one
    document (contiguous spans required) and carries its supporting flag.  A
    LongBench pack records the prefix and suffix lengths: its context region is
    cut into pages of ``page_tokens`` (the last page may be short), the
    documents of the schedule (reference: pd_progressive_kv_pipeline.py's
    ``--context-page-tokens``).
    """
    from ..synthetic import RAGRequest

    pack_dir = Path(pack_dir)
    reqs = [json.loads(x) for x in (pack_dir / "requests.jsonl").read_text().splitlines() if x.strip()]
    meta = [json.loads(x) for x in (pack_dir / "metadata.jsonl").read_text().splitlines() if x.strip()]
    if len(reqs) != len(meta):
        raise ValueError("request and metadata row counts differ")
    if page_tokens <= 0:
        raise ValueError("page_tokens must be positive")
    end = len(reqs) if limit is None else min(len(reqs), offset + limit)
    out = []
    for i in range(offset, end):
        prompt, m = [int(t) for t in reqs[i]["prompt"]], meta[i]
        if m.get("document_spans"):
            spans = m["document_spans"]
            for a, b in zip(spans, spans[1:]):
                if int(a["end_token"]) != int(b["start_token"]):
                    raise ValueError(f"row {i}: document spans are not contiguous")
            docs = tuple(tuple(prompt[int(s["start_token"]):int(s["end_token"])]) for s in spans)
            flags = [bool(s.get("supporting")) for s in spans]
            head, tail = int(spans[0]["start_token"]), int(spans[-1]["end_token"])
        else:
            head, tail = int(m["prefix_tokens"]), len(prompt) - int(m["suffix_tokens"])
            if not 0 < head < tail <= len(prompt):
                raise ValueError(f"row {i}: prefix / suffix lengths leave no context")
            docs = tuple(tuple(prompt[a:min(a + page_tokens, tail)]) for a in range(head, tail, page_tokens))
            flags = [None] * len(docs)
        out.append((RAGRequest(index=i, prefix=tuple(prompt[:head]), documents=docs, suffix=tuple(prompt[tail:])),
                    flags))
    if not out:
        raise ValueError("the pack window holds no requests")
    return out


def exclusive_gpu_or_exit(*, command_runner=None, max_used_memory_mib: float = 1024.0,
                          max_utilization_pct: float = 5.0) -> dict[str, Any]:
    """Fail closed unless the GPU this process uses has no compute process and is idle.

    The physical index is the first entry of CUDA_VISIBLE_DEVICES when that is
    set, else the current CUDA device (reference: the P/D pipeline's
    ``--require-exclusive-gpu`` check).
    """
    import os

    from ..serving.live import gate

    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")[0].strip()
    index = int(vis) if vis.isdecimal() else int(torch.cuda.current_device())
    states = gate.inspect_gpus(**({"command_runner": command_runner} if command_runner else {}))
    res = gate.evaluate_exclusivity(states, [index], max_used_memory_mib=max_used_memory_mib,
                                    max_utilization_pct=max_utilization_pct)
    if res["status"] != "passed":
        raise SystemExit(f"GPU {index} is not exclusive: {json.dumps(res['failures'])}")
    return res


def score_pack_row(row: dict[str, Any], meta: dict[str, Any], decode) -> None:
    """Score the full target's and every chain's timing tokens with the pack's task metric (in place).

    ``meta`` is the request's pack metadata (``dataset``, ``answers``,
    ``all_classes``); ``decode`` turns token ids into text.
    """
    from ..evaluation.longbench import score_prediction

    answers = meta.get("answers") or []
    dataset = meta.get("dataset", "")
    if not answers or not dataset:
        return

    def score(cell: dict) -> None:
        text = decode(list(cell["timing_token_ids"]))
        metric, em, value = score_prediction(dataset, text, answers, meta.get("all_classes"))
        cell.update(answer=text, metric=metric, exact_match=em, score=value)

    for sched in row["schedules"].values():
        score(sched["full_target"])
        for chain in sched["chains"].values():
            score(chain)
            if chain.get("paired_fixed_control"):
                score(chain["paired_fixed_control"])


def main(argv=None) -> None:
    from ..config import get_model_config
    from ..models.engine import B200Engine
    from ..synthetic import make_requests

    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--workload", default="pd_long")
    p.add_argument("--requests", type=int, default=8)
    p.add_argument("--schedule", default="query",
                   choices=("sequential", "uniform", "query", "p_attention", "oracle", "support_last", "random"))
    p.add_argument("--stage-fractions", default="0.25,0.5,0.75,1.0")
    p.add_argument("--max-new-tokens", type=int, default=32)
    p.add_argument("--draft-tokens", type=int, default=7)
    p.add_argument("--transport-gbps", type=float, default=100.0)
    p.add_argument("--auto-draft-tpot-ms", type=float, default=None)
    p.add_argument("--auto-draft-utilization", type=float, default=1.0)
    p.add_argument("--paired-fixed-control", action="store_true",
                   help="also run the fixed first-stage-view chain on the same staged request")
    p.add_argument("--pack", type=Path, default=None, help="P/D request pack (replaces --workload)")
    p.add_argument("--request-offset", type=int, default=0)
    p.add_argument("--context-page-tokens", type=int, default=256)
    p.add_argument("--model-dir", type=Path, default=None,
                   help="model directory (config.json + model.safetensors) instead of random-init --model")
    p.add_argument("--eager-serial-wire", action="store_true",
                   help="tranches leave on one serial wire as soon as the request starts (cumulative deadlines)")
    p.add_argument("--require-exclusive-gpu", action="store_true",
                   help="refuse to run unless the GPU has no other compute process and is idle")
    p.add_argument("--output", type=Path, required=True)
    a = p.parse_args(argv)
    if a.require_exclusive_gpu:
        exclusive_gpu_or_exit()
    free, total = torch.cuda.mem_get_info()
    if a.model_dir is not None:
        from ..models.checkpoint import load_oracle

        eng = B200Engine.from_oracle(load_oracle(a.model_dir, dtype=torch.bfloat16), device="cuda",
                                     max_positions=65536)
        cfg = eng.cfg
        a.model = str(a.model_dir)
    else:
        cfg = get_model_config(a.model)
        eng = B200Engine.random(cfg, seed=0, device="cuda", max_positions=65536)
    pack_meta, decode = {}, None
    if a.pack is not None:
        packed = requests_from_pack(a.pack, page_tokens=a.context_page_tokens, offset=a.request_offset,
                                    limit=a.requests)
        reqs, flags = [r for r, _ in packed], [f for _, f in packed]
        a.workload = str(a.pack)
        manifest = json.loads((a.pack / "manifest.json").read_text())
        lines = (a.pack / "metadata.jsonl").read_text().splitlines()
        pack_meta = {i: {"dataset": manifest.get("dataset", ""), **json.loads(x)} for i, x in enumerate(lines)
                     if x.strip()}
        if a.model_dir is not None:  # the pack's tokenizer ships with the model: score the answers
            from ..tokenizer import load_tokenizer

            tok = load_tokenizer(a.model_dir, cfg.vocab, max(cfg.n_special, 4), cfg.eos_token_ids)
            decode = lambda ids: tok.decode(ids, skip_special_tokens=True)  # noqa: E731
    else:
        reqs = make_requests(a.workload, cfg)[a.request_offset:a.request_offset + a.requests]
        flags = [[None] * len(r.documents) for r in reqs]
    fractions = tuple(float(x) for x in a.stage_fractions.split(","))
    bytes_per_token = cfg.n_layers * 2 * cfg.n_kv_heads * cfg.head_dim * 2
    rows = []
    window = "inf"
    protocol = {"schedules": [a.schedule], "commit_windows": [window], "transport_gbps": a.transport_gbps,
                "draft_tokens": a.draft_tokens, "max_new_tokens": a.max_new_tokens,
                "stage_fractions": list(fractions), "fixed_token_horizon": True, "paired_measurement": True,
                "paired_fixed_control": a.paired_fixed_control, "model": a.model, "workload": a.workload,
                "require_exclusive_gpu": bool(a.require_exclusive_gpu), "eager_serial_wire": bool(a.eager_serial_wire),
                "initial_gpu_used_bytes": int(total - free)}
    with open(a.output, "w") as f:
        for i, r in enumerate(reqs):
            T = r.prompt_tokens
            docs = [Document(tuple(d), " ".join(map(str, d[:64])), supporting=sup, start=b, end=e)
                    for d, (b, e), sup in zip(r.documents, r.document_ranges(), flags[i])]
            # producer: prefill the whole prompt once; its slot is the tranches' source
            src = eng.new_slot(T + a.max_new_tokens + 64)
            ids = torch.tensor(r.prompt, dtype=torch.int32, device=eng.device)
            q_rows = slice(T - min(16, len(r.suffix)), T)  # question rows scored by p_attention
            score_layers = sorted({round(j * (cfg.n_layers - 1) / 3) for j in range(4)})
            captured: dict[int, torch.Tensor] = {}

            def hook(layer, hh):
                if layer in score_layers:
                    captured[layer] = hh[q_rows].clone()

            p0 = time.perf_counter()
            h = eng.prefill(ids, src, layer_hook=hook if a.schedule == "p_attention" else None)
            seed = int(eng.first_token(h[T - 1:T], position=T, max_new=1)["tok"][0].item())
            prefill_ms = (time.perf_counter() - p0) * 1e3
            att = None
            if a.schedule == "p_attention":
                att = question_attention_document_scores(
                    cfg, captured, {l: (eng.w.layers[l].ln1, eng.w.layers[l].w_qkv) for l in captured},
                    {l: src.k(l) for l in captured}, torch.arange(T)[q_rows], T, r.document_ranges())
            ranking = ranked_document_indices(a.schedule, question=" ".join(map(str, r.suffix)), documents=docs,
                                              random_seed=i, attention_scores=att)
            sets = stage_document_sets(ranking, docs, fractions)
            first = len(r.prefix) + len(r.suffix) + sum(len(docs[j].token_ids) for j in sets[0])
            gamma, residual = (a.draft_tokens, None)
            if a.auto_draft_tpot_ms is not None:
                gamma, residual = auto_draft_tokens(prompt_tokens=T, first_stage_tokens=first,
                                                    bytes_per_token=bytes_per_token,
                                                    transport_gbps=a.transport_gbps, tpot_ms=a.auto_draft_tpot_ms,
                                                    max_draft_tokens=a.draft_tokens,
                                                    utilization=a.auto_draft_utilization)
            host = src.data[:, :, :, :T].cpu().pin_memory()
            arms = ["full_target", "chain"] + (["fixed"] if a.paired_fixed_control else [])
            if i % 2:
                arms = arms[::-1]
            out: dict[str, Any] = {}
            for arm in arms:
                dst = eng.new_slot(T + a.max_new_tokens + 64)
                stager = TrancheStager(host, dst, prefix_tokens=len(r.prefix), documents=docs,
                                       suffix_tokens=len(r.suffix), ranking=ranking, selected_sets=sets,
                                       transport_gbps=a.transport_gbps, eager_serial_wire=a.eager_serial_wire)
                if arm == "full_target":
                    out[arm] = run_full_target(eng, stager, seed_token=seed, prompt_tokens=T,
                                               max_new_tokens=a.max_new_tokens)
                else:
                    out[arm] = continuous_graft_chain(eng, stager, seed_token=seed, prompt_tokens=T,
                                                      max_draft_tokens=gamma, max_new_tokens=a.max_new_tokens,
                                                      grow_view=(arm == "chain"))
            row = build_result_row(r.index, r, a.schedule, ranking, sets, out, arms=arms, gamma=gamma, residual=residual,
                                   bytes_per_token=bytes_per_token, prefill_ms=prefill_ms, protocol=protocol)
            if decode is not None and r.index in pack_meta:
                score_pack_row(row, pack_meta[r.index], decode)
            rows.append(row)
            f.write(json.dumps(row, default=str) + "\n")
    print(json.dumps(aggregate(rows), indent=2))


if __name__ == "__main__":
    main()
