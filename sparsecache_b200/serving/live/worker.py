"""OpenAI-style completion endpoints over a prefill or decode worker.

A worker process serves one role of a 1P1D deployment:
  * ``prefill``: prefills the prompt, makes its KV available to the decode
    side, answers with the seed token (``choices[0].token_ids[0]``, always
    returned: the proxy needs it), then reports store completion to the
    proxy's telemetry endpoint (``{"request_ids_set": [id]}``);
  * ``decode``: given the prompt and the proxy-owned ``kv_transfer_params``
    (the producer seed token, progressive-draft settings, the request's chunk
    priority), streams the greedy continuation as server-sent events, one
    token per event, and appends scheduler / input-trace / sparse-attention
    (the prompt view each draft step read) records to JSONL telemetry files
    for the aggregator and the trace verifier.

The HTTP contract is the one the reference's vLLM/LMCache workers expose to
its proxy (experiments/progressive_pd_proxy.py:123-214), so the same proxy
and benchmark client drive either.  ``EngineWorker`` runs this package's
engine on one GPU; ``ToyWorker`` is a deterministic CPU stand-in with the
same telemetry, used by the harness tests.
"""
from __future__ import annotations

import json
import math
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Iterator, Protocol, Sequence

from fastapi import Request  # module level: FastAPI resolves handler annotations here


def now_ns() -> int:
    return time.perf_counter_ns()


@dataclass
class DecodeSettings:
    max_tokens: int
    seed_token_id: int | None = None
    progressive: dict | None = None        # {seed_token_id, max_draft_tokens, start_fraction, visibility_mode}
    priority_chunks: list[int] | None = None
    stop_token_ids: tuple[int, ...] = ()


class Worker(Protocol):
    model_name: str

    def prefill(self, request_id: str, prompt: Sequence[int]) -> int: ...

    def decode(self, request_id: str, prompt: Sequence[int], settings: DecodeSettings) -> Iterator[int]: ...


@dataclass
class TelemetrySink:
    """Append-only JSONL files (scheduler records, worker input trace, link trace)."""

    directory: Path | None = None
    records: dict[str, list[dict]] = field(default_factory=dict)
    lock: threading.Lock = field(default_factory=threading.Lock)

    def emit(self, kind: str, row: dict) -> None:
        with self.lock:
            self.records.setdefault(kind, []).append(row)
            if self.directory is not None:
                self.directory.mkdir(parents=True, exist_ok=True)
                with open(self.directory / f"{kind}.jsonl", "a", encoding="utf-8") as f:
                    f.write(json.dumps(row) + "\n")


def visibility_snapshot(prompt_tokens: int, order: Sequence[int], k: int, chunk: int) -> dict:
    """The prompt view after the first ``k`` chunks of ``order`` arrived: merged [lo, hi) token ranges,
    visible token fraction, visible / candidate chunk counts."""
    n_chunks = max(1, -(-prompt_tokens // chunk))
    vis = sorted({int(c) for c in order[:k] if 0 <= int(c) < n_chunks})
    ranges: list[list[int]] = []
    for c in vis:
        lo, hi = c * chunk, min(prompt_tokens, (c + 1) * chunk)
        if ranges and ranges[-1][1] == lo:
            ranges[-1][1] = hi
        else:
            ranges.append([lo, hi])
    seen = sum(hi - lo for lo, hi in ranges)
    return {"visible_token_ranges": ranges, "visible_fraction": seen / max(1, prompt_tokens),
            "visible_pages": len(vis), "candidate_pages": n_chunks}


def emit_attention_step(telemetry: "TelemetrySink", request_id: str, mode: str, step: int, snapshot: dict,
                        layers: int) -> None:
    """One request-attributed record of the view a sparse draft step attended to (every layer reads it)."""
    telemetry.emit("attention", {"request_id": request_id, "visibility_mode": mode, "decode_step": step,
                                 "layers": layers, **snapshot})


def stage_chunks(mode: str, start_fraction: float, n_chunks: int, step: int) -> int:
    """Chunks visible to draft ``step``: the first stage for ``fixed_s1``, one more per step for ``continuous``."""
    first = max(1, min(n_chunks, math.ceil(float(start_fraction) * n_chunks)))
    return first if mode == "fixed_s1" else min(n_chunks, first + step)


class ToyWorker:
    """Deterministic greedy "model" on the CPU with the real worker's telemetry.

    next(token history) = (31 * last + 7 * len(history) + sum(prompt)) % vocab.
    Progressive decoding drafts ``max_draft_tokens`` from a sparse view (the
    draft is right for the first ``accept`` positions, ``accept`` derived from
    the visibility fraction), verifies them in one batch and continues with
    the target; the streamed tokens are identical to baseline decoding.
    """

    def __init__(self, model_name: str = "toy", vocab: int = 1000, telemetry: TelemetrySink | None = None,
                 step_s: float = 0.0) -> None:
        self.model_name, self.vocab = model_name, vocab
        self.telemetry = telemetry or TelemetrySink()
        self.step_s = step_s

    def _next(self, prompt: Sequence[int], hist: list[int]) -> int:
        return (31 * hist[-1] + 7 * len(hist) + sum(prompt)) % self.vocab

    def prefill(self, request_id: str, prompt: Sequence[int]) -> int:
        return (sum(prompt) * 13 + len(prompt)) % self.vocab

    def _link_trace(self, request_id: str, prompt: Sequence[int], s: DecodeSettings) -> None:
        """The KV bundles this decode received (anchor chunks first, then the priority order)."""
        n_chunks = max(1, -(-len(prompt) // 256))
        order = list(s.priority_chunks or range(n_chunks))
        self.telemetry.emit("link", {"request_id": request_id, "bundles": [
            {"index": i, "chunks": [c], "bytes": 2 * 256, "wire_ms": 0.05} for i, c in enumerate(order)],
            "residual_modeled_wire_ms": 0.05 * max(0, len(order) - 1)})

    def _progressive_trace(self, request_id: str, prompt: Sequence[int], s: DecodeSettings, seed: int,
                           out: list[int]) -> None:
        """Scheduler record + worker input trace of one draft-while-loading episode.

        The draft of γ tokens runs as γ single-token forwards over the sparse
        view ([seed, d0, .., d_{γ-2}] at contiguous positions from the seed's
        position); after the full KV arrives one verifier batch rewinds to the
        seed and consumes [seed, d0, .., d_{γ-1}].  Draft token i is right for
        the first ``accept`` positions (accept grows with the visible fraction).
        """
        gamma = int(s.progressive["max_draft_tokens"])
        accept = min(gamma, max(0, int(round(gamma * (1.0 - float(s.progressive["start_fraction"]))))) - 1)
        accept = max(0, accept)
        target = out[1:gamma + 1] + [0] * max(0, gamma + 1 - len(out))
        drafts = [t if i < accept else (t + 1) % self.vocab for i, t in enumerate(target[:gamma])]
        pos0 = len(prompt)
        n_chunks = max(1, -(-pos0 // 256))
        order = list(s.priority_chunks or range(n_chunks))
        t = now_ns()
        started = t
        for i, tok in enumerate([seed] + drafts[:-1]):
            t += 1000
            k = stage_chunks(s.progressive["visibility_mode"], s.progressive["start_fraction"], n_chunks, i)
            emit_attention_step(self.telemetry, request_id, s.progressive["visibility_mode"], i,
                                visibility_snapshot(pos0, order, k, 256), layers=1)
            self.telemetry.emit("input_trace", {"request_id": request_id, "recorded_at_ns": t,
                                                "input_token_ids": [tok], "positions": [pos0 + i],
                                                "num_scheduled_tokens": 1})
        last_draft = t
        full_arrival = t + 500
        verify_start = full_arrival + 100
        self.telemetry.emit("input_trace", {"request_id": request_id, "recorded_at_ns": verify_start + 10,
                                            "input_token_ids": [seed] + drafts,
                                            "positions": list(range(pos0, pos0 + gamma + 1)),
                                            "num_scheduled_tokens": gamma + 1})
        accepted = 0
        for d, tgt in zip(drafts, target):
            if d != tgt:
                break
            accepted += 1
        self.telemetry.emit("scheduler", {
            "request_id": request_id, "seed_token_id": int(seed), "draft_token_ids": drafts, "draft_tokens": gamma,
            "max_draft_tokens": gamma, "accepted_tokens": accepted,
            "visibility_mode": s.progressive["visibility_mode"], "priority_chunks": s.priority_chunks,
            "transitions": ["WAIT_ANCHOR", "DRAFT_WHILE_LOADING", "READY_TO_VERIFY", "TARGET_DECODING", "FINISHED"],
            "started_at_ns": started, "draft_completed_at_ns": [started + 1000 * (i + 1) for i in range(gamma)],
            "last_draft_at_ns": last_draft, "full_arrival_at_ns": full_arrival, "verify_started_at_ns": verify_start,
            "verify_completed_at_ns": verify_start + 2000, "verify_ns": 2000})

    def decode(self, request_id: str, prompt: Sequence[int], s: DecodeSettings) -> Iterator[int]:
        seed = s.seed_token_id if s.progressive is None else s.progressive["seed_token_id"]
        out = [int(seed)]
        while len(out) < s.max_tokens:
            out.append(self._next(prompt, out))
        self._link_trace(request_id, prompt, s)
        if s.progressive is not None:
            self._progressive_trace(request_id, prompt, s, seed, out)
        for t in out:
            if self.step_s:
                time.sleep(self.step_s)
            yield t


class EngineWorker:
    """This package's engine on one GPU: prefill, first token, CUDA-graph decode.

    Both roles may run in one process on one GPU ("aggregated"): the decode
    side then holds the whole prompt's K/V after its own prefill, and the
    link is modeled (one bundle per 256-token chunk, in the request's
    priority order).  A progressive request drafts ``max_draft_tokens``
    tokens as single-token forwards over a sparse view of the prompt (the
    chunks that would have arrived: the first stage for ``fixed_s1``, one
    more priority chunk per draft for ``continuous``), verifies
    [seed, drafts] in one batched forward over the full prompt, and
    continues with greedy decoding; the verifier's rows equal greedy
    decoding's bit for bit, so every arm streams the same tokens.  The
    scheduler and input-trace records are those the aggregator and the
    trace verifier read (``ToyWorker`` writes the same).
    """

    CHUNK = 256  # tokens per link bundle

    def __init__(self, engine, *, capacity: int = 32768, model_name: str = "sparsecache-b200",
                 telemetry: TelemetrySink | None = None) -> None:
        import torch

        self.engine, self.model_name = engine, model_name
        self.telemetry = telemetry or TelemetrySink()
        self.slot = engine.new_slot(capacity)
        self._torch = torch
        self._lock = threading.Lock()
        cfg = engine.cfg
        self.kv_bytes_per_token = cfg.n_layers * 2 * cfg.n_kv_heads * cfg.head_dim * 2

    def _prefill_seed(self, prompt: Sequence[int], max_new: int) -> int:
        torch = self._torch
        ids = torch.tensor(list(prompt), dtype=torch.int32, device=self.engine.device)
        h = self.engine.prefill(ids, self.slot)
        b = self.engine.first_token(h[-1:], position=len(prompt), max_new=max_new)
        return int(b["tok"][0].item())

    def prefill(self, request_id: str, prompt: Sequence[int]) -> int:
        with self._lock:
            return self._prefill_seed(prompt, 1)

    def _chunk_order(self, s: DecodeSettings, n_chunks: int) -> list[int]:
        order = [int(c) for c in (s.priority_chunks or range(n_chunks)) if 0 <= int(c) < n_chunks]
        seen = set()
        order = [c for c in order if not (c in seen or seen.add(c))]
        return order + [c for c in range(n_chunks) if c not in seen]

    def _link_trace(self, request_id: str, T: int, order: Sequence[int]) -> None:
        bundles = [{"index": i, "chunks": [c], "wire_ms": 0.0,
                    "bytes": (min(T, (c + 1) * self.CHUNK) - c * self.CHUNK) * self.kv_bytes_per_token}
                   for i, c in enumerate(order)]
        self.telemetry.emit("link", {"request_id": request_id, "bundles": bundles, "residual_modeled_wire_ms": 0.0})

    def _continue(self, out: list[int], T: int, n: int) -> list[int]:
        """Greedy decode after ``out`` (its last token's K/V not yet written) up to ``n`` tokens."""
        eng = self.engine
        if len(out) >= n:
            return out[:n]
        b = eng._decode_buffers(n)
        b["ids"][:1].fill_(out[-1])
        eng.ext.embedding(b["ids"][:1], eng.w.embed, b["h"][:1])
        b["gen"].zero_()
        eng.set_decode_state(position=T + len(out) - 1)
        eng.decode(self.slot, n - len(out), max_new=n)
        return out + eng.generated_tokens(n - len(out)).tolist()

    def _progressive(self, request_id: str, prompt: Sequence[int], s: DecodeSettings, n: int,
                     order: Sequence[int]) -> list[int]:
        torch, eng, emit = self._torch, self.engine, self.telemetry.emit
        p = s.progressive
        T = len(prompt)
        seed = int(p["seed_token_id"])
        gamma = max(1, min(int(p["max_draft_tokens"]), eng.MAX_ROWS - 1))  # one verifier batch of gamma + 1 rows
        mode = str(p["visibility_mode"])
        n_chunks = len(order)
        view = torch.zeros(self.slot.capacity, dtype=torch.int32, device=eng.device)
        started = now_ns()
        drafts, done_at = [], []
        tok = seed
        for i in range(gamma):
            snap = visibility_snapshot(T, order, stage_chunks(mode, p["start_fraction"], n_chunks, i), self.CHUNK)
            emit_attention_step(self.telemetry, request_id, mode, i, snap, layers=eng.cfg.n_layers)
            vis = [t for lo, hi in snap["visible_token_ranges"] for t in range(lo, hi)]
            # virtual keys: the visible prompt slots, the earlier drafts' slots, then this row's own slot
            view[: len(vis) + i + 1].copy_(torch.tensor(vis + list(range(T, T + i + 1)), dtype=torch.int32))
            t_in = now_ns()
            pred = eng.verify(self.slot, torch.tensor([tok], dtype=torch.int32), position=T + i, slot_start=T + i,
                              view=view, n_visible=len(vis) + i, sparse=True)
            emit("input_trace", {"request_id": request_id, "recorded_at_ns": t_in, "input_token_ids": [tok],
                                 "positions": [T + i], "num_scheduled_tokens": 1})
            tok = int(pred[0].item())
            drafts.append(tok)
            done_at.append(now_ns())
        last_draft = now_ns()
        full_arrival = now_ns()  # aggregated: the whole prompt's K/V is resident
        verify_start = now_ns()
        seq = [seed] + drafts
        t_in = now_ns()
        preds = eng.verify(self.slot, torch.tensor(seq, dtype=torch.int32), position=T, slot_start=T).tolist()
        emit("input_trace", {"request_id": request_id, "recorded_at_ns": t_in, "input_token_ids": seq,
                             "positions": list(range(T, T + len(seq))), "num_scheduled_tokens": len(seq)})
        verify_done = now_ns()
        accepted = 0
        for d, t in zip(drafts, preds):
            if d != t:
                break
            accepted += 1
        out = [seed] + drafts[:accepted] + [int(preds[accepted])]
        emit("scheduler", {
            "request_id": request_id, "seed_token_id": seed, "draft_token_ids": drafts, "draft_tokens": gamma,
            "max_draft_tokens": gamma, "accepted_tokens": accepted, "visibility_mode": mode,
            "priority_chunks": s.priority_chunks,
            "transitions": ["WAIT_ANCHOR", "DRAFT_WHILE_LOADING", "READY_TO_VERIFY", "TARGET_DECODING", "FINISHED"],
            "started_at_ns": started, "draft_completed_at_ns": done_at, "last_draft_at_ns": last_draft,
            "full_arrival_at_ns": full_arrival, "verify_started_at_ns": verify_start,
            "verify_completed_at_ns": verify_done, "verify_ns": verify_done - verify_start})
        return self._continue(out, T, n)

    def decode(self, request_id: str, prompt: Sequence[int], s: DecodeSettings) -> Iterator[int]:
        with self._lock:
            n = max(1, s.max_tokens)
            T = len(prompt)
            order = self._chunk_order(s, max(1, -(-T // self.CHUNK)))
            seed = self._prefill_seed(prompt, n)  # stands for the transferred prompt K/V
            if s.progressive is None:
                if n > 1:
                    self.engine.decode(self.slot, n - 1, max_new=n)
                toks = self.engine.generated_tokens(n).cpu().tolist()
            else:
                if int(s.progressive["seed_token_id"]) != seed:
                    raise RuntimeError("the producer seed differs from this worker's prefill")
                toks = self._progressive(request_id, prompt, s, n, order)
            self._link_trace(request_id, T, order)
        yield from toks


def make_app(worker: Worker, role: str, *, telemetry_url: str | None = None,
             notify: Callable[[str], None] | None = None):
    """FastAPI app of one worker role ("prefill", "decode")."""
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, StreamingResponse

    if role not in ("prefill", "decode"):
        raise ValueError("role must be prefill or decode")
    app = FastAPI()

    def _prompt_ids(body: dict) -> list[int]:
        p = body.get("prompt")
        if not isinstance(p, list) or not p or any(not isinstance(t, int) or isinstance(t, bool) for t in p):
            raise HTTPException(status_code=400, detail="prompt must be a non-empty list of token ids")
        return p

    async def _store_complete(request_id: str) -> None:
        if notify is not None:
            notify(request_id)
        elif telemetry_url:
            import httpx

            async with httpx.AsyncClient(trust_env=False, timeout=10.0) as c:
                await c.post(telemetry_url, json={"request_ids_set": [request_id]})

    @app.get("/health")
    async def health():
        return {"status": "ok", "role": role}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": worker.model_name, "object": "model"}]}

    @app.post("/v1/completions")
    async def completions(request: Request):
        body = await request.json()
        request_id = request.headers.get("X-Request-Id") or "anon"
        prompt = _prompt_ids(body)
        if role == "prefill":
            seed = worker.prefill(request_id, prompt)
            await _store_complete(request_id)
            return JSONResponse({"id": f"cmpl-{request_id}", "object": "text_completion",
                                 "choices": [{"index": 0, "text": "", "token_ids": [seed], "finish_reason": "length"}]})
        params = body.get("kv_transfer_params") or {}
        prog = params.get("progressive_sparse_draft")
        seed = prog["seed_token_id"] if prog else params.get("producer_seed_token_id")
        settings = DecodeSettings(max_tokens=int(body.get("max_tokens", 16)), seed_token_id=seed, progressive=prog,
                                  priority_chunks=params.get("progressive_priority_chunks"))
        if seed is None:
            raise HTTPException(status_code=400, detail="decode requires the producer seed token")
        tokens = worker.decode(request_id, prompt, settings)
        if body.get("stream", False):
            def events():
                for t in tokens:
                    yield "data: " + json.dumps({"id": f"cmpl-{request_id}", "choices": [
                        {"index": 0, "text": "", "token_ids": [t]}]}) + "\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(events(), media_type="text/event-stream")
        out = list(tokens)
        return JSONResponse({"id": f"cmpl-{request_id}", "choices": [{"index": 0, "text": "", "token_ids": out,
                                                                     "finish_reason": "length"}]})

    return app
