"""OpenAI-style completion endpoints over a prefill or decode worker.

A worker process serves one role of a 1P1D deployment:
  * ``prefill``: prefills the prompt, makes its KV available to the decode
    side, answers with the seed token (``choices[0].token_ids[0]``, always
    returned: the proxy needs it), then reports store completion to the
    proxy's telemetry endpoint (``{"request_ids_set": [id]}``);
  * ``decode``: given the prompt and the proxy-owned ``kv_transfer_params``
    (the producer seed token, progressive-draft settings, the request's chunk
    priority), streams the greedy continuation as server-sent events, one
    token per event, and appends scheduler / input-trace records to JSONL
    telemetry files for the aggregator and the trace verifier.

The HTTP contract is the one the reference's vLLM/LMCache workers expose to
its proxy (experiments/progressive_pd_proxy.py:123-214), so the same proxy
and benchmark client drive either.  ``EngineWorker`` runs this package's
engine on one GPU; ``ToyWorker`` is a deterministic CPU stand-in with the
same telemetry, used by the harness tests.
"""
from __future__ import annotations

import json
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
        t = now_ns()
        started = t
        for i, tok in enumerate([seed] + drafts[:-1]):
            t += 1000
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
    side then finds the prompt KV in the slot the prefill wrote.  Progressive
    drafting uses the sparse-view decode of ``B200Engine.decode(view=...)``
    followed by one batched verification.
    """

    def __init__(self, engine, *, capacity: int = 32768, model_name: str = "sparsecache-b200",
                 telemetry: TelemetrySink | None = None) -> None:
        import torch

        self.engine, self.model_name = engine, model_name
        self.telemetry = telemetry or TelemetrySink()
        self.slot = engine.new_slot(capacity)
        self._prompts: dict[str, tuple[list[int], int]] = {}
        self._torch = torch
        self._lock = threading.Lock()

    def prefill(self, request_id: str, prompt: Sequence[int]) -> int:
        torch = self._torch
        with self._lock:
            ids = torch.tensor(list(prompt), dtype=torch.int32, device=self.engine.device)
            t0 = now_ns()
            h = self.engine.prefill(ids, self.slot)
            b = self.engine.first_token(h[-1:], position=len(prompt), max_new=1)
            seed = int(b["tok"][0].item())
            self.telemetry.emit("link", {"request_id": request_id, "bundles": [
                {"index": 0, "chunks": list(range(-(-len(prompt) // 256))), "bytes": 0,
                 "wire_ms": (now_ns() - t0) / 1e6}], "residual_modeled_wire_ms": 0.0})
            self._prompts[request_id] = (list(prompt), seed)
            return seed

    def decode(self, request_id: str, prompt: Sequence[int], s: DecodeSettings) -> Iterator[int]:
        torch = self._torch
        with self._lock:
            n = max(1, s.max_tokens)
            h = self.engine.prefill(torch.tensor(list(prompt), dtype=torch.int32, device=self.engine.device),
                                    self.slot)
            self.engine.first_token(h[-1:], position=len(prompt), max_new=n)
            if n > 1:
                self.engine.decode(self.slot, n - 1, max_new=n)
            toks = self.engine.generated_tokens(n).cpu().tolist()
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
