"""Single-GPU RAG serving front end: dedup store -> composer -> CacheBlend -> graph decode.

This is the public serving call (``RAGServer.serve``) used by the CLI, the
data-parallel router and the benchmark.  One request at a time per GPU
(batch 1, greedy), as the reference measures (reuse_cacheblend_pipeline.py:
835-893 ``run_full_cacheblend``; modeling.py:33-327); ``serve_batch`` serves
up to 32 requests together with a batched greedy decode.

Device timing: CUDA events on the serving stream bracket TTFT (first token
ready on the device) and the full response (all new tokens ready).  Nothing
in ``serve`` synchronises the host unless ``sync=True``; the caller decides
when to read results.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from ..config import CacheBlendConfig
from ..models.engine import B200Engine, KVSlot
from ..store import DocumentKVStore
from ..synthetic import RAGRequest


@dataclass
class ServeHandle:
    """In-flight request: events and the pinned host buffer receiving its tokens."""

    request: RAGRequest
    mode: str
    start: torch.cuda.Event
    first: torch.cuda.Event
    end: torch.cuda.Event
    tokens_host: torch.Tensor
    max_new: int
    eos: frozenset
    meta: dict[str, Any] = field(default_factory=dict)

    def result(self) -> "ServeResult":
        self.end.synchronize()
        toks = [int(t) for t in self.tokens_host[: self.max_new].tolist()]
        for i, t in enumerate(toks):
            if t in self.eos:
                toks = toks[: i + 1]
                break
        ttft = self.start.elapsed_time(self.first)
        total = self.start.elapsed_time(self.end)
        return ServeResult(tuple(toks), ttft, total, total - ttft, self.mode, dict(self.meta))


@dataclass
class ServeResult:
    token_ids: tuple[int, ...]
    ttft_ms: float
    response_ms: float
    decode_ms: float
    mode: str
    metadata: dict[str, Any]


@dataclass
class BatchResult:
    """A batch served together: one CacheBlend prefill per request, then batched greedy decode."""

    token_ids: list[tuple[int, ...]]
    ttft_ms: list[float]        # request i's first token ready, from the batch start
    response_ms: float          # all tokens of all requests ready, from the batch start
    decode_step_ms: float       # one batched greedy step
    metadata: dict[str, Any]


class RAGServer:
    def __init__(
        self,
        engine: B200Engine,
        store: DocumentKVStore,
        *,
        capacity: int,
        blend: CacheBlendConfig | None = None,
    ) -> None:
        self.engine = engine
        self.store = store
        self.blend = blend or CacheBlendConfig()
        self.slot: KVSlot = engine.new_slot(capacity)
        self.eos = frozenset(engine.cfg.eos_token_ids)
        self._ids_dev = torch.empty(capacity, dtype=torch.int32, device=engine.device)
        self._batch_slots: dict[int, list[KVSlot]] = {}

    # ---------------------------------------------------------- producer
    def encode_local(self, tokens) -> torch.Tensor:
        """Prefill one document alone at positions 0..n-1; returns its [L,2,Hkv,n,D] block."""
        n = len(tokens)
        block = KVSlot(self.engine.cfg, n, self.engine.device)
        ids = torch.tensor(tokens, dtype=torch.int32).to(self.engine.device, non_blocking=True)
        self.engine.prefill(ids, block)
        return block.data

    def produce(self, requests) -> dict[str, Any]:
        docs = [d for r in requests for d in r.documents]
        return self.store.produce(self.encode_local, docs)

    # ------------------------------------------------------------- serve
    def serve(
        self,
        request: RAGRequest,
        *,
        mode: str = "cacheblend",
        ids_host: torch.Tensor | None = None,
        store: DocumentKVStore | None = None,
        max_new_tokens: int | None = None,
        blend: CacheBlendConfig | None = None,
        sync: bool = False,
    ) -> ServeHandle | ServeResult:
        """Serve one request.  ``ids_host`` (pinned int32) is copied H2D inside the timed region.

        ``blend`` overrides the server's CacheBlend parameters for this call
        (e.g. recompute ratio 1.0 as the correctness gate against full prefill).
        """
        eng = self.engine
        store = store or self.store
        blend = blend or self.blend
        max_new = max_new_tokens or blend.max_new_tokens
        T = request.prompt_tokens
        if T + max_new > self.slot.capacity:
            raise ValueError("request does not fit the serving slot")
        start, first, end = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        tokens_host = torch.empty(max_new, dtype=torch.int32, pin_memory=True)
        start.record()
        ids = self._ids_dev[:T]
        if ids_host is None:
            ids_host = torch.tensor(request.prompt, dtype=torch.int32).pin_memory()
        ids.copy_(ids_host, non_blocking=True)
        meta: dict[str, Any] = {"prompt_tokens": T}
        if mode == "cacheblend":
            blocks = [store[d].kv for d in request.documents]
            eng.compose(self.slot, blocks, first_slot=len(request.prefix), layer_begin=blend.check_layer)
            h_a, A, dmeta = eng.cacheblend(
                ids, self.slot, prefix_tokens=len(request.prefix), suffix_tokens=len(request.suffix), blend=blend
            )
            last = h_a[A - 1 : A]
            meta.update(active_rows=A, document_tokens=dmeta["document_tokens"],
                        document_tokens_selected=dmeta["k_selected"], checksum_dev=dmeta["checksum"])
        elif mode == "full":
            h = eng.prefill(ids, self.slot)
            last = h[T - 1 : T]
        elif mode == "direct":
            blocks = [store[d].kv for d in request.documents]
            P = len(request.prefix)
            # the system prefix is prefilled, documents reused as-is, suffix prefilled after them
            eng.prefill(ids[:P], self.slot)
            eng.compose(self.slot, blocks, first_slot=P)
            h = eng.prefill(ids[P + request.document_tokens :], self.slot, start=P + request.document_tokens)
            last = h[len(request.suffix) - 1 : len(request.suffix)]
        else:
            raise ValueError(f"unknown mode {mode!r}")
        eng.first_token(last, position=T, max_new=max_new)
        first.record()
        eng.decode(self.slot, max_new - 1, max_new=max_new)
        tokens_host.copy_(eng.generated_tokens(max_new), non_blocking=True)
        end.record()
        handle = ServeHandle(request, mode, start, first, end, tokens_host, max_new, self.eos, meta)
        return handle.result() if sync else handle

    # ------------------------------------------------------ batched serve
    def serve_batch(self, requests: list[RAGRequest], *, ids_host: list[torch.Tensor] | None = None,
                    store: DocumentKVStore | None = None, max_new_tokens: int | None = None,
                    blend: CacheBlendConfig | None = None) -> BatchResult:
        """Serve up to ``B200Engine.MAX_BATCH`` requests together (greedy, CacheBlend).

        Each request is composed and CacheBlend-prefilled into its own slot of
        a batch buffer (the slots are reused by later batches of the same
        size); the last prompt rows go through one LM-head GEMM on the tensor
        cores for the first tokens; then every step decodes all sequences at
        once (skinny tcgen05 GEMMs over the batch rows, one attention launch
        for all sequences, one CUDA graph per step).  Synchronises the host at
        the end and returns the tokens and device timings.
        """
        eng = self.engine
        store = store or self.store
        blend = blend or self.blend
        max_new = max_new_tokens or blend.max_new_tokens
        B = len(requests)
        cap = self.slot.capacity
        if any(r.prompt_tokens + max_new > cap for r in requests):
            raise ValueError("a request does not fit the serving slots")
        slots = self._batch_slots.get(B)
        if slots is None:
            slots = self._batch_slots[B] = eng.batch_slots(B, cap)
        last = eng.ws.get("serve_batch_last", (eng.MAX_BATCH, eng.cfg.d_model), torch.bfloat16)[:B]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(B + 3)]
        ev[0].record()
        actives = []
        for i, r in enumerate(requests):
            T = r.prompt_tokens
            ids = self._ids_dev[:T]
            host = ids_host[i] if ids_host is not None else torch.tensor(r.prompt, dtype=torch.int32).pin_memory()
            ids.copy_(host, non_blocking=True)
            blocks = [store[d].kv for d in r.documents]
            eng.compose(slots[i], blocks, first_slot=len(r.prefix), layer_begin=blend.check_layer)
            h_a, A, _ = eng.cacheblend(ids, slots[i], prefix_tokens=len(r.prefix), suffix_tokens=len(r.suffix),
                                       blend=blend)
            last[i].copy_(h_a[A - 1])
            actives.append(A)
            ev[1 + i].record()
        firsts = eng.batch_first_tokens(last)
        eng.start_batch(slots, firsts, [r.prompt_tokens for r in requests], max_new=max_new)
        ev[B + 1].record()
        eng.decode_batch(slots, max_new - 1)
        toks = torch.empty(max_new, B, dtype=torch.int32, pin_memory=True)
        toks.copy_(eng.batch_tokens(B, max_new), non_blocking=True)
        ev[B + 2].record()
        ev[B + 2].synchronize()
        out = []
        for b in range(B):
            seq = [int(t) for t in toks[:, b].tolist()]
            for k, t in enumerate(seq):
                if t in self.eos:
                    seq = seq[: k + 1]
                    break
            out.append(tuple(seq))
        first_ms = ev[0].elapsed_time(ev[B + 1])
        total = ev[0].elapsed_time(ev[B + 2])
        return BatchResult(out, [ev[0].elapsed_time(e) for e in ev[1:B + 1]], total,
                           (total - first_ms) / max(1, max_new - 1),
                           {"batch": B, "active_rows": actives, "first_tokens_ms": first_ms})
