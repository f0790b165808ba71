"""Public generation API: full prefill, direct KV reuse, CacheBlend.

Same call surface as the reference (src/sparsecache/modeling.py:19-327):
``baseline_generate``, ``direct_reuse_generate`` and ``cacheblend_generate``
return a ``GenerationResult``.  ``model`` is either a ``B200Engine`` (the
sm_100a kernel path) or a ``LlamaOracle`` (the PyTorch CPU/oracle path).
Prefix caches use the legacy per-layer layout ``[(key, value)]`` with
tensors ``[1, n_kv_heads, tokens, head_dim]``.

``cacheblend_generate`` defaults to the reference's semantics for this entry
point (key deviation; only the question suffix is mandatory; the system
prefix comes from the cache).  ``deviation_metric="value"`` with
``keep_prefix=True`` is the strict independent-document protocol.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from time import perf_counter
from typing import Any

import torch

from .cacheblend import cacheblend_prefill_oracle
from .config import CacheBlendConfig
from .models.llama import LegacyCache, LlamaOracle


@dataclass(frozen=True)
class GenerationResult:
    token_ids: tuple[int, ...]
    prefill_ms: float
    decode_ms: float
    metadata: dict[str, Any]

    def as_dict(self) -> dict[str, Any]:
        return asdict(self)


def _is_engine(model) -> bool:
    from .models.engine import B200Engine

    return isinstance(model, B200Engine)


def _truncate_eos(tokens, eos) -> tuple[int, ...]:
    out = []
    for t in tokens:
        out.append(int(t))
        if int(t) in eos:
            break
    return tuple(out)


# ------------------------------------------------------------------ engine
def _engine_slot(engine, needed: int):
    slot = getattr(engine, "_api_slot", None)
    if slot is None or slot.capacity < needed:
        cap = max(needed, 1024)
        cap = (cap + 1023) // 1024 * 1024
        engine.release_graphs()
        slot = engine.new_slot(cap)
        engine._api_slot = slot
    return slot


def _load_prefix(engine, slot, prefix_cache: LegacyCache) -> int:
    n = prefix_cache[0][0].shape[2]
    for layer, (k, v) in enumerate(prefix_cache):
        slot.data[layer, 0, :, :n].copy_(k[0], non_blocking=True)
        slot.data[layer, 1, :, :n].copy_(v[0], non_blocking=True)
    return n


def _engine_finish(engine, slot, last_row, position, max_new, eos, ev_start, ev_first, meta):
    engine.first_token(last_row, position=position, max_new=max_new)
    ev_first.record()
    engine.decode(slot, max_new - 1, max_new=max_new)
    ev_end = torch.cuda.Event(enable_timing=True)
    ev_end.record()
    tokens = engine.generated_tokens(max_new).cpu().tolist()
    ev_end.synchronize()
    return GenerationResult(_truncate_eos(tokens, eos), ev_start.elapsed_time(ev_first),
                            ev_first.elapsed_time(ev_end), meta)


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


# ------------------------------------------------------------------ API
@torch.inference_mode()
def baseline_generate(model, *, full_ids, max_new_tokens: int, eos_token_ids) -> GenerationResult:
    """Ordinary full-prompt prefill followed by greedy decode."""
    eos = set(eos_token_ids)
    if _is_engine(model):
        T = len(full_ids)
        slot = _engine_slot(model, T + max_new_tokens)
        start, first = _events()
        ids = torch.tensor(full_ids, dtype=torch.int32).to(model.device, non_blocking=True)
        start.record()
        h = model.prefill(ids, slot)
        return _engine_finish(model, slot, h[T - 1:T], T, max_new_tokens, eos, start, first, {"full_prefill": True})
    started = perf_counter()
    logits, cache = model.prefill(full_ids)
    prefill_ms = (perf_counter() - started) * 1000
    started = perf_counter()
    tokens = model.greedy(logits, cache, len(full_ids), max_new_tokens, eos)
    return GenerationResult(tokens, prefill_ms, (perf_counter() - started) * 1000, {"full_prefill": True})


@torch.inference_mode()
def direct_reuse_generate(model, *, prefix_cache: LegacyCache, suffix_ids, max_new_tokens: int,
                          eos_token_ids) -> GenerationResult:
    """Load the complete reusable prefix KV and prefill only the question suffix."""
    eos = set(eos_token_ids)
    P = prefix_cache[0][0].shape[2]
    S = len(suffix_ids)
    meta = {"full_prefill": False, "document_prefill_tokens": 0, "online_suffix_tokens": S}
    if _is_engine(model):
        slot = _engine_slot(model, P + S + max_new_tokens)
        t0 = perf_counter()
        _load_prefix(model, slot, prefix_cache)
        torch.cuda.synchronize(model.device)
        meta["prefix_h2d_ms"] = (perf_counter() - t0) * 1000
        start, first = _events()
        ids = torch.tensor(suffix_ids, dtype=torch.int32).to(model.device, non_blocking=True)
        start.record()
        h = model.prefill(ids, slot, start=P)
        return _engine_finish(model, slot, h[S - 1:S], P + S, max_new_tokens, eos, start, first, meta)
    device = model.device
    t0 = perf_counter()
    past = tuple((k.to(device, model.dtype), v.to(device, model.dtype)) for k, v in prefix_cache)
    meta["prefix_h2d_ms"] = (perf_counter() - t0) * 1000
    started = perf_counter()
    positions = torch.arange(P, P + S)
    hidden, cache = model.forward_tokens(torch.tensor(suffix_ids), positions, past=past)
    logits = model.logits(hidden[:, -1])[0]
    prefill_ms = (perf_counter() - started) * 1000
    started = perf_counter()
    tokens = model.greedy(logits, cache, P + S, max_new_tokens, eos)
    return GenerationResult(tokens, prefill_ms, (perf_counter() - started) * 1000, meta)


@torch.inference_mode()
def cacheblend_generate(
    model,
    *,
    full_ids,
    prefix_cache: LegacyCache,
    system_tokens: int,
    suffix_tokens: int,
    check_layer: int,
    recompute_ratio: float,
    max_new_tokens: int,
    eos_token_ids,
    deviation_metric: str = "key",
    keep_prefix: bool = False,
) -> GenerationResult:
    """CacheBlend layerwise selective recomputation against a composed prefix cache."""
    eos = set(eos_token_ids)
    T = len(full_ids)
    P = T - suffix_tokens
    if prefix_cache[0][0].shape[2] != P:
        raise ValueError("prefix cache and full prompt lengths disagree")
    blend = CacheBlendConfig(check_layer=check_layer, recompute_ratio=recompute_ratio,
                             deviation_metric=deviation_metric, keep_prefix=keep_prefix,
                             max_new_tokens=max_new_tokens)
    n_layers = model.cfg.n_layers if _is_engine(model) else len(model.layers)
    if not 0 <= check_layer < n_layers:
        raise ValueError("check_layer lies outside the model")
    if _is_engine(model):
        slot = _engine_slot(model, T + max_new_tokens)
        t0 = perf_counter()
        _load_prefix(model, slot, prefix_cache)
        torch.cuda.synchronize(model.device)
        h2d_ms = (perf_counter() - t0) * 1000
        start, first = _events()
        ids = torch.tensor(full_ids, dtype=torch.int32).to(model.device, non_blocking=True)
        start.record()
        h_a, A, dmeta = model.cacheblend(ids, slot, prefix_tokens=system_tokens, suffix_tokens=suffix_tokens,
                                         blend=blend)
        n_doc = P - system_tokens
        meta = {"check_layer": check_layer, "recompute_ratio": recompute_ratio,
                "document_tokens_selected": dmeta["k_selected"], "document_tokens": n_doc,
                "mandatory_suffix_tokens": suffix_tokens, "prefix_h2d_ms": h2d_ms,
                "selected_document_fraction": dmeta["k_selected"] / max(1, n_doc),
                "approximate_layer_token_fraction":
                    (check_layer * T + T + (n_layers - check_layer - 1) * A) / (n_layers * T)}
        result = _engine_finish(model, slot, h_a[A - 1:A], T, max_new_tokens, eos, start, first, meta)
        result.metadata["selection_checksum"] = int(dmeta["checksum"].item())
        return result
    t0 = perf_counter()
    composed = tuple((k.to(model.device, model.dtype), v.to(model.device, model.dtype)) for k, v in prefix_cache)
    h2d_ms = (perf_counter() - t0) * 1000
    started = perf_counter()
    out = cacheblend_prefill_oracle(model, full_ids, composed, prefix_tokens=system_tokens,
                                    suffix_tokens=suffix_tokens, blend=blend)
    prefill_ms = (perf_counter() - started) * 1000
    started = perf_counter()
    tokens = model.greedy(out.logits, out.cache, T, max_new_tokens, eos)
    meta = dict(out.metadata)
    meta.update(mandatory_suffix_tokens=suffix_tokens, prefix_h2d_ms=h2d_ms)
    return GenerationResult(tokens, prefill_ms, (perf_counter() - started) * 1000, meta)


__all__ = ["GenerationResult", "baseline_generate", "direct_reuse_generate", "cacheblend_generate",
           "LlamaOracle"]
