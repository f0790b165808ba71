"""CacheBlend selective recomputation over a composed document cache (oracle path).

This is the algorithm of the reference, expressed on the PyTorch oracle
model; the B200 engine (models/engine.py) implements the same contract with
fused sm_100a kernels and is tested against it.

Algorithm (reference modeling.py:126-327 and the strict variant
reuse_cacheblend_pipeline.py:512-706):
  * layers before ``check_layer`` recompute every prompt row with full
    causal attention and replace the cached K/V;
  * at ``check_layer`` every row is projected, document rows are ranked by
    the deviation between the fresh and the cached K or V (squared L2 by
    default, L1 and K+V variants selectable), the top ceil(ratio * N_doc)
    are kept, and the mandatory rows (the question suffix, plus the system
    prefix in the strict protocol) are always kept; only those rows continue;
  * later layers recompute only the active rows, scatter their fresh K/V
    into the composed cache and attend over all positions with the
    predicate key_pos <= query_pos (positions, not a triangular mask).
Ratio 1.0 reproduces full prefill exactly (every row active).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Sequence

import torch

from .config import CacheBlendConfig, ModelConfig
from .models.llama import LegacyCache, LlamaOracle
from .rope import relocate_positions


def recompute_count(n_document_tokens: int, ratio: float) -> int:
    """Number of document rows recomputed (reference: max(1, ceil(N * ratio)))."""
    if n_document_tokens <= 0:
        return 0
    return min(n_document_tokens, max(1, math.ceil(n_document_tokens * ratio)))


def deviation_scores(
    fresh_k: torch.Tensor,
    fresh_v: torch.Tensor,
    cached_k: torch.Tensor,
    cached_v: torch.Tensor,
    metric: str,
) -> torch.Tensor:
    """Per-token deviation [T] of fresh vs cached K/V ([1, Hkv, T, D] each)."""
    def reduce(fresh, cached, l1):
        diff = fresh.float() - cached.float()
        return (diff.abs() if l1 else diff.square()).sum(dim=(0, 1, 3))

    l1 = metric.endswith("_l1")
    base = metric.replace("_l1", "")
    score = None
    if base in ("key", "kv"):
        score = reduce(fresh_k, cached_k, l1)
    if base in ("value", "kv"):
        value_score = reduce(fresh_v, cached_v, l1)
        score = value_score if score is None else score + value_score
    if score is None:
        raise ValueError(f"unknown deviation metric {metric!r}")
    return score


def select_active(
    scores: torch.Tensor,
    *,
    doc_begin: int,
    doc_end: int,
    total: int,
    ratio: float,
    keep_prefix: bool,
) -> tuple[torch.Tensor, torch.Tensor]:
    """(sorted active positions, selected document positions)."""
    device = scores.device
    n_doc = doc_end - doc_begin
    k = recompute_count(n_doc, ratio)
    if k > 0:
        local = torch.topk(scores, k=k, sorted=False).indices
        selected = local + doc_begin
    else:
        selected = torch.empty(0, dtype=torch.long, device=device)
    parts = []
    if keep_prefix:
        parts.append(torch.arange(0, doc_begin, device=device))
    parts.append(selected)
    parts.append(torch.arange(doc_end, total, device=device))
    return torch.cat(parts).sort().values, selected


def selection_checksum(selected: torch.Tensor) -> int:
    """sum(rank * position) over the sorted selection (reuse_cacheblend_pipeline.py:661-668)."""
    ordered = selected.sort().values.to(torch.int64)
    ranks = torch.arange(1, ordered.numel() + 1, dtype=torch.int64, device=ordered.device)
    return int((ordered * ranks).sum())


@dataclass
class BlendOutput:
    cache: LegacyCache
    logits: torch.Tensor
    active_positions: torch.Tensor
    selected_positions: torch.Tensor
    metadata: dict[str, Any] = field(default_factory=dict)


def compose_documents(
    config: ModelConfig,
    document_caches: Sequence[LegacyCache],
    *,
    prefix_tokens: int,
    system_cache: LegacyCache | None = None,
    source_starts: Sequence[int] | None = None,
) -> LegacyCache:
    """Concatenate per-document caches after a prefix and relocate their keys.

    Documents were produced at positions ``source_starts`` (0 for the
    independent-document producer); they land contiguously after the
    prefix.  The prefix region holds ``system_cache`` when given, zeros
    otherwise (the reference's zero placeholder, README.md:73-75).
    """
    n_layers = config.n_layers
    sample_k = document_caches[0][0][0]
    keys: list[list[torch.Tensor]] = [[] for _ in range(n_layers)]
    values: list[list[torch.Tensor]] = [[] for _ in range(n_layers)]
    for layer in range(n_layers):
        if system_cache is not None:
            keys[layer].append(system_cache[layer][0].to(sample_k.dtype))
            values[layer].append(system_cache[layer][1].to(sample_k.dtype))
        elif prefix_tokens:
            shape = (1, config.n_kv_heads, prefix_tokens, config.head_dim)
            keys[layer].append(torch.zeros(shape, dtype=sample_k.dtype, device=sample_k.device))
            values[layer].append(torch.zeros(shape, dtype=sample_k.dtype, device=sample_k.device))
    cursor = prefix_tokens
    for index, cache in enumerate(document_caches):
        n = cache[0][0].shape[2]
        src = 0 if source_starts is None else int(source_starts[index])
        for layer in range(n_layers):
            key, value = cache[layer]
            if src != cursor:
                key = relocate_positions(
                    config, key, torch.arange(src, src + n), torch.arange(cursor, cursor + n)
                )
            keys[layer].append(key)
            values[layer].append(value)
        cursor += n
    return tuple(
        (torch.cat(keys[layer], dim=2), torch.cat(values[layer], dim=2)) for layer in range(n_layers)
    )


@torch.no_grad()
def cacheblend_prefill_oracle(
    model: LlamaOracle,
    ids: Sequence[int] | torch.Tensor,
    composed: LegacyCache,
    *,
    prefix_tokens: int,
    suffix_tokens: int,
    blend: CacheBlendConfig,
    global_positions: torch.Tensor | None = None,
) -> BlendOutput:
    """CacheBlend prefill of ``ids`` against ``composed`` (prefix + documents).

    With a gradual schedule (several check layers) every later check layer
    projects the rows still active, writes their fresh K/V, ranks the active
    document rows by deviation from the composed cache and keeps the top
    ``ratio * N_doc`` of them (ratios relative to the original document count).
    """
    device = model.device
    ids = torch.as_tensor(ids, dtype=torch.long, device=device).view(1, -1)
    total = ids.shape[1]
    raw_len = total - suffix_tokens
    if composed[0][0].shape[2] != raw_len:
        raise ValueError("composed cache and prompt lengths disagree")
    sched = blend.schedule
    if sched[-1][0] >= len(model.layers):
        raise ValueError("check_layer lies outside the model")
    first = sched[0][0]
    ratio_at = dict(sched)
    local = torch.arange(total, device=device)
    gpos = local if global_positions is None else global_positions.to(device)
    hidden = model.embed_tokens(ids)
    cos, sin = model.rope(gpos)
    active = local
    selected = None
    cache = []
    work = 0  # rows projected, summed over layers
    for index, layer in enumerate(model.layers):
        residual = hidden
        normed = layer.input_layernorm(hidden)
        work += int(active.numel())
        q, k, v = model.project_qkv(layer, normed, cos.index_select(0, active), sin.index_select(0, active))
        if index < first:
            attended = model.attention(q, k, v, query_positions=gpos, key_positions=gpos)
            cache_k, cache_v = k, v
        else:
            if index == first:
                cache_k, cache_v = k, v
            else:
                old_k, old_v = composed[index]
                pad = total - old_k.shape[2]
                cache_k = torch.nn.functional.pad(old_k, (0, 0, 0, pad)).clone()
                cache_v = torch.nn.functional.pad(old_v, (0, 0, 0, pad)).clone()
                cache_k[:, :, active] = k.to(cache_k.dtype)
                cache_v[:, :, active] = v.to(cache_v.dtype)
            if index in ratio_at:
                old_k, old_v = composed[index]
                doc = slice(prefix_tokens, raw_len)
                scores = deviation_scores(cache_k[:, :, doc], cache_v[:, :, doc], old_k[:, :, doc], old_v[:, :, doc],
                                          blend.deviation_metric)
                if index != first:  # only rows still active compete
                    live = torch.zeros(raw_len - prefix_tokens, dtype=torch.bool, device=device)
                    live[(selected - prefix_tokens)] = True
                    scores = torch.where(live, scores, torch.full_like(scores, float("-inf")))
                new_active, selected = select_active(scores, doc_begin=prefix_tokens, doc_end=raw_len, total=total,
                                                     ratio=ratio_at[index], keep_prefix=blend.keep_prefix)
                keep = torch.searchsorted(active, new_active)  # rows of ``hidden`` that stay
                q = q.index_select(2, keep)
                residual = residual.index_select(1, keep)
                active = new_active
            attended = model.attention(q, cache_k, cache_v, query_positions=gpos.index_select(0, active),
                                       key_positions=gpos)
        hidden = model.block_rest(layer, residual, attended)
        cache.append((cache_k, cache_v))
    last = (active == total - 1).nonzero()
    if last.numel() != 1:
        raise RuntimeError("the final suffix token is not active")
    logits = model.logits(hidden[:, int(last[0, 0])])[0]
    assert selected is not None
    n_doc = raw_len - prefix_tokens
    trace = blend.layer_document_trace(len(model.layers))
    return BlendOutput(
        cache=tuple(cache),
        logits=logits,
        active_positions=active,
        selected_positions=selected,
        metadata={
            "check_layer": blend.check_layer,
            "recompute_ratio": blend.recompute_ratio,
            "deviation_metric": blend.deviation_metric,
            "document_tokens": n_doc,
            "document_tokens_selected": int(selected.numel()),
            "selected_document_fraction": int(selected.numel()) / max(1, n_doc),
            "active_rows": int(active.numel()),
            "approximate_layer_token_fraction": work / (len(model.layers) * total),
            "check_layers": [c for c, _ in blend.schedule],
            "recompute_ratios": [r for _, r in blend.schedule],
            "layer_document_trace": trace,
            "layer_document_mean": blend.check_target(len(model.layers)),
            "selection_checksum": selection_checksum(selected),
        },
    )
