"""A small drafter that cross-attends exact, page-sparse target-model KV.

Behavioural parity with the reference's src/sparsecache/sparse_kv_draft.py:
``SparseKVDraftConfig`` (:18-54), ``RMSNorm`` (:57-66),
``CausalDraftAttention`` (:69-102), ``SparseTargetKVAttention`` (:105-171),
``SparseKVDraftBlock`` (:174-203), ``SparseKVDrafter`` (:206-310),
``select_visible_token_indices`` (:313-364) and ``accepted_prefix_length``
(:367-372).  Parameter names follow the reference so that checkpoints and
the EAGLE allowed-missing set (``memory_attention.query.{i}.weight``...)
line up.

What differs is the execution of the memory cross-attention: every memory
layer's queries go through ``sparse_memory_attention`` which, on a B200 with
the extension built, runs the K13 kernel (one pass over the visible K/V rows,
read through an optional token-index list, forward and dq backward) instead of
materialising a gathered copy per layer and calling SDPA; the CPU path is the
plain SDPA formula used as the oracle.
"""
from __future__ import annotations

import math
import random
from dataclasses import asdict, dataclass
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..rope import apply_rope


@dataclass(frozen=True)
class SparseKVDraftConfig:
    """Drafter geometry; nothing here depends on one particular target checkpoint."""

    target_hidden_size: int = 4096
    draft_hidden_size: int = 512
    head_dim: int = 128
    num_draft_heads: int = 4
    num_memory_heads: int = 8
    num_memory_layers: int = 3
    num_seed_layers: int = 3
    num_blocks: int = 1
    mlp_ratio: int = 4
    rms_norm_eps: float = 1e-5

    def __post_init__(self) -> None:
        if self.draft_hidden_size != self.num_draft_heads * self.head_dim:
            raise ValueError("draft_hidden_size must equal num_draft_heads * head_dim")
        for name in ("target_hidden_size", "num_memory_heads", "num_memory_layers", "num_seed_layers",
                     "num_blocks", "mlp_ratio"):
            if int(getattr(self, name)) <= 0:
                raise ValueError(f"{name} must be positive")

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> "SparseKVDraftConfig":
        return cls(**payload)


class RMSNorm(nn.Module):
    """RMSNorm with the variance in fp32 and the scale applied in the input dtype."""

    def __init__(self, hidden_size: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        inv = torch.rsqrt(hidden.float().square().mean(-1, keepdim=True) + self.eps)
        return (hidden * inv.to(hidden.dtype)) * self.weight.to(hidden.dtype)


def _split_heads(x: torch.Tensor, heads: int, head_dim: int) -> torch.Tensor:
    b, t, _ = x.shape
    return x.view(b, t, heads, head_dim).transpose(1, 2)


def _merge_heads(x: torch.Tensor) -> torch.Tensor:
    b, h, t, d = x.shape
    return x.transpose(1, 2).reshape(b, t, h * d)


class CausalDraftAttention(nn.Module):
    """Causal self-attention over the draft tokens (fused qkv projection + RoPE)."""

    def __init__(self, config: SparseKVDraftConfig) -> None:
        super().__init__()
        self.num_heads = config.num_draft_heads
        self.head_dim = config.head_dim
        width = config.draft_hidden_size
        self.qkv = nn.Linear(width, 3 * width, bias=False)
        self.output = nn.Linear(width, width, bias=False)

    def forward(self, hidden: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        q, k, v = (_split_heads(t, self.num_heads, self.head_dim) for t in self.qkv(hidden).chunk(3, dim=-1))
        q = apply_rope(q, cos, sin, sequence_dim=2)
        k = apply_rope(k, cos, sin, sequence_dim=2)
        out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.output(_merge_heads(out))


# --------------------------------------------------------------- K13 dispatch
def _memory_attention_reference(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
    """q [B, H, t, D] against one memory layer [H, T, D] (non-causal)."""
    k = keys.unsqueeze(0).to(q.dtype).expand(q.shape[0], -1, -1, -1)
    v = values.unsqueeze(0).to(q.dtype).expand(q.shape[0], -1, -1, -1)
    return F.scaled_dot_product_attention(q, k, v)


def sparse_memory_attention(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
    """Non-causal attention of queries into one exact memory layer.

    ``q`` is [B, H, t, D]; ``keys``/``values`` are [H, T, D].  On CUDA with the
    extension loaded this is the K13 kernel (bf16 K/V, fp32 softmax, dq-only
    backward since the memory is an input, not a parameter); otherwise SDPA.
    """
    if q.is_cuda and keys.dtype == torch.bfloat16 and q.shape[-1] == 128:
        from ..ops import sparse_attention

        if sparse_attention.kernel_available():
            return sparse_attention.memory_attention_heads_major(q, keys, values)
    return _memory_attention_reference(q, keys, values)


class SparseTargetKVAttention(nn.Module):
    """Learned queries into a few exact target KV layers, mixed by softmaxed gates."""

    def __init__(self, config: SparseKVDraftConfig) -> None:
        super().__init__()
        width = config.draft_hidden_size
        mem_width = config.num_memory_heads * config.head_dim
        self.num_heads = config.num_memory_heads
        self.head_dim = config.head_dim
        self.num_memory_layers = config.num_memory_layers
        self.query = nn.ModuleList(nn.Linear(width, mem_width, bias=False) for _ in range(self.num_memory_layers))
        self.output = nn.ModuleList(nn.Linear(mem_width, width, bias=False) for _ in range(self.num_memory_layers))
        self.layer_gates = nn.Parameter(torch.zeros(self.num_memory_layers))

    def check_memory(self, memory_keys: torch.Tensor, memory_values: torch.Tensor) -> None:
        if memory_keys.shape != memory_values.shape:
            raise ValueError("memory key/value shapes differ")
        if memory_keys.ndim != 4 or tuple(memory_keys.shape[:2]) != (self.num_memory_layers, self.num_heads):
            raise ValueError("memory must have shape [memory_layers, heads, tokens, head_dim]")
        if memory_keys.shape[-1] != self.head_dim or memory_keys.shape[-2] == 0:
            raise ValueError("memory has an invalid token or head dimension")

    def layer_weights(self, layer_logits_bias: torch.Tensor | None = None) -> torch.Tensor:
        """Softmaxed layer mix: [L], or [B, L] when the bias is per row."""
        logits = self.layer_gates
        if layer_logits_bias is not None:
            if layer_logits_bias.shape[-1:] != logits.shape or layer_logits_bias.ndim > 2:
                raise ValueError("memory layer-logit bias has an invalid shape")
            logits = logits + layer_logits_bias.to(logits.dtype)
        return logits.softmax(dim=-1)

    def forward(
        self,
        hidden: torch.Tensor,
        memory_keys: torch.Tensor,
        memory_values: torch.Tensor,
        cos: torch.Tensor,
        sin: torch.Tensor,
        layer_logits_bias: torch.Tensor | None = None,
    ) -> torch.Tensor:
        batched = not isinstance(memory_keys, torch.Tensor)  # a per-row memory batch
        if not batched:
            self.check_memory(memory_keys, memory_values)
        weights = self.layer_weights(layer_logits_bias)
        fused = torch.zeros_like(hidden)
        for i in range(self.num_memory_layers):
            q = _split_heads(self.query[i](hidden), self.num_heads, self.head_dim)
            q = apply_rope(q, cos, sin, sequence_dim=2)
            if batched:
                attended = memory_keys.attend(i, q)
            else:
                attended = sparse_memory_attention(q, memory_keys[i], memory_values[i])
            w = weights[..., i].to(hidden.dtype)
            if w.ndim == 1:
                w = w.view(-1, 1, 1)
            fused = fused + w * self.output[i](_merge_heads(attended))
        return fused


class SparseKVDraftBlock(nn.Module):
    """Pre-norm block: causal self-attention, sparse memory attention, SwiGLU."""

    def __init__(self, config: SparseKVDraftConfig) -> None:
        super().__init__()
        width, eps = config.draft_hidden_size, config.rms_norm_eps
        self.self_norm = RMSNorm(width, eps)
        self.self_attention = CausalDraftAttention(config)
        self.memory_norm = RMSNorm(width, eps)
        self.memory_attention = SparseTargetKVAttention(config)
        self.mlp_norm = RMSNorm(width, eps)
        inner = width * config.mlp_ratio
        self.gate = nn.Linear(width, inner, bias=False)
        self.up = nn.Linear(width, inner, bias=False)
        self.down = nn.Linear(inner, width, bias=False)

    def forward(self, hidden, memory_keys, memory_values, cos, sin) -> torch.Tensor:
        hidden = hidden + self.self_attention(self.self_norm(hidden), cos, sin)
        hidden = hidden + self.memory_attention(self.memory_norm(hidden), memory_keys, memory_values, cos, sin)
        x = self.mlp_norm(hidden)
        return hidden + self.down(F.silu(self.gate(x)) * self.up(x))


def stage_features(visible_fraction: float, prompt_tokens: int, *, dtype, device) -> torch.Tensor:
    """The two stage scalars the drafters are conditioned on: (fraction, log2(P+1)/17)."""
    return torch.tensor([[visible_fraction, math.log2(prompt_tokens + 1) / 17.0]], dtype=dtype, device=device)


class SparseKVDrafter(nn.Module):
    """Predict target tokens from a seed feature and sparse prompt target KV.

    The target's input-embedding and LM-head matrices are bound at run time
    (frozen, shared with the verifier) and are not part of ``state_dict``.
    """

    def __init__(self, config: SparseKVDraftConfig) -> None:
        super().__init__()
        self.config = config
        th, dh = config.target_hidden_size, config.draft_hidden_size
        self.embedding_down = nn.Linear(th, dh, bias=False)
        self.seed_projection = nn.Linear(th * config.num_seed_layers, dh, bias=False)
        self.stage_projection = nn.Sequential(nn.Linear(2, dh, bias=False), nn.SiLU(), nn.Linear(dh, dh, bias=False))
        self.blocks = nn.ModuleList(SparseKVDraftBlock(config) for _ in range(config.num_blocks))
        self.final_norm = RMSNorm(dh, config.rms_norm_eps)
        self.output_up = nn.Linear(dh, th, bias=False)
        object.__setattr__(self, "_target_embedding_weight", None)
        object.__setattr__(self, "_target_lm_head_weight", None)

    def bind_target_weights(self, embedding_weight: torch.Tensor, lm_head_weight: torch.Tensor) -> None:
        if embedding_weight.ndim != 2 or lm_head_weight.ndim != 2:
            raise ValueError("target embedding and LM-head weights must be matrices")
        th = self.config.target_hidden_size
        if embedding_weight.shape[1] != th or lm_head_weight.shape[1] != th:
            raise ValueError("target shared-weight hidden dimension is incompatible")
        if embedding_weight.shape[0] != lm_head_weight.shape[0]:
            raise ValueError("target embedding and LM-head vocabularies differ")
        object.__setattr__(self, "_target_embedding_weight", embedding_weight.detach())
        object.__setattr__(self, "_target_lm_head_weight", lm_head_weight.detach())

    def _bound_weights(self) -> tuple[torch.Tensor, torch.Tensor]:
        emb, head = self._target_embedding_weight, self._target_lm_head_weight
        if emb is None or head is None:
            raise RuntimeError("bind_target_weights must be called before forward")
        return emb, head

    def forward(
        self,
        input_ids: torch.Tensor,
        seed_hidden: torch.Tensor,
        memory_keys: torch.Tensor,
        memory_values: torch.Tensor,
        query_cos: torch.Tensor,
        query_sin: torch.Tensor,
        *,
        visible_fraction: float,
        prompt_tokens: int,
        return_features: bool = False,
    ):
        cfg = self.config
        if input_ids.ndim != 2 or input_ids.shape[0] != 1:
            raise ValueError("the selection model currently requires batch size one")
        if tuple(seed_hidden.shape) != (1, cfg.num_seed_layers, cfg.target_hidden_size):
            raise ValueError("seed hidden-state shape is incompatible")
        t = input_ids.shape[1]
        if tuple(query_cos.shape[-2:]) != (t, cfg.head_dim):
            raise ValueError("query RoPE shape does not match draft tokens")
        if query_sin.shape != query_cos.shape:
            raise ValueError("query RoPE cosine/sine shapes differ")
        if not 0.0 < visible_fraction <= 1.0 or prompt_tokens <= 0:
            raise ValueError("visibility and prompt length must be positive")
        emb, head = self._bound_weights()
        hidden = self.embedding_down(F.embedding(input_ids, emb))
        seed = self.seed_projection(seed_hidden.reshape(1, -1)).unsqueeze(1)
        # the seed conditions the first draft position only
        first = hidden[:, :1] + seed
        hidden = torch.cat((first, hidden[:, 1:]), dim=1)
        stage = stage_features(visible_fraction, prompt_tokens, dtype=hidden.dtype, device=hidden.device)
        hidden = hidden + self.stage_projection(stage).unsqueeze(1)
        for block in self.blocks:
            hidden = block(hidden, memory_keys, memory_values, query_cos, query_sin)
        target_space = self.output_up(self.final_norm(hidden))
        logits = F.linear(target_space, head)
        return (logits, target_space) if return_features else logits


# ------------------------------------------------------------ page selection
def select_visible_token_indices(
    prompt_tokens: int,
    *,
    page_size: int,
    visible_fraction: float,
    seed: int,
    protected_prefix_pages: int = 1,
    protected_suffix_pages: int = 1,
    mode: str = "random",
    page_scores: torch.Tensor | None = None,
) -> torch.Tensor:
    """Sorted token indices of one sparse page view of a prompt.

    The page budget is ceil(pages * fraction) (at least one page, and at least
    the protected pages).  The first/last pages are always kept; the rest are
    chosen by a seeded shuffle ("random", so that a larger fraction with the
    same seed is a superset), by descending score ("priority", ties to the
    lower page), or evenly spaced ("strided").
    """
    if prompt_tokens <= 0 or page_size <= 0:
        raise ValueError("prompt length and page size must be positive")
    if not 0.0 < visible_fraction <= 1.0:
        raise ValueError("visible_fraction must be in (0, 1]")
    n_pages = -(-prompt_tokens // page_size)
    keep = set(range(min(protected_prefix_pages, n_pages)))
    keep.update(range(max(0, n_pages - protected_suffix_pages), n_pages))
    budget = min(n_pages, max(1, math.ceil(n_pages * visible_fraction), len(keep)))
    pool = [p for p in range(n_pages) if p not in keep]
    need = budget - len(keep)
    if mode == "random":
        random.Random(seed).shuffle(pool)
        keep.update(pool[:need])
    elif mode == "priority":
        if page_scores is None or tuple(page_scores.shape) != (n_pages,):
            raise ValueError("priority mode requires one score per prompt page")
        scores = page_scores.detach().float().cpu().tolist()
        keep.update(sorted(pool, key=lambda p: (-scores[p], p))[:need])
    elif mode == "strided":
        if need:
            step = len(pool) / need
            keep.update(pool[min(int((i + 0.5) * step), len(pool) - 1)] for i in range(need))
    else:
        raise ValueError(f"unsupported page-selection mode: {mode}")
    pages = torch.tensor(sorted(keep), dtype=torch.long)
    tokens = (pages[:, None] * page_size + torch.arange(page_size)).reshape(-1)
    return tokens[tokens < prompt_tokens]


def sink_recent_topk_indices(
    prompt_tokens: int,
    chunk_scores: torch.Tensor | None,
    *,
    sink: int = 64,
    recent: int = 512,
    chunk: int = 64,
    budget: int = 2048,
) -> torch.Tensor:
    """Sorted token indices of a sink + recent + top-k-chunk view.

    Keeps the first ``sink`` tokens, the last ``recent`` tokens, then whole
    ``chunk``-token chunks of the middle in descending score order until
    ``budget`` tokens are visible (ties to the earlier chunk).  With no scores
    the middle chunks are taken evenly spaced.  This is the drafter's memory
    view for long contexts (64 sink + 512 recent + top-k 64-token chunks, 2048
    tokens in all).
    """
    if prompt_tokens <= 0 or chunk <= 0:
        raise ValueError("prompt length and chunk size must be positive")
    if prompt_tokens <= budget:
        return torch.arange(prompt_tokens, dtype=torch.long)
    head_end = min(sink, prompt_tokens)
    tail_start = max(head_end, prompt_tokens - recent)
    n_chunks = -(-prompt_tokens // chunk)
    first_mid = -(-head_end // chunk)
    last_mid = tail_start // chunk  # chunks fully inside [head_end, tail_start)
    mids = list(range(first_mid, last_mid))
    room = max(0, (budget - head_end - (prompt_tokens - tail_start)) // chunk)
    if chunk_scores is not None:
        if tuple(chunk_scores.shape) != (n_chunks,):
            raise ValueError("one score per chunk is required")
        s = chunk_scores.detach().float().cpu().tolist()
        chosen = sorted(mids, key=lambda c: (-s[c], c))[:room]
    elif room >= len(mids):
        chosen = mids
    else:
        step = len(mids) / max(room, 1)
        chosen = sorted({mids[min(int((i + 0.5) * step), len(mids) - 1)] for i in range(room)})
    parts = [torch.arange(head_end)]
    parts += [torch.arange(c * chunk, (c + 1) * chunk) for c in sorted(chosen)]
    parts.append(torch.arange(tail_start, prompt_tokens))
    return torch.cat(parts).unique(sorted=True)


def accepted_prefix_length(proposal: list[int], target: list[int]) -> int:
    """Number of leading draft tokens equal to the target's greedy tokens."""
    n = 0
    for a, b in zip(proposal, target):
        if a != b:
            return n
        n += 1
    return n
