"""Pure-PyTorch Llama decoder: the CPU plumbing model and the numerics oracle.

This is a self-contained Llama-style decoder (RMSNorm, GQA attention with
rotate-half RoPE, SwiGLU MLP), written against ModelConfig instead of HF
Transformers so that it runs anywhere (fp32 on CPU for the tiny plumbing
config, or any dtype on GPU).  It exposes the layer-level pieces the
CacheBlend algorithm needs (project_qkv / attention / mlp), mirroring the
manual layer loop of the reference (modeling.py:126-327,
reuse_cacheblend_pipeline.py:512-706).

KV caches use the reference's legacy layout: a tuple over layers of
(key, value) tensors shaped [1, n_kv_heads, tokens, head_dim]
(store.py:30-54).  The B200 engine (models/engine.py) is tested against
this module.
"""
from __future__ import annotations

import math

import torch
from torch import nn
from torch.nn import functional as F

from ..config import ModelConfig
from ..rope import apply_rope, rope_cos_sin

LegacyCache = tuple[tuple[torch.Tensor, torch.Tensor], ...]


class RMSNorm(nn.Module):
    """LlamaRMSNorm: fp32 variance, normalised value cast back before the weight."""

    def __init__(self, dim: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        xf = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps)
        return self.weight * xf.to(x.dtype)


class LlamaLayer(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        d, hd = cfg.d_model, cfg.head_dim
        self.q_proj = nn.Linear(d, cfg.n_heads * hd, bias=False)
        self.k_proj = nn.Linear(d, cfg.n_kv_heads * hd, bias=False)
        self.v_proj = nn.Linear(d, cfg.n_kv_heads * hd, bias=False)
        self.o_proj = nn.Linear(cfg.n_heads * hd, d, bias=False)
        self.gate_proj = nn.Linear(d, cfg.ffn, bias=False)
        self.up_proj = nn.Linear(d, cfg.ffn, bias=False)
        self.down_proj = nn.Linear(cfg.ffn, d, bias=False)
        self.input_layernorm = RMSNorm(d, cfg.rms_eps)
        self.post_attention_layernorm = RMSNorm(d, cfg.rms_eps)

    def mlp(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class LlamaOracle(nn.Module):
    """Llama decoder with explicit-position prefill, decode and layer access."""

    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.config = cfg
        self.embed_tokens = nn.Embedding(cfg.vocab, cfg.d_model)
        self.layers = nn.ModuleList(LlamaLayer(cfg) for _ in range(cfg.n_layers))
        self.norm = RMSNorm(cfg.d_model, cfg.rms_eps)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab, bias=False)
        self.scaling = 1.0 / math.sqrt(cfg.head_dim)

    # ------------------------------------------------------------ creation
    @classmethod
    def random_init(
        cls,
        cfg: ModelConfig,
        *,
        seed: int = 0,
        dtype: torch.dtype = torch.float32,
        device: torch.device | str = "cpu",
        std: float = 0.02,
    ) -> "LlamaOracle":
        """Seeded random initialisation (normal(0, std) matrices, unit norms)."""
        gen = torch.Generator(device="cpu").manual_seed(seed)
        model = cls(cfg)
        with torch.no_grad():
            for name, param in model.named_parameters():
                if name.endswith("layernorm.weight") or name == "norm.weight":
                    param.fill_(1.0)
                else:
                    param.copy_(torch.randn(param.shape, generator=gen) * std)
        return model.to(device=device, dtype=dtype).eval()

    @property
    def device(self) -> torch.device:
        return self.embed_tokens.weight.device

    @property
    def dtype(self) -> torch.dtype:
        return self.embed_tokens.weight.dtype

    # ------------------------------------------------------- layer pieces
    def rope(self, positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """cos/sin [T, head_dim] in the model dtype (HF rotary_emb semantics)."""
        return rope_cos_sin(self.config, positions, dtype=self.dtype, device=self.device)

    def project_qkv(
        self, layer: LlamaLayer, normed: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor
    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """[B, T, d] -> post-RoPE q [B, H, T, D], k/v [B, Hkv, T, D]."""
        hd = self.config.head_dim
        shape = (*normed.shape[:-1], -1, hd)
        q = layer.q_proj(normed).view(shape).transpose(1, 2)
        k = layer.k_proj(normed).view(shape).transpose(1, 2)
        v = layer.v_proj(normed).view(shape).transpose(1, 2)
        return apply_rope(q, cos, sin, sequence_dim=2), apply_rope(k, cos, sin, sequence_dim=2), v

    def attention(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        *,
        query_positions: torch.Tensor,
        key_positions: torch.Tensor,
    ) -> torch.Tensor:
        """Attention with the predicate key_pos <= query_pos (GQA by head repeat)."""
        groups = q.shape[1] // k.shape[1]
        if groups > 1:
            k = k.repeat_interleave(groups, dim=1)
            v = v.repeat_interleave(groups, dim=1)
        mask = key_positions.unsqueeze(0) <= query_positions.unsqueeze(1)
        return F.scaled_dot_product_attention(
            q, k, v, attn_mask=mask[None, None], dropout_p=0.0, scale=self.scaling
        )

    def block_rest(
        self, layer: LlamaLayer, residual: torch.Tensor, attended: torch.Tensor
    ) -> torch.Tensor:
        """o_proj + residual, then the MLP block."""
        attended = attended.transpose(1, 2).reshape(residual.shape[0], residual.shape[1], -1)
        hidden = residual + layer.o_proj(attended)
        return hidden + layer.mlp(layer.post_attention_layernorm(hidden))

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.lm_head(self.norm(hidden))

    # ------------------------------------------------------- whole passes
    @torch.no_grad()
    def forward_tokens(
        self,
        ids: torch.Tensor,
        positions: torch.Tensor,
        past: LegacyCache | None = None,
        past_positions: torch.Tensor | None = None,
    ) -> tuple[torch.Tensor, LegacyCache]:
        """Run ``ids`` [T] at ``positions`` [T] after an optional past cache.

        Returns (hidden [1, T, d] after the final layer, new cache covering
        past + these tokens).  Keys are visible iff key_pos <= query_pos.
        """
        ids = ids.to(self.device).view(1, -1)
        positions = positions.to(self.device)
        hidden = self.embed_tokens(ids)
        cos, sin = self.rope(positions)
        if past is not None:
            if past_positions is None:
                past_positions = torch.arange(past[0][0].shape[2], device=self.device)
            key_positions = torch.cat((past_positions.to(self.device), positions))
        else:
            key_positions = positions
        cache = []
        for index, layer in enumerate(self.layers):
            residual = hidden
            q, k, v = self.project_qkv(layer, layer.input_layernorm(hidden), cos, sin)
            if past is not None:
                k = torch.cat((past[index][0].to(k.dtype), k), dim=2)
                v = torch.cat((past[index][1].to(v.dtype), v), dim=2)
            attended = self.attention(q, k, v, query_positions=positions, key_positions=key_positions)
            hidden = self.block_rest(layer, residual, attended)
            cache.append((k, v))
        return hidden, tuple(cache)

    @torch.no_grad()
    def prefill(self, ids, start: int = 0) -> tuple[torch.Tensor, LegacyCache]:
        """Causal prefill at positions start..start+T-1; returns (last logits [V], cache)."""
        ids = torch.as_tensor(ids, dtype=torch.long)
        positions = torch.arange(start, start + ids.numel())
        hidden, cache = self.forward_tokens(ids, positions)
        return self.logits(hidden[:, -1])[0], cache

    @torch.no_grad()
    def decode_step(self, token: int, position: int, cache: LegacyCache) -> tuple[torch.Tensor, LegacyCache]:
        ids = torch.tensor([token], dtype=torch.long)
        hidden, cache = self.forward_tokens(ids, torch.tensor([position]), past=cache)
        return self.logits(hidden[:, -1])[0], cache

    @torch.no_grad()
    def greedy(
        self, logits: torch.Tensor, cache: LegacyCache, position: int, max_new_tokens: int, eos: set[int]
    ) -> tuple[int, ...]:
        """Greedy continuation (reference modeling.py:383-417)."""
        out = []
        for step in range(max_new_tokens):
            token = int(logits.float().argmax())
            out.append(token)
            if token in eos or step + 1 == max_new_tokens:
                break
            logits, cache = self.decode_step(token, position, cache)
            position += 1
        return tuple(out)

    @torch.no_grad()
    def encode_local(self, ids) -> LegacyCache:
        """KV of a segment prefilled alone at local positions 0..n-1 (the producer)."""
        _, cache = self.prefill(ids, start=0)
        return cache
