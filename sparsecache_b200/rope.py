"""Rotate-half RoPE with Llama-3.1 frequency scaling, and cached-key relocation.

API parity with the reference's src/sparsecache/rope.py: ``rotate_half``
(rope.py:9-12), ``apply_rope`` (:15-24), ``remove_rope`` (:27-36),
``relocate_key`` (:61-91).  The reference reads cos/sin from an HF model's
``rotary_emb``; this module computes the same schedule from a ModelConfig:
inverse frequencies in fp32 (with the published llama3 scaling rule when the
config has one), angles ``fp32(pos * inv_freq)``, cos/sin in fp32 with the
64 frequencies duplicated over both halves of the head.

``rope_table`` returns the same numbers as a dense [positions, 64, 2]
(cos, sin) fp32 table: the CUDA kernels (QKV epilogue, decode GEMV,
composer) index it by position, so the oracle and the kernels rotate with
bit-identical coefficients.
"""
from __future__ import annotations

import math
from functools import lru_cache

import torch

from .config import ModelConfig


def rotate_half(tensor: torch.Tensor) -> torch.Tensor:
    """[x1, x2] -> [-x2, x1] over the last dimension."""
    half = tensor.shape[-1] // 2
    return torch.cat((-tensor[..., half:], tensor[..., :half]), dim=-1)


def _shape_like(tensor: torch.Tensor, table: torch.Tensor, sequence_dim: int) -> torch.Tensor:
    """Broadcast a [T, D] (or [B, T, D]) table against ``tensor``."""
    sequence_dim %= tensor.ndim
    if table.shape[-1] != tensor.shape[-1]:
        raise ValueError("RoPE head dimension does not match tensor")
    if table.shape[-2] != tensor.shape[sequence_dim]:
        raise ValueError("RoPE token dimension does not match tensor")
    shape = [1] * tensor.ndim
    shape[sequence_dim] = table.shape[-2]
    shape[-1] = table.shape[-1]
    if table.ndim == 3:
        if table.shape[0] != tensor.shape[0]:
            raise ValueError("RoPE batch dimension does not match tensor")
        shape[0] = table.shape[0]
    elif table.ndim != 2:
        raise ValueError("RoPE tables must have two or three dimensions")
    return table.reshape(shape)


def apply_rope(
    tensor: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *, sequence_dim: int = -2
) -> torch.Tensor:
    """Rotate ``tensor`` by the given angles: x*cos + rotate_half(x)*sin."""
    if cos.shape != sin.shape:
        raise ValueError("cos and sin shapes differ")
    c = _shape_like(tensor, cos, sequence_dim)
    s = _shape_like(tensor, sin, sequence_dim)
    return tensor * c + rotate_half(tensor) * s


def remove_rope(
    tensor: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *, sequence_dim: int = -2
) -> torch.Tensor:
    """Undo a rotation (rotations are orthogonal): x*cos - rotate_half(x)*sin."""
    if cos.shape != sin.shape:
        raise ValueError("cos and sin shapes differ")
    c = _shape_like(tensor, cos, sequence_dim)
    s = _shape_like(tensor, sin, sequence_dim)
    return tensor * c - rotate_half(tensor) * s


def inverse_frequencies(config: ModelConfig) -> torch.Tensor:
    """fp32 inverse frequencies, llama3-scaled when the config asks for it.

    The scaling rule is the one published with Llama 3.1: wavelengths longer
    than original_ctx / low_freq_factor are divided by ``factor``; shorter
    than original_ctx / high_freq_factor are kept; the band in between is
    interpolated linearly in 1/wavelength.
    """
    dim = config.head_dim
    exponents = torch.arange(0, dim, 2, dtype=torch.int64).to(torch.float32) / dim
    inv = 1.0 / (config.rope_theta ** exponents)
    scaling = config.rope_scaling
    if scaling is None:
        return inv
    low_wavelen = scaling.original_max_position_embeddings / scaling.low_freq_factor
    high_wavelen = scaling.original_max_position_embeddings / scaling.high_freq_factor
    wavelen = 2 * math.pi / inv
    scaled = torch.where(wavelen > low_wavelen, inv / scaling.factor, inv)
    smooth = (scaling.original_max_position_embeddings / wavelen - scaling.low_freq_factor) / (
        scaling.high_freq_factor - scaling.low_freq_factor
    )
    interpolated = (1 - smooth) * scaled / scaling.factor + smooth * scaled
    in_band = (wavelen >= high_wavelen) & (wavelen <= low_wavelen)
    return torch.where(in_band, interpolated, scaled).to(torch.float32)


def rope_cos_sin(
    config: ModelConfig,
    positions: torch.Tensor,
    *,
    dtype: torch.dtype = torch.float32,
    device: torch.device | str | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin of shape [..., head_dim] for integer ``positions`` (fp32 math)."""
    inv = inverse_frequencies(config)
    pos = positions.to(device="cpu", dtype=torch.float32)
    angles = pos.unsqueeze(-1) * inv  # fp32 product, as HF's rotary embedding
    emb = torch.cat((angles, angles), dim=-1)
    cos, sin = emb.cos(), emb.sin()
    target = device if device is not None else positions.device
    return cos.to(device=target, dtype=dtype), sin.to(device=target, dtype=dtype)


@lru_cache(maxsize=8)
def _host_table(config_json: str, n_positions: int) -> torch.Tensor:
    config = ModelConfig.from_dict(__import__("json").loads(config_json))
    cos, sin = rope_cos_sin(config, torch.arange(n_positions))
    half = config.head_dim // 2
    return torch.stack((cos[:, :half], sin[:, :half]), dim=-1).reshape(n_positions, 2 * half)


def rope_table(config: ModelConfig, n_positions: int, device: torch.device | str = "cpu") -> torch.Tensor:
    """[n_positions, head_dim] fp32 table of interleaved (cos_i, sin_i) pairs."""
    return _host_table(config.to_json(), int(n_positions)).to(device)


def relocate_key(
    config: ModelConfig, key: torch.Tensor, *, source_start: int, target_start: int
) -> torch.Tensor:
    """Move a post-RoPE key [B, H, T, D] from positions source_start.. to target_start..

    Removes the source rotation and applies the target one in fp32, then
    casts back to the key's dtype (reference rope.py:61-91).
    """
    if source_start == target_start:
        return key
    tokens = key.shape[2]
    return relocate_positions(
        config,
        key,
        torch.arange(source_start, source_start + tokens),
        torch.arange(target_start, target_start + tokens),
    )


def relocate_positions(
    config: ModelConfig,
    key: torch.Tensor,
    source_positions: torch.Tensor,
    target_positions: torch.Tensor,
) -> torch.Tensor:
    """Per-token relocation of a [B, H, T, D] key between arbitrary positions.

    Batched form of the reference's relocate_document_keys
    (reuse_cacheblend_pipeline.py:407-449): one fp32 pass for a concatenation
    of documents whose local positions restart at 0.
    """
    if source_positions.numel() != key.shape[2] or target_positions.numel() != key.shape[2]:
        raise ValueError("relocation maps must cover every token")
    src_cos, src_sin = rope_cos_sin(config, source_positions, device=key.device)
    dst_cos, dst_sin = rope_cos_sin(config, target_positions, device=key.device)
    canonical = remove_rope(key.float(), src_cos, src_sin, sequence_dim=2)
    return apply_rope(canonical, dst_cos, dst_sin, sequence_dim=2).to(key.dtype)
