"""Frozen linear layers on the tcgen05 GEMM, forward and backward (drafter trunk training).

The EAGLE trunk of the sparse-KV drafter is frozen: its projections need the
activation gradient dX = dY @ W but no weight gradient.  ``FrozenTCLinear``
replaces an ``nn.Linear``'s forward with

    forward : Y  = X @ W^T      (tcgen05, bf16 in / bf16 out, fp32 accumulate)
    backward: dX = dY @ W       (the same on a transposed copy W^T [K, N], made once)

Up to 64 rows (the trainer's batch rows per recurrent position) the product
runs on the swap-AB skinny GEMM, which streams the weight at HBM rate with the
rows as the MMA's N; above, on the tiled tcgen05 GEMM.

so the trunk's fc / q / k / v / o / gate / up / down run on this package's
kernels instead of cuBLAS through autograd (reference trunk:
src/sparsecache/sparse_kv_eagle.py:69-170, trained with the adapter in
experiments/train_sparse_kv_eagle.py:521-525, 683-686).  Shapes the GEMM does
not take (N not a multiple of 32, K not a multiple of 8) and CPU tensors keep
``F.linear``.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import available, ext


def _tc_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (available() and x.is_cuda and w.dtype == torch.bfloat16 and w.shape[0] % 32 == 0
            and w.shape[1] % 8 == 0 and x.shape[-1] == w.shape[1])


_SPLITS: dict[tuple[int, int], int] = {}


def _matmul_t(x2: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
    """out = x2 @ w^T on the tensor cores: the swap-AB skinny GEMM (weight streaming) up to 64 rows,
    the tiled tcgen05 GEMM above."""
    M, (N, K) = x2.shape[0], w.shape
    if M == 0:
        return
    if M <= 64 and K % 64 == 0:
        key = (N, K)
        if key not in _SPLITS:
            _SPLITS[key] = int(ext().skinny_splits(N, K))
        bn = 16 if M <= 16 else (32 if M <= 32 else 64)
        ws = torch.empty(_SPLITS[key] * N * bn, device=x2.device, dtype=torch.float32)
        ext().skinny_gemm(x2, w, 0, out, None, ws)
    else:
        ext().gemm_store(x2, w, out, 256, -1)


class _FrozenLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, w_t):
        K = w.shape[1]
        x2 = x.reshape(-1, K)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = x2.contiguous()
        out = torch.empty(x2.shape[0], w.shape[0], device=x.device, dtype=torch.bfloat16)
        _matmul_t(x2, w, out)
        ctx.save_for_backward(w_t)
        ctx.in_shape, ctx.in_dtype = x.shape, x.dtype
        return out.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, g):
        (w_t,) = ctx.saved_tensors
        N = w_t.shape[1]
        g2 = g.reshape(-1, N)
        if g2.dtype != torch.bfloat16:
            g2 = g2.to(torch.bfloat16)
        g2 = g2.contiguous()
        dx = torch.empty(g2.shape[0], w_t.shape[0], device=g.device, dtype=torch.bfloat16)
        _matmul_t(g2, w_t, dx)
        dx = dx.view(ctx.in_shape)
        return (dx if ctx.in_dtype == torch.bfloat16 else dx.to(ctx.in_dtype)), None, None


class FrozenTCLinear:
    """Callable standing in for a frozen bias-free ``nn.Linear``'s forward."""

    def __init__(self, weight: torch.Tensor) -> None:
        if weight.requires_grad:
            raise ValueError("FrozenTCLinear is for frozen weights")
        self.weight = weight
        self.weight_t = weight.t().contiguous() if weight.is_cuda else None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.weight_t is None or not _tc_ok(x, self.weight):
            return F.linear(x.to(self.weight.dtype), self.weight)
        return _FrozenLinear.apply(x, self.weight, self.weight_t)


def use_tc_for_frozen_linears(module: nn.Module) -> list[str]:
    """Route every frozen, bias-free bf16 ``nn.Linear`` under ``module`` through the tcgen05 GEMM.

    Trainable linears (the adapter) keep autograd's path.  Returns the names
    of the layers switched."""
    switched = []
    for name, sub in module.named_modules():
        if (isinstance(sub, nn.Linear) and sub.bias is None and not sub.weight.requires_grad
                and sub.weight.dtype == torch.bfloat16 and sub.weight.is_cuda):
            sub.forward = FrozenTCLinear(sub.weight)  # instance attribute: shadows nn.Linear.forward
            switched.append(name)
    return switched


class _RecurrentAttention(torch.autograd.Function):
    """softmax(q K^T * scale) V for one query position per head over all past keys (no mask)."""

    @staticmethod
    def forward(ctx, q, k, v, scale):
        q3 = q.reshape(q.shape[0], q.shape[1], q.shape[-1]).to(torch.bfloat16).contiguous()
        k4, v4 = k.to(torch.bfloat16).contiguous(), v.to(torch.bfloat16).contiguous()
        out, lse = ext().recurrent_attention_fwd(q3, k4, v4, float(scale))
        ctx.save_for_backward(q3, k4, v4, out, lse)
        ctx.scale = float(scale)
        ctx.dtypes = (q.dtype, k.dtype, v.dtype)
        ctx.q_shape = q.shape
        return out.view(q.shape)

    @staticmethod
    def backward(ctx, g):
        q3, k4, v4, out, lse = ctx.saved_tensors
        dout = g.reshape(out.shape).to(torch.bfloat16).contiguous()
        dq, dk, dv = ext().recurrent_attention_bwd(q3, k4, v4, out, lse, dout, ctx.scale)
        qd, kd, vd = ctx.dtypes
        return dq.view(ctx.q_shape).to(qd), dk.to(kd), dv.to(vd), None


# the K14 kernels serve recurrent_attention on CUDA; False routes it to SDPA (A/B measurements)
USE_RECURRENT_ATTENTION_KERNEL = True


def recurrent_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None):
    """Attention of one new position (q [B, Hq, 1, D]) over keys / values [B, Hkv, P, D], Hq = G * Hkv.

    On CUDA with the extension: this package's forward / backward kernels (K14); otherwise PyTorch
    SDPA with the query heads of a KV group folded into the query length."""
    b, hq, t, d = q.shape
    hkv = k.shape[1]
    scale = d ** -0.5 if scale is None else scale
    if (USE_RECURRENT_ATTENTION_KERNEL and available() and q.is_cuda and t == 1 and d == 128 and hq % hkv == 0
            and hq // hkv <= 8 and 1 <= k.shape[2] <= 1024):
        return _RecurrentAttention.apply(q, k, v, scale)
    qg = q.reshape(b, hkv, (hq // hkv) * t, d)
    return F.scaled_dot_product_attention(qg, k, v, scale=scale).reshape(b, hq, t, d)
