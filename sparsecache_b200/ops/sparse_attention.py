"""Autograd wrapper and per-row memory batches for the K13 memory attention.

``MemoryAttention`` is a ``torch.autograd.Function`` over the extension's
``mem_attn_fwd`` / ``mem_attn_bwd``: queries [L, R, H, 128] bf16 attend to
strided bf16 memory; the backward returns dq only (memory K/V are inputs of
the drafter, never trained).

``MemoryBatch`` holds the memories of several sequences in one token-major
buffer [S, L, T, H, 128] with a per-sequence visible-token index list, so a
batch of drafter rows, each with its own sparse view (sink + recent + top
chunks, or a random/priority page view), is attended in one launch per
memory layer, reading K/V rows in place.  Its CPU path gathers and runs
masked SDPA; that is the oracle the kernel is tested against.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _C, ext


def kernel_available() -> bool:
    return _C is not None


class MemoryAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, strides, row_seq, idx, idx_stride, n_vis, n_fixed, scale):
        x = ext()
        q = q.contiguous()
        out = torch.empty_like(q)
        lse = torch.empty(q.shape[:3], device=q.device, dtype=torch.float32)
        x.mem_attn_fwd(q, k, v, *strides, row_seq, idx, idx_stride, n_vis, n_fixed, scale, out, lse)
        ctx.save_for_backward(q, k, v, out, lse, row_seq, idx, n_vis)
        ctx.meta = (strides, idx_stride, n_fixed, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, row_seq, idx, n_vis = ctx.saved_tensors
        strides, idx_stride, n_fixed, scale = ctx.meta
        dq = torch.empty(q.shape, device=q.device, dtype=torch.float32)
        ext().mem_attn_bwd(q, k, v, *strides, row_seq, idx, idx_stride, n_vis, n_fixed, scale, out,
                           dout.contiguous().to(torch.bfloat16), lse, dq)
        return dq.to(q.dtype), None, None, None, None, None, None, None, None, None


def _rows_major(q: torch.Tensor) -> torch.Tensor:
    """[B, H, t, D] -> [1, B*t, H, D] (row r = b*t + i)."""
    b, h, t, d = q.shape
    return q.transpose(1, 2).reshape(1, b * t, h, d)


def _rows_to_heads(o: torch.Tensor, b: int, t: int) -> torch.Tensor:
    _, _, h, d = o.shape
    return o.view(b, t, h, d).transpose(1, 2)


def memory_attention_heads_major(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
    """q [B, H, t, 128] into one shared memory layer [H, T, 128] (all rows see all T)."""
    b, h, t, d = q.shape
    keys = keys.contiguous()
    values = values.contiguous()
    T = keys.shape[1]
    q_rows = _rows_major(q.to(torch.bfloat16))
    strides = (0, 0, d, T * d)
    out = MemoryAttention.apply(q_rows, keys, values, strides, None, None, 0, None, T, 1.0 / math.sqrt(d))
    return _rows_to_heads(out, b, t).to(q.dtype)


class MemoryBatch:
    """Sparse memories of S sequences for a batch of drafter rows.

    ``keys``/``values``: [S, L, T, H, D] bf16 (token-major, as the target's KV
    caches are); ``idx``: [S, V] int32 visible token indices (each row sorted,
    padded past ``n_vis``); ``n_vis``: [S] int32; ``row_seq``: [B] int32, the
    memory sequence of each batch row (rows of a negative/contrast pass simply
    point at another sequence).  ``zero`` replaces the memory by zeros (the
    "zero memory" ablation) without a copy on the kernel path.
    """

    def __init__(self, keys, values, idx, n_vis, row_seq, zero: bool = False) -> None:
        if keys.shape != values.shape or keys.ndim != 5:
            raise ValueError("memory must be [S, L, T, H, D] keys and values")
        self.keys, self.values = keys, values
        self.idx, self.n_vis, self.row_seq = idx, n_vis, row_seq
        self.zero = zero

    @property
    def num_layers(self) -> int:
        return self.keys.shape[1]

    def with_rows(self, row_seq: torch.Tensor) -> "MemoryBatch":
        return MemoryBatch(self.keys, self.values, self.idx, self.n_vis, row_seq, self.zero)

    def _use_kernel(self, q: torch.Tensor) -> bool:
        return q.is_cuda and kernel_available() and self.keys.dtype == torch.bfloat16 and q.shape[-1] == 128

    def attend(self, layer: int, q: torch.Tensor) -> torch.Tensor:
        """q [B, H, t, D] (row b uses sequence row_seq[b]) -> [B, H, t, D]."""
        b, h, t, d = q.shape
        if self.zero:
            # softmax over equal (zero) scores of zero values: exactly zero output
            return torch.zeros_like(q) + 0.0 * q
        if self._use_kernel(q):
            S, L, T, H, D = self.keys.shape
            row_seq = self.row_seq if t == 1 else self.row_seq.repeat_interleave(t)
            strides = (T * H * D, L * T * H * D, H * D, D)
            kl = self.keys[:, layer:layer + 1]  # layer offset via the base pointer
            vl = self.values[:, layer:layer + 1]
            out = MemoryAttention.apply(_rows_major(q.to(torch.bfloat16)), kl, vl, strides, row_seq, self.idx,
                                        self.idx.shape[1], self.n_vis, 0, 1.0 / math.sqrt(d))
            return _rows_to_heads(out, b, t).to(q.dtype)
        return self.attend_reference(layer, q)

    def attend_reference(self, layer: int, q: torch.Tensor) -> torch.Tensor:
        b, h, t, d = q.shape
        seq = self.row_seq.long().to(self.keys.device)
        V = self.idx.shape[1]
        idx = self.idx.long().to(self.keys.device)[seq]  # [B, V]
        k = self.keys[seq, layer]  # [B, T, H, D]
        v = self.values[seq, layer]
        gather = idx[:, :, None, None].expand(-1, -1, h, d).clamp_min(0)
        ks = torch.gather(k, 1, gather).transpose(1, 2).to(q.dtype)  # [B, H, V, D]
        vs = torch.gather(v, 1, gather).transpose(1, 2).to(q.dtype)
        valid = torch.arange(V, device=idx.device)[None, :] < self.n_vis.long().to(idx.device)[seq][:, None]
        mask = valid[:, None, None, :].expand(b, 1, t, V)
        return F.scaled_dot_product_attention(q, ks, vs, attn_mask=mask)
