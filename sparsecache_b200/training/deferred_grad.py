"""Adapter weight gradients formed after the recurrence, one tensor-core GEMM per weight.

The drafter adapter's memory projections (``memory_attention.query[i]`` and
``memory_attention.output[i]``) are applied at every one of the 256 teacher-
forced positions of a training step.  Under plain autograd each position adds
its own ``x_t^T dy_t`` product to each weight's gradient: 256 small GEMMs per
weight and step, summed in bf16 by the autograd engine (every use shares the
one cached bf16 cast of the weight), and no weight's gradient is final before
the whole backward has returned, so a data-parallel exchange cannot start
earlier.

Here those linears propagate activation gradients only.  Their forward
stores its input rows and their backward stores the output-gradient rows,
both transposed (feature-major, so the rows of all positions form the K
dimension of one GEMM), and after the backward one tcgen05 GEMM per weight
forms ``dW = dY^T X`` over all positions with fp32 accumulation, straight
into the weight's slice of the flat gradient buffer.  Each finished weight
is reported to a callback: the data-parallel optimizer starts that weight's
peer-memory reduce-scatter on a side stream while the next GEMM runs.

The function computed is the reference's (experiments/train_sparse_kv_eagle.py
trains the same adapter with ``loss.backward()`` at :521-525 and steps the
optimizer at :683-686); only the order of the summation over positions and
its precision (fp32 instead of bf16) differ.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops

ROW_ALIGN = 64  # the GEMM's K tile: stashes are padded to it with zero columns


class WeightGradStash:
    """Feature-major stores of the inputs and output gradients of deferred linears."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.linears: list[nn.Linear] = []
        self.xT: list[torch.Tensor] = []
        self.dyT: list[torch.Tensor] = []
        self.w16: list[torch.Tensor] = []
        self.calls: list[int] = []
        self.rows_per_call = 0
        self.max_calls = 0
        self.active = False
        # bf16 on the GPU (the trainer's autocast dtype, the GEMM's operand type); fp32 on the
        # host, where the trainer runs without autocast
        self.dtype = torch.bfloat16 if device.type == "cuda" else torch.float32

    def register(self, linear: nn.Linear) -> int:
        if linear.bias is not None:
            raise ValueError("deferred weight gradients cover bias-free linears only")
        self.linears.append(linear)
        self.calls.append(0)
        return len(self.linears) - 1

    def begin(self, rows_per_call: int, max_calls: int) -> None:
        """Start a forward pass whose deferred linears see ``rows_per_call`` rows per call."""
        if (rows_per_call, max_calls) != (self.rows_per_call, self.max_calls):
            self._allocate(rows_per_call, max_calls)
        self.calls = [0] * len(self.linears)
        self.active = True

    def _allocate(self, rows_per_call: int, max_calls: int) -> None:
        total = rows_per_call * max_calls
        padded = -(-total // ROW_ALIGN) * ROW_ALIGN
        bf = self.dtype
        # zero columns past the last call contribute nothing to dW
        self.xT = [torch.zeros(l.in_features, padded, device=self.device, dtype=bf) for l in self.linears]
        self.dyT = [torch.zeros(l.out_features, padded, device=self.device, dtype=bf) for l in self.linears]
        self.w16 = [torch.empty(l.out_features, l.in_features, device=self.device, dtype=bf) for l in self.linears]
        self.rows_per_call, self.max_calls = rows_per_call, max_calls

    def next_call(self, key: int, weight: torch.Tensor) -> int:
        idx = self.calls[key]
        if idx >= self.max_calls:
            raise RuntimeError(f"deferred linear {key} called more than {self.max_calls} times in one pass")
        if idx == 0:  # the weights change only at the optimizer step: one bf16 copy per pass
            self.w16[key].copy_(weight.detach())
        self.calls[key] = idx + 1
        return idx

    def _cols(self, idx: int) -> slice:
        return slice(idx * self.rows_per_call, (idx + 1) * self.rows_per_call)

    def put_x(self, key: int, idx: int, rows: torch.Tensor) -> None:
        if rows.shape[0] != self.rows_per_call:
            raise ValueError(f"deferred linear expected {self.rows_per_call} rows per call, got {rows.shape[0]}")
        self.xT[key][:, self._cols(idx)].copy_(rows.t())

    def put_dy(self, key: int, idx: int, rows: torch.Tensor) -> None:
        self.dyT[key][:, self._cols(idx)].copy_(rows.t())

    def finish(self, on_weight: Callable[[int], None] | None = None,
               order: Sequence[int] | None = None) -> None:
        """dW = dY^T X of every deferred linear into its ``.grad`` (overwritten), in ``order``.

        ``on_weight(key)`` runs after each weight's GEMM has been enqueued.
        Every call of the pass must have gone through the backward.
        """
        self.active = False
        for key in (order if order is not None else range(len(self.linears))):
            w = self.linears[key].weight
            g = w.grad
            if g is None or g.dtype != torch.float32 or not g.is_contiguous():
                raise RuntimeError("deferred weights need a contiguous fp32 .grad (a flat-buffer view)")
            if self.device.type == "cuda":
                ops.ext().gemm_f32(self.dyT[key], self.xT[key], g)
            else:  # host oracle of the same product (CPU tests)
                torch.mm(self.dyT[key].float(), self.xT[key].float().t(), out=g)
            if on_weight is not None:
                on_weight(key)


class _DeferredLinearFn(torch.autograd.Function):
    """y = x W^T in the stash dtype; the backward returns dX only and stores dY for the stash."""

    @staticmethod
    def forward(ctx, x, weight, stash: WeightGradStash, key: int):  # noqa: ARG004 (weight: graph link only)
        idx = stash.next_call(key, weight)
        xb = x.to(stash.dtype)
        stash.put_x(key, idx, xb.reshape(-1, xb.shape[-1]))
        ctx.stash, ctx.key, ctx.idx, ctx.x_dtype = stash, key, idx, x.dtype
        return F.linear(xb, stash.w16[key])

    @staticmethod
    def backward(ctx, gy):
        stash = ctx.stash
        g = gy.to(stash.dtype)
        stash.put_dy(ctx.key, ctx.idx, g.reshape(-1, g.shape[-1]))
        gx = torch.matmul(g, stash.w16[ctx.key]).to(ctx.x_dtype)
        return gx, None, None, None


class DeferredGradLinear(nn.Linear):
    """An ``nn.Linear`` (same parameters and state-dict names) whose weight gradient the stash forms.

    Outside a stash pass (no-grad evaluation, drafting) it is a plain linear.
    """

    _stash: WeightGradStash
    _key: int

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        st = self._stash
        if st.active and torch.is_grad_enabled() and self.weight.requires_grad:
            return _DeferredLinearFn.apply(x, self.weight, st, self._key)
        return F.linear(x, self.weight, self.bias)


def defer_adapter_linears(model: nn.Module, device: torch.device) -> WeightGradStash | None:
    """Switch the trainable memory projections of a ``SparseKVEagleDrafter`` to deferred gradients.

    Returns the stash, or None when no such projection is trainable.  The
    modules keep their parameters (same objects, same names).
    """
    mem = getattr(model, "memory_attention", None)
    if mem is None:
        return None
    stash = WeightGradStash(device)
    for lin in (*mem.query, *mem.output):
        if type(lin) is nn.Linear and lin.bias is None and lin.weight.requires_grad:
            key = stash.register(lin)
            lin.__class__ = DeferredGradLinear
            lin._stash, lin._key = stash, key
    return stash if stash.linears else None


def restore_linears(stash: WeightGradStash | None) -> None:
    """Turn the deferred linears back into plain ``nn.Linear`` modules."""
    if stash is None:
        return
    for lin in stash.linears:
        if isinstance(lin, DeferredGradLinear):
            del lin._stash, lin._key
            lin.__class__ = nn.Linear
