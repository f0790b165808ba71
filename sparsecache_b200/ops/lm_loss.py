"""LM head + log-sum-exp + logit gathers for the drafter losses (no fp32 [rows, vocab] tensors).

Every drafter loss term reads the log-softmax only at a few ids per row
(label, teacher top-k): logp[id] = z[id] - lse.  ``lm_head_lse_gather``
returns (lse [R], z [R, G]) for feature rows and an id table; its backward
turns the small gradients (g_lse, g_z) into the logits gradient
g_lse * softmax + sum_j g_z[j] * onehot(ids[j]) with one kernel pass and
multiplies by the frozen LM head with the tcgen05 GEMM:

    forward : logits = feats @ W^T (tcgen05 GEMM, bf16)   -> lse_gather kernel
    backward: dlogits (lse_gather_backward, in place)     -> dfeats = dlogits @ W (tcgen05 GEMM, W^T copy)

The bf16 logits are kept for the backward (one [R, V] bf16 buffer; the
log-probabilities, their gradient and the one-hot gathers of the plain
PyTorch formulation are fp32 [R, V] each).  On the CPU (no extension) the
same decomposition runs in PyTorch, which the tests compare against the
log-softmax formulation.
"""
from __future__ import annotations

import torch

from . import available, ext


def lse_gather_reference(logits: torch.Tensor, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(logsumexp over the last dim, logits at ``ids`` (0 where id < 0)) in fp32, differentiable."""
    x = logits.float()
    lse = x.logsumexp(-1)
    z = x.gather(-1, ids.clamp_min(0).long()) * (ids >= 0)
    return lse, z


class _LseGather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, ids):
        R, G = ids.shape
        lse = torch.empty(R, device=logits.device, dtype=torch.float32)
        z = torch.empty(R, G, device=logits.device, dtype=torch.float32)
        ext().lse_gather(logits, ids, lse, z)
        ctx.save_for_backward(logits, ids, lse)
        return lse, z

    @staticmethod
    def backward(ctx, g_lse, g_z):
        logits, ids, lse = ctx.saved_tensors
        d = torch.empty_like(logits)
        ext().lse_gather_backward(logits, ids, lse, None if g_lse is None else g_lse.float().contiguous(),
                                  None if g_z is None else g_z.float().contiguous(), d)
        return d, None


class _LMHeadLseGather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, feats, w, w_t, ids):
        R = feats.shape[0]
        V = w.shape[0]
        logits = torch.empty(R, V, device=feats.device, dtype=torch.bfloat16)
        ext().gemm_store(feats, w, logits, 256, -1)
        lse = torch.empty(R, device=feats.device, dtype=torch.float32)
        z = torch.empty(R, ids.shape[1], device=feats.device, dtype=torch.float32)
        ext().lse_gather(logits, ids, lse, z)
        ctx.save_for_backward(logits, ids, lse, w_t)
        return lse, z

    @staticmethod
    def backward(ctx, g_lse, g_z):
        logits, ids, lse, w_t = ctx.saved_tensors
        ext().lse_gather_backward(logits, ids, lse, None if g_lse is None else g_lse.float().contiguous(),
                                  None if g_z is None else g_z.float().contiguous(), logits)  # in place
        dfeats = torch.empty(logits.shape[0], w_t.shape[0], device=logits.device, dtype=torch.bfloat16)
        ext().gemm_store(logits, w_t, dfeats, 256, -1)
        return dfeats, None, None, None


def _kernel_ok(t: torch.Tensor) -> bool:
    return t.is_cuda and available() and t.dtype == torch.bfloat16


def lse_gather(logits: torch.Tensor, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(lse [R], z [R, G]) of 2-D logits and an int32 id table (kernel on CUDA bf16)."""
    if _kernel_ok(logits):
        return _LseGather.apply(logits.contiguous(), ids.to(torch.int32).contiguous())
    return lse_gather_reference(logits, ids)


class FrozenLMHead:
    """A frozen LM head ([V, d]) with its transposed copy for the fused loss path."""

    def __init__(self, weight: torch.Tensor) -> None:
        self.w = weight.detach().to(torch.bfloat16).contiguous()
        self.w_t = self.w.t().contiguous() if self.w.is_cuda else None

    def lse_gather(self, feats: torch.Tensor, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(lse, z) of feats [R, d] against the head; differentiable in ``feats`` only."""
        ids = ids.to(torch.int32).contiguous()
        if _kernel_ok(self.w) and feats.is_cuda:
            return _LMHeadLseGather.apply(feats.to(torch.bfloat16).contiguous(), self.w, self.w_t, ids)
        return lse_gather_reference(feats.to(self.w.dtype) @ self.w.t(), ids)
