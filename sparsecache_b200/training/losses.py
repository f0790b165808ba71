"""Drafter training losses.

Same definitions as the reference trainers:
  * ``weighted_distillation_loss``: prefix-decayed hard CE on the greedy
    labels plus soft CE against the renormalised teacher top-k
    (experiments/train_sparse_kv_drafter.py:57-97);
  * ``prefix_weights`` (:100-113), ``feature_distillation_loss`` (cosine
    distance to the verifier's normalised LM-head input, :116-135) and
    ``target_sequence_score`` (prefix-weighted label log-probability used by
    the memory-contrast margin, :138-152);
  * ``compressed_distillation_loss`` / ``compressed_target_score``: the same
    losses in EAGLE's compressed draft vocabulary, skipping labels and
    teacher ids that have no draft id (experiments/train_sparse_kv_eagle.py:97-175).
    They are written on (row log-sum-exp, logits at the label / top-k ids):
    logp[id] = z[id] - lse, so the ``*_from_lse`` forms take the output of
    the fused LM-head path (``ops.lm_loss``) and never need [B, t, V].

Every function accepts a leading batch dimension (``[B, t, V]`` logits and
``[B, t]`` labels) in addition to the reference's batch-1 shapes; the batch
losses are the mean of the per-sequence losses.  Nothing here calls
``.item()`` in the loss itself, so a training step built on these functions
can be captured in a CUDA graph; ``components`` holds device tensors.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def prefix_weights(tokens: int, *, prefix_decay: float, device=None) -> torch.Tensor:
    """decay**i normalised to sum 1 over ``tokens`` positions."""
    if tokens <= 0 or not 0.0 < prefix_decay <= 1.0:
        raise ValueError("invalid prefix-weight parameters")
    w = prefix_decay ** torch.arange(tokens, dtype=torch.float32, device=device)
    return w / w.sum()


def _batched(logits: torch.Tensor, labels: torch.Tensor):
    if logits.ndim != 3:
        raise ValueError("logits must have shape [batch, tokens, vocabulary]")
    if labels.ndim == 1:
        labels = labels.unsqueeze(0)
    if labels.shape != logits.shape[:2]:
        raise ValueError("labels do not match logits")
    return logits, labels


def weighted_distillation_loss(
    logits: torch.Tensor,
    labels: torch.Tensor,
    teacher_topk_ids: torch.Tensor,
    teacher_topk_logprobs: torch.Tensor,
    *,
    prefix_decay: float,
    hard_weight: float,
    soft_weight: float,
):
    """Hard CE on greedy labels + soft CE on the renormalised teacher top-k."""
    if teacher_topk_ids.shape != teacher_topk_logprobs.shape:
        raise ValueError("teacher top-k IDs and log-probabilities differ")
    if not 0.0 < prefix_decay <= 1.0:
        raise ValueError("prefix_decay must be in (0, 1]")
    if min(hard_weight, soft_weight) < 0.0 or hard_weight + soft_weight <= 0.0:
        raise ValueError("loss weights must be non-negative and non-zero")
    if logits.ndim == 3 and logits.shape[0] != 1 and labels.ndim == 1:
        raise ValueError("labels do not match logits")
    logits, labels = _batched(logits, labels)
    ids = teacher_topk_ids if teacher_topk_ids.ndim == 3 else teacher_topk_ids.unsqueeze(0)
    lps = teacher_topk_logprobs if teacher_topk_logprobs.ndim == 3 else teacher_topk_logprobs.unsqueeze(0)
    if ids.shape[:2] != labels.shape:
        raise ValueError("teacher top-k length does not match logits")
    logp = logits.float().log_softmax(-1)
    hard = -logp.gather(-1, labels.unsqueeze(-1)).squeeze(-1)  # [B, t]
    soft = -(lps.float().softmax(-1) * logp.gather(-1, ids)).sum(-1)
    w = prefix_weights(labels.shape[1], prefix_decay=prefix_decay, device=logits.device)
    hard_loss = (hard * w).sum(-1).mean()
    soft_loss = (soft * w).sum(-1).mean()
    total = hard_weight * hard_loss + soft_weight * soft_loss
    return total, {"hard_loss": hard_loss.detach(), "soft_loss": soft_loss.detach()}


def feature_distillation_loss(features: torch.Tensor, teacher_hidden: torch.Tensor, *, prefix_decay: float):
    """Prefix-weighted cosine distance between student and verifier features."""
    if features.ndim != 3:
        raise ValueError("student features must have shape [batch, tokens, hidden]")
    if teacher_hidden.ndim == 2:
        teacher_hidden = teacher_hidden.unsqueeze(0)
    if teacher_hidden.shape != features.shape:
        raise ValueError("teacher hidden states do not match student features")
    cos = (F.normalize(features.float(), dim=-1) * F.normalize(teacher_hidden.float(), dim=-1)).sum(-1)
    w = prefix_weights(features.shape[1], prefix_decay=prefix_decay, device=features.device)
    return ((1.0 - cos) * w).sum(-1).mean()


def target_sequence_score(logits: torch.Tensor, labels: torch.Tensor, *, prefix_decay: float) -> torch.Tensor:
    """Prefix-weighted log-probability of the labels ([B] for batched input)."""
    batched = labels.ndim == 2
    logits, labels = _batched(logits, labels)
    lp = logits.float().log_softmax(-1).gather(-1, labels.unsqueeze(-1)).squeeze(-1)
    w = prefix_weights(labels.shape[1], prefix_decay=prefix_decay, device=logits.device)
    score = (lp * w).sum(-1)
    return score if batched else score[0]


def compressed_id_table(model, labels: torch.Tensor, teacher_ids: torch.Tensor | None) -> torch.Tensor:
    """Draft-vocabulary id table [B, t, 1 + K]: the label, then the teacher top-k (-1 = unmapped)."""
    d_lab = model.draft_ids(labels).unsqueeze(-1)
    if teacher_ids is None:
        return d_lab
    ids = teacher_ids if teacher_ids.ndim == 3 else teacher_ids.unsqueeze(0)
    return torch.cat((d_lab, model.draft_ids(ids)), dim=-1)


def compressed_distillation_from_lse(
    lse: torch.Tensor,
    z: torch.Tensor,
    table: torch.Tensor,
    teacher_logprobs: torch.Tensor,
    *,
    prefix_decay: float,
    hard_weight: float,
    soft_weight: float,
    check_coverage: bool = True,
):
    """``compressed_distillation_loss`` from the row log-sum-exp and the logits at ``table``.

    ``lse`` [B, t]; ``z`` / ``table`` [B, t, 1 + K] (label column first, ids
    < 0 unmapped).  logp[id] = z - lse, so the loss needs no [B, t, V] tensor.
    """
    lps = teacher_logprobs if teacher_logprobs.ndim == 3 else teacher_logprobs.unsqueeze(0)
    B, t = lse.shape
    w = prefix_weights(t, prefix_decay=prefix_decay, device=lse.device)
    d_lab, d_ids = table[..., 0], table[..., 1:]
    ok_hard = d_lab >= 0
    hw = w * ok_hard.float()
    hard = -(z[..., 0] - lse)
    h_den = hw.sum(-1)
    hard_loss = torch.where(h_den > 0, (hard * hw).sum(-1) / h_den.clamp_min(1.0), torch.zeros_like(h_den))
    ok_soft = d_ids >= 0
    ok_rows = ok_soft.any(-1)
    t_logits = lps.float().masked_fill(~ok_soft, float("-inf"))
    t_logits = torch.where(ok_rows.unsqueeze(-1), t_logits, torch.zeros_like(t_logits))
    probs = t_logits.softmax(-1)
    soft = -(probs * (z[..., 1:] - lse.unsqueeze(-1))).sum(-1)
    sw = w * ok_rows.float()
    s_den = sw.sum(-1)
    soft_loss = torch.where(s_den > 0, (soft * sw).sum(-1) / s_den.clamp_min(1.0), torch.zeros_like(s_den))
    if check_coverage and bool(((h_den == 0) & (s_den == 0)).any()):
        raise ValueError("teacher labels and top-k are outside EAGLE vocabulary")
    hard_loss, soft_loss = hard_loss.mean(), soft_loss.mean()
    loss = hard_weight * hard_loss + soft_weight * soft_loss
    return loss, {
        "hard_loss": hard_loss.detach(),
        "soft_loss": soft_loss.detach(),
        "label_coverage": ok_hard.float().mean().detach(),
        "topk_coverage": ok_soft.float().mean().detach(),
    }


def compressed_target_score_from_lse(lse: torch.Tensor, z_label: torch.Tensor, d_label: torch.Tensor, *,
                                     prefix_decay: float) -> torch.Tensor:
    """``compressed_target_score`` ([B]) from lse [B, t] and the label logits [B, t]."""
    w = prefix_weights(lse.shape[1], prefix_decay=prefix_decay, device=lse.device) * (d_label >= 0).float()
    sel = z_label - lse
    den = w.sum(-1)
    return torch.where(den > 0, (w * sel).sum(-1) / den.clamp_min(1.0), lse.sum(-1) * 0.0)


def compressed_distillation_loss(
    model,
    logits: torch.Tensor,
    labels: torch.Tensor,
    teacher_ids: torch.Tensor,
    teacher_logprobs: torch.Tensor,
    *,
    prefix_decay: float,
    hard_weight: float,
    soft_weight: float,
    check_coverage: bool = True,
):
    """Distillation in the EAGLE draft vocabulary; unmapped targets are skipped.

    Hard CE averages over labels that have a draft id (prefix-weighted);
    the soft term renormalises the teacher top-k over the ids that map and
    skips rows where none does.  With ``check_coverage`` a batch whose labels
    and top-k all fall outside the draft vocabulary raises (this reads one
    device scalar; the graph-captured trainer passes False).
    """
    from ..ops.lm_loss import lse_gather

    logits, labels = _batched(logits, labels)
    table = compressed_id_table(model, labels, teacher_ids)
    B, t, V = logits.shape
    lse, z = lse_gather(logits.reshape(B * t, V), table.reshape(B * t, -1))
    return compressed_distillation_from_lse(lse.view(B, t), z.view(B, t, -1), table, teacher_logprobs,
                                            prefix_decay=prefix_decay, hard_weight=hard_weight,
                                            soft_weight=soft_weight, check_coverage=check_coverage)


def compressed_target_score(model, logits: torch.Tensor, labels: torch.Tensor, *, prefix_decay: float):
    """Prefix-weighted draft-vocabulary log-probability of the mapped labels."""
    from ..ops.lm_loss import lse_gather

    batched = labels.ndim == 2
    logits, labels = _batched(logits, labels)
    table = compressed_id_table(model, labels, None)
    B, t, V = logits.shape
    lse, z = lse_gather(logits.reshape(B * t, V), table.reshape(B * t, 1))
    score = compressed_target_score_from_lse(lse.view(B, t), z.view(B, t), table[..., 0], prefix_decay=prefix_decay)
    return score if batched else score[0]


def components_to_floats(components: dict) -> dict[str, float]:
    """Host copy of a components dict (one sync), for logging."""
    return {k: float(v) for k, v in components.items()}
