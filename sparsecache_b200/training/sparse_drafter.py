"""Training and evaluation of the 512-wide ``SparseKVDrafter``.

Parity with the reference's experiments/train_sparse_kv_drafter.py (the
training loop :575-897: page-view memory per step with the visibility
fraction cycled per sample, optional windows, seed dropout, prefix-decayed
hard + top-k soft distillation, cosine feature loss, a margin contrast
against another request's memory, AdamW with gradient clipping, checkpoint
``sparsecache.sparse-kv-drafter.v1`` without the target's shared weights),
its ``evaluate`` (:383-509: teacher-forced top-1 and the accepted prefix of
greedy drafts under exact / zero / shuffled memory and exact / zero seed),
experiments/eval_sparse_kv_boundaries.py (post-verification windows at
evenly spaced offsets, summarised by source group :30-178) and
experiments/eval_sparse_kv_drafter.py (the five-cell memory x seed ablation
:45-171).  On a B200 the memory attention inside the drafter runs the K13
kernel; the drafter's batch-1 API is kept, as the reference's.
"""
from __future__ import annotations

import json
import random
import time
from collections import defaultdict
from pathlib import Path
from typing import Any, Sequence

import torch
import torch.nn.functional as F

from ..models.sparse_kv_draft import SparseKVDraftConfig, SparseKVDrafter, accepted_prefix_length
from .losses import feature_distillation_loss, target_sequence_score, weighted_distillation_loss
from .teacher import TeacherSample, sample_inputs, select_memory, training_window_inputs

CHECKPOINT_FORMAT = "sparsecache.sparse-kv-drafter.v1"


def _autocast(device):
    dev = torch.device(device)
    return torch.autocast(device_type=dev.type, dtype=torch.bfloat16, enabled=dev.type == "cuda")


def train_sparse_drafter(model: SparseKVDrafter, train: Sequence[TeacherSample], *, fractions: Sequence[float],
                         steps: int, device, page_size: int = 64, selection_mode: str = "random", lr: float = 3e-4,
                         weight_decay: float = 0.01, prefix_decay: float = 0.9, hard_weight: float = 1.0,
                         soft_weight: float = 0.5, feature_weight: float = 1.0, seed_dropout_prob: float = 0.25,
                         contrast_weight: float = 0.5, contrast_margin: float = 0.5, gradient_clip: float = 1.0,
                         window_tokens: int = 0, initial_window_prob: float = 0.25, seed: int = 0,
                         log_every: int = 10, log=None) -> list[dict[str, Any]]:
    """The reference's training loop (batch size 1, one sample per step)."""
    rng = random.Random(seed)
    opt = torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=weight_decay)
    history = []
    model.train()
    t0 = time.perf_counter()
    for step in range(1, steps + 1):
        si, epoch = (step - 1) % len(train), (step - 1) // len(train)
        sample = train[si]
        frac = fractions[(si + epoch) % len(fractions)]
        keys, values, actual, visible = select_memory(sample, page_size=page_size, requested_fraction=frac,
                                                      seed=seed + step * 7919 + sample.request_index, device=device,
                                                      selection_mode=selection_mode)
        offset = 0
        if window_tokens > 0 and sample.horizon > 1 and rng.random() >= initial_window_prob:
            offset = rng.randrange(1, sample.horizon)
        if window_tokens > 0:
            ids, seed_h, cos, sin, labels, tids, tlp = training_window_inputs(sample, device, offset=offset,
                                                                              window_tokens=window_tokens)
        else:
            ids, seed_h, cos, sin, labels, tids, tlp = sample_inputs(sample, device)
        th = sample.tensors.get("teacher_hidden")
        if feature_weight > 0 and th is None:
            raise ValueError("feature loss requires teacher hidden states")
        if th is not None:
            if offset == 0 and "initial_teacher_hidden" in sample.tensors:
                th = sample.tensors["initial_teacher_hidden"]
            th = th[offset:offset + ids.shape[1]].to(device)
        seed_h = torch.zeros_like(seed_h) if rng.random() < seed_dropout_prob else seed_h
        opt.zero_grad(set_to_none=True)
        with _autocast(device):
            logits, feats = model(ids, seed_h, keys, values, cos, sin, visible_fraction=actual,
                                  prompt_tokens=sample.prompt_tokens, return_features=True)
            loss, comps = weighted_distillation_loss(logits, labels, tids, tlp, prefix_decay=prefix_decay,
                                                     hard_weight=hard_weight, soft_weight=soft_weight)
            if feature_weight > 0:
                f_loss = feature_distillation_loss(feats, th, prefix_decay=prefix_decay)
                loss = loss + feature_weight * f_loss
                comps["feature_loss"] = f_loss.detach()
            if contrast_weight > 0:
                neg = train[step % len(train)]
                nk, nv, _, _ = select_memory(neg, page_size=page_size, requested_fraction=frac,
                                             seed=seed + step * 7919 + neg.request_index, device=device,
                                             selection_mode=selection_mode)
                neg_logits = model(ids, seed_h, nk, nv, cos, sin, visible_fraction=actual,
                                   prompt_tokens=sample.prompt_tokens)
                c = F.relu(contrast_margin - target_sequence_score(logits, labels, prefix_decay=prefix_decay)
                           + target_sequence_score(neg_logits, labels, prefix_decay=prefix_decay))
                loss = loss + contrast_weight * c
                comps["contrast_loss"] = c.detach()
        if not torch.isfinite(loss):
            raise FloatingPointError(f"non-finite loss at step {step}")
        loss.backward()
        gnorm = torch.nn.utils.clip_grad_norm_(model.parameters(), gradient_clip)
        opt.step()
        if step % log_every == 0 or step == steps:
            row = {"step": step, "request_index": sample.request_index, "requested_fraction": frac,
                   "actual_fraction": actual, "visible_tokens": visible, "loss": float(loss.detach()),
                   "grad_norm": float(gnorm), "elapsed_s": time.perf_counter() - t0,
                   **{k: float(v) for k, v in comps.items()}}
            history.append(row)
            if log is not None:
                log(row)
    return history


@torch.inference_mode()
def evaluate_sparse_drafter(model, samples: Sequence[TeacherSample], fractions: Sequence[float], *, device,
                            page_size: int = 64, selection_seed: int = 0, memory_mode: str = "exact",
                            seed_mode: str = "exact", selection_mode: str = "random",
                            max_proposal_tokens: int = 8) -> list[dict[str, Any]]:
    """Teacher-forced top-1 and greedy accepted prefix per visibility fraction."""
    if memory_mode not in {"exact", "zero", "shuffled"} or seed_mode not in {"exact", "zero"}:
        raise ValueError("unsupported memory or seed mode")
    model.eval()
    out = []
    for frac in fractions:
        accepted, horizons, correct, total, visible = [], [], 0, 0, []
        for i, s in enumerate(samples):
            ms = samples[(i + 1) % len(samples)] if memory_mode == "shuffled" else s
            k, v, actual, nvis = select_memory(ms, page_size=page_size, requested_fraction=frac,
                                               seed=selection_seed + ms.request_index * 1009, device=device,
                                               selection_mode=selection_mode)
            if memory_mode == "zero":
                k, v = torch.zeros_like(k), torch.zeros_like(v)
            ids, seed_h, cos, sin, labels, _, _ = sample_inputs(s, device)
            n = min(labels.numel(), max_proposal_tokens)
            ids, cos, sin, labels = ids[:, :n], cos[:n], sin[:n], labels[:n]
            if seed_mode == "zero":
                seed_h = torch.zeros_like(seed_h)
            with _autocast(device):
                pred = model(ids, seed_h, k, v, cos, sin, visible_fraction=actual,
                             prompt_tokens=s.prompt_tokens)[0].argmax(-1)
            correct += int((pred == labels).sum())
            total += n
            prefix, prop = ids[:, :1], []
            for _ in range(n):
                with _autocast(device):
                    lg = model(prefix, seed_h, k, v, cos[:prefix.shape[1]], sin[:prefix.shape[1]],
                               visible_fraction=actual, prompt_tokens=s.prompt_tokens)
                t = int(lg[0, -1].argmax())
                prop.append(t)
                prefix = torch.cat((prefix, torch.tensor([[t]], device=prefix.device)), dim=1)
            accepted.append(accepted_prefix_length(prop, labels.tolist()))
            horizons.append(n)
            visible.append(nvis)
        out.append({"memory_mode": memory_mode, "seed_mode": seed_mode, "selection_mode": selection_mode,
                    "requested_fraction": frac, "samples": len(samples),
                    "mean_visible_tokens": sum(visible) / len(visible), "teacher_forced_top1": correct / total,
                    "mean_accepted_prefix": sum(accepted) / len(accepted),
                    "full_accept_rate": sum(a == h for a, h in zip(accepted, horizons)) / len(samples),
                    "accepted_prefixes": accepted})
    return out


def five_cell_ablation(model, samples, fractions, *, device, **kw) -> dict[str, list[dict]]:
    """exact/exact, zero memory, shuffled memory, zero seed, zero/zero."""
    cells = {"exact": ("exact", "exact"), "zero_memory": ("zero", "exact"), "shuffled_memory": ("shuffled", "exact"),
             "zero_seed": ("exact", "zero"), "zero_memory_zero_seed": ("zero", "zero")}
    return {name: evaluate_sparse_drafter(model, samples, fractions, device=device, memory_mode=m, seed_mode=sd, **kw)
            for name, (m, sd) in cells.items()}


def select_offsets(horizon: int, maximum: int) -> tuple[int, ...]:
    """Up to ``maximum`` evenly spaced post-verification offsets in [1, horizon)."""
    if horizon <= 1 or maximum <= 0:
        return ()
    cand = list(range(1, horizon))
    if len(cand) <= maximum:
        return tuple(cand)
    return tuple(cand[min(len(cand) - 1, i * len(cand) // maximum)] for i in range(maximum))


def summarize_windows(rows: Sequence[dict]) -> dict[str, Any]:
    tokens = sum(int(r["tokens"]) for r in rows)
    return {"windows": len(rows), "tokens": tokens,
            "teacher_forced_top1": sum(int(r["correct"]) for r in rows) / max(tokens, 1),
            "mean_accepted_prefix": sum(int(r["accepted"]) for r in rows) / max(len(rows), 1),
            "full_accept_rate": sum(int(r["accepted"]) == int(r["tokens"]) for r in rows) / max(len(rows), 1)}


@torch.inference_mode()
def evaluate_boundaries(model, samples: Sequence[TeacherSample], fractions: Sequence[float], *, device,
                        page_size: int = 64, selection_seed: int = 0, selection_mode: str = "random",
                        memory_mode: str = "exact", window_tokens: int = 8,
                        maximum_windows_per_sample: int = 4) -> list[dict[str, Any]]:
    """Drafts that start after a verification boundary (v5 data), by source group."""
    if memory_mode not in {"exact", "zero", "shuffled"}:
        raise ValueError("unsupported boundary memory mode")
    model.eval()
    results = []
    for frac in fractions:
        rows = []
        for i, s in enumerate(samples):
            ms = samples[(i + 1) % len(samples)] if memory_mode == "shuffled" else s
            k, v, actual, _ = select_memory(ms, page_size=page_size, requested_fraction=frac,
                                            seed=selection_seed + ms.request_index * 1009, device=device,
                                            selection_mode=selection_mode)
            if memory_mode == "zero":
                k, v = torch.zeros_like(k), torch.zeros_like(v)
            for off in select_offsets(s.horizon, maximum_windows_per_sample):
                ids, seed_h, cos, sin, labels, _, _ = training_window_inputs(s, device, offset=off,
                                                                             window_tokens=window_tokens)
                with _autocast(device):
                    lg = model(ids, seed_h, k, v, cos, sin, visible_fraction=actual, prompt_tokens=s.prompt_tokens)
                pred = lg[0].argmax(-1)
                if hasattr(model, "target_ids"):
                    pred = model.target_ids(pred)
                prefix, prop = ids[:, :1], []
                for _ in range(labels.numel()):
                    with _autocast(device):
                        sl = model(prefix, seed_h, k, v, cos[:prefix.shape[1]], sin[:prefix.shape[1]],
                                   visible_fraction=actual, prompt_tokens=s.prompt_tokens)
                    t = sl[0, -1].argmax()
                    if hasattr(model, "target_ids"):
                        t = model.target_ids(t)
                    prop.append(int(t))
                    prefix = torch.cat((prefix, torch.tensor([[prop[-1]]], device=prefix.device)), dim=1)
                rows.append({"request_index": s.request_index, "source_group": s.source_group, "offset": off,
                             "tokens": labels.numel(), "correct": int((pred == labels).sum()),
                             "accepted": accepted_prefix_length(prop, labels.tolist())})
        groups = defaultdict(list)
        for r in rows:
            groups[str(r["source_group"])].append(r)
        results.append({"memory_mode": memory_mode, "requested_fraction": frac, "overall": summarize_windows(rows),
                        "by_source_group": {g: summarize_windows(rr) for g, rr in sorted(groups.items())}})
    return results


def save_checkpoint(model: SparseKVDrafter, path: Path, *, target_model: str, target_fingerprint: str,
                    completed_steps: int, training_args: dict | None = None) -> None:
    """``sparsecache.sparse-kv-drafter.v1``: config + state dict (no target weights)."""
    ckpt = {"format": CHECKPOINT_FORMAT, "config": model.config.to_dict(), "state_dict": model.state_dict(),
            "target_model": target_model, "target_fingerprint": target_fingerprint,
            "completed_steps": completed_steps, "training_args": training_args or {}}
    tmp = Path(path).with_suffix(".tmp")
    torch.save(ckpt, tmp)
    tmp.replace(path)


def load_checkpoint(path: Path, *, target_fingerprint: str | None = None) -> tuple[SparseKVDrafter, dict]:
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    if ckpt.get("format") != CHECKPOINT_FORMAT:
        raise ValueError("unsupported drafter checkpoint")
    if target_fingerprint is not None and ckpt["target_fingerprint"] != target_fingerprint:
        raise ValueError("target fingerprints differ")
    model = SparseKVDrafter(SparseKVDraftConfig.from_dict(ckpt["config"]))
    model.load_state_dict(ckpt["state_dict"])
    return model, ckpt


def write_history(path: Path, rows: Sequence[dict]) -> None:
    with open(path, "w") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")
