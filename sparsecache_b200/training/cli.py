"""Command-line drafter trainers over the teacher-data formats.

    python -m sparsecache_b200.training.cli train-eagle --teacher-manifest T/manifest.json \\
        --output-dir runs/eagle --steps 2000 --global-batch 32
    python -m sparsecache_b200.training.cli train-drafter --teacher-manifest T/manifest.json \\
        --output-dir runs/drafter --steps 2000

Counterparts of the reference's experiments/train_sparse_kv_eagle.py (flags
:384-436) and experiments/train_sparse_kv_drafter.py (flags :536-572) with the
same flag names where the behaviour is the same.  Train / evaluation split:
explicit ``--train-indices`` / ``--eval-indices`` (``0-99,120``), else every
index with ``i % eval_modulus == eval_remainder`` is held out.

``train-eagle``: the EAGLE-3 trunk (from ``--eagle-checkpoint`` or random
init) frozen, the sparse target-KV adapter trained by
``EagleDrafterTrainer`` (batched recurrence, fused LM-head losses, fused
AdamW, CUDA graph on a GPU), ``--save-every`` adapter snapshots,
``--resume-adapter`` restores adapter weights with a fresh optimizer and counts
the steps as additional steps; the held-out rows are evaluated with memory
exact and disabled (4-token draft acceptance, teacher-forced top-1).

``train-drafter``: ``SparseKVDrafter`` trained by ``train_sparse_drafter``
over visibility fractions, then the five-cell ablation on held-out samples.
The target's embedding / LM head come from ``--target-embedding`` (a tensor
file) or the seeded random-init weights of ``--target-model``.
"""
from __future__ import annotations

import argparse
import json
from dataclasses import replace
from pathlib import Path

import torch


def parse_indices(text: str | None) -> set[int] | None:
    """``"0-3,7"`` -> {0, 1, 2, 3, 7}; empty / None -> None."""
    if not text:
        return None
    out: set[int] = set()
    for part in text.split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            a, b = (int(x) for x in part.split("-"))
            if b < a:
                raise ValueError(f"bad index range {part!r}")
            out.update(range(a, b + 1))
        else:
            out.add(int(part))
    return out


def split_indices(available, *, train: str | None, evaluate: str | None, eval_modulus: int,
                  eval_remainder: int) -> tuple[list[int], list[int]]:
    avail = sorted(available)
    tr, ev = parse_indices(train), parse_indices(evaluate)
    if tr is None and ev is None:
        if eval_modulus <= 0:
            return avail, []
        ev = {i for i in avail if i % eval_modulus == eval_remainder}
    if ev is None:
        ev = set(avail) - tr
    if tr is None:
        tr = set(avail) - ev
    missing = (tr | ev) - set(avail)
    if missing:
        raise ValueError(f"indices not in the teacher data: {sorted(missing)[:8]}")
    if tr & ev:
        raise ValueError("train and evaluation indices overlap")
    return sorted(tr), sorted(ev)


def _target_tensors(a, vocab: int, hidden: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """(embedding, lm_head) of the target model, [vocab, hidden] bf16."""
    if a.target_embedding:
        t = torch.load(a.target_embedding, map_location="cpu")
        emb = t["embed"] if isinstance(t, dict) else t
        head = t.get("lm_head", emb) if isinstance(t, dict) else emb
    else:  # the seeded random-init target the teacher data was extracted from
        from ..config import get_model_config
        from ..models.engine import EngineWeights

        full = EngineWeights.random(get_model_config(a.target_model), seed=a.target_seed, device=device)
        emb, head = full.embed, full.lm_head
        del full
    if tuple(emb.shape) != (vocab, hidden):
        raise ValueError(f"target embedding {tuple(emb.shape)} does not match ({vocab}, {hidden})")
    return emb.to(device=device, dtype=torch.bfloat16), head.to(device=device, dtype=torch.bfloat16)


def _rope(a, head_dim: int, max_pos: int, device):
    from ..config import get_model_config
    from ..rope import rope_cos_sin

    cfg = replace(get_model_config(a.target_model), head_dim=head_dim)
    return rope_cos_sin(cfg, torch.arange(max_pos), device=device)


def cmd_train_eagle(a) -> dict:
    from ..models.sparse_kv_eagle import SparseKVEagleConfig, SparseKVEagleDrafter
    from .drafter_trainer import (DrafterTrainConfig, EagleDrafterTrainer, configure_trainable_modules,
                                  evaluate_drafter, prepare_for_training, random_eagle_drafter, write_json)
    from .teacher import bank_from_samples, load_teacher_dataset

    dev = torch.device(a.device)
    manifest, samples = load_teacher_dataset(a.teacher_manifest)
    train_ids, eval_ids = split_indices(samples, train=a.train_indices, evaluate=a.eval_indices,
                                        eval_modulus=a.eval_modulus, eval_remainder=a.eval_remainder)
    if not train_ids:
        raise ValueError("no training samples")
    ecfg = (SparseKVEagleConfig.from_dict(json.loads(Path(a.drafter_config).read_text()))
            if a.drafter_config else SparseKVEagleConfig(fusion_mode=a.fusion_mode))
    torch.manual_seed(a.seed)
    if a.eagle_checkpoint:
        model = SparseKVEagleDrafter(ecfg)
        model.load_eagle_checkpoint(a.eagle_checkpoint)
    else:  # random-init trunk with the identity draft<->target vocabulary maps
        model = random_eagle_drafter(ecfg, seed=a.seed)
    model.freeze_eagle()
    configure_trainable_modules(model, train_fc=a.train_fc, train_midlayer=a.train_midlayer,
                                adapter_scale_init=a.adapter_scale_init)
    emb, _ = _target_tensors(a, ecfg.target_vocab_size, ecfg.target_hidden_size, dev)
    if dev.type == "cuda":  # bf16 trunk + fp32 adapter under autocast
        prepare_for_training(model, dev)
    else:  # no autocast on the CPU: everything in fp32
        model.to(dev)
        emb = emb.float()
    model.bind_target_embedding(emb)
    train = [samples[i] for i in train_ids]
    bank = bank_from_samples(train, dev)
    max_pos = max(s.prompt_tokens + s.horizon for s in samples.values()) + 8
    cos, sin = _rope(a, ecfg.head_dim, max_pos, dev)
    tcfg = DrafterTrainConfig(lr=a.learning_rate, weight_decay=a.weight_decay, grad_clip=a.gradient_clip,
                              prefix_decay=a.prefix_decay, hard_weight=a.hard_weight, soft_weight=a.soft_weight,
                              contrast_weight=a.contrast_weight, contrast_margin=a.contrast_margin,
                              base_contrast_weight=a.base_contrast_weight, feature_weight=a.feature_weight,
                              global_batch=min(a.global_batch, len(train)),
                              window_tokens=a.training_window_tokens, use_graph=dev.type == "cuda", seed=a.seed)
    trainer = EagleDrafterTrainer(model, bank, cos, sin, tcfg)
    out = Path(a.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    resumed = 0
    if a.resume_adapter:  # adapter weights only; a fresh optimizer, steps counted on top
        resumed = int(trainer.resume(a.resume_adapter, restore_optimizer=False).get("completed_steps", 0))
    history = []
    target_steps = resumed + a.steps
    trainer.warmup_and_capture(warmup=min(1, a.steps))
    while trainer.steps_done < target_steps:
        trainer.train_step()
        if a.log_every and trainer.steps_done % a.log_every == 0:
            history.append(trainer.log_row())
            print(json.dumps({"event": "train", **history[-1]}), flush=True)
        if a.save_every and trainer.steps_done % a.save_every == 0:
            trainer.save(out / f"adapter_step{trainer.steps_done:06d}.pt", training_args=vars(a))
    trainer.save(out / "adapter.pt", training_args=vars(a))
    trainer.release()
    evals = {}
    if eval_ids:
        ebank = bank_from_samples([samples[i] for i in eval_ids], dev)
        rows = list(range(len(eval_ids)))
        for mode in ("exact", "disabled"):
            evals[mode] = evaluate_drafter(model, ebank, rows, cos, sin, memory_mode=mode, draft_tokens=4,
                                           batch=min(32, len(rows)))
    summary = {"format": manifest.get("format"), "train_samples": len(train_ids), "eval_samples": len(eval_ids),
               "completed_steps": trainer.steps_done, "resumed_from_step": resumed, "history": history,
               "evaluation": evals}
    write_json(out / "summary.json", summary)
    return summary


def cmd_train_drafter(a) -> dict:
    from ..models.sparse_kv_draft import SparseKVDraftConfig, SparseKVDrafter
    from . import sparse_drafter
    from .teacher import load_teacher_dataset

    dev = torch.device(a.device)
    manifest, samples = load_teacher_dataset(a.teacher_manifest)
    train_ids, eval_ids = split_indices(samples, train=a.train_indices, evaluate=a.eval_indices,
                                        eval_modulus=a.eval_modulus, eval_remainder=a.eval_remainder)
    s0 = samples[train_ids[0]].tensors
    L, Hm, _, D = s0["memory_keys"].shape
    n_seed, HT = s0["seed_hidden"].shape
    if a.draft_hidden_size % D:
        raise ValueError(f"--draft-hidden-size must be a multiple of the head dim {D}")
    cfg = SparseKVDraftConfig(target_hidden_size=HT, draft_hidden_size=a.draft_hidden_size, head_dim=D,
                              num_draft_heads=a.draft_hidden_size // D, num_memory_heads=Hm,
                              num_memory_layers=L, num_seed_layers=n_seed, num_blocks=a.num_blocks,
                              mlp_ratio=a.mlp_ratio)
    torch.manual_seed(a.seed)
    model = SparseKVDrafter(cfg).to(dev)
    vocab = int(manifest.get("vocab_size", 0)) or int(max(int(s.tensors["labels"].max()) for s in samples.values())) + 1
    emb, head = _target_tensors(a, vocab, HT, dev)
    model.bind_target_weights(emb.float() if dev.type == "cpu" else emb, head.float() if dev.type == "cpu" else head)
    fractions = tuple(float(x) for x in a.visibility_fractions.split(","))
    hist = sparse_drafter.train_sparse_drafter(
        model, [samples[i] for i in train_ids], fractions=fractions, steps=a.steps, device=dev,
        log_every=a.log_every, lr=a.learning_rate, window_tokens=a.training_window_tokens or None)
    out = Path(a.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    sparse_drafter.save_checkpoint(model, out / "checkpoint.pt", target_model=a.target_model,
                                   target_fingerprint=manifest.get("target_fingerprint", ""),
                                   completed_steps=a.steps)
    sparse_drafter.write_history(out / "history.jsonl", hist)
    ablation = {}
    if eval_ids:
        ablation = sparse_drafter.five_cell_ablation(model, [samples[i] for i in eval_ids], fractions, device=dev,
                                                     max_proposal_tokens=a.max_eval_tokens)
    summary = {"train_samples": len(train_ids), "eval_samples": len(eval_ids), "steps": a.steps,
               "history": hist, "ablation": ablation}
    (out / "summary.json").write_text(json.dumps(summary, indent=2, default=float) + "\n")
    return summary


def _common(p: argparse.ArgumentParser) -> None:
    p.add_argument("--teacher-manifest", required=True)
    p.add_argument("--output-dir", required=True)
    p.add_argument("--train-indices", default=None)
    p.add_argument("--eval-indices", default=None)
    p.add_argument("--eval-modulus", type=int, default=10)
    p.add_argument("--eval-remainder", type=int, default=0)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--learning-rate", type=float, default=1e-4)
    p.add_argument("--weight-decay", type=float, default=0.01)
    p.add_argument("--prefix-decay", type=float, default=0.9)
    p.add_argument("--hard-weight", type=float, default=1.0)
    p.add_argument("--soft-weight", type=float, default=0.5)
    p.add_argument("--feature-weight", type=float, default=0.0)
    p.add_argument("--gradient-clip", type=float, default=1.0)
    p.add_argument("--training-window-tokens", type=int, default=0)
    p.add_argument("--max-eval-tokens", type=int, default=8)
    p.add_argument("--log-every", type=int, default=50)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", default="cuda")
    p.add_argument("--target-model", default="llama3-8b", help="random-init target preset (embedding, RoPE)")
    p.add_argument("--target-seed", type=int, default=0)
    p.add_argument("--target-embedding", default=None, help="tensor file: embedding or {embed, lm_head}")


def main(argv=None) -> dict:
    p = argparse.ArgumentParser()
    sub = p.add_subparsers(dest="cmd", required=True)
    e = sub.add_parser("train-eagle")
    _common(e)
    e.add_argument("--eagle-checkpoint", default=None)
    e.add_argument("--drafter-config", default=None, help="SparseKVEagleConfig JSON (default: 8B width)")
    e.add_argument("--contrast-weight", type=float, default=0.5)
    e.add_argument("--contrast-margin", type=float, default=0.25)
    e.add_argument("--base-contrast-weight", type=float, default=0.25)
    e.add_argument("--train-fc", action="store_true")
    e.add_argument("--train-midlayer", action="store_true")
    e.add_argument("--fusion-mode", choices=("scalar", "gated_delta"), default="scalar")
    e.add_argument("--adapter-scale-init", type=float, default=-4.0)
    e.add_argument("--resume-adapter", default=None)
    e.add_argument("--save-every", type=int, default=0)
    e.add_argument("--global-batch", type=int, default=32)
    d = sub.add_parser("train-drafter")
    _common(d)
    d.add_argument("--visibility-fractions", default="0.05,0.1,0.2")
    d.add_argument("--draft-hidden-size", type=int, default=512)
    d.add_argument("--num-blocks", type=int, default=1)
    d.add_argument("--mlp-ratio", type=int, default=4)
    a = p.parse_args(argv)
    return cmd_train_eagle(a) if a.cmd == "train-eagle" else cmd_train_drafter(a)


if __name__ == "__main__":
    main()
