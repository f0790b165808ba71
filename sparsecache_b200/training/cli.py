"""Command-line drafter trainers over the teacher-data formats.

    python -m sparsecache_b200.training.cli train-eagle --teacher-manifest T/manifest.json \\
        --output-dir runs/eagle --steps 2000 --global-batch 32
    python -m sparsecache_b200.training.cli train-drafter --teacher-manifest T/manifest.json \\
        --output-dir runs/drafter --steps 2000
    python -m sparsecache_b200.training.cli extract-teacher --model M --requests-jsonl C/requests.jsonl \\
        --output-dir T --request-indices 0-255 --continuation-tokens 8
    python -m sparsecache_b200.training.cli extend-teacher --base-manifest T/manifest.json \\
        --output-dir T5 --continuation-tokens 64
    python -m sparsecache_b200.training.cli eval-drafter --checkpoint runs/drafter/checkpoint.pt \\
        --teacher-manifest T/manifest.json --output runs/drafter/eval.json
    python -m sparsecache_b200.training.cli eval-boundaries --checkpoint runs/drafter/checkpoint.pt \\
        --teacher-manifest T5/manifest.json --output runs/drafter/boundaries.json

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

``extract-teacher`` (reference: experiments/extract_sparse_kv_teacher.py,
flags :326-341, manifest :393-431): the v3 teacher records of the chosen
rows of a corpus ``requests.jsonl`` from a model directory (``config.json``
+ ``model.safetensors``), one ``sample_XXXXX.safetensors`` per request and a
manifest that records the corpus hash, the model fingerprint, each prompt's
hash and its seed token.  ``extend-teacher`` (reference:
experiments/extend_sparse_kv_teacher.py:138-260): a longer greedy
continuation per request with the seed-layer hidden state after every token,
written as ``trace_XXXXX.safetensors`` + a v5 manifest chained to the v3
base; it refuses a changed corpus, a changed model, a changed prompt or a
seed token that does not reproduce.  On a CUDA device the B200 engine does
the extraction (prefill hooks, CUDA-graph greedy decode); on the CPU the
plain-PyTorch oracle model does.
"""
from __future__ import annotations

import argparse
import json
import time
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


def parse_layer_list(raw: str, *, name: str) -> tuple[int, ...]:
    """``"8,20,31"`` -> (8, 20, 31); empty, negative or duplicate entries are rejected."""
    values = tuple(int(x) for x in raw.split(",") if x.strip())
    if not values or min(values) < 0 or len(set(values)) != len(values):
        raise ValueError(f"{name} must be distinct non-negative integers")
    return values


def load_request_rows(path: Path, indices, max_context_tokens: int) -> list[dict]:
    """Rows ``indices`` of a corpus ``requests.jsonl`` (prompt token ids), sorted by index."""
    wanted = set(int(i) for i in indices)
    rows = []
    with Path(path).open(encoding="utf-8") as f:
        for index, line in enumerate(f):
            if index not in wanted:
                continue
            row = json.loads(line)
            prompt = row.get("prompt")
            if not isinstance(prompt, list) or not prompt or any(type(t) is not int for t in prompt):
                raise ValueError(f"request {index} has invalid prompt token ids")
            if len(prompt) > max_context_tokens:
                raise ValueError(f"request {index} has {len(prompt)} prompt tokens, above the "
                                 f"{max_context_tokens}-token cap")
            rows.append({"request_index": index, "prompt": prompt, "source_dataset": row.get("source_dataset"),
                         "source_index": row.get("source_index")})
    missing = wanted - {r["request_index"] for r in rows}
    if missing:
        raise ValueError(f"missing request indices: {sorted(missing)}")
    return sorted(rows, key=lambda r: r["request_index"])


class _TeacherModel:
    """The target of a model directory: the B200 engine on a CUDA device, the fp32 oracle on the CPU."""

    def __init__(self, model_dir: str, device: torch.device, max_positions: int) -> None:
        from ..models.checkpoint import load_oracle

        self.device = device
        if device.type == "cuda":
            from ..models.engine import B200Engine

            oracle = load_oracle(model_dir, dtype=torch.bfloat16, device="cpu")
            self.engine, self.oracle = B200Engine.from_oracle(oracle, device=device,
                                                              max_positions=max_positions), None
            del oracle
        else:
            self.engine, self.oracle = None, load_oracle(model_dir, dtype=torch.float32, device="cpu")
        self.config = self.engine.cfg if self.engine is not None else self.oracle.config

    def extract(self, prompt: list[int], **kw) -> dict[str, torch.Tensor]:
        from .teacher import extract_teacher, extract_teacher_oracle

        ids = torch.tensor(prompt, dtype=torch.int32)
        if self.engine is not None:
            return extract_teacher(self.engine, [ids], keep_full_memory=True, **kw)[0].tensors
        return extract_teacher_oracle(self.oracle, [ids], **kw)[0].tensors


def _eos_ids(model_dir: str, config) -> set[int]:
    """End-of-sequence ids: the model config's, else a Hugging Face ``eos_token_id`` entry."""
    if config.eos_token_ids:
        return {int(x) for x in config.eos_token_ids}
    raw = json.loads((Path(model_dir) / "config.json").read_text()).get("eos_token_id")
    if raw is None:
        return set()
    return {int(raw)} if isinstance(raw, int) else {int(x) for x in raw}


def _save_record(tensors: dict[str, torch.Tensor], path: Path) -> tuple[str, int]:
    from .teacher import _atomic_save, sha256_file

    _atomic_save(tensors, path)
    return sha256_file(path), sum(t.numel() * t.element_size() for t in tensors.values())


def cmd_extract_teacher(a) -> dict:
    from ..store import model_fingerprint
    from .teacher import TEACHER_FORMATS, prompt_sha256, required_fields, sha256_file, truncate_at_eos

    indices = sorted(parse_indices(a.request_indices) or ())
    kv_layers = parse_layer_list(a.kv_layers, name="KV layers")
    seed_layers = parse_layer_list(a.seed_layers, name="seed layers")
    if min(a.max_context_tokens, a.continuation_tokens, a.teacher_topk, a.priority_page_size) <= 0:
        raise ValueError("context, continuation and top-k sizes must be positive")
    requests = Path(a.requests_jsonl)
    rows = load_request_rows(requests, indices, a.max_context_tokens)
    out = Path(a.output_dir)
    out.mkdir(parents=True, exist_ok=False)
    dev = torch.device(a.device)
    target = _TeacherModel(a.model, dev, a.max_context_tokens + a.continuation_tokens + 128)
    cfg = target.config
    if max(kv_layers + seed_layers) >= cfg.n_layers:
        raise ValueError("a requested target layer is out of range")
    eos = _eos_ids(a.model, cfg)
    v3 = required_fields(3)
    sample_rows = []
    for row in rows:
        t0 = time.perf_counter()
        tensors = truncate_at_eos(target.extract(row["prompt"], kv_layers=kv_layers, seed_layers=seed_layers,
                                                 continuation_tokens=a.continuation_tokens,
                                                 teacher_topk=a.teacher_topk, page_size=a.priority_page_size),
                                  eos)
        i = row["request_index"]
        f = out / f"sample_{i:05d}.safetensors"
        digest, nbytes = _save_record({k: tensors[k] for k in v3}, f)
        sample = {"request_index": i, "file": f.name, "prompt_tokens": len(row["prompt"]),
                  "draft_training_tokens": int(tensors["labels"].numel()),
                  "seed_token_id": int(tensors["input_ids"][0]), "prompt_sha256": prompt_sha256(row["prompt"]),
                  "logical_bytes": nbytes, "file_sha256": digest,
                  "elapsed_ms": (time.perf_counter() - t0) * 1000.0,
                  "source_dataset": row["source_dataset"], "source_index": row["source_index"]}
        sample_rows.append(sample)
        print(json.dumps({"event": "teacher_sample", **sample}), flush=True)
    manifest = {"schema_version": 3, "format": TEACHER_FORMATS[2], "created_at_ns": time.time_ns(),
                "target_model": str(Path(a.model).resolve()), "target_fingerprint": model_fingerprint(a.model),
                "requests_jsonl": str(requests.resolve()), "requests_sha256": sha256_file(requests),
                "request_indices": indices, "max_context_tokens": a.max_context_tokens,
                "continuation_tokens": a.continuation_tokens, "teacher_topk": a.teacher_topk,
                "priority_page_size": a.priority_page_size, "kv_layers": list(kv_layers),
                "seed_layers": list(seed_layers), "dtype": "bfloat16", "head_dim": cfg.head_dim,
                "kv_heads": cfg.n_kv_heads, "target_hidden_size": cfg.d_model, "vocab_size": cfg.vocab,
                "samples": sample_rows, "extractor": "sparsecache_b200.training.cli extract-teacher",
                "extractor_backend": "b200-engine" if target.engine is not None else "oracle-cpu"}
    (out / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    print(json.dumps({"event": "teacher_manifest", "samples": len(sample_rows)}), flush=True)
    return manifest


_BASE_KEYS = ("target_model", "target_fingerprint", "requests_jsonl", "requests_sha256", "max_context_tokens",
              "priority_page_size", "kv_layers", "seed_layers", "dtype", "head_dim", "kv_heads",
              "target_hidden_size", "vocab_size")


def cmd_extend_teacher(a) -> dict:
    from ..store import model_fingerprint
    from .teacher import TEACHER_FORMATS, _TRACE_FIELDS, prompt_sha256, sha256_file, truncate_at_eos

    if min(a.continuation_tokens, a.teacher_topk) <= 0:
        raise ValueError("continuation length and teacher top-k must be positive")
    base_path = Path(a.base_manifest).resolve()
    base = json.loads(base_path.read_text(encoding="utf-8"))
    if base.get("format") != TEACHER_FORMATS[2]:
        raise ValueError("trace extension requires a v3 base teacher manifest")
    base_rows = {int(r["request_index"]): r for r in base["samples"]}
    indices = sorted(parse_indices(a.request_indices) or base_rows)
    missing = set(indices) - set(base_rows)
    if missing:
        raise ValueError(f"base teacher data is missing {sorted(missing)}")
    requests = Path(base["requests_jsonl"])
    if sha256_file(requests) != base["requests_sha256"]:
        raise ValueError("request corpus hash differs from the base manifest")
    rows = load_request_rows(requests, indices, int(base["max_context_tokens"]))
    model_dir = str(base["target_model"])
    if model_fingerprint(model_dir) != base["target_fingerprint"]:
        raise ValueError("target model fingerprint differs from the base manifest")
    out = Path(a.output_dir)
    out.mkdir(parents=True, exist_ok=False)
    dev = torch.device(a.device)
    target = _TeacherModel(model_dir, dev, int(base["max_context_tokens"]) + a.continuation_tokens + 128)
    eos = _eos_ids(model_dir, target.config)
    sample_rows = []
    for row in rows:
        t0 = time.perf_counter()
        i = row["request_index"]
        brow = base_rows[i]
        if prompt_sha256(row["prompt"]) != brow["prompt_sha256"]:
            raise ValueError(f"request {i} prompt hash differs")
        tensors = truncate_at_eos(target.extract(row["prompt"], kv_layers=tuple(base["kv_layers"]),
                                                 seed_layers=tuple(base["seed_layers"]),
                                                 continuation_tokens=a.continuation_tokens,
                                                 teacher_topk=a.teacher_topk,
                                                 page_size=int(base["priority_page_size"])), eos)
        if int(tensors["input_ids"][0]) != int(brow["seed_token_id"]):
            raise ValueError(f"request {i} seed token is not reproducible")
        f = out / f"trace_{i:05d}.safetensors"
        digest, nbytes = _save_record({k: tensors[k] for k in _TRACE_FIELDS}, f)
        sample = {"request_index": i, "file": f.name, "file_sha256": digest,
                  "draft_training_tokens": int(tensors["labels"].numel()), "seed_token_id": int(brow["seed_token_id"]),
                  "prompt_tokens": len(row["prompt"]), "prompt_sha256": brow["prompt_sha256"],
                  "logical_bytes": nbytes, "elapsed_ms": (time.perf_counter() - t0) * 1000.0,
                  "source_dataset": brow.get("source_dataset"), "source_index": brow.get("source_index")}
        sample_rows.append(sample)
        print(json.dumps({"event": "teacher_trace", **sample}), flush=True)
    manifest = {k: base[k] for k in _BASE_KEYS}
    manifest.update({"schema_version": 5, "format": TEACHER_FORMATS[4], "created_at_ns": time.time_ns(),
                     "base_manifest": str(base_path), "request_indices": indices,
                     "continuation_tokens": a.continuation_tokens, "teacher_topk": a.teacher_topk,
                     "samples": sample_rows, "extractor": "sparsecache_b200.training.cli extend-teacher"})
    (out / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    print(json.dumps({"event": "teacher_trace_manifest", "samples": len(sample_rows),
                      "tokens": sum(r["draft_training_tokens"] for r in sample_rows)}), flush=True)
    return manifest


def _eval_setup(a):
    """(manifest, samples, held-out ids, drafter with the target embedding / LM head bound, device)."""
    from . import sparse_drafter
    from .teacher import load_teacher_dataset

    dev = torch.device(a.device)
    manifest, samples = load_teacher_dataset(a.teacher_manifest)
    _, eval_ids = split_indices(samples, train=None, evaluate=a.eval_indices, eval_modulus=a.eval_modulus,
                                eval_remainder=a.eval_remainder)
    if not eval_ids:
        raise ValueError("no evaluation samples")
    model, _ = sparse_drafter.load_checkpoint(a.checkpoint, target_fingerprint=manifest.get("target_fingerprint"))
    cfg = model.config
    vocab = int(manifest.get("vocab_size", 0)) or int(max(int(s.tensors["labels"].max()) for s in samples.values())) + 1
    emb, head = _target_tensors(a, vocab, cfg.target_hidden_size, dev)
    model.to(dev)
    model.bind_target_weights(emb.float() if dev.type == "cpu" else emb, head.float() if dev.type == "cpu" else head)
    return manifest, samples, eval_ids, model, dev


def cmd_eval_drafter(a) -> dict:
    """Five-cell ablation (memory x seed) of a drafter checkpoint on held-out samples.

    Reference: experiments/eval_sparse_kv_drafter.py:45-171.
    """
    from . import sparse_drafter

    manifest, samples, eval_ids, model, dev = _eval_setup(a)
    fractions = tuple(float(x) for x in a.visibility_fractions.split(","))
    cells = sparse_drafter.five_cell_ablation(model, [samples[i] for i in eval_ids], fractions, device=dev,
                                              page_size=a.page_size, selection_seed=a.selection_seed,
                                              selection_mode=a.selection_mode, max_proposal_tokens=a.max_eval_tokens)
    out = {"checkpoint": str(a.checkpoint), "teacher_format": manifest.get("format"), "eval_indices": eval_ids,
           "visibility_fractions": list(fractions), "selection_mode": a.selection_mode, "cells": cells}
    Path(a.output).parent.mkdir(parents=True, exist_ok=True)
    Path(a.output).write_text(json.dumps(out, indent=2, default=float) + "\n")
    return out


def cmd_eval_boundaries(a) -> dict:
    """Drafts that start after a verification boundary (v5 teacher data), by source group, for exact /
    zero / shuffled memory.  Reference: experiments/eval_sparse_kv_boundaries.py:30-178."""
    from . import sparse_drafter

    manifest, samples, eval_ids, model, dev = _eval_setup(a)
    if not str(manifest.get("format", "")).endswith(".v5"):
        raise ValueError("boundary evaluation needs v5 teacher data (continuation_seed_hidden)")
    fractions = tuple(float(x) for x in a.visibility_fractions.split(","))
    held = [samples[i] for i in eval_ids]
    modes = {m: sparse_drafter.evaluate_boundaries(model, held, fractions, device=dev, page_size=a.page_size,
                                                   selection_seed=a.selection_seed, selection_mode=a.selection_mode,
                                                   memory_mode=m, window_tokens=a.window_tokens,
                                                   maximum_windows_per_sample=a.max_windows_per_sample)
             for m in ("exact", "zero", "shuffled")}
    out = {"checkpoint": str(a.checkpoint), "eval_indices": eval_ids, "visibility_fractions": list(fractions),
           "window_tokens": a.window_tokens, "memory_modes": modes}
    Path(a.output).parent.mkdir(parents=True, exist_ok=True)
    Path(a.output).write_text(json.dumps(out, indent=2, default=float) + "\n")
    return out


def _eval_common(p: argparse.ArgumentParser, fractions: str) -> None:
    p.add_argument("--checkpoint", required=True)
    p.add_argument("--teacher-manifest", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--eval-indices", default=None)
    p.add_argument("--eval-modulus", type=int, default=5)
    p.add_argument("--eval-remainder", type=int, default=0)
    p.add_argument("--visibility-fractions", default=fractions)
    p.add_argument("--page-size", type=int, default=64)
    p.add_argument("--selection-mode", choices=("random", "priority", "strided"), default="priority")
    p.add_argument("--selection-seed", type=int, default=20960827)
    p.add_argument("--device", default="cuda")
    p.add_argument("--target-model", default="llama3-8b", help="random-init target preset (embedding, LM head)")
    p.add_argument("--target-seed", type=int, default=0)
    p.add_argument("--target-embedding", default=None, help="tensor file: embedding or {embed, lm_head}")


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
    x = sub.add_parser("extract-teacher")
    x.add_argument("--model", required=True, help="model directory (config.json + model.safetensors)")
    x.add_argument("--requests-jsonl", required=True)
    x.add_argument("--output-dir", required=True)
    x.add_argument("--request-indices", default="0,1,5,8")
    x.add_argument("--max-context-tokens", type=int, default=16384)
    x.add_argument("--continuation-tokens", type=int, default=8)
    x.add_argument("--kv-layers", default="8,20,31")
    x.add_argument("--seed-layers", default="2,16,29")
    x.add_argument("--teacher-topk", type=int, default=64)
    x.add_argument("--priority-page-size", type=int, default=64)
    x.add_argument("--device", default="cuda")
    t = sub.add_parser("extend-teacher")
    t.add_argument("--base-manifest", required=True)
    t.add_argument("--output-dir", required=True)
    t.add_argument("--request-indices", default=None)
    t.add_argument("--continuation-tokens", type=int, default=64)
    t.add_argument("--teacher-topk", type=int, default=64)
    t.add_argument("--device", default="cuda")
    ed = sub.add_parser("eval-drafter")
    _eval_common(ed, "0.05,0.10,0.20,1.0")
    ed.add_argument("--max-eval-tokens", type=int, default=8)
    eb = sub.add_parser("eval-boundaries")
    _eval_common(eb, "0.05,0.10,0.20")
    eb.add_argument("--window-tokens", type=int, default=8)
    eb.add_argument("--max-windows-per-sample", type=int, default=8)
    a = p.parse_args(argv)
    return {"train-eagle": cmd_train_eagle, "train-drafter": cmd_train_drafter,
            "extract-teacher": cmd_extract_teacher, "extend-teacher": cmd_extend_teacher,
            "eval-drafter": cmd_eval_drafter, "eval-boundaries": cmd_eval_boundaries}[a.cmd](a)


if __name__ == "__main__":
    main()
