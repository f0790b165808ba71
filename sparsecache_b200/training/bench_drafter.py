"""Sparse-KV EAGLE drafter training throughput and draft acceptance.

    python -m sparsecache_b200.training.bench_drafter --steps 10 --warmup 3
    torchrun --nproc-per-node N -m sparsecache_b200.training.bench_drafter ...

Workload: the drafter is one Llama-3.1-8B-width EAGLE layer (d 4096, 32/8
heads, FFN 14336, draft vocabulary 32000 over a 128256-token target) fed the
concatenated hidden states of 3 target layers; each sequence attends to a
2048-token sparse view (64 sink + 512 recent + top 64-token chunks) of a
16k-token context's K/V at 3 target layers; 256 teacher-forced continuation
tokens per sequence; AdamW with fp32 master weights over the trainable
adapter; global batch 32 sequences split over the ranks.  Weights are random
(no checkpoint is available offline) and the teacher bank is synthetic of
that geometry (``--teacher extract`` derives it from the random-init 8B
target with this package's engine instead, for a smaller sample count).

Timing: W warm-up steps (they include the CUDA-graph capture), then K steps
bracketed by a barrier and a device synchronize, CUDA events on the training
stream, max over ranks.  Each step's batch indices are copied from pinned
host memory; the bank itself (inputs larger than L2) is resident in HBM.
Prints one JSON line on rank 0: training tokens/s (global batch x horizon
per step), ms per step, and the accepted prefix of 4-token greedy drafts on
held-out sequences (exact / disabled memory).
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--samples", type=int, default=600)
    p.add_argument("--eval-samples", type=int, default=64)
    p.add_argument("--horizon", type=int, default=256)
    p.add_argument("--prompt-tokens", type=int, default=16384)
    p.add_argument("--visible", type=int, default=2048)
    p.add_argument("--global-batch", type=int, default=32)
    p.add_argument("--teacher", choices=("synthetic", "extract"), default="synthetic")
    p.add_argument("--fusion-mode", choices=("scalar", "gated_delta"), default="scalar")
    p.add_argument("--train-fc", action="store_true")
    p.add_argument("--train-midlayer", action="store_true")
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--tc-linears", action="store_true",
                   help="frozen trunk projections on this package's tensor-core GEMMs instead of autograd's linears")
    p.add_argument("--no-k14", action="store_true", help="trunk self-attention on SDPA instead of the K14 kernels")
    p.add_argument("--no-defer", action="store_true",
                   help="adapter weight gradients through autograd (per position) instead of one GEMM per weight")
    p.add_argument("--nccl-control", action="store_true",
                   help="data parallel: ncclAllReduce of the gradient after the backward (the control arm)")
    p.add_argument("--no-overlap", action="store_true",
                   help="data parallel: one reduce-scatter after the backward instead of per-bucket overlap")
    p.add_argument("--small", action="store_true", help="tiny geometry (smoke runs)")
    args = p.parse_args(argv)

    import torch.distributed as dist

    from ..config import get_model_config
    from ..models.sparse_kv_eagle import SparseKVEagleConfig
    from ..rope import rope_cos_sin
    from .drafter_trainer import (DrafterTrainConfig, EagleDrafterTrainer, configure_trainable_modules,
                                  evaluate_drafter, prepare_for_training, random_eagle_drafter)
    from .teacher import synthetic_bank

    if args.no_k14:
        from ..ops import linear as _linear

        _linear.USE_RECURRENT_ATTENTION_KERNEL = False

    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    distributed = world > 1
    if distributed:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    rank = dist.get_rank() if distributed else 0
    try:
        target = get_model_config("llama3-8b")
        if args.small:
            ecfg = SparseKVEagleConfig(target_hidden_size=512, hidden_size=512, intermediate_size=1024,
                                       num_attention_heads=4, num_key_value_heads=2, num_memory_heads=8,
                                       target_vocab_size=4096, draft_vocab_size=1024)
        else:
            ecfg = SparseKVEagleConfig(fusion_mode=args.fusion_mode)
        model = random_eagle_drafter(ecfg, seed=0)
        model.freeze_eagle()
        configure_trainable_modules(model, train_fc=args.train_fc, train_midlayer=args.train_midlayer,
                                    adapter_scale_init=0.0)
        prepare_for_training(model, dev)
        g = torch.Generator(device=dev).manual_seed(7)
        emb = torch.empty(ecfg.target_vocab_size, ecfg.target_hidden_size, device=dev, dtype=torch.bfloat16)
        model.bind_target_embedding(emb.normal_(0.0, 0.02, generator=g))
        n_total = args.samples + args.eval_samples
        if args.teacher == "synthetic":
            bank = synthetic_bank(n_samples=n_total, horizon=args.horizon, n_layers=ecfg.num_memory_layers,
                                  n_heads=ecfg.num_memory_heads, n_seed=ecfg.num_seed_layers,
                                  target_hidden=ecfg.target_hidden_size, hidden=ecfg.hidden_size,
                                  vocab=ecfg.draft_vocab_size, visible=args.visible,
                                  prompt_tokens=args.prompt_tokens, topk=64, device=dev, seed=1)
        else:
            bank = _extracted_bank(target, n_total, args, dev)
        cos, sin = rope_cos_sin(target, torch.arange(args.prompt_tokens + args.horizon + 8), device=dev)
        train_bank_rows = args.samples
        tcfg = DrafterTrainConfig(global_batch=args.global_batch, use_graph=not args.no_graph,
                                  tc_linears=args.tc_linears, defer_weight_grads=not args.no_defer,
                                  overlap_exchange=not args.no_overlap, nccl_exchange=args.nccl_control)
        trainer = EagleDrafterTrainer(model, _head(bank, train_bank_rows), cos, sin, tcfg, distributed=distributed)
        trainer.warmup_and_capture(warmup=max(1, args.warmup))
        if distributed:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(True), torch.cuda.Event(True)
        t0.record()
        for _ in range(args.steps):
            trainer.train_step()
        t1.record()
        torch.cuda.synchronize(dev)
        ms = t0.elapsed_time(t1) / args.steps
        if distributed:
            if not trainer.nccl:
                trainer.opt.check()
            mt = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(mt, op=dist.ReduceOp.MAX)
            ms = float(mt.item())
        row = trainer.log_row()
        evals = {}
        if rank == 0 and args.eval_samples > 0:
            rows = list(range(args.samples, n_total))
            for mode in ("exact", "disabled"):
                evals[mode] = evaluate_drafter(model, bank, rows, cos, sin, memory_mode=mode, draft_tokens=4,
                                               batch=32)
        # the optimizer phase on its own (eager, after the evaluation): with several ranks it is
        # the peer-memory reduce-scatter + clip + AdamW + all-gather, which runs after the
        # backward (every adapter weight is shared by all 256 positions of the recurrence),
        # so its time is the exposed exchange of a step
        if distributed:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(3):
            if trainer.nccl:
                dist.all_reduce(trainer.flat.grad, op=dist.ReduceOp.AVG)
            elif distributed:
                trainer.opt.begin_step()
            trainer.opt.step()
        e1.record()
        torch.cuda.synchronize(dev)
        opt_ms = e0.elapsed_time(e1) / 3
        # the backward's tail as captured CUDA graphs (launch costs as inside the step): the deferred
        # weight-gradient GEMMs alone, then the GEMMs followed by each exchange variant; the difference
        # is the exchange time the step cannot hide
        parts = {}
        if trainer.stash is not None:
            tail = _tail_graph_ms(trainer, dev, distributed)
            parts.update({f"tail_{k}_ms": v for k, v in tail.items()})
            for k, v in tail.items():
                if k != "dw_gemms":
                    parts[f"exposed_{k}_ms"] = v - tail["dw_gemms"]
        if distributed:
            if not trainer.nccl:
                trainer.opt.check()
            keys = sorted(parts)
            mt = torch.tensor([opt_ms] + [parts[k] for k in keys], device=dev, dtype=torch.float64)
            dist.all_reduce(mt, op=dist.ReduceOp.MAX)
            opt_ms = float(mt[0].item())
            parts = {k: float(v) for k, v in zip(keys, mt[1:].tolist())}
        tokens = args.global_batch * trainer.horizon
        trainable = sum(p.numel() for p in model.adapter_parameters())
        if rank == 0:
            print(json.dumps({
                "metric": "drafter_training_tokens_per_s", "value": tokens / (ms / 1e3), "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "dtype": "bf16 (fp32 master)",
                "data": f"{args.teacher} teacher bank, random-init weights",
                "config": {"model": "EAGLE-3 layer, Llama-3.1-8B width", "global_batch": args.global_batch,
                           "horizon": trainer.horizon, "prompt_tokens": args.prompt_tokens,
                           "visible_tokens": args.visible, "samples": args.samples,
                           "trainable_params": trainable, "fusion_mode": ecfg.fusion_mode,
                           "parallelism": f"dp{world}", "graph": not args.no_graph,
                           "trunk_linears": "tcgen05 GEMM" if trainer.tc_linears else "autograd (library)",
                           "trunk_self_attention": "SDPA (library)" if args.no_k14 else "K14 kernels",
                           "inputs": "bank resident in HBM (larger than L2)"},
                "final_loss": row["loss"], "grad_norm": row["grad_norm"],
                "optimizer_exchange_ms": opt_ms,
                "optimizer_exchange": ("ncclAllReduce of the whole gradient + clip + AdamW on every rank, timed "
                                       "alone" if trainer.nccl else
                                       "peer-memory reduce-scatter + clip + AdamW + all-gather of the whole "
                                       "buffer, timed alone" if distributed else "fused clip + AdamW"),
                "weight_grads": "deferred: one GEMM per adapter weight" if trainer.stash is not None
                                else "autograd, per position",
                "exchange_overlap": bool(distributed and getattr(trainer.opt, "buckets", None)),
                **parts,
                "acceptance_4tok": {k: v["mean_accepted_prefix"] for k, v in evals.items()},
                "teacher_forced_top1": {k: v["teacher_forced_top1"] for k, v in evals.items()},
                "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 1e9,
            }), flush=True)
        trainer.release()
    finally:
        if distributed:
            dist.barrier()
            dist.destroy_process_group()


def _tail_graph_ms(trainer, dev, distributed: bool, reps: int = 10) -> dict[str, float]:
    """Per-replay device time of the backward's tail variants, each captured once as a CUDA graph.

    Every variant runs the same kernels on every rank in the same order (the
    exchanges wait on each other across ranks); each replay also applies one
    optimizer update, harmless after the timed steps.
    """
    import torch.distributed as dist

    st, opt = trainer.stash, trainer.opt
    variants = {"dw_gemms": lambda: st.finish()}
    if trainer.nccl:
        def nccl():
            st.finish()
            dist.all_reduce(trainer.flat.grad, op=dist.ReduceOp.AVG)
            opt.step()
        variants["nccl_allreduce"] = nccl
    elif distributed:
        def serial():
            opt.begin_step()
            st.finish()
            opt.step()
        variants["peer_serial"] = serial
        if getattr(opt, "buckets", None):
            def overlap():
                opt.begin_step()
                opt.bucket_ready(0)
                st.finish(on_weight=lambda k: opt.bucket_ready(1 + k))
                opt.step_reduced()
            variants["peer_overlap"] = overlap
    out = {}
    for name, fn in variants.items():
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()  # eager once: workspaces and communicators exist before the capture
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        if distributed:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        out[name] = e0.elapsed_time(e1) / reps
        del g
    return out


def _head(bank, n):
    """The first ``n`` sequences of a bank (the rest are held out for evaluation)."""
    from dataclasses import replace

    fields = ("mem_k", "mem_v", "idx", "n_vis", "seed_hidden", "input_ids", "labels", "topk_ids", "topk_logprobs",
              "prompt_tokens", "visible_fraction")
    kw = {f: getattr(bank, f)[:n] for f in fields}
    kw["teacher_hidden"] = None if bank.teacher_hidden is None else bank.teacher_hidden[:n]
    kw["groups"] = bank.groups[:n]
    return replace(bank, **kw)


def _extracted_bank(target_cfg, n, args, dev):
    """Teacher bank from the random-init 8B target (engine prefill + graph decode)."""
    from ..models.engine import B200Engine
    from .teacher import bank_from_extracted, extract_teacher

    engine = B200Engine.random(target_cfg, seed=0, device=dev,
                               max_positions=args.prompt_tokens + args.horizon + 256)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(1000, 120000, (args.prompt_tokens,), generator=g, dtype=torch.int32) for _ in range(n)]
    slot = engine.new_slot(args.prompt_tokens + args.horizon + 128)
    samples = extract_teacher(engine, prompts, kv_layers=(8, 16, 24), seed_layers=(2, 16, 29),
                              continuation_tokens=args.horizon, teacher_topk=64, view_budget=args.visible,
                              slot=slot)
    for i, s in enumerate(samples):
        s.source_group = i % 8
    del engine
    torch.cuda.empty_cache()
    return bank_from_extracted(samples, dev)


if __name__ == "__main__":
    main()
