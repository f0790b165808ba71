"""Tensor-parallel prefill/decode timing: fused peer-memory collectives vs NCCL.

    torchrun --nproc-per-node N -m sparsecache_b200.parallel.tp_bench --model llama3-8b --tokens 8192

Every rank generates its own weight shard (seeded per tensor and rank; no
full-model materialisation), so the 70B geometry fits at TP8.  Reported, as
the max over ranks of CUDA-event device time:
  * prefill_ms (fused, whole model) and decode tpot_ms (fused, CUDA graph);
  * per-op at the prompt length: the fused AG->QKV GEMM vs NCCL all-gather +
    the same GEMM, and the fused o_proj GEMM->RS (+ owner reduce) vs the same
    GEMM + NCCL reduce-scatter; each with its roofline, the slower of
    FLOPs / measured bf16 peak and NVLink bytes / 770 GB/s.
"""
from __future__ import annotations

import argparse
import json
import os
import zlib
from datetime import timedelta

import torch
import torch.distributed as dist

from ..config import get_model_config
from ..models.engine import EngineWeights, LayerWeights
from .tp import FLAG_RS_O, FLAG_STAGE_X, FLAG_X, TIMEOUT_NS, TPEngine, TPGroup, local_config

BF16_TFLOPS = 1676.9
NVLINK_GBS = 770.0


def stable_seed(*parts) -> int:
    """Seed from a tuple, identical in every process (``hash`` of a str is salted per process)."""
    return zlib.crc32(repr(parts).encode()) & 0x7FFFFFFF


def random_shard(cfg, rank: int, tp: int, seed: int, device) -> EngineWeights:
    """Seeded random weight shard of ``rank`` (the full model is the concatenation)."""
    lc = local_config(cfg, tp)
    bf = torch.bfloat16
    gen = torch.Generator(device=device)

    def mat(rows, cols, tag):
        gen.manual_seed(stable_seed(seed, tag, rank))
        w = torch.empty(rows, cols, device=device, dtype=bf)
        return w.normal_(0.0, 0.02, generator=gen)

    def rep(rows, cols, tag):  # replicated tensors: same on every rank
        gen.manual_seed(stable_seed(seed, tag))
        w = torch.empty(rows, cols, device=device, dtype=bf)
        return w.normal_(0.0, 0.02, generator=gen)

    d = cfg.d_model
    ones = torch.ones(d, device=device, dtype=bf)
    layers = [LayerWeights(ln1=ones, w_qkv=mat(lc.qkv_rows, d, ("qkv", i)), w_o=mat(d, lc.q_size, ("o", i)),
                           ln2=ones, w_gu=mat(2 * lc.ffn, d, ("gu", i)), w_down=mat(d, lc.ffn, ("down", i)))
              for i in range(cfg.n_layers)]
    return EngineWeights(embed=rep(cfg.vocab, d, "embed"), layers=layers, norm=ones,
                         lm_head=rep(cfg.vocab, d, "lm_head"))


def device_time(fn, iters: int, warmup: int = 2) -> float:
    for _ in range(warmup):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--tokens", type=int, default=8192)
    p.add_argument("--new-tokens", type=int, default=32)
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--breakdown", action="store_true", help="per-op decode step breakdown (eager, CUDA events)")
    p.add_argument("--decode-only", action="store_true", help="skip the per-op prefill comparisons")
    args = p.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    try:
        cfg = get_model_config(args.model)
        if args.layers:
            cfg = cfg.with_layers(args.layers)
        group = TPGroup()
        tp, rank = group.size, group.rank
        w = random_shard(cfg, rank, tp, 0, dev)
        T = args.tokens
        tpe = TPEngine(cfg, w, group, max_rows=(T + tp * 128) // tp, max_positions=T + args.new_tokens + 1024)
        lc, eng, ext = tpe.lcfg, tpe.engine, tpe.ext
        g = torch.Generator().manual_seed(1)
        ids = torch.randint(0, 128000 if cfg.vocab > 128000 else cfg.vocab, (T,), generator=g).to(torch.int32).to(dev)
        slot = tpe.new_slot(T + tp * 128 + args.new_tokens + 64)
        out = {"model": cfg.name, "layers": cfg.n_layers, "tp": tp, "tokens": T}

        # ---- whole-model fused prefill + decode ----
        def prefill():
            tpe.prefill(ids, slot)

        out["prefill_ms"] = device_time(prefill, max(1, args.iters // 2))
        tpe.check_status()
        x, rows, Tp = tpe.prefill(ids, slot)
        tpe.first_token(x, rows, T, max_new=args.new_tokens)
        tpe.decode(slot, 2)  # capture + warm
        out["tpot_ms"] = device_time(lambda: tpe.decode(slot, 1), 16)
        tpe.check_status()
        if args.breakdown:  # eager step with events around every op, max over ranks
            bd = tpe.decode_breakdown(slot)
            t = torch.tensor([bd[k] for k in sorted(bd)], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out["decode_breakdown_ms"] = dict(zip(sorted(bd), t.tolist()))
            tpe.check_status()

        if args.decode_only:
            dist.barrier()
            eng.release_graphs()
            if rank == 0:
                print(json.dumps(out), flush=True)
            dist.barrier()
            tpe.close()
            return
        # ---- per-op: AG -> QKV GEMM ----
        d = cfg.d_model
        lw = eng.w.layers[0]
        pos = eng._arange("bench_pos", Tp)
        q = torch.empty(Tp, lc.q_size, device=dev, dtype=torch.bfloat16)
        xs = tpe.x_buf.view(torch.bfloat16)[: rows * d].view(rows, d)
        xs.normal_()

        def fused_ag():
            tpe.epoch += 1
            tpe._signal_all(FLAG_X, tpe.epoch)
            bases = tpe._pull_shards(FLAG_X, FLAG_STAGE_X, tpe.x_ptrs, tpe.stage_x, rows, tpe.epoch)
            ext.gemm_ag_qkv(bases, rows, rank, tpe.flags[FLAG_STAGE_X], tpe.epoch, d, lw.w_qkv, q, slot.k(0),
                            slot.v(0), pos, pos, eng.rope, lc.n_heads, lc.n_kv_heads, eng.bn)

        x_full = torch.empty(Tp, d, device=dev, dtype=torch.bfloat16)

        def nccl_ag():
            dist.all_gather_into_tensor(x_full, xs)
            ext.gemm_qkv(x_full, lw.w_qkv, q, slot.k(0), slot.v(0), pos, pos, eng.rope, lc.n_heads, lc.n_kv_heads,
                         None, 0, eng.bn)

        flops = 2.0 * Tp * lc.qkv_rows * d
        nvl = (tp - 1) / tp * Tp * d * 2
        roof_ms = max(flops / (BF16_TFLOPS * 1e12), nvl / (NVLINK_GBS * 1e9)) * 1e3
        t_f, t_n = device_time(fused_ag, args.iters), device_time(nccl_ag, args.iters)
        out["ag_qkv"] = {"fused_ms": t_f, "nccl_ms": t_n, "roofline_ms": roof_ms, "fused_frac_of_roofline": roof_ms / t_f,
                         "nccl_frac_of_roofline": roof_ms / t_n, "speedup": t_n / t_f}

        # ---- per-op: o_proj GEMM -> RS (+ owner reduce with residual) ----
        attn = torch.randn(Tp, lc.q_size, device=dev).to(torch.bfloat16)
        h = torch.randn(rows, d, device=dev).to(torch.bfloat16)
        recv = tpe.recv_o_buf.view(torch.bfloat16)[: tp * rows * d].view(tp, rows, d)
        x2 = tpe.x2_buf.view(torch.bfloat16)[: rows * d].view(rows, d)

        def fused_rs():
            tpe.epoch += 1
            ext.gemm_rs(attn, lw.w_o, tpe.recv_o_ptrs, rows, rank, eng.bn)
            tpe._signal_all(FLAG_RS_O, tpe.epoch)
            ext.rs_reduce(recv, tpe.flags[FLAG_RS_O], tpe.epoch, TIMEOUT_NS, tpe.status, h, h, lw.ln2, x2,
                          cfg.rms_eps)

        partial = torch.empty(Tp, d, device=dev, dtype=torch.bfloat16)
        shard = torch.empty(rows, d, device=dev, dtype=torch.bfloat16)

        def nccl_rs():
            ext.gemm_store(attn, lw.w_o, partial, eng.bn)
            dist.reduce_scatter_tensor(shard, partial)
            h.add_(shard)
            ext.rmsnorm(h, None, lw.ln2, cfg.rms_eps, x2)

        flops = 2.0 * Tp * d * lc.q_size
        nvl = (tp - 1) / tp * Tp * d * 2  # bf16 partials cross NVLink
        roof_ms = max(flops / (BF16_TFLOPS * 1e12), nvl / (NVLINK_GBS * 1e9)) * 1e3
        t_f, t_n = device_time(fused_rs, args.iters), device_time(nccl_rs, args.iters)
        out["gemm_rs_o"] = {"fused_ms": t_f, "nccl_ms": t_n, "roofline_ms": roof_ms,
                            "fused_frac_of_roofline": roof_ms / t_f, "nccl_frac_of_roofline": roof_ms / t_n,
                            "speedup": t_n / t_f, "partials": "bf16 (both)"}
        tpe.check_status()
        dist.barrier()
        eng.release_graphs()
        if rank == 0:
            print(json.dumps(out), flush=True)
        dist.barrier()
        tpe.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
