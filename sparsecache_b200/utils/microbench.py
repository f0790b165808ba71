"""Isolated timings of the sm_100a kernels at Llama-3.1-8B shapes.

    python -m sparsecache_b200.utils.microbench [--only gemm,gemv,gemm_f32,attn_decode,attn_prefill,mem_attn,adamw]

CUDA events on the launching stream, 10 warm-up launches, mean over N timed
launches; every case uses tensors that are re-read each launch, so the
bandwidth figures of the GEMV / decode-attention rows are HBM figures when
the operand exceeds L2 (126 MB) and L2-assisted otherwise (noted per row).
Fractions are against the measured copy bandwidth and cuBLAS bf16 burst rate
of this machine class (``_measured_peaks``).
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from ..models.engine import ATTN_CNT_PER_KVH, ATTN_WS_PER_KVH


def _measured_peaks() -> tuple[float, float]:
    """Copy bandwidth (GB/s) and cuBLAS bf16 burst rate (TFLOP/s) measured on
    this machine class (MEASURED_PEAKS.json at the repository root when it is
    there; otherwise an earlier measurement of the same B200 pool)."""
    import os

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 6558.7, 1661.6


HBM_GBS, BF16_TFLOPS = _measured_peaks()


def timeit(fn, n: int = 50, warm: int = 10) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    for _ in range(n):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n * 1000.0  # us


def main() -> None:
    from .. import ops

    p = argparse.ArgumentParser()
    p.add_argument("--only", default="gemm,gemm_small,gemv,attn_decode,attn_prefill,mem_attn,adamw")
    args = p.parse_args()
    only = set(args.only.split(","))
    ext = ops.ext()
    dev = torch.device("cuda:0")
    res: dict[str, dict] = {}
    bf = torch.bfloat16

    if "gemv_rows" in only:
        # batched-verify rows at 70B widths (one GPU): weight bytes per launch / time
        for name, N, K in (("qkv", 10240, 8192), ("down", 8192, 28672), ("gate_up", 57344, 8192)):
            w = (torch.randn(N, K, device=dev) * 0.02).to(bf)
            for M in (1, 2, 5, 8):
                x = torch.randn(M, K, device=dev).to(bf)
                if name == "gate_up":
                    o = torch.empty(M, N // 2, device=dev, dtype=bf)
                    fn = lambda: ext.gemv_swiglu(x, w, None, 1e-5, o)  # noqa: E731
                else:
                    o = torch.empty(M, N, device=dev, dtype=bf)
                    fn = lambda: ext.gemv_residual(x, w, None, 1e-5, o, o)  # noqa: E731
                t = timeit(fn, n=20, warm=5)
                gbs = N * K * 2 / (t * 1e-6) / 1e9
                res[f"gemv_rows_{name}_M{M}"] = {"us": t, "GBps": gbs, "frac_of_measured_hbm": gbs / HBM_GBS}
            del w

    if "skinny" in only:
        # tensor-core skinny GEMM vs the CUDA-core GEMV at batched-verify row counts (70B widths)
        for name, N, K in (("qkv", 10240, 8192), ("down", 8192, 28672), ("gate_up", 57344, 8192)):
            w = (torch.randn(N, K, device=dev) * 0.02).to(bf)
            splits = int(ext.skinny_splits(N, K))
            ws = torch.empty(splits * N * 16, device=dev)
            for M in (1, 2, 5, 8, 16):
                x = torch.randn(M, K, device=dev).to(bf)
                epi = 2 if name == "gate_up" else 1
                o = torch.empty(M, N // 2 if epi == 2 else N, device=dev, dtype=bf)
                t = timeit(lambda: ext.skinny_gemm(x, w, epi, o, o if epi == 1 else None, ws), n=20, warm=5)
                gbs = N * K * 2 / (t * 1e-6) / 1e9
                res[f"skinny_{name}_M{M}"] = {"us": t, "GBps": gbs, "frac_of_measured_hbm": gbs / HBM_GBS,
                                               "splits": splits}
            del w

    if "gemm_f32" in only:
        # drafter weight gradients: dW [out, in] = dY^T X over 64 rows x 256 positions (fp32 result)
        R = 64 * 256
        for name, M, N in (("query_dw", 1024, 4096), ("output_dw", 4096, 1024)):
            a = (torch.randn(M, R, device=dev) * 0.02).to(bf)
            w = (torch.randn(N, R, device=dev) * 0.02).to(bf)
            out = torch.empty(M, N, device=dev)
            t = timeit(lambda: ext.gemm_f32(a, w, out), n=20)
            tf = 2.0 * M * N * R / (t * 1e-6) / 1e12
            res[f"gemm_f32_{name}"] = {"us": t, "TFLOPs": tf, "frac_of_measured_bf16": tf / BF16_TFLOPS}
            del a, w, out

    if "gemv" in only:
        for name, N, K in (("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 28672, 4096),
                           ("down", 4096, 14336), ("lm_head", 128256, 4096)):
            w = (torch.randn(N, K, device=dev) * 0.02).to(bf)
            x = torch.randn(1, K, device=dev).to(bf)
            o = torch.empty(1, N, device=dev, dtype=bf)
            t = timeit(lambda: ext.gemv_store(x, w, None, 1e-5, o))
            gbs = N * K * 2 / (t * 1e-6) / 1e9
            res[f"gemv_{name}"] = {"us": t, "GBps": gbs, "frac_of_measured_hbm": gbs / HBM_GBS}
            del w

    if "gemm" in only:
        K = 4096
        for M in (300, 1700, 8192):
            for name, N in (("qkv", 6144), ("gate_up", 28672)):
                a = torch.randn(M, K, device=dev).to(bf)
                w = (torch.randn(N, K, device=dev) * 0.02).to(bf)
                o = torch.empty(M, N, device=dev, dtype=bf)
                t = timeit(lambda: ext.gemm_store(a, w, o, 256), n=20)
                tf = 2 * M * N * K / (t * 1e-6) / 1e12
                res[f"gemm_M{M}_{name}"] = {"us": t, "TFLOPs": tf, "frac_of_measured_bf16": tf / BF16_TFLOPS,
                                            "weight_GBps": N * K * 2 / (t * 1e-6) / 1e9}

    if "gemm_small" in only or "gemm_down_splitk" in only or "gemm_gate_up" in only or "gemm_gate_up_big" in only:
        # CacheBlend active rows (~15% of a 1.7k-token prompt): the layer's four
        # projections as the engine issues them (128-wide QKV tiles, split-K o/down);
        # gemm_gate_up_big: the SwiGLU projection of a full 2048-row prefill
        M = 2048 if "gemm_gate_up_big" in only else 300
        cases = (("qkv_bn128", 6144, 4096, "store", 128), ("o_splitk", 4096, 4096, "residual", 256),
                 ("gate_up", 28672, 4096, "swiglu", 256), ("down_splitk", 4096, 14336, "residual", 256))
        if "gemm_small" not in only:
            cases = cases[3:] if "gemm_down_splitk" in only else cases[2:3]
        for name, N, K, kind, bn in cases:
            a = torch.randn(M, K, device=dev).to(bf)
            w = (torch.randn(N, K, device=dev) * 0.02).to(bf)
            o = torch.empty(M, N // 2 if kind == "swiglu" else N, device=dev, dtype=bf)
            if kind == "store":
                fn = lambda: ext.gemm_store(a, w, o, bn, -1)  # noqa: E731
            elif kind == "residual":
                fn = lambda: ext.gemm_residual(a, w, o, o, bn, -1)  # noqa: E731
            else:
                fn = lambda: ext.gemm_swiglu(a, w, o, bn)  # noqa: E731
            t = timeit(fn, n=20)
            tf = 2 * M * N * K / (t * 1e-6) / 1e12
            res[f"gemm_M{M}_{name}"] = {"us": t, "TFLOPs": tf, "frac_of_measured_bf16": tf / BF16_TFLOPS,
                                        "weight_GBps": N * K * 2 / (t * 1e-6) / 1e9,
                                        "weight_frac_of_measured_hbm": N * K * 2 / (t * 1e-6) / 1e9 / HBM_GBS}

    if "gemm_shapes" in only:
        # 128-row tiles (one accumulator) vs 256-row tiles (two accumulators sharing B)
        # vs the automatic choice, for the CacheBlend active-row and full-prefill shapes
        for M in (300, 1676):
            for name, N, K, kind in (("qkv", 6144, 4096, "store"), ("o", 4096, 4096, "residual"),
                                     ("gate_up", 28672, 4096, "swiglu"), ("down", 4096, 14336, "residual")):
                a = torch.randn(M, K, device=dev).to(bf)
                w = (torch.randn(N, K, device=dev) * 0.02).to(bf)
                o = torch.empty(M, N // 2 if kind == "swiglu" else N, device=dev, dtype=bf)
                for rows, bn in ((128, 128), (128, 256), (256, 256), (0, 256)):
                    ext.set_gemm_rows_per_tile(rows)
                    if kind == "store":
                        fn = lambda: ext.gemm_store(a, w, o, bn, -1)  # noqa: E731
                    elif kind == "residual":
                        fn = lambda: ext.gemm_residual(a, w, o, o, bn, -1)  # noqa: E731
                    else:
                        fn = lambda: ext.gemm_swiglu(a, w, o, bn)  # noqa: E731
                    t = timeit(fn, n=20)
                    tf = 2 * M * N * K / (t * 1e-6) / 1e12
                    res[f"gemm_M{M}_{name}_rows{rows or 'auto'}_bn{bn}"] = {
                        "us": t, "TFLOPs": tf, "frac_of_measured_bf16": tf / BF16_TFLOPS}
                ext.set_gemm_rows_per_tile(0)
                del a, w, o

    if "gemm_wide_gu" in only:
        # one shape for a profiler capture: the SwiGLU gate/up projection of the 8B layer at 330 rows
        M, N, K = 330, 28672, 4096
        w = (torch.randn(N, K, device=dev) * 0.02).to(bf)
        a = torch.randn(M, K, device=dev).to(bf)
        o = torch.empty(M, N // 2, device=dev, dtype=bf)
        for sk in (True, False):
            ext.set_wide_stream_k(sk)
            t = timeit(lambda: ext.wide_swiglu(a, w, o), n=5, warm=3)
            tf = 2 * M * N * K / (t * 1e-6) / 1e12
            res[f"gemm_M330_gate_up_tokencol_streamk{int(sk)}"] = {
                "us": t, "TFLOPs": tf, "frac_of_measured_bf16": tf / BF16_TFLOPS, "plan": ext.wide_plan(M, N, K, 1)}
        ext.set_wide_stream_k(True)
        del w, a, o

    if "gemm_wide" in only:
        # token-column GEMM (weights as the MMA's M, tokens as its N) against the row-tile GEMM at
        # CacheBlend's active-row counts; weights cycled over copies so every call streams them
        # from HBM (as in a layer loop), inputs of the real shapes
        for M in (300, 330, 512):
            for name, N, K, kind in (("qkv", 6144, 4096, "qkv"), ("o", 4096, 4096, "residual"),
                                     ("gate_up", 28672, 4096, "swiglu"), ("down", 4096, 14336, "residual")):
                copies = max(1, -(-(256 << 20) // (N * K * 2)))
                ws_ = [(torch.randn(N, K, device=dev) * 0.02).to(bf) for _ in range(copies)]
                a = torch.randn(M, K, device=dev).to(bf)
                o = torch.empty(M, N // 2 if kind == "swiglu" else N, device=dev, dtype=bf)
                cap, nq, nkv = 2048, 32, 8
                qo = torch.empty(M, nq * 128, device=dev, dtype=bf)
                kc = torch.zeros(nkv, cap, 128, device=dev, dtype=bf)
                vc = torch.zeros(nkv, cap, 128, device=dev, dtype=bf)
                pos = torch.arange(M, device=dev, dtype=torch.int32) * 5
                table = torch.zeros(4096, 128, device=dev)
                it = [0]

                def nxt():
                    it[0] = (it[0] + 1) % copies
                    return ws_[it[0]]

                if kind == "qkv":
                    tc = lambda: ext.gemm_qkv(a, nxt(), qo, kc, vc, pos, pos, table, nq, nkv, None, 0,  # noqa: E731
                                              128 if -(-M // 128) * (N // 256) < ext.num_sms() else 256, 0, 0)
                    wd = lambda: ext.wide_qkv(a, nxt(), qo, kc, vc, pos, pos, table, nq, nkv)  # noqa: E731
                elif kind == "residual":
                    tc = lambda: ext.gemm_residual(a, nxt(), o, o, 256, -1)  # noqa: E731
                    wd = lambda: ext.wide_residual(a, nxt(), o, o)  # noqa: E731
                else:
                    tc = lambda: ext.gemm_swiglu(a, nxt(), o, 256)  # noqa: E731
                    wd = lambda: ext.wide_swiglu(a, nxt(), o)  # noqa: E731
                for arm, fn in (("rowtile", tc), ("tokencol", wd)):
                    t = timeit(fn, n=20)
                    tf = 2 * M * N * K / (t * 1e-6) / 1e12
                    res[f"gemm_M{M}_{name}_{arm}"] = {"us": t, "TFLOPs": tf, "frac_of_measured_bf16": tf / BF16_TFLOPS}
                res[f"gemm_M{M}_{name}_tokencol"]["plan"] = ext.wide_plan(M, N, K, 1 if kind == "swiglu" else 0)
                del ws_, a, o

    if "attn_decode" in only or "attn_decode_sweep" in only:
        H, Hkv = 32, 8
        for cap in (2048, 18000):
            kc = torch.randn(Hkv, cap, 128, device=dev).to(bf)
            vc = torch.randn(Hkv, cap, 128, device=dev).to(bf)
            q = torch.randn(1, H * 128, device=dev).to(bf)
            pos = torch.tensor([cap - 16], device=dev, dtype=torch.int32)
            out = torch.empty(1, H * 128, device=dev, dtype=bf)
            S = int(ext.attention_decode_cluster(cap, Hkv))
            if "attn_decode_sweep" in only:  # cluster-size sweep
                for s_try in (4, 8, 16):
                    t_s = timeit(lambda: ext.attention_decode(q, kc, vc, pos, H, 1 / math.sqrt(128), s_try, out))
                    res[f"attn_decode_ctx{cap}_S{s_try}"] = {"us": t_s}
            ws = torch.zeros(Hkv * ATTN_WS_PER_KVH, device=dev)
            cnt = torch.zeros(Hkv * ATTN_CNT_PER_KVH, device=dev, dtype=torch.int32)
            R = int(ext.attention_decode_outer(cap, Hkv, S, ext.num_sms()))
            t = timeit(lambda: ext.attention_decode(q, kc, vc, pos, H, 1 / math.sqrt(128), S, out, ws=ws,
                                                    counters=cnt))
            kv_bytes = 2 * Hkv * (cap - 15) * 128 * 2
            gbs = kv_bytes / (t * 1e-6) / 1e9
            res[f"attn_decode_ctx{cap}"] = {"us": t, "GBps": gbs, "frac_of_measured_hbm": gbs / HBM_GBS,
                                            "cluster": S, "clusters_per_kv_head": R,
                                            "l2_resident": kv_bytes < 126e6}

    if "attn_decode_serving" in only:
        # the 8B serving shape: 32 layer caches of one slot (cycled, so K/V come
        # from HBM as in a decode step) at the bench capacity, keys = a typical
        # and a long prompt; cluster size x clusters per kv head
        H, Hkv, cap, layers = 32, 8, 2768, 32
        kcs = [torch.randn(Hkv, cap, 128, device=dev).to(bf) for _ in range(layers)]
        vcs = [torch.randn(Hkv, cap, 128, device=dev).to(bf) for _ in range(layers)]
        q = torch.randn(1, H * 128, device=dev).to(bf)
        out = torch.empty(1, H * 128, device=dev, dtype=bf)
        ws = torch.zeros(Hkv * ATTN_WS_PER_KVH, device=dev)
        cnt = torch.zeros(Hkv * ATTN_CNT_PER_KVH, device=dev, dtype=torch.int32)
        auto = (int(ext.attention_decode_cluster(cap, Hkv)),
                int(ext.attention_decode_outer(cap, Hkv, int(ext.attention_decode_cluster(cap, Hkv)), ext.num_sms())))
        for n_keys in (1676, 2600):
            pos = torch.tensor([n_keys - 1], device=dev, dtype=torch.int32)
            for S in (4, 8, 16):
                for R in (1, 2, 3, 4, 6, 8):
                    def run_all():
                        for i in range(layers):
                            ext.attention_decode(q, kcs[i], vcs[i], pos, H, 1 / math.sqrt(128), S, out, ws=ws,
                                                 counters=cnt, outer=R)
                    t = timeit(run_all, n=10, warm=3) / layers
                    kv_bytes = 2 * Hkv * n_keys * 128 * 2
                    res[f"attn_decode_serving_keys{n_keys}_S{S}_R{R}"] = {
                        "us": t, "frac_of_measured_hbm": kv_bytes / (t * 1e-6) / 1e9 / HBM_GBS,
                        "automatic": (S, R) == auto}

    if "attn_decode_batch" in only:
        # batched decode attention: 32 sequences, each with its own slot (stride apart) at ~1676 keys,
        # 4 layers' caches cycled so K/V come from HBM (32 x 6.9 MB per layer); one launch per layer
        H, Hkv, cap, B, layers = 32, 8, 2768, 32, 4
        per = Hkv * cap * 128
        kbuf = [torch.randn(B * per, device=dev).to(bf) for _ in range(layers)]
        vbuf = [torch.randn(B * per, device=dev).to(bf) for _ in range(layers)]
        q = torch.randn(B, H * 128, device=dev).to(bf)
        out = torch.empty(B, H * 128, device=dev, dtype=bf)
        pos_rows = torch.full((B,), 1675, device=dev, dtype=torch.int32)
        S_auto = int(ext.attention_decode_cluster(cap, Hkv))
        kv_bytes = B * 2 * Hkv * 1676 * 128 * 2
        for S in sorted({1, 2, 4, 8, S_auto}):
            def run_layers():
                for i in range(layers):
                    ext.attention_decode(q, kbuf[i][:per].view(Hkv, cap, 128), vbuf[i][:per].view(Hkv, cap, 128),
                                         pos_rows, H, 1 / math.sqrt(128), S, out, pos_rows=pos_rows, seq_stride=per)
            t = timeit(run_layers, n=10, warm=3) / layers
            res[f"attn_decode_batch32_keys1676_S{S}"] = {
                "us": t, "frac_of_measured_hbm": kv_bytes / (t * 1e-6) / 1e9 / HBM_GBS, "cluster": S}

    if "attn_decode_grid" in only:
        # cluster size x (one / several clusters per kv head) for the decode shapes that matter
        for H, Hkv, cap in ((32, 8, 2048), (32, 8, 18000), (8, 1, 16384), (16, 4, 4096)):
            kc = torch.randn(Hkv, cap, 128, device=dev).to(bf)
            vc = torch.randn(Hkv, cap, 128, device=dev).to(bf)
            q = torch.randn(1, H * 128, device=dev).to(bf)
            pos = torch.tensor([cap - 16], device=dev, dtype=torch.int32)
            out = torch.empty(1, H * 128, device=dev, dtype=bf)
            ws = torch.zeros(Hkv * ATTN_WS_PER_KVH, device=dev)
            cnt = torch.zeros(Hkv * ATTN_CNT_PER_KVH, device=dev, dtype=torch.int32)
            for S in (4, 8, 16):
                for two in (False, True):
                    kw = {"ws": ws, "counters": cnt} if two else {}
                    R = int(ext.attention_decode_outer(cap, Hkv, S, ext.num_sms())) if two else 1
                    t = timeit(lambda: ext.attention_decode(q, kc, vc, pos, H, 1 / math.sqrt(128), S, out, **kw))
                    res[f"grid_H{H}_kv{Hkv}_ctx{cap}_S{S}_R{R}"] = {"us": t}

    if "attn_decode_tp" in only:
        # one kv head per GPU (70B at TP8), 16k context: one cluster vs several clusters per kv head
        H, Hkv, cap = 8, 1, 16384
        kc = torch.randn(Hkv, cap, 128, device=dev).to(bf)
        vc = torch.randn(Hkv, cap, 128, device=dev).to(bf)
        q = torch.randn(1, H * 128, device=dev).to(bf)
        pos = torch.tensor([cap - 16], device=dev, dtype=torch.int32)
        out = torch.empty(1, H * 128, device=dev, dtype=bf)
        ws = torch.zeros(Hkv * ATTN_WS_PER_KVH, device=dev)
        cnt = torch.zeros(Hkv * ATTN_CNT_PER_KVH, device=dev, dtype=torch.int32)
        kv_bytes = 2 * Hkv * (cap - 15) * 128 * 2
        for name, S, kw in (("one_cluster", 16, {}), ("two_level", int(ext.attention_decode_cluster(cap, Hkv)),
                                                          {"ws": ws, "counters": cnt})):
            t = timeit(lambda: ext.attention_decode(q, kc, vc, pos, H, 1 / math.sqrt(128), S, out, **kw))
            res[f"attn_decode_tp8_70b_ctx{cap}_{name}"] = {"us": t, "GBps": kv_bytes / (t * 1e-6) / 1e9}

    if "attn_prefill" in only or "attn_prefill_ab" in only or "attn_prefill_split" in only:
        # CacheBlend shapes of the 8B serving case: the full layers (every row,
        # causal) and the selective layers (300 active rows over 1676 keys);
        # the tcgen05 kernel against the mma.sync kernel it replaced
        H, Hkv, T = 32, 8, 1676
        kc = torch.randn(Hkv, T, 128, device=dev).to(bf)
        vc = torch.randn(Hkv, T, 128, device=dev).to(bf)
        q = torch.randn(T, H * 128, device=dev).to(bf)
        allpos = torch.arange(T, device=dev, dtype=torch.int32)
        sel = torch.sort(torch.randperm(T - 40, device=dev)[:260]).values.to(torch.int32)
        sel = torch.cat([sel, allpos[-40:]]).sort().values
        for name, rows in (("causal", None), ("selective300", sel)):
            R = T if rows is None else rows.numel()
            qpos = allpos if rows is None else rows
            out = torch.empty(R, H * 128, device=dev, dtype=bf)
            flops = 4 * 128 * H * float(sum(int(x) + 1 for x in qpos.tolist()))
            split_ws = torch.empty(4 * 512 * H * 132, device=dev)  # the engine's key-split workspace
            for kern in ("attention_prefill", "attention_prefill_mma"):
                fn = getattr(ext, kern)
                if kern == "attention_prefill":
                    call = lambda: fn(q, rows, qpos, kc, vc, None, T, H, 1 / math.sqrt(128), out,  # noqa: E731
                                      ws=split_ws if R <= 512 else None)
                else:
                    call = lambda: fn(q, rows, qpos, kc, vc, None, T, H, 1 / math.sqrt(128), out)  # noqa: E731
                t = timeit(call, n=20)
                tf = flops / (t * 1e-6) / 1e12
                res[f"{kern}_{name}_T{T}"] = {"us": t, "TFLOPs": tf, "frac_of_measured_bf16": tf / BF16_TFLOPS}
            if "attn_prefill_split" in only and R <= 512:
                # key split forced to 1..4 CTAs per row tile (+ the merge kernel)
                for s_try in (1, 2, 3, 4):
                    ext.set_attention_prefill_splits(s_try)
                    t = timeit(lambda: ext.attention_prefill(q, rows, qpos, kc, vc, None, T, H, 1 / math.sqrt(128), out,
                                                             ws=split_ws), n=20)
                    res[f"attention_prefill_{name}_T{T}_splits{s_try}"] = {
                        "us": t, "frac_of_measured_bf16": flops / (t * 1e-6) / 1e12 / BF16_TFLOPS}
                ext.set_attention_prefill_splits(0)
    if "attn_trace" in only:
        # timeline of one CTA (head 0, the longest row tile) of the causal case
        H, Hkv, T = 32, 8, 1676
        kc = torch.randn(Hkv, T, 128, device=dev).to(bf)
        vc = torch.randn(Hkv, T, 128, device=dev).to(bf)
        q = torch.randn(T, H * 128, device=dev).to(bf)
        pos = torch.arange(T, device=dev, dtype=torch.int32)
        out = torch.empty(T, H * 128, device=dev, dtype=bf)
        tr = torch.zeros(640, device=dev, dtype=torch.int64)
        for _ in range(3):
            ext.attention_prefill(q, None, pos, kc, vc, None, T, H, 1 / math.sqrt(128), out, trace=tr)
        torch.cuda.synchronize()
        t = tr.view(64, 10).cpu()
        t0 = int(t[63, 0])
        names = ("K_issued", "V_issued", "QK_issued", "P_ready_seen", "PV_issued", "S_ready_seen", "S_in_regs",
                 "max_exchanged", "P_written", "P_arrived")
        rows = {}
        for j in range(63):
            if int(t[j].abs().sum()) == 0:
                continue
            rows[j] = {n: (int(t[j, e]) - t0) / 1000.0 for e, n in enumerate(names) if int(t[j, e])}
        res["attn_trace_us_from_cta_start"] = {"tiles": rows, "kernel": {
            n: (int(t[63, e]) - t0) / 1000.0 for e, n in enumerate(("start", "prologue_done", "o_final_seen", "end"))}}
    if "attn_prefill" in only:
        H, Hkv = 32, 8
        for T in (2048, 16384):
            kc = torch.randn(Hkv, T, 128, device=dev).to(bf)
            vc = torch.randn(Hkv, T, 128, device=dev).to(bf)
            q = torch.randn(T, H * 128, device=dev).to(bf)
            pos = torch.arange(T, device=dev, dtype=torch.int32)
            out = torch.empty(T, H * 128, device=dev, dtype=bf)
            t = timeit(lambda: ext.attention_prefill(q, None, pos, kc, vc, None, T, H, 1 / math.sqrt(128), out), n=10)
            flops = 4 * 128 * H * T * (T + 1) / 2
            tf = flops / (t * 1e-6) / 1e12
            res[f"attn_prefill_causal_T{T}"] = {"us": t, "TFLOPs": tf, "frac_of_measured_bf16": tf / BF16_TFLOPS}

    if "mem_attn" in only:
        # drafter training step: 64 rows (32 positive + 32 contrast), 8 memory heads,
        # one memory layer of a [64 seq, 3 layers, 2048 visible, 8, 128] bank (1.6 GB > L2)
        S, L, V, H = 64, 3, 2048, 8
        mk = torch.randn(S, L, V, H, 128, device=dev).to(bf)
        mv = torch.randn(S, L, V, H, 128, device=dev).to(bf)
        q = torch.randn(1, S, H, 128, device=dev).to(bf)
        rows = torch.arange(S, device=dev, dtype=torch.int32)
        idx = torch.arange(V, device=dev, dtype=torch.int32).repeat(S, 1)
        nv = torch.full((S,), V, device=dev, dtype=torch.int32)
        out = torch.empty_like(q)
        lse = torch.empty(1, S, H, device=dev)
        dq = torch.empty(1, S, H, 128, device=dev)
        strides = (V * H * 128, L * V * H * 128, H * 128, 128)
        layer = [0]

        def fwd():
            layer[0] = (layer[0] + 1) % L
            k, v = mk[:, layer[0]:], mv[:, layer[0]:]
            ext.mem_attn_fwd(q, k, v, *strides, rows, idx, V, nv, 0, 1 / math.sqrt(128), out, lse)

        def bwd():
            layer[0] = (layer[0] + 1) % L
            k, v = mk[:, layer[0]:], mv[:, layer[0]:]
            ext.mem_attn_bwd(q, k, v, *strides, rows, idx, V, nv, 0, 1 / math.sqrt(128), out, out, lse, dq)

        kv_bytes = 2 * S * V * H * 128 * 2
        for name, fn in (("fwd", fwd), ("dq_bwd", bwd)):
            t = timeit(fn, n=30)
            gbs = kv_bytes / (t * 1e-6) / 1e9
            res[f"mem_attn_{name}_64x8x2048"] = {"us": t, "GBps": gbs, "frac_of_measured_hbm": gbs / HBM_GBS}
        del mk, mv

    if "adamw" in only:
        n = 25_169_920  # the 8B-width EAGLE adapter
        p_, g_ = torch.randn(n, device=dev), torch.randn(n, device=dev)
        m_, v_ = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
        hyper = torch.tensor([1e-4, 0.9, 0.999, 1e-8, 0.01, 1.0, 0.0, 0.0], device=dev)
        state = torch.zeros(8, device=dev)
        part = torch.zeros(296, device=dev)
        cnt = torch.zeros(1, device=dev, dtype=torch.int32)
        t = timeit(lambda: ext.adamw_step(p_, g_, m_, v_, hyper, state, part, cnt), n=30)
        byts = n * 4 * (1 + 5 + 2)  # norm pass reads g; update reads p,g,m,v and writes p,m,v
        gbs = byts / (t * 1e-6) / 1e9
        res["adamw_25M"] = {"us": t, "GBps": gbs, "frac_of_measured_hbm": gbs / HBM_GBS}
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
