// Weight-streaming small-M GEMV for decode and batched verification.
//
// At batch 1 a Llama decode step reads every weight once and does two FLOPs
// per weight, so it is bound by HBM bandwidth, not by the tensor cores.  This
// kernel streams W with 128-bit L1-bypassing loads (several in flight per
// lane), keeps the M <= 8 input rows in shared memory, and fuses the
// neighbouring pointwise work so a decode layer is five launches:
//   prologue  optional RMSNorm of x (HF LlamaRMSNorm rounding order)
//   GEMV_QKV      rows (d, d+64) of one head per warp -> RoPE in registers,
//                 Q to a buffer, K/V appended to the layer cache at *pos + m
//   GEMV_RESIDUAL out = residual + bf16(W x)          (o_proj / down_proj)
//   GEMV_SWIGLU   gate/up rows of one output per warp -> silu(g) * u
//   GEMV_ARGMAX   LM head: per-CTA (max, first index) partials, the last CTA
//                 reduces them, logs the token, loads the next embedding row
//                 and advances the device-side position (decode feedback
//                 without a host round trip; graph-replayable).
// Rows are processed in pairs; the pair layout matches the tcgen05 GEMM
// weight layout (fused QKV, gate/up interleaved in 128-row blocks).
//
// Reference behaviour: HF decode step per token (modeling.py:383-417,
// progressive_kv_feasibility.py:561-613) with argmax over bf16 logits.
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 8;
constexpr int kArMaxPairs = 32;  // pairs per CTA of the all-reduce epilogue (launcher keeps it there)

// Inner product: bf16 pairs widened into packed fp32x2 registers and
// multiplied with the sm_100 two-lane FMA (fma.rn.f32x2), which halves the
// FMA instructions per weight; each row keeps two interleaved fp32 chains
// (even / odd elements) that are added at the end.
typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 widen_bf16x2(uint32_t v) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(v << 16), "r"(v & 0xffff0000u));
  return r;
}

__device__ __forceinline__ void fma2(f32x2& acc, f32x2 a, f32x2 b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

__device__ __forceinline__ float sum2(f32x2 v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}

// Pair p -> the two weight rows it reads.
__device__ __forceinline__ void pair_rows(int epi, int p, int& r0, int& r1) {
  if (epi == GEMV_QKV) {
    const int head = p >> 6, i = p & 63;
    r0 = head * 128 + i;
    r1 = r0 + 64;
  } else if (epi == GEMV_SWIGLU) {
    const int blk = p >> 7, i = p & 127;
    r0 = blk * 256 + i;
    r1 = r0 + 128;
  } else {
    r0 = 2 * p;
    r1 = 2 * p + 1;
  }
}

__device__ __forceinline__ void load_batch(const uint4* w0, const uint4* w1, int c0, int nchunk,
                                           uint4 (&wa)[kUnroll], uint4 (&wb)[kUnroll]) {
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int c = c0 + u * 32;
    if (c < nchunk) {
      wa[u] = ld_stream_u4(w0 + c);
      wb[u] = ld_stream_u4(w1 + c);
    } else {
      wa[u] = make_uint4(0, 0, 0, 0);
      wb[u] = make_uint4(0, 0, 0, 0);
    }
  }
}

}  // namespace

// kXG: x is read from global memory (L1/L2-resident) instead of being staged
// in shared memory; used when M * K * 2 bytes exceed the shared-memory budget
// (the batched verifier's down projection at large FFN widths).  No prologue
// RMSNorm in that mode.
template <int MR, bool kXG>
__device__ __forceinline__ void gemv_body(const GemvArgs& a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem);  // [MR][K]
  __shared__ float red[kWarps][MR];
  __shared__ float s_bval[kWarps][MR];
  __shared__ int s_bidx[kWarps][MR];
  __shared__ int s_last;
  __shared__ __align__(16) float s_ar[MR][2 * kArMaxPairs];  // all-reduce chunk of this CTA

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.K;
  const int M = a.M;
  const int n_pairs = a.N / 2;
  const int nchunk = K / 8;

  // Pair schedule.  The all-reduce epilogue gives every CTA a contiguous run
  // of pairs (its outputs form one contiguous chunk, sent to the peers with
  // vector stores); the other epilogues interleave pairs over all warps.
  const bool ar = a.epi == GEMV_ALLREDUCE;
  const int ar_ppc = ar ? (((n_pairs + (int)gridDim.x - 1) / (int)gridDim.x + 1) & ~1) : 0;
  const int ar_p0 = ar ? (int)blockIdx.x * ar_ppc : 0;
  const int ar_p1 = ar ? max(ar_p0, min(ar_p0 + ar_ppc, n_pairs)) : 0;  // empty for CTAs past the end
  const int p_step = ar ? kWarps : (int)gridDim.x * kWarps;
  const int p_end = ar ? ar_p1 : n_pairs;

  // Prefetch this warp's first weight batch before waiting on the previous
  // kernel: weights never depend on it, so the prologue below overlaps HBM.
  uint4 wa[kUnroll], wb[kUnroll];
  const int first_p = ar ? ar_p0 + warp : (int)blockIdx.x * kWarps + warp;
  if (first_p < p_end) {
    int r0, r1;
    pair_rows(a.epi, first_p, r0, r1);
    load_batch(reinterpret_cast<const uint4*>(a.w + (size_t)r0 * K),
               reinterpret_cast<const uint4*>(a.w + (size_t)r1 * K), lane, nchunk, wa, wb);
  }
  pdl_wait();
  // Dependents may launch once this kernel has passed its own wait: anything
  // they read before their wait was written at least two kernels back.
  pdl_launch_dependents();

  // ---- stage x (optionally RMS-normalised) into shared memory ----
  if (kXG) {
    // x stays in global memory
  } else if (a.norm_w == nullptr) {
    for (int m = 0; m < M; ++m) {
      const uint4* src = reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx);
      uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)m * K);
      for (int c = tid; c < K / 8; c += kThreads) dst[c] = src[c];
    }
  } else {
    float ss[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) ss[m] = 0.f;
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      if (m >= M) break;
      const uint4* src = reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx);
      for (int c = tid; c < K / 8; c += kThreads) {
        const uint4 v = src[c];
        const float2 f0 = unpack_bf16x2(v.x), f1 = unpack_bf16x2(v.y), f2 = unpack_bf16x2(v.z),
                     f3 = unpack_bf16x2(v.w);
        ss[m] += f0.x * f0.x + f0.y * f0.y + f1.x * f1.x + f1.y * f1.y + f2.x * f2.x +
                 f2.y * f2.y + f3.x * f3.x + f3.y * f3.y;
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      const float v = warp_sum(ss[m]);
      if (lane == 0) red[warp][m] = v;
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      if (m >= M) break;
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) tot += red[w][m];
      const float r = rsqrtf(tot / (float)K + a.eps);
      const uint4* src = reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx);
      const uint4* wn = reinterpret_cast<const uint4*>(a.norm_w);
      uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)m * K);
      for (int c = tid; c < K / 8; c += kThreads) {
        const uint4 v = src[c], g = wn[c];
        const uint32_t vi[4] = {v.x, v.y, v.z, v.w};
        const uint32_t gi[4] = {g.x, g.y, g.z, g.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 xf = unpack_bf16x2(vi[q]), gf = unpack_bf16x2(gi[q]);
          o[q] = pack_bf16x2(gf.x * bf16_round(xf.x * r), gf.y * bf16_round(xf.y * r));
        }
        dst[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  __syncthreads();

  const uint4* xs4 = kXG ? reinterpret_cast<const uint4*>(a.x) : reinterpret_cast<const uint4*>(xs);
  const int pos0 = (a.epi == GEMV_QKV) ? *a.pos : 0;
  const int slot0 = (a.epi == GEMV_QKV) ? (a.slot != nullptr ? *a.slot : pos0) : 0;

  float best_v[MR];
  int best_i[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) best_v[m] = -INFINITY, best_i[m] = 0x7fffffff;

  bool preloaded = true;
  for (int p = first_p; p < p_end; p += p_step) {
    int r0, r1;
    pair_rows(a.epi, p, r0, r1);
    const uint4* w0 = reinterpret_cast<const uint4*>(a.w + (size_t)r0 * K);
    const uint4* w1 = reinterpret_cast<const uint4*>(a.w + (size_t)r1 * K);
    float acc0[MR], acc1[MR];
    f32x2 pacc0[MR], pacc1[MR];  // multi-row accumulators (packed even / odd chains)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc0[m] = acc1[m] = 0.f, pacc0[m] = pacc1[m] = 0ull;
    for (int c0 = lane; c0 < nchunk; c0 += 32 * kUnroll) {
      if (!preloaded) load_batch(w0, w1, c0, nchunk, wa, wb);
      preloaded = false;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32;
        if (c < nchunk) {
          {
            // widen the weight pair once and each row's x once; the same
            // arithmetic for every M keeps a row's result independent of M
            const f32x2 w0[4] = {widen_bf16x2(wa[u].x), widen_bf16x2(wa[u].y), widen_bf16x2(wa[u].z),
                                 widen_bf16x2(wa[u].w)};
            const f32x2 w1[4] = {widen_bf16x2(wb[u].x), widen_bf16x2(wb[u].y), widen_bf16x2(wb[u].z),
                                 widen_bf16x2(wb[u].w)};
#pragma unroll
            for (int m = 0; m < MR; ++m) {
              if (m < M) {
                const uint4 xv = kXG ? __ldg(xs4 + m * nchunk + c) : xs4[m * nchunk + c];
                const f32x2 xf[4] = {widen_bf16x2(xv.x), widen_bf16x2(xv.y), widen_bf16x2(xv.z),
                                     widen_bf16x2(xv.w)};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  fma2(pacc0[m], w0[i], xf[i]);
                  fma2(pacc1[m], w1[i], xf[i]);
                }
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) acc0[m] = sum2(pacc0[m]), acc1[m] = sum2(pacc1[m]);
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      acc0[m] = warp_sum(acc0[m]);
      acc1[m] = warp_sum(acc1[m]);
    }
    if (lane != 0) continue;
    // ---- epilogue (lane 0) ----
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      if (m >= M) break;
      const float v0 = acc0[m], v1 = acc1[m];
      switch (a.epi) {
        case GEMV_STORE:
          a.out[(size_t)m * a.ldo + r0] = __float2bfloat16_rn(v0);
          a.out[(size_t)m * a.ldo + r1] = __float2bfloat16_rn(v1);
          break;
        case GEMV_RESIDUAL: {
          const float q0 = __bfloat162float(a.residual[(size_t)m * a.ldr + r0]);
          const float q1 = __bfloat162float(a.residual[(size_t)m * a.ldr + r1]);
          a.out[(size_t)m * a.ldo + r0] = __float2bfloat16_rn(q0 + bf16_round(v0));
          a.out[(size_t)m * a.ldo + r1] = __float2bfloat16_rn(q1 + bf16_round(v1));
          break;
        }
        case GEMV_SWIGLU: {
          const float g = bf16_round(v0), u = bf16_round(v1);
          a.out[(size_t)m * a.ldo + p] = __float2bfloat16_rn(bf16_round(silu_f(g)) * u);
          break;
        }
        case GEMV_QKV: {
          const int head = p >> 6, i = p & 63;
          const int pos = pos0 + m;
          float o0 = v0, o1 = v1;
          const bool is_q = head < a.n_q_heads;
          const bool is_k = !is_q && head < a.n_q_heads + a.n_kv_heads;
          if (is_q || is_k) {
            const float2 cs = a.rope_table[(size_t)pos * 64 + i];
            o0 = v0 * cs.x - v1 * cs.y;
            o1 = v1 * cs.x + v0 * cs.y;
          }
          __nv_bfloat16* dst;
          if (is_q) {
            dst = a.q_out + (size_t)m * a.ldq + head * 128;
          } else {
            const int kvh = is_k ? head - a.n_q_heads : head - a.n_q_heads - a.n_kv_heads;
            dst = (is_k ? a.k_cache : a.v_cache) + ((size_t)kvh * a.cache_cap + slot0 + m) * 128;
          }
          dst[i] = __float2bfloat16_rn(o0);
          dst[i + 64] = __float2bfloat16_rn(o1);
          break;
        }
        case GEMV_ALLREDUCE: {
          // staged: the CTA sends its whole contiguous chunk after the loop
          s_ar[m][2 * (p - ar_p0)] = v0;
          s_ar[m][2 * (p - ar_p0) + 1] = v1;
          break;
        }
        case GEMV_ARGMAX: {
          // argmax over bf16-rounded logits, first index on ties
          const float b0 = bf16_round(v0), b1 = bf16_round(v1);
          if (b0 > best_v[m] || (b0 == best_v[m] && r0 < best_i[m])) best_v[m] = b0, best_i[m] = r0;
          if (b1 > best_v[m] || (b1 == best_v[m] && r1 < best_i[m])) best_v[m] = b1, best_i[m] = r1;
          break;
        }
      }
    }
  }

  if (a.epi == GEMV_ALLREDUCE) {
    // this CTA's outputs [2 * ar_p0, 2 * ar_p1) of every row go to every
    // rank's receive slot of this sender as 16-byte stores (NVLink for
    // peers); the chunk start is 16-byte aligned because ar_ppc is even
    __syncthreads();
    const int n_vec = (ar_p1 - ar_p0) / 2;  // float4 per row (2 pairs = 4 outputs)
    const int per_rank = M * n_vec;
    for (int i = tid; i < a.ar_tp * per_rank; i += kThreads) {
      const int r = i / per_rank, rem = i - r * per_rank;
      const int m = rem / n_vec, v = rem - m * n_vec;
      float4* dst = reinterpret_cast<float4*>(a.ar_dst[r] + ((size_t)a.ar_sender * M + m) * a.N + 2 * ar_p0);
      dst[v] = *reinterpret_cast<const float4*>(&s_ar[m][4 * v]);
    }
    if ((ar_p1 - ar_p0) & 1) {  // odd tail pair (only the last CTA can have one)
      for (int i = tid; i < a.ar_tp * M; i += kThreads) {
        const int r = i / M, m = i - r * M;
        float2* dst = reinterpret_cast<float2*>(a.ar_dst[r] + ((size_t)a.ar_sender * M + m) * a.N + 2 * (ar_p1 - 1));
        *dst = make_float2(s_ar[m][2 * (ar_p1 - 1 - ar_p0)], s_ar[m][2 * (ar_p1 - 1 - ar_p0) + 1]);
      }
    }
    // the last CTA to finish publishes this rank's partial to every rank
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
      const unsigned prev = atomicAdd(a.counter, 1u);
      s_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (s_last) {
      __threadfence_system();
      const int epoch = a.ar_epoch_ptr ? *a.ar_epoch_ptr * a.ar_epoch_mul + a.ar_epoch : a.ar_epoch;
      if (tid < a.ar_tp)
        asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(a.ar_flag[tid]), "r"(epoch) : "memory");
      if (tid == 0) *a.counter = 0u;
      if (a.ar_recv != nullptr) {
        // fused reduction (replaces a separate reduce kernel): wait (bounded)
        // for every rank's partial, sum them in rank order, add the residual
        // with the HF rounding order (residual + bf16(sum))
        __shared__ int s_fail;
        if (tid == 0) {
          s_fail = (a.status != nullptr && *((volatile int*)a.status) != 0) ? 1 : 0;
          unsigned long long t0;
          asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t0));
          for (int r = 0; r < a.ar_tp && !s_fail; ++r) {
            while (true) {
              int v;
              asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(a.ar_wait_flags + r) : "memory");
              if (v >= epoch) break;
              unsigned long long t1;
              asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t1));
              if ((long long)(t1 - t0) > a.ar_timeout_ns) {
                report_status(a.status, kStatusTimeoutPeerFlag);
                s_fail = 1;
                break;
              }
              __nanosleep(64);
            }
          }
        }
        __syncthreads();
        if (!s_fail) {
          const int n4 = a.N / 4;
          for (int i = tid; i < M * n4; i += kThreads) {
            const int m = i / n4, c = i - m * n4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < a.ar_tp; ++r) {
              const float4 p = __ldcg(reinterpret_cast<const float4*>(a.ar_recv + ((size_t)r * M + m) * a.N) + c);
              acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
            }
            const uint2 rr = *reinterpret_cast<const uint2*>(a.ar_residual + (size_t)m * a.N + 4 * c);
            const float2 r0 = unpack_bf16x2(rr.x), r1 = unpack_bf16x2(rr.y);
            *reinterpret_cast<uint2*>(a.ar_out + (size_t)m * a.N + 4 * c) =
                make_uint2(pack_bf16x2(r0.x + bf16_round(acc.x), r0.y + bf16_round(acc.y)),
                           pack_bf16x2(r1.x + bf16_round(acc.z), r1.y + bf16_round(acc.w)));
          }
        }
      }
    }
    return;
  }
  if (a.epi != GEMV_ARGMAX) return;

  // ---- argmax: CTA partials, then the last CTA reduces ----
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MR; ++m) s_bval[warp][m] = best_v[m], s_bidx[warp][m] = best_i[m];
  }
  __syncthreads();
  if (tid < M) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < kWarps; ++w) {
      const float v = s_bval[w][tid];
      const int i = s_bidx[w][tid];
      if (v > bv || (v == bv && i < bi)) bv = v, bi = i;
    }
    a.part_val[(size_t)tid * gridDim.x + blockIdx.x] = bv;
    a.part_idx[(size_t)tid * gridDim.x + blockIdx.x] = bi;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(a.counter, 1u);
    s_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Reduce partials of every row: warp m handles row m.
  if (warp < M) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int b = lane; b < (int)gridDim.x; b += 32) {
      const float v = __ldcg(a.part_val + (size_t)warp * gridDim.x + b);
      const int i = __ldcg(a.part_idx + (size_t)warp * gridDim.x + b);
      if (v > bv || (v == bv && i < bi)) bv = v, bi = i;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
    }
    if (lane == 0) {
      // no logit compared (all NaN): report token 0, never an index past the
      // vocabulary (the token feeds the embedding load below)
      if (bi < 0 || bi >= a.N) bi = 0;
      a.out_token[warp] = bi;
      s_bidx[0][warp] = bi;
    }
  }
  __syncthreads();
  const int last_tok = s_bidx[0][M - 1];
  if (tid == 0) {
    if (a.token_log != nullptr) {
      const int n = *a.gen_count;
      a.token_log[n] = last_tok;
      *a.gen_count = n + 1;
    }
    if (a.pos_advance != nullptr) {
      const int n = a.n_advance > 0 ? a.n_advance : 1;
      for (int i = 0; i < n; ++i) a.pos_advance[i] += M;
    }
    *a.counter = 0u;
  }
  if (a.embed != nullptr) {
    const uint4* src = reinterpret_cast<const uint4*>(a.embed + (size_t)last_tok * K);
    uint4* dst = reinterpret_cast<uint4*>(a.next_hidden);
    for (int c = tid; c < K / 8; c += kThreads) dst[c] = src[c];
  }
}

template <int MR, bool kXG = false>
__global__ void __launch_bounds__(kThreads) gemv_kernel(GemvArgs a) {
  gemv_body<MR, kXG>(a);
}

// One-row calls whose grid needs 2-3 waves at 2 CTAs per SM (e.g. the 8B QKV
// projection's 384 CTAs): registers capped so three CTAs fit an SM and the
// grid runs as one wave.  The same body, so the same arithmetic and bits.
__global__ void __launch_bounds__(kThreads, 3) gemv_kernel_one_wave(GemvArgs a) {
  gemv_body<1, false>(a);
}

// One-wave variant for 2-3-wave one-row grids; SC_GEMV_THREE_PER_SM=0 turns it off (A/B runs).
static bool gemv_three_per_sm() {
  static const bool on = [] {
    const char* e = getenv("SC_GEMV_THREE_PER_SM");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

cudaError_t gemv_bf16(const GemvArgs& a, cudaStream_t stream) {
  if (a.M < 1 || a.M > 8 || (a.K % 8) != 0 || (a.N % 2) != 0) return cudaErrorInvalidValue;
  const size_t smem = (size_t)a.M * a.K * 2;
  const bool xg = smem > 200 * 1024;
  if (xg && (a.norm_w != nullptr || a.ldx != a.K || a.M <= 2)) return cudaErrorInvalidValue;
  const int n_pairs = a.N / 2;
  int grid = (n_pairs + kWarps - 1) / kWarps;
  const int cap = (a.num_sms > 0 ? a.num_sms : 148) * 8;
  if (grid > cap) grid = cap;
  if (a.epi == GEMV_ALLREDUCE) {
    // at most kArMaxPairs (rounded to even) pairs per CTA
    const int need = (n_pairs + kArMaxPairs - 2) / (kArMaxPairs - 1);
    if (grid < need) grid = need;
    if (a.N % 4 != 0) return cudaErrorInvalidValue;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = xg ? 0 : smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
#define SC_LAUNCH_GEMV(MRV)                                        \
  {                                                                \
    ensure_smem_attr(gemv_kernel<MRV>, 200 * 1024);                \
    return cudaLaunchKernelEx(&cfg, gemv_kernel<MRV>, a);          \
  }
  if (xg) {
    if (a.M <= 4) return cudaLaunchKernelEx(&cfg, gemv_kernel<4, true>, a);
    return cudaLaunchKernelEx(&cfg, gemv_kernel<8, true>, a);
  }
  if (a.M == 1 && gemv_three_per_sm() && grid > 2 * (a.num_sms > 0 ? a.num_sms : 148) &&
      grid <= 3 * (a.num_sms > 0 ? a.num_sms : 148)) {
    ensure_smem_attr(gemv_kernel_one_wave, 200 * 1024);
    return cudaLaunchKernelEx(&cfg, gemv_kernel_one_wave, a);
  }
  if (a.M == 1) SC_LAUNCH_GEMV(1)
  else if (a.M <= 2) SC_LAUNCH_GEMV(2)
  else if (a.M <= 4) SC_LAUNCH_GEMV(4)
  else SC_LAUNCH_GEMV(8)
#undef SC_LAUNCH_GEMV
  return cudaErrorInvalidValue;
}

}  // namespace sc

// ===========================================================================
// Allocation-free entry point (declared in no_alloc.h; no counterpart in the
// reference).  The LM-head/argmax kernel above needs scratch for its per-CTA
// (max, index) partials and its completion counter; here that scratch is a
// fixed-size file-scope device array instead of caller-provided buffers, for
// callers that cannot allocate device memory.
// ===========================================================================
#include "no_alloc.h"

namespace sc {
namespace {

struct NoAllocScratch {
  float part_val[SC_NOALLOC_MAX_PARTIALS];
  int part_idx[SC_NOALLOC_MAX_PARTIALS];
  unsigned int counter;
};

// One copy per device that loads the library (~129 KiB), alive until exit.
static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

// Device address of g_noalloc_scratch, looked up once per device.  In host
// code the symbol itself is only a host-side stand-in, never a device
// address, so it is never passed to a kernel directly.
NoAllocScratch* g_noalloc_ptr[64] = {nullptr};
std::mutex g_noalloc_setup_lock;

}  // namespace
}  // namespace sc

extern "C" __attribute__((visibility("default"))) const char* sc_noalloc_error_string(int code) {
  switch (code) {
    case SC_NOALLOC_OK: return "ok";
    case SC_NOALLOC_EBADSHAPE:
      return "shape outside the limits: 1 <= M <= 8, K % 8 == 0, N even, M*K*2 <= 200 KiB";
    case SC_NOALLOC_ETOOLARGE: return "launch grid * M exceeds the fixed scratch (16384 partials)";
    case SC_NOALLOC_ESYMBOL: return "cudaGetSymbolAddress of the scratch array failed";
    case SC_NOALLOC_ELAUNCH: return "memset of the counter or kernel launch failed";
    case SC_NOALLOC_EBADPOINTER:
      return "x, w, norm_w must be 16-byte aligned device pointers (x, w non-NULL); out_token non-NULL, "
             "4-byte aligned";
  }
  return "unknown error code";
}

extern "C" __attribute__((visibility("default"))) int sc_lm_head_argmax_noalloc(
    const void* x, const void* w, const void* norm_w, float eps, int M, int N, int K,
    int* out_token, cudaStream_t stream) {
  using namespace sc;
  if (M < 1 || M > SC_NOALLOC_MAX_ROWS || K < 8 || (K % 8) != 0 || N < 2 || (N % 2) != 0 ||
      (size_t)M * K * 2 > 200 * 1024)
    return SC_NOALLOC_EBADSHAPE;
  // the kernel reads x, w and norm_w with 16-byte loads and writes int32 tokens
  if (x == nullptr || w == nullptr || out_token == nullptr ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
        reinterpret_cast<uintptr_t>(norm_w)) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(out_token) & 3u) != 0)
    return SC_NOALLOC_EBADPOINTER;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SC_NOALLOC_ESYMBOL;
  // Set-up on the first call on this device (the device is current here),
  // under a lock so that concurrent first calls from several host threads
  // look the address up once.
  NoAllocScratch* scratch = nullptr;
  {
    std::lock_guard<std::mutex> guard(g_noalloc_setup_lock);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
        return SC_NOALLOC_ESYMBOL;
      g_noalloc_ptr[dev] = reinterpret_cast<NoAllocScratch*>(p);
    }
    scratch = g_noalloc_ptr[dev];
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 148;
  int grid = (N / 2 + kWarps - 1) / kWarps;
  if (grid > sms * 8) grid = sms * 8;
  if ((long long)grid * M > SC_NOALLOC_MAX_PARTIALS) return SC_NOALLOC_ETOOLARGE;

  // The completion counter must start at zero; the partials are overwritten.
  if (cudaMemsetAsync(&scratch->counter, 0, sizeof(unsigned int), stream) != cudaSuccess)
    return SC_NOALLOC_ELAUNCH;
  GemvArgs a{};
  a.w = reinterpret_cast<const __nv_bfloat16*>(w);
  a.x = reinterpret_cast<const __nv_bfloat16*>(x);
  a.ldx = K;
  a.M = M;
  a.N = N;
  a.K = K;
  a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.epi = GEMV_ARGMAX;
  a.part_val = scratch->part_val;
  a.part_idx = scratch->part_idx;
  a.counter = &scratch->counter;
  a.out_token = out_token;
  a.num_sms = sms;
  if (gemv_bf16(a, stream) != cudaSuccess) return SC_NOALLOC_ELAUNCH;
  return SC_NOALLOC_OK;
}
