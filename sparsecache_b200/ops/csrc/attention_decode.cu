// Split-K decode / verify attention over a paged layer cache, merged through
// distributed shared memory inside a thread-block cluster.
//
// The query block is M <= 8 consecutive new tokens (M = 1 for greedy decode,
// M = gamma + 1 for the batched speculative verifier) at positions
// *pos .. *pos + M - 1; row m sees keys [0, *pos + m].  The position lives in
// device memory so a captured CUDA graph replays the same launch every step.
//
// Grid (S, n_kv_heads), cluster (S, 1, 1): the S CTAs of a cluster split the
// keys of one kv head.  Each CTA stages 128-key K/V sub-chunks into shared
// memory with cp.async (64 KB in flight per CTA), scores them for all
// G = H/H_kv query heads and all M rows at once (GQA packing: K/V are read
// once per kv head), keeps an online softmax per query vector, and leaves its
// partial (max, sum, o[128]) in its own shared memory.  After a cluster
// barrier every CTA merges a slice of the outputs by reading its peers'
// partials over DSMEM; a second barrier keeps the partials alive until all
// peers are done.  No global scratch, no atomics, one launch.
//
// Replaces the reference's per-token HF DynamicCache concatenation + SDPA
// (modeling.py:383-417; progressive_kv_feasibility.py:561-613, 616-682).
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace sc {

namespace {
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kSub = 64;      // keys per staged sub-chunk (double-buffered)
constexpr int kMaxQV = 32;    // M * G
constexpr int kMaxRows = 8;   // largest query block M
constexpr int kRow = 256;     // bytes per K/V row (128 bf16)
constexpr int kMaxOuter = 16; // clusters per kv head (second split level)

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz)
               : "memory");
}
}  // namespace

struct DecodeSmem {
  __nv_bfloat16 k[2][kSub * 128];  // double-buffered sub-chunks
  __nv_bfloat16 v[2][kSub * 128];
  float s[kMaxQV][kSub];
  float o[kMaxQV][128];  // partial output of this CTA (unnormalised)
  float m[kMaxQV];       // running max (log2 domain)
  float l[kMaxQV];       // running sum
  float corr[kMaxQV];
};

// QVT is the compile-time query-vector count (M * G rounded up); the exact
// decode shapes (QVT == M * G) carry no per-vector guards in the inner loops.
template <int QVT>
__global__ void __launch_bounds__(kThreads)
    attention_decode_kernel(AttnDecodeArgs a, int chunk, int outer) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();

  const int G = a.n_heads / a.n_kv_heads;
  const int QV = a.M * G;
  const int S = gridDim.x / outer;          // CTAs of one cluster
  const int split = blockIdx.x % S;         // rank within the cluster
  const int cidx = blockIdx.x / S;          // cluster index of this kv head
  const int kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // *pos and the cache rows [0, *pos) were written at least two launches
  // back (the LM-head kernel of the previous step and earlier QKV kernels),
  // so they are read before the programmatic wait; q and the M new rows come
  // from the QKV kernel right before this one and are read after it.
  const int n_keys = a.n_virtual != nullptr ? *a.n_virtual : *a.pos + a.M;
  const int pos0 = n_keys - a.M;  // virtual index of query row 0
  const int page_mask = (1 << a.page_shift) - 1;
  auto phys = [&](int v) -> int {
    return a.page_table != nullptr ? (a.page_table[v >> a.page_shift] << a.page_shift) + (v & page_mask) : v;
  };
  const int k_begin = blockIdx.x * chunk;  // global split index over all clusters
  const int k_end = min(n_keys, k_begin + chunk);
  const float sl2 = a.scale * 1.4426950408889634f;
  const __nv_bfloat16* kb = a.k_cache + (size_t)kvh * a.cache_cap * 128;
  const __nv_bfloat16* vb = a.v_cache + (size_t)kvh * a.cache_cap * 128;
  const uint32_t sk0 = smem_u32(sm.k[0]), sv0 = smem_u32(sm.v[0]);
  constexpr uint32_t kBufBytes = kSub * kRow;
  // stage rows [base, base + nk) whose key index lies in [lo, hi) into buffer
  // buf; rows past nk are zero-filled when zero_tail is set
  auto stage = [&](int buf, int base, int nk, int lo, int hi, bool zero_tail) {
    const uint32_t sk = sk0 + buf * kBufBytes, sv = sv0 + buf * kBufBytes;
    for (int i = tid; i < kSub * 16; i += kThreads) {
      const int r = i >> 4, c = i & 15;
      const int key = base + r;
      const bool in = r < nk;
      if (in ? (key < lo || key >= hi) : !zero_tail) continue;
      const size_t off = (size_t)(in ? phys(key) : 0) * 128 + c * 8;
      cp_async16(sk + r * kRow + c * 16, kb + off, in);
      cp_async16(sv + r * kRow + c * 16, vb + off, in);
    }
  };
  if (k_begin < k_end) stage(0, k_begin, min(kSub, k_end - k_begin), 0, pos0, true);
  for (int i = tid; i < QV * 128; i += kThreads) sm.o[i / 128][i % 128] = 0.f;
  if (tid < QV) sm.m[tid] = -INFINITY, sm.l[tid] = 0.f;
  pdl_wait();
  pdl_launch_dependents();

  // Scores use LPK lanes per key (LPK = 8 for small query blocks: 4 keys per
  // warp step and a 3-level shuffle reduction); lane owns DPL dims of every
  // query vector in registers.
  constexpr int LPK = QVT <= 8 ? 8 : 32;
  constexpr int DPL = 128 / LPK;
  const int sub = lane % LPK;        // dim slice
  const int kgrp = lane / LPK;       // key slot within the warp step
  float q[QVT][DPL];
#pragma unroll
  for (int qv = 0; qv < QVT; ++qv) {
    if (qv < QV) {
      const int m = qv / G, gi = qv % G;
      const __nv_bfloat16* qp = a.q + (size_t)m * a.n_heads * 128 + (kvh * G + gi) * 128 + DPL * sub;
#pragma unroll
      for (int c = 0; c < DPL / 4; ++c) {
        const uint2 raw = *reinterpret_cast<const uint2*>(qp + 4 * c);
        const float2 f0 = unpack_bf16x2(raw.x), f1 = unpack_bf16x2(raw.y);
        q[qv][4 * c] = f0.x; q[qv][4 * c + 1] = f0.y; q[qv][4 * c + 2] = f1.x; q[qv][4 * c + 3] = f1.y;
      }
    }
  }
  int it = 0;
  for (int base = k_begin; base < k_end; base += kSub, ++it) {
    const int nk = min(kSub, k_end - base);
    const int buf = it & 1;
    if (it == 0) {
      stage(0, base, nk, pos0, n_keys, false);  // the new rows, now visible
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // prefetch the next sub-chunk into the other buffer while this one runs
    const int nbase = base + kSub;
    if (nbase < k_end) stage(buf ^ 1, nbase, min(kSub, k_end - nbase), 0, n_keys, true);
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 1;" ::: "memory");
    __syncthreads();

    // scores: each warp step covers 32/LPK keys; LPK lanes split the dims
    constexpr int KPW = 32 / LPK;
    for (int j0 = warp * KPW; j0 < nk; j0 += kWarps * KPW) {
      const int j = j0 + kgrp;
      const bool valid = j < nk;
      float kf[DPL];
      {
        const __nv_bfloat16* kr = sm.k[buf] + (valid ? j : 0) * 128 + DPL * sub;
#pragma unroll
        for (int c = 0; c < DPL / 4; ++c) {
          const uint2 raw = *reinterpret_cast<const uint2*>(kr + 4 * c);
          const float2 f0 = unpack_bf16x2(raw.x), f1 = unpack_bf16x2(raw.y);
          kf[4 * c] = f0.x; kf[4 * c + 1] = f0.y; kf[4 * c + 2] = f1.x; kf[4 * c + 3] = f1.y;
        }
      }
      const int key = base + j;
#pragma unroll
      for (int qv = 0; qv < QVT; ++qv) {
        if (qv < QV) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < DPL; ++e) d = fmaf(q[qv][e], kf[e], d);
#pragma unroll
          for (int o = LPK / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
          if (valid && sub == (qv % LPK)) sm.s[qv][j] = (key <= pos0 + qv / G) ? d * sl2 : -INFINITY;
        }
      }
    }
    __syncthreads();

    // online softmax update, one warp per query vector
    for (int qv = warp; qv < QV; qv += kWarps) {
      float mx = -INFINITY;
      for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sm.s[qv][j]);
      mx = warp_max(mx);
      const float m_old = sm.m[qv];
      const float m_new = fmaxf(m_old, mx);
      const float base_m = (m_new == -INFINITY) ? 0.f : m_new;
      float sum = 0.f;
      for (int j = lane; j < nk; j += 32) {
        const float e = exp2f(sm.s[qv][j] - base_m);
        sm.s[qv][j] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float c = exp2f(m_old - base_m);
        sm.corr[qv] = c;
        sm.l[qv] = sm.l[qv] * c + sum;
        sm.m[qv] = m_new;
      }
    }
    __syncthreads();

    // o[qv][d] = o * corr + sum_j p[qv][j] * v[j][d]; thread t owns dim
    // d = t % 128 for the query vectors qv = t / 128 (mod 2)
    {
      constexpr int kHalf = (QVT + 1) / 2;
      const int d = tid & 127;
      const int q0 = tid >> 7;
      float acc[kHalf];
#pragma unroll
      for (int i = 0; i < kHalf; ++i) acc[i] = 0.f;
      float acc2[kHalf];
#pragma unroll
      for (int i = 0; i < kHalf; ++i) acc2[i] = 0.f;
      int j = 0;
      for (; j + 1 < nk; j += 2) {  // two keys per step: independent FMA chains
        const float v0 = __bfloat162float(sm.v[buf][j * 128 + d]);
        const float v1 = __bfloat162float(sm.v[buf][(j + 1) * 128 + d]);
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          const int qv = q0 + 2 * i;
          if (qv < QV) {
            acc[i] = fmaf(sm.s[qv][j], v0, acc[i]);
            acc2[i] = fmaf(sm.s[qv][j + 1], v1, acc2[i]);
          }
        }
      }
      if (j < nk) {
        const float v0 = __bfloat162float(sm.v[buf][j * 128 + d]);
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          const int qv = q0 + 2 * i;
          if (qv < QV) acc[i] = fmaf(sm.s[qv][j], v0, acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < kHalf; ++i) acc[i] += acc2[i];
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        const int qv = q0 + 2 * i;
        if (qv < QV) sm.o[qv][d] = sm.o[qv][d] * sm.corr[qv] + acc[i];
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }

  // ---- merge the S partials of this kv head through DSMEM ----
  cluster.sync();
  for (int idx = split * kThreads + tid; idx < QV * 128; idx += S * kThreads) {
    const int qv = idx >> 7, d = idx & 127;
    // all peer loads are independent: issue them together (<= 16 peers)
    float mr[16], lr[16], orr[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      if (r < S) {
        const DecodeSmem* peer = cluster.map_shared_rank(&sm, r);
        mr[r] = peer->m[qv];
        lr[r] = peer->l[qv];
        orr[r] = peer->o[qv][d];
      }
    }
    float gmax = -INFINITY;
#pragma unroll
    for (int r = 0; r < 16; ++r)
      if (r < S) gmax = fmaxf(gmax, mr[r]);
    float num = 0.f, den = 0.f;
    if (gmax != -INFINITY) {
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        if (r < S && mr[r] != -INFINITY) {
          const float w = exp2f(mr[r] - gmax);
          num += w * orr[r];
          den += w * lr[r];
        }
      }
    }
    if (outer == 1) {
      const int m = qv / G, gi = qv % G;
      a.out[(size_t)m * a.n_heads * 128 + (kvh * G + gi) * 128 + d] =
          __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
    } else {
      float* part = a.ws + (((size_t)kvh * kMaxOuter + cidx) * kMaxQV + qv) * 130;
      part[2 + d] = num;
      if (d == 0) {
        part[0] = gmax;
        part[1] = den;
      }
    }
  }
  cluster.sync();
  if (outer == 1) return;
  // the last CTA of this kv head merges the clusters' partials in cluster order
  __shared__ unsigned s_ticket;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(a.counters + kvh, 1u);
  __syncthreads();
  if (s_ticket != (unsigned)(S * outer - 1)) return;
  __threadfence();
  for (int idx = tid; idx < QV * 128; idx += kThreads) {
    const int qv = idx >> 7, d = idx & 127;
    const float* base = a.ws + ((size_t)kvh * kMaxOuter * kMaxQV + qv) * 130;
    float gmax = -INFINITY;
    for (int c = 0; c < outer; ++c) gmax = fmaxf(gmax, __ldcg(base + (size_t)c * kMaxQV * 130));
    float num = 0.f, den = 0.f;
    if (gmax != -INFINITY) {
      for (int c = 0; c < outer; ++c) {
        const float* pc = base + (size_t)c * kMaxQV * 130;
        const float mc = __ldcg(pc);
        if (mc == -INFINITY) continue;
        const float w = exp2f(mc - gmax);
        num += w * __ldcg(pc + 2 + d);
        den += w * __ldcg(pc + 1);
      }
    }
    const int m = qv / G, gi = qv % G;
    a.out[(size_t)m * a.n_heads * 128 + (kvh * G + gi) * 128 + d] =
        __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
  }
  if (tid == 0) a.counters[kvh] = 0u;
}

// Clusters per kv head: enough CTAs for about two per SM when the kv heads are
// few (tensor parallelism) or the context long, at least 128 keys per CTA.
int attention_decode_outer(int cache_cap, int n_kv_heads, int cluster, int num_sms) {
  int r = (2 * num_sms + cluster * n_kv_heads / 2) / (cluster * n_kv_heads);
  const int by_keys = cache_cap / (cluster * 128);
  if (r > by_keys) r = by_keys;
  if (r > kMaxOuter) r = kMaxOuter;
  return r < 1 ? 1 : r;
}

int attention_decode_cluster(int cache_cap) {
  // 16-CTA clusters (non-portable, supported by B200) when the context is long
  // enough to give each CTA at least a sub-chunk; 8 otherwise.
  return cache_cap > 8 * kSub ? 16 : 8;
}

cudaError_t attention_decode(const AttnDecodeArgs& a, cudaStream_t stream) {
  const int G = a.n_heads / a.n_kv_heads;
  if (a.M < 1 || a.M * G > kMaxQV) return cudaErrorInvalidValue;
  const int S = a.splits;
  if (S < 1 || S > 16) return cudaErrorInvalidValue;
  int outer = 1;
  if (a.ws != nullptr && a.counters != nullptr) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    outer = attention_decode_outer(a.cache_cap, a.n_kv_heads, S, sms);
  }
  // keys per CTA: the cache capacity (+ the largest row block) split evenly
  // over all S * outer CTAs, rounded to 16 keys; independent of M so a row
  // sees the same split boundaries (and the same rounding) in decode and in
  // batched verification
  const int total = S * outer;
  int chunk = (a.cache_cap + kMaxRows + total - 1) / total;
  chunk = (chunk + 15) / 16 * 16;
  const int smem = (int)sizeof(DecodeSmem);
  const int qv = a.M * G;
  auto kern = qv <= 4 ? attention_decode_kernel<4>
            : qv <= 8 ? attention_decode_kernel<8>
            : qv <= 16 ? attention_decode_kernel<16> : attention_decode_kernel<32>;
  ensure_smem_attr(kern, smem);
  {
    static const void* nonportable_done[8] = {nullptr};
    bool done = false;
    for (auto* p : nonportable_done) done |= (p == reinterpret_cast<const void*>(kern));
    if (!done) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      for (auto*& p : nonportable_done)
        if (p == nullptr) { p = reinterpret_cast<const void*>(kern); break; }
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S * outer, a.n_kv_heads, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, a, chunk, outer);
}

}  // namespace sc
