// Split-K decode / verify attention over a paged layer cache.
//
// The query block is M <= 8 consecutive new tokens (M = 1 for greedy decode,
// M = gamma + 1 for the batched speculative verifier) at positions
// *pos .. *pos + M - 1; row m sees keys [0, *pos + m].  The position lives in
// device memory so a captured CUDA graph replays the same launch every step.
//
// Grid: (kv_head, split).  A CTA scores one key chunk for all G = H/H_kv
// query heads sharing the kv head and all M rows (GQA packing: the K/V chunk
// is read once for every query vector), writes (max, sum, o[128]) partials,
// and the last CTA of each kv head merges the splits (a per-head counter,
// reset by that CTA, makes the merge graph-replayable without a second
// launch).  Replaces the reference's HF DynamicCache concatenation + SDPA per
// token (modeling.py:383-417; progressive_kv_feasibility.py:561-613, 616-682).
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {
constexpr int kThreads = 128;
constexpr int kMaxQV = 64;  // M * G
}  // namespace

__global__ void __launch_bounds__(kThreads)
    attention_decode_kernel(AttnDecodeArgs a, int chunk_cap) {
  extern __shared__ __align__(16) float dsm[];
  const int G = a.n_heads / a.n_kv_heads;
  const int QV = a.M * G;
  float* qs = dsm;                  // [QV][128]
  float* sc = qs + QV * 128;        // [QV][chunk_cap]
  __shared__ int s_last;

  const int kvh = blockIdx.x, split = blockIdx.y, splits = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos0 = *a.pos;
  const int n_keys = pos0 + a.M;
  const int chunk = (n_keys + splits - 1) / splits;
  const int k_begin = split * chunk;
  const int k_end = min(n_keys, k_begin + chunk);
  const int nk = max(0, k_end - k_begin);
  const float sl2 = a.scale * 1.4426950408889634f;

  // q vectors: qv = m * G + gi  -> head kvh * G + gi of row m
  for (int idx = tid; idx < QV * 128; idx += kThreads) {
    const int qv = idx >> 7, d = idx & 127;
    const int m = qv / G, gi = qv % G;
    qs[idx] = __bfloat162float(a.q[(size_t)m * a.n_heads * 128 + (kvh * G + gi) * 128 + d]);
  }
  __syncthreads();

  const __nv_bfloat16* kb = a.k_cache + (size_t)kvh * a.cache_cap * 128;
  const __nv_bfloat16* vb = a.v_cache + (size_t)kvh * a.cache_cap * 128;

  // ---- scores: one key per thread, all query vectors ----
  for (int j = tid; j < nk; j += kThreads) {
    const int key = k_begin + j;
    const uint4* kr = reinterpret_cast<const uint4*>(kb + (size_t)key * 128);
    float kf[128];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint4 v = kr[c];
      const float2 f0 = unpack_bf16x2(v.x), f1 = unpack_bf16x2(v.y), f2 = unpack_bf16x2(v.z),
                   f3 = unpack_bf16x2(v.w);
      kf[8 * c + 0] = f0.x; kf[8 * c + 1] = f0.y; kf[8 * c + 2] = f1.x; kf[8 * c + 3] = f1.y;
      kf[8 * c + 4] = f2.x; kf[8 * c + 5] = f2.y; kf[8 * c + 6] = f3.x; kf[8 * c + 7] = f3.y;
    }
    for (int qv = 0; qv < QV; ++qv) {
      const float* q = qs + qv * 128;
      float s = 0.f;
#pragma unroll
      for (int d = 0; d < 128; ++d) s = fmaf(q[d], kf[d], s);
      const int m = qv / G;
      sc[qv * chunk_cap + j] = (key <= pos0 + m) ? s * sl2 : -INFINITY;
    }
  }
  __syncthreads();

  // ---- per query vector: max and exp-sum over the chunk (one warp each) ----
  __shared__ float s_max[kMaxQV], s_sum[kMaxQV];
  for (int qv = warp; qv < QV; qv += kThreads / 32) {
    float mx = -INFINITY;
    for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sc[qv * chunk_cap + j]);
    mx = warp_max(mx);
    const float base = (mx == -INFINITY) ? 0.f : mx;
    float sum = 0.f;
    for (int j = lane; j < nk; j += 32) {
      const float e = exp2f(sc[qv * chunk_cap + j] - base);
      sc[qv * chunk_cap + j] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    if (lane == 0) s_max[qv] = mx, s_sum[qv] = sum;
  }
  __syncthreads();

  // ---- o = p . V : thread owns dims (2*(tid%64), +1) for query vectors tid/64, +2, ... ----
  {
    const int d = 2 * (tid & 63);
    const int q0 = tid >> 6;
    float acc[kMaxQV / 2][2];
    const int nq = (QV - q0 + 1) / 2;
#pragma unroll
    for (int i = 0; i < kMaxQV / 2; ++i) acc[i][0] = acc[i][1] = 0.f;
    for (int j = 0; j < nk; ++j) {
      const float2 v = unpack_bf16x2(
          *reinterpret_cast<const uint32_t*>(vb + (size_t)(k_begin + j) * 128 + d));
#pragma unroll
      for (int i = 0; i < kMaxQV / 2; ++i) {
        if (i < nq) {
          const float pj = sc[(q0 + 2 * i) * chunk_cap + j];
          acc[i][0] = fmaf(pj, v.x, acc[i][0]);
          acc[i][1] = fmaf(pj, v.y, acc[i][1]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kMaxQV / 2; ++i) {
      if (i < nq) {
        const int qv = q0 + 2 * i;
        const int m = qv / G, gi = qv % G;
        const int h = kvh * G + gi;
        float* po = a.part_o + (((size_t)h * a.M + m) * splits + split) * 128;
        po[d] = acc[i][0];
        po[d + 1] = acc[i][1];
      }
    }
  }
  if (tid < QV) {
    const int m = tid / G, gi = tid % G;
    const int h = kvh * G + gi;
    float* pm = a.part_ml + (((size_t)h * a.M + m) * splits + split) * 2;
    pm[0] = s_max[tid];
    pm[1] = s_sum[tid];
  }

  // ---- last CTA of this kv head merges the splits ----
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(a.counters + kvh, 1u);
    s_last = (prev == (unsigned)splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = tid; idx < QV * 128; idx += kThreads) {
    const int qv = idx >> 7, d = idx & 127;
    const int m = qv / G, gi = qv % G;
    const int h = kvh * G + gi;
    const float* pm = a.part_ml + ((size_t)h * a.M + m) * splits * 2;
    const float* po = a.part_o + ((size_t)h * a.M + m) * splits * 128;
    float gmax = -INFINITY;
    for (int s = 0; s < splits; ++s) gmax = fmaxf(gmax, __ldcg(pm + 2 * s));
    float num = 0.f, den = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float ms = __ldcg(pm + 2 * s);
      if (ms == -INFINITY) continue;
      const float w = exp2f(ms - gmax);
      num += w * __ldcg(po + (size_t)s * 128 + d);
      den += w * __ldcg(pm + 2 * s + 1);
    }
    a.out[(size_t)m * a.n_heads * 128 + h * 128 + d] =
        __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
  }
  if (tid == 0) a.counters[kvh] = 0u;
}

cudaError_t attention_decode(const AttnDecodeArgs& a, cudaStream_t stream) {
  const int G = a.n_heads / a.n_kv_heads;
  if (a.M < 1 || a.M * G > kMaxQV || a.splits < 1) return cudaErrorInvalidValue;
  // worst case keys per split given the cache capacity
  const int chunk_cap = (a.cache_cap + a.M + a.splits - 1) / a.splits;
  const size_t smem = (size_t)(a.M * G * 128 + a.M * G * chunk_cap) * sizeof(float);
  if (smem > 220 * 1024) return cudaErrorInvalidValue;
  ensure_smem_attr(attention_decode_kernel, 220 * 1024);
  dim3 grid(a.n_kv_heads, a.splits);
  attention_decode_kernel<<<grid, kThreads, smem, stream>>>(a, chunk_cap);
  return cudaGetLastError();
}

}  // namespace sc
