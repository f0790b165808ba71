// Producer-side attention scores of prompt tokens (page / document priority).
//
//   score[t] = mean over (layer l, query row r, query head h) of
//              softmax_t'( q[l, r, h] . k[l, kvh(h), t'] * scale )[t]
//
// for t < n_tokens, with the query heads of a GQA group sharing one key head.
// The caller sums the scores per page or per document range.  This is the
// fp32 softmax(q K^T) the reference evaluates with einsum on [heads, keys]
// tensors and averages over heads (and layers) to rank KV pages or documents
// for progressive transfer and for the drafter teacher's page priorities
// (experiments/pd_progressive_kv_pipeline.py:117-141,
// experiments/extract_sparse_kv_teacher.py:193-237).
//
// It is bound by reading the keys once (layers x kv heads x tokens x 256 B),
// so it runs as three small kernels:
//   1. logits   one thread per key of one (layer, kv head): the key row is
//               loaded once (16-byte loads) and dotted with every query row
//               of its group (queries in shared memory, broadcast reads);
//               fp32 logits go to a scratch buffer and every 256-key chunk
//               leaves its (max, sum of exp) per query row;
//   2. stats    one warp per (layer, query row): the chunk partials merge
//               into the row's softmax max and denominator;
//   3. scores   one thread per token sums the normalised probabilities over
//               (layer, query row) in a fixed order (deterministic).
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {

constexpr int kPsThreads = 256;
constexpr int kPsD = 128;

__global__ void __launch_bounds__(kPsThreads) page_logits_kernel(PageScoreArgs a) {
  extern __shared__ float qs[];  // [rows_per_group = R * G][128] fp32 queries of this (layer, kv head)
  __shared__ float red_m[kPsThreads / 32][kPsMaxRowsPerGroup];
  __shared__ float red_s[kPsThreads / 32][kPsMaxRowsPerGroup];
  const int layer = blockIdx.y / a.n_kv_heads;
  const int kvh = blockIdx.y % a.n_kv_heads;
  const int G = a.n_q_heads / a.n_kv_heads;
  const int RG = a.n_rows * G;  // query rows of this group: (row r, head kvh*G + g) -> r * G + g
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < RG * kPsD; i += kPsThreads) {
    const int rg = i / kPsD, d = i % kPsD;
    const int r = rg / G, g = rg % G;
    qs[i] = a.q[(((size_t)layer * a.n_rows + r) * a.n_q_heads + kvh * G + g) * kPsD + d];
  }
  __syncthreads();
  const int t = blockIdx.x * kPsThreads + tid;
  const bool valid = t < a.n_tokens;
  uint4 kr[16];
  if (valid) {
    const uint4* src = reinterpret_cast<const uint4*>(a.keys[layer] + ((size_t)kvh * a.cache_cap + t) * kPsD);
#pragma unroll
    for (int c = 0; c < 16; ++c) kr[c] = src[c];
  }
  const int chunk = blockIdx.x;
  const int n_chunks = gridDim.x;
  for (int rg = 0; rg < RG; ++rg) {
    float dot = 0.f;
    if (valid) {
      const float* qv = qs + rg * kPsD;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint32_t w[4] = {kr[c].x, kr[c].y, kr[c].z, kr[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(w[e]);
          dot = fmaf(f.x, qv[c * 8 + 2 * e], dot);
          dot = fmaf(f.y, qv[c * 8 + 2 * e + 1], dot);
        }
      }
    }
    const float logit = valid ? dot * a.scale : -INFINITY;
    const int r = rg / G, g = rg % G;
    const int qrow = r * a.n_q_heads + kvh * G + g;  // (row, head) index of this query row
    if (valid) a.logits[((size_t)layer * a.n_rows * a.n_q_heads + qrow) * a.n_tokens + t] = logit;
    // chunk max and sum of exp(logit - max)
    const float m = warp_max(logit);
    const float s = warp_sum(valid ? __expf(logit - m) : 0.f);
    if (lane == 0) red_m[warp][rg % kPsMaxRowsPerGroup] = m, red_s[warp][rg % kPsMaxRowsPerGroup] = s;
    __syncthreads();
    if (tid == 0) {
      float mm = -INFINITY;
      for (int w = 0; w < kPsThreads / 32; ++w) mm = fmaxf(mm, red_m[w][rg % kPsMaxRowsPerGroup]);
      float ss = 0.f;
      for (int w = 0; w < kPsThreads / 32; ++w) {
        const float wm = red_m[w][rg % kPsMaxRowsPerGroup];
        if (wm != -INFINITY) ss += red_s[w][rg % kPsMaxRowsPerGroup] * __expf(wm - mm);
      }
      float2* part = a.partials + ((size_t)layer * a.n_rows * a.n_q_heads + qrow) * n_chunks + chunk;
      *part = make_float2(mm, ss);
    }
    __syncthreads();
  }
}

__global__ void page_stats_kernel(PageScoreArgs a, int n_chunks) {
  // one warp per (layer, query row): merge the chunk partials
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int n = a.n_layers * a.n_rows * a.n_q_heads;
  if (w >= n) return;
  const float2* part = a.partials + (size_t)w * n_chunks;
  float m = -INFINITY;
  for (int c = lane; c < n_chunks; c += 32) m = fmaxf(m, part[c].x);
  m = warp_max(m);
  float s = 0.f;
  for (int c = lane; c < n_chunks; c += 32) {
    const float2 p = part[c];
    if (p.x != -INFINITY) s += p.y * __expf(p.x - m);
  }
  s = warp_sum(s);
  if (lane == 0) a.stats[w] = make_float2(m, s);
}

__global__ void page_token_scores_kernel(PageScoreArgs a) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= a.n_tokens) return;
  const int n = a.n_layers * a.n_rows * a.n_q_heads;
  float acc = 0.f;
  for (int i = 0; i < n; ++i) {
    const float2 st = a.stats[i];
    const float l = a.logits[(size_t)i * a.n_tokens + t];
    acc += st.y > 0.f ? __expf(l - st.x) / st.y : 0.f;
  }
  a.token_scores[t] = acc / (float)n;
}

}  // namespace

cudaError_t page_token_scores(const PageScoreArgs& a, cudaStream_t stream) {
  if (a.n_layers < 1 || a.n_layers > kPsMaxLayers || a.n_rows < 1 || a.n_kv_heads < 1 ||
      a.n_q_heads % a.n_kv_heads != 0 || a.n_tokens < 1 || a.n_tokens > a.cache_cap)
    return cudaErrorInvalidValue;
  const int G = a.n_q_heads / a.n_kv_heads;
  if (a.n_rows * G > kPsMaxRowsPerGroup) return cudaErrorInvalidValue;
  const int n_chunks = (a.n_tokens + kPsThreads - 1) / kPsThreads;
  const size_t smem = (size_t)a.n_rows * G * kPsD * sizeof(float);
  ensure_smem_attr(page_logits_kernel, (int)smem);
  page_logits_kernel<<<dim3(n_chunks, a.n_layers * a.n_kv_heads), kPsThreads, smem, stream>>>(a);
  const int n_rows_total = a.n_layers * a.n_rows * a.n_q_heads;
  page_stats_kernel<<<(n_rows_total * 32 + 255) / 256, 256, 0, stream>>>(a, n_chunks);
  page_token_scores_kernel<<<(a.n_tokens + 255) / 256, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace sc
