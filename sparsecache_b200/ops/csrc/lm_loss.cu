// Row log-sum-exp + logit gathers over bf16 logits, and their backward.
//
// The drafter losses (hard CE on the label, soft CE on the teacher's top-k,
// the prefix-weighted label score of the memory-contrast margin; reference
// experiments/train_sparse_kv_drafter.py:57-152 and
// experiments/train_sparse_kv_eagle.py:97-175) read the log-softmax only at
// a few ids per row: logp[id] = z[id] - lse.  So a row needs its lse and the
// logits at its ids, and the gradient of any such loss with respect to the
// logits is
//     d z[v] = g_lse * softmax(z)[v] + sum_j g_z[j] * [v == id_j],
// with g_lse, g_z from autograd on the small (lse, gathered) tensors.  These
// kernels produce (lse, gathered) in one read of the row and the bf16
// gradient row in one read + one write (in place over the logits allowed),
// instead of materialising fp32 log-probabilities, their gradient and the
// one-hot gathers over the whole vocabulary.  The LM-head GEMM before and
// the dX GEMM after are the tcgen05 GEMM (ops/lm_loss.py).
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {
constexpr int kLseThreads = 256;

__device__ __forceinline__ void merge_max_sum(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2, s = s2;
    return;
  }
  const float mn = fmaxf(m, m2);
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}
}  // namespace

__global__ void __launch_bounds__(kLseThreads) lse_gather_kernel(LseGatherArgs a) {
  const int r = blockIdx.x;
  const int tid = threadIdx.x;
  const __nv_bfloat16* row = a.logits + (size_t)r * a.ld;
  const uint4* row4 = reinterpret_cast<const uint4*>(row);
  float m = -INFINITY, s = 0.f;
  for (int c = tid; c < a.V / 8; c += kLseThreads) {
    const uint4 u = row4[c];
    float x[8];
    const float2 p0 = unpack_bf16x2(u.x), p1 = unpack_bf16x2(u.y), p2 = unpack_bf16x2(u.z), p3 = unpack_bf16x2(u.w);
    x[0] = p0.x, x[1] = p0.y, x[2] = p1.x, x[3] = p1.y, x[4] = p2.x, x[5] = p2.y, x[6] = p3.x, x[7] = p3.y;
    float cm = x[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) cm = fmaxf(cm, x[i]);
    float cs = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) cs += __expf(x[i] - cm);
    merge_max_sum(m, s, cm, cs);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge_max_sum(m, s, m2, s2);
  }
  __shared__ float sm[kLseThreads / 32], ss[kLseThreads / 32];
  const int warp = tid >> 5, lane = tid & 31;
  if (lane == 0) sm[warp] = m, ss[warp] = s;
  __syncthreads();
  if (tid == 0) {
    float M = sm[0], S = ss[0];
    for (int w = 1; w < kLseThreads / 32; ++w) merge_max_sum(M, S, sm[w], ss[w]);
    a.lse[r] = M + __logf(S);
  }
  for (int j = tid; j < a.G; j += kLseThreads) {
    const int id = a.ids[(size_t)r * a.G + j];
    a.z[(size_t)r * a.G + j] = (id >= 0 && id < a.V) ? __bfloat162float(row[id]) : 0.f;
  }
}

__global__ void __launch_bounds__(kLseThreads) lse_gather_backward_kernel(LseGatherArgs a) {
  const int r = blockIdx.x;
  const int tid = threadIdx.x;
  const float l = a.lse[r];
  const float g = a.g_lse != nullptr ? a.g_lse[r] : 0.f;
  const uint4* src = reinterpret_cast<const uint4*>(a.logits + (size_t)r * a.ld);
  __nv_bfloat16* drow = a.dlogits + (size_t)r * a.ldd;
  uint4* dst = reinterpret_cast<uint4*>(drow);
  for (int c = tid; c < a.V / 8; c += kLseThreads) {
    const uint4 u = src[c];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = unpack_bf16x2(w[i]);
      o[i] = pack_bf16x2(g * __expf(x.x - l), g * __expf(x.y - l));
    }
    dst[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  // the gathered ids, one thread in id order (duplicates add up, deterministically)
  if (tid == 0 && a.g_z != nullptr) {
    for (int j = 0; j < a.G; ++j) {
      const int id = a.ids[(size_t)r * a.G + j];
      if (id < 0 || id >= a.V) continue;
      drow[id] = __float2bfloat16_rn(__bfloat162float(drow[id]) + a.g_z[(size_t)r * a.G + j]);
    }
  }
}

cudaError_t lse_gather(const LseGatherArgs& a, cudaStream_t stream) {
  if (a.R < 1 || a.V % 8 != 0 || a.ld % 8 != 0) return cudaErrorInvalidValue;
  lse_gather_kernel<<<a.R, kLseThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t lse_gather_backward(const LseGatherArgs& a, cudaStream_t stream) {
  if (a.R < 1 || a.V % 8 != 0 || a.ld % 8 != 0 || a.ldd % 8 != 0) return cudaErrorInvalidValue;
  lse_gather_backward_kernel<<<a.R, kLseThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace sc
