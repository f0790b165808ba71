// K13: drafter cross-attention into exact, page-sparse target KV.
//
// One query per (memory layer, row, head) attends, non-causally, to the
// visible token rows of one sequence's memory.  Visibility is an int32 index
// list per sequence (sink + recent + top chunks, or a page view); there is no
// gathered copy of K/V: rows are read in place through the list.  Memory
// heads equal KV heads (no GQA), so each query is a GEMV over its rows and the
// kernel is bound by HBM/L2 bandwidth, not by tensor cores: 8 lanes per key
// (16 dims each, two 16-byte loads for K and two for V), two keys in flight
// per lane group with a warp-uniform loop (the 8-lane shuffles need the whole
// warp), fp32 online softmax in base 2, and a shared-memory merge of
// the CTA's lane groups.
//
// Backward computes dq only (the memory is an input, not a parameter):
//   dq = scale * sum_j p_j (dO.v_j - dO.o) k_j,  p_j = exp2(s_j - lse2)
// re-reading K/V once, with the forward's base-2 log-sum-exp.
//
// Layouts (elements): K/V address = base + l*layer_stride + seq*seq_stride +
// tok*tok_stride + h*head_stride + d; q/o/dO are [L, R, H, 128] bf16,
// lse [L, R, H] fp32, dq [L, R, H, 128] fp32.
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {
// 4 warps a CTA in both directions; the forward keeps the loads of the next
// key pair in flight while the current pair is computed
constexpr int kFwdThreads = 128;
constexpr int kBwdThreads = 128;

__device__ __forceinline__ void load16(const __nv_bfloat16* p, float (&x)[16]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
  const uint4 b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
  const unsigned w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ float group_sum8(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  return v;
}

struct RowCtx {
  const __nv_bfloat16* kb;
  const __nv_bfloat16* vb;
  const int* idx;
  int n;
  long long tok_stride;
};

__device__ __forceinline__ RowCtx row_ctx(const MemAttnArgs& a, int l, int r, int h, int sub) {
  RowCtx c;
  const int seq = a.row_seq ? a.row_seq[r] : 0;
  const long long off = (long long)l * a.layer_stride + (long long)seq * a.seq_stride +
                        (long long)h * a.head_stride + sub * 16;
  c.kb = a.k + off;
  c.vb = a.v + off;
  c.idx = a.idx ? a.idx + (long long)seq * a.idx_stride : nullptr;
  c.n = a.n_vis ? a.n_vis[seq] : a.n_fixed;
  c.tok_stride = a.tok_stride;
  return c;
}

__device__ __forceinline__ long long tok_off(const RowCtx& c, int j) {
  return (long long)(c.idx ? __ldg(c.idx + j) : j) * c.tok_stride;
}

// The K/V bytes one lane needs for its two keys of one loop iteration, kept
// packed (32 registers) so that the next iteration's loads can be in flight
// while this one is computed.
struct KvRaw {
  uint4 k0[2], v0[2], k1[2], v1[2];
};

__device__ __forceinline__ void fetch(const RowCtx& c, int base, int lane, KvRaw& r) {
  const int j0 = base + (lane >> 3), j1 = j0 + 4;
  const long long o0 = tok_off(c, j0 < c.n ? j0 : base);
  const long long o1 = tok_off(c, j1 < c.n ? j1 : base);
  const uint4* k0 = reinterpret_cast<const uint4*>(c.kb + o0);
  const uint4* v0 = reinterpret_cast<const uint4*>(c.vb + o0);
  const uint4* k1 = reinterpret_cast<const uint4*>(c.kb + o1);
  const uint4* v1 = reinterpret_cast<const uint4*>(c.vb + o1);
  r.k0[0] = __ldg(k0); r.k0[1] = __ldg(k0 + 1);
  r.v0[0] = __ldg(v0); r.v0[1] = __ldg(v0 + 1);
  r.k1[0] = __ldg(k1); r.k1[1] = __ldg(k1 + 1);
  r.v1[0] = __ldg(v1); r.v1[1] = __ldg(v1 + 1);
}

__device__ __forceinline__ void unpack16(const uint4 (&u)[2], float (&x)[16]) {
  const unsigned w[8] = {u[0].x, u[0].y, u[0].z, u[0].w, u[1].x, u[1].y, u[1].z, u[1].w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
}  // namespace

__global__ void __launch_bounds__(kFwdThreads) mem_attn_fwd_kernel(MemAttnArgs a) {
  constexpr int kGroups = kFwdThreads / 8, kKeysPerIter = kFwdThreads / 4;
  __shared__ float s_acc[kGroups][128];
  __shared__ float s_m[kGroups], s_l[kGroups];
  const int h = blockIdx.x, r = blockIdx.y, l = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane & 7, grp = warp * 4 + (lane >> 3);
  const RowCtx c = row_ctx(a, l, r, h, sub);
  const long long qoff = (((long long)l * a.R + r) * a.H + h) * 128;

  float q[16];
  load16(a.q + qoff + sub * 16, q);
#pragma unroll
  for (int i = 0; i < 16; ++i) q[i] *= a.scale_log2;

  float m = -INFINITY, lsum = 0.f, acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;

  // The trip count depends on the warp only (shuffles below need all 32 lanes):
  // warp w takes keys [base, base + 8) with base = 8w, 8w + 8 * warps, ...;
  // lane group g of the warp takes keys base + g and base + 4 + g.  The next
  // iteration's K/V rows are fetched before this iteration is computed.
  KvRaw cur, nxt;
  int base = warp * 8;
  if (base < c.n) fetch(c, base, lane, cur);
  for (; base < c.n; base += kKeysPerIter) {
    if (base + kKeysPerIter < c.n) fetch(c, base + kKeysPerIter, lane, nxt);
    const int j0 = base + (lane >> 3), j1 = j0 + 4;
    const bool has0 = j0 < c.n, has1 = j1 < c.n;
    float kk0[16], kk1[16];
    unpack16(cur.k0, kk0);
    unpack16(cur.k1, kk1);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      s0 = fmaf(q[i], kk0[i], s0);
      s1 = fmaf(q[i], kk1[i], s1);
    }
    s0 = group_sum8(s0);
    s1 = group_sum8(s1);
    if (!has0) s0 = -INFINITY;
    if (!has1) s1 = -INFINITY;
    const float mn = fmaxf(m, fmaxf(s0, s1));
    if (mn != -INFINITY) {  // else nothing valid yet in this lane group
      const float corr = exp2f(m - mn);
      const float p0 = exp2f(s0 - mn), p1 = exp2f(s1 - mn);
      lsum = lsum * corr + p0 + p1;
      float vv0[16], vv1[16];
      unpack16(cur.v0, vv0);
      unpack16(cur.v1, vv1);
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = fmaf(acc[i], corr, fmaf(p0, vv0[i], p1 * vv1[i]));
      m = mn;
    }
    cur = nxt;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) s_acc[grp][sub * 16 + i] = acc[i];
  if (sub == 0) {
    s_m[grp] = m;
    s_l[grp] = lsum;
  }
  __syncthreads();
  const int d = threadIdx.x;
  if (d >= 128) return;
  float mx = -INFINITY;
#pragma unroll
  for (int g = 0; g < kGroups; ++g) mx = fmaxf(mx, s_m[g]);
  float tot = 0.f, o = 0.f;
  if (mx != -INFINITY) {
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
      const float w = exp2f(s_m[g] - mx);
      tot += s_l[g] * w;
      o += s_acc[g][d] * w;
    }
  }
  o = tot > 0.f ? o / tot : 0.f;
  a.out[qoff + d] = __float2bfloat16(o);
  if (d == 0) a.lse[((long long)l * a.R + r) * a.H + h] = tot > 0.f ? mx + log2f(tot) : -INFINITY;
}

__global__ void __launch_bounds__(kBwdThreads) mem_attn_bwd_kernel(MemAttnArgs a) {
  constexpr int kGroups = kBwdThreads / 8, kKeysPerIter = kBwdThreads / 4;
  __shared__ float s_dq[kGroups][128];
  const int h = blockIdx.x, r = blockIdx.y, l = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane & 7, grp = warp * 4 + (lane >> 3);
  const RowCtx c = row_ctx(a, l, r, h, sub);
  const long long qoff = (((long long)l * a.R + r) * a.H + h) * 128;
  const float lse2 = a.lse[((long long)l * a.R + r) * a.H + h];

  float q[16], dout[16], o[16];
  load16(a.q + qoff + sub * 16, q);
  load16(a.dout + qoff + sub * 16, dout);
  load16(a.o + qoff + sub * 16, o);
  float dd = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    q[i] *= a.scale_log2;
    dd = fmaf(dout[i], o[i], dd);
  }
  dd = group_sum8(dd);

  float dq[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) dq[i] = 0.f;
  if (lse2 != -INFINITY) {
    // warp-uniform trip count (see forward); no register prefetch here: the
    // backward already holds q, dO and the dq accumulator, and measured
    // faster with 4 resident CTAs an SM than with the prefetch buffers
    for (int base = warp * 8; base < c.n; base += kKeysPerIter) {
      const int j0 = base + (lane >> 3), j1 = j0 + 4;
      const bool has0 = j0 < c.n, has1 = j1 < c.n;
      float k0[16], v0[16], k1[16], v1[16];
      const long long o0 = tok_off(c, has0 ? j0 : base);
      const long long o1 = tok_off(c, has1 ? j1 : base);
      load16(c.kb + o0, k0);
      load16(c.vb + o0, v0);
      load16(c.kb + o1, k1);
      load16(c.vb + o1, v1);
      float s0 = 0.f, s1 = 0.f, dp0 = 0.f, dp1 = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        s0 = fmaf(q[i], k0[i], s0);
        s1 = fmaf(q[i], k1[i], s1);
        dp0 = fmaf(dout[i], v0[i], dp0);
        dp1 = fmaf(dout[i], v1[i], dp1);
      }
      s0 = group_sum8(s0);
      s1 = group_sum8(s1);
      dp0 = group_sum8(dp0);
      dp1 = group_sum8(dp1);
      const float ds0 = has0 ? exp2f(s0 - lse2) * (dp0 - dd) : 0.f;
      const float ds1 = has1 ? exp2f(s1 - lse2) * (dp1 - dd) : 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) dq[i] = fmaf(ds0, k0[i], fmaf(ds1, k1[i], dq[i]));
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) s_dq[grp][sub * 16 + i] = dq[i];
  __syncthreads();
  const int d = threadIdx.x;
  if (d >= 128) return;
  float t = 0.f;
#pragma unroll
  for (int g = 0; g < kGroups; ++g) t += s_dq[g][d];
  a.dq[qoff + d] = t * a.scale;
}

cudaError_t mem_attn_fwd(const MemAttnArgs& a, cudaStream_t stream) {
  if (a.L < 1 || a.R < 1 || a.H < 1 || a.H > 65535 || a.R > 65535 || a.L > 64) return cudaErrorInvalidValue;
  mem_attn_fwd_kernel<<<dim3(a.H, a.R, a.L), kFwdThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t mem_attn_bwd(const MemAttnArgs& a, cudaStream_t stream) {
  if (a.L < 1 || a.R < 1 || a.H < 1 || a.H > 65535 || a.R > 65535 || a.L > 64) return cudaErrorInvalidValue;
  mem_attn_bwd_kernel<<<dim3(a.H, a.R, a.L), kBwdThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace sc
