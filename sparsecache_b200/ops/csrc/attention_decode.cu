// Split-K decode / verify attention over a paged layer cache, merged through
// distributed shared memory inside a thread-block cluster (and, for few kv
// heads or long contexts, across several clusters per kv head).
//
// The query block is M <= 8 consecutive new tokens (M = 1 for greedy decode,
// M = gamma + 1 for the batched speculative verifier) at positions
// *pos .. *pos + M - 1; row m sees keys [0, *pos + m].  The position lives in
// device memory so a captured CUDA graph replays the same launch every step.
//
// Grid (S * R, n_kv_heads, ceil(M * G / 4)), cluster (S, 1, 1): the S CTAs of
// a cluster split a key range of one kv head; R clusters per kv head split
// the keys further.  K/V rows are read once per kv head for the 4 query
// vectors of a z-block (GQA packing) straight into registers; each CTA leaves
// its partial (max, sum, o[128]) in shared memory, the cluster merges them
// over DSMEM, and with R > 1 the last CTA of the kv head merges the clusters'
// partials from a small global workspace (atomic ticket, reset by that CTA).
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
constexpr int kSub = 64;      // minimum keys per CTA for 16-CTA clusters
constexpr int kMaxQV = 64;    // M * G (M <= 8 rows, G <= 8 query heads per kv head)
constexpr int kMaxRows = 8;   // largest query block M
constexpr int kMaxOuter = 16; // clusters per kv head (second split level)

}  // namespace

// ---------------------------------------------------------------------------
// Register-resident decode attention: no shared-memory staging and no block
// barrier inside the key loop.  Grid (S * R, n_kv_heads, ceil(QV / 4)):
// z-block z handles query vectors 4z .. 4z + 3 (a query vector = one row m and
// one query head of the kv head's group), so each vector's arithmetic is the
// same whatever M is (decode M = 1 and batched verification M <= 8 give
// bit-identical rows).  In a CTA, lane group g (8 lanes, 16 dims each) of warp
// w takes keys base + g and base + 4 + g of base = k_begin + 8w, + 64, ...;
// the next pair's K/V rows are loaded into registers while the current pair
// is scored, so the loop is one load latency per 64 keys.  Per vector, the
// lane group keeps an online softmax (max, sum, 16-dim accumulator); the 4
// groups of a warp merge through shuffles, the 8 warps through shared memory,
// and the CTAs of the cluster through DSMEM.
constexpr int kRQ = 4;  // query vectors per z-block

// 2^x by the MUFU ex2 instruction (flush-to-zero; 2^-inf = +0): the key
// loop's three exponentials per key pair and vector are its costliest
// instructions, and a softmax weight needs no more than this precision
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct RegSmem {
  float wo[kWarps][kRQ][128];  // per-warp partial accumulators
  float wm[kWarps][kRQ], wl[kWarps][kRQ];
  float o[kRQ][128];           // this CTA's partial (DSMEM-visible)
  float m[kRQ], l[kRQ];
};

__device__ __forceinline__ void reg_load16(const __nv_bfloat16* p, uint4 (&u)[2]) {
  u[0] = __ldg(reinterpret_cast<const uint4*>(p));
  u[1] = __ldg(reinterpret_cast<const uint4*>(p) + 1);
}

__device__ __forceinline__ void reg_unpack16(const uint4 (&u)[2], float (&x)[16]) {
  const unsigned w[8] = {u[0].x, u[0].y, u[0].z, u[0].w, u[1].x, u[1].y, u[1].z, u[1].w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

__global__ void __launch_bounds__(kThreads)
    attention_decode_reg_kernel(AttnDecodeArgs a, int chunk, int outer) {
  __shared__ RegSmem sm;
  cg::cluster_group cluster = cg::this_cluster();
  const int G = a.n_heads / a.n_kv_heads;
  const int QV = a.M * G;
  const int S = gridDim.x / outer;
  const int split = blockIdx.x % S;
  const int cidx = blockIdx.x / S;
  const int kvh = blockIdx.y;
  // batched sequences (pos_rows): z = sequence * z-blocks + z-block, one row
  // per sequence, its own position and cache (seq_stride elements apart)
  const int nzb = (QV + kRQ - 1) / kRQ;
  const int seq = a.pos_rows != nullptr ? (int)blockIdx.z / nzb : 0;
  const int qv0 = (a.pos_rows != nullptr ? (int)blockIdx.z % nzb : (int)blockIdx.z) * kRQ;
  const __nv_bfloat16* qbase = a.q + (size_t)seq * a.n_heads * 128;
  __nv_bfloat16* obase = a.out + (size_t)seq * a.n_heads * 128;
  const int nq = min(kRQ, QV - qv0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sub = lane & 7, grp = lane >> 3;
  const float sl2 = a.scale * 1.4426950408889634f;
  const size_t seq_off = (size_t)seq * (size_t)a.seq_stride;
  const __nv_bfloat16* kb = a.k_cache + seq_off + (size_t)kvh * a.cache_cap * 128 + sub * 16;
  const __nv_bfloat16* vb = a.v_cache + seq_off + (size_t)kvh * a.cache_cap * 128 + sub * 16;
  const int page_mask = (1 << a.page_shift) - 1;
  pdl_wait();  // q and the new rows come from the QKV kernel right before
  pdl_launch_dependents();
  if (warp == kWarps - 1 && (a.pf_bytes[0] > 0 || a.pf_bytes[1] > 0)) {
    const int cta = ((int)blockIdx.z * (int)gridDim.y + (int)blockIdx.y) * (int)gridDim.x + (int)blockIdx.x;
    prefetch_l2_share(a.pf_ptr, a.pf_bytes, 2, cta, (int)(gridDim.x * gridDim.y * gridDim.z), lane);
  }
  const int n_keys = a.pos_rows != nullptr ? a.pos_rows[seq] + 1 : (a.n_virtual != nullptr ? *a.n_virtual : *a.pos + a.M);
  const int pos0 = n_keys - a.M;
  const int k_begin = blockIdx.x * chunk;
  const int k_end = min(n_keys, k_begin + chunk);
  auto row_off = [&](int v) -> size_t {
    const int p = a.page_table != nullptr ? (a.page_table[v >> a.page_shift] << a.page_shift) + (v & page_mask) : v;
    return (size_t)p * 128;
  };

  float q[kRQ][16];
  int last[kRQ];  // last visible key of each vector (its row's position)
#pragma unroll
  for (int i = 0; i < kRQ; ++i) {
    const int qv = qv0 + (i < nq ? i : 0);
    const int m = qv / G, gi = qv % G;
    uint4 u[2];
    reg_load16(qbase + (size_t)m * a.n_heads * 128 + (kvh * G + gi) * 128 + sub * 16, u);
    reg_unpack16(u, q[i]);
#pragma unroll
    for (int e = 0; e < 16; ++e) q[i][e] *= sl2;
    last[i] = i < nq ? pos0 + m : -1;
  }
  float mx[kRQ], ls[kRQ], acc[kRQ][16];
#pragma unroll
  for (int i = 0; i < kRQ; ++i) {
    mx[i] = -INFINITY;
    ls[i] = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[i][e] = 0.f;
  }

  // key loop: warp-uniform trip count (the 8-lane shuffles need all 32 lanes)
  uint4 ck0[2], cv0[2], ck1[2], cv1[2], nk0[2], nv0[2], nk1[2], nv1[2];
  int base = k_begin + warp * 8;
  auto fetch = [&](int b, uint4 (&k0)[2], uint4 (&v0)[2], uint4 (&k1)[2], uint4 (&v1)[2]) {
    const int j0 = b + grp, j1 = j0 + 4;
    const size_t o0 = row_off(j0 < k_end ? j0 : b), o1 = row_off(j1 < k_end ? j1 : b);
    reg_load16(kb + o0, k0);
    reg_load16(vb + o0, v0);
    reg_load16(kb + o1, k1);
    reg_load16(vb + o1, v1);
  };
  if (base < k_end) fetch(base, ck0, cv0, ck1, cv1);
  for (; base < k_end; base += kWarps * 8) {
    if (base + kWarps * 8 < k_end) fetch(base + kWarps * 8, nk0, nv0, nk1, nv1);
    const int j0 = base + grp, j1 = j0 + 4;
    float s0[kRQ], s1[kRQ];
    {
      float kf0[16], kf1[16];
      reg_unpack16(ck0, kf0);
      reg_unpack16(ck1, kf1);
#pragma unroll
      for (int i = 0; i < kRQ; ++i) {
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          a0 = fmaf(q[i][e], kf0[e], a0);
          a1 = fmaf(q[i][e], kf1[e], a1);
        }
        s0[i] = a0;
        s1[i] = a1;
      }
    }
#pragma unroll
    for (int i = 0; i < kRQ; ++i) {
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) {
        s0[i] += __shfl_xor_sync(0xffffffffu, s0[i], o);
        s1[i] += __shfl_xor_sync(0xffffffffu, s1[i], o);
      }
      if (j0 >= k_end || j0 > last[i]) s0[i] = -INFINITY;
      if (j1 >= k_end || j1 > last[i]) s1[i] = -INFINITY;
    }
    // online softmax: the (corr, p0, p1) of every vector, then one pass over the dims
    float corr[kRQ], p0[kRQ], p1[kRQ];
#pragma unroll
    for (int i = 0; i < kRQ; ++i) {
      const float mn = fmaxf(mx[i], fmaxf(s0[i], s1[i]));
      if (mn == -INFINITY) {  // nothing visible yet for this vector
        corr[i] = 1.f, p0[i] = 0.f, p1[i] = 0.f;
      } else {
        corr[i] = ex2_fast(mx[i] - mn);
        p0[i] = ex2_fast(s0[i] - mn);
        p1[i] = ex2_fast(s1[i] - mn);
        mx[i] = mn;
      }
      ls[i] = ls[i] * corr[i] + p0[i] + p1[i];
    }
    {
      const unsigned w0[8] = {cv0[0].x, cv0[0].y, cv0[0].z, cv0[0].w, cv0[1].x, cv0[1].y, cv0[1].z, cv0[1].w};
      const unsigned w1[8] = {cv1[0].x, cv1[0].y, cv1[0].z, cv1[0].w, cv1[1].x, cv1[1].y, cv1[1].z, cv1[1].w};
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        const float2 va = unpack_bf16x2(w0[h]), vb = unpack_bf16x2(w1[h]);
#pragma unroll
        for (int i = 0; i < kRQ; ++i) {
          acc[i][2 * h] = fmaf(acc[i][2 * h], corr[i], fmaf(p0[i], va.x, p1[i] * vb.x));
          acc[i][2 * h + 1] = fmaf(acc[i][2 * h + 1], corr[i], fmaf(p0[i], va.y, p1[i] * vb.y));
        }
      }
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      ck0[c] = nk0[c]; cv0[c] = nv0[c]; ck1[c] = nk1[c]; cv1[c] = nv1[c];
    }
  }

  // merge the 4 lane groups of the warp (lanes with the same dims: xor 8, 16)
#pragma unroll
  for (int i = 0; i < kRQ; ++i) {
    float wm = mx[i];
    wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, 8));
    wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, 16));
    const float w = (mx[i] == -INFINITY) ? 0.f : exp2f(mx[i] - wm);
    float l = ls[i] * w;
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      float x = acc[i][e] * w;
      x += __shfl_xor_sync(0xffffffffu, x, 8);
      x += __shfl_xor_sync(0xffffffffu, x, 16);
      if (grp == 0) sm.wo[warp][i][sub * 16 + e] = x;
    }
    if (lane == 0) {
      sm.wm[warp][i] = wm;
      sm.wl[warp][i] = l;
    }
  }
  __syncthreads();
  // merge the 8 warps (fixed order) into this CTA's partial
  for (int idx = tid; idx < kRQ * 128; idx += kThreads) {
    const int i = idx >> 7, d = idx & 127;
    float gm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) gm = fmaxf(gm, sm.wm[w][i]);
    float o = 0.f, l = 0.f;
    if (gm != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float c = sm.wm[w][i] == -INFINITY ? 0.f : exp2f(sm.wm[w][i] - gm);
        o += sm.wo[w][i][d] * c;
        l += sm.wl[w][i] * c;
      }
    }
    sm.o[i][d] = o;
    if (d == 0) {
      sm.m[i] = gm;
      sm.l[i] = l;
    }
  }

  // ---- merge the S partials of this kv head through DSMEM ----
  cluster.sync();
  for (int idx = split * kThreads + tid; idx < nq * 128; idx += S * kThreads) {
    const int i = idx >> 7, d = idx & 127;
    float mr[16], lr[16], orr[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      if (r < S) {
        const RegSmem* peer = cluster.map_shared_rank(&sm, r);
        mr[r] = peer->m[i];
        lr[r] = peer->l[i];
        orr[r] = peer->o[i][d];
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
    const int qv = qv0 + i;
    if (outer == 1) {
      const int m = qv / G, gi = qv % G;
      obase[(size_t)m * a.n_heads * 128 + (kvh * G + gi) * 128 + d] =
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
  __shared__ unsigned s_ticket;
  unsigned* counter = a.counters + kvh * (kMaxQV / kRQ) + blockIdx.z;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(counter, 1u);
  __syncthreads();
  if (s_ticket != (unsigned)(S * outer - 1)) return;
  __threadfence();
  for (int idx = tid; idx < nq * 128; idx += kThreads) {
    const int qv = qv0 + (idx >> 7), d = idx & 127;
    const float* b0 = a.ws + ((size_t)kvh * kMaxOuter * kMaxQV + qv) * 130;
    float gmax = -INFINITY;
    for (int c = 0; c < outer; ++c) gmax = fmaxf(gmax, __ldcg(b0 + (size_t)c * kMaxQV * 130));
    float num = 0.f, den = 0.f;
    if (gmax != -INFINITY) {
      for (int c = 0; c < outer; ++c) {
        const float* pc = b0 + (size_t)c * kMaxQV * 130;
        const float mc = __ldcg(pc);
        if (mc == -INFINITY) continue;
        const float w = exp2f(mc - gmax);
        num += w * __ldcg(pc + 2 + d);
        den += w * __ldcg(pc + 1);
      }
    }
    const int m = qv / G, gi = qv % G;
    obase[(size_t)m * a.n_heads * 128 + (kvh * G + gi) * 128 + d] =
        __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
  }
  if (tid == 0) *counter = 0u;
}

// Launch geometry (measured on B200, one query row, 8/4/1 kv heads, 2k-18k
// keys): up to ~512 keys per CTA a single cluster per kv head is fastest (8
// CTAs with 8 kv heads, 16 with fewer); beyond that, 4-CTA clusters with
// several clusters per kv head (about 128 CTAs in all, at least 128 keys a
// CTA) beat larger clusters, which schedule poorly at one CTA per SM.  Both
// depend on the capacity and the head count only, never on M.
int attention_decode_cluster(int cache_cap, int n_kv_heads) {
  const int s1 = n_kv_heads >= 8 ? 8 : 16;
  return cache_cap / s1 <= 512 ? s1 : 4;
}

int attention_decode_outer(int cache_cap, int n_kv_heads, int cluster, int num_sms) {
  if (cluster != 4) return 1;
  int r = (num_sms < 128 ? num_sms : 128) / (cluster * n_kv_heads);
  const int by_keys = cache_cap / (cluster * 128);
  if (r > by_keys) r = by_keys;
  if (r > kMaxOuter) r = kMaxOuter;
  return r < 1 ? 1 : r;
}

cudaError_t attention_decode(const AttnDecodeArgs& a, cudaStream_t stream) {
  const int G = a.n_heads / a.n_kv_heads;
  if (a.M < 1 || a.M * G > kMaxQV) return cudaErrorInvalidValue;
  const int S = a.splits;
  if (S < 1 || S > 16) return cudaErrorInvalidValue;
  if (a.pos_rows != nullptr && (a.M != 1 || a.n_seq < 1 || a.page_table != nullptr)) return cudaErrorInvalidValue;
  if (a.key_cap < 0) return cudaErrorInvalidValue;
  const int cap = a.key_cap > 0 ? a.key_cap : a.cache_cap;  // keys the geometry is sized for
  int outer = 1;
  if (a.ws != nullptr && a.counters != nullptr && a.pos_rows == nullptr) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    outer = a.outer > 0 ? a.outer : attention_decode_outer(cap, a.n_kv_heads, S, sms);
    if (outer > kMaxOuter) return cudaErrorInvalidValue;
  }
  // keys per CTA: the capacity (+ the largest row block) split evenly over
  // all S * outer CTAs, rounded to 16 keys; independent of M so a row sees
  // the same split boundaries (and the same rounding) in decode and in
  // batched verification
  const int total = S * outer;
  int chunk = (cap + kMaxRows + total - 1) / total;
  chunk = (chunk + 15) / 16 * 16;
  const int qv = a.M * G;
  auto kern = attention_decode_reg_kernel;
  {
    static bool nonportable_done = false;
    if (!nonportable_done) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      nonportable_done = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S * outer, a.n_kv_heads, ((qv + kRQ - 1) / kRQ) * (a.pos_rows != nullptr ? a.n_seq : 1));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
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
