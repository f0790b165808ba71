// LEGACY (kept only to A/B-measure the tcgen05 kernel in attention_prefill.cu):
// flash attention over a paged layer cache with per-row position vectors.
//
//   out[r, h, :] = softmax_j( q[r,h,:] . k[j,kvh(h),:] * scale | kpos[j] <= qpos[r] ) v[j,kvh,:]
//
// One kernel covers both prefill flavours of the reference:
//   * full causal prefill (qpos = kpos = arange) - HF SDPA is_causal=True
//     (modeling.py:196-206, reuse_cacheblend_pipeline.py:557-567)
//   * CacheBlend selective recompute: the query rows are an arbitrary sorted
//     subset of positions and the keys are the whole composed cache; the
//     reference materialises a dense [A, T] boolean mask
//     (modeling.py:345-369, reuse_cacheblend_pipeline.py:464-488); here the
//     predicate kpos[j] <= qpos[r] is evaluated per tile from two int vectors.
// Query rows can be gathered through q_rows (row r reads q[q_rows[r]]), so
// the check layer attends only its active rows without a separate gather.
// kpos must be non-decreasing (it is: cache slots are laid out in position
// order), which lets every CTA stop at the last key any of its rows can see.
//
// Tiles: 64 query rows x 64 keys, head_dim 128, 4 warps of 16 rows, bf16
// m16n8k16 tensor-core MMAs with fp32 accumulation, online softmax in exp2
// space, K/V double-buffered with cp.async into XOR-swizzled shared memory.
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace legacy_mma {

constexpr int kBM = 64;
constexpr int kBN = 64;
constexpr int kD = 128;
constexpr int kThreads = 128;
constexpr int kRowBytes = kD * 2;  // 256 B = 16 chunks of 16 B

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return row * kRowBytes + ((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Load a [64 rows x 128] bf16 tile (rows row0.., clipped at nrows) into
// swizzled smem.  Each of the 128 threads moves 8 chunks of 16 B.
__device__ __forceinline__ void load_tile(uint32_t sbase, const __nv_bfloat16* g, size_t row_stride,
                                          int row0, int nrows) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = tid + i * kThreads;  // 0..1023
    const int r = idx >> 4, c = idx & 15;
    const int grow = row0 + r;
    const bool ok = grow < nrows;
    const __nv_bfloat16* src = g + (size_t)(ok ? grow : 0) * row_stride + c * 8;
    cp_async16(sbase + swz(r, c), src, ok);
  }
}

}  // namespace legacy_mma
using namespace legacy_mma;

__global__ void __launch_bounds__(kThreads, 2)
    attention_prefill_mma_kernel(AttnPrefillArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + kBM * kRowBytes;       // 2 stages
  const uint32_t sV = sK + 2 * kBN * kRowBytes;   // 2 stages
  __shared__ int s_qpos[kBM];
  __shared__ int s_qmin, s_qmax, s_nkeys;

  const int h = blockIdx.y;
  const int kvh = h / (p.n_heads / p.n_kv_heads);
  const int r0 = blockIdx.x * kBM;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- query positions of this tile; bound of visible keys ----
  if (tid < kBM) {
    const int r = r0 + tid;
    s_qpos[tid] = (r < p.n_rows) ? p.qpos[r] : -1;
  }
  __syncthreads();
  if (tid == 0) {
    int mn = 0x7fffffff, mx = -1;
    for (int i = 0; i < kBM; ++i) {
      const int q = s_qpos[i];
      if (q >= 0) { mn = min(mn, q); mx = max(mx, q); }
    }
    // number of keys with kpos <= mx (kpos non-decreasing)
    int lo = 0, hi = p.n_keys;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      const int kp = p.kpos ? p.kpos[mid] : mid;
      if (kp <= mx) lo = mid + 1; else hi = mid;
    }
    s_qmin = mn; s_qmax = mx; s_nkeys = (mx < 0) ? 0 : lo;
  }

  // ---- Q tile (gathered rows) ----
  {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + i * kThreads;
      const int r = idx >> 4, c = idx & 15;
      const int grow = r0 + r;
      const bool ok = grow < p.n_rows;
      const int src_row = ok ? (p.q_rows ? p.q_rows[grow] : grow) : 0;
      const __nv_bfloat16* src = p.q + (size_t)src_row * p.ldq + h * kD + c * 8;
      cp_async16(sQ + swz(r, c), src, ok);
    }
    cp_async_commit();
  }
  __syncthreads();
  const int n_keys = s_nkeys;
  const int qmin = s_qmin;
  const int n_tiles = (n_keys + kBN - 1) / kBN;

  const __nv_bfloat16* kbase = p.k_cache + (size_t)kvh * p.cache_cap * kD;
  const __nv_bfloat16* vbase = p.v_cache + (size_t)kvh * p.cache_cap * kD;
  if (n_tiles > 0) {
    load_tile(sK, kbase, kD, 0, n_keys);
    load_tile(sV, vbase, kD, 0, n_keys);
  }
  cp_async_commit();

  // Q fragments
  cp_async_wait<1>();
  __syncthreads();
  uint32_t qf[8][4];
  {
    const int mi = lane >> 3, rr = lane & 7;
    const int row = warp * 16 + (mi & 1) * 8 + rr;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int chunk = kk * 2 + (mi >> 1);
      ldsm_x4(sQ + swz(row, chunk), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }

  const int g = lane >> 2, t4 = lane & 3;
  const int my_row0 = warp * 16 + g;  // tile-local rows my_row0 and my_row0 + 8
  const int qp0 = s_qpos[my_row0], qp1 = s_qpos[my_row0 + 8];
  const float sl2 = p.scale * 1.4426950408889634f;

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int it = 0; it < n_tiles; ++it) {
    const int stage = it & 1;
    if (it + 1 < n_tiles) {
      const int ns = stage ^ 1;
      load_tile(sK + ns * kBN * kRowBytes, kbase, kD, (it + 1) * kBN, n_keys);
      load_tile(sV + ns * kBN * kRowBytes, vbase, kD, (it + 1) * kBN, n_keys);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t k_s = sK + stage * kBN * kRowBytes;
    const uint32_t v_s = sV + stage * kBN * kRowBytes;

    // S = Q K^T : 16 x 64 per warp -> 8 n-tiles of 8 keys
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        // two n-tiles (16 keys) x 16 dims per ldmatrix.x4
        const int mi = lane >> 3, rr = lane & 7;
        const int key = jp * 16 + (mi >> 1) * 8 + rr;
        const int chunk = kk * 2 + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(k_s + swz(key, chunk), b0, b1, b2, b3);
        mma_bf16(s[2 * jp], qf[kk], b0, b1);
        mma_bf16(s[2 * jp + 1], qf[kk], b2, b3);
      }
    }

    // masking
    const int key0 = it * kBN;
    const int last_key = min(key0 + kBN, n_keys) - 1;
    const int last_kpos = p.kpos ? p.kpos[last_key] : last_key;
    const bool need_mask = (key0 + kBN > n_keys) || (last_kpos > qmin);
    if (need_mask) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = key0 + j * 8 + 2 * t4 + e;
          int kp = 0x7fffffff;
          if (key < n_keys) kp = p.kpos ? p.kpos[key] : key;
          if (kp > qp0) s[j][e] = -INFINITY;
          if (kp > qp1) s[j][2 + e] = -INFINITY;
        }
      }
    }

    // online softmax (rows g and g+8 of this warp; each row shared by 4 lanes)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0 * sl2), mn1 = fmaxf(m1, mx1 * sl2);
    const float base0 = (mn0 == -INFINITY) ? 0.f : mn0;
    const float base1 = (mn1 == -INFINITY) ? 0.f : mn1;
    const float c0 = exp2f(m0 - base0), c1 = exp2f(m1 - base1);
    m0 = mn0; m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pf[4][4];  // P as A fragments for 4 k-steps of 16 keys
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = exp2f(s[j][0] * sl2 - base0);
      const float p1 = exp2f(s[j][1] * sl2 - base0);
      const float p2 = exp2f(s[j][2] * sl2 - base1);
      const float p3 = exp2f(s[j][3] * sl2 - base1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      const int kk = j >> 1, hi = j & 1;
      pf[kk][hi * 2 + 0] = pack_bf16x2(p0, p1);
      pf[kk][hi * 2 + 1] = pack_bf16x2(p2, p3);
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= c0; o[i][1] *= c0;
      o[i][2] *= c1; o[i][3] *= c1;
    }

    // O += P V : V tile [64 keys x 128 dims], B fragments via ldmatrix.trans
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        // two n-tiles of 8 dims (16 dims) x 16 keys
        const int mi = lane >> 3, rr = lane & 7;
        const int key = kk * 16 + (mi & 1) * 8 + rr;
        const int chunk = dp * 2 + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(v_s + swz(key, chunk), b0, b1, b2, b3);
        mma_bf16(o[2 * dp], pf[kk], b0, b1);
        mma_bf16(o[2 * dp + 1], pf[kk], b2, b3);
      }
    }
    __syncthreads();
  }

  // finalize: reduce row sums across the 4 lanes sharing a row
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int row_a = r0 + my_row0, row_b = row_a + 8;
#pragma unroll
  for (int dn = 0; dn < 16; ++dn) {
    const int d = dn * 8 + 2 * t4;
    if (row_a < p.n_rows) {
      *reinterpret_cast<uint32_t*>(p.out + (size_t)row_a * p.ldo + h * kD + d) =
          pack_bf16x2(o[dn][0] * inv0, o[dn][1] * inv0);
    }
    if (row_b < p.n_rows) {
      *reinterpret_cast<uint32_t*>(p.out + (size_t)row_b * p.ldo + h * kD + d) =
          pack_bf16x2(o[dn][2] * inv1, o[dn][3] * inv1);
    }
  }
}

cudaError_t attention_prefill_mma(const AttnPrefillArgs& p, cudaStream_t stream) {
  if (p.head_dim != kD || p.n_rows <= 0) return p.n_rows == 0 ? cudaSuccess : cudaErrorInvalidValue;
  const int smem = kBM * kRowBytes + 4 * kBN * kRowBytes;  // 80 KB
  ensure_smem_attr(attention_prefill_mma_kernel, smem);
  dim3 grid((p.n_rows + kBM - 1) / kBM, p.n_heads);
  attention_prefill_mma_kernel<<<grid, kThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace sc
