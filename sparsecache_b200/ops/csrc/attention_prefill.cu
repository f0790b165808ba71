// Flash attention over a layer cache with per-row position vectors, on the
// 5th-generation tensor cores (tcgen05.mma, accumulators in TMEM, K/V tiles
// by TMA).
//
//   out[r, h, :] = softmax_j( q[r,h,:] . k[j,kvh(h),:] * scale | kpos[j] <= qpos[r] ) v[j,kvh,:]
//
// One kernel covers both prefill flavours of the reference:
//   * full causal prefill (qpos = kpos = arange) - HF SDPA is_causal=True
//     (src/sparsecache/modeling.py:196-206, reuse_cacheblend_pipeline.py:557-567)
//   * CacheBlend selective recompute: the query rows are an arbitrary sorted
//     subset of positions and the keys are the whole composed cache; the
//     reference materialises a dense [A, T] boolean mask
//     (src/sparsecache/modeling.py:345-369, reuse_cacheblend_pipeline.py:464-488).
//     Here kpos is non-decreasing (cache slots are in position order), so row
//     r sees exactly the key prefix [0, nvis[r]) with nvis[r] = #{j : kpos[j]
//     <= qpos[r]}: one binary search per row replaces the mask.
// Query rows can be gathered through q_rows (row r reads q[q_rows[r]]), so
// the check layer attends only its active rows without a separate gather.
//
// CTA = one kv head and 128 / G query positions, where G query heads share
// the kv head: the 128 rows of the tcgen05 tile are (query head g, position
// i) pairs, so every K/V tile is loaded once for the whole GQA group (a
// kv-head-major packing; K/V traffic from L2 drops by G against one CTA per
// query head).  192 threads:
//   warp 0     TMA producer: K and V tiles of 128 keys (two 128-byte-swizzled
//              boxes of 64 dims each) into a 2-deep ring; rows past n_keys
//              are zero-filled by the tensor map, never read from the cache.
//   warp 1     MMA issuer and TMEM owner:
//                S_j = Q K_j^T   M=128 N=128 K=128 -> TMEM S[j & 1] (fp32)
//                O  += P_j V_j   M=128 N=128 K=128 -> TMEM O       (fp32)
//              Q and P_j are K-major operands in shared memory; V_j is the
//              MN-major B operand straight from its [keys][dims] tile.  QK of
//              tile j+1 is issued before PV of tile j, so the tensor core
//              works on the next scores while the softmax of this tile runs.
//   warps 2-5  softmax + epilogue, one tile row per thread (its TMEM lane):
//              tcgen05.ld the 128 scores, mask by nvis, online softmax in
//              exp2 space, P_j as bf16 into the swizzled K-major smem tile,
//              then one arrive.  The running max is rescaled lazily: O in
//              TMEM is rescaled (tcgen05.ld/st) only when a row max grows by
//              more than 2^8, so P stays <= 256 and most tiles touch O not at
//              all.  The epilogue reads O once, divides by the row sum and
//              stores bf16.
// TMEM: S[0] cols 0-127, S[1] cols 128-255, O cols 256-383 (512 allocated).
// Shared memory: Q 32 KB + 2 x (K 32 KB + V 32 KB) + 2 x P 32 KB = 224 KB.
// Every wait is bounded; an expired wait records a status code and the CTA
// winds down (TMA loads in flight are drained, TMEM is freed).  No cluster,
// no multicast: safe inside multi-GPU programs.
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {

constexpr int kD = 128;
constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kStages = 2;
constexpr int kThreads = 192;
constexpr float kRescaleLog2 = 8.0f;

constexpr int kQBytes = kBM * kD * 2;      // two 16 KB k-blocks (dims 0-63, 64-127)
constexpr int kKVBytes = kBN * kD * 2;     // two 16 KB halves (dims 0-63, 64-127)
constexpr int kHalfBytes = kBN * 128;      // one 128-key x 128-byte half
constexpr int kPBytes = kBM * kBN * 2;     // two 16 KB k-blocks (keys 0-63, 64-127)
constexpr int kPBlock = kBM * 128;
constexpr int kOffK = kQBytes;
constexpr int kOffV = kOffK + kStages * kKVBytes;
constexpr int kOffP = kOffV + kStages * kKVBytes;
constexpr int kOffBars = kOffP + 2 * kPBytes;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 256;

struct alignas(8) AttnBars {
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done;
  uint64_t o_final;
  uint64_t drain;
  uint32_t tmem_base;
  int max_vis;
};
static_assert(sizeof(AttnBars) <= 256, "barrier block");
constexpr int kNeedBytes = kOffBars + 256;  // from the 1024-aligned base
// the largest opt-in dynamic shared memory of a CTA; the base is aligned up
// to 1024 inside it, which leaves kSmemBytes - kNeedBytes bytes of slack
constexpr int kSmemBytes = 232448;
static_assert(kNeedBytes <= kSmemBytes, "shared-memory plan");

// Optional debug timeline of one CTA (kv head 0, the first scheduled row tile):
// trace[tile * 10 + event] = globaltimer ns; tile 63 holds kernel-level events.
__device__ __forceinline__ void trace_at(const AttnPrefillArgs& p, int tile, int event) {
  if (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && tile < 64) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    p.trace[tile * 10 + event] = t;
  }
}

// 2^x by the MUFU ex2 instruction (flush-to-zero; 2^-inf = +0)
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// byte offset of 16-byte chunk c of row r in a K-major, 128-byte-swizzled
// block of 128-byte rows (the layout TMA SWIZZLE_128B writes)
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    attention_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                                const __grid_constant__ CUtensorMap tm_v, AttnPrefillArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  AttnBars* bars = reinterpret_cast<AttnBars*>(smem + kOffBars);
  int* status = p.status;
  // the swizzled operand tiles need a 1024-byte aligned base; the dynamic
  // window is aligned that way on sm_100, and if it ever were not by enough,
  // the kernel reports it and does nothing rather than overrun shared memory
  if ((smem - smem_raw) + kNeedBytes > kSmemBytes) {
    if (threadIdx.x == 0) report_status(status, kStatusBadArgument);
    return;
  }

  const int warp = warp_id();
  const int lane = lane_id();
  const int kvh = blockIdx.x;
  const int G = p.n_heads / p.n_kv_heads;  // query heads per kv head (divides 128)
  const int span = kBM / G;                // query positions per CTA
  const int n_row_tiles = gridDim.y;
  const int r0 = (n_row_tiles - 1 - (int)blockIdx.y) * span;  // longest row tiles first

  if (threadIdx.x == 0) {
    trace_at(p, 63, 0);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_full[b], 128);
    }
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->o_final, 1);
    mbar_init(&bars->drain, 1);
    bars->max_vis = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  __syncthreads();
  // q, the positions and the new K/V rows come from the previous kernels
  pdl_wait();
  pdl_launch_dependents();

  // ---- softmax warps: stage the (gathered) Q tile, find each row's visible prefix ----
  // tile row = TMEM lane = warp quarter * 32 + lane; row -> (query head
  // kvh * G + row / span, position r0 + row % span)
  const int quarter = warp & 3;  // TMEM lane quarter this warp may access
  const int row = quarter * 32 + lane;
  const int head = kvh * G + row / span;
  const int g = r0 + row % span;  // query row index of this tile row
  int nvis = 0;
  if (warp >= 2) {
    uint8_t* sq = smem;
    int qp = -1;
    if (g < p.n_rows) {
      qp = p.qpos[g];
      const int src = p.q_rows ? p.q_rows[g] : g;
      const uint4* qsrc = reinterpret_cast<const uint4*>(p.q + (size_t)src * p.ldq + (size_t)head * kD);
#pragma unroll
      for (int c = 0; c < 16; ++c)
        *reinterpret_cast<uint4*>(sq + (c >> 3) * (kBM * 128) + sw128(row, c & 7)) = qsrc[c];
    } else {
#pragma unroll
      for (int c = 0; c < 16; ++c)
        *reinterpret_cast<uint4*>(sq + (c >> 3) * (kBM * 128) + sw128(row, c & 7)) = make_uint4(0, 0, 0, 0);
    }
    if (qp >= 0) {
      if (p.kpos == nullptr) {
        nvis = qp + 1 < p.n_keys ? qp + 1 : p.n_keys;
      } else {
        int lo = 0, hi = p.n_keys;  // first key with kpos > qp
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (p.kpos[mid] <= qp) lo = mid + 1; else hi = mid;
        }
        nvis = lo;
      }
    }
    fence_proxy_async_smem();  // Q written by threads, read by the tensor core
    const int wmax = __reduce_max_sync(0xffffffffu, nvis);
    if (lane == 0) atomicMax(&bars->max_vis, wmax);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  // key tiles of the row tile, and this CTA's share of them (key split z of
  // gridDim.z); below, j counts this CTA's tiles and t0 + j is the key tile
  const int n_tiles_all = (bars->max_vis + kBN - 1) / kBN;
  const int t0 = (int)blockIdx.z * n_tiles_all / (int)gridDim.z;
  const int n_tiles = ((int)blockIdx.z + 1) * n_tiles_all / (int)gridDim.z - t0;
  if (threadIdx.x == 0) trace_at(p, 63, 1);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int k_last[kStages], v_last[kStages];
      for (int s = 0; s < kStages; ++s) k_last[s] = v_last[s] = -1;
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (uint32_t)(j / kStages) & 1u;
        uint8_t* sk = smem + kOffK + s * kKVBytes;
        uint8_t* sv = smem + kOffV + s * kKVBytes;
        if (!mbar_wait(&bars->k_empty[s], ph ^ 1u, status, kStatusTimeoutSmemEmpty)) break;
        mbar_arrive_expect_tx(&bars->k_full[s], kKVBytes);
        tma_load_3d(sk, &tm_k, &bars->k_full[s], 0, (t0 + j) * kBN, kvh);
        tma_load_3d(sk + kHalfBytes, &tm_k, &bars->k_full[s], 64, (t0 + j) * kBN, kvh);
        trace_at(p, j, 0);
        k_last[s] = (int)ph;
        if (!mbar_wait(&bars->v_empty[s], ph ^ 1u, status, kStatusTimeoutSmemEmpty)) break;
        mbar_arrive_expect_tx(&bars->v_full[s], kKVBytes);
        tma_load_3d(sv, &tm_v, &bars->v_full[s], 0, (t0 + j) * kBN, kvh);
        tma_load_3d(sv + kHalfBytes, &tm_v, &bars->v_full[s], 64, (t0 + j) * kBN, kvh);
        trace_at(p, j, 1);
        v_last[s] = (int)ph;
      }
      // every TMA load issued must land before the CTA exits
      for (int s = 0; s < kStages; ++s) {
        if (k_last[s] >= 0) mbar_wait(&bars->k_full[s], (uint32_t)k_last[s], status, kStatusTimeoutDrain);
        if (v_last[s] >= 0) mbar_wait(&bars->v_full[s], (uint32_t)v_last[s], status, kStatusTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16(kBM, kBN);
      constexpr uint32_t idesc_pv = make_idesc_bf16(kBM, kD, /*b_mn_major=*/true);
      const uint32_t sq = smem_u32(smem);
      bool ok = true;
      auto issue_qk = [&](int j) -> bool {
        const int s = j % kStages;
        if (!mbar_wait(&bars->k_full[s], (uint32_t)(j / kStages) & 1u, status, kStatusTimeoutTmaFull))
          return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + kOffK + s * kKVBytes);
        const uint32_t d = tmem_base + (uint32_t)(j & 1) * kBN;
#pragma unroll
        for (int t = 0; t < kD / 16; ++t) {
          const uint64_t ad = make_desc_kmajor_sw128(sq + (t >> 2) * (kBM * 128) + (t & 3) * 32);
          const uint64_t bd = make_desc_kmajor_sw128(sk + (t >> 2) * kHalfBytes + (t & 3) * 32);
          tc_mma_f16(d, ad, bd, idesc_qk, t > 0 ? 1u : 0u);
        }
        tc_commit(&bars->s_full[j & 1]);
        tc_commit(&bars->k_empty[s]);
        trace_at(p, j, 2);
        return true;
      };
      ok = issue_qk(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles && !(ok = issue_qk(j + 1))) break;
        const int s = j % kStages;
        if (!mbar_wait(&bars->p_full[j & 1], (uint32_t)(j >> 1) & 1u, status, kStatusTimeoutTmemFull)) {
          ok = false;
          break;
        }
        trace_at(p, j, 3);
        if (!mbar_wait(&bars->v_full[s], (uint32_t)(j / kStages) & 1u, status, kStatusTimeoutTmaFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sp = smem_u32(smem + kOffP + (j & 1) * kPBytes);
        const uint32_t sv = smem_u32(smem + kOffV + s * kKVBytes);
#pragma unroll
        for (int t = 0; t < kBN / 16; ++t) {
          const uint64_t ad = make_desc_kmajor_sw128(sp + (t >> 2) * kPBlock + (t & 3) * 32);
          const uint64_t bd = make_desc_mnmajor_sw128(sv + t * 2048, kHalfBytes);
          tc_mma_f16(tmem_base + kTmemO, ad, bd, idesc_pv, (j > 0 || t > 0) ? 1u : 0u);
        }
        tc_commit(&bars->o_done);
        tc_commit(&bars->v_empty[s]);
        trace_at(p, j, 4);
      }
      // o_final completes once every MMA above has completed (also on the
      // error path, so the epilogue and the teardown never read a live TMEM)
      tc_commit(&bars->o_final);
    }
  } else {
    // ---------------- softmax (warps 2-5: one tile row per thread) ----------------
    const float c = p.scale * 1.4426950408889634f;
    const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
    float m_ref = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int b = j & 1;
      // exits stay warp-uniform: the tcgen05 loads below are warp-collective
      const bool got = mbar_wait(&bars->s_full[b], (uint32_t)(j >> 1) & 1u, status, kStatusTimeoutTmemFull);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0) trace_at(p, j, 5);
      tc_fence_after();
      uint32_t sv[kBN];
#pragma unroll
      for (int q4 = 0; q4 < kBN / 32; ++q4)
        tmem_ld_32x32b_x32(lane_base + b * kBN + q4 * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[q4 * 32]));
      tmem_ld_wait();
      if (warp == 2 && lane == 0) trace_at(p, j, 6);
      const int vis = nvis - (t0 + j) * kBN;  // keys [0, vis) of this tile are visible to my row
      if (!__all_sync(0xffffffffu, vis >= kBN)) {
#pragma unroll
        for (int i = 0; i < kBN; ++i)
          if (i >= vis) sv[i] = 0xff800000u;  // -inf
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int i = 0; i < kBN; i += 4) {
        mx0 = fmaxf(mx0, __uint_as_float(sv[i]));
        mx1 = fmaxf(mx1, __uint_as_float(sv[i + 1]));
        mx2 = fmaxf(mx2, __uint_as_float(sv[i + 2]));
        mx3 = fmaxf(mx3, __uint_as_float(sv[i + 3]));
      }
      if (warp == 2 && lane == 0) trace_at(p, j, 7);
      const float m_tile = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c;
      const bool need = m_tile > m_ref + kRescaleLog2;  // false when the tile is fully masked
      float f = 1.f;
      if (need) {
        f = exp2_approx(m_ref - m_tile);  // 0 while nothing was visible (m_ref = -inf)
        m_ref = m_tile;
        l *= f;
      }
      // O holds P_0..P_{j-1} V: rescale it (warp-uniformly, tcgen05 ld/st are
      // warp-collective) once PV(j-1) has completed.  s_full(j) implies PV(j-2)
      // completed, so waiting on o_done's phase j-1 is unambiguous.
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        const bool done = mbar_wait(&bars->o_done, (uint32_t)(j - 1) & 1u, status, kStatusTimeoutTmemFull);
        if (!__all_sync(0xffffffffu, done)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < kD / 32; ++cc) {
          uint32_t o[32];
          const uint32_t at = lane_base + kTmemO + cc * 32;
          tmem_ld_32x32b_x32(at, o);
          tmem_ld_wait();
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            lo[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            hi[i] = __float_as_uint(__uint_as_float(o[16 + i]) * f);
          }
          tmem_st_32x32b_x16(at, lo);
          tmem_st_32x32b_x16(at + 16, hi);
        }
        tmem_st_wait();
      }
      const float base = (m_ref == -INFINITY) ? 0.f : m_ref;
      float sum0 = 0.f, sum1 = 0.f;
      uint8_t* sp = smem + kOffP + b * kPBytes;
#pragma unroll
      for (int cc = 0; cc < kBN / 8; ++cc) {  // 8 keys = one 16-byte chunk of the P row
        float e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = exp2_approx(fmaf(__uint_as_float(sv[8 * cc + i]), c, -base));
        sum0 += (e[0] + e[1]) + (e[2] + e[3]);
        sum1 += (e[4] + e[5]) + (e[6] + e[7]);
        *reinterpret_cast<uint4*>(sp + (cc >> 3) * kPBlock + sw128(row, cc & 7)) =
            make_uint4(pack_bf16x2(e[0], e[1]), pack_bf16x2(e[2], e[3]), pack_bf16x2(e[4], e[5]),
                       pack_bf16x2(e[6], e[7]));
      }
      l += sum0 + sum1;
      if (warp == 2 && lane == 0) trace_at(p, j, 8);
      fence_proxy_async_smem();  // P written by threads, read by the tensor core
      tc_fence_before();
      mbar_arrive(&bars->p_full[b]);
      if (warp == 2 && lane == 0) trace_at(p, j, 9);
    }
    // ---- epilogue: O / l -> bf16 (or the fp32 partial of a key split) ----
    if (n_tiles > 0 && ok) ok = mbar_wait(&bars->o_final, 0, status, kStatusTimeoutTmemFull);
    if (warp == 2 && lane == 0) trace_at(p, 63, 2);
    __nv_bfloat16* dst = p.out + (size_t)g * p.ldo + (size_t)head * kD;
    if (gridDim.z > 1) {
      // partial (O relative to m_ref, m_ref, l) of this split; rows whose keys
      // all lie in other splits leave m = -inf, l = 0 and are ignored by the merge
      float* part = p.ws + (((size_t)blockIdx.z * p.n_rows + (g < p.n_rows ? g : 0)) * p.n_heads + head) * 132;
      const bool have = n_tiles > 0 && __all_sync(0xffffffffu, ok);
      if (have) tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < kD / 32; ++cc) {
        uint32_t o[32];
        if (have) {
          tmem_ld_32x32b_x32(lane_base + kTmemO + cc * 32, o);
          tmem_ld_wait();
        }
        if (g < p.n_rows) {
          float4* d4 = reinterpret_cast<float4*>(part + cc * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            d4[i] = have ? make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                       __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      if (g < p.n_rows) {
        part[128] = have ? m_ref : -INFINITY;
        part[129] = have ? l : 0.f;
      }
    } else if (n_tiles > 0 && __all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int cc = 0; cc < kD / 32; ++cc) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(lane_base + kTmemO + cc * 32, o);
        tmem_ld_wait();
        if (g < p.n_rows) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + cc * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                               pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                               pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                               pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
        }
      }
    } else if (g < p.n_rows && n_tiles == 0) {
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < 16; ++i) d4[i] = make_uint4(0, 0, 0, 0);
    }
  }

  // teardown: the MMA thread's o_final commit covers every MMA it issued; a
  // CTA that failed early still waits (bounded) for it before freeing TMEM
  if (warp == 1 && lane == 0 && n_tiles > 0) mbar_wait(&bars->o_final, 0, status, kStatusTimeoutDrain);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
  if (threadIdx.x == 0) trace_at(p, 63, 3);
}

// Merge of the key-split partials: one warp per (row, head), 4 dims a lane,
// splits combined in split order (deterministic).
__global__ void __launch_bounds__(256) attention_prefill_merge_kernel(AttnPrefillArgs p) {
  pdl_wait();
  pdl_launch_dependents();
  const long long pair = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pair >= (long long)p.n_rows * p.n_heads) return;
  const int lane = threadIdx.x & 31;
  const int row = (int)(pair / p.n_heads), head = (int)(pair % p.n_heads);
  const size_t stride = (size_t)p.n_rows * p.n_heads * 132;
  const float* base = p.ws + (size_t)pair * 132;
  float mx = -INFINITY;
  for (int s = 0; s < p.splits; ++s) mx = fmaxf(mx, base[s * stride + 128]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float den = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < p.splits; ++s) {
      const float* part = base + s * stride;
      const float m = part[128];
      if (m == -INFINITY) continue;
      const float w = exp2_approx(m - mx);
      const float4 o = reinterpret_cast<const float4*>(part)[lane];
      acc.x = fmaf(w, o.x, acc.x);
      acc.y = fmaf(w, o.y, acc.y);
      acc.z = fmaf(w, o.z, acc.z);
      acc.w = fmaf(w, o.w, acc.w);
      den = fmaf(w, part[129], den);
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  uint2 packed = make_uint2(pack_bf16x2(acc.x * inv, acc.y * inv), pack_bf16x2(acc.z * inv, acc.w * inv));
  *reinterpret_cast<uint2*>(p.out + (size_t)row * p.ldo + (size_t)head * kD + lane * 4) = packed;
}

cudaError_t attention_prefill(const AttnPrefillArgs& p, cudaStream_t stream) {
  if (p.head_dim != kD || p.n_rows < 0 || p.n_kv_heads <= 0 || p.n_heads % p.n_kv_heads != 0 ||
      kBM % (p.n_heads / p.n_kv_heads) != 0)
    return cudaErrorInvalidValue;
  if (p.n_rows == 0) return cudaSuccess;
  if (p.n_keys < 0 || p.n_keys > p.cache_cap) return cudaErrorInvalidValue;
  // [n_kv_heads][n_keys][128] view of the layer cache: rows past n_keys are
  // outside the tensor and arrive as zeros
  const uint64_t rows = p.n_keys > 0 ? (uint64_t)p.n_keys : 1;
  CUtensorMap tk, tv;
  if (!make_tmap_3d_bf16(&tk, p.k_cache, kD, rows, (uint64_t)p.n_kv_heads, kD, (uint64_t)p.cache_cap * kD, 64,
                         kBN))
    return cudaErrorInvalidValue;
  if (!make_tmap_3d_bf16(&tv, p.v_cache, kD, rows, (uint64_t)p.n_kv_heads, kD, (uint64_t)p.cache_cap * kD, 64,
                         kBN))
    return cudaErrorInvalidValue;
  ensure_smem_attr(attention_prefill_tc_kernel, kSmemBytes);
  const int span = kBM / (p.n_heads / p.n_kv_heads);
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  AttnPrefillArgs a = p;
  a.splits = attention_prefill_splits(p, sms);
  dim3 grid(p.n_kv_heads, (p.n_rows + span - 1) / span, a.splits);
  cudaError_t err = launch_pdl(attention_prefill_tc_kernel, grid, dim3(kThreads), kSmemBytes, stream, tk, tv, a);
  if (err != cudaSuccess || a.splits == 1) return err;
  const long long pairs = (long long)p.n_rows * p.n_heads;
  return launch_pdl(attention_prefill_merge_kernel, dim3((unsigned)((pairs + 7) / 8)), dim3(256), 0, stream, a);
}

// A grid of fewer CTAs than SMs (a few hundred selective rows over a long
// cache) gets its key tiles split over up to 4 CTAs per row tile, each split
// keeping at least 16 key tiles (2048 keys: below that a CTA's fixed costs -
// TMEM allocation, Q staging, pipeline fill - outweigh the shorter key loop;
// 300 rows over 1676 keys ran 31.7 us whole and 41.5 us split three ways);
// full prefills (a wave of row tiles or more) never split.
static int g_forced_splits = 0;  // measurement hook: 0 = the cost rule below
void set_attention_prefill_splits(int s) { g_forced_splits = s < 0 ? 0 : s; }

int attention_prefill_splits(const AttnPrefillArgs& p, int num_sms) {
  if (p.ws == nullptr || p.n_rows <= 0 || p.n_kv_heads <= 0 || num_sms <= 0) return 1;
  if (g_forced_splits > 0) {
    const int key_tiles = (p.n_keys + kBN - 1) / kBN;
    int s = g_forced_splits < key_tiles ? g_forced_splits : key_tiles;
    if (s > 4) s = 4;
    if ((long long)s * p.n_rows * p.n_heads * 132 > p.ws_floats) return 1;
    return s < 1 ? 1 : s;
  }
  const int span = kBM / (p.n_heads / p.n_kv_heads);
  const int ctas = p.n_kv_heads * ((p.n_rows + span - 1) / span);
  if (ctas >= num_sms) return 1;
  const int key_tiles = (p.n_keys + kBN - 1) / kBN;
  // one CTA per SM (224 KB of shared memory): s splits take ceil(ctas * s /
  // SMs) waves of 1/s of the work each, plus a merge; pick the cheapest
  int best_s = 1;
  double best = 1.0;
  for (int s = 2; s <= 4 && key_tiles >= 16 * s; ++s) {
    const int waves = (ctas * s + num_sms - 1) / num_sms;
    const double cost = (double)waves / s + 0.1;
    if (cost < best) best = cost, best_s = s;
  }
  if ((long long)best_s * p.n_rows * p.n_heads * 132 > p.ws_floats) return 1;
  return best_s;
}

}  // namespace sc
