// Token-column tensor-core GEMM for a few hundred token rows (CacheBlend's
// active rows: 64 < M <= 512):  out[m, n] = sum_k x[m, k] * w[n, k].
//
// At M ~ 300 the row-major GEMM (gemm_tc.cu, tokens as the 128-row MMA M)
// pads the token count to whole 128-row tiles (300 -> 384), and its
// 128 x 256 tiles land on the 148 SMs in 2.27 rounds (gate/up) or need a
// 3-way K split; both cost more than the FLOPs.  Here the roles are swapped:
// the weight tile is the MMA's M (128 rows; a unit may take two consecutive
// weight tiles, e.g. the gate block and the up block of one SwiGLU block) and
// the tokens are its N, padded only to a multiple of 16 (300 -> 2 x 160, or
// one column tile up to 256).  A unit (weight tiles, token tile, K slice) is
// streamed through a deep TMA ring (128-byte swizzle, no multicast) and
// accumulated in TMEM; adjacent units share their weight tiles (the token
// tile is the fastest index), so concurrent CTAs read each weight byte from
// HBM once and from L2 otherwise.
//
// Epilogues:
//   WIDE_PARTIAL  the fp32 partial of K slice s goes to ws[s][m][n] (the
//                 layout of the split-K reduce kernels, which apply the
//                 residual / RMSNorm or the QKV RoPE + cache scatter)
//   WIDE_SWIGLU   two weight tiles per unit = one gate block and its up block
//                 (gate/up interleaved in 128-row blocks): out[m, blk*128+i] =
//                 silu(gate) * up with the HF rounding order, no K split
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer (one
// lane), warps 2-5 epilogue (TMEM lane quarter = warp % 4).  Every wait is
// bounded and reports through the status word.
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {
constexpr int kWdBM = 128;                   // weight rows per accumulator (MMA M)
constexpr int kWdBK = 64;                    // 128 bytes of bf16 per row
constexpr int kWdTileBytes = kWdBM * kWdBK * 2;  // 16 KB per weight tile and k-block
constexpr int kWdMaxStages = 8;
constexpr int kWdThreads = 192;
constexpr int kWdSmemLimit = 227 * 1024;

struct alignas(8) WdBars {
  uint64_t full[kWdMaxStages];
  uint64_t empty[kWdMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t sk_ticket;
};

__device__ __forceinline__ void wd_tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// One work item of a CTA: a whole unit, or a run of k-blocks of a stream-K
// tail unit (piece `piece` of `n_pieces`; n_pieces == 1 is a whole unit).
struct WdItem {
  int g, t, s, kb0, kb1;
  int tail;      // index among the tail units (-1: data-parallel unit)
  int piece, n_pieces;
};

// Walks the items of one CTA in order: its data-parallel units (one per
// round of the grid), then its run [lo, hi) of the tail's k-block space.
struct WdIter {
  int r;
  long long w, hi;
  bool tail;
};

__device__ __forceinline__ void wd_decode(const WideArgs& a, int u, int num_kb, WdItem& it) {
  it.t = u % a.n_tt;
  const int r = u / a.n_tt;
  it.s = r % a.splits;
  it.g = r / a.splits;
  it.kb0 = it.s * num_kb / a.splits;
  it.kb1 = (it.s + 1) * num_kb / a.splits;
}

// CTA whose tail run holds k-block x: the largest c with floor(c * Wt / C) <= x
__device__ __forceinline__ int wd_sk_owner(long long x, long long Wt, int C) {
  long long c = ((x + 1) * C + Wt - 1) / Wt - 1;
  return (int)(c < 0 ? 0 : (c >= C ? C - 1 : c));
}

__device__ __forceinline__ void wd_begin(const WideArgs& a, int num_kb, WdIter& it) {
  it.r = 0;
  it.tail = false;
  it.w = it.hi = 0;
  if (a.sk_tail > 0 && (int)blockIdx.x < a.sk_ctas) {
    const long long Wt = (long long)a.sk_tail * num_kb;
    it.w = (long long)blockIdx.x * Wt / a.sk_ctas;
    it.hi = (long long)(blockIdx.x + 1) * Wt / a.sk_ctas;
  }
}

__device__ __forceinline__ bool wd_next(const WideArgs& a, int num_kb, int units, WdIter& it, WdItem& out) {
  const int dp_units = units - a.sk_tail;
  if (!it.tail) {
    const int u = (int)blockIdx.x + it.r * (int)gridDim.x;
    if (u < dp_units) {
      ++it.r;
      wd_decode(a, u, num_kb, out);
      out.tail = -1;
      out.piece = 0;
      out.n_pieces = 1;
      return true;
    }
    it.tail = true;
  }
  if (it.w >= it.hi) return false;
  const long long Wt = (long long)a.sk_tail * num_kb;
  const int tu = (int)(it.w / num_kb);
  const long long u0 = (long long)tu * num_kb;
  const int kb0 = (int)(it.w - u0);
  const int kb1 = (int)((it.hi < u0 + num_kb ? it.hi : u0 + num_kb) - u0);
  it.w = u0 + kb1;
  wd_decode(a, dp_units + tu, num_kb, out);
  out.kb0 = kb0;
  out.kb1 = kb1;
  const int first = wd_sk_owner(u0, Wt, a.sk_ctas);
  out.n_pieces = wd_sk_owner(u0 + num_kb - 1, Wt, a.sk_ctas) - first + 1;
  out.piece = (int)blockIdx.x - first;
  out.tail = tu;
  return true;
}

__device__ __forceinline__ void wd_epi_barrier() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
}  // namespace

template <int ACC, int EPI>
__global__ void __launch_bounds__(kWdThreads, 1)
    wide_mma_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    WideArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stage_bytes = ACC * kWdTileBytes + a.bn * kWdBK * 2;
  const int stages = a.stages;
  WdBars* bars = reinterpret_cast<WdBars*>(smem + stages * stage_bytes);
  const int warp = warp_id(), lane = lane_id();
  const int num_kb = a.K / kWdBK;
  const int groups = a.N / (kWdBM * ACC);
  const int units = groups * a.n_tt * a.splits;
  const int acc_cols = ACC * a.bn;  // TMEM columns of one unit's accumulators

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&bars->full[s], 1), mbar_init(&bars->empty[s], 1);
    for (int b = 0; b < 2; ++b) mbar_init(&bars->tmem_full[b], 1), mbar_init(&bars->tmem_empty[b], 4);
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, (uint32_t)a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // The weight tiles of the first ring fill do not depend on the previous
      // kernel: issue them before waiting on it, the token tiles after.
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int pre = 0;  // stages whose weight half was issued before the wait
      {
        WdIter it;
        WdItem w;
        wd_begin(a, num_kb, it);
        if (wd_next(a, num_kb, units, it, w)) {
          for (int kb = w.kb0; kb < w.kb1 && pre < stages; ++kb, ++pre) {
            uint8_t* sa = smem + pre * stage_bytes;
            mbar_arrive_expect_tx(&bars->full[pre], (uint32_t)stage_bytes);
            tma_load_2d(sa, &tmap_w, &bars->full[pre], kb * kWdBK, w.g * kWdBM * ACC);
          }
        }
      }
      pdl_wait();
      pdl_launch_dependents();
      bool issued[kWdMaxStages];
      uint32_t issued_phase[kWdMaxStages];
      for (int s = 0; s < kWdMaxStages; ++s) issued[s] = false, issued_phase[s] = 0;
      int done_pre = 0;
      WdIter it;
      WdItem w;
      wd_begin(a, num_kb, it);
      while (ok && wd_next(a, num_kb, units, it, w)) {
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          uint8_t* sa = smem + stage * stage_bytes;
          if (done_pre < pre) {
            // first ring fill: the weight half is in flight, add the tokens
            ++done_pre;
          } else {
            if (!mbar_wait(&bars->empty[stage], phase ^ 1, a.status, kStatusTimeoutSmemEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars->full[stage], (uint32_t)stage_bytes);
            tma_load_2d(sa, &tmap_w, &bars->full[stage], kb * kWdBK, w.g * kWdBM * ACC);
          }
          tma_load_2d(sa + ACC * kWdTileBytes, &tmap_x, &bars->full[stage], kb * kWdBK, w.t * a.bn);
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == stages) stage = 0, phase ^= 1;
        }
      }
      // every stage that was armed must see its bytes land before the CTA exits
      for (int s = 0; s < stages; ++s)
        if (issued[s]) mbar_wait(&bars->full[s], issued_phase[s], a.status, kStatusTimeoutDrain);
    } else {
      pdl_wait();
      pdl_launch_dependents();
    }
  } else if (warp == 1) {
    pdl_wait();
    pdl_launch_dependents();
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16(kWdBM, a.bn);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true, any = false;
      WdIter it;
      WdItem w;
      wd_begin(a, num_kb, it);
      for (; ok && wd_next(a, num_kb, units, it, w); ++local) {
        const int buf = local % a.nbuf;
        const uint32_t tphase = (uint32_t)((local / a.nbuf) & 1);
        if (!mbar_wait(&bars->tmem_empty[buf], tphase ^ 1, a.status, kStatusTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tacc = tmem_base + (uint32_t)(buf * acc_cols);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&bars->full[stage], phase, a.status, kStatusTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * stage_bytes);
          const uint32_t sb = sa + ACC * kWdTileBytes;
#pragma unroll
          for (int k = 0; k < kWdBK / 16; ++k) {
            const uint64_t bdesc = make_desc_kmajor_sw128(sb + k * 32);
#pragma unroll
            for (int c = 0; c < ACC; ++c)
              tc_mma_f16(tacc + (uint32_t)(c * a.bn), make_desc_kmajor_sw128(sa + c * kWdTileBytes + k * 32), bdesc,
                         idesc, (kb != w.kb0 || k != 0) ? 1u : 0u);
          }
          any = true;
          tc_commit(&bars->empty[stage]);
          if (++stage == stages) stage = 0, phase ^= 1;
        }
        if (!ok) break;
        tc_commit(&bars->tmem_full[buf]);
      }
      if (any) {
        tc_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, a.status, kStatusTimeoutDrain);
      }
    }
  } else {
    pdl_wait();
    pdl_launch_dependents();
    const int quarter = warp & 3;
    const int i = quarter * 32 + lane;  // row of the 128-row weight tile
    int local = 0;
    WdIter it;
    WdItem w;
    wd_begin(a, num_kb, it);
    for (; wd_next(a, num_kb, units, it, w); ++local) {
      const int buf = local % a.nbuf;
      const uint32_t tphase = (uint32_t)((local / a.nbuf) & 1);
      if (!mbar_wait(&bars->tmem_full[buf], tphase, a.status, kStatusTimeoutTmemFull)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * acc_cols);
      const int m0 = w.t * a.bn;
      bool finish = true;  // this CTA applies the epilogue of the unit
      // stream-K partials of the unit: [piece][acc * bn / 4][128 rows] float4
      // (4 consecutive token columns of one weight row per float4)
      const float4* others = nullptr;
      int oth0 = 0, oth1 = 0;  // the other pieces, in piece order
      if (w.n_pieces > 1) {
        // stream-K piece: leave the fp32 partial, count the arrival; the last
        // piece to arrive sums all pieces in piece order and finishes the unit
        float4* slots = reinterpret_cast<float4*>(a.sk_ws) + (size_t)w.tail * a.sk_max_pieces * (acc_cols / 4) * kWdBM;
        float4* mine = slots + (size_t)w.piece * (acc_cols / 4) * kWdBM;
#pragma unroll 1
        for (int c0 = 0; c0 < acc_cols; c0 += 16) {
          uint32_t r[16];
          wd_tmem_ld16(tbase + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 4; ++q)
            mine[(size_t)(c0 / 4 + q) * kWdBM + i] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                                                 __uint_as_float(r[4 * q + 2]),
                                                                 __uint_as_float(r[4 * q + 3]));
        }
        __threadfence();
        wd_epi_barrier();
        if (warp == 2 && lane == 0) bars->sk_ticket = atomicAdd(a.sk_tickets + w.tail, 1u);
        wd_epi_barrier();
        finish = bars->sk_ticket == (uint32_t)(w.n_pieces - 1);
        if (finish) {
          __threadfence();
          others = slots;
          oth0 = w.piece == 0 ? 1 : 0;
          oth1 = w.piece == 2 ? 1 : 2;  // used only with three pieces
          if (warp == 2 && lane == 0) a.sk_tickets[w.tail] = 0u;
        }
      }
      if (finish) {
#pragma unroll 2
        for (int c0 = 0; c0 < a.bn; c0 += 16) {
          float v[ACC][16];
          float4 o0[ACC][4], o1[ACC][4];
          if (others != nullptr) {
            // every load of the chunk in flight before the first use
#pragma unroll
            for (int c = 0; c < ACC; ++c) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const size_t col4 = (size_t)((c * a.bn + c0) / 4 + q) * kWdBM + i;
                o0[c][q] = __ldcg(others + (size_t)oth0 * (acc_cols / 4) * kWdBM + col4);
                o1[c][q] = w.n_pieces == 3 ? __ldcg(others + (size_t)oth1 * (acc_cols / 4) * kWdBM + col4)
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
          }
#pragma unroll
          for (int c = 0; c < ACC; ++c) {
            uint32_t r[16];
            wd_tmem_ld16(tbase + (uint32_t)(c * a.bn + c0), r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[c][j] = __uint_as_float(r[j]);
          }
          if (others != nullptr) {
            // fixed piece order (x0 + x1) + x2: the sum does not depend on
            // which piece arrived last
#pragma unroll
            for (int c = 0; c < ACC; ++c) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float4 f0 = o0[c][j / 4], f1 = o1[c][j / 4];
                const float a0 = (j & 3) == 0 ? f0.x : (j & 3) == 1 ? f0.y : (j & 3) == 2 ? f0.z : f0.w;
                const float a1 = (j & 3) == 0 ? f1.x : (j & 3) == 1 ? f1.y : (j & 3) == 2 ? f1.z : f1.w;
                const float mine_v = v[c][j];
                float x0, x1, x2;
                if (w.piece == 0) x0 = mine_v, x1 = a0, x2 = a1;
                else if (w.piece == 1) x0 = a0, x1 = mine_v, x2 = a1;
                else x0 = a0, x1 = a1, x2 = mine_v;
                v[c][j] = w.n_pieces == 3 ? (x0 + x1) + x2 : x0 + x1;
              }
            }
          }
          if constexpr (EPI == WIDE_SWIGLU) {
            __nv_bfloat16* dst = a.out + (size_t)w.g * kWdBM + i;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = m0 + c0 + j;
              if (m < a.M) {
                const float gb = bf16_round(v[0][j]);
                const float ub = bf16_round(v[ACC - 1][j]);
                dst[(size_t)m * a.ldo] = __float2bfloat16_rn(bf16_round(silu_f(gb)) * ub);
              }
            }
          } else {
#pragma unroll
            for (int c = 0; c < ACC; ++c) {
              const int n = (w.g * ACC + c) * kWdBM + i;
              float* dst = a.ws + (size_t)w.s * a.M * a.N + n;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int m = m0 + c0 + j;
                if (m < a.M) dst[(size_t)m * a.N] = v[c][j];
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tmem_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, (uint32_t)a.tmem_cols);
}

// ---------------------------------------------------------------------------
// Plan: weight tiles per unit, token tile, K split.  A roofline-style cost
// per unit (k-blocks x the slower of tensor time and L2->SM time, plus a
// fixed pipeline fill and the epilogue), times the rounds of units over the
// SMs, plus the split-K partials' round trip; the cheapest plan wins.
// ---------------------------------------------------------------------------
static double wide_cost(int M, int N, int K, int acc, int n_tt, int splits, int epi, int num_sms, bool stream_k,
                        WidePlan* out) {
  const int bn = ((M + n_tt - 1) / n_tt + 15) / 16 * 16;
  if (bn < 16 || bn > 256) return -1.0;
  if (N % (kWdBM * acc) != 0) return -1.0;
  const int num_kb = K / kWdBK;
  if (splits > num_kb) return -1.0;
  const int stage_bytes = acc * kWdTileBytes + bn * kWdBK * 2;
  int stages = (kWdSmemLimit - 1024 - (int)sizeof(WdBars)) / stage_bytes;
  if (stages > kWdMaxStages) stages = kWdMaxStages;
  if (stages < 2) return -1.0;
  const int cols = acc * bn;
  const int nbuf = 2 * cols <= 512 ? 2 : 1;
  int alloc = 32;
  while (alloc < nbuf * cols) alloc *= 2;
  if (alloc > 512) return -1.0;
  const long long units = (long long)(N / (kWdBM * acc)) * n_tt * splits;
  const int grid = units < num_sms ? (int)units : num_sms;
  const long long rounds = (units + num_sms - 1) / num_sms;
  const double busy = (double)grid;
  // stream-K tail (SwiGLU only: the other epilogues balance through the K split)
  int sk_tail = 0, sk_ctas = 0, sk_max_pieces = 0;
  if (stream_k && epi == WIDE_SWIGLU && units > grid && units % grid != 0) {
    sk_tail = (int)(units % grid);
    const long long Wt = (long long)sk_tail * num_kb;
    // runs of at least 8 k-blocks and half a unit: a unit meets at most 3 pieces
    const long long min_run = num_kb / 2 > 8 ? (num_kb + 1) / 2 : 8;
    sk_ctas = (int)(Wt / min_run < grid ? Wt / min_run : grid);
    if (sk_ctas < 2) {
      sk_tail = sk_ctas = 0;
    } else {
      const long long run = Wt / sk_ctas;  // shortest run of k-blocks of a CTA
      sk_max_pieces = (int)((num_kb + run - 1) / run) + 1;
      if (sk_max_pieces > 3) sk_tail = sk_ctas = sk_max_pieces = 0;
    }
  }
  // per-SM rates (B200, measured): ~11.2 TFLOP/s of bf16 MMA, L2->SM share of ~13 TB/s
  const double l2_per_sm = 13.0e12 / busy;
  const double kb_flops = 2.0 * kWdBM * acc * bn * kWdBK;
  const double kb_time = fmax(kb_flops / 11.2e12, stage_bytes / (l2_per_sm < 120e9 ? l2_per_sm : 120e9));
  const double kb_per_unit = (double)num_kb / splits;
  const double epi_time = (epi == WIDE_SWIGLU ? 1.0 : 2.0) * (double)kWdBM * cols * 2.0 / 60e9;
  const double unit_time = kb_per_unit * kb_time + 1.5e-6 + (nbuf == 2 ? 0.0 : epi_time);
  double cost;
  if (sk_tail > 0) {
    // whole rounds, then each CTA's run of the tail; the pieces' partials go
    // through L2 (written by every piece, read by the last)
    const double run_kb = (double)sk_tail * num_kb / sk_ctas;
    const double fix = (double)sk_tail * (sk_max_pieces + 1) * cols * kWdBM * 4.0 / 5.0e12;
    cost = (double)(units / grid) * unit_time + run_kb * kb_time + 1.5e-6 + 2.0 * epi_time + fix;
  } else {
    cost = rounds * unit_time + (nbuf == 2 ? epi_time : 0.0);
  }
  if (epi == WIDE_PARTIAL) cost += ((double)M * N * 4.0 * (splits + 1) + (double)M * N * 2.0) / 5.0e12 + 2e-6;
  if (out != nullptr) {
    out->acc = acc;
    out->bn = bn;
    out->n_tt = n_tt;
    out->splits = splits;
    out->stages = stages;
    out->nbuf = nbuf;
    out->tmem_cols = alloc;
    out->smem = stages * stage_bytes + 1024 + (int)sizeof(WdBars);
    out->grid = grid;
    out->sk_tail = sk_tail;
    out->sk_ctas = sk_ctas;
    out->sk_max_pieces = sk_max_pieces;
  }
  return cost;
}

bool wide_plan(int M, int N, int K, int epi, int num_sms, int acc_req, int n_tt_req, int splits_req,
               bool stream_k, WidePlan* plan) {
  if (M < 1 || M > 512 || K % kWdBK != 0 || num_sms < 1) return false;
  double best = -1.0;
  WidePlan bp{};
  const int tt_min = (M + 255) / 256;
  for (int acc = 1; acc <= 2; ++acc) {
    if (epi == WIDE_SWIGLU && acc != 2) continue;
    if (acc_req > 0 && acc != acc_req) continue;
    for (int n_tt = tt_min; n_tt <= tt_min + 3; ++n_tt) {
      if (n_tt_req > 0 && n_tt != n_tt_req) continue;
      for (int s = 1; s <= (epi == WIDE_SWIGLU ? 1 : 16); ++s) {
        if (splits_req > 0 && s != splits_req) continue;
        WidePlan p{};
        const double c = wide_cost(M, N, K, acc, n_tt, s, epi, num_sms, stream_k, &p);
        if (c < 0.0) continue;
        if (best < 0.0 || c < best) best = c, bp = p;
      }
    }
  }
  if (best < 0.0) return false;
  *plan = bp;
  return true;
}

template <int ACC, int EPI>
static cudaError_t launch_wide(const WideArgs& a, const CUtensorMap& tw, const CUtensorMap& tx, int grid,
                               cudaStream_t stream) {
  auto kern = wide_mma_kernel<ACC, EPI>;
  ensure_smem_attr(kern, a.smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kWdThreads, 1, 1);
  cfg.dynamicSmemBytes = a.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tw, tx, a);
}

cudaError_t wide_gemm(const WideArgs& args, cudaStream_t stream) {
  WideArgs a = args;
  if (a.M < 1 || a.M > 512 || a.K % kWdBK != 0 || a.bn < 16 || a.bn > 256 || a.bn % 16 != 0) return cudaErrorInvalidValue;
  if (a.acc < 1 || a.acc > 2 || a.N % (kWdBM * a.acc) != 0 || a.n_tt * a.bn < a.M) return cudaErrorInvalidValue;
  if (a.stages < 2 || a.stages > kWdMaxStages || a.splits < 1 || a.splits > a.K / kWdBK) return cudaErrorInvalidValue;
  if (a.nbuf < 1 || a.nbuf > 2 || a.tmem_cols > 512 || a.nbuf * a.acc * a.bn > a.tmem_cols) return cudaErrorInvalidValue;
  if (a.epi == WIDE_SWIGLU && (a.acc != 2 || a.splits != 1 || a.out == nullptr)) return cudaErrorInvalidValue;
  if (a.epi == WIDE_PARTIAL && a.ws == nullptr) return cudaErrorInvalidValue;
  CUtensorMap tw, tx;
  if (!make_tmap_2d_bf16(&tw, a.w, a.K, a.N, a.ldw, kWdBK, kWdBM * a.acc, true)) return cudaErrorInvalidValue;
  if (!make_tmap_2d_bf16(&tx, a.x, a.K, a.M, a.ldx, kWdBK, a.bn, true)) return cudaErrorInvalidValue;
  const int units = a.N / (kWdBM * a.acc) * a.n_tt * a.splits;
  const int grid = a.grid;
  if (grid < 1 || grid > units || grid > a.num_sms) return cudaErrorInvalidValue;
  if (a.sk_tail > 0) {
    if (a.sk_tail >= units || a.sk_ctas < 1 || a.sk_ctas > grid || a.sk_ws == nullptr || a.sk_tickets == nullptr ||
        (units - a.sk_tail) % grid != 0)
      return cudaErrorInvalidValue;
    const long long run = (long long)a.sk_tail * (a.K / kWdBK) / a.sk_ctas;
    if (run < 1 || ((a.K / kWdBK) + run - 1) / run + 1 > a.sk_max_pieces || a.sk_max_pieces > 3)
      return cudaErrorInvalidValue;
  } else if ((units + grid - 1) / grid * grid < units) {
    return cudaErrorInvalidValue;
  }
  if (a.epi == WIDE_SWIGLU) return launch_wide<2, WIDE_SWIGLU>(a, tw, tx, grid, stream);
  return a.acc == 2 ? launch_wide<2, WIDE_PARTIAL>(a, tw, tx, grid, stream)
                    : launch_wide<1, WIDE_PARTIAL>(a, tw, tx, grid, stream);
}

}  // namespace sc
