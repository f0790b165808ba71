// Persistent tcgen05 BF16 GEMM for sm_100a with fused epilogues.
//
//   C[M, N] = A[M, K] . B[N, K]^T      (A activations, B nn.Linear weights)
//
// One CTA per SM walks a static tile schedule.  Warp roles:
//   warp 0      TMA producer: 128B-swizzled A/B tiles into a STAGES-deep ring
//   warp 1      MMA issuer: tcgen05.mma (M=128, N=BN, K=16) into TMEM,
//               owns the TMEM allocation
//   warps 2..   epilogue: tcgen05.ld the fp32 accumulator (one row per
//               thread), apply the fused epilogue and store bf16
// Two tile shapes (ACC = accumulators per tile):
//   ACC = 1   128 x BN tiles, the accumulator double-buffered in TMEM so the
//             epilogue of tile i overlaps the MMAs of tile i+1; 4 epilogue warps.
//   ACC = 2   256 x 256 tiles: every B k-block in shared memory feeds two
//             M=128 MMAs (rows 0-127 and 128-255 of the A k-block) into two
//             accumulators that fill the 512 TMEM columns (no double buffer;
//             8 epilogue warps drain both halves at once).  Per k-block the
//             CTA moves 64 KB from L2 for 256x256 outputs instead of 48 KB for
//             128x256: the 128x256 shape is L2-bandwidth-bound on B200 (ncu:
//             L2 throughput ~80 % with the tensor pipe ~55 % busy), this one
//             a third less so.  A last m-tile with <= 128 valid rows runs one
//             accumulator only.  Not used with row-sharded A (TP all-gather)
//             or the reduce-scatter epilogue.
// No cluster multicast is used anywhere, so the same kernel is safe inside
// multi-GPU programs.
//
// Fused epilogues (the hot projections of a Llama layer):
//   EPI_STORE     C = acc
//   EPI_RESIDUAL  C = R + bf16(acc)                         (o_proj, down_proj)
//   EPI_SWIGLU    C = silu(gate) * up, gate/up interleaved in 128-col blocks
//   EPI_PARTIAL   split-K: the fp32 partial of K-slice ks goes to
//                 ws[ks][M][N]; splitk_reduce sums the slices in slice order
//                 and applies the STORE / RESIDUAL epilogue.  Used when a
//                 small-M GEMM has fewer output tiles than SMs (the o_proj and
//                 down_proj of CacheBlend's active rows).
//   EPI_QKV       RoPE on Q/K heads at per-row positions; Q to a row-major
//                 buffer, K/V scattered into the paged layer cache at per-row
//                 slots; optional per-(row, kv-head) deviation partials of the
//                 fresh K/V against the cache contents they overwrite (the
//                 CacheBlend check-layer score, fused).
//
// Reference behaviour reproduced: modeling.py:330-342 (_project_qkv with
// apply_rope), modeling.py:257-264 (scatter of fresh K/V into the composed
// cache), modeling.py:215-226 / reuse_cacheblend_pipeline.py:586-604
// (squared deviation of fresh vs cached K or V), HF LlamaMLP SwiGLU.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace sc {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kPrefetchKb = 6;  // k-blocks of L2 prefetch ahead of the smem ring

template <int BN, int ACC = 1>
struct GemmCfg {
  static_assert(ACC == 1 || (ACC == 2 && BN == 256), "two accumulators only with 256-column tiles");
  static constexpr int kBM = kGemmBM * ACC;  // rows per tile
  static constexpr int kStages = ACC == 2 ? 3 : ((BN == 256) ? 4 : 6);
  static constexpr int kABytes = kBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kNumBuf = ACC == 2 ? 1 : 2;  // TMEM accumulator buffers
  static constexpr int kTmemCols = kNumBuf * ACC * BN;  // 256 or 512 columns
  static constexpr int kEpiWarps = 4 * ACC;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kEpiStageBytes = ACC == 1 ? 4 * 32 * 33 * 4 : 0;  // per-warp transpose tiles (EPI_RS)
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256 + kEpiStageBytes;
};

struct alignas(8) GemmBarriers {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
};

// --------------------------------------------------------------------------
// Epilogue helpers (one thread = one output row, 32 columns per TMEM load)
// --------------------------------------------------------------------------
__device__ __forceinline__ void store_row32(__nv_bfloat16* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
    w.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
    w.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
    w.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
    d[i] = w;
  }
}

__device__ __forceinline__ void load_row32(const __nv_bfloat16* src, float* v) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 w = s[i];
    float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z),
           d = unpack_bf16x2(w.w);
    v[8 * i + 0] = a.x; v[8 * i + 1] = a.y; v[8 * i + 2] = b.x; v[8 * i + 3] = b.y;
    v[8 * i + 4] = c.x; v[8 * i + 5] = c.y; v[8 * i + 6] = d.x; v[8 * i + 7] = d.y;
  }
}

template <int BN, int EPI>
__device__ __forceinline__ void gemm_epilogue_tile(const GemmEpilogue& ep, uint32_t tacc,
                                                   int row, int tile_n, int M, int N, uint32_t* stage,
                                                   int ks) {
  const bool row_ok = row < M;
  if constexpr (EPI == EPI_PARTIAL) {
    float* dst = ep.ws + ((size_t)ks * M + row) * N;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tacc + c * 32, r);
      tmem_ld_wait();
      const int col = tile_n * BN + c * 32;
      if (row_ok && col < N) {
        float4* d4 = reinterpret_cast<float4*>(dst + col);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          d4[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                              __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
      }
    }
  } else if constexpr (EPI == EPI_STORE || EPI == EPI_RESIDUAL) {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tacc + c * 32, r);
      tmem_ld_wait();
      const int col = tile_n * BN + c * 32;
      if (row_ok && col < N) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if constexpr (EPI == EPI_RESIDUAL) {
          float res[32];
          load_row32(ep.residual + (size_t)row * ep.ldr + col, res);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = res[i] + bf16_round(v[i]);
        }
        store_row32(ep.out + (size_t)row * ep.ldo + col, v);
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    // Tile columns [0, BN/2) are gate rows, [BN/2, BN) the matching up rows.
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(tacc + c * 32, g);
      tmem_ld_32x32b_x32(tacc + BN / 2 + c * 32, u);
      tmem_ld_wait();
      const int col = tile_n * (BN / 2) + c * 32;
      if (row_ok) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float gb = bf16_round(__uint_as_float(g[i]));
          const float ub = bf16_round(__uint_as_float(u[i]));
          v[i] = bf16_round(silu_f(gb)) * ub;
        }
        store_row32(ep.out + (size_t)row * ep.ldo + col, v);
      }
    }
  } else if constexpr (EPI == EPI_RS) {
    // fused reduce-scatter: this warp's 32 rows (one owner, rs_rows is a
    // multiple of 128) are converted to bf16 partials and staged through
    // shared memory, so every warp store writes one contiguous 128-byte row
    // segment into the owner's receive slot (NVLink stores for peers)
    const int lane = threadIdx.x & 31;
    const int row_base = row - lane;
    const int shard = row_base < M ? row_base / ep.rs_rows : 0;
    const int lrow_base = row_base - shard * ep.rs_rows;
    __nv_bfloat16* dst_base = reinterpret_cast<__nv_bfloat16*>(ep.rs_dst[shard]) +
                              ((size_t)ep.rs_sender * ep.rs_rows + lrow_base) * N;
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      uint32_t a[32], b[32];
      tmem_ld_32x32b_x32(tacc + c * 64, a);
      tmem_ld_32x32b_x32(tacc + c * 64 + 32, b);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        stage[lane * 33 + i] = pack_bf16x2(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]));
        stage[lane * 33 + 16 + i] = pack_bf16x2(__uint_as_float(b[2 * i]), __uint_as_float(b[2 * i + 1]));
      }
      __syncwarp();
      const int col = tile_n * BN + c * 64;
      if (col < N) {
#pragma unroll 4
        for (int r = 0; r < 32; ++r) {
          if (row_base + r < M)
            *reinterpret_cast<uint32_t*>(dst_base + (size_t)r * N + col + 2 * lane) = stage[r * 33 + lane];
        }
      }
      __syncwarp();
    }
  } else if constexpr (EPI == EPI_QKV) {
    int pos = 0, slot = 0;
    if (row_ok) {
      pos = ep.rope_pos[row];
      slot = ep.cache_slot[row];
    }
#pragma unroll 1
    for (int j = 0; j < BN / 128; ++j) {
      const int head = tile_n * (BN / 128) + j;  // index in [q heads | k heads | v heads]
      const bool is_q = head < ep.n_q_heads;
      const bool is_k = !is_q && head < ep.n_q_heads + ep.n_kv_heads;
      const bool is_v = !is_q && !is_k;
      const int kvh = is_k ? head - ep.n_q_heads : head - ep.n_q_heads - ep.n_kv_heads;
      __nv_bfloat16* dst = nullptr;
      if (is_q) {
        dst = ep.q_out + (size_t)row * ep.ldq + head * 128;
      } else {
        __nv_bfloat16* cache = is_k ? ep.k_cache : ep.v_cache;
        dst = cache + ((size_t)kvh * ep.cache_cap + slot) * 128;
      }
      const bool want_dev = ep.dev_part != nullptr &&
                            ((is_k && (ep.dev_mode & DEV_KEY)) ||
                             (is_v && (ep.dev_mode & DEV_VALUE)));
      const bool l1 = (ep.dev_mode & DEV_L1) != 0;
      float dev = 0.f;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t a[32], b[32];
        tmem_ld_32x32b_x32(tacc + j * 128 + half * 32, a);
        tmem_ld_32x32b_x32(tacc + j * 128 + 64 + half * 32, b);
        tmem_ld_wait();
        if (!row_ok) continue;
        float xa[32], xb[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          xa[i] = __uint_as_float(a[i]);
          xb[i] = __uint_as_float(b[i]);
        }
        if (!is_v) {
          const float2* tab = ep.rope_table + (size_t)pos * 64 + half * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float2 cs = tab[i];
            const float oa = xa[i] * cs.x - xb[i] * cs.y;
            const float ob = xb[i] * cs.x + xa[i] * cs.y;
            xa[i] = oa;
            xb[i] = ob;
          }
        }
        if (want_dev) {
          float olda[32], oldb[32];
          load_row32(dst + half * 32, olda);
          load_row32(dst + 64 + half * 32, oldb);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float da = bf16_round(xa[i]) - olda[i];
            const float db = bf16_round(xb[i]) - oldb[i];
            dev += l1 ? (fabsf(da) + fabsf(db)) : (da * da + db * db);
          }
        }
        store_row32(dst + half * 32, xa);
        store_row32(dst + 64 + half * 32, xb);
        if (!is_q && ep.k_peer != nullptr) {
          // fused P->D push: the same row into the decode GPU's slot (NVLink)
          __nv_bfloat16* peer = (is_k ? ep.k_peer : ep.v_peer) + ((size_t)kvh * ep.cache_cap + slot) * 128;
          store_row32(peer + half * 32, xa);
          store_row32(peer + 64 + half * 32, xb);
        }
      }
      if (want_dev && row_ok) {
        ep.dev_part[(size_t)row * (2 * ep.n_kv_heads) + (is_v ? ep.n_kv_heads : 0) + kvh] = dev;
      }
    }
  }
}

// One TMA descriptor per A shard (only maps[0] is used by ordinary GEMMs).
struct AMaps {
  CUtensorMap m[kMaxShards];
};

// Tile t -> (m-tile, n-tile).  The m-tiles of one n-tile are consecutive, so
// CTAs working at the same time share B k-blocks through L2.  With a
// row-sharded A the m-tiles are rotated so that every rank starts on its own
// shard while its peers finish theirs.  With `round_rotate` (256-row tiles,
// whose last m-tile may be half empty) the m-tile order is rotated by the
// schedule round t / grid, so a CTA that took a full tile in one round takes
// the short one in the next; grid % num_m == 0 keeps every n-tile's units
// inside one round, which keeps the map one to one.
__device__ __forceinline__ void tile_coords(int t, int num_m, const AShards& sh, int& tm, int& tn,
                                            bool round_rotate = false, int grid = 1) {
  tm = t % num_m;
  tn = t / num_m;
  if (sh.n > 1) tm = (tm + sh.own * (sh.rows / kGemmBM)) % num_m;
  if (round_rotate && grid > 0 && grid % num_m == 0) tm = (tm + t / grid) % num_m;
}

// Bounded acquire-poll of a peer shard's ready flag (written over NVLink).
__device__ __forceinline__ bool wait_shard_ready(const int* flag, int epoch, int* status) {
  const long long start = clock64();
  while (true) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= epoch) return true;
    if (clock64() - start > kSpinLimitCycles) {
      report_status(status, kStatusTimeoutPeerFlag);
      return false;
    }
    if (status != nullptr && *((volatile int*)status) != 0) return false;  // another wait failed
    __nanosleep(64);
  }
}

template <int BN, int EPI, int ACC>
__global__ void __launch_bounds__(GemmCfg<BN, ACC>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ AMaps amaps,
                   const __grid_constant__ CUtensorMap tmap_b, int M, int N, int K,
                   GemmEpilogue ep, AShards shards, int splits, int* status) {
  using Cfg = GemmCfg<BN, ACC>;
  constexpr int S = Cfg::kStages;
  constexpr int BM = Cfg::kBM;
  constexpr int NB = Cfg::kNumBuf;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GemmBarriers* bars = reinterpret_cast<GemmBarriers*>(smem + S * Cfg::kStageBytes);
  uint32_t* epi_stage = reinterpret_cast<uint32_t*>(smem + S * Cfg::kStageBytes + 256);

  const int warp = warp_id();
  const int lane = lane_id();
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_kb = (K + kGemmBK - 1) / kGemmBK;
  // work unit u = (tile u / splits, K-slice u % splits); slice ks covers
  // k-blocks [ks * num_kb / splits, (ks + 1) * num_kb / splits)
  const int num_units = num_m * num_n * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], Cfg::kEpiWarps);
    }
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    for (int r = 0; r < shards.n; ++r) tma_prefetch_desc(&amaps.m[r]);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  // the A rows (and the residual / cache rows of the epilogues) come from the
  // previous kernel; the setup above overlapped its tail
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued_phase[8];
      bool issued[8];
      for (int s = 0; s < S; ++s) issued[s] = false, issued_phase[s] = 0;
      bool ok = true;
      unsigned confirmed = 1u << shards.own;  // shards known to be ready
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int tm, tn;
        tile_coords(u / splits, num_m, shards, tm, tn, ACC == 2, gridDim.x / splits);
        const int ks = u % splits;
        const int kb0 = ks * num_kb / splits, kb1 = (ks + 1) * num_kb / splits;
        int map = 0, ay = tm * BM;
        if (shards.n > 1) {
          map = ay / shards.rows;
          ay -= map * shards.rows;
          if (!((confirmed >> map) & 1u) && shards.ready != nullptr) {
            if (!wait_shard_ready(shards.ready + map, shards.epoch, status)) {
              ok = false;
              break;
            }
            confirmed |= 1u << map;
          }
        }
        // L2 prefetch runs kPrefetchKb k-blocks ahead of the loads: the
        // weight tiles stream from DRAM into L2 while earlier stages are
        // consumed, so each tiled load waits on an L2 hit instead of DRAM
        for (int kb = kb0; kb < kb0 + kPrefetchKb && kb < kb1; ++kb) {
          tma_prefetch_l2_2d(&tmap_b, kb * kGemmBK, tn * BN);
          tma_prefetch_l2_2d(&amaps.m[map], kb * kGemmBK, ay);
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (kb + kPrefetchKb < kb1) {
            tma_prefetch_l2_2d(&tmap_b, (kb + kPrefetchKb) * kGemmBK, tn * BN);
            tma_prefetch_l2_2d(&amaps.m[map], (kb + kPrefetchKb) * kGemmBK, ay);
          }
          if (!mbar_wait(&bars->empty[stage], phase ^ 1, status, kStatusTimeoutSmemEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          mbar_arrive_expect_tx(&bars->full[stage], Cfg::kStageBytes);
          tma_load_2d(sa, &amaps.m[map], &bars->full[stage], kb * kGemmBK, ay);
          tma_load_2d(sb, &tmap_b, &bars->full[stage], kb * kGemmBK, tn * BN);
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == S) stage = 0, phase ^= 1;
        }
      }
      // Drain: every TMA load issued must have landed before the CTA exits.
      for (int s = 0; s < S; ++s)
        if (issued[s]) mbar_wait(&bars->full[s], issued_phase[s], status, kStatusTimeoutDrain);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kGemmBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      bool any = false;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++local) {
        const int ks = u % splits;
        const int kb0 = ks * num_kb / splits, kb1 = (ks + 1) * num_kb / splits;
        const int buf = local % NB;
        const uint32_t tphase = (uint32_t)(local / NB) & 1u;
        // accumulators with valid rows in this tile (ACC = 2: the last m-tile may need one)
        int n_acc = 1;
        if constexpr (ACC == 2) {
          int tm, tn;
          tile_coords(u / splits, num_m, shards, tm, tn, true, gridDim.x / splits);
          n_acc = M - tm * BM > kGemmBM ? 2 : 1;
        }
        if (!mbar_wait(&bars->tmem_empty[buf], tphase ^ 1, status, kStatusTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tacc = tmem_base + buf * ACC * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&bars->full[stage], phase, status, kStatusTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t bd = make_desc_kmajor_sw128(sb + k * 32);
#pragma unroll
            for (int a = 0; a < ACC; ++a) {
              // rows 128a.. of the A k-block start 128a * 128 bytes in (a whole number of 8-row atoms)
              if (a < n_acc) {
                const uint64_t ad = make_desc_kmajor_sw128(sa + a * (kGemmBM * 128) + k * 32);
                tc_mma_f16(tacc + a * BN, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
              }
            }
          }
          any = true;
          tc_commit(&bars->empty[stage]);
          if (++stage == S) stage = 0, phase ^= 1;
        }
        if (!ok) break;
        tc_commit(&bars->tmem_full[buf]);
      }
      if (any) {
        // Wait for every MMA of this CTA to complete before teardown.
        tc_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, status, kStatusTimeoutDrain);
      }
    }
  } else {
    // ---------------- Epilogue (warps 2..) ----------------
    const int quarter = warp & 3;     // TMEM lane quarter this warp may access
    const int acc = (warp - 2) >> 2;  // accumulator this warp drains (ACC = 2: warps 6.. take the second)
    int local = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(u / splits, num_m, shards, tm, tn, ACC == 2, gridDim.x / splits);
      const int buf = local % NB;
      const uint32_t tphase = (uint32_t)(local / NB) & 1u;
      if (!mbar_wait(&bars->tmem_full[buf], tphase, status, kStatusTimeoutTmemFull)) break;
      tc_fence_after();
      const int row0 = tm * BM + acc * kGemmBM;
      if (row0 < M) {  // the second accumulator of a short last m-tile holds nothing
        const uint32_t tacc = tmem_base + ((uint32_t)(quarter * 32) << 16) + (buf * ACC + acc) * BN;
        gemm_epilogue_tile<BN, EPI>(ep, tacc, row0 + quarter * 32 + lane, tn, M, N, epi_stage + quarter * (32 * 33),
                                    u % splits);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tmem_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------
static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

bool make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                       bool swizzle128) {
  PFN_encodeTiled enc = get_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t mid, uint64_t outer,
                       uint64_t mid_stride_elems, uint64_t outer_stride_elems, uint32_t box_inner,
                       uint32_t box_mid) {
  PFN_encodeTiled enc = get_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[3] = {inner, mid, outer};
  cuuint64_t strides[2] = {mid_stride_elems * 2, outer_stride_elems * 2};
  cuuint32_t box[3] = {box_inner, box_mid, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, int EPI, int ACC>
static cudaError_t launch_gemm(const GemmArgs& g, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, ACC>;
  AMaps maps;
  CUtensorMap tb;
  AShards sh = g.shards;
  if (sh.n <= 1) {
    sh.n = 1;
    sh.rows = g.M;
    sh.own = 0;
    sh.ready = nullptr;
    if (!make_tmap_2d_bf16(&maps.m[0], g.a, g.K, g.M, g.lda, kGemmBK, Cfg::kBM, true))
      return cudaErrorInvalidValue;
  } else {
    if (ACC != 1) return cudaErrorInvalidValue;  // an m-tile must not span two shards
    if (sh.n > kMaxShards || sh.rows % kGemmBM != 0 || sh.rows * sh.n != g.M) return cudaErrorInvalidValue;
    for (int r = 0; r < sh.n; ++r)
      if (!make_tmap_2d_bf16(&maps.m[r], g.a_shards[r], g.K, sh.rows, g.lda, kGemmBK, kGemmBM, true))
        return cudaErrorInvalidValue;
  }
  if (!make_tmap_2d_bf16(&tb, g.b, g.K, g.N, g.ldb, kGemmBK, BN, true)) return cudaErrorInvalidValue;
  auto kern = gemm_tc_kernel<BN, EPI, ACC>;
  ensure_smem_attr(kern, Cfg::kSmemBytes);
  const int splits = EPI == EPI_PARTIAL ? (g.splits < 1 ? 1 : g.splits) : 1;
  if (splits > (g.K + kGemmBK - 1) / kGemmBK) return cudaErrorInvalidValue;  // every slice needs a k-block
  const int num_units = ((g.M + Cfg::kBM - 1) / Cfg::kBM) * ((g.N + BN - 1) / BN) * splits;
  int grid = num_units < g.num_sms ? num_units : g.num_sms;
  if (grid < 1) grid = 1;
  return launch_pdl(kern, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, maps, tb, g.M, g.N, g.K, g.ep,
                    sh, splits, g.status);
}

template <int EPI>
static cudaError_t launch_gemm_bn(const GemmArgs& g, cudaStream_t stream) {
  if (g.rows_per_tile == 256) {
    if constexpr (EPI == EPI_RS) {
      return cudaErrorInvalidValue;
    } else {
      return g.bn == 256 ? launch_gemm<256, EPI, 2>(g, stream) : cudaErrorInvalidValue;
    }
  }
  return g.bn == 128 ? launch_gemm<128, EPI, 1>(g, stream) : launch_gemm<256, EPI, 1>(g, stream);
}

cudaError_t gemm_bf16_tc(const GemmArgs& g, cudaStream_t stream) {
  if (g.rows_per_tile != 128 && g.rows_per_tile != 256 && g.rows_per_tile != 0) return cudaErrorInvalidValue;
  switch (g.epi) {
    case EPI_STORE: return launch_gemm_bn<EPI_STORE>(g, stream);
    case EPI_RESIDUAL: return launch_gemm_bn<EPI_RESIDUAL>(g, stream);
    case EPI_SWIGLU: return launch_gemm_bn<EPI_SWIGLU>(g, stream);
    case EPI_QKV: return launch_gemm_bn<EPI_QKV>(g, stream);
    case EPI_RS: return launch_gemm_bn<EPI_RS>(g, stream);
    case EPI_PARTIAL: return launch_gemm_bn<EPI_PARTIAL>(g, stream);
  }
  return cudaErrorInvalidValue;
}

// Estimated device cycles of a GEMM with the given tile shape: every CTA's
// units summed (static round-robin schedule), a unit costing the larger of
// its MMA cycles (512 per 128x256x64 k-block and accumulator) and its
// L2->SM bytes at the CTAs' share of ~15 TB/s of L2 bandwidth.  Only the
// ratio between shapes is used.
double gemm_cost_estimate(int M, int N, int K, int bn, int rows_per_tile, int splits, int num_sms) {
  const int acc = rows_per_tile / kGemmBM;
  const int num_m = (M + rows_per_tile - 1) / rows_per_tile;
  const int num_n = (N + bn - 1) / bn;
  const int units = num_m * num_n * (splits < 1 ? 1 : splits);
  const int grid = units < num_sms ? units : num_sms;
  const double kb = (double)((K + kGemmBK - 1) / kGemmBK) / (splits < 1 ? 1 : splits);
  const double share = std::min(128.0, 15.0e12 / (grid * 1.9e9));  // bytes per cycle per CTA
  const int sp = splits < 1 ? 1 : splits;
  const int tgrid = grid / sp;
  auto unit_cost = [&](int u) {
    const int t = u / sp;
    int tm = t % num_m;
    if (acc == 2 && tgrid > 0 && tgrid % num_m == 0) tm = (tm + t / tgrid) % num_m;
    const int rows = std::min(rows_per_tile, M - tm * rows_per_tile);
    const int n_acc = acc == 2 && rows <= kGemmBM ? 1 : acc;
    const double mma = kb * 512.0 * n_acc * bn / 256.0;
    const double l2 = kb * (double)(std::min(rows, rows_per_tile) + bn) * 128.0 / share;
    return std::max(mma, l2);
  };
  double worst = 0.0;
  for (int c = 0; c < grid; ++c) {
    double t = 0.0;
    for (int u = c; u < units; u += grid) t += unit_cost(u);
    worst = std::max(worst, t);
  }
  return worst;
}

// Sum of the K-slice partials in slice order, then the STORE or RESIDUAL
// epilogue (out = residual + bf16(sum), the HF rounding order).
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M, int N,
                                     const __nv_bfloat16* residual, int ldr, __nv_bfloat16* out, int ldo) {
  pdl_wait();
  pdl_launch_dependents();
  const int n4 = N / 4;
  const long long total = (long long)M * n4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / n4), c = (int)(i % n4) * 4;
    float4 acc = __ldcs(reinterpret_cast<const float4*>(ws + (size_t)row * N + c));
    for (int s = 1; s < splits; ++s) {
      const float4 p = __ldcs(reinterpret_cast<const float4*>(ws + ((size_t)s * M + row) * N + c));
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    float v[4] = {acc.x, acc.y, acc.z, acc.w};
    if (residual != nullptr) {
      const uint2 rr = *reinterpret_cast<const uint2*>(residual + (size_t)row * ldr + c);
      const float2 r0 = unpack_bf16x2(rr.x), r1 = unpack_bf16x2(rr.y);
      v[0] = r0.x + bf16_round(v[0]);
      v[1] = r0.y + bf16_round(v[1]);
      v[2] = r1.x + bf16_round(v[2]);
      v[3] = r1.y + bf16_round(v[3]);
    }
    *reinterpret_cast<uint2*>(out + (size_t)row * ldo + c) =
        make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  }
}

// Split-K reduce + RESIDUAL epilogue + the RMSNorm of each finished row (the
// next projection's input), one CTA of 256 threads per row.  Thread t owns
// the 8-column chunks t, t + 256, ...; the sum of squares runs over the
// bf16-rounded outputs in exactly the order of rmsnorm_kernel (same chunk
// ownership, same pair order, same warp / block reduction), so norm_out is
// bit-identical to running rmsnorm_bf16 on the stored rows.
constexpr int kRedNormMaxChunks = 4;  // N <= 256 threads * 4 chunks * 8 = 8192
__global__ void __launch_bounds__(256) splitk_reduce_norm_kernel(const float* __restrict__ ws, int splits, int M,
                                                                 int N, const __nv_bfloat16* residual, int ldr,
                                                                 __nv_bfloat16* out, int ldo,
                                                                 const __nv_bfloat16* norm_w, float eps,
                                                                 __nv_bfloat16* norm_out, int ldn) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int n8 = N / 8;
  uint32_t keep[kRedNormMaxChunks][4];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kRedNormMaxChunks; ++k) {
    const int c = threadIdx.x + k * 256;
    if (c >= n8) break;
    float acc[8];
    {
      const float4 a0 = __ldcs(reinterpret_cast<const float4*>(ws + (size_t)row * N + 8 * c));
      const float4 a1 = __ldcs(reinterpret_cast<const float4*>(ws + (size_t)row * N + 8 * c) + 1);
      acc[0] = a0.x; acc[1] = a0.y; acc[2] = a0.z; acc[3] = a0.w;
      acc[4] = a1.x; acc[5] = a1.y; acc[6] = a1.z; acc[7] = a1.w;
    }
    for (int s = 1; s < splits; ++s) {
      const float* src = ws + ((size_t)s * M + row) * N + 8 * c;
      const float4 p0 = __ldcs(reinterpret_cast<const float4*>(src));
      const float4 p1 = __ldcs(reinterpret_cast<const float4*>(src) + 1);
      acc[0] += p0.x; acc[1] += p0.y; acc[2] += p0.z; acc[3] += p0.w;
      acc[4] += p1.x; acc[5] += p1.y; acc[6] += p1.z; acc[7] += p1.w;
    }
    const uint4 rr = *reinterpret_cast<const uint4*>(residual + (size_t)row * ldr + 8 * c);
    const uint32_t ri[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 r = unpack_bf16x2(ri[q]);
      keep[k][q] = pack_bf16x2(r.x + bf16_round(acc[2 * q]), r.y + bf16_round(acc[2 * q + 1]));
      const float2 f = unpack_bf16x2(keep[k][q]);
      ss += f.x * f.x + f.y * f.y;
    }
    *reinterpret_cast<uint4*>(out + (size_t)row * ldo + 8 * c) = make_uint4(keep[k][0], keep[k][1], keep[k][2], keep[k][3]);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rinv = rsqrtf(red[0] / (float)N + eps);
#pragma unroll
  for (int k = 0; k < kRedNormMaxChunks; ++k) {
    const int c = threadIdx.x + k * 256;
    if (c >= n8) break;
    const uint4 g = *reinterpret_cast<const uint4*>(norm_w + 8 * c);
    const uint32_t gi[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 xf = unpack_bf16x2(keep[k][q]), gf = unpack_bf16x2(gi[q]);
      o[q] = pack_bf16x2(gf.x * bf16_round(xf.x * rinv), gf.y * bf16_round(xf.y * rinv));
    }
    *reinterpret_cast<uint4*>(norm_out + (size_t)row * ldn + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

cudaError_t splitk_reduce_norm(const float* ws, int splits, int M, int N, const __nv_bfloat16* residual, int ldr,
                               __nv_bfloat16* out, int ldo, const __nv_bfloat16* norm_w, float eps,
                               __nv_bfloat16* norm_out, int ldn, cudaStream_t stream) {
  if (N % 8 != 0 || N / 8 > 256 * kRedNormMaxChunks || splits < 1 || residual == nullptr) return cudaErrorInvalidValue;
  if (M <= 0) return cudaSuccess;
  return launch_pdl(splitk_reduce_norm_kernel, dim3(M), dim3(256), 0, stream, ws, splits, M, N, residual, ldr, out,
                    ldo, norm_w, eps, norm_out, ldn);
}

cudaError_t splitk_reduce(const float* ws, int splits, int M, int N, const __nv_bfloat16* residual, int ldr,
                          __nv_bfloat16* out, int ldo, cudaStream_t stream) {
  if (N % 4 != 0 || splits < 1) return cudaErrorInvalidValue;
  const long long total = (long long)M * (N / 4);
  const int grid = (int)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
  return launch_pdl(splitk_reduce_kernel, dim3(grid < 1 ? 1 : grid), dim3(256), 0, stream, ws, splits, M, N, residual,
                    ldr, out, ldo);
}

}  // namespace sc
