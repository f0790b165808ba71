// Skinny GEMM on the tensor cores for a few token rows (batched verification,
// small decode batches, drafter-trunk rows): out[m, n] = sum_k x[m, k] * w[n, k], M <= 64.
//
// At M <= 16 the work is a weight stream; the CUDA-core GEMV (gemv.cu) keeps
// up with HBM only at M = 1-2 because every extra row costs an unpack and
// FMAs per weight.  Here the roles are swapped so the tensor core does the
// rows: the weight tile is the 128-row A operand (TMA, 128-byte swizzle,
// `tcgen05.mma.cta_group::1.kind::f16` with M = 128), the token rows padded to
// N = 16 (M <= 16), 32 (M <= 32) or 64 (M <= 64) are the B operand (TMA zero-fills rows
// >= M), and the 128 x N fp32 accumulator lives in TMEM (two buffers).  Work
// units are (128-row weight tile, K slice) so that ~one unit per SM streams
// its slice with a deep (10-stage) TMA pipeline; each unit writes its fp32
// partial tile to a workspace [slice][token row][weight row], and a small reduce kernel sums the K slices
// in a fixed order and applies the epilogue (store, residual add with the
// HF rounding order, SwiGLU over 128-row interleaved gate/up blocks).  The
// result of a row m does not depend on M (columns never mix in the MMA and
// the K split depends on N and K only).
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer (one
// elected lane), warps 2-5 epilogue (TMEM lane quarter = warp % 4).  Every
// wait is bounded (mbar_wait) and reports through the status word.
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {
constexpr int kSkBM = 128;  // weight rows per tile (MMA M)
constexpr int kSkBK = 64;   // 128 bytes of bf16 per row
constexpr int kSkStages = 10;
constexpr int kSkABytes = kSkBM * kSkBK * 2;  // 16 KB
constexpr int kSkThreads = 192;

// BN = token rows padded to the MMA N: 16 (M <= 16), 32 (M <= 32) or 64 (M <= 64)
template <int BN>
struct SkCfg {
  static constexpr int kBBytes = BN * kSkBK * 2;  // 2 / 4 / 8 KB
  static constexpr int kStageBytes = kSkABytes + kBBytes;
  static constexpr int kStages = BN == 64 ? 8 : kSkStages;  // 8 x 24 KB fits shared memory
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
  static constexpr uint32_t kTmemCols = BN == 16 ? 32 : 2 * BN;  // two accumulators, power of two >= 32
};

struct alignas(8) SkBars {
  uint64_t full[kSkStages];
  uint64_t empty[kSkStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
};

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
}  // namespace

template <int BN>
__global__ void __launch_bounds__(kSkThreads, 1)
    skinny_mma_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                      int M, int N, int K, int splits, float* ws, int* status) {
  using Cfg = SkCfg<BN>;
  constexpr int kSkStageBytes = Cfg::kStageBytes;
  constexpr int kSkStages = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SkBars* bars = reinterpret_cast<SkBars*>(smem + kSkStages * kSkStageBytes);
  const int warp = warp_id(), lane = lane_id();
  const int tiles = (N + kSkBM - 1) / kSkBM;
  const int num_kb = (K + kSkBK - 1) / kSkBK;
  const int units = tiles * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSkStages; ++s) mbar_init(&bars->full[s], 1), mbar_init(&bars->empty[s], 1);
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
    tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  pdl_wait();  // x comes from the previous kernel
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool issued[kSkStages];
      uint32_t issued_phase[kSkStages];
      for (int s = 0; s < kSkStages; ++s) issued[s] = false, issued_phase[s] = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int tile = u / splits, ks = u % splits;
        const int kb0 = ks * num_kb / splits, kb1 = (ks + 1) * num_kb / splits;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&bars->empty[stage], phase ^ 1, status, kStatusTimeoutSmemEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * kSkStageBytes;
          mbar_arrive_expect_tx(&bars->full[stage], kSkStageBytes);
          tma_load_2d(sa, &tmap_w, &bars->full[stage], kb * kSkBK, tile * kSkBM);
          tma_load_2d(sa + kSkABytes, &tmap_x, &bars->full[stage], kb * kSkBK, 0);
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == kSkStages) stage = 0, phase ^= 1;
        }
      }
      for (int s = 0; s < kSkStages; ++s)
        if (issued[s]) mbar_wait(&bars->full[s], issued_phase[s], status, kStatusTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kSkBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true, any = false;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++local) {
        const int ks = u % splits;
        const int kb0 = ks * num_kb / splits, kb1 = (ks + 1) * num_kb / splits;
        const int buf = local & 1;
        const uint32_t tphase = (local >> 1) & 1;
        if (!mbar_wait(&bars->tmem_empty[buf], tphase ^ 1, status, kStatusTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tacc = tmem_base + buf * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&bars->full[stage], phase, status, kStatusTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kSkStageBytes);
          const uint32_t sb = sa + kSkABytes;
#pragma unroll
          for (int k = 0; k < kSkBK / 16; ++k)
            tc_mma_f16(tacc, make_desc_kmajor_sw128(sa + k * 32), make_desc_kmajor_sw128(sb + k * 32), idesc,
                       (kb != kb0 || k != 0) ? 1u : 0u);
          any = true;
          tc_commit(&bars->empty[stage]);
          if (++stage == kSkStages) stage = 0, phase ^= 1;
        }
        if (!ok) break;
        tc_commit(&bars->tmem_full[buf]);
      }
      if (any) {
        tc_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, status, kStatusTimeoutDrain);
      }
    }
  } else {
    const int quarter = warp & 3;
    int local = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
      const int tile = u / splits, ks = u % splits;
      const int buf = local & 1;
      const uint32_t tphase = (local >> 1) & 1;
      if (!mbar_wait(&bars->tmem_full[buf], tphase, status, kStatusTimeoutTmemFull)) break;
      tc_fence_after();
      uint32_t r[BN];
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN;
      if constexpr (BN == 16) {
        tmem_ld_32x32b_x16(taddr, r);
      } else {
#pragma unroll
        for (int h = 0; h < BN / 32; ++h)
          tmem_ld_32x32b_x32(taddr + h * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[h * 32]));
      }
      tmem_ld_wait();
      const int row = tile * kSkBM + quarter * 32 + lane;
      if (row < N) {
        // partials laid out [slice][token row m][weight row n]: a warp's 32
        // weight rows are 128 contiguous bytes per token row, and the reduce
        // kernel reads them back along n with coalesced loads
        float* d = ws + (size_t)ks * M * N + row;
#pragma unroll
        for (int m = 0; m < BN; ++m)
          if (m < M) d[(size_t)m * N] = __uint_as_float(r[m]);
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

// Sum the K slices in order and apply the epilogue; one thread per (row m, output j)
// (QKV: per (row, rotation pair)).  No thread leaves before the block barrier of
// the all-reduce publication.
__global__ void skinny_reduce_kernel(SkinnyArgs a) {
  __shared__ int s_last;
  pdl_wait();
  pdl_launch_dependents();
  const int outs = (a.epi == SKINNY_SWIGLU || a.epi == SKINNY_QKV) ? a.N / 2 : a.N;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = idx < outs * a.M;
  const int m = active ? idx / outs : 0, j = active ? idx % outs : 0;
  auto sum_row = [&](int n) {
    float v = 0.f;
    for (int s = 0; s < a.splits; ++s) v += a.ws[((size_t)s * a.M + m) * a.N + n];
    return v;
  };
  if (active) {
    if (a.epi == SKINNY_SWIGLU) {
      const int blk = j >> 7, i = j & 127;
      const float g = bf16_round(sum_row(blk * 256 + i)), u = bf16_round(sum_row(blk * 256 + 128 + i));
      a.out[(size_t)m * a.ldo + j] = __float2bfloat16_rn(bf16_round(silu_f(g)) * u);
    } else if (a.epi == SKINNY_QKV) {
      const int head = j >> 6, i = j & 63;
      const int r0 = head * 128 + i;
      const float v0 = sum_row(r0), v1 = sum_row(r0 + 64);
      int pos, slot;
      size_t seq_off = 0;
      if (a.pos_rows != nullptr && a.slot_rows != nullptr) {  // one sequence, per-row position and slot
        pos = a.pos_rows[m];
        slot = a.slot_rows[m];
      } else if (a.pos_rows != nullptr) {  // batched decode: one sequence per row
        pos = slot = a.pos_rows[m];
        seq_off = (size_t)m * (size_t)a.seq_stride;
      } else {
        pos = *a.pos + m;
        slot = (a.slot != nullptr ? *a.slot : *a.pos) + m;
      }
      const bool is_q = head < a.n_q_heads;
      const bool is_k = !is_q && head < a.n_q_heads + a.n_kv_heads;
      float o0 = v0, o1 = v1;
      if (is_q || is_k) {
        const float2 cs = a.rope_table[(size_t)pos * 64 + i];
        o0 = v0 * cs.x - v1 * cs.y;
        o1 = v1 * cs.x + v0 * cs.y;
      }
      __nv_bfloat16* dst;
      if (is_q) {
        dst = a.q_out + (size_t)m * a.ldq + head * 128;
      } else {
        const int kvh = is_k ? head - a.n_q_heads : head - a.n_q_heads - a.n_kv_heads;
        dst = (is_k ? a.k_cache : a.v_cache) + seq_off + ((size_t)kvh * a.cache_cap + slot) * 128;
      }
      dst[i] = __float2bfloat16_rn(o0);
      dst[i + 64] = __float2bfloat16_rn(o1);
    } else if (a.epi == SKINNY_ALLREDUCE) {
      const float v = sum_row(j);
      for (int r = 0; r < a.ar_tp; ++r) a.ar_dst[r][((size_t)a.ar_sender * a.M + m) * a.N + j] = v;
    } else {
      float out = sum_row(j);
      if (a.epi == SKINNY_RESIDUAL) out = __bfloat162float(a.residual[(size_t)m * a.ldr + j]) + bf16_round(out);
      a.out[(size_t)m * a.ldo + j] = __float2bfloat16_rn(out);
    }
  }
  if (a.epi != SKINNY_ALLREDUCE) return;
  // the last block to finish publishes this rank's partial to every rank
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last) {
    __threadfence_system();
    const int epoch = a.ar_epoch_ptr ? *a.ar_epoch_ptr * a.ar_epoch_mul + a.ar_epoch : a.ar_epoch;
    if ((int)threadIdx.x < a.ar_tp)
      asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(a.ar_flag[threadIdx.x]), "r"(epoch) : "memory");
    if (threadIdx.x == 0) *a.counter = 0u;
  }
}

// One block per row: argmax over bf16 logits, first index on ties (the GEMV
// LM head's rule).
__global__ void row_argmax_kernel(const __nv_bfloat16* logits, int ld, int V, int* out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  pdl_wait();
  pdl_launch_dependents();
  const __nv_bfloat16* row = logits + (size_t)blockIdx.x * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < V / 8; c += blockDim.x) {
    const uint4 u = reinterpret_cast<const uint4*>(row)[c];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(w[q]);
      const int i0 = c * 8 + 2 * q;
      if (f.x > bv || (f.x == bv && i0 < bi)) bv = f.x, bi = i0;
      if (f.y > bv || (f.y == bv && i0 + 1 < bi)) bv = f.y, bi = i0 + 1;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
  }
  if ((threadIdx.x & 31) == 0) sv[threadIdx.x >> 5] = bv, si[threadIdx.x >> 5] = bi;
  __syncthreads();
  if (threadIdx.x == 0) {
    bv = sv[0], bi = si[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) bv = sv[w], bi = si[w];
    out[blockIdx.x] = (bi < 0 || bi >= V) ? 0 : bi;  // all-NaN row: token 0, never out of range
  }
}

cudaError_t row_argmax_bf16(const __nv_bfloat16* logits, int ld, int M, int V, int* out_token, cudaStream_t stream) {
  if (M < 1 || V % 8 != 0 || ld % 8 != 0) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, row_argmax_kernel, logits, ld, V, out_token);
}

// K slices per tile: the smallest split whose units fill the persistent CTAs'
// rounds to >= 90% (units / (rounds * SMs)), at least 4 k-blocks per unit;
// else the best filling found.
int skinny_splits(int N, int K, int num_sms) {
  const int tiles = (N + kSkBM - 1) / kSkBM;
  const int num_kb = (K + kSkBK - 1) / kSkBK;
  const int max_s = num_kb / 4 < 1 ? 1 : (num_kb / 4 > 32 ? 32 : num_kb / 4);
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= max_s; ++s) {
    const int units = tiles * s;
    const int rounds = (units + num_sms - 1) / num_sms;
    const double eff = (double)units / ((double)rounds * num_sms);
    if (eff >= 0.9) return s;
    if (eff > best_eff + 1e-9) best_eff = eff, best = s;
  }
  return best;
}

int skinny_bn(int M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

cudaError_t skinny_gemm(const SkinnyArgs& args, cudaStream_t stream) {
  SkinnyArgs a = args;
  if (a.M < 1 || a.M > 64 || a.K % kSkBK != 0 || a.N % 2 != 0) return cudaErrorInvalidValue;
  a.bn = skinny_bn(a.M);
  if (a.epi == SKINNY_SWIGLU && a.N % 256 != 0) return cudaErrorInvalidValue;
  if (a.epi == SKINNY_QKV && (a.N % 128 != 0 || a.N != (a.n_q_heads + 2 * a.n_kv_heads) * 128))
    return cudaErrorInvalidValue;
  if (a.epi == SKINNY_ALLREDUCE && (a.ar_tp < 1 || a.ar_tp > 8 || a.counter == nullptr)) return cudaErrorInvalidValue;
  CUtensorMap tw, tx;
  if (!make_tmap_2d_bf16(&tw, a.w, a.K, a.N, a.ldw, kSkBK, kSkBM, true)) return cudaErrorInvalidValue;
  if (!make_tmap_2d_bf16(&tx, a.x, a.K, a.M, a.ldx, kSkBK, a.bn, true)) return cudaErrorInvalidValue;
  ensure_smem_attr(skinny_mma_kernel<16>, SkCfg<16>::kSmem);
  ensure_smem_attr(skinny_mma_kernel<32>, SkCfg<32>::kSmem);
  ensure_smem_attr(skinny_mma_kernel<64>, SkCfg<64>::kSmem);
  const int tiles = (a.N + kSkBM - 1) / kSkBM;
  const int units = tiles * a.splits;
  const int grid = units < a.num_sms ? units : a.num_sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kSkThreads, 1, 1);
  cfg.dynamicSmemBytes = a.bn == 16 ? SkCfg<16>::kSmem : (a.bn == 32 ? SkCfg<32>::kSmem : SkCfg<64>::kSmem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e =
      a.bn == 16   ? cudaLaunchKernelEx(&cfg, skinny_mma_kernel<16>, tw, tx, a.M, a.N, a.K, a.splits, a.ws, a.status)
      : a.bn == 32 ? cudaLaunchKernelEx(&cfg, skinny_mma_kernel<32>, tw, tx, a.M, a.N, a.K, a.splits, a.ws, a.status)
                   : cudaLaunchKernelEx(&cfg, skinny_mma_kernel<64>, tw, tx, a.M, a.N, a.K, a.splits, a.ws, a.status);
  if (e != cudaSuccess) return e;
  return skinny_reduce(a, stream);
}

cudaError_t skinny_reduce(const SkinnyArgs& a, cudaStream_t stream) {
  if (a.M < 1 || a.splits < 1 || a.ws == nullptr || a.N % 2 != 0) return cudaErrorInvalidValue;
  if (a.epi == SKINNY_SWIGLU && a.N % 256 != 0) return cudaErrorInvalidValue;
  if (a.epi == SKINNY_QKV && (a.N % 128 != 0 || a.N != (a.n_q_heads + 2 * a.n_kv_heads) * 128))
    return cudaErrorInvalidValue;
  const int outs = ((a.epi == SKINNY_SWIGLU || a.epi == SKINNY_QKV) ? a.N / 2 : a.N) * a.M;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((outs + 255) / 256, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, skinny_reduce_kernel, a);
}

}  // namespace sc
