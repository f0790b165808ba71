// Shared device helpers for the sm_100a kernels of sparsecache_b200.
//
// Everything here is written directly against the PTX ISA for sm_100a:
// mbarriers, TMA tiled loads (cp.async.bulk.tensor into this CTA's own
// shared memory only), and the tcgen05 family (alloc / mma / commit / ld).
// Every spin-wait is bounded by a clock64 deadline; on expiry the waiting
// thread records an error code in a device status word and the kernel winds
// down instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <mutex>
#include <utility>

namespace sc {

// ----------------------------------------------------------------------------
// Status word written by kernels when a bounded wait expires.
// ----------------------------------------------------------------------------
enum StatusCode : int {
  kStatusOk = 0,
  kStatusTimeoutTmaFull = 1,
  kStatusTimeoutSmemEmpty = 2,
  kStatusTimeoutTmemFull = 3,
  kStatusTimeoutTmemEmpty = 4,
  kStatusTimeoutDrain = 5,
  kStatusTimeoutPeerFlag = 6,
  kStatusBadArgument = 7,
};

// ~1.5 s at 1.9 GHz.  Correct kernels never come close; this only turns a
// protocol bug into an error status instead of a hung GPU.
constexpr long long kSpinLimitCycles = 3000000000LL;

__device__ __forceinline__ void report_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// ----------------------------------------------------------------------------
// Address-space helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one_lane() {
  return (threadIdx.x & 31) == 0;
}

__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

// ----------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], "
      "%1;\n}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], "
      "%2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (after recording `code`) if the phase with the
// given parity did not complete within kSpinLimitCycles.
// try_wait suspends the thread until the phase completes or a hardware time
// limit passes, so the loop wakes as soon as the phase flips; the deadline
// and the shared status word (a global load) are looked at only every 32nd
// round, keeping them off the wake-up path of a handoff.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  for (uint32_t round = 1;; ++round) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((round & 31u) == 0) {
      if (clock64() - start > kSpinLimitCycles) {
        report_status(status, code);
        return false;
      }
      if (status != nullptr && *((volatile int*)status) != 0) {
        // Another role already failed: stop waiting so the kernel can drain.
        return false;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// TMA (tiled, no multicast)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map))
               : "memory");
}

// Load a 2D box whose innermost coordinate is x (elements) and outer is y.
// The caller guarantees x * sizeof(elem) % 16 == 0.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Prefetch a 2D box of a tensor map into L2 (no shared memory, no barrier):
// a later tiled load of the same box then hits L2 instead of DRAM.  Same
// alignment rule on x as the loads.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// Untiled bulk prefetch of [p, p + bytes) into L2 (the copy engine of the
// SM fetches it in the background; nothing waits on it).  p and bytes must be
// multiples of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
               : "memory");
}

// Spread the L2 prefetch of up to two byte ranges over every CTA of a grid:
// CTA b takes the b-th of n_cta equal 16-byte-aligned shares of each range
// and the 32 lanes of the calling warp issue it in 32 KB pieces.
__device__ __forceinline__ void prefetch_l2_share(const void* const* ptr, const long long* bytes, int n_ranges,
                                                  int cta, int n_cta, int lane) {
  constexpr long long kPiece = 32 << 10;
  for (int r = 0; r < n_ranges; ++r) {
    const long long total = bytes[r];
    if (ptr[r] == nullptr || total <= 0) continue;
    const long long share = ((total + n_cta - 1) / n_cta + 15) & ~15LL;
    const long long beg = (long long)cta * share;
    const long long end = beg + share < total ? beg + share : total;
    const char* base = static_cast<const char*>(ptr[r]);
    for (long long off = beg + (long long)lane * kPiece; off < end; off += 32 * kPiece) {
      const long long n = end - off < kPiece ? end - off : kPiece;
      prefetch_l2_bulk(base + off, (unsigned)n);
    }
  }
}

// 3D box: coordinates (x innermost, y, z).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y),
      "r"(z)
      : "memory");
}

// ----------------------------------------------------------------------------
// tcgen05 (5th generation tensor core, accumulators in TMEM)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(smem_result)),
      "r"(ncols)
      : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (bf16 in, f32 acc).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc,
                                           uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Variant whose A operand is read from TMEM (used for P*V in attention).
__device__ __forceinline__ void tc_mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem,
                                                  uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05.mma of this
// thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 columns of 32-bit data: thread t of the warp receives row
// (lane base + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
        "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]),
        "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 16 columns store (registers -> TMEM).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
      "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),
      "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored with the
// 128-byte swizzle: rows of 64 bf16 (128 B), 8-row atoms of 1024 B.  The
// stage buffers are 1024-byte aligned so the base offset field is 0.
//   bits  0-13 start address >> 4
//   bits 16-29 leading byte offset >> 4 (unused for swizzled K-major: 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 61-63 layout: 2 = 128-byte swizzle
__device__ __forceinline__ uint64_t make_desc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Descriptor for an MN-major operand with the 128-byte swizzle: 64 elements
// of the N (or M) dimension are contiguous per 128-byte row, rows advance
// along K, 8-row atoms are 1024 B apart (SBO), and the next 64-element group
// of N lies `lbo_bytes` further on (LBO).
__device__ __forceinline__ uint64_t make_desc_mnmajor_sw128(uint32_t smem_addr,
                                                            uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B, f32 accumulator.
//   bits 4-5 D format (1 = f32); 7-9 A format (1 = bf16); 10-12 B format
//   bit 15 A major (0 = K); bit 16 B major (0 = K, 1 = MN)
//   bits 17-22 N >> 3; bits 24-28 M >> 4
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool b_mn_major = false,
                                                       bool a_mn_major = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// ----------------------------------------------------------------------------
// bf16 helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may start while its predecessor drains.
// Everything before pdl_wait() must not read data the predecessor writes
// (weights are fine); pdl_wait() returns once the predecessor has completed
// and its memory is visible.  Both are no-ops without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 128-bit streaming load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace sc

namespace sc {
// Raise a kernel's dynamic shared-memory limit once per (kernel, device)
// rather than on every launch: the attribute call is host work and must stay
// out of CUDA-graph capture.  Keyed by the kernel's address (template
// instantiations share a signature but are distinct kernels).
template <typename F>
inline void ensure_smem_attr(F* func, int bytes) {
  struct Entry { const void* fn; int dev; int bytes; };
  static Entry table[256];
  static int used = 0;
  // host threads may launch concurrently (one per device, or a plugin's
  // worker threads): the table is shared, so look-up and insert are locked
  static std::mutex lock;
  std::lock_guard<std::mutex> guard(lock);
  int dev = 0;
  cudaGetDevice(&dev);
  const void* key = reinterpret_cast<const void*>(func);
  for (int i = 0; i < used; ++i) {
    if (table[i].fn == key && table[i].dev == dev) {
      if (table[i].bytes < bytes) {
        cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        table[i].bytes = bytes;
      }
      return;
    }
  }
  cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (used < 256) table[used++] = Entry{key, dev, bytes};
}
}  // namespace sc

namespace sc {
// Programmatic dependent launch is on unless SC_PDL=0 (an experiment and
// safety switch: every kernel stays correct without it).
inline bool pdl_enabled() {
  static int enabled = -1;
  if (enabled < 0) {
    const char* e = getenv("SC_PDL");
    enabled = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return enabled != 0;
}

// Launch with programmatic stream serialization when PDL is on: the kernel
// may start while its predecessor drains and must call pdl_wait() before it
// touches anything the predecessor writes or reads.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
}  // namespace sc
