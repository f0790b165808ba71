// Peer-memory plumbing for the prefill -> decode KV push over NVLink.
//
//   shared buffers   cudaMalloc'd device memory exported with a CUDA IPC
//                    handle; the peer process maps it with
//                    cudaIpcOpenMemHandle (plain peer mapping: no NVLink
//                    multicast object is created, so a dying peer cannot
//                    fault this GPU through a multicast binding)
//   signal           after the writes it orders (previous kernels on the
//                    stream), publish `value` into a flag word that lives in
//                    the peer's memory: system-scope fence + release store
//   wait             bounded spin (acquire loads, globaltimer deadline) until
//                    a local flag word reaches a target; on time-out it
//                    records an error code in a status word and returns, so
//                    the stream and the context stay usable
// The K/V stores themselves are fused into the QKV GEMM epilogue
// (gemm_tc.cu, EPI_QKV with peer pointers).
#include "common.cuh"
#include "kernels.h"

namespace sc {

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__global__ void peer_signal_kernel(int* flag, int value, const int* value_src,
                                   unsigned long long* stamp) {
  if (threadIdx.x == 0) {
    if (value_src != nullptr) value = *value_src;
    __threadfence_system();
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
    if (stamp != nullptr) *stamp = global_ns();
  }
}

__global__ void wait_flag_kernel(const int* flag, int target, long long timeout_ns, int* status,
                                 unsigned long long* stamp) {
  if (threadIdx.x != 0) return;
  // an earlier wait on this status already failed: fail fast instead of
  // spending another full time-out (the host raises at its next check)
  if (status != nullptr && *((volatile int*)status) != 0) return;
  const unsigned long long start = global_ns();
  while (true) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= target) break;
    if ((long long)(global_ns() - start) > timeout_ns) {
      report_status(status, kStatusTimeoutPeerFlag);
      return;
    }
    __nanosleep(200);
  }
  if (stamp != nullptr) *stamp = global_ns();
}

struct FlagList {
  int* addr[kMaxShards];
  int n;
};

// One launch releases `value` into up to 8 flag words (one per rank).
__global__ void peer_signal_many_kernel(FlagList flags, int value) {
  if (threadIdx.x == 0) __threadfence_system();
  __syncwarp();
  if (threadIdx.x < flags.n)
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flags.addr[threadIdx.x]), "r"(value) : "memory");
}

cudaError_t peer_signal_many(int* const* addrs, int n, int value, cudaStream_t stream) {
  if (n < 1 || n > kMaxShards) return cudaErrorInvalidValue;
  FlagList fl{};
  for (int i = 0; i < n; ++i) fl.addr[i] = addrs[i];
  fl.n = n;
  peer_signal_many_kernel<<<1, 32, 0, stream>>>(fl, value);
  return cudaGetLastError();
}

cudaError_t peer_signal(int* flag, int value, const int* value_src, unsigned long long* stamp,
                        cudaStream_t stream) {
  peer_signal_kernel<<<1, 32, 0, stream>>>(flag, value, value_src, stamp);
  return cudaGetLastError();
}

cudaError_t wait_flag(const int* flag, int target, long long timeout_ns, int* status,
                      unsigned long long* stamp, cudaStream_t stream) {
  wait_flag_kernel<<<1, 32, 0, stream>>>(flag, target, timeout_ns, status, stamp);
  return cudaGetLastError();
}

// ------------------------------------------------------------ rs_reduce
// One CTA per owned row.  Thread 0 waits (bounded) for every sender's flag,
// then the CTA sums the tp fp32 partials in rank order, adds the residual with
// the HF rounding order (residual + bf16(sum)), and optionally emits the
// RMSNorm of the new row for the next projection.
constexpr int kRsThreads = 256;
constexpr int kRsMaxVec = 8;  // float4 per thread: N <= 8192

__global__ void __launch_bounds__(kRsThreads) rs_reduce_kernel(RsReduceArgs a) {
  __shared__ int s_fail;
  __shared__ float red[kRsThreads / 32];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  // launched programmatically after the partial-sending kernel: the flags
  // (acquire) order every partial, including this rank's own, so the CTAs
  // can sit resident and poll while that kernel finishes; the next kernel
  // may launch now and prefetch its weights (it waits before reading ours)
  pdl_launch_dependents();
  if (tid == 0) {
    s_fail = (a.status != nullptr && *((volatile int*)a.status) != 0) ? 1 : 0;  // fail fast
    const int epoch = a.epoch_ptr ? *a.epoch_ptr * a.epoch_mul + a.epoch : a.epoch;
    const unsigned long long start = global_ns();
    for (int s = 0; s < a.tp && !s_fail; ++s) {
      while (true) {
        int v;
        asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(a.flags + s) : "memory");
        if (v >= epoch) break;
        if ((long long)(global_ns() - start) > a.timeout_ns) {
          report_status(a.status, kStatusTimeoutPeerFlag);
          s_fail = 1;
          break;
        }
        __nanosleep(100);
      }
    }
  }
  __syncthreads();
  if (s_fail) return;
  pdl_wait();  // the residual row and the output buffers: the predecessor has completed
  // column block of this CTA (several blocks per row only without the norm,
  // which needs the whole row)
  const int nvec_row = a.N / 4;
  const int per_block = (nvec_row + gridDim.y - 1) / gridDim.y;
  const int cbase = blockIdx.y * per_block;
  const int nvec = min(nvec_row, cbase + per_block);
  float vals[kRsMaxVec][4];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kRsMaxVec; ++i) {
    const int c = cbase + tid + i * kRsThreads;
    if (c >= nvec) break;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < a.tp; ++s) {
      const size_t off = ((size_t)s * a.rows + row) * a.N;
      if (a.recv_bf16) {
        const uint2 p = __ldcg(reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(a.recv) + off) + c);
        const float2 p0 = unpack_bf16x2(p.x), p1 = unpack_bf16x2(p.y);
        acc.x += p0.x; acc.y += p0.y; acc.z += p1.x; acc.w += p1.y;
      } else {
        const float4 p = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.recv) + off) + c);
        acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
      }
    }
    const uint2 rr = *reinterpret_cast<const uint2*>(a.residual + (size_t)row * a.N + 4 * c);
    const float2 r0 = unpack_bf16x2(rr.x), r1 = unpack_bf16x2(rr.y);
    vals[i][0] = bf16_round(r0.x + bf16_round(acc.x));
    vals[i][1] = bf16_round(r0.y + bf16_round(acc.y));
    vals[i][2] = bf16_round(r1.x + bf16_round(acc.z));
    vals[i][3] = bf16_round(r1.y + bf16_round(acc.w));
    *reinterpret_cast<uint2*>(a.out + (size_t)row * a.N + 4 * c) =
        make_uint2(pack_bf16x2(vals[i][0], vals[i][1]), pack_bf16x2(vals[i][2], vals[i][3]));
    ss += vals[i][0] * vals[i][0] + vals[i][1] * vals[i][1] + vals[i][2] * vals[i][2] +
          vals[i][3] * vals[i][3];
  }
  if (a.norm_w == nullptr) return;
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kRsThreads / 32; ++w) tot += red[w];
  const float rinv = rsqrtf(tot / (float)a.N + a.eps);
#pragma unroll
  for (int i = 0; i < kRsMaxVec; ++i) {
    const int c = cbase + tid + i * kRsThreads;
    if (c >= nvec) break;
    const uint2 gw = *reinterpret_cast<const uint2*>(a.norm_w + 4 * c);
    const float2 g0 = unpack_bf16x2(gw.x), g1 = unpack_bf16x2(gw.y);
    *reinterpret_cast<uint2*>(a.norm_out + (size_t)row * a.N + 4 * c) =
        make_uint2(pack_bf16x2(g0.x * bf16_round(vals[i][0] * rinv), g0.y * bf16_round(vals[i][1] * rinv)),
                   pack_bf16x2(g1.x * bf16_round(vals[i][2] * rinv), g1.y * bf16_round(vals[i][3] * rinv)));
  }
}

cudaError_t rs_reduce(const RsReduceArgs& a, cudaStream_t stream) {
  if (a.N % 4 != 0 || a.N / 4 > kRsThreads * kRsMaxVec || a.tp < 1 || a.rows < 1) return cudaErrorInvalidValue;
  // few rows (decode, verify): spread each row over column blocks of 256
  // float4 so the tp partials are summed by many SMs; the fused RMSNorm
  // needs whole rows and keeps one CTA per row
  int blocks = 1;
  if (a.norm_w == nullptr && a.rows < 64) blocks = (a.N / 4 + kRsThreads - 1) / kRsThreads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.rows, blocks, 1);
  cfg.blockDim = dim3(kRsThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rs_reduce_kernel, a);
}

}  // namespace sc
