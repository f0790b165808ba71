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

}  // namespace sc
