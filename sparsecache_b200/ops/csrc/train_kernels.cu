// K16: AdamW with device-side global-norm clipping, and the data-parallel
// gradient reduce-scatter + AdamW + parameter all-gather over peer memory.
//
// All scalars that change between steps (step count, learning rate, clip
// coefficient) live in device memory, so a captured training step replays
// without host involvement.  Every wait on another rank is a bounded poll of
// a flag word (acquire loads, globaltimer deadline) that records
// kStatusTimeoutPeerFlag and makes the kernel return on expiry.
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {
constexpr int kOptThreads = 256;

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread 0 waits until flags[0..n) >= target; returns false (and records the
// status) on time-out.  The result is broadcast to the block.
__device__ bool block_wait_all(const int* flags, int n, int target, long long timeout_ns, int* status) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_ok = (status != nullptr && *((volatile int*)status) != 0) ? 0 : 1;  // fail fast after a time-out
    const unsigned long long t0 = now_ns();
    for (int s = 0; s < n && s_ok; ++s) {
      while (ld_acquire(flags + s) < target) {
        if ((long long)(now_ns() - t0) > timeout_ns) {
          report_status(status, kStatusTimeoutPeerFlag);
          s_ok = 0;
          break;
        }
        __nanosleep(128);
      }
    }
  }
  __syncthreads();
  return s_ok != 0;
}

__device__ float block_sum(float v) {
  __shared__ float red[kOptThreads / 32];
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kOptThreads / 32; ++w) t += red[w];
  return t;
}

// Returns true in exactly one CTA: the last to finish (after a fence).
__device__ bool last_cta(unsigned* counter) {
  __shared__ unsigned s_ticket;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_ticket = atomicAdd(counter, 1u);
  __syncthreads();
  return s_ticket == gridDim.x - 1;
}

__device__ __forceinline__ void clip_and_bias(float total_sq, float step, const float* hyper, float* st) {
  const float norm = sqrtf(total_sq);
  const float max_norm = hyper[5];
  const float coef = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
  st[0] = step;
  st[1] = 1.f - powf(hyper[1], step);
  st[2] = 1.f - powf(hyper[2], step);
  st[3] = norm;
  st[4] = coef;
}

struct AdamScalars {
  float lr, b1, b2, eps, wd, coef, step_size, bc2_sqrt;
};

__device__ __forceinline__ AdamScalars adam_scalars(const float* hyper, const float* st) {
  AdamScalars s;
  s.lr = hyper[0];
  s.b1 = hyper[1];
  s.b2 = hyper[2];
  s.eps = hyper[3];
  s.wd = hyper[4];
  s.coef = st[4];
  s.step_size = s.lr / st[1];
  s.bc2_sqrt = sqrtf(st[2]);
  return s;
}

// torch.optim.AdamW (non-amsgrad, maximize=False) on one element.
__device__ __forceinline__ float adam_elem(float p, float g, float& m, float& v, const AdamScalars& s) {
  g *= s.coef;
  p *= 1.f - s.lr * s.wd;
  m = m + (1.f - s.b1) * (g - m);
  v = v * s.b2 + (1.f - s.b2) * g * g;
  const float denom = sqrtf(v) / s.bc2_sqrt + s.eps;
  return p - s.step_size * (m / denom);
}
}  // namespace

// ------------------------------------------------------------ single GPU
__global__ void __launch_bounds__(kOptThreads) adamw_norm_kernel(AdamArgs a) {
  float ss = 0.f;
  for (long long i = blockIdx.x * (long long)kOptThreads + threadIdx.x; i < a.n;
       i += (long long)gridDim.x * kOptThreads) {
    const float g = a.grad[i];
    ss = fmaf(g, g, ss);
  }
  ss = block_sum(ss);
  if (threadIdx.x == 0) a.partial[blockIdx.x] = ss;
  if (!last_cta(a.counter)) return;
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int b = 0; b < (int)gridDim.x; ++b) tot += __ldcg(a.partial + b);
    clip_and_bias(tot, a.state[0] + 1.f, a.hyper, a.state);
    *a.counter = 0u;
  }
}

__global__ void __launch_bounds__(kOptThreads) adamw_update_kernel(AdamArgs a) {
  const AdamScalars s = adam_scalars(a.hyper, a.state);
  for (long long i = blockIdx.x * (long long)kOptThreads + threadIdx.x; i < a.n;
       i += (long long)gridDim.x * kOptThreads) {
    float m = a.exp_avg[i], v = a.exp_avg_sq[i];
    a.param[i] = adam_elem(a.param[i], a.grad[i], m, v, s);
    a.exp_avg[i] = m;
    a.exp_avg_sq[i] = v;
  }
}

cudaError_t adamw_norm(const AdamArgs& a, int grid, cudaStream_t stream) {
  if (a.n < 0 || grid < 1) return cudaErrorInvalidValue;
  adamw_norm_kernel<<<grid, kOptThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t adamw_update(const AdamArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return cudaSuccess;
  const long long blocks = (a.n + kOptThreads - 1) / kOptThreads;
  const int grid = (int)(blocks < 148 * 16 ? blocks : 148 * 16);
  adamw_update_kernel<<<grid, kOptThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

// ------------------------------------------------------------ data parallel
// Mean over ranks of one gradient element, summed in rank order (the same
// bits on every rank whichever kernel reduces it).
__device__ __forceinline__ float rank_mean(const DpArgs& a, long long i) {
  float g = 0.f;
  for (int s = 0; s < a.world; ++s) g += __ldcg(a.grads[s] + i);
  return g * (1.f / (float)a.world);  // each rank's loss is a mean over its rows
}

__global__ void __launch_bounds__(kOptThreads) dp_reduce_norm_kernel(DpArgs a) {
  const int epoch = *a.epoch_ptr;
  // pre_reduced: per-bucket kernels already wrote red_grad (overlapped with
  // the backward); only the sum of squares is left
  if (!a.pre_reduced && !block_wait_all(a.flag_grads, a.world, epoch, a.timeout_ns, a.status)) return;
  const long long base = (long long)a.rank * a.shard;
  long long len = a.n_total - base;
  len = len < 0 ? 0 : (len > a.shard ? a.shard : len);
  float ss = 0.f;
  for (long long i = blockIdx.x * (long long)kOptThreads + threadIdx.x; i < len;
       i += (long long)gridDim.x * kOptThreads) {
    float g;
    if (a.pre_reduced) {
      g = a.red_grad[i];
    } else {
      g = rank_mean(a, base + i);
      a.red_grad[i] = g;
    }
    ss = fmaf(g, g, ss);
  }
  ss = block_sum(ss);
  if (threadIdx.x == 0) a.partial[blockIdx.x] = ss;
  if (!last_cta(a.counter)) return;
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int b = 0; b < (int)gridDim.x; ++b) tot += __ldcg(a.partial + b);
    for (int s = 0; s < a.world; ++s) a.norms[s][a.rank] = tot;
    __threadfence_system();
    for (int s = 0; s < a.world; ++s) st_release(a.peer_flag_norms[s], epoch);
    *a.counter = 0u;
  }
}

__global__ void __launch_bounds__(kOptThreads) dp_adamw_gather_kernel(DpArgs a) {
  const int epoch = *a.epoch_ptr;
  if (!block_wait_all(a.flag_norms, a.world, epoch, a.timeout_ns, a.status)) return;
  __shared__ float s_st[5];
  if (threadIdx.x == 0) {
    float tot = 0.f;  // rank order: the same sum, bit for bit, on every rank
    for (int s = 0; s < a.world; ++s) tot += __ldcg(a.norms[a.rank] + s);
    clip_and_bias(tot, (float)epoch + a.hyper[6], a.hyper, s_st);
  }
  __syncthreads();
  const AdamScalars sc = adam_scalars(a.hyper, s_st);
  const long long base = (long long)a.rank * a.shard;
  long long len = a.n_total - base;
  len = len < 0 ? 0 : (len > a.shard ? a.shard : len);
  const float* own = a.params[a.rank] + base;
  for (long long i = blockIdx.x * (long long)kOptThreads + threadIdx.x; i < len;
       i += (long long)gridDim.x * kOptThreads) {
    float m = a.exp_avg[i], v = a.exp_avg_sq[i];
    const float p = adam_elem(own[i], a.red_grad[i], m, v, sc);
    a.exp_avg[i] = m;
    a.exp_avg_sq[i] = v;
    for (int s = 0; s < a.world; ++s) a.params[s][base + i] = p;
  }
  if (!last_cta(a.counter)) return;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < 5; ++i) a.state[i] = s_st[i];
    __threadfence_system();
    for (int s = 0; s < a.world; ++s) st_release(a.peer_flag_params[s], epoch);
    *a.counter = 0u;
  }
}

// One gradient bucket (flat range [lo, hi)) of the reduce-scatter: after a
// bounded wait until every rank released the bucket's flag for this epoch,
// this rank sums its shard's part of the range over all ranks into red_grad.
// Launched on a side stream while the backward still computes later buckets.
__global__ void __launch_bounds__(kOptThreads) dp_reduce_range_kernel(DpArgs a, const int* flags, long long lo,
                                                                     long long hi) {
  const int epoch = *a.epoch_ptr;
  if (!block_wait_all(flags, a.world, epoch, a.timeout_ns, a.status)) return;
  const long long base = (long long)a.rank * a.shard;
  long long end = a.n_total < base + a.shard ? a.n_total : base + a.shard;
  if (hi < end) end = hi;
  const long long begin = lo > base ? lo : base;
  // 4 elements per thread and iteration when the range and the shard allow 16-byte loads
  const bool vec = ((begin | end | base) & 3) == 0;
  if (vec) {
    const long long n4 = (end - begin) / 4;
    for (long long j = blockIdx.x * (long long)kOptThreads + threadIdx.x; j < n4;
         j += (long long)gridDim.x * kOptThreads) {
      const long long i = begin + 4 * j;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = 0; s < a.world; ++s) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(a.grads[s] + i));
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      const float inv = 1.f / (float)a.world;
      acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
      *reinterpret_cast<float4*>(a.red_grad + (i - base)) = acc;
    }
  } else {
    for (long long i = begin + blockIdx.x * (long long)kOptThreads + threadIdx.x; i < end;
         i += (long long)gridDim.x * kOptThreads)
      a.red_grad[i - base] = rank_mean(a, i);
  }
}

cudaError_t dp_reduce_range(const DpArgs& a, const int* flags, long long lo, long long hi, int grid,
                            cudaStream_t stream) {
  if (a.world < 1 || a.world > kMaxShards || a.rank < 0 || a.rank >= a.world || grid < 1 || lo < 0 || hi < lo)
    return cudaErrorInvalidValue;
  dp_reduce_range_kernel<<<grid, kOptThreads, 0, stream>>>(a, flags, lo, hi);
  return cudaGetLastError();
}

cudaError_t dp_reduce_norm(const DpArgs& a, int grid, cudaStream_t stream) {
  if (a.world < 1 || a.world > kMaxShards || a.rank < 0 || a.rank >= a.world || grid < 1)
    return cudaErrorInvalidValue;
  dp_reduce_norm_kernel<<<grid, kOptThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t dp_adamw_gather(const DpArgs& a, int grid, cudaStream_t stream) {
  if (a.world < 1 || a.world > kMaxShards || a.rank < 0 || a.rank >= a.world || grid < 1)
    return cudaErrorInvalidValue;
  dp_adamw_gather_kernel<<<grid, kOptThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

__global__ void bump_counter_kernel(int* c) {
  if (threadIdx.x == 0) *c += 1;
}

cudaError_t bump_counter(int* counter, cudaStream_t stream) {
  bump_counter_kernel<<<1, 32, 0, stream>>>(counter);
  return cudaGetLastError();
}

// ------------------------------------------ epoch-valued signal / multi-wait
__global__ void signal_epoch_kernel(FlagPtrs flags, const int* epoch_ptr, int offset) {
  if (threadIdx.x == 0) __threadfence_system();
  __syncwarp();
  if (threadIdx.x < flags.n) st_release(flags.addr[threadIdx.x], *epoch_ptr + offset);
}

__global__ void wait_all_kernel(const int* flags, int n, const int* epoch_ptr, int offset, long long timeout_ns,
                                int* status) {
  block_wait_all(flags, n, *epoch_ptr + offset, timeout_ns, status);
}

cudaError_t signal_epoch(const FlagPtrs& flags, const int* epoch_ptr, int offset, cudaStream_t stream) {
  if (flags.n < 1 || flags.n > kMaxShards) return cudaErrorInvalidValue;
  signal_epoch_kernel<<<1, 32, 0, stream>>>(flags, epoch_ptr, offset);
  return cudaGetLastError();
}

cudaError_t wait_all(const int* flags, int n, const int* epoch_ptr, int offset, long long timeout_ns, int* status,
                     cudaStream_t stream) {
  if (n < 1 || n > kMaxShards) return cudaErrorInvalidValue;
  wait_all_kernel<<<1, 32, 0, stream>>>(flags, n, epoch_ptr, offset, timeout_ns, status);
  return cudaGetLastError();
}

}  // namespace sc
