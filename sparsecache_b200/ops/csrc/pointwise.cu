// Memory-bound kernels of the prefill / compose path:
//   rmsnorm_bf16       HF LlamaRMSNorm rounding order, optional row gather
//   embedding_bf16     token-id row gather of the embedding table
//   gather_rows_bf16   residual-row gather at the CacheBlend check layer
//   compose_relocate   the cache composer: gather every document's K/V (from
//                      HBM or from mapped pinned host memory) into the
//                      request's layer caches and re-rotate each key's RoPE
//                      from its source to its target position in fp32
//                      (rope.py:61-91 relocate_key, store.py:99-149
//                      compose_cache, reuse_cacheblend_pipeline.py:407-449)
//   cacheblend_select  fixed-order reduction of the fused deviation partials,
//                      radix top-k over the document rows, merge with the
//                      mandatory system/suffix rows, sorted active list
//                      (modeling.py:215-242, reuse_cacheblend_pipeline.py:586-616)
#include "common.cuh"
#include "kernels.h"

namespace sc {

// ------------------------------------------------------------------ RMSNorm
__global__ void rmsnorm_kernel(const __nv_bfloat16* x, int ldx, const int* rows,
                               const __nv_bfloat16* w, __nv_bfloat16* out, int ldo, int D,
                               float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const int r = blockIdx.x;
  const int src_row = rows ? rows[r] : r;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)src_row * ldx);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)r * ldo);
  float ss = 0.f;
  for (int c = threadIdx.x; c < D / 8; c += blockDim.x) {
    const uint4 v = xr[c];
    const uint32_t vi[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(vi[q]);
      ss += f.x * f.x + f.y * f.y;
    }
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
  const float rinv = rsqrtf(red[0] / (float)D + eps);
  for (int c = threadIdx.x; c < D / 8; c += blockDim.x) {
    const uint4 v = xr[c], g = wr[c];
    const uint32_t vi[4] = {v.x, v.y, v.z, v.w};
    const uint32_t gi[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 xf = unpack_bf16x2(vi[q]), gf = unpack_bf16x2(gi[q]);
      o[q] = pack_bf16x2(gf.x * bf16_round(xf.x * rinv), gf.y * bf16_round(xf.y * rinv));
    }
    orow[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

cudaError_t rmsnorm_bf16(const __nv_bfloat16* x, int ldx, const int* rows, const __nv_bfloat16* w,
                         __nv_bfloat16* out, int ldo, int M, int D, float eps,
                         cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  if (D % 8) return cudaErrorInvalidValue;
  return launch_pdl(rmsnorm_kernel, dim3(M), dim3(256), 0, stream, x, ldx, rows, w, out, ldo, D, eps);
}

// ---------------------------------------------------------------- gathers
__global__ void gather_rows_kernel(const __nv_bfloat16* in, int ldi, const int* rows,
                                   __nv_bfloat16* out, int ldo, int D) {
  const int r = blockIdx.x;
  const int src = rows ? rows[r] : r;
  const uint4* s = reinterpret_cast<const uint4*>(in + (size_t)src * ldi);
  uint4* d = reinterpret_cast<uint4*>(out + (size_t)r * ldo);
  for (int c = threadIdx.x; c < D / 8; c += blockDim.x) d[c] = s[c];
}

cudaError_t embedding_bf16(const int* ids, const __nv_bfloat16* table, __nv_bfloat16* out, int M,
                           int D, cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  gather_rows_kernel<<<M, 128, 0, stream>>>(table, D, ids, out, D, D);
  return cudaGetLastError();
}

cudaError_t gather_rows_bf16(const __nv_bfloat16* in, int ldi, const int* rows,
                             __nv_bfloat16* out, int ldo, int M, int D, cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  gather_rows_kernel<<<M, 128, 0, stream>>>(in, ldi, rows, out, ldo, D);
  return cudaGetLastError();
}

// ------------------------------------------------------- compose/relocate
// Thread layout: one thread per (layer, kv in {K,V}, head, token, 8-dim
// chunk c in [0, 8)).  For keys the thread rotates the dim pairs
// (8c + i, 64 + 8c + i); for values it copies both 16-byte chunks.
__global__ void compose_relocate_kernel(ComposeArgs a) {
  const long long total = (long long)(a.layer_end - a.layer_begin) * 2 * a.n_kv_heads *
                          a.total_tokens * 8;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= total) return;
  const int c = (int)(tid & 7);
  long long rest = tid >> 3;
  const int tok = (int)(rest % a.total_tokens);
  rest /= a.total_tokens;
  const int head = (int)(rest % a.n_kv_heads);
  rest /= a.n_kv_heads;
  const int kv = (int)(rest & 1);
  const int layer = a.layer_begin + (int)(rest >> 1);

  // token -> document (n_docs is small: linear scan over the offsets)
  int d = 0;
  while (d + 1 < a.n_docs && a.doc_token_offset[d + 1] <= tok) ++d;
  const ComposeDoc doc = a.docs[d];
  const int t = tok - a.doc_token_offset[d];

  const size_t src_off =
      ((((size_t)layer * 2 + kv) * a.n_kv_heads + head) * doc.n_tokens + t) * 128;
  const size_t dst_off =
      ((((size_t)layer * 2 + kv) * a.n_kv_heads + head) * a.cache_cap + doc.dst_slot + t) * 128;
  const uint4* src = reinterpret_cast<const uint4*>(doc.src + src_off);
  uint4* dst = reinterpret_cast<uint4*>(a.cache + dst_off);
  const uint4 lo = src[c];
  const uint4 hi = src[8 + c];
  const int sp = doc.src_pos + t, tp = doc.dst_pos + t;
  if (kv == 1 || sp == tp) {
    dst[c] = lo;
    dst[8 + c] = hi;
    return;
  }
  const uint32_t li[4] = {lo.x, lo.y, lo.z, lo.w};
  const uint32_t hi4[4] = {hi.x, hi.y, hi.z, hi.w};
  uint32_t lo_o[4], hi_o[4];
  const float2* ts = a.rope_table + (size_t)sp * 64 + 8 * c;
  const float2* tt = a.rope_table + (size_t)tp * 64 + 8 * c;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 x1 = unpack_bf16x2(li[q]), x2 = unpack_bf16x2(hi4[q]);
    float r1[2], r2[2];
    const float a1[2] = {x1.x, x1.y}, a2[2] = {x2.x, x2.y};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float2 s = ts[2 * q + e], g = tt[2 * q + e];
      // remove the source rotation, then apply the target rotation (fp32)
      const float c1 = a1[e] * s.x + a2[e] * s.y;
      const float c2 = a2[e] * s.x - a1[e] * s.y;
      r1[e] = c1 * g.x - c2 * g.y;
      r2[e] = c2 * g.x + c1 * g.y;
    }
    lo_o[q] = pack_bf16x2(r1[0], r1[1]);
    hi_o[q] = pack_bf16x2(r2[0], r2[1]);
  }
  dst[c] = make_uint4(lo_o[0], lo_o[1], lo_o[2], lo_o[3]);
  dst[8 + c] = make_uint4(hi_o[0], hi_o[1], hi_o[2], hi_o[3]);
}

cudaError_t compose_relocate(const ComposeArgs& a, cudaStream_t stream) {
  const long long total = (long long)(a.layer_end - a.layer_begin) * 2 * a.n_kv_heads *
                          a.total_tokens * 8;
  if (total <= 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  compose_relocate_kernel<<<(unsigned)blocks, threads, 0, stream>>>(a);
  return cudaGetLastError();
}

// ------------------------------------------------------ CacheBlend select
// One CTA of 1024 threads.  Scores are non-negative floats, so their bit
// patterns order like unsigned integers: a 4-pass 8-bit radix select finds
// the k-th largest value; rows above it are taken, ties go to the lowest
// rows.  The active list is emitted in position order by a block scan.
namespace {
constexpr int kSelThreads = 1024;

__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;
  }
  __syncthreads();
  const int warp_prefix = warp > 0 ? s_warp[warp - 1] : 0;
  total = s_warp[31];
  __syncthreads();
  return warp_prefix + x - v;
}
}  // namespace

__global__ void __launch_bounds__(kSelThreads) cacheblend_select_kernel(SelectArgs a) {
  __shared__ unsigned int hist[256];
  __shared__ int s_warp[32];
  __shared__ unsigned int s_prefix, s_mask;
  __shared__ int s_remaining;
  const int tid = threadIdx.x;
  const int n_doc = max(0, a.doc_end - a.doc_begin);
  const int H = a.n_kv_heads;

  // 1. scores (fixed reduction order over kv heads; key part then value part)
  for (int i = tid; i < n_doc; i += kSelThreads) {
    float s = 0.f;
    for (int part = 0; part < max(1, a.n_parts); ++part) {
      const float* p = a.dev_part + part * a.part_stride + (size_t)(a.doc_begin + i) * 2 * H;
      if (a.dev_mode & DEV_KEY)
        for (int h = 0; h < H; ++h) s += p[h];
      if (a.dev_mode & DEV_VALUE)
        for (int h = 0; h < H; ++h) s += p[H + h];
    }
    a.scores[i] = s;
  }
  __syncthreads();

  // 2. radix select of the k-th largest bit pattern
  const int k = min(a.k, n_doc);
  if (tid == 0) s_prefix = 0u, s_mask = 0u, s_remaining = k;
  __syncthreads();
  for (int pass = 0; pass < 4 && k > 0; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = tid; b < 256; b += kSelThreads) hist[b] = 0u;
    __syncthreads();
    const unsigned prefix = s_prefix, mask = s_mask;
    for (int i = tid; i < n_doc; i += kSelThreads) {
      const unsigned bits = __float_as_uint(a.scores[i]);
      if ((bits & mask) == prefix) atomicAdd(&hist[(bits >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      int rem = s_remaining;
      int b = 255;
      for (; b > 0; --b) {
        if ((int)hist[b] >= rem) break;
        rem -= (int)hist[b];
      }
      s_prefix = prefix | ((unsigned)b << shift);
      s_mask = mask | (255u << shift);
      s_remaining = rem;
    }
    __syncthreads();
  }
  const unsigned thresh = s_prefix;
  const int ties_needed = s_remaining;  // how many rows equal to thresh to take

  // 3. emit active rows in position order
  int tie_base = 0, out_base = 0, sel_base = 0;
  long long checksum = 0;
  for (int base = 0; base < a.total_rows; base += kSelThreads) {
    const int r = base + tid;
    int is_tie = 0, take = 0, is_doc = 0;
    if (r < a.total_rows) {
      if (r >= a.doc_begin && r < a.doc_end) {
        is_doc = 1;
        if (k > 0) {
          const unsigned bits = __float_as_uint(a.scores[r - a.doc_begin]);
          if (bits > thresh) take = 1;
          else if (bits == thresh) is_tie = 1;
        }
      } else if (r >= a.doc_end || a.keep_prefix) {
        take = 1;
      }
    }
    int tie_total;
    const int tie_rank = block_exclusive_scan(is_tie, s_warp, tie_total);
    if (is_tie && tie_base + tie_rank < ties_needed) take = 1;
    tie_base += tie_total;
    int take_total;
    const int out_idx = block_exclusive_scan(take, s_warp, take_total);
    if (take) a.active[out_base + out_idx] = r;
    out_base += take_total;
    int seld = take && is_doc;
    int sel_total;
    const int sel_rank = block_exclusive_scan(seld, s_warp, sel_total);
    if (seld) checksum += (long long)r * (long long)(sel_base + sel_rank + 1);
    sel_base += sel_total;
  }
  if (tid == 0) *a.n_active = out_base;
  if (a.checksum != nullptr) {
    // reduce the per-thread checksum contributions
    __shared__ long long s_ck[32];
    long long v = checksum;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((tid & 31) == 0) s_ck[tid >> 5] = v;
    __syncthreads();
    if (tid == 0) {
      long long t = 0;
      for (int w = 0; w < kSelThreads / 32; ++w) t += s_ck[w];
      *a.checksum = t;
    }
  }
}

cudaError_t cacheblend_select(const SelectArgs& a, cudaStream_t stream) {
  cacheblend_select_kernel<<<1, kSelThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- small ops
__global__ void arange_kernel(int* out, int n, int start) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = start + i;
}
cudaError_t fill_arange_i32(int* out, int n, int start, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  arange_kernel<<<(n + 255) / 256, 256, 0, stream>>>(out, n, start);
  return cudaGetLastError();
}

__global__ void index_kernel(const int* src, const int* idx, int* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = src[idx[i]];
}
cudaError_t index_i32(const int* src, const int* idx, int* out, int n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  index_kernel<<<(n + 255) / 256, 256, 0, stream>>>(src, idx, out, n);
  return cudaGetLastError();
}

}  // namespace sc
