// Attention of one new position over its own past keys, forward and backward:
// the self-attention of the recurrent EAGLE drafter trunk (K14).
//
//   out[b, h]  = sum_j softmax_j(q[b, h] . k[b, g(h), j] * scale) v[b, g(h), j]
//   lse[b, h]  = log-sum-exp of the scaled scores (saved for the backward)
//
// Every recurrent step of the drafter appends one position and attends to all
// positions so far (no mask; reference src/sparsecache/sparse_kv_eagle.py:
// 69-110, where the trunk runs HF SDPA with the query heads of a KV group
// folded into the query length).  Shapes: q [B, Hq, 128], k / v [B, Hkv, P,
// 128] contiguous bf16, Hq = G * Hkv with G <= 8, P <= kMaxKeys.
//
// One CTA per (sequence, kv head), one warp per query head of the group:
//   forward   lanes take keys j = lane, lane + 32, ... and form whole-row dot
//             products against q staged in shared memory; warp max / sum give
//             the softmax; then lanes take 4 dims each and accumulate
//             sum_j p_j v_j with coalesced 256-byte row reads.
//   backward  recompute p_j from the saved lse; dp_j = dO . v_j (lanes over
//             keys); D = sum_j p_j dp_j; ds_j = p_j (dp_j - D); dq = scale sum_j ds_j k_j
//             (lanes over dims); then all threads of the CTA form dk_j = scale
//             sum_h ds[h][j] q[h] and dv_j = sum_h p[h][j] dO[h] over the group.
// fp32 arithmetic throughout, bf16 in and out.
#include "common.cuh"
#include "kernels.h"

namespace sc {

namespace {
constexpr int kD = 128;

__device__ __forceinline__ float dot_row_bf16(const __nv_bfloat16* row, const float* vec) {
  const uint4* r = reinterpret_cast<const uint4*>(row);
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < kD / 8; ++c) {
    const uint4 u = r[c];
    const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), e = unpack_bf16x2(u.z), f = unpack_bf16x2(u.w);
    const float* v = vec + 8 * c;
    acc = fmaf(a.x, v[0], acc);
    acc = fmaf(a.y, v[1], acc);
    acc = fmaf(b.x, v[2], acc);
    acc = fmaf(b.y, v[3], acc);
    acc = fmaf(e.x, v[4], acc);
    acc = fmaf(e.y, v[5], acc);
    acc = fmaf(f.x, v[6], acc);
    acc = fmaf(f.y, v[7], acc);
  }
  return acc;
}

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
}  // namespace

// dynamic shared memory: q [G][128] fp32, p [G][P] fp32
__global__ void recurrent_attention_fwd_kernel(RecurrentAttnArgs a) {
  extern __shared__ float sm[];
  const int G = a.n_heads / a.n_kv_heads;
  const int b = blockIdx.x / a.n_kv_heads, kvh = blockIdx.x % a.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = a.n_keys;
  float* sq = sm;
  float* sp = sm + G * kD;
  const __nv_bfloat16* K = a.k + ((size_t)b * a.n_kv_heads + kvh) * (size_t)P * kD;
  const __nv_bfloat16* V = a.v + ((size_t)b * a.n_kv_heads + kvh) * (size_t)P * kD;
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const int h = kvh * G + i / kD;
    sq[i] = __bfloat162float(a.q[((size_t)b * a.n_heads + h) * kD + i % kD]) * a.scale;
  }
  __syncthreads();
  if (warp >= G) return;
  const int h = kvh * G + warp;
  float* p = sp + warp * P;
  float mx = -INFINITY;
  for (int j = lane; j < P; j += 32) {
    const float s = dot_row_bf16(K + (size_t)j * kD, sq + warp * kD);
    p[j] = s;
    mx = fmaxf(mx, s);
  }
  mx = warp_max_f(mx);
  float sum = 0.f;
  for (int j = lane; j < P; j += 32) {
    const float e = __expf(p[j] - mx);
    p[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  __syncwarp();
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < P; ++j) {
    const float w = p[j];
    const uint2 u = *reinterpret_cast<const uint2*>(V + (size_t)j * kD + lane * 4);
    const float2 v0 = unpack_bf16x2(u.x), v1 = unpack_bf16x2(u.y);
    o[0] = fmaf(w, v0.x, o[0]);
    o[1] = fmaf(w, v0.y, o[1]);
    o[2] = fmaf(w, v1.x, o[2]);
    o[3] = fmaf(w, v1.y, o[3]);
  }
  __nv_bfloat16* out = a.out + ((size_t)b * a.n_heads + h) * kD + lane * 4;
  *reinterpret_cast<uint2*>(out) = make_uint2(pack_bf16x2(o[0] * inv, o[1] * inv), pack_bf16x2(o[2] * inv, o[3] * inv));
  if (lane == 0) a.lse[(size_t)b * a.n_heads + h] = mx + logf(sum);
}

// dynamic shared memory: q [G][128], dO [G][128], p [G][P], ds [G][P] (fp32)
__global__ void recurrent_attention_bwd_kernel(RecurrentAttnArgs a) {
  extern __shared__ float sm[];
  const int G = a.n_heads / a.n_kv_heads;
  const int b = blockIdx.x / a.n_kv_heads, kvh = blockIdx.x % a.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = a.n_keys;
  float* sq = sm;
  float* sdo = sq + G * kD;
  float* sp = sdo + G * kD;
  float* sds = sp + G * P;
  const size_t kv_off = ((size_t)b * a.n_kv_heads + kvh) * (size_t)P * kD;
  const __nv_bfloat16* K = a.k + kv_off;
  const __nv_bfloat16* V = a.v + kv_off;
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const size_t qi = ((size_t)b * a.n_heads + kvh * G + i / kD) * kD + i % kD;
    sq[i] = __bfloat162float(a.q[qi]);
    sdo[i] = __bfloat162float(a.dout[qi]);
  }
  __syncthreads();
  if (warp < G) {
    const int h = kvh * G + warp;
    const float lse = a.lse[(size_t)b * a.n_heads + h];
    float* p = sp + warp * P;
    float* ds = sds + warp * P;
    // p_j and dp_j = dO . v_j; D = sum_j p_j dp_j (= dO . O, formed in fp32
    // from the recomputed probabilities rather than from the bf16 output)
    float dsum = 0.f;
    for (int j = lane; j < P; j += 32) {
      const float s = dot_row_bf16(K + (size_t)j * kD, sq + warp * kD) * a.scale;
      const float pj = __expf(s - lse);
      const float dp = dot_row_bf16(V + (size_t)j * kD, sdo + warp * kD);
      p[j] = pj;
      ds[j] = dp;
      dsum = fmaf(pj, dp, dsum);
    }
    const float dd = warp_sum(dsum);
    for (int j = lane; j < P; j += 32) ds[j] = p[j] * (ds[j] - dd);
    __syncwarp();
    // dq = scale * sum_j ds_j k_j  (lanes over 4 dims each)
    float dq[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < P; ++j) {
      const float w = ds[j];
      const uint2 u = *reinterpret_cast<const uint2*>(K + (size_t)j * kD + lane * 4);
      const float2 k0 = unpack_bf16x2(u.x), k1 = unpack_bf16x2(u.y);
      dq[0] = fmaf(w, k0.x, dq[0]);
      dq[1] = fmaf(w, k0.y, dq[1]);
      dq[2] = fmaf(w, k1.x, dq[2]);
      dq[3] = fmaf(w, k1.y, dq[3]);
    }
    __nv_bfloat16* dqo = a.dq + ((size_t)b * a.n_heads + h) * kD + lane * 4;
    *reinterpret_cast<uint2*>(dqo) = make_uint2(pack_bf16x2(dq[0] * a.scale, dq[1] * a.scale),
                                                pack_bf16x2(dq[2] * a.scale, dq[3] * a.scale));
  }
  __syncthreads();
  // dk_j = scale * sum_h ds[h][j] q[h];  dv_j = sum_h p[h][j] dO[h]   (threads over (j, 4-dim chunk))
  for (int i = threadIdx.x; i < P * (kD / 4); i += blockDim.x) {
    const int j = i / (kD / 4), c = (i % (kD / 4)) * 4;
    float dk[4] = {0.f, 0.f, 0.f, 0.f}, dv[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g = 0; g < G; ++g) {
      const float w = sds[g * P + j], pj = sp[g * P + j];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        dk[e] = fmaf(w, sq[g * kD + c + e], dk[e]);
        dv[e] = fmaf(pj, sdo[g * kD + c + e], dv[e]);
      }
    }
    __nv_bfloat16* dko = a.dk + kv_off + (size_t)j * kD + c;
    __nv_bfloat16* dvo = a.dv + kv_off + (size_t)j * kD + c;
    *reinterpret_cast<uint2*>(dko) = make_uint2(pack_bf16x2(dk[0] * a.scale, dk[1] * a.scale),
                                                pack_bf16x2(dk[2] * a.scale, dk[3] * a.scale));
    *reinterpret_cast<uint2*>(dvo) = make_uint2(pack_bf16x2(dv[0], dv[1]), pack_bf16x2(dv[2], dv[3]));
  }
}

static bool recurrent_attn_ok(const RecurrentAttnArgs& a) {
  return a.n_kv_heads > 0 && a.n_heads % a.n_kv_heads == 0 && a.n_heads / a.n_kv_heads <= 8 && a.batch > 0 &&
         a.n_keys > 0 && a.n_keys <= kRecurrentAttnMaxKeys;
}

cudaError_t recurrent_attention_fwd(const RecurrentAttnArgs& a, cudaStream_t stream) {
  if (!recurrent_attn_ok(a)) return cudaErrorInvalidValue;
  const int G = a.n_heads / a.n_kv_heads;
  const size_t smem = (size_t)G * (kD + a.n_keys) * sizeof(float);
  ensure_smem_attr(recurrent_attention_fwd_kernel, (int)smem);
  recurrent_attention_fwd_kernel<<<a.batch * a.n_kv_heads, 32 * G, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t recurrent_attention_bwd(const RecurrentAttnArgs& a, cudaStream_t stream) {
  if (!recurrent_attn_ok(a)) return cudaErrorInvalidValue;
  const int G = a.n_heads / a.n_kv_heads;
  const size_t smem = (size_t)G * (2 * kD + 2 * a.n_keys) * sizeof(float);
  ensure_smem_attr(recurrent_attention_bwd_kernel, (int)smem);
  recurrent_attention_bwd_kernel<<<a.batch * a.n_kv_heads, 256, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace sc
