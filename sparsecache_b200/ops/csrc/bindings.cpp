// PyTorch bindings of the sm_100a kernels.  Every op launches on the
// current torch CUDA stream and validates shapes, dtypes and alignment
// before launch (TMA needs 16-byte aligned bases and row strides).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>

#include "kernels.h"

namespace {

using torch::Tensor;

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == torch::kBFloat16, #x " must be bf16")
#define CHECK_I32(x) TORCH_CHECK((x).scalar_type() == torch::kInt32, #x " must be int32")
#define CHECK_F32(x) TORCH_CHECK((x).scalar_type() == torch::kFloat32, #x " must be float32")
#define CHECK_ALIGN16(x) \
  TORCH_CHECK((reinterpret_cast<uintptr_t>((x).data_ptr()) & 15) == 0, #x " must be 16-byte aligned")

void check_cuda(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

int num_sms() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (n[dev] == 0) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev];
}

// Per-device status word the tcgen05 kernels write when a bounded wait expires.
Tensor& status_tensor(const Tensor& like) {
  static Tensor st[64];
  const int dev = like.get_device();
  if (!st[dev].defined()) {
    st[dev] = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(like.device()));
  }
  return st[dev];
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

void check_matrix(const Tensor& t, const char* name) {
  CHECK_CUDA(t);
  CHECK_BF16(t);
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must be row-major");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0, name, " row stride must be a multiple of 16 bytes");
  CHECK_ALIGN16(t);
}

sc::GemmArgs base_gemm(const Tensor& a, const Tensor& w, int epi, int bn) {
  check_matrix(a, "a");
  check_matrix(w, "w");
  TORCH_CHECK(a.size(1) == w.size(1), "K mismatch");
  TORCH_CHECK(bn == 128 || bn == 256, "bn must be 128 or 256");
  sc::GemmArgs g{};
  g.a = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
  g.b = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  g.M = (int)a.size(0);
  g.N = (int)w.size(0);
  g.K = (int)a.size(1);
  g.lda = (int)a.stride(0);
  g.ldb = (int)w.stride(0);
  g.epi = epi;
  g.bn = bn;
  g.num_sms = num_sms();
  g.status = status_tensor(a).data_ptr<int>();
  return g;
}

void run_gemm(const sc::GemmArgs& g) {
  if (g.M == 0 || g.N == 0) return;
  check_cuda(sc::gemm_bf16_tc(g, cur_stream()), "gemm_bf16_tc");
}

// Split-K for STORE/RESIDUAL GEMMs whose output has too few tiles to fill the
// SMs (small M): K-slices write fp32 partials, an ordered reduce applies the
// epilogue.  splits < 0 picks automatically; 1 disables.
int auto_splits(const sc::GemmArgs& g, int rows_per_tile) {
  const int tiles = ((g.M + rows_per_tile - 1) / rows_per_tile) * ((g.N + g.bn - 1) / g.bn);
  const int num_kb = (g.K + 63) / 64;
  if (2 * tiles > g.num_sms) return 1;
  int s = g.num_sms / tiles;
  if (s > num_kb / 8) s = num_kb / 8;  // at least 8 k-blocks (K = 512) per slice
  if (s > 8) s = 8;
  return s < 2 ? 1 : s;
}

// Tile rows forced for every GEMM (0: chosen per call); a test hook.
static int g_rows_policy = 0;
void set_gemm_rows_per_tile(int64_t rows) {
  TORCH_CHECK(rows == 0 || rows == 128 || rows == 256, "rows per tile: 0 (automatic), 128 or 256");
  g_rows_policy = (int)rows;
}

// Tile shape of an unsharded GEMM: 128-row tiles, or 256-row tiles (two TMEM
// accumulators sharing each B k-block) when the cost model prefers them; with
// `may_split`, the split-K count of each shape is priced in as well (partials
// written and read back by the ordered reduce).  Returns the split count.
int choose_shape(sc::GemmArgs& g, bool may_split, int64_t splits_req) {
  // 256-row tiles pay off from ~3 full m-tiles on (B200, 8B shapes: o / gate-up / down 1.2-1.4x
  // faster at 1676 rows, equal or slower at 300 rows where the k-loop is latency-bound)
  const bool two_ok = g.bn == 256 && g.shards.n <= 1 && g.epi != sc::EPI_RS &&
                      (g.M >= 768 || (g_rows_policy == 256 && g.M > 128));
  double best = 0.0;
  int best_rows = 128, best_s = 1;
  bool have = false;
  for (int rows : {128, 256}) {
    if (rows == 256 && !two_ok) continue;
    if (g_rows_policy != 0 && rows != g_rows_policy && !(rows == 128 && !two_ok)) continue;
    const int s = !may_split ? 1 : (splits_req < 0 ? auto_splits(g, rows) : (int)splits_req);
    double cost = sc::gemm_cost_estimate(g.M, g.N, g.K, g.bn, rows, s, g.num_sms);
    if (s > 1) cost += ((double)g.M * g.N * 4.0 * (s + 1) + (double)g.M * g.N * 4.0) / (6.5e12 / 1.9e9);
    if (!have || cost < best) best = cost, best_rows = rows, best_s = s, have = true;
  }
  g.rows_per_tile = best_rows;
  return best_s;
}

struct NormOut {  // optional RMSNorm of the finished rows (the next projection's input)
  const __nv_bfloat16* w = nullptr;
  float eps = 0.f;
  __nv_bfloat16* out = nullptr;
  int ld = 0;
};

bool run_gemm_split(sc::GemmArgs g, int s, const Tensor& like, const NormOut& norm = NormOut{}) {
  if (s <= 1 || g.M == 0) return false;
  Tensor ws = torch::empty({s, g.M, g.N}, like.options().dtype(torch::kFloat32));
  const __nv_bfloat16* residual = g.epi == sc::EPI_RESIDUAL ? g.ep.residual : nullptr;
  const int ldr = g.ep.ldr;
  __nv_bfloat16* out = g.ep.out;
  const int ldo = g.ep.ldo;
  g.epi = sc::EPI_PARTIAL;
  g.splits = s;
  g.ep.ws = ws.data_ptr<float>();
  check_cuda(sc::gemm_bf16_tc(g, cur_stream()), "gemm_bf16_tc (split-K)");
  if (norm.w != nullptr) {
    check_cuda(sc::splitk_reduce_norm(g.ep.ws, s, g.M, g.N, residual, ldr, out, ldo, norm.w, norm.eps, norm.out,
                                      norm.ld, cur_stream()),
               "splitk_reduce_norm");
  } else {
    check_cuda(sc::splitk_reduce(g.ep.ws, s, g.M, g.N, residual, ldr, out, ldo, cur_stream()), "splitk_reduce");
  }
  return true;
}

// out = a @ w^T
int64_t gemm_store(Tensor a, Tensor w, Tensor out, int64_t bn, int64_t splits) {
  const c10::cuda::CUDAGuard guard(a.device());
  auto g = base_gemm(a, w, sc::EPI_STORE, (int)bn);
  check_matrix(out, "out");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == w.size(0), "out shape");
  TORCH_CHECK(g.N % 32 == 0, "N must be a multiple of 32");
  g.ep.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  g.ep.ldo = (int)out.stride(0);
  const int s = choose_shape(g, true, splits);
  if (run_gemm_split(g, s, a)) return 2;  // kernels launched
  run_gemm(g);
  return 1;
}

// out = residual + bf16(a @ w^T)   (out may alias residual); with norm_w also
// norm_out = RMSNorm(out) (fused into the split-K reduce when split-K runs,
// else the RMSNorm kernel after the GEMM).  Returns the kernels launched.
int64_t gemm_residual(Tensor a, Tensor w, Tensor out, Tensor residual, int64_t bn, int64_t splits,
                      c10::optional<Tensor> norm_w, double eps, c10::optional<Tensor> norm_out) {
  const c10::cuda::CUDAGuard guard(a.device());
  auto g = base_gemm(a, w, sc::EPI_RESIDUAL, (int)bn);
  check_matrix(out, "out");
  check_matrix(residual, "residual");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == w.size(0), "out shape");
  TORCH_CHECK(residual.sizes() == out.sizes(), "residual shape");
  TORCH_CHECK(g.N % 32 == 0, "N must be a multiple of 32");
  g.ep.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  g.ep.ldo = (int)out.stride(0);
  g.ep.residual = reinterpret_cast<const __nv_bfloat16*>(residual.data_ptr());
  g.ep.ldr = (int)residual.stride(0);
  NormOut norm;
  if (norm_w.has_value() && norm_w->defined()) {
    TORCH_CHECK(norm_out.has_value() && norm_out->defined(), "norm_out required with norm_w");
    CHECK_BF16(*norm_w); check_matrix(*norm_out, "norm_out");
    TORCH_CHECK(norm_w->numel() == g.N && norm_out->sizes() == out.sizes(), "norm shapes");
    TORCH_CHECK(g.N % 8 == 0 && g.N <= 8192, "fused norm: N % 8 == 0, N <= 8192");
    norm.w = reinterpret_cast<const __nv_bfloat16*>(norm_w->data_ptr());
    norm.eps = (float)eps;
    norm.out = reinterpret_cast<__nv_bfloat16*>(norm_out->data_ptr());
    norm.ld = (int)norm_out->stride(0);
  }
  const int s = choose_shape(g, true, splits);
  if (run_gemm_split(g, s, a, norm)) return 2;  // kernels launched (the norm is fused into the reduce)
  run_gemm(g);
  if (norm.w == nullptr) return 1;
  check_cuda(sc::rmsnorm_bf16(g.ep.out, g.ep.ldo, nullptr, norm.w, norm.out, norm.ld, g.M, g.N, norm.eps,
                              cur_stream()),
             "rmsnorm");
  return 2;
}

// out[:, j] = silu(gate_j) * up_j with w_gu rows interleaved in blocks of bn/2
void gemm_swiglu(Tensor a, Tensor w_gu, Tensor out, int64_t bn) {
  const c10::cuda::CUDAGuard guard(a.device());
  auto g = base_gemm(a, w_gu, sc::EPI_SWIGLU, (int)bn);
  check_matrix(out, "out");
  TORCH_CHECK(w_gu.size(0) % bn == 0, "gate/up rows must be a multiple of bn");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == w_gu.size(0) / 2, "out shape");
  g.ep.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  g.ep.ldo = (int)out.stride(0);
  choose_shape(g, false, 1);
  run_gemm(g);
}

// Fused QKV projection + RoPE + K/V cache scatter (+ optional deviation partials).
void gemm_qkv(Tensor a, Tensor w_qkv, Tensor q_out, Tensor k_cache, Tensor v_cache,
              Tensor rope_pos, Tensor cache_slot, Tensor rope_table, int64_t n_q_heads,
              int64_t n_kv_heads, c10::optional<Tensor> dev_part, int64_t dev_mode, int64_t bn,
              int64_t k_peer, int64_t v_peer) {
  const c10::cuda::CUDAGuard guard(a.device());
  auto g = base_gemm(a, w_qkv, sc::EPI_QKV, (int)bn);
  check_matrix(q_out, "q_out");
  TORCH_CHECK(w_qkv.size(0) == (n_q_heads + 2 * n_kv_heads) * 128, "w_qkv rows");
  TORCH_CHECK(q_out.size(0) >= a.size(0) && q_out.size(1) == n_q_heads * 128, "q_out shape");
  CHECK_CUDA(k_cache); CHECK_BF16(k_cache); CHECK_CUDA(v_cache); CHECK_BF16(v_cache);
  TORCH_CHECK(k_cache.dim() == 3 && k_cache.size(0) == n_kv_heads && k_cache.size(2) == 128 &&
                  k_cache.is_contiguous(), "k_cache must be [n_kv_heads, cap, 128] contiguous");
  TORCH_CHECK(v_cache.sizes() == k_cache.sizes() && v_cache.is_contiguous(), "v_cache shape");
  CHECK_I32(rope_pos); CHECK_I32(cache_slot); CHECK_F32(rope_table);
  TORCH_CHECK(rope_pos.numel() >= a.size(0) && cache_slot.numel() >= a.size(0), "positions");
  TORCH_CHECK(rope_table.dim() == 2 && rope_table.size(1) == 128, "rope_table [P, 64*2]");
  g.ep.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  g.ep.ldq = (int)q_out.stride(0);
  g.ep.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  g.ep.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  g.ep.cache_cap = (int)k_cache.size(1);
  g.ep.rope_pos = rope_pos.data_ptr<int>();
  g.ep.cache_slot = cache_slot.data_ptr<int>();
  g.ep.rope_table = reinterpret_cast<const float2*>(rope_table.data_ptr<float>());
  g.ep.n_q_heads = (int)n_q_heads;
  g.ep.n_kv_heads = (int)n_kv_heads;
  if (dev_part.has_value() && dev_part->defined()) {
    CHECK_F32(*dev_part);
    TORCH_CHECK(dev_part->numel() >= a.size(0) * 2 * n_kv_heads, "dev_part size");
    g.ep.dev_part = dev_part->data_ptr<float>();
    g.ep.dev_mode = (int)dev_mode;
  }
  // peer pointers (int64 addresses of the decode GPU's layer cache, mapped
  // into this process with CUDA IPC); 0 disables the push
  g.ep.k_peer = reinterpret_cast<__nv_bfloat16*>(k_peer);
  g.ep.v_peer = reinterpret_cast<__nv_bfloat16*>(v_peer);
  TORCH_CHECK((k_peer == 0) == (v_peer == 0), "k_peer and v_peer go together");
  choose_shape(g, false, 1);
  run_gemm(g);
}

sc::GemvArgs base_gemv(const Tensor& x, const Tensor& w, c10::optional<Tensor> norm_w, double eps, int epi);
void run_gemv(const sc::GemvArgs& g);

// ------------------------------------------------- tensor-parallel GEMMs
// A is row-sharded over `shard_ptrs` (device addresses, peers' shards mapped
// with CUDA IPC), each [rows, K] with row stride K; the all-gather is fused
// into the GEMM's TMA producer (see AShards).
sc::GemmArgs sharded_gemm(const std::vector<int64_t>& shard_ptrs, int64_t rows, int64_t own,
                          const Tensor& ready, int64_t epoch, int64_t K, const Tensor& w, int epi,
                          int64_t bn) {
  check_matrix(w, "w");
  TORCH_CHECK(!shard_ptrs.empty() && (int)shard_ptrs.size() <= sc::kMaxShards, "1..8 shards");
  TORCH_CHECK(rows % 128 == 0, "rows per shard must be a multiple of 128");
  TORCH_CHECK(K == w.size(1) && (K * 2) % 16 == 0, "K");
  CHECK_I32(ready);
  sc::GemmArgs g{};
  for (size_t r = 0; r < shard_ptrs.size(); ++r) {
    TORCH_CHECK((shard_ptrs[r] & 15) == 0, "shard base must be 16-byte aligned");
    g.a_shards[r] = reinterpret_cast<const __nv_bfloat16*>(shard_ptrs[r]);
  }
  g.a = g.a_shards[0];
  g.shards.n = (int)shard_ptrs.size();
  g.shards.rows = (int)rows;
  g.shards.own = (int)own;
  g.shards.ready = ready.data_ptr<int>();
  g.shards.epoch = (int)epoch;
  g.b = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  g.M = (int)(rows * shard_ptrs.size());
  g.N = (int)w.size(0);
  g.K = (int)K;
  g.lda = (int)K;
  g.ldb = (int)w.stride(0);
  g.epi = epi;
  g.bn = (int)bn;
  g.num_sms = num_sms();
  g.status = status_tensor(w).data_ptr<int>();
  return g;
}

void gemm_ag_qkv(std::vector<int64_t> shard_ptrs, int64_t rows, int64_t own, Tensor ready, int64_t epoch,
                 int64_t K, Tensor w_qkv, Tensor q_out, Tensor k_cache, Tensor v_cache, Tensor rope_pos,
                 Tensor cache_slot, Tensor rope_table, int64_t n_q_heads, int64_t n_kv_heads, int64_t bn,
                 c10::optional<Tensor> dev_part, int64_t dev_mode, int64_t k_peer, int64_t v_peer) {
  const c10::cuda::CUDAGuard guard(w_qkv.device());
  auto g = sharded_gemm(shard_ptrs, rows, own, ready, epoch, K, w_qkv, sc::EPI_QKV, bn);
  // optional push of this rank's K/V rows into a peer slot of the same
  // local geometry (the decode rank with the same TP index); 0 disables it
  TORCH_CHECK((k_peer == 0) == (v_peer == 0), "k_peer and v_peer go together");
  TORCH_CHECK((k_peer & 15) == 0 && (v_peer & 15) == 0, "peer K/V bases must be 16-byte aligned");
  g.ep.k_peer = reinterpret_cast<__nv_bfloat16*>(k_peer);
  g.ep.v_peer = reinterpret_cast<__nv_bfloat16*>(v_peer);
  if (dev_part.has_value() && dev_part->defined()) {
    CHECK_F32(*dev_part);
    TORCH_CHECK(dev_part->numel() >= (int64_t)g.M * 2 * n_kv_heads, "dev_part size");
    g.ep.dev_part = dev_part->data_ptr<float>();
    g.ep.dev_mode = (int)dev_mode;
  }
  check_matrix(q_out, "q_out");
  TORCH_CHECK(w_qkv.size(0) == (n_q_heads + 2 * n_kv_heads) * 128, "w_qkv rows");
  TORCH_CHECK(k_cache.dim() == 3 && k_cache.size(0) == n_kv_heads && k_cache.is_contiguous(), "k_cache");
  g.ep.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  g.ep.ldq = (int)q_out.stride(0);
  g.ep.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  g.ep.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  g.ep.cache_cap = (int)k_cache.size(1);
  g.ep.rope_pos = rope_pos.data_ptr<int>();
  g.ep.cache_slot = cache_slot.data_ptr<int>();
  g.ep.rope_table = reinterpret_cast<const float2*>(rope_table.data_ptr<float>());
  g.ep.n_q_heads = (int)n_q_heads;
  g.ep.n_kv_heads = (int)n_kv_heads;
  run_gemm(g);
}

void gemm_ag_swiglu(std::vector<int64_t> shard_ptrs, int64_t rows, int64_t own, Tensor ready, int64_t epoch,
                    int64_t K, Tensor w_gu, Tensor out, int64_t bn) {
  const c10::cuda::CUDAGuard guard(w_gu.device());
  auto g = sharded_gemm(shard_ptrs, rows, own, ready, epoch, K, w_gu, sc::EPI_SWIGLU, bn);
  check_matrix(out, "out");
  TORCH_CHECK(out.size(0) == g.M && out.size(1) == w_gu.size(0) / 2, "out shape");
  g.ep.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  g.ep.ldo = (int)out.stride(0);
  run_gemm(g);
}

// partial = a @ w^T; rows of owner r are stored into dst_ptrs[r] at slot `sender`
void gemm_rs(Tensor a, Tensor w, std::vector<int64_t> dst_ptrs, int64_t rows, int64_t sender, int64_t bn) {
  const c10::cuda::CUDAGuard guard(a.device());
  auto g = base_gemm(a, w, sc::EPI_RS, (int)bn);
  TORCH_CHECK(!dst_ptrs.empty() && (int)dst_ptrs.size() <= sc::kMaxShards, "1..8 owners");
  TORCH_CHECK(rows % 128 == 0 && rows * (int64_t)dst_ptrs.size() == a.size(0), "rows per owner");
  TORCH_CHECK(g.N % 32 == 0, "N must be a multiple of 32");
  for (size_t r = 0; r < dst_ptrs.size(); ++r) g.ep.rs_dst[r] = reinterpret_cast<void*>(dst_ptrs[r]);
  TORCH_CHECK(g.N % 64 == 0, "N must be a multiple of 64");
  g.ep.rs_rows = (int)rows;
  g.ep.rs_sender = (int)sender;
  run_gemm(g);
}

void rs_reduce(Tensor recv, Tensor flags, int64_t epoch, int64_t timeout_ns, Tensor status, Tensor residual,
               Tensor out, c10::optional<Tensor> norm_w, c10::optional<Tensor> norm_out, double eps,
               c10::optional<Tensor> epoch_ptr, int64_t epoch_mul) {
  const c10::cuda::CUDAGuard guard(recv.device());
  TORCH_CHECK(recv.scalar_type() == torch::kFloat32 || recv.scalar_type() == torch::kBFloat16, "recv fp32/bf16");
  CHECK_I32(flags); CHECK_I32(status);
  TORCH_CHECK(recv.dim() == 3 && recv.is_contiguous(), "recv [tp, rows, N]");
  check_matrix(residual, "residual");
  check_matrix(out, "out");
  sc::RsReduceArgs a{};
  a.recv = recv.data_ptr();
  a.recv_bf16 = recv.scalar_type() == torch::kBFloat16 ? 1 : 0;
  a.tp = (int)recv.size(0);
  a.rows = (int)recv.size(1);
  a.N = (int)recv.size(2);
  TORCH_CHECK(flags.numel() >= a.tp, "one flag per sender");
  TORCH_CHECK(residual.size(0) == a.rows && residual.size(1) == a.N, "residual shape");
  a.flags = flags.data_ptr<int>();
  a.epoch = (int)epoch;
  a.timeout_ns = timeout_ns;
  a.status = status.data_ptr<int>();
  a.residual = reinterpret_cast<const __nv_bfloat16*>(residual.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (norm_w.has_value() && norm_w->defined()) {
    TORCH_CHECK(norm_out.has_value() && norm_out->defined(), "norm_out required");
    a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w->data_ptr());
    a.norm_out = reinterpret_cast<__nv_bfloat16*>(norm_out->data_ptr());
  }
  a.eps = (float)eps;
  if (epoch_ptr.has_value() && epoch_ptr->defined()) {
    CHECK_I32(*epoch_ptr);
    a.epoch_ptr = epoch_ptr->data_ptr<int>();
    a.epoch_mul = (int)epoch_mul;
  }
  check_cuda(sc::rs_reduce(a, cur_stream()), "rs_reduce");
}

// Row-parallel decode projection with the all-reduce fused into the epilogue.
void gemv_allreduce(Tensor x, Tensor w, c10::optional<Tensor> norm_w, double eps, std::vector<int64_t> dst_ptrs,
                    std::vector<int64_t> flag_ptrs, int64_t sender, int64_t epoch, c10::optional<Tensor> epoch_ptr,
                    int64_t epoch_mul, Tensor counter, c10::optional<Tensor> recv, c10::optional<Tensor> wait_flags,
                    c10::optional<Tensor> residual, int64_t timeout_ns, c10::optional<Tensor> status) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto g = base_gemv(x, w, norm_w, eps, sc::GEMV_ALLREDUCE);
  TORCH_CHECK(dst_ptrs.size() == flag_ptrs.size() && !dst_ptrs.empty() && dst_ptrs.size() <= 8, "1..8 ranks");
  for (size_t r = 0; r < dst_ptrs.size(); ++r) {
    g.ar_dst[r] = reinterpret_cast<float*>(dst_ptrs[r]);
    g.ar_flag[r] = reinterpret_cast<int*>(flag_ptrs[r]);
  }
  g.ar_tp = (int)dst_ptrs.size();
  g.ar_sender = (int)sender;
  g.ar_epoch = (int)epoch;
  if (epoch_ptr.has_value() && epoch_ptr->defined()) {
    CHECK_I32(*epoch_ptr);
    g.ar_epoch_ptr = epoch_ptr->data_ptr<int>();
    g.ar_epoch_mul = (int)epoch_mul;
  }
  CHECK_I32(counter);
  g.counter = reinterpret_cast<unsigned int*>(counter.data_ptr<int>());
  if (recv.has_value() && recv->defined()) {
    // fused reduction: residual (in place) += sum over ranks of the partial rows
    TORCH_CHECK(wait_flags.has_value() && residual.has_value() && status.has_value(),
                "fused reduce needs wait_flags, residual and status");
    CHECK_F32(*recv); CHECK_I32(*wait_flags); CHECK_BF16(*residual); CHECK_I32(*status);
    TORCH_CHECK(recv->numel() >= (int64_t)g.ar_tp * g.M * g.N, "recv [tp, M, N]");
    TORCH_CHECK(wait_flags->numel() >= g.ar_tp, "one wait flag per rank");
    TORCH_CHECK(residual->dim() == 2 && residual->size(0) == g.M && residual->size(1) == g.N &&
                    residual->is_contiguous(), "residual [M, N] contiguous");
    TORCH_CHECK(g.N % 4 == 0, "N % 4");
    g.ar_recv = recv->data_ptr<float>();
    g.ar_wait_flags = wait_flags->data_ptr<int>();
    g.ar_residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    g.ar_out = reinterpret_cast<__nv_bfloat16*>(residual->data_ptr());
    g.ar_timeout_ns = timeout_ns;
    g.status = status->data_ptr<int>();
  }
  run_gemv(g);
}

// ------------------------------------------------------- page scores (K11)
Tensor page_token_scores(Tensor q, std::vector<Tensor> keys, int64_t n_tokens, double scale) {
  const c10::cuda::CUDAGuard guard(q.device());
  CHECK_CUDA(q); CHECK_F32(q);
  TORCH_CHECK(q.dim() == 4 && q.size(3) == 128 && q.is_contiguous(), "q [layers, rows, q_heads, 128] fp32");
  const int L = (int)q.size(0);
  TORCH_CHECK(L >= 1 && L <= sc::kPsMaxLayers && (int)keys.size() == L, "1..8 layers, one key tensor each");
  sc::PageScoreArgs a{};
  a.q = q.data_ptr<float>();
  for (int l = 0; l < L; ++l) {
    const Tensor& k = keys[l];
    CHECK_CUDA(k); CHECK_BF16(k); CHECK_ALIGN16(k);
    TORCH_CHECK(k.dim() == 3 && k.size(2) == 128 && k.is_contiguous(), "keys [kv_heads, capacity, 128]");
    TORCH_CHECK(k.sizes() == keys[0].sizes(), "every layer's keys have the same shape");
    a.keys[l] = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  }
  a.cache_cap = (int)keys[0].size(1);
  a.n_layers = L;
  a.n_rows = (int)q.size(1);
  a.n_q_heads = (int)q.size(2);
  a.n_kv_heads = (int)keys[0].size(0);
  a.n_tokens = (int)n_tokens;
  a.scale = (float)scale;
  const int64_t n = (int64_t)L * a.n_rows * a.n_q_heads;
  const int64_t chunks = (n_tokens + 255) / 256;
  auto f32 = torch::TensorOptions().dtype(torch::kFloat32).device(q.device());
  Tensor logits = torch::empty({n, std::max<int64_t>(n_tokens, 1)}, f32);
  Tensor partials = torch::empty({n, std::max<int64_t>(chunks, 1), 2}, f32);
  Tensor stats = torch::empty({n, 2}, f32);
  Tensor out = torch::empty({std::max<int64_t>(n_tokens, 1)}, f32);
  a.logits = logits.data_ptr<float>();
  a.partials = reinterpret_cast<float2*>(partials.data_ptr<float>());
  a.stats = reinterpret_cast<float2*>(stats.data_ptr<float>());
  a.token_scores = out.data_ptr<float>();
  check_cuda(sc::page_token_scores(a, cur_stream()), "page_token_scores");
  return out;
}

// ---------------------------------------------------------------- p2p
std::tuple<Tensor, py::bytes> shared_empty(int64_t nbytes, int64_t device) {
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  check_cuda(cudaMalloc(&p, (size_t)nbytes), "cudaMalloc (shared buffer)");
  check_cuda(cudaMemset(p, 0, (size_t)nbytes), "cudaMemset (shared buffer)");
  cudaIpcMemHandle_t h;
  check_cuda(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  Tensor t = torch::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
  return {t, py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

int64_t shared_open(py::bytes handle) {
  std::string raw = handle;
  TORCH_CHECK(raw.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, raw.data(), sizeof(h));
  void* p = nullptr;
  check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}

void shared_close(int64_t ptr) {
  check_cuda(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle");
}

void peer_signal(int64_t flag_ptr, int64_t value, c10::optional<Tensor> stamp,
                 c10::optional<Tensor> value_src) {
  unsigned long long* st = nullptr;
  if (stamp.has_value() && stamp->defined()) st = reinterpret_cast<unsigned long long*>(stamp->data_ptr<int64_t>());
  const int* src = nullptr;
  if (value_src.has_value() && value_src->defined()) { CHECK_I32(*value_src); src = value_src->data_ptr<int>(); }
  check_cuda(sc::peer_signal(reinterpret_cast<int*>(flag_ptr), (int)value, src, st, cur_stream()), "peer_signal");
}

void wait_flag(Tensor flags, int64_t index, int64_t target, int64_t timeout_ns, Tensor status,
               c10::optional<Tensor> stamp) {
  const c10::cuda::CUDAGuard guard(flags.device());
  CHECK_I32(flags); CHECK_I32(status);
  TORCH_CHECK(index >= 0 && index < flags.numel(), "flag index");
  unsigned long long* st = nullptr;
  if (stamp.has_value() && stamp->defined()) st = reinterpret_cast<unsigned long long*>(stamp->data_ptr<int64_t>());
  check_cuda(sc::wait_flag(flags.data_ptr<int>() + index, (int)target, (long long)timeout_ns,
                           status.data_ptr<int>(), st, cur_stream()), "wait_flag");
}

// ---------------------------------------------------------------- GEMV
sc::GemvArgs base_gemv(const Tensor& x, const Tensor& w, c10::optional<Tensor> norm_w, double eps,
                       int epi) {
  check_matrix(x, "x");
  check_matrix(w, "w");
  TORCH_CHECK(x.size(1) == w.size(1), "K mismatch");
  sc::GemvArgs g{};
  g.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  g.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  g.ldx = (int)x.stride(0);
  g.M = (int)x.size(0);
  g.N = (int)w.size(0);
  g.K = (int)w.size(1);
  if (norm_w.has_value() && norm_w->defined()) {
    CHECK_BF16(*norm_w);
    CHECK_ALIGN16(*norm_w);
    g.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w->data_ptr());
  }
  g.eps = (float)eps;
  g.epi = epi;
  g.num_sms = num_sms();
  return g;
}

void run_gemv(const sc::GemvArgs& g) { check_cuda(sc::gemv_bf16(g, cur_stream()), "gemv_bf16"); }

void gemv_store(Tensor x, Tensor w, c10::optional<Tensor> norm_w, double eps, Tensor out) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto g = base_gemv(x, w, norm_w, eps, sc::GEMV_STORE);
  CHECK_BF16(out);
  g.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  g.ldo = (int)out.stride(0);
  run_gemv(g);
}

void gemv_residual(Tensor x, Tensor w, c10::optional<Tensor> norm_w, double eps, Tensor out,
                   Tensor residual) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto g = base_gemv(x, w, norm_w, eps, sc::GEMV_RESIDUAL);
  CHECK_BF16(out); CHECK_BF16(residual);
  g.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  g.ldo = (int)out.stride(0);
  g.residual = reinterpret_cast<const __nv_bfloat16*>(residual.data_ptr());
  g.ldr = (int)residual.stride(0);
  run_gemv(g);
}

void gemv_swiglu(Tensor x, Tensor w_gu, c10::optional<Tensor> norm_w, double eps, Tensor out) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto g = base_gemv(x, w_gu, norm_w, eps, sc::GEMV_SWIGLU);
  CHECK_BF16(out);
  TORCH_CHECK(w_gu.size(0) % 256 == 0, "gate/up rows must be a multiple of 256");
  g.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  g.ldo = (int)out.stride(0);
  run_gemv(g);
}

void gemv_qkv(Tensor x, Tensor w_qkv, c10::optional<Tensor> norm_w, double eps, Tensor q_out,
              Tensor k_cache, Tensor v_cache, Tensor pos, Tensor rope_table, int64_t n_q_heads,
              int64_t n_kv_heads, c10::optional<Tensor> slot) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto g = base_gemv(x, w_qkv, norm_w, eps, sc::GEMV_QKV);
  CHECK_I32(pos); CHECK_F32(rope_table);
  TORCH_CHECK(w_qkv.size(0) == (n_q_heads + 2 * n_kv_heads) * 128, "w_qkv rows");
  TORCH_CHECK(k_cache.dim() == 3 && k_cache.size(2) == 128 && k_cache.is_contiguous(), "k_cache");
  g.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  g.ldq = (int)q_out.stride(0);
  g.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  g.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  g.cache_cap = (int)k_cache.size(1);
  g.pos = pos.data_ptr<int>();
  if (slot.has_value() && slot->defined()) {
    CHECK_I32(*slot);
    g.slot = slot->data_ptr<int>();
  }
  g.rope_table = reinterpret_cast<const float2*>(rope_table.data_ptr<float>());
  g.n_q_heads = (int)n_q_heads;
  g.n_kv_heads = (int)n_kv_heads;
  run_gemv(g);
}

int64_t gemv_argmax_grid(int64_t n_rows) {
  const int64_t pairs = n_rows / 2;
  int64_t grid = (pairs + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 8;
  return grid < cap ? grid : cap;
}

void gemv_argmax(Tensor x, Tensor w, c10::optional<Tensor> norm_w, double eps, Tensor part_val,
                 Tensor part_idx, Tensor counter, Tensor out_token,
                 c10::optional<Tensor> token_log, c10::optional<Tensor> gen_count,
                 c10::optional<Tensor> embed, c10::optional<Tensor> next_hidden,
                 c10::optional<Tensor> pos_advance, int64_t n_advance) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto g = base_gemv(x, w, norm_w, eps, sc::GEMV_ARGMAX);
  CHECK_F32(part_val); CHECK_I32(part_idx); CHECK_I32(out_token);
  const int64_t grid = gemv_argmax_grid(w.size(0));
  TORCH_CHECK(part_val.numel() >= grid * x.size(0) && part_idx.numel() >= grid * x.size(0),
              "argmax partial buffers too small");
  g.part_val = part_val.data_ptr<float>();
  g.part_idx = part_idx.data_ptr<int>();
  g.counter = reinterpret_cast<unsigned int*>(counter.data_ptr<int>());
  g.out_token = out_token.data_ptr<int>();
  if (token_log.has_value() && token_log->defined()) {
    TORCH_CHECK(gen_count.has_value() && gen_count->defined(), "gen_count required");
    g.token_log = token_log->data_ptr<int>();
    g.gen_count = gen_count->data_ptr<int>();
  }
  if (embed.has_value() && embed->defined()) {
    TORCH_CHECK(next_hidden.has_value() && next_hidden->defined(), "next_hidden required");
    g.embed = reinterpret_cast<const __nv_bfloat16*>(embed->data_ptr());
    g.next_hidden = reinterpret_cast<__nv_bfloat16*>(next_hidden->data_ptr());
  }
  if (pos_advance.has_value() && pos_advance->defined()) {
    CHECK_I32(*pos_advance);
    TORCH_CHECK(pos_advance->numel() >= std::max<int64_t>(1, n_advance), "pos_advance too short");
    g.pos_advance = pos_advance->data_ptr<int>();
    g.n_advance = (int)n_advance;
  }
  run_gemv(g);
}

// ----------------------------------------------------------- attention
int64_t attention_prefill_impl(Tensor q, c10::optional<Tensor> q_rows, Tensor qpos, Tensor k_cache,
                            Tensor v_cache, c10::optional<Tensor> kpos, int64_t n_keys,
                            int64_t n_heads, double scale, Tensor out, bool legacy,
                            c10::optional<Tensor> trace = c10::nullopt,
                            c10::optional<Tensor> ws = c10::nullopt) {
  const c10::cuda::CUDAGuard guard(q.device());
  check_matrix(q, "q");
  check_matrix(out, "out");
  CHECK_I32(qpos);
  TORCH_CHECK(k_cache.dim() == 3 && k_cache.size(2) == 128 && k_cache.is_contiguous(), "k_cache");
  TORCH_CHECK(v_cache.sizes() == k_cache.sizes() && v_cache.is_contiguous(), "v_cache");
  TORCH_CHECK(n_keys <= k_cache.size(1), "n_keys exceeds cache capacity");
  sc::AttnPrefillArgs p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.ldq = (int)q.stride(0);
  if (q_rows.has_value() && q_rows->defined()) {
    CHECK_I32(*q_rows);
    p.q_rows = q_rows->data_ptr<int>();
  }
  p.qpos = qpos.data_ptr<int>();
  p.n_rows = (int)out.size(0);
  TORCH_CHECK(qpos.numel() >= p.n_rows, "qpos too short");
  p.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  p.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  p.cache_cap = (int)k_cache.size(1);
  if (kpos.has_value() && kpos->defined()) {
    CHECK_I32(*kpos);
    TORCH_CHECK(kpos->numel() >= n_keys, "kpos too short");
    p.kpos = kpos->data_ptr<int>();
  }
  p.n_keys = (int)n_keys;
  p.n_heads = (int)n_heads;
  p.n_kv_heads = (int)k_cache.size(0);
  p.head_dim = 128;
  p.scale = (float)scale;
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldo = (int)out.stride(0);
  p.status = status_tensor(q).data_ptr<int>();
  if (trace.has_value() && trace->defined()) {
    TORCH_CHECK(trace->scalar_type() == torch::kInt64 && trace->numel() >= 640 && trace->is_cuda(),
                "trace must be a CUDA int64 tensor of >= 640 entries");
    p.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  if (ws.has_value() && ws->defined()) {
    CHECK_F32(*ws);
    CHECK_ALIGN16(*ws);
    p.ws = ws->data_ptr<float>();
    p.ws_floats = ws->numel();
  }
  TORCH_CHECK(k_cache.is_cuda() && v_cache.is_cuda(), "caches must be CUDA tensors");
  CHECK_BF16(k_cache); CHECK_BF16(v_cache);
  CHECK_ALIGN16(k_cache); CHECK_ALIGN16(v_cache);
  TORCH_CHECK(n_heads % k_cache.size(0) == 0, "n_heads must be a multiple of the kv heads");
  TORCH_CHECK(q.size(1) >= n_heads * 128 && out.size(1) >= n_heads * 128, "q / out narrower than n_heads * 128");
  if (legacy) {
    check_cuda(sc::attention_prefill_mma(p, cur_stream()), "attention_prefill_mma");
    return 1;
  } else {
    check_cuda(sc::attention_prefill(p, cur_stream()), "attention_prefill");
    return sc::attention_prefill_splits(p, num_sms()) > 1 ? 2 : 1;  // + the merge kernel
  }
}

// returns the kernels launched (2 when the keys were split: + the merge)
int64_t attention_prefill(Tensor q, c10::optional<Tensor> q_rows, Tensor qpos, Tensor k_cache,
                          Tensor v_cache, c10::optional<Tensor> kpos, int64_t n_keys,
                          int64_t n_heads, double scale, Tensor out, c10::optional<Tensor> trace,
                          c10::optional<Tensor> ws) {
  return attention_prefill_impl(q, q_rows, qpos, k_cache, v_cache, kpos, n_keys, n_heads, scale, out, false, trace, ws);
}

int64_t attention_prefill_mma(Tensor q, c10::optional<Tensor> q_rows, Tensor qpos, Tensor k_cache,
                              Tensor v_cache, c10::optional<Tensor> kpos, int64_t n_keys,
                              int64_t n_heads, double scale, Tensor out) {
  return attention_prefill_impl(q, q_rows, qpos, k_cache, v_cache, kpos, n_keys, n_heads, scale, out, true);
}

void attention_decode(Tensor q, Tensor k_cache, Tensor v_cache, Tensor pos, int64_t n_heads,
                      double scale, int64_t splits, Tensor out, c10::optional<Tensor> page_table,
                      int64_t page_shift, c10::optional<Tensor> n_virtual, c10::optional<Tensor> ws,
                      c10::optional<Tensor> counters, int64_t outer, c10::optional<Tensor> pos_rows,
                      int64_t seq_stride, std::vector<Tensor> l2_prefetch, int64_t l2_prefetch_bytes,
                      int64_t key_capacity) {
  const c10::cuda::CUDAGuard guard(q.device());
  CHECK_BF16(q); CHECK_BF16(out); CHECK_I32(pos);
  // key_capacity > 0 sizes the split for that many keys (it must bound the call's key count:
  // a sparse view's visible keys plus the query rows); 0 sizes it for the whole cache
  TORCH_CHECK(key_capacity >= 0 && key_capacity <= k_cache.size(1) + 64, "key_capacity");
  TORCH_CHECK(key_capacity == 0 || (page_table.has_value() && page_table->defined()),
              "key_capacity applies to paged views only");
  TORCH_CHECK(k_cache.dim() == 3 && k_cache.size(2) == 128 && k_cache.is_contiguous(), "k_cache");
  sc::AttnDecodeArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.M = (int)q.size(0);
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  a.cache_cap = (int)k_cache.size(1);
  a.pos = pos.data_ptr<int>();
  a.n_heads = (int)n_heads;
  a.n_kv_heads = (int)k_cache.size(0);
  a.scale = (float)scale;
  a.splits = (int)splits;
  a.key_cap = (int)key_capacity;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (page_table.has_value() && page_table->defined()) {
    CHECK_I32(*page_table);
    a.page_table = page_table->data_ptr<int>();
    a.page_shift = (int)page_shift;
  }
  if (n_virtual.has_value() && n_virtual->defined()) {
    CHECK_I32(*n_virtual);
    a.n_virtual = n_virtual->data_ptr<int>();
  }
  if (ws.has_value() && ws->defined()) {
    TORCH_CHECK(counters.has_value() && counters->defined(), "counters required with ws");
    CHECK_F32(*ws); CHECK_I32(*counters);
    TORCH_CHECK(ws->numel() >= (int64_t)a.n_kv_heads * 16 * 64 * 130, "ws too small");
    TORCH_CHECK(counters->numel() >= (int64_t)a.n_kv_heads * 16, "16 counters per kv head");
    a.ws = ws->data_ptr<float>();
    a.counters = reinterpret_cast<unsigned*>(counters->data_ptr<int>());
  }
  TORCH_CHECK(outer >= 0 && outer <= 16, "outer: 0 (automatic) or 1..16 clusters per kv head");
  a.outer = (int)outer;
  if (pos_rows.has_value() && pos_rows->defined()) {
    CHECK_I32(*pos_rows);
    TORCH_CHECK(q.size(0) == pos_rows->numel() && out.size(0) == pos_rows->numel(),
                "batched decode attention: one q / out row per sequence");
    TORCH_CHECK(seq_stride >= 0 && seq_stride % 8 == 0, "seq_stride (elements) must keep rows 16-byte aligned");
    a.pos_rows = pos_rows->data_ptr<int>();
    a.seq_stride = seq_stride;
    a.n_seq = (int)pos_rows->numel();
    a.M = 1;
  }
  // L2 prefetch: the listed tensors in order, the first fully, the rest while
  // the byte budget lasts (whole 16-byte units)
  TORCH_CHECK(l2_prefetch.size() <= 2, "at most two l2_prefetch tensors");
  TORCH_CHECK(l2_prefetch_bytes >= 0, "l2_prefetch_bytes");
  long long left = l2_prefetch_bytes;
  for (size_t i = 0; i < l2_prefetch.size(); ++i) {
    const Tensor& t = l2_prefetch[i];
    TORCH_CHECK(t.is_cuda() && t.device() == q.device() && t.is_contiguous(), "l2_prefetch: contiguous tensors on q's device");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, "l2_prefetch: 16-byte aligned base");
    const long long nb = (long long)(t.numel() * t.element_size()) & ~15LL;
    const long long take = std::min(nb, left);
    a.pf_ptr[i] = t.data_ptr();
    a.pf_bytes[i] = take;
    left -= take;
  }
  check_cuda(sc::attention_decode(a, cur_stream()), "attention_decode");
}

// ------------------------------------------------- recurrent attention (K14)
static sc::RecurrentAttnArgs recurrent_args(const Tensor& q, const Tensor& k, const Tensor& v, double scale) {
  CHECK_BF16(q); CHECK_BF16(k); CHECK_BF16(v);
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "CUDA tensors");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && q.is_contiguous(), "q [B, Hq, 128] contiguous");
  TORCH_CHECK(k.dim() == 4 && k.size(3) == 128 && k.is_contiguous() && k.size(0) == q.size(0),
              "k [B, Hkv, P, 128] contiguous");
  TORCH_CHECK(v.sizes() == k.sizes() && v.is_contiguous(), "v like k");
  TORCH_CHECK(q.size(1) % k.size(1) == 0 && q.size(1) / k.size(1) <= 8, "Hq = G * Hkv, G <= 8");
  TORCH_CHECK(k.size(2) >= 1 && k.size(2) <= sc::kRecurrentAttnMaxKeys, "1..1024 keys");
  sc::RecurrentAttnArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.batch = (int)q.size(0);
  a.n_heads = (int)q.size(1);
  a.n_kv_heads = (int)k.size(1);
  a.n_keys = (int)k.size(2);
  a.scale = (float)scale;
  return a;
}

std::vector<Tensor> recurrent_attention_fwd(Tensor q, Tensor k, Tensor v, double scale) {
  const c10::cuda::CUDAGuard guard(q.device());
  auto a = recurrent_args(q, k, v, scale);
  Tensor out = torch::empty_like(q);
  Tensor lse = torch::empty({q.size(0), q.size(1)}, q.options().dtype(torch::kFloat32));
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  check_cuda(sc::recurrent_attention_fwd(a, cur_stream()), "recurrent_attention_fwd");
  return {out, lse};
}

std::vector<Tensor> recurrent_attention_bwd(Tensor q, Tensor k, Tensor v, Tensor out, Tensor lse, Tensor dout,
                                            double scale) {
  const c10::cuda::CUDAGuard guard(q.device());
  auto a = recurrent_args(q, k, v, scale);
  CHECK_BF16(out); CHECK_BF16(dout); CHECK_F32(lse);
  TORCH_CHECK(out.sizes() == q.sizes() && dout.sizes() == q.sizes() && out.is_contiguous() &&
                  dout.is_contiguous(), "out / dout like q");
  TORCH_CHECK(lse.numel() == q.size(0) * q.size(1), "lse [B, Hq]");
  Tensor dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  check_cuda(sc::recurrent_attention_bwd(a, cur_stream()), "recurrent_attention_bwd");
  return {dq, dk, dv};
}

// ------------------------------------------------------------ pointwise
void rmsnorm(Tensor x, c10::optional<Tensor> rows, Tensor w, double eps, Tensor out) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_matrix(x, "x");
  check_matrix(out, "out");
  const int* r = nullptr;
  if (rows.has_value() && rows->defined()) { CHECK_I32(*rows); r = rows->data_ptr<int>(); }
  check_cuda(sc::rmsnorm_bf16(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                              (int)x.stride(0), r,
                              reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                              reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)out.stride(0),
                              (int)out.size(0), (int)out.size(1), (float)eps, cur_stream()),
             "rmsnorm");
}

void embedding(Tensor ids, Tensor table, Tensor out) {
  const c10::cuda::CUDAGuard guard(ids.device());
  CHECK_I32(ids);
  check_matrix(table, "table");
  check_matrix(out, "out");
  check_cuda(sc::embedding_bf16(ids.data_ptr<int>(),
                                reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
                                reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)ids.numel(),
                                (int)table.size(1), cur_stream()),
             "embedding");
}

void gather_rows(Tensor x, Tensor rows, Tensor out) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_matrix(x, "x");
  check_matrix(out, "out");
  CHECK_I32(rows);
  check_cuda(sc::gather_rows_bf16(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                  (int)x.stride(0), rows.data_ptr<int>(),
                                  reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                  (int)out.stride(0), (int)out.size(0), (int)out.size(1),
                                  cur_stream()),
             "gather_rows");
}

// docs: int32 [n_docs, 6] = (ptr_lo, ptr_hi, n_tokens, src_pos, dst_slot, dst_pos), on device
void compose_relocate(Tensor docs, Tensor offsets, int64_t total_tokens, int64_t layer_begin,
                      int64_t layer_end, int64_t n_layers, Tensor cache, int64_t n_kv_heads,
                      Tensor rope_table) {
  const c10::cuda::CUDAGuard guard(cache.device());
  CHECK_I32(docs); CHECK_I32(offsets); CHECK_BF16(cache); CHECK_F32(rope_table);
  TORCH_CHECK(docs.is_cuda() && offsets.is_cuda(), "docs/offsets on device");
  TORCH_CHECK(docs.dim() == 2 && docs.size(1) == 6 && docs.is_contiguous(), "docs [n, 6]");
  TORCH_CHECK(cache.dim() == 5 && cache.size(1) == 2 && cache.size(2) == n_kv_heads &&
                  cache.size(4) == 128 && cache.is_contiguous(),
              "cache must be [L, 2, n_kv_heads, cap, 128]");
  static_assert(sizeof(sc::ComposeDoc) == 24, "ComposeDoc layout");
  sc::ComposeArgs a{};
  a.docs = reinterpret_cast<const sc::ComposeDoc*>(docs.data_ptr<int>());
  a.n_docs = (int)docs.size(0);
  a.doc_token_offset = offsets.data_ptr<int>();
  a.total_tokens = (int)total_tokens;
  a.layer_begin = (int)layer_begin;
  a.layer_end = (int)layer_end;
  a.n_layers = (int)n_layers;
  a.cache = reinterpret_cast<__nv_bfloat16*>(cache.data_ptr());
  a.cache_cap = (int)cache.size(3);
  a.n_kv_heads = (int)n_kv_heads;
  a.rope_table = reinterpret_cast<const float2*>(rope_table.data_ptr<float>());
  check_cuda(sc::compose_relocate(a, cur_stream()), "compose_relocate");
}

void cacheblend_select(Tensor dev_part, int64_t n_kv_heads, int64_t dev_mode, int64_t total_rows,
                       int64_t doc_begin, int64_t doc_end, int64_t k, bool keep_prefix,
                       Tensor active, Tensor n_active, Tensor scores,
                       c10::optional<Tensor> checksum, int64_t n_parts, int64_t part_stride) {
  const c10::cuda::CUDAGuard guard(dev_part.device());
  CHECK_F32(dev_part); CHECK_I32(active); CHECK_I32(n_active); CHECK_F32(scores);
  TORCH_CHECK(scores.numel() >= std::max<int64_t>(1, doc_end - doc_begin), "scores scratch");
  sc::SelectArgs a{};
  a.dev_part = dev_part.data_ptr<float>();
  a.n_kv_heads = (int)n_kv_heads;
  a.dev_mode = (int)dev_mode;
  a.total_rows = (int)total_rows;
  a.doc_begin = (int)doc_begin;
  a.doc_end = (int)doc_end;
  a.k = (int)k;
  a.keep_prefix = keep_prefix ? 1 : 0;
  a.active = active.data_ptr<int>();
  a.n_active = n_active.data_ptr<int>();
  a.scores = scores.data_ptr<float>();
  TORCH_CHECK(n_parts >= 1 && (n_parts == 1 || part_stride >= total_rows * 2 * n_kv_heads), "partial layout");
  TORCH_CHECK(dev_part.numel() >= (n_parts - 1) * part_stride + total_rows * 2 * n_kv_heads, "dev_part size");
  a.n_parts = (int)n_parts;
  a.part_stride = part_stride;
  if (checksum.has_value() && checksum->defined()) {
    TORCH_CHECK(checksum->scalar_type() == torch::kInt64, "checksum int64");
    a.checksum = reinterpret_cast<long long*>(checksum->data_ptr<int64_t>());
  }
  check_cuda(sc::cacheblend_select(a, cur_stream()), "cacheblend_select");
}

sc::SkinnyArgs skinny_base(const Tensor& x, const Tensor& w, int64_t epi, const Tensor& ws, int64_t splits) {
  check_matrix(x, "x");
  check_matrix(w, "w");
  TORCH_CHECK(x.size(1) == w.size(1), "K mismatch");
  CHECK_F32(ws);
  sc::SkinnyArgs a{};
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  a.M = (int)x.size(0);
  a.N = (int)w.size(0);
  a.K = (int)w.size(1);
  a.ldx = (int)x.stride(0);
  a.ldw = (int)w.stride(0);
  a.epi = (int)epi;
  a.num_sms = num_sms();
  a.splits = splits > 0 ? (int)splits : sc::skinny_splits(a.N, a.K, a.num_sms);
  TORCH_CHECK(a.M >= 1 && a.M <= 64, "the skinny GEMM takes 1..64 rows");
  TORCH_CHECK(ws.numel() >= (int64_t)a.splits * a.N * sc::skinny_bn(a.M), "workspace [splits][N][bn] too small");
  a.ws = ws.data_ptr<float>();
  a.status = status_tensor(w).data_ptr<int>();
  return a;
}

// out = epilogue(x @ w^T) for M <= 64 rows on the tensor cores; returns kernels launched.
int64_t skinny_gemm(Tensor x, Tensor w, int64_t epi, Tensor out, c10::optional<Tensor> residual, Tensor ws,
                    int64_t splits) {
  const c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(epi == sc::SKINNY_STORE || epi == sc::SKINNY_RESIDUAL || epi == sc::SKINNY_SWIGLU, "epilogue");
  auto a = skinny_base(x, w, epi, ws, splits);
  check_matrix(out, "out");
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = (int)out.stride(0);
  TORCH_CHECK(out.size(0) >= a.M && out.size(1) == (epi == sc::SKINNY_SWIGLU ? a.N / 2 : a.N), "out shape");
  if (epi == sc::SKINNY_RESIDUAL) {
    TORCH_CHECK(residual.has_value() && residual->defined(), "residual required");
    check_matrix(*residual, "residual");
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ldr = (int)residual->stride(0);
  }
  check_cuda(sc::skinny_gemm(a, cur_stream()), "skinny_gemm");
  return 2;
}

// Fused QKV (RoPE + K/V cache write) for M <= 64 rows on the tensor cores.
int64_t skinny_qkv(Tensor x, Tensor w_qkv, Tensor q_out, Tensor k_cache, Tensor v_cache, Tensor pos,
                   Tensor rope_table, int64_t n_q_heads, int64_t n_kv_heads, Tensor ws, c10::optional<Tensor> slot,
                   c10::optional<Tensor> pos_rows, int64_t seq_stride) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto a = skinny_base(x, w_qkv, sc::SKINNY_QKV, ws, -1);
  TORCH_CHECK(w_qkv.size(0) == (n_q_heads + 2 * n_kv_heads) * 128, "w_qkv rows");
  TORCH_CHECK(k_cache.dim() == 3 && k_cache.size(2) == 128 && k_cache.is_contiguous(), "k_cache");
  CHECK_I32(pos); CHECK_F32(rope_table);
  a.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  a.ldq = (int)q_out.stride(0);
  a.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  a.cache_cap = (int)k_cache.size(1);
  a.pos = pos.data_ptr<int>();
  if (slot.has_value() && slot->defined()) { CHECK_I32(*slot); a.slot = slot->data_ptr<int>(); }
  if (pos_rows.has_value() && pos_rows->defined()) {
    CHECK_I32(*pos_rows);
    TORCH_CHECK(pos_rows->numel() >= a.M && seq_stride >= 0, "pos_rows [M] and a sequence stride");
    a.pos_rows = pos_rows->data_ptr<int>();
    a.seq_stride = seq_stride;
  }
  a.rope_table = reinterpret_cast<const float2*>(rope_table.data_ptr<float>());
  a.n_q_heads = (int)n_q_heads;
  a.n_kv_heads = (int)n_kv_heads;
  check_cuda(sc::skinny_gemm(a, cur_stream()), "skinny_qkv");
  return 2;
}

// Row-parallel projection whose fp32 partial rows go to every rank's receive slot (tensor parallel).
int64_t skinny_allreduce(Tensor x, Tensor w, std::vector<int64_t> dst_ptrs, std::vector<int64_t> flag_ptrs,
                         int64_t sender, int64_t epoch, c10::optional<Tensor> epoch_ptr, int64_t epoch_mul,
                         Tensor counter, Tensor ws) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto a = skinny_base(x, w, sc::SKINNY_ALLREDUCE, ws, -1);
  TORCH_CHECK(dst_ptrs.size() == flag_ptrs.size() && !dst_ptrs.empty() && dst_ptrs.size() <= 8, "1..8 ranks");
  for (size_t r = 0; r < dst_ptrs.size(); ++r) {
    a.ar_dst[r] = reinterpret_cast<float*>(dst_ptrs[r]);
    a.ar_flag[r] = reinterpret_cast<int*>(flag_ptrs[r]);
  }
  a.ar_tp = (int)dst_ptrs.size();
  a.ar_sender = (int)sender;
  a.ar_epoch = (int)epoch;
  if (epoch_ptr.has_value() && epoch_ptr->defined()) {
    CHECK_I32(*epoch_ptr);
    a.ar_epoch_ptr = epoch_ptr->data_ptr<int>();
    a.ar_epoch_mul = (int)epoch_mul;
  }
  CHECK_I32(counter);
  a.counter = reinterpret_cast<unsigned int*>(counter.data_ptr<int>());
  check_cuda(sc::skinny_gemm(a, cur_stream()), "skinny_allreduce");
  return 2;
}

// ------------------------------------------- token-column GEMM (64 < M <= 512)
// stream-K arrival counters of the token-column GEMM: one zeroed buffer per
// device, every counter returned to zero by the launch that used it
static Tensor wide_tickets(const Tensor& like) {
  static std::mutex lock;
  static std::map<int, Tensor> bufs;
  std::lock_guard<std::mutex> guard(lock);
  const int dev = like.get_device();
  auto it = bufs.find(dev);
  if (it == bufs.end()) it = bufs.emplace(dev, torch::zeros({4096}, like.options().dtype(torch::kInt32))).first;
  return it->second;
}

static bool g_wide_stream_k = true;

static sc::WideArgs wide_base(const Tensor& x, const Tensor& w, int epi, int64_t acc, int64_t n_tt, int64_t splits) {
  check_matrix(x, "x");
  check_matrix(w, "w");
  TORCH_CHECK(x.size(1) == w.size(1), "K mismatch");
  sc::WideArgs a{};
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  a.M = (int)x.size(0);
  a.N = (int)w.size(0);
  a.K = (int)w.size(1);
  a.ldx = (int)x.stride(0);
  a.ldw = (int)w.stride(0);
  a.epi = epi;
  a.num_sms = num_sms();
  a.status = status_tensor(w).data_ptr<int>();
  TORCH_CHECK(a.M >= 1 && a.M <= 512, "the token-column GEMM takes 1..512 rows");
  sc::WidePlan p{};
  TORCH_CHECK(sc::wide_plan(a.M, a.N, a.K, epi, a.num_sms, (int)acc, (int)n_tt, (int)splits, g_wide_stream_k, &p),
              "no token-column GEMM plan for this shape (K % 64, N % 128 or % 256 for SwiGLU)");
  static_cast<sc::WidePlan&>(a) = p;
  return a;
}

// stream-K tail workspace (allocated by the caller's stream-ordered allocator)
static Tensor wide_stream_k(sc::WideArgs& a, const Tensor& like) {
  if (a.sk_tail <= 0) return Tensor();
  TORCH_CHECK(a.sk_tail <= 4096, "too many stream-K tail units");
  Tensor ws = torch::empty({(int64_t)a.sk_tail * a.sk_max_pieces * a.acc * a.bn * 128},
                           like.options().dtype(torch::kFloat32));
  a.sk_ws = ws.data_ptr<float>();
  a.sk_tickets = reinterpret_cast<unsigned*>(wide_tickets(like).data_ptr<int>());
  return ws;
}

static Tensor wide_partials(sc::WideArgs& a, const Tensor& like) {
  Tensor ws = torch::empty({a.splits, a.M, a.N}, like.options().dtype(torch::kFloat32));
  a.ws = ws.data_ptr<float>();
  Tensor sk = wide_stream_k(a, like);
  check_cuda(sc::wide_gemm(a, cur_stream()), "wide_gemm");
  return ws;
}

// out = silu(gate) * up for gate/up interleaved in 128-row blocks; one kernel.
int64_t wide_swiglu(Tensor x, Tensor w_gu, Tensor out) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto a = wide_base(x, w_gu, sc::WIDE_SWIGLU, 2, 0, 1);
  check_matrix(out, "out");
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == w_gu.size(0) / 2, "out shape");
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = (int)out.stride(0);
  Tensor sk = wide_stream_k(a, x);
  check_cuda(sc::wide_gemm(a, cur_stream()), "wide_swiglu");
  return 1;
}

// out = [residual +] bf16(x @ w^T), optionally norm_out = RMSNorm(out) (fused
// into the reduce); two kernels.
int64_t wide_residual(Tensor x, Tensor w, Tensor out, c10::optional<Tensor> residual, c10::optional<Tensor> norm_w,
                      double eps, c10::optional<Tensor> norm_out, int64_t acc, int64_t n_tt, int64_t splits) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto a = wide_base(x, w, sc::WIDE_PARTIAL, acc, n_tt, splits);
  check_matrix(out, "out");
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == w.size(0), "out shape");
  TORCH_CHECK(a.N % 8 == 0, "N % 8");
  const __nv_bfloat16* res = nullptr;
  int ldr = 0;
  if (residual.has_value() && residual->defined()) {
    check_matrix(*residual, "residual");
    TORCH_CHECK(residual->sizes() == out.sizes(), "residual shape");
    res = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    ldr = (int)residual->stride(0);
  }
  Tensor ws = wide_partials(a, x);
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (norm_w.has_value() && norm_w->defined()) {
    TORCH_CHECK(res != nullptr, "the fused norm needs the residual epilogue");
    TORCH_CHECK(norm_out.has_value() && norm_out->defined(), "norm_out required with norm_w");
    CHECK_BF16(*norm_w); check_matrix(*norm_out, "norm_out");
    TORCH_CHECK(norm_w->numel() == a.N && norm_out->sizes() == out.sizes() && a.N <= 8192, "norm shapes");
    check_cuda(sc::splitk_reduce_norm(a.ws, a.splits, a.M, a.N, res, ldr, o, (int)out.stride(0),
                                      reinterpret_cast<const __nv_bfloat16*>(norm_w->data_ptr()), (float)eps,
                                      reinterpret_cast<__nv_bfloat16*>(norm_out->data_ptr()), (int)norm_out->stride(0),
                                      cur_stream()),
               "splitk_reduce_norm");
  } else {
    check_cuda(sc::splitk_reduce(a.ws, a.splits, a.M, a.N, res, ldr, o, (int)out.stride(0), cur_stream()),
               "splitk_reduce");
  }
  return 2;
}

// Fused QKV rows -> RoPE at rope_pos[m], Q to q_out, K/V to cache slot cache_slot[m]; two kernels.
int64_t wide_qkv(Tensor x, Tensor w_qkv, Tensor q_out, Tensor k_cache, Tensor v_cache, Tensor rope_pos,
                 Tensor cache_slot, Tensor rope_table, int64_t n_q_heads, int64_t n_kv_heads, int64_t acc,
                 int64_t n_tt, int64_t splits) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto a = wide_base(x, w_qkv, sc::WIDE_PARTIAL, acc, n_tt, splits);
  TORCH_CHECK(w_qkv.size(0) == (n_q_heads + 2 * n_kv_heads) * 128, "w_qkv rows");
  check_matrix(q_out, "q_out");
  TORCH_CHECK(q_out.size(0) >= x.size(0) && q_out.size(1) == n_q_heads * 128, "q_out shape");
  TORCH_CHECK(k_cache.dim() == 3 && k_cache.size(0) == n_kv_heads && k_cache.size(2) == 128 &&
                  k_cache.is_contiguous() && v_cache.sizes() == k_cache.sizes() && v_cache.is_contiguous(),
              "k_cache / v_cache [n_kv_heads, cap, 128]");
  CHECK_I32(rope_pos); CHECK_I32(cache_slot); CHECK_F32(rope_table);
  TORCH_CHECK(rope_pos.numel() >= x.size(0) && cache_slot.numel() >= x.size(0), "positions");
  Tensor ws = wide_partials(a, x);
  sc::SkinnyArgs r{};
  r.M = a.M;
  r.N = a.N;
  r.K = a.K;
  r.epi = sc::SKINNY_QKV;
  r.ws = a.ws;
  r.splits = a.splits;
  r.num_sms = a.num_sms;
  r.status = a.status;
  r.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  r.ldq = (int)q_out.stride(0);
  r.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  r.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  r.cache_cap = (int)k_cache.size(1);
  r.pos_rows = rope_pos.data_ptr<int>();
  r.slot_rows = cache_slot.data_ptr<int>();
  r.rope_table = reinterpret_cast<const float2*>(rope_table.data_ptr<float>());
  r.n_q_heads = (int)n_q_heads;
  r.n_kv_heads = (int)n_kv_heads;
  check_cuda(sc::skinny_reduce(r, cur_stream()), "wide_qkv reduce");
  return 2;
}

py::dict wide_plan(int64_t M, int64_t N, int64_t K, int64_t epi, int64_t acc, int64_t n_tt, int64_t splits,
                   int64_t sms) {
  sc::WidePlan p{};
  py::dict d;
  if (!sc::wide_plan((int)M, (int)N, (int)K, (int)epi, sms > 0 ? (int)sms : num_sms(), (int)acc, (int)n_tt,
                     (int)splits, g_wide_stream_k, &p))
    return d;
  d["acc"] = p.acc; d["bn"] = p.bn; d["n_tt"] = p.n_tt; d["splits"] = p.splits; d["stages"] = p.stages;
  d["nbuf"] = p.nbuf; d["tmem_cols"] = p.tmem_cols; d["smem"] = p.smem; d["grid"] = p.grid;
  d["sk_tail"] = p.sk_tail; d["sk_ctas"] = p.sk_ctas; d["sk_max_pieces"] = p.sk_max_pieces;
  return d;
}

// experiment switch: stream-K tail of the token-column GEMM on / off
void set_wide_stream_k(bool on) { g_wide_stream_k = on; }

void row_argmax(Tensor logits, Tensor out_token) {
  const c10::cuda::CUDAGuard guard(logits.device());
  check_matrix(logits, "logits");
  CHECK_I32(out_token);
  TORCH_CHECK(out_token.numel() >= logits.size(0), "out_token [M]");
  check_cuda(sc::row_argmax_bf16(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), (int)logits.stride(0),
                                 (int)logits.size(0), (int)logits.size(1), out_token.data_ptr<int>(), cur_stream()),
             "row_argmax");
}

int64_t skinny_splits(int64_t N, int64_t K) { return sc::skinny_splits((int)N, (int)K, num_sms()); }

sc::LseGatherArgs lse_args(const Tensor& logits, const Tensor& ids, const Tensor& lse) {
  check_matrix(logits, "logits");
  CHECK_I32(ids); CHECK_F32(lse);
  TORCH_CHECK(ids.dim() == 2 && ids.size(0) == logits.size(0) && ids.is_contiguous(), "ids [R, G]");
  TORCH_CHECK(lse.numel() == logits.size(0) && lse.is_contiguous(), "lse [R]");
  TORCH_CHECK(logits.size(1) % 8 == 0, "vocabulary must be a multiple of 8");
  sc::LseGatherArgs a{};
  a.logits = reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr());
  a.ld = (int)logits.stride(0);
  a.R = (int)logits.size(0);
  a.V = (int)logits.size(1);
  a.ids = ids.data_ptr<int>();
  a.G = (int)ids.size(1);
  a.lse = lse.data_ptr<float>();
  return a;
}

void lse_gather(Tensor logits, Tensor ids, Tensor lse, Tensor z) {
  const c10::cuda::CUDAGuard guard(logits.device());
  auto a = lse_args(logits, ids, lse);
  CHECK_F32(z);
  TORCH_CHECK(z.sizes() == ids.sizes() && z.is_contiguous(), "z [R, G]");
  a.z = z.data_ptr<float>();
  check_cuda(sc::lse_gather(a, cur_stream()), "lse_gather");
}

void lse_gather_backward(Tensor logits, Tensor ids, Tensor lse, c10::optional<Tensor> g_lse,
                         c10::optional<Tensor> g_z, Tensor dlogits) {
  const c10::cuda::CUDAGuard guard(logits.device());
  auto a = lse_args(logits, ids, lse);
  check_matrix(dlogits, "dlogits");
  TORCH_CHECK(dlogits.sizes() == logits.sizes(), "dlogits shape");
  if (g_lse.has_value() && g_lse->defined()) {
    CHECK_F32(*g_lse);
    TORCH_CHECK(g_lse->numel() == a.R && g_lse->is_contiguous(), "g_lse [R]");
    a.g_lse = g_lse->data_ptr<float>();
  }
  if (g_z.has_value() && g_z->defined()) {
    CHECK_F32(*g_z);
    TORCH_CHECK(g_z->sizes() == ids.sizes() && g_z->is_contiguous(), "g_z [R, G]");
    a.g_z = g_z->data_ptr<float>();
  }
  a.dlogits = reinterpret_cast<__nv_bfloat16*>(dlogits.data_ptr());
  a.ldd = (int)dlogits.stride(0);
  check_cuda(sc::lse_gather_backward(a, cur_stream()), "lse_gather_backward");
}

void arange_i32(Tensor out, int64_t start) {
  const c10::cuda::CUDAGuard guard(out.device());
  CHECK_I32(out);
  check_cuda(sc::fill_arange_i32(out.data_ptr<int>(), (int)out.numel(), (int)start, cur_stream()),
             "arange");
}

void index_i32(Tensor src, Tensor idx, Tensor out) {
  const c10::cuda::CUDAGuard guard(out.device());
  CHECK_I32(src); CHECK_I32(idx); CHECK_I32(out);
  check_cuda(sc::index_i32(src.data_ptr<int>(), idx.data_ptr<int>(), out.data_ptr<int>(),
                           (int)out.numel(), cur_stream()),
             "index_i32");
}

Tensor status(Tensor like) { return status_tensor(like); }

// ------------------------------------------------------- K13 memory attention
sc::MemAttnArgs mem_args(const Tensor& q, const Tensor& k, const Tensor& v, int64_t layer_stride,
                         int64_t seq_stride, int64_t tok_stride, int64_t head_stride,
                         const c10::optional<Tensor>& row_seq, const c10::optional<Tensor>& idx,
                         int64_t idx_stride, const c10::optional<Tensor>& n_vis, int64_t n_fixed, double scale) {
  CHECK_CUDA(q); CHECK_BF16(q); CHECK_CUDA(k); CHECK_BF16(k); CHECK_CUDA(v); CHECK_BF16(v);
  TORCH_CHECK(q.dim() == 4 && q.size(3) == 128 && q.is_contiguous(), "q must be contiguous [L, R, H, 128]");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(), "memory on another device");
  TORCH_CHECK(tok_stride % 8 == 0 && head_stride % 8 == 0 && seq_stride % 8 == 0 && layer_stride % 8 == 0,
              "memory strides must be multiples of 8 elements (16-byte rows)");
  CHECK_ALIGN16(k); CHECK_ALIGN16(v);
  sc::MemAttnArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.layer_stride = layer_stride; a.seq_stride = seq_stride; a.tok_stride = tok_stride; a.head_stride = head_stride;
  a.L = (int)q.size(0); a.R = (int)q.size(1); a.H = (int)q.size(2);
  if (row_seq.has_value() && row_seq->defined()) {
    CHECK_I32(*row_seq);
    TORCH_CHECK(row_seq->numel() >= a.R, "row_seq too short");
    a.row_seq = row_seq->data_ptr<int>();
  }
  if (idx.has_value() && idx->defined()) { CHECK_I32(*idx); a.idx = idx->data_ptr<int>(); a.idx_stride = idx_stride; }
  if (n_vis.has_value() && n_vis->defined()) { CHECK_I32(*n_vis); a.n_vis = n_vis->data_ptr<int>(); }
  a.n_fixed = (int)n_fixed;
  a.scale = (float)scale;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  return a;
}

void mem_attn_fwd(Tensor q, Tensor k, Tensor v, int64_t layer_stride, int64_t seq_stride, int64_t tok_stride,
                  int64_t head_stride, c10::optional<Tensor> row_seq, c10::optional<Tensor> idx, int64_t idx_stride,
                  c10::optional<Tensor> n_vis, int64_t n_fixed, double scale, Tensor out, Tensor lse) {
  const c10::cuda::CUDAGuard guard(q.device());
  auto a = mem_args(q, k, v, layer_stride, seq_stride, tok_stride, head_stride, row_seq, idx, idx_stride, n_vis,
                    n_fixed, scale);
  CHECK_BF16(out); CHECK_F32(lse);
  TORCH_CHECK(out.sizes() == q.sizes() && out.is_contiguous(), "out shape");
  TORCH_CHECK(lse.numel() == (int64_t)a.L * a.R * a.H && lse.is_contiguous(), "lse shape");
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  check_cuda(sc::mem_attn_fwd(a, cur_stream()), "mem_attn_fwd");
}

void mem_attn_bwd(Tensor q, Tensor k, Tensor v, int64_t layer_stride, int64_t seq_stride, int64_t tok_stride,
                  int64_t head_stride, c10::optional<Tensor> row_seq, c10::optional<Tensor> idx, int64_t idx_stride,
                  c10::optional<Tensor> n_vis, int64_t n_fixed, double scale, Tensor o, Tensor dout, Tensor lse,
                  Tensor dq) {
  const c10::cuda::CUDAGuard guard(q.device());
  auto a = mem_args(q, k, v, layer_stride, seq_stride, tok_stride, head_stride, row_seq, idx, idx_stride, n_vis,
                    n_fixed, scale);
  CHECK_BF16(o); CHECK_BF16(dout); CHECK_F32(lse); CHECK_F32(dq);
  TORCH_CHECK(o.sizes() == q.sizes() && o.is_contiguous() && dout.sizes() == q.sizes() && dout.is_contiguous(),
              "o/dout shape");
  TORCH_CHECK(dq.sizes() == q.sizes() && dq.is_contiguous(), "dq shape");
  a.o = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.dq = dq.data_ptr<float>();
  check_cuda(sc::mem_attn_bwd(a, cur_stream()), "mem_attn_bwd");
}

// ------------------------------------------------------------- K16 AdamW / DP
void adamw_step(Tensor param, Tensor grad, Tensor exp_avg, Tensor exp_avg_sq, Tensor hyper, Tensor state,
                Tensor partial, Tensor counter) {
  const c10::cuda::CUDAGuard guard(param.device());
  for (const Tensor* t : {&param, &grad, &exp_avg, &exp_avg_sq, &hyper, &state, &partial}) {
    CHECK_CUDA(*t); CHECK_F32(*t);
    TORCH_CHECK(t->is_contiguous(), "optimizer buffers must be contiguous");
  }
  TORCH_CHECK(grad.numel() == param.numel() && exp_avg.numel() == param.numel() &&
              exp_avg_sq.numel() == param.numel(), "flat buffer sizes differ");
  TORCH_CHECK(hyper.numel() >= 6 && state.numel() >= 5, "hyper[6] / state[5]");
  TORCH_CHECK(counter.scalar_type() == torch::kInt32 && counter.numel() >= 1, "counter int32");
  sc::AdamArgs a{};
  a.param = param.data_ptr<float>();
  a.grad = grad.data_ptr<float>();
  a.exp_avg = exp_avg.data_ptr<float>();
  a.exp_avg_sq = exp_avg_sq.data_ptr<float>();
  a.n = param.numel();
  a.hyper = hyper.data_ptr<float>();
  a.state = state.data_ptr<float>();
  a.partial = partial.data_ptr<float>();
  a.counter = reinterpret_cast<unsigned*>(counter.data_ptr<int>());
  check_cuda(sc::adamw_norm(a, (int)partial.numel(), cur_stream()), "adamw_norm");
  check_cuda(sc::adamw_update(a, cur_stream()), "adamw_update");
}

void dp_adamw_step(int64_t world, int64_t rank, int64_t n_total, int64_t shard, std::vector<int64_t> grads,
                   std::vector<int64_t> params, std::vector<int64_t> norms, Tensor flag_grads, Tensor flag_norms,
                   std::vector<int64_t> peer_flag_norms, std::vector<int64_t> peer_flag_params, Tensor epoch,
                   int64_t timeout_ns, Tensor status, Tensor red_grad, Tensor exp_avg, Tensor exp_avg_sq,
                   Tensor hyper, Tensor state, Tensor partial, Tensor counter, bool pre_reduced) {
  const c10::cuda::CUDAGuard guard(red_grad.device());
  TORCH_CHECK(world >= 1 && world <= sc::kMaxShards && rank >= 0 && rank < world, "world/rank");
  TORCH_CHECK((int64_t)grads.size() == world && (int64_t)params.size() == world && (int64_t)norms.size() == world &&
              (int64_t)peer_flag_norms.size() == world && (int64_t)peer_flag_params.size() == world,
              "one pointer per rank");
  TORCH_CHECK(shard * world >= n_total, "shards do not cover the buffer");
  for (const Tensor* t : {&red_grad, &exp_avg, &exp_avg_sq, &hyper, &state, &partial}) {
    CHECK_CUDA(*t); CHECK_F32(*t);
  }
  TORCH_CHECK(red_grad.numel() >= shard && exp_avg.numel() >= shard && exp_avg_sq.numel() >= shard, "shard buffers");
  TORCH_CHECK(hyper.numel() >= 7 && state.numel() >= 5, "hyper[7] / state[5]");
  CHECK_I32(flag_grads); CHECK_I32(flag_norms); CHECK_I32(epoch); CHECK_I32(status); CHECK_I32(counter);
  sc::DpArgs a{};
  a.world = (int)world; a.rank = (int)rank; a.n_total = n_total; a.shard = shard;
  for (int s = 0; s < world; ++s) {
    a.grads[s] = reinterpret_cast<const float*>(grads[s]);
    a.params[s] = reinterpret_cast<float*>(params[s]);
    a.norms[s] = reinterpret_cast<float*>(norms[s]);
    a.peer_flag_norms[s] = reinterpret_cast<int*>(peer_flag_norms[s]);
    a.peer_flag_params[s] = reinterpret_cast<int*>(peer_flag_params[s]);
  }
  a.flag_grads = flag_grads.data_ptr<int>();
  a.flag_norms = flag_norms.data_ptr<int>();
  a.epoch_ptr = epoch.data_ptr<int>();
  a.timeout_ns = timeout_ns;
  a.status = status.data_ptr<int>();
  a.red_grad = red_grad.data_ptr<float>();
  a.exp_avg = exp_avg.data_ptr<float>();
  a.exp_avg_sq = exp_avg_sq.data_ptr<float>();
  a.hyper = hyper.data_ptr<float>();
  a.state = state.data_ptr<float>();
  a.partial = partial.data_ptr<float>();
  a.counter = reinterpret_cast<unsigned*>(counter.data_ptr<int>());
  a.pre_reduced = pre_reduced ? 1 : 0;
  const int grid = (int)partial.numel();
  check_cuda(sc::dp_reduce_norm(a, grid, cur_stream()), "dp_reduce_norm");
  check_cuda(sc::dp_adamw_gather(a, grid, cur_stream()), "dp_adamw_gather");
}

// One bucket of the data-parallel reduce-scatter (flat range [lo, hi)):
// bounded wait on flags[0..world) (one per sender) for the current epoch,
// then this rank's shard of the range, summed over every rank's gradient in
// rank order, into red_grad.  grid CTAs (a few: it shares the GPU with the
// backward's GEMMs).
void dp_reduce_range(int64_t world, int64_t rank, int64_t n_total, int64_t shard, std::vector<int64_t> grads,
                     Tensor flags, Tensor epoch, int64_t lo, int64_t hi, int64_t timeout_ns, Tensor status,
                     Tensor red_grad, int64_t grid) {
  const c10::cuda::CUDAGuard guard(red_grad.device());
  TORCH_CHECK(world >= 1 && world <= sc::kMaxShards && rank >= 0 && rank < world, "world/rank");
  TORCH_CHECK((int64_t)grads.size() == world, "one gradient pointer per rank");
  TORCH_CHECK(shard * world >= n_total, "shards do not cover the buffer");
  TORCH_CHECK(lo >= 0 && lo <= hi && hi <= n_total, "bucket range");
  TORCH_CHECK(grid >= 1 && grid <= 1024, "grid");
  CHECK_CUDA(red_grad); CHECK_F32(red_grad);
  TORCH_CHECK(red_grad.numel() >= shard, "red_grad holds a shard");
  CHECK_I32(flags); CHECK_I32(epoch); CHECK_I32(status);
  TORCH_CHECK(flags.numel() >= world, "one flag per rank");
  sc::DpArgs a{};
  a.world = (int)world; a.rank = (int)rank; a.n_total = n_total; a.shard = shard;
  for (int s = 0; s < world; ++s) a.grads[s] = reinterpret_cast<const float*>(grads[s]);
  a.epoch_ptr = epoch.data_ptr<int>();
  a.timeout_ns = timeout_ns;
  a.status = status.data_ptr<int>();
  a.red_grad = red_grad.data_ptr<float>();
  check_cuda(sc::dp_reduce_range(a, flags.data_ptr<int>(), lo, hi, (int)grid, cur_stream()), "dp_reduce_range");
}

// out (fp32, [M, N], contiguous) = a @ w^T on the tensor cores with no
// epilogue: the weight gradient of a linear layer over a whole batch of
// positions (a = dY^T [out, rows], w = X^T [in, rows]; K = rows).
void gemm_f32(Tensor a, Tensor w, Tensor out) {
  const c10::cuda::CUDAGuard guard(a.device());
  auto g = base_gemm(a, w, sc::EPI_PARTIAL, 256);
  CHECK_CUDA(out); CHECK_F32(out);
  TORCH_CHECK(out.is_contiguous() && out.dim() == 2 && out.size(0) == a.size(0) && out.size(1) == w.size(0),
              "out must be a contiguous [M, N] fp32 matrix");
  CHECK_ALIGN16(out);
  TORCH_CHECK(g.N % 32 == 0, "N must be a multiple of 32");
  g.splits = 1;
  g.ep.ws = out.data_ptr<float>();
  g.rows_per_tile = 128;  // one accumulator per tile: the partial epilogue's tested layout
  run_gemm(g);
}

void bump_counter(Tensor counter) {
  const c10::cuda::CUDAGuard guard(counter.device());
  CHECK_I32(counter);
  check_cuda(sc::bump_counter(counter.data_ptr<int>(), cur_stream()), "bump_counter");
}

void signal_epoch(std::vector<int64_t> flag_ptrs, Tensor epoch, int64_t offset) {
  const c10::cuda::CUDAGuard guard(epoch.device());
  CHECK_I32(epoch);
  TORCH_CHECK(!flag_ptrs.empty() && flag_ptrs.size() <= (size_t)sc::kMaxShards, "1..8 flags");
  sc::FlagPtrs f{};
  for (size_t i = 0; i < flag_ptrs.size(); ++i) f.addr[i] = reinterpret_cast<int*>(flag_ptrs[i]);
  f.n = (int)flag_ptrs.size();
  check_cuda(sc::signal_epoch(f, epoch.data_ptr<int>(), (int)offset, cur_stream()), "signal_epoch");
}

void wait_all(Tensor flags, int64_t n, Tensor epoch, int64_t offset, int64_t timeout_ns, Tensor status) {
  const c10::cuda::CUDAGuard guard(flags.device());
  CHECK_I32(flags); CHECK_I32(epoch); CHECK_I32(status);
  TORCH_CHECK(n >= 1 && n <= sc::kMaxShards && flags.numel() >= n, "1..8 flags");
  check_cuda(sc::wait_all(flags.data_ptr<int>(), (int)n, epoch.data_ptr<int>(), (int)offset, timeout_ns,
                          status.data_ptr<int>(), cur_stream()),
             "wait_all");
}


}  // namespace

namespace sc {
void register_disk_loader(py::module& m);
void register_host_pack(py::module& m);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  sc::register_disk_loader(m);
  sc::register_host_pack(m);
  m.doc() = "sm_100a kernels of sparsecache_b200";
  m.def("gemm_store", &gemm_store, py::arg("a"), py::arg("w"), py::arg("out"), py::arg("bn"),
        py::arg("splits") = -1);
  m.def("gemm_residual", &gemm_residual, py::arg("a"), py::arg("w"), py::arg("out"), py::arg("residual"),
        py::arg("bn"), py::arg("splits") = -1, py::arg("norm_w") = py::none(), py::arg("eps") = 1e-5,
        py::arg("norm_out") = py::none());
  m.def("gemm_swiglu", &gemm_swiglu);
  m.def("gemm_qkv", &gemm_qkv, py::arg("a"), py::arg("w_qkv"), py::arg("q_out"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("rope_pos"), py::arg("cache_slot"), py::arg("rope_table"),
        py::arg("n_q_heads"), py::arg("n_kv_heads"), py::arg("dev_part"), py::arg("dev_mode"), py::arg("bn"),
        py::arg("k_peer") = 0, py::arg("v_peer") = 0);
  m.def("peer_signal_many", [](std::vector<int64_t> addrs, int64_t value) {
    std::vector<int*> p;
    for (auto a : addrs) p.push_back(reinterpret_cast<int*>(a));
    check_cuda(sc::peer_signal_many(p.data(), (int)p.size(), (int)value, cur_stream()), "peer_signal_many");
  });
  m.def("memcpy_async", [](int64_t dst, int64_t src, int64_t nbytes) {
    // copy-engine transfer on the current stream (peer addresses included: UVA)
    check_cuda(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), (size_t)nbytes,
                               cudaMemcpyDefault, cur_stream()),
               "memcpy_async");
  });
  m.def("gemm_ag_qkv", &gemm_ag_qkv, py::arg("shard_ptrs"), py::arg("rows"), py::arg("own"), py::arg("ready"),
        py::arg("epoch"), py::arg("K"), py::arg("w_qkv"), py::arg("q_out"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("rope_pos"), py::arg("cache_slot"), py::arg("rope_table"), py::arg("n_q_heads"),
        py::arg("n_kv_heads"), py::arg("bn"), py::arg("dev_part") = py::none(), py::arg("dev_mode") = 0,
        py::arg("k_peer") = 0, py::arg("v_peer") = 0);
  m.def("gemm_ag_swiglu", &gemm_ag_swiglu);
  m.def("set_gemm_rows_per_tile", &set_gemm_rows_per_tile);
  m.def("gemm_cost_estimate", [](int64_t M, int64_t N, int64_t K, int64_t bn, int64_t rows, int64_t splits,
                                 int64_t sms) {
    return sc::gemm_cost_estimate((int)M, (int)N, (int)K, (int)bn, (int)rows, (int)splits,
                                  sms > 0 ? (int)sms : num_sms());
  }, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("bn"), py::arg("rows"), py::arg("splits"),
     py::arg("sms") = 0);
  m.def("gemm_rs", &gemm_rs);
  m.def("rs_reduce", &rs_reduce, py::arg("recv"), py::arg("flags"), py::arg("epoch"), py::arg("timeout_ns"),
        py::arg("status"), py::arg("residual"), py::arg("out"), py::arg("norm_w"), py::arg("norm_out"),
        py::arg("eps"), py::arg("epoch_ptr") = py::none(), py::arg("epoch_mul") = 0);
  m.def("gemv_allreduce", &gemv_allreduce, py::arg("x"), py::arg("w"), py::arg("norm_w"), py::arg("eps"),
        py::arg("dst_ptrs"), py::arg("flag_ptrs"), py::arg("sender"), py::arg("epoch"), py::arg("epoch_ptr"),
        py::arg("epoch_mul"), py::arg("counter"), py::arg("recv") = py::none(), py::arg("wait_flags") = py::none(),
        py::arg("residual") = py::none(), py::arg("timeout_ns") = 20000000000LL, py::arg("status") = py::none());
  m.def("shared_empty", &shared_empty);
  m.def("shared_open", &shared_open);
  m.def("shared_close", &shared_close);
  m.def("peer_signal", &peer_signal, py::arg("flag_ptr"), py::arg("value"), py::arg("stamp") = py::none(),
        py::arg("value_src") = py::none());
  m.def("wait_flag", &wait_flag, py::arg("flags"), py::arg("index"), py::arg("target"), py::arg("timeout_ns"),
        py::arg("status"), py::arg("stamp") = py::none());
  m.def("gemv_store", &gemv_store);
  m.def("gemv_residual", &gemv_residual);
  m.def("gemv_swiglu", &gemv_swiglu);
  m.def("gemv_qkv", &gemv_qkv, py::arg("x"), py::arg("w_qkv"), py::arg("norm_w"), py::arg("eps"),
        py::arg("q_out"), py::arg("k_cache"), py::arg("v_cache"), py::arg("pos"), py::arg("rope_table"),
        py::arg("n_q_heads"), py::arg("n_kv_heads"), py::arg("slot") = py::none());
  m.def("gemv_argmax", &gemv_argmax, py::arg("x"), py::arg("w"), py::arg("norm_w"), py::arg("eps"),
        py::arg("part_val"), py::arg("part_idx"), py::arg("counter"), py::arg("out_token"),
        py::arg("token_log"), py::arg("gen_count"), py::arg("embed"), py::arg("next_hidden"),
        py::arg("pos_advance"), py::arg("n_advance") = 1);
  m.def("gemv_argmax_grid", &gemv_argmax_grid);
  m.def("attention_prefill", &attention_prefill, py::arg("q"), py::arg("q_rows"), py::arg("qpos"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("kpos"), py::arg("n_keys"), py::arg("n_heads"),
        py::arg("scale"), py::arg("out"), py::arg("trace") = py::none(), py::arg("ws") = py::none());
  m.def("attention_prefill_splits", [](int64_t n_rows, int64_t n_heads, int64_t n_kv_heads, int64_t n_keys,
                                       int64_t ws_floats, int64_t num_sms) {
    sc::AttnPrefillArgs p{};
    p.n_rows = (int)n_rows;
    p.n_heads = (int)n_heads;
    p.n_kv_heads = (int)n_kv_heads;
    p.n_keys = (int)n_keys;
    p.ws = ws_floats > 0 ? reinterpret_cast<float*>(16) : nullptr;  // only tested for null
    p.ws_floats = ws_floats;
    return sc::attention_prefill_splits(p, (int)num_sms);
  });
  m.def("attention_prefill_mma", &attention_prefill_mma);
  m.def("recurrent_attention_fwd", &recurrent_attention_fwd);
  m.def("recurrent_attention_bwd", &recurrent_attention_bwd);
  m.def("page_token_scores", &page_token_scores, py::arg("q"), py::arg("keys"), py::arg("n_tokens"),
        py::arg("scale"));
  m.def("attention_decode", &attention_decode, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("pos"), py::arg("n_heads"), py::arg("scale"), py::arg("splits"), py::arg("out"),
        py::arg("page_table") = py::none(), py::arg("page_shift") = 6, py::arg("n_virtual") = py::none(),
        py::arg("ws") = py::none(), py::arg("counters") = py::none(), py::arg("outer") = 0,
        py::arg("pos_rows") = py::none(), py::arg("seq_stride") = 0,
        py::arg("l2_prefetch") = std::vector<Tensor>{}, py::arg("l2_prefetch_bytes") = 0,
        py::arg("key_capacity") = 0);
  m.def("attention_decode_outer", [](int64_t cap, int64_t kvh, int64_t cluster, int64_t sms) {
    return sc::attention_decode_outer((int)cap, (int)kvh, (int)cluster, (int)sms);
  });
  m.def("attention_decode_cluster", [](int64_t cap, int64_t n_kv_heads) {
    return sc::attention_decode_cluster((int)cap, (int)n_kv_heads);
  }, py::arg("cache_cap"), py::arg("n_kv_heads") = 8);
  m.def("rmsnorm", &rmsnorm);
  m.def("embedding", &embedding);
  m.def("gather_rows", &gather_rows);
  m.def("compose_relocate", &compose_relocate);
  m.def("cacheblend_select", &cacheblend_select, py::arg("dev_part"), py::arg("n_kv_heads"), py::arg("dev_mode"),
        py::arg("total_rows"), py::arg("doc_begin"), py::arg("doc_end"), py::arg("k"), py::arg("keep_prefix"),
        py::arg("active"), py::arg("n_active"), py::arg("scores"), py::arg("checksum") = py::none(),
        py::arg("n_parts") = 1, py::arg("part_stride") = 0);
  m.def("arange_i32", &arange_i32);
  m.def("lse_gather", &lse_gather);
  m.def("skinny_gemm", &skinny_gemm, py::arg("x"), py::arg("w"), py::arg("epi"), py::arg("out"),
        py::arg("residual") = py::none(), py::arg("ws"), py::arg("splits") = -1);
  m.def("skinny_splits", &skinny_splits);
  m.def("wide_swiglu", &wide_swiglu, py::arg("x"), py::arg("w_gu"), py::arg("out"));
  m.def("wide_residual", &wide_residual, py::arg("x"), py::arg("w"), py::arg("out"), py::arg("residual") = py::none(),
        py::arg("norm_w") = py::none(), py::arg("eps") = 1e-5, py::arg("norm_out") = py::none(), py::arg("acc") = 0,
        py::arg("n_tt") = 0, py::arg("splits") = 0);
  m.def("wide_qkv", &wide_qkv, py::arg("x"), py::arg("w_qkv"), py::arg("q_out"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("rope_pos"), py::arg("cache_slot"), py::arg("rope_table"), py::arg("n_q_heads"),
        py::arg("n_kv_heads"), py::arg("acc") = 0, py::arg("n_tt") = 0, py::arg("splits") = 0);
  m.def("set_wide_stream_k", &set_wide_stream_k);
  m.def("set_attention_prefill_splits", [](int64_t s) { sc::set_attention_prefill_splits((int)s); });
  m.def("wide_plan", &wide_plan, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("epi"), py::arg("acc") = 0,
        py::arg("n_tt") = 0, py::arg("splits") = 0, py::arg("sms") = 0);
  m.def("skinny_qkv", &skinny_qkv, py::arg("x"), py::arg("w_qkv"), py::arg("q_out"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("pos"), py::arg("rope_table"), py::arg("n_q_heads"), py::arg("n_kv_heads"),
        py::arg("ws"), py::arg("slot") = py::none(), py::arg("pos_rows") = py::none(), py::arg("seq_stride") = 0);
  m.def("skinny_allreduce", &skinny_allreduce);
  m.def("row_argmax", &row_argmax);
  m.def("lse_gather_backward", &lse_gather_backward, py::arg("logits"), py::arg("ids"), py::arg("lse"),
        py::arg("g_lse"), py::arg("g_z"), py::arg("dlogits"));
  m.def("index_i32", &index_i32);
  m.def("status", &status);
  m.def("num_sms", &num_sms);
  m.def("mem_attn_fwd", &mem_attn_fwd);
  m.def("mem_attn_bwd", &mem_attn_bwd);
  m.def("adamw_step", &adamw_step);
  m.def("dp_adamw_step", &dp_adamw_step, py::arg("world"), py::arg("rank"), py::arg("n_total"), py::arg("shard"),
        py::arg("grads"), py::arg("params"), py::arg("norms"), py::arg("flag_grads"), py::arg("flag_norms"),
        py::arg("peer_flag_norms"), py::arg("peer_flag_params"), py::arg("epoch"), py::arg("timeout_ns"),
        py::arg("status"), py::arg("red_grad"), py::arg("exp_avg"), py::arg("exp_avg_sq"), py::arg("hyper"),
        py::arg("state"), py::arg("partial"), py::arg("counter"), py::arg("pre_reduced") = false);
  m.def("dp_reduce_range", &dp_reduce_range);
  m.def("gemm_f32", &gemm_f32, py::arg("a"), py::arg("w"), py::arg("out"));
  m.def("bump_counter", &bump_counter);
  m.def("signal_epoch", &signal_epoch);
  m.def("wait_all", &wait_all);
}
