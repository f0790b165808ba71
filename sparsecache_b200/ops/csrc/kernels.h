// Host-visible argument structs and launchers of the sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sc {

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                       bool swizzle128);
// 3-D [outer][mid][inner] bf16 view, 128-byte swizzle, box {box_inner, box_mid, 1};
// coordinates past mid / outer load as zeros
bool make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t mid, uint64_t outer,
                       uint64_t mid_stride_elems, uint64_t outer_stride_elems, uint32_t box_inner,
                       uint32_t box_mid);

// ---------------------------------------------------------------- GEMM ----
enum Epi : int { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_QKV = 3, EPI_RS = 4, EPI_PARTIAL = 5 };
constexpr int kMaxShards = 8;
enum DevMode : int { DEV_KEY = 1, DEV_VALUE = 2, DEV_L1 = 4 };

struct GemmEpilogue {
  __nv_bfloat16* out;  // EPI_STORE / RESIDUAL / SWIGLU
  int ldo;
  const __nv_bfloat16* residual;  // EPI_RESIDUAL (may alias out)
  int ldr;
  // EPI_QKV
  __nv_bfloat16* q_out;
  int ldq;
  __nv_bfloat16* k_cache;  // [n_kv_heads, cache_cap, 128]
  __nv_bfloat16* v_cache;
  int cache_cap;
  const int* rope_pos;      // [M]
  const int* cache_slot;    // [M]
  const float2* rope_table; // [max_pos, 64] (cos, sin)
  int n_q_heads;
  int n_kv_heads;
  float* dev_part;  // [M, 2 * n_kv_heads] or null
  int dev_mode;
  // optional peer copies of this layer's cache (same layout and capacity):
  // every K/V row written locally is also stored into the peer GPU's slot
  __nv_bfloat16* k_peer;
  __nv_bfloat16* v_peer;
  // EPI_RS (GEMM -> reduce-scatter): rows [r * rs_rows, (r + 1) * rs_rows)
  // belong to rank r; their bf16 partial tile is stored into rank r's receive
  // buffer (local or peer-mapped) at slot rs_sender: rs_dst[r][rs_sender][row][N]
  void* rs_dst[kMaxShards];
  int rs_rows;
  int rs_sender;
  // EPI_PARTIAL (split-K): fp32 partial of K-slice ks at ws[ks][row][col]
  float* ws;
};

// A operand split by rows over ranks (all-gather fused into the GEMM): shard
// r holds rows [r * rows, (r + 1) * rows) in its own buffer (peer-mapped for
// r != own); its TMA map is maps[r].  Before a peer shard is first read the
// producer waits (bounded) until ready[r] >= epoch.
struct AShards {
  int n;       // 1 = ordinary GEMM (maps[0] covers all of A)
  int rows;    // rows per shard, a multiple of 128
  int own;
  const int* ready;
  int epoch;
};

struct GemmArgs {
  const __nv_bfloat16* a;  // [M, K], row stride lda (shard 0 when sharded)
  const __nv_bfloat16* a_shards[kMaxShards];  // per-rank shard bases when shards.n > 1
  AShards shards;
  const __nv_bfloat16* b;  // [N, K], row stride ldb
  int M, N, K, lda, ldb;
  int epi;
  int bn;  // 128 or 256
  int rows_per_tile;  // 128 (one accumulator) or 256 (two; bn 256, unsharded, not EPI_RS); 0 = 128
  int splits;  // EPI_PARTIAL: number of K slices (>= 1)
  int num_sms;
  GemmEpilogue ep;
  int* status;
};

cudaError_t gemm_bf16_tc(const GemmArgs& g, cudaStream_t stream);
// relative device-cycle estimate of a tile shape (used to pick rows_per_tile and split-K)
double gemm_cost_estimate(int M, int N, int K, int bn, int rows_per_tile, int splits, int num_sms);
cudaError_t splitk_reduce(const float* ws, int splits, int M, int N, const __nv_bfloat16* residual, int ldr,
                          __nv_bfloat16* out, int ldo, cudaStream_t stream);
// the same with the RESIDUAL epilogue and the RMSNorm of every finished row
// (bit-identical to rmsnorm_bf16 on the stored rows); N % 8 == 0, N <= 8192
cudaError_t splitk_reduce_norm(const float* ws, int splits, int M, int N, const __nv_bfloat16* residual, int ldr,
                               __nv_bfloat16* out, int ldo, const __nv_bfloat16* norm_w, float eps,
                               __nv_bfloat16* norm_out, int ldn, cudaStream_t stream);

// ---------------------------------------------------------------- GEMV ----
// Small-M (1..8 rows) weight-streaming kernel for decode / verify.
enum GemvEpi : int {
  GEMV_STORE = 0,
  GEMV_RESIDUAL = 1,
  GEMV_SWIGLU = 2,
  GEMV_QKV = 3,
  GEMV_ARGMAX = 4,
  GEMV_ALLREDUCE = 5
};

struct GemvArgs {
  const __nv_bfloat16* w;  // [N, K]
  const __nv_bfloat16* x;  // [M, K] (row stride ldx)
  int ldx;
  int M, N, K;
  const __nv_bfloat16* norm_w;  // optional fused RMSNorm of x (weight [K])
  float eps;
  int epi;
  __nv_bfloat16* out;  // STORE/RESIDUAL/SWIGLU: [M, ldo]
  int ldo;
  const __nv_bfloat16* residual;
  int ldr;
  // QKV
  __nv_bfloat16* q_out;  // [M, n_q_heads*128]
  int ldq;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int cache_cap;
  const int* pos;  // device scalar: position of row 0 (row m at pos + m)
  const int* slot; // optional device scalar: cache slot of row 0 (default: *pos)
  const float2* rope_table;
  int n_q_heads, n_kv_heads;
  // ARGMAX (LM head)
  float* part_val;     // [M, gridDim]
  int* part_idx;       // [M, gridDim]
  unsigned int* counter;  // one word, zero on entry, restored to zero
  int* out_token;      // [M] argmax per row
  int* token_log;      // optional: token_log[*gen_count] = token of row M-1
  int* gen_count;      // device scalar advanced by one per call when token_log is set
  const __nv_bfloat16* embed;  // optional: writes embed[token] of the last row to next_hidden
  __nv_bfloat16* next_hidden;
  int* pos_advance;    // optional device scalars [n_advance] each incremented by M at the end
  int n_advance;       // number of scalars at pos_advance (0 means 1)
  // ALLREDUCE (row-parallel decode projection under tensor parallelism): the
  // fp32 partial of every row goes to every rank's receive buffer
  // ar_dst[r][ar_sender][m][N] (NVLink stores); the last CTA then releases
  // ar_flag[r] = ar_epoch on every rank (fence.sys + st.release.sys).
  float* ar_dst[8];
  int* ar_flag[8];
  int ar_tp;
  int ar_sender;
  int ar_epoch;          // epoch = ar_epoch_ptr ? *ar_epoch_ptr * ar_epoch_mul + ar_epoch : ar_epoch
  const int* ar_epoch_ptr;
  int ar_epoch_mul;
  // optional fused reduction by the last CTA (null ar_recv: a separate reduce
  // kernel follows): wait until ar_wait_flags[0..tp) reach the epoch, then
  // ar_out[m] = ar_residual[m] + bf16(sum_r ar_recv[r][m][N]) in rank order
  const float* ar_recv;
  const int* ar_wait_flags;
  const __nv_bfloat16* ar_residual;
  __nv_bfloat16* ar_out;
  long long ar_timeout_ns;
  int* status;
  int num_sms;
};

cudaError_t gemv_bf16(const GemvArgs& a, cudaStream_t stream);

// ----------------------------------------------------------- attention ----
struct AttnPrefillArgs {
  const __nv_bfloat16* q;  // [rows_total, n_heads*128] row stride ldq
  int ldq;
  const int* q_rows;  // optional gather of query rows
  const int* qpos;    // [n_rows]
  int n_rows;
  const __nv_bfloat16* k_cache;  // [n_kv_heads, cache_cap, 128]
  const __nv_bfloat16* v_cache;
  int cache_cap;
  const int* kpos;  // optional [n_keys], non-decreasing; null -> kpos[j] = j
  int n_keys;
  int n_heads, n_kv_heads, head_dim;
  float scale;
  __nv_bfloat16* out;  // [n_rows, n_heads*128]
  int ldo;
  int* status;  // bounded-wait status word
  unsigned long long* trace;  // optional debug timeline (640 entries), null in production
  // Optional key split for grids that leave SMs idle (few query rows): CTA z
  // of `splits` streams its share of the row tile's key tiles and leaves
  // fp32 (O, running max, sum) partials in ws[split][row][head][132]; a merge
  // kernel combines them.  ws = null or ws_floats too small: no split.
  float* ws;
  long long ws_floats;
  int splits;  // set by the launcher
};

cudaError_t attention_prefill(const AttnPrefillArgs& p, cudaStream_t stream);

// Attention of one new position over its past keys (recurrent drafter trunk,
// K14): q [B, Hq, 128], k / v [B, Hkv, P, 128] bf16 contiguous, Hq / Hkv <= 8.
constexpr int kRecurrentAttnMaxKeys = 1024;
struct RecurrentAttnArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* out;   // [B, Hq, 128]
  float* lse;           // [B, Hq] (written by the forward, read by the backward)
  const __nv_bfloat16* dout;  // backward: dO [B, Hq, 128]
  __nv_bfloat16* dq;    // backward outputs
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int batch, n_heads, n_kv_heads, n_keys;
  float scale;
};
cudaError_t recurrent_attention_fwd(const RecurrentAttnArgs& a, cudaStream_t stream);
cudaError_t recurrent_attention_bwd(const RecurrentAttnArgs& a, cudaStream_t stream);
// key splits the launcher would use for these arguments (1 = none)
int attention_prefill_splits(const AttnPrefillArgs& p, int num_sms);
void set_attention_prefill_splits(int s);  // measurement hook (0 = automatic)
// the mma.sync kernel the tcgen05 one replaced, kept for A/B measurement only
cudaError_t attention_prefill_mma(const AttnPrefillArgs& p, cudaStream_t stream);

struct AttnDecodeArgs {
  const __nv_bfloat16* q;  // [M, n_heads*128]
  int M;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  int cache_cap;
  const int* pos;  // device scalar: position of query row 0; row m sees keys [0, pos+m]
  // Optional paged view: virtual key v lives in physical slot
  // (page_table[v >> page_shift] << page_shift) + (v & page_mask); the view
  // holds *n_virtual keys, the last M of which are the query rows themselves
  // (row m sees virtual keys [0, *n_virtual - M + m]).  Without a page table
  // the view is the identity over [0, *pos + M).
  const int* page_table;
  int page_shift;
  const int* n_virtual;
  int n_heads, n_kv_heads;
  float scale;
  int splits;  // CTAs per cluster = thread-block cluster size (1..16)
  __nv_bfloat16* out;  // [M, n_heads*128]
  // Optional second split level for long contexts / few kv heads: R clusters
  // per kv head, each merging its CTAs through DSMEM and leaving a partial
  // (max, sum, numerator) in ws; the last CTA of the kv head (atomic ticket
  // in counters[kvh], reset to zero by it) merges the R partials in cluster
  // order.  R is chosen from the capacity and the head count only, so a row's
  // result does not depend on M.
  float* ws;           // [n_kv_heads][16][32][130] fp32 (null: one cluster per kv head)
  unsigned* counters;  // [n_kv_heads][8] (one per kv head and group of 4 query vectors), zero between launches
  int outer;           // clusters per kv head; 0 = chosen from the capacity (attention_decode_outer)
  // Batched sequences (null: one sequence): n_seq independent sequences of
  // one query row each (M = 1); sequence s's row is q/out row s, it sits at
  // position pos_rows[s] (keys [0, pos_rows[s]]) and its caches start
  // s * seq_stride elements after k_cache / v_cache.  One cluster per kv head.
  const int* pos_rows;
  long long seq_stride;
  int n_seq;
  // Geometry key count (0: cache_cap): keys per CTA and clusters per kv head
  // are sized for this many keys instead of the whole cache.  Must bound the
  // call's key count.  Sparse draft steps over a small view of a long cache
  // set it to the view's keys (their boundaries need not match the verifier's);
  // decode and verification keep 0, so a row sees the same split boundaries
  // in both.
  int key_cap;
  // Optional L2 prefetch of the next kernels' weights (bytes multiples of 16,
  // 16-byte-aligned bases): the key loop leaves HBM mostly idle, so the
  // o-projection and the start of the gate/up weights can stream into L2
  // while it runs.  Issued after the wait on the predecessor, spread over all
  // CTAs; a hint only, nothing waits on it.
  const void* pf_ptr[2];
  long long pf_bytes[2];
};

cudaError_t attention_decode(const AttnDecodeArgs& a, cudaStream_t stream);
int attention_decode_cluster(int cache_cap, int n_kv_heads);
int attention_decode_outer(int cache_cap, int n_kv_heads, int cluster, int num_sms);

// ------------------------------------------------------------ pointwise ----
cudaError_t rmsnorm_bf16(const __nv_bfloat16* x, int ldx, const int* rows, const __nv_bfloat16* w,
                         __nv_bfloat16* out, int ldo, int M, int D, float eps,
                         cudaStream_t stream);
cudaError_t embedding_bf16(const int* ids, const __nv_bfloat16* table, __nv_bfloat16* out, int M,
                           int D, cudaStream_t stream);
cudaError_t gather_rows_bf16(const __nv_bfloat16* in, int ldi, const int* rows,
                             __nv_bfloat16* out, int ldo, int M, int D, cudaStream_t stream);

// Relocate cached keys: rotate every key of [n_kv_heads, n_tokens, 128]
// blocks from source to target positions (fp32 math, bf16 storage).
struct ComposeDoc {
  const __nv_bfloat16* src;  // [L, 2, n_kv_heads, n_tokens, 128] (device or mapped host)
  int n_tokens;
  int src_pos;   // RoPE position of the first source token
  int dst_slot;  // first destination slot
  int dst_pos;   // RoPE position of the first destination token
};
struct ComposeArgs {
  const ComposeDoc* docs;  // device array
  int n_docs;
  const int* doc_token_offset;  // [n_docs + 1] prefix sum of n_tokens
  int total_tokens;
  int layer_begin, layer_end, n_layers;
  __nv_bfloat16* cache;  // [L, 2, n_kv_heads, cache_cap, 128]
  int cache_cap;
  int n_kv_heads;
  const float2* rope_table;
};
cudaError_t compose_relocate(const ComposeArgs& a, cudaStream_t stream);

// CacheBlend selection: from deviation partials [T, 2*n_kv_heads] choose the
// top ceil(ratio * n_doc) document rows in [doc_begin, doc_end), merge with
// mandatory rows and emit the sorted active list.
struct SelectArgs {
  const float* dev_part;
  int n_kv_heads;
  int dev_mode;
  int total_rows;   // T
  int doc_begin, doc_end;
  int k;            // number of document rows to select
  int keep_prefix;  // keep [0, doc_begin) active
  int* active;      // out [A]
  int* n_active;    // out scalar
  float* scores;    // scratch [T]
  long long* checksum;  // optional out: sum over sorted selected doc positions * rank
  // tensor parallel: the partials of n_parts ranks (each [T][2 * n_kv_heads]
  // over its own kv heads) lie part_stride floats apart; scores sum them all
  int n_parts;
  long long part_stride;
};
cudaError_t cacheblend_select(const SelectArgs& a, cudaStream_t stream);

// Skinny tensor-core GEMM for M <= 16 token rows (skinny_tc.cu).
enum SkinnyEpi { SKINNY_STORE = 0, SKINNY_RESIDUAL = 1, SKINNY_SWIGLU = 2, SKINNY_QKV = 3, SKINNY_ALLREDUCE = 4 };
struct SkinnyArgs {
  const __nv_bfloat16* x;  // [M, K] row stride ldx
  const __nv_bfloat16* w;  // [N, K] row stride ldw
  int M, N, K, ldx, ldw;
  int epi;
  __nv_bfloat16* out;      // [M, N] (SwiGLU: [M, N / 2]) row stride ldo
  int ldo;
  const __nv_bfloat16* residual;  // [M, N] row stride ldr (SKINNY_RESIDUAL; may alias out)
  int ldr;
  float* ws;               // [splits][M][N] fp32 (at least splits * N * bn floats, bn = skinny_bn(M))
  int splits;
  int bn;                  // token-row tile (16, 32 or 64), set by the launcher
  int num_sms;
  int* status;
  // SKINNY_QKV: fused QKV rows (q heads, k heads, v heads of 128): RoPE on
  // q/k at position *pos + m, q to q_out, k/v to the cache at slot (*slot or
  // *pos) + m -- the GEMV_QKV epilogue
  __nv_bfloat16* q_out;
  int ldq;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int cache_cap;
  const int* pos;
  const int* slot;
  const float2* rope_table;
  int n_q_heads, n_kv_heads;
  // batched decode: row m belongs to sequence m, at position pos_rows[m], and
  // its cache starts seq_stride elements after row m-1's (null: one sequence)
  const int* pos_rows;
  long long seq_stride;
  // with pos_rows: row m's K/V go to cache slot slot_rows[m] of the one
  // sequence (CacheBlend's active rows: RoPE position and slot differ)
  const int* slot_rows;
  // SKINNY_ALLREDUCE: fp32 partial rows to every rank's receive slot
  // ar_dst[r][sender][m][N], then the last CTA releases ar_flag[r] = epoch
  float* ar_dst[8];
  int* ar_flag[8];
  int ar_tp, ar_sender, ar_epoch;
  const int* ar_epoch_ptr;
  int ar_epoch_mul;
  unsigned int* counter;
};
int skinny_splits(int N, int K, int num_sms);
// The reduce + epilogue half of skinny_gemm alone (a.ws holds the [splits][M][N]
// partials of another producer, e.g. the token-column GEMM); any M.
cudaError_t skinny_reduce(const SkinnyArgs& a, cudaStream_t stream);

// Token-column tensor-core GEMM for 64 < M <= 512 token rows (gemm_wide.cu):
// weight tiles are the MMA's 128-row M, token rows its N (multiple of 16).
enum WideEpi { WIDE_PARTIAL = 0, WIDE_SWIGLU = 1 };
struct WidePlan {
  int acc;        // 128-row weight tiles per unit (1, or 2 = a SwiGLU gate/up block pair)
  int bn;         // token columns per unit (multiple of 16, <= 256)
  int n_tt;       // token tiles (n_tt * bn >= M)
  int splits;     // K slices
  int stages;     // TMA ring depth
  int nbuf;       // TMEM accumulator buffers
  int tmem_cols;  // TMEM allocation (power of two)
  int smem;       // dynamic shared memory bytes
  int grid;       // persistent CTAs
  // stream-K tail: when the units do not fill whole rounds of the grid, the
  // last sk_tail units are cut into sk_ctas equal runs of k-blocks, one per
  // CTA; the pieces of a unit meet in sk_ws and the last to finish applies
  // the epilogue (0 = every unit runs whole)
  int sk_tail;
  int sk_ctas;
  int sk_max_pieces;
};
struct WideArgs : WidePlan {
  const __nv_bfloat16* x;  // [M, K] row stride ldx
  const __nv_bfloat16* w;  // [N, K] row stride ldw
  int M, N, K, ldx, ldw;
  int epi;
  float* ws;               // WIDE_PARTIAL: [splits][M][N] fp32
  __nv_bfloat16* out;      // WIDE_SWIGLU: [M, N / 2] row stride ldo
  int ldo;
  int num_sms;
  int* status;
  float* sk_ws;            // [sk_tail][sk_max_pieces][acc][bn][128] fp32 partials of split tail units
  unsigned* sk_tickets;    // [sk_tail] arrival counters, zero between launches (the last arrival resets)
};
// Cheapest plan for the shape (a *_req of 0 leaves that choice free); false if none fits.
bool wide_plan(int M, int N, int K, int epi, int num_sms, int acc_req, int n_tt_req, int splits_req,
               bool stream_k, WidePlan* plan);
cudaError_t wide_gemm(const WideArgs& a, cudaStream_t stream);
// token-row tile of the skinny GEMM for M rows: 16 (M <= 16), 32 (M <= 32) or 64 (M <= 64)
int skinny_bn(int M);
cudaError_t skinny_gemm(const SkinnyArgs& a, cudaStream_t stream);
// Row argmax over bf16 logits [M, V] (first index on ties) -> out_token[M].
cudaError_t row_argmax_bf16(const __nv_bfloat16* logits, int ld, int M, int V, int* out_token, cudaStream_t stream);

// Row log-sum-exp + logit gathers (forward) and the logits gradient
// g_lse * softmax + sum_j g_z[j] * onehot(ids[j]) (backward), lm_loss.cu.
struct LseGatherArgs {
  const __nv_bfloat16* logits;  // [R, V] row stride ld
  int ld, R, V;
  const int* ids;  // [R, G], -1 = no id
  int G;
  float* lse;      // [R]
  float* z;        // [R, G]
  const float* g_lse;  // backward inputs (g_lse may be null)
  const float* g_z;
  __nv_bfloat16* dlogits;  // [R, V] row stride ldd (may alias logits)
  int ldd;
};
cudaError_t lse_gather(const LseGatherArgs& a, cudaStream_t stream);
cudaError_t lse_gather_backward(const LseGatherArgs& a, cudaStream_t stream);

cudaError_t fill_arange_i32(int* out, int n, int start, cudaStream_t stream);

// Owner-side reduction of GEMM -> reduce-scatter partials: waits (bounded)
// until every sender released flags[s] >= epoch, then
//   out[row] = residual[row] + bf16(sum_s recv[s][row])   (fixed rank order)
// and optionally norm_out[row] = RMSNorm(out[row]) * norm_w.
struct RsReduceArgs {
  const void* recv;   // [tp, rows, N], fp32 or bf16 (recv_bf16)
  int recv_bf16;
  int tp, rows, N;
  const int* flags;   // [tp]
  int epoch;          // epoch = epoch_ptr ? *epoch_ptr * epoch_mul + epoch : epoch
  const int* epoch_ptr;
  int epoch_mul;
  long long timeout_ns;
  int* status;
  const __nv_bfloat16* residual;  // [rows, N]
  __nv_bfloat16* out;             // [rows, N] (may alias residual)
  const __nv_bfloat16* norm_w;    // optional [N]
  __nv_bfloat16* norm_out;        // optional [rows, N]
  float eps;
};
cudaError_t rs_reduce(const RsReduceArgs& a, cudaStream_t stream);

// -------------------------------------------------------- page scores ----
constexpr int kPsMaxLayers = 8;
constexpr int kPsMaxRowsPerGroup = 64;
struct PageScoreArgs {
  const float* q;                       // [n_layers, n_rows, n_q_heads, 128] fp32 (RoPE applied)
  const __nv_bfloat16* keys[kPsMaxLayers];  // per layer [n_kv_heads, cache_cap, 128]
  int cache_cap;
  int n_layers, n_rows, n_q_heads, n_kv_heads, n_tokens;
  float scale;
  float* logits;        // scratch [n_layers * n_rows * n_q_heads, n_tokens]
  float2* partials;     // scratch [n_layers * n_rows * n_q_heads, ceil(n_tokens / 256)]
  float2* stats;        // scratch [n_layers * n_rows * n_q_heads]
  float* token_scores;  // [n_tokens]
};
cudaError_t page_token_scores(const PageScoreArgs& a, cudaStream_t stream);

// ------------------------------------------------------------------- p2p ----
cudaError_t peer_signal(int* flag, int value, const int* value_src, unsigned long long* stamp,
                        cudaStream_t stream);
cudaError_t wait_flag(const int* flag, int target, long long timeout_ns, int* status,
                      unsigned long long* stamp, cudaStream_t stream);
cudaError_t peer_signal_many(int* const* addrs, int n, int value, cudaStream_t stream);
cudaError_t index_i32(const int* src, const int* idx, int* out, int n, cudaStream_t stream);

// ------------------------------------------------- K13 sparse memory attention
struct MemAttnArgs {
  const __nv_bfloat16* q;     // [L, R, H, 128]
  const __nv_bfloat16* k;     // memory keys (strided, see below)
  const __nv_bfloat16* v;     // memory values (same strides)
  long long layer_stride, seq_stride, tok_stride, head_stride;  // elements
  const int* row_seq;         // [R] row -> sequence (null: all rows sequence 0)
  const int* idx;             // [S, idx_stride] visible token rows (null: 0..n-1)
  long long idx_stride;
  const int* n_vis;           // [S] visible count (null: n_fixed)
  int n_fixed;
  int L, R, H;
  float scale, scale_log2;
  __nv_bfloat16* out;         // fwd: [L, R, H, 128]
  float* lse;                 // [L, R, H] base-2 log-sum-exp of the scaled scores
  const __nv_bfloat16* o;     // bwd: forward output
  const __nv_bfloat16* dout;  // bwd: gradient of the output
  float* dq;                  // bwd: [L, R, H, 128] fp32
};
cudaError_t mem_attn_fwd(const MemAttnArgs& a, cudaStream_t stream);
cudaError_t mem_attn_bwd(const MemAttnArgs& a, cudaStream_t stream);

// ------------------------------------------------------ K16 optimizer / DP
// AdamW over one flat fp32 parameter range with device-side step, learning
// rate and global gradient-norm clipping (graph-replayable: no host scalars
// change between steps).  ``hyper`` (device, fp32) holds
//   [0] lr  [1] beta1  [2] beta2  [3] eps  [4] weight_decay  [5] max_norm
//   [6] step offset (data parallel: the step is *epoch_ptr + [6], so a resumed
//       run keeps its bias correction while its flags restart from zero)
// and ``state`` (device, fp32) is written by the norm pass:
//   [0] step  [1] 1-beta1^step  [2] 1-beta2^step  [3] grad norm  [4] clip coef
struct AdamArgs {
  float* param;        // master fp32 (this rank's shard for DP)
  const float* grad;   // fp32 gradient (reduced)
  float* exp_avg;
  float* exp_avg_sq;
  long long n;
  const float* hyper;
  float* state;
  float* partial;      // [grid] sum-of-squares partials
  unsigned* counter;   // last-CTA ticket (zeroed by the kernel that consumes it)
};
cudaError_t adamw_norm(const AdamArgs& a, int grid, cudaStream_t stream);
cudaError_t adamw_update(const AdamArgs& a, cudaStream_t stream);

// Data-parallel gradient reduce-scatter + AdamW + parameter all-gather over
// CUDA-IPC peer memory.  Rank r owns elements [r*shard, (r+1)*shard) of the
// flat buffers.  Phase 1 (dp_reduce_norm): wait for every rank's "grads
// ready" flag, sum the peers' gradients of the owned shard in rank order
// (deterministic and identical on every rank), write the shard's
// sum-of-squares into every peer's norm slot and release "norms ready".
// Phase 2 (dp_adamw_gather): wait for every norm, form the global clip
// coefficient, run AdamW on the shard and store the new parameters into
// every peer's parameter buffer, then release "params ready".
struct DpArgs {
  int world, rank;
  long long n_total, shard;         // elements; shard * world >= n_total
  const float* grads[kMaxShards];   // every rank's flat gradient (peer pointers)
  float* params[kMaxShards];        // every rank's flat parameters (peer pointers)
  float* norms[kMaxShards];         // every rank's [world] sum-of-squares slots
  int* flag_grads;                  // this rank's [world] flags (peers release into them)
  int* flag_norms;
  int* peer_flag_norms[kMaxShards]; // where this rank releases its "norm ready"
  int* peer_flag_params[kMaxShards];
  const int* epoch_ptr;             // device step counter (epoch = *epoch_ptr)
  long long timeout_ns;
  int* status;
  float* red_grad;                  // [shard] reduced gradient of the owned shard
  float* exp_avg;                   // [shard]
  float* exp_avg_sq;                // [shard]
  const float* hyper;
  float* state;
  float* partial;
  unsigned* counter;
  int pre_reduced;                  // 1: red_grad already holds the reduced shard (bucketed reduce)
};
cudaError_t dp_reduce_norm(const DpArgs& a, int grid, cudaStream_t stream);
cudaError_t dp_reduce_range(const DpArgs& a, const int* flags, long long lo, long long hi, int grid,
                            cudaStream_t stream);
cudaError_t dp_adamw_gather(const DpArgs& a, int grid, cudaStream_t stream);
cudaError_t bump_counter(int* counter, cudaStream_t stream);

// Release (*epoch_ptr + offset) into up to 8 flag words; bounded wait until
// flags[0..n) >= *epoch_ptr + offset.
struct FlagPtrs {
  int* addr[kMaxShards];
  int n;
};
cudaError_t signal_epoch(const FlagPtrs& flags, const int* epoch_ptr, int offset, cudaStream_t stream);
cudaError_t wait_all(const int* flags, int n, const int* epoch_ptr, int offset, long long timeout_ns, int* status,
                     cudaStream_t stream);

}  // namespace sc
