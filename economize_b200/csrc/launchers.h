// Host-side entry points of the CUDA kernels (raw pointers; the torch bindings check shapes and dtypes).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ecz {

constexpr int kMaxPeers = 8;
struct PeerPtrs {
  void* ptr[kMaxPeers];
};

// Where a row-parallel GEMM pushes its output in tensor-parallel push mode (world == 0: ordinary output).
//   mode 0 (all-reduce push): every output element goes into slot `rank` of every peer's buffer (parity `parity`).
//   mode 1 (reduce-scatter, sequence-parallel buffers of tp_sp.cu): output row m goes only to its owner rank
//   m / shard_rows, into that rank's partial slot [parity][rank][m % shard_rows]; the parity is the device-side round
//   counter of this rank's own control block (read after the predecessor grid completed).
struct PeerOut {
  PeerPtrs ptrs;
  int world = 0;
  int rank = 0;
  int parity = 0;
  long slot_elems = 0;
  long control_bytes = 256;
  int mode = 0;
  int shard_rows = 0;   // mode 1: tokens per rank (the last ranks may own fewer or none)
  int shard_max = 0;    // mode 1: rows of one partial slot
  long data_off = 0;    // mode 1: byte offset of the partial slots in every peer's buffer
};

// Control words (unsigned) at the start of a sequence-parallel buffer (tp_sp.cu). Rounds of each kind alternate
// between two parities; the round counters live on the device so captured CUDA graphs replay with the right ones.
constexpr int kSpRsArrive = 0;     // [2] source ranks whose reduce-scatter partials of a round arrived here
constexpr int kSpPushDone = 4;     // CTAs of this rank's current reduce-scatter GEMM that finished
constexpr int kSpReduceDone = 5;   // CTAs of this rank's current reduce kernel that finished
constexpr int kSpRsRound = 6;      // reduce-scatter rounds this rank has consumed
constexpr int kSpAgArrive = 8;     // [2] source ranks whose all-gather rows of a round arrived here
constexpr int kSpAgDone = 10;      // CTAs of this rank's current all-gather consumer that finished waiting
constexpr int kSpAgRound = 11;     // all-gather rounds this rank has consumed
constexpr int kSpControlBytes = 256;

// An all-gather -> GEMM consumer: the TMA producer of every CTA waits (bounded) until all `world` ranks' rows of the
// current all-gather round arrived in this rank's buffer, then loads X from the round's parity (tensor map 0 or 1);
// the last CTA resets the arrival count and advances the round. ctrl == nullptr: an ordinary GEMM.
struct AgWait {
  unsigned* ctrl = nullptr;
  int world = 0;
};

// Paged KV caches: where (sequence, KV head, logical slot) rows live; the device-side mapping is kv_row /
// kv_layer_row in common.cuh, which documents the layouts.
struct KVPages {
  const int* table = nullptr;
  int max_chunks = 0;
  int page_rows = 0;
};

struct KVLayout {
  KVPages pages;
  long table_stride = 0;
  long layer_rows = 0;
  long v_rows = 0;
};

// Score options of an attention launch: tanh soft-cap of the scaled scores (0: off), one sink logit per query head
// (fp32 [H], natural-log units; nullptr: off), sliding window in positions (0: off).
struct AttnOpts {
  float softcap = 0.f;
  const float* sinks = nullptr;
  int window = 0;
};

struct AttnPlan {
  int m_tiles = 1;
  int splits = 1;
  int chunks_per_split = 1;
  long ws_floats = 0;
  bool tail = false;  // exact-tail mode: partials always staged in the workspace
};

// elementwise.cu
// x_parts / qkv_parts / gu_parts: optional fp32 split-K partials [splits][...] of the input, summed in split order
// and rounded to bf16 in place of reading the bf16 input.
int launch_rmsnorm(const void* x, const void* resid, const void* w, void* out, void* resid_out, int rows, int hidden,
                   float eps, cudaStream_t stream, const float* x_parts = nullptr, int splits = 0);
int launch_rope_store(const void* qkv, const int* positions, const float* cos_t, const float* sin_t, void* q_out,
                      void* k_cache, void* v_cache, const int* kv_len, const int* n_new, const void* q_norm,
                      const void* k_norm, float eps, int B, int T, int H, int Hkv, int D, int S, int q_offset,
                      cudaStream_t stream, const float* k_scale = nullptr, const float* v_scale = nullptr,
                      const float* qkv_parts = nullptr, int splits = 0, const KVPages& pages = KVPages(),
                      int table_rows = 1 << 30, unsigned* status = nullptr);
// act(gate) * up of a fused [gate; up] projection: act 0 = SiLU, 1 = GELU (tanh approximation), 2 = clamped SwiGLU
// ((clamp(up, -limit, limit) + 1) * g * sigmoid(1.702 g), g = min(gate, limit))
int launch_glu(const void* gu, void* out, int rows, int F, cudaStream_t stream, const float* gu_parts, int splits,
               int act,
               float limit = 7.f);
int launch_silu_mul(const void* gu, void* out, int rows, int F, cudaStream_t stream, const float* gu_parts = nullptr,
                    int splits = 0);
// Block Walsh-Hadamard transform x H_b / sqrt(b) of every row (blocks of b = 2^p, 8 <= b <= 8192, dividing F); with
// glu_act_kind >= 0 the input is the fused [gate; up] projection and the transformed value is act(gate) * up
// (glu_act_kind as launch_glu's act; -1: x is the bf16 [rows, F] input itself)
int launch_hadamard(const void* x, void* out, int rows, int F, int block, cudaStream_t stream, int glu_act_kind = -1,
                    const float* gu_parts = nullptr, int splits = 0, float limit = 7.f);
// MInference vertical-slash keep bitmap of `rows` (row, KV head) pairs: cols [rows, nv] key columns, offsets [rows, ns]
// slash diagonals (query position - key position) of a chunk of t queries at `base`; keys >= limit are dropped;
// keep [rows, S / 32] bit words (S a multiple of 32, at most 262144)
int launch_vs_keep(const int64_t* cols, int nv, const int64_t* offsets, int ns, int base, int t, int limit, int rows,
                   int S, uint32_t* keep, cudaStream_t stream);
int argmax_slices(int rows, int V);
int launch_argmax(const void* x, bool is_bf16, int64_t* out, float* part_v, int* part_i, int rows, int V,
                  cudaStream_t stream);
// ok [B, T] (optional): node t is acceptable given its parent; without it, tokens[t] == pred[parent].
int launch_greedy_accept(const int64_t* tokens, const int64_t* parents, const int64_t* pred, const uint8_t* ok,
                         int* n_acc, int* path, int64_t* out, int B, int T, cudaStream_t stream);
int launch_kv_compact(void* cache, const int* kv_len, const int* path, const int* n_acc, int L, int B, int Hkv,
                      int S, int row_bytes, int T, int max_depth, cudaStream_t stream, const KVLayout& layout);

// gemm_tc.cu
int gemm_block_n(int M);
int gemm_splits(int M, int N, int K, int num_sms);
// With `counters` (a zeroed int array of at least num_sms entries, private to the stream) the split-K partials are
// reduced inside the GEMM by the last CTA of each tile; without, by a second kernel.
int launch_gemm_bf16(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, float* ws, int M, int N, int K,
                     int splits, unsigned* status, cudaStream_t stream, int* counters = nullptr,
                     const PeerOut* peer = nullptr, int flags = 0, const AgWait* ag = nullptr,
                     const CUtensorMap* tm_x1 = nullptr);

// Cluster split-K GEMM (partials reduced over DSMEM inside each tile's cluster; no workspace).
int gemm_cluster_splits(int M, int N, int K, int num_sms);
int gemm_cluster_capacity(int M, int splits);
int launch_gemm_cluster(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, int M, int N, int K, int splits,
                        unsigned* status, cudaStream_t stream, const PeerOut* peer = nullptr,
                        const AgWait* ag = nullptr, const CUtensorMap* tm_x1 = nullptr);

// Persistent stream-K GEMM: `ws` holds gemm_persistent_ws_floats() floats, `counters` >= num_sms zeroed ints
// private to the stream (the kernel resets them).
int gemm_persistent_ctas(int M, int N, int K, int num_sms);
long gemm_persistent_ws_floats(int M, int N, int K, int num_sms);
int launch_gemm_persistent(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, float* ws, int* counters, int M,
                           int N, int K, int num_sms, unsigned* status, cudaStream_t stream);

// attention.cu
AttnPlan attention_plan(int B, int T, int H, int Hkv, int S, int num_sms, bool tail = false, int D = 128,
                        int window = 0);
int launch_attention(const void* q, const CUtensorMap* tm_k, const CUtensorMap* tm_v, void* out, float* ws,
                     const int* kv_len, const int* n_new, const int64_t* mask, int B, int T, int H, int Hkv, int D,
                     int S, float scale, int q_offset, const AttnPlan& plan, unsigned* status, cudaStream_t stream,
                     unsigned long long* trace = nullptr, const float* k_scale = nullptr,
                     const float* v_scale = nullptr, const uint32_t* keep = nullptr, float* lse_out = nullptr,
                     const uint8_t* kivi = nullptr, const int* kivi_chunks = nullptr, int kivi_bits = 0,
                     int tail_w = 0, const void* k_cache = nullptr, const void* v_cache = nullptr,
                     const AttnOpts& opts = AttnOpts(), const KVPages& pages = KVPages());
// KIVI: bytes of one quantized 128-key chunk; quantise committed chunks of a bf16 cache [L, 2, B, Hkv, S, D] into
// kivi [L, B, Hkv, S / 128, chunk bytes] and advance chunks [B] (at most max_new chunks per row and call)
int kivi_chunk_size(int bits);
int launch_kivi_quantize(const void* cache, void* kivi, const int* kv_len, int* chunks, int L, int B, int Hkv, int S,
                         int D, int bits, int residual, int max_new, cudaStream_t stream,
                         const KVLayout& layout);
// KV-eviction scores: scores[b, kvh, s] += attention probability mass of slot s (see attention.cu)
int launch_attention_scores(const void* q, const CUtensorMap* tm_k, const float* lse2, float* scores,
                            const int* kv_len, const int* n_new, const int64_t* mask, int B, int T, int H, int Hkv,
                            int D, int S, float scale, int q_offset, unsigned* status, cudaStream_t stream,
                            const KVPages& pages = KVPages());

// sampling.cu
int launch_topk_logp(const float* logits, const int64_t* d2t, float* vals, int64_t* ids, int rows, int V, int k,
                     float floor_v, cudaStream_t stream, int splits = 1, void* workspace = nullptr,
                     int* counters = nullptr);
// chunks per row of the split top-k (1: one CTA per row) and its workspace; counters: `rows` zeroed ints
int topk_splits(int rows, int V, int num_sms);
size_t topk_workspace_bytes(int rows, int splits);
int launch_sample(const float* probs, const float* u, int64_t* out, int rows, int V, cudaStream_t stream);
int launch_rejection(const float* p, const float* q, const int64_t* drafts, const float* u_acc, const float* u_draw,
                     int* n_acc, int64_t* out, int B, int k, int V, cudaStream_t stream);

// ngram.cu
int launch_ngram(const int64_t* history, const int* len, int64_t* drafts, int B, int cap, int k, int min_n, int max_n,
                 bool earliest, cudaStream_t stream);

// comm.cu: fused NVLink all-reduce (+ residual add + RMSNorm) on IPC-mapped symmetric buffers
size_t symm_control_bytes();
// tp_sp.cu: sequence-parallel tensor parallelism. `layout` describes one rank's buffer (see tp_sp.cu).
struct SpLayout {
  int world = 0, rank = 0, hidden = 0, max_rows = 0, shard_max = 0, n_cap = 0;
  long rs_off = 0, ag_off = 0, cap_off = 0, bytes = 0;
};
SpLayout sp_layout(int world, int rank, int hidden, int max_rows, int n_cap);
// Sum this rank's reduce-scatter partials (partials = true) of rows [row0, row0 + rows) in rank order, add the
// residual shard, write the new residual, RMSNorm, and push the normed rows (and, with cap_slot >= 0, the residual
// rows) into every rank's all-gather buffer; then signal the round. rows may be 0 (a rank that owns no token).
int launch_sp_reduce_norm(const PeerPtrs& peers, const SpLayout& L, bool partials, const void* resid_in,
                          void* resid_out, const void* w, int rows, int row0, float eps, int cap_slot,
                          unsigned* status, cudaStream_t stream);
// Wait for the current all-gather round and copy its rows [0, rows) into out (an all-gather consumer).
int launch_sp_fetch(const PeerPtrs& peers, const SpLayout& L, void* out, int rows, unsigned* status,
                    cudaStream_t stream);
int launch_push(const void* src, long elems, const PeerPtrs& peers, int rank, int world, int parity, long slot_elems,
                int num_sms, cudaStream_t stream);
int launch_reduce_rmsnorm(const PeerPtrs& peers, int rank, int world, int parity, long slot_elems, const void* resid,
                          const void* w, void* out, void* resid_out, int rows, int hidden, float eps,
                          unsigned* status, cudaStream_t stream);

// gemm_wq.cu: weight-only quantized GEMM (W4A16 / W8A16 / fp8-weight); see the file comment for the layouts.
enum WqFormat : int { kWqInt4 = 0, kWqInt8 = 1, kWqFp8 = 2, kWqSp24 = 3, kWqInt2 = 4, kWqMxfp4 = 5, kWqNvfp4 = 6 };
struct WqMaps {
  const CUtensorMap* w = nullptr;  // packed weights, uint8 [N, K * bits / 8], box {64 * bits / 8, 128}
  const CUtensorMap* s = nullptr;  // scales bf16 [K / group, N], box {128, 1}
  const CUtensorMap* z = nullptr;  // zeros bf16 [K / group, N], box {128, 1} (int4 only)
  const CUtensorMap* x = nullptr;  // activations bf16 [M, K], box {64, BN} with the 128-byte swizzle
};
int gemm_wq_splits(int M, int N, int K, int fmt, int num_sms);
int launch_gemm_wq(const WqMaps& maps, void* y, int M, int N, int K, int group, int fmt, int splits,
                   unsigned* status, cudaStream_t stream);

// moe.cu: top-k routing, token permutation, grouped expert GEMM (weights stacked [E * N, K]) and weighted combine.
int launch_moe_route(const void* logits, int T, int E, int k, int* ids, float* weights, int* pos, int* offsets,
                     cudaStream_t stream);
int launch_moe_gather(const void* x, const int* pos, void* xs, int T, int k, int H, cudaStream_t stream);
int launch_moe_combine(const void* y, const int* pos, const float* w, void* out, int T, int k, int H,
                       cudaStream_t stream);
int grouped_block_n(int rows, int E);
int launch_gemm_grouped(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, const int* offsets, int E,
                        int rows, int N, int K, unsigned* status, cudaStream_t stream);

// gemm_fp8.cu: block-scaled fp8 GEMM (e4m3 weights [N, K] with fp32 scales [N / 128, K / 128]; activations
// quantised per token and 128-wide K block by launch_act_quant_fp8 into codes [M, K] and scales [K / 128, >= M]).
int fp8_block_n(int M);
// sx rows are `sx_stride` floats apart (>= M, a multiple of 4 so that a TMA map can read them).
int launch_act_quant_fp8(const void* x, void* q, float* sx, int M, int K, int sx_stride, cudaStream_t stream);
int launch_gemm_fp8(const CUtensorMap* tm_w, const CUtensorMap* tm_x, const CUtensorMap* tm_sx, const float* sw,
                    void* y, float* ws, int M, int N, int K, int splits, unsigned* status, cudaStream_t stream);

int launch_gemm_segments(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, const int* seg_start,
                         const int* seg_end, const int* seg_expert, int G, int max_rows, int N, int K,
                         unsigned* status, cudaStream_t stream);

// act_sparse.cu: activation-sparse GEMVs (<= 16 rows). splits = colsparse_splits(...); with splits > 8, ws holds
// (splits / 8) * M * N floats and counters (zeroed, one per 256 output columns, private to the stream) are reset by
// the kernel.
int colsparse_splits(int M, int N, int K, int num_sms);
int launch_colsparse_gemv(const void* x, int ldx, const void* wt, const float* thr, void* out, float* ws,
                          int* counters, int M, int N, int K, int splits, cudaStream_t stream);
int launch_glu_rows(const void* x, int ldx, const void* w, const void* gate_pre, int ld_gate, const uint8_t* keep,
                    const float* thr, void* h, int M, int F, int H, cudaStream_t stream);

// binary.cu: out[m, n] = sum_k s[n, k] x[m, k] with sign bits packed 32 per word along k (bit set = -1), M <= 16.
int launch_sign_matvec(const uint32_t* bits, const float* x, float* out, int M, int N, int K, cudaStream_t stream);

// tree.cu: dynamic-tree drafting bookkeeping (one CTA per row).
int launch_tree_expand(const float* c_vals, const int64_t* c_ids, float* f_scores, int64_t* f_cand, int64_t* f_tokens,
                       int64_t* parent_fwd, int64_t* fwd_bits, int64_t* origin, int64_t* bits_next,
                       int64_t* cand_tokens, float* cand_scores, int64_t* cand_parents, int B, int k, int d,
                       int n_cand, int n_fwd, bool next, cudaStream_t stream);
int launch_tree_select(const int64_t* cand_tokens, const float* cand_scores, const int64_t* cand_parents, int B,
                       int n_cand, int k, int total, int64_t* out_tokens, int64_t* out_parents, cudaStream_t stream);
int launch_tree_layout(const int64_t* parents, const int* kv_len, int64_t* bits, int* positions, int B, int T,
                       cudaStream_t stream);

// ep.cu: expert-parallel dispatch / combine over IPC-mapped symmetric buffers (layout below, per rank).
struct EpLayout {
  int world = 1, experts_local = 1, cap = 1, hidden = 8, ret_rows = 1;
  long counts_off = 0, meta_off = 0, recv_off = 0, ret_off = 0, bytes = 0;
};
EpLayout ep_layout(int world, int experts_local, int cap, int hidden, int ret_rows);
int launch_ep_dispatch(const void* xs, const int* offsets, const PeerPtrs& peers, const EpLayout& L, int rank,
                       int rows, cudaStream_t stream);
int launch_ep_segments(const PeerPtrs& peers, const EpLayout& L, int rank, int* seg_start, int* seg_end,
                       int* seg_expert, unsigned* status, cudaStream_t stream);
int launch_ep_combine(const void* y, const int* seg_start, const int* seg_end, const PeerPtrs& peers,
                      const EpLayout& L, int rank, cudaStream_t stream);
int launch_ep_finish(const PeerPtrs& peers, const EpLayout& L, int rank, const int* pos, const float* w, void* out,
                     int tokens, int k, unsigned* status, cudaStream_t stream);

// tmap.cpp: a 2-D tensor map over a row-major [rows, cols] matrix of 1- or 2-byte elements (elem_bytes), with a
// {box_cols, box_rows} box and the given swizzle (0, 32, 64 or 128 bytes). Returns 0 on success.
int make_tmap_2d(CUtensorMap* map, int elem_bytes, const void* base, uint64_t rows, uint64_t cols,
                 uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows, int swizzle_bytes);

// tmap.cpp: a 2-D bf16 tensor map over a row-major [rows, cols] matrix with a {64, box_rows} box and the 128-byte
// swizzle (cols * 2 bytes must be a multiple of 16). Returns 0 on success.
int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                      uint32_t box_rows);

}  // namespace ecz
