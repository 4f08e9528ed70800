// Draft-tree bookkeeping of the engine's dynamic-tree drafting (EAGLE-2 expansion), one CTA per row:
//
//   tree_expand_kernel  after a depth's top-k expansion: the children's cumulative scores, tokens and parents are
//                       written into the candidate buffers, and the next frontier (the k best children, ties to the
//                       lower child index), its parents among the forwarded nodes, its ancestor bits and the
//                       origin of every frontier node (for the state gather) are computed
//   tree_select_kernel  the `total` best candidates (key = score - 1e-9 depth in double, ties to the lower index)
//                       in candidate order, with every parent mapped to its position among them
//   tree_layout_kernel  the verified tree's ancestor bits and token positions from its parents (every drafting
//                       mode), in place of pointer doubling and a bit count in tensor operations
//
// Both replace chains of small tensor operations that a captured cycle would otherwise launch one by one.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

constexpr int kTreeThreads = 256;

// d >= 1: c_vals / c_ids [B, k, k] expand the frontier of depth d (k nodes); the children are candidates
// [k + (d - 1) k^2, k + d k^2). With next = 1 the frontier of depth d + 1 is produced.
__global__ void __launch_bounds__(kTreeThreads) tree_expand_kernel(
    const float* __restrict__ c_vals, const int64_t* __restrict__ c_ids, float* __restrict__ f_scores,
    int64_t* __restrict__ f_cand, int64_t* __restrict__ f_tokens, int64_t* __restrict__ parent_fwd,
    int64_t* __restrict__ fwd_bits, int64_t* __restrict__ origin, int64_t* __restrict__ bits_next,
    int64_t* __restrict__ cand_tokens, float* __restrict__ cand_scores, int64_t* __restrict__ cand_parents, int k,
    int d, int n_cand, int n_fwd, int next) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, t = threadIdx.x;
  const int n = k * k;
  __shared__ float sc[kTreeThreads];
  __shared__ int pick[16];
  const int off = k + (d - 1) * n;
  float v = -INFINITY;
  if (t < n) {
    const int f = t / k;
    v = f_scores[b * k + f] + c_vals[static_cast<size_t>(b) * n + t];
    cand_scores[static_cast<size_t>(b) * n_cand + off + t] = v;
    cand_tokens[static_cast<size_t>(b) * n_cand + off + t] = c_ids[static_cast<size_t>(b) * n + t];
    cand_parents[static_cast<size_t>(b) * n_cand + off + t] = f_cand[b * k + f];
  }
  sc[t] = v;
  __syncthreads();
  if (!next) return;
  if (t < n) {  // rank among the children: the k best become the next frontier
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const float o = sc[j];
      rank += (o > v || (o == v && j < t)) ? 1 : 0;
    }
    if (rank < k) pick[rank] = t;
  }
  __syncthreads();
  if (t < k) {
    const int p = pick[t];
    const int org = p / k;
    f_scores[b * k + t] = sc[p];
    f_tokens[b * k + t] = c_ids[static_cast<size_t>(b) * n + p];
    f_cand[b * k + t] = off + p;
    origin[b * k + t] = org;
    const int64_t pf = static_cast<int64_t>(d - 1) * k + org;  // the parent's index among the forwarded nodes
    parent_fwd[b * k + t] = pf;
    const int64_t own = 1ll << (d * k + t);
    const int64_t bits = own | fwd_bits[static_cast<size_t>(b) * n_fwd + pf];
    bits_next[b * k + t] = bits;
    if (d * k + t < n_fwd) fwd_bits[static_cast<size_t>(b) * n_fwd + d * k + t] = bits;
  }
}

__global__ void __launch_bounds__(512) tree_select_kernel(const int64_t* __restrict__ cand_tokens,
                                                          const float* __restrict__ cand_scores,
                                                          const int64_t* __restrict__ cand_parents, int n_cand,
                                                          int k, int total, int64_t* __restrict__ out_tokens,
                                                          int64_t* __restrict__ out_parents) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ double key[];  // [n_cand]
  int* place = reinterpret_cast<int*>(key + n_cand);  // [n_cand]: position among the chosen, or -1
  const int b = blockIdx.x;
  const size_t row = static_cast<size_t>(b) * n_cand;
  for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {
    const int depth = i < k ? 0 : 1 + (i - k) / (k * k);
    key[i] = static_cast<double>(cand_scores[row + i]) - static_cast<double>(depth) * 1e-9;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {
    const double v = key[i];
    int rank = 0;
    for (int j = 0; j < n_cand; ++j) rank += (key[j] > v || (key[j] == v && j < i)) ? 1 : 0;
    place[i] = rank < total ? 1 : -1;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {  // position = chosen candidates before it
    if (place[i] < 0) continue;
    int pos = 0;
    for (int j = 0; j < i; ++j) pos += place[j] >= 0 ? 1 : 0;
    key[i] = static_cast<double>(pos);  // the key is no longer needed
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {
    if (place[i] < 0) continue;
    const int pos = static_cast<int>(key[i]);
    const int64_t p = cand_parents[row + i];
    out_tokens[static_cast<size_t>(b) * total + pos] = cand_tokens[row + i];
    out_parents[static_cast<size_t>(b) * total + pos] =
        p >= 0 && place[p] >= 0 ? static_cast<int64_t>(key[p]) : -1;
  }
}

// parents [B, T] (parents[b, i] < i for i >= 1; node 0 is the root): bits[b, i] has bit j set when node j is i or
// one of its ancestors, positions[b, i] = kv_len[b] + depth(i). One CTA of T threads per row; thread i walks up its
// ancestor chain in shared memory (at most T - 1 steps, so a malformed row cannot loop).
__global__ void __launch_bounds__(64) tree_layout_kernel(const int64_t* __restrict__ parents,
                                                         const int* __restrict__ kv_len, int64_t* __restrict__ bits,
                                                         int* __restrict__ positions, int T) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, i = threadIdx.x;
  __shared__ int par[64];
  if (i < T) par[i] = static_cast<int>(parents[static_cast<size_t>(b) * T + i]);
  __syncthreads();
  if (i >= T) return;
  uint64_t m = 1ull << i;
  int depth = 0;
  for (int j = i, steps = 0; j > 0 && steps < T; ++steps) {
    const int p = par[j];
    j = (p >= 0 && p < j) ? p : 0;  // parents precede their children; anything else ends the walk at the root
    m |= 1ull << j;
    ++depth;
  }
  bits[static_cast<size_t>(b) * T + i] = static_cast<int64_t>(m);
  positions[static_cast<size_t>(b) * T + i] = kv_len[b] + depth;
}

}  // namespace

int launch_tree_layout(const int64_t* parents, const int* kv_len, int64_t* bits, int* positions, int B, int T,
                       cudaStream_t stream) {
  if (T < 1 || T > 64) return -1;
  if (B == 0) return 0;
  launch_pdl(tree_layout_kernel, dim3(B), dim3(64), 0, stream, parents, kv_len, bits, positions, T);
  return 0;
}

int launch_tree_expand(const float* c_vals, const int64_t* c_ids, float* f_scores, int64_t* f_cand, int64_t* f_tokens,
                       int64_t* parent_fwd, int64_t* fwd_bits, int64_t* origin, int64_t* bits_next,
                       int64_t* cand_tokens, float* cand_scores, int64_t* cand_parents, int B, int k, int d,
                       int n_cand, int n_fwd, bool next, cudaStream_t stream) {
  if (k < 1 || k > 16 || d < 1 || (next && (d + 1) * k > 64)) return -1;
  launch_pdl(tree_expand_kernel, dim3(B), dim3(kTreeThreads), 0, stream, c_vals, c_ids, f_scores, f_cand, f_tokens,
             parent_fwd, fwd_bits, origin, bits_next, cand_tokens, cand_scores, cand_parents, k, d, n_cand, n_fwd,
             next ? 1 : 0);
  return 0;
}

int launch_tree_select(const int64_t* cand_tokens, const float* cand_scores, const int64_t* cand_parents, int B,
                       int n_cand, int k, int total, int64_t* out_tokens, int64_t* out_parents, cudaStream_t stream) {
  if (total < 1 || total > n_cand || n_cand > 4096) return -1;
  const size_t smem = static_cast<size_t>(n_cand) * (sizeof(double) + sizeof(int));
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(tree_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  }
  launch_pdl(tree_select_kernel, dim3(B), dim3(512), smem, stream, cand_tokens, cand_scores, cand_parents, n_cand, k,
             total, out_tokens, out_parents);
  return 0;
}

}  // namespace ecz
