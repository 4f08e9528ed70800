// Sampling kernels of the speculative cycle (no host synchronization, CUDA-graph safe):
//
//   sample_kernel       one token per row of a probability matrix by inverse CDF with a given uniform number
//   rejection_kernel    lossless speculative sampling of a draft chain (Leviathan et al. 2023 / Chen et al. 2023):
//                       draft token x_j (drawn from q_j) is accepted with probability min(1, p_j(x_j) / q_j(x_j));
//                       at the first rejection the correction is drawn from norm(max(0, p_j - q_j)); if every draft
//                       is accepted the bonus token is drawn from p_k. The output distribution equals sampling
//                       from p step by step.
//
// One CTA of 1024 threads per row. A draw over V entries: every thread sums a contiguous slice, the CTA scans the
// slice sums, and the thread whose slice holds u * total scans it sequentially. Uniforms come from the caller
// (torch's Philox generator), so replays of a captured graph draw fresh numbers.
#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

constexpr int kThreads = 1024;

// Inverse-CDF draw from weights w[0..V) (w(i) computed by `weight`), target u in [0, 1). Returns the index; -1 if
// the total weight is zero. All threads of the CTA call it.
template <typename F>
__device__ int draw(int V, float u, F weight, float* scan, float* total_out) {
  const int per = (V + kThreads - 1) / kThreads;
  const int lo = threadIdx.x * per, hi = min(V, lo + per);
  float part = 0.f;
  for (int i = lo; i < hi; ++i) part += weight(i);
  // inclusive block scan of the slice sums (Hillis-Steele over shared memory)
  scan[threadIdx.x] = part;
  __syncthreads();
  for (int off = 1; off < kThreads; off <<= 1) {
    const float add = threadIdx.x >= off ? scan[threadIdx.x - off] : 0.f;
    __syncthreads();
    scan[threadIdx.x] += add;
    __syncthreads();
  }
  const float total = scan[kThreads - 1];
  if (total_out != nullptr && threadIdx.x == 0) *total_out = total;
  __shared__ int found;
  if (threadIdx.x == 0) found = -1;
  __syncthreads();
  if (total > 0.f) {
    const float target = u * total;
    const float before = threadIdx.x > 0 ? scan[threadIdx.x - 1] : 0.f;
    if (target >= before && (target < scan[threadIdx.x] || threadIdx.x == kThreads - 1)) {
      float run = before;
      int pick = -1;
      for (int i = lo; i < hi; ++i) {
        const float w = weight(i);
        if (w > 0.f) pick = i;  // last positive entry: guards rounding at the slice end
        run += w;
        if (run > target && w > 0.f) { pick = i; break; }
      }
      if (pick >= 0) atomicMax(&found, pick);  // at most one thread matches; max keeps it simple
    }
  }
  __syncthreads();
  int result = found;
  if (result < 0 && total > 0.f) {
    // the target fell on a slice boundary with an empty slice: take the last positive entry overall
    __shared__ int last;
    if (threadIdx.x == 0) last = -1;
    __syncthreads();
    for (int i = hi - 1; i >= lo; --i) {
      if (weight(i) > 0.f) { atomicMax(&last, i); break; }
    }
    __syncthreads();
    result = last;
  }
  __syncthreads();
  return result;
}

__global__ void __launch_bounds__(kThreads) sample_kernel(const float* __restrict__ probs,
                                                          const float* __restrict__ u, int64_t* __restrict__ out,
                                                          int V) {
  pdl_trigger();
  pdl_wait();
  __shared__ float scan[kThreads];
  const float* p = probs + static_cast<size_t>(blockIdx.x) * V;
  const int idx = draw(V, u[blockIdx.x], [&](int i) { return p[i]; }, scan, nullptr);
  if (threadIdx.x == 0) out[blockIdx.x] = idx < 0 ? 0 : idx;
}

// p [B, k + 1, V] target probabilities at the root and after every draft; q [B, k, V] the draft distributions the
// drafts were drawn from; drafts [B, k]; u_acc [B, k] and u_draw [B] uniforms. Outputs n_acc [B] and
// out [B, k + 1] (accepted drafts, then the correction or bonus token).
__global__ void __launch_bounds__(kThreads) rejection_kernel(const float* __restrict__ p, const float* __restrict__ q,
                                                             const int64_t* __restrict__ drafts,
                                                             const float* __restrict__ u_acc,
                                                             const float* __restrict__ u_draw, int* __restrict__ n_acc,
                                                             int64_t* __restrict__ out, int k, int V) {
  pdl_trigger();
  pdl_wait();
  __shared__ float scan[kThreads];
  __shared__ int accepted;
  const int b = blockIdx.x;
  const float* pb = p + static_cast<size_t>(b) * (k + 1) * V;
  const float* qb = q + static_cast<size_t>(b) * k * V;
  const int64_t* xb = drafts + static_cast<size_t>(b) * k;
  int64_t* ob = out + static_cast<size_t>(b) * (k + 1);
  if (threadIdx.x == 0) {
    int j = 0;
    for (; j < k; ++j) {
      const int64_t x = xb[j];
      const float px = pb[static_cast<size_t>(j) * V + x], qx = qb[static_cast<size_t>(j) * V + x];
      // accept when u < p/q, i.e. u * q < p (q > 0 for a drawn token)
      if (!(u_acc[b * k + j] * qx < px)) break;
      ob[j] = x;
    }
    accepted = j;
  }
  __syncthreads();
  const int j = accepted;
  int tok;
  if (j < k) {
    const float* pj = pb + static_cast<size_t>(j) * V;
    const float* qj = qb + static_cast<size_t>(j) * V;
    tok = draw(V, u_draw[b], [&](int i) { return fmaxf(pj[i] - qj[i], 0.f); }, scan, nullptr);
    if (tok < 0) {  // p == q on the support: the residual is empty, sample p itself
      tok = draw(V, u_draw[b], [&](int i) { return pj[i]; }, scan, nullptr);
    }
  } else {
    const float* pk = pb + static_cast<size_t>(k) * V;
    tok = draw(V, u_draw[b], [&](int i) { return pk[i]; }, scan, nullptr);
  }
  if (threadIdx.x == 0) {
    ob[j] = tok < 0 ? 0 : tok;
    for (int i = j + 1; i <= k; ++i) ob[i] = 0;
    n_acc[b] = j;
  }
}

// ---- fused log-softmax + top-k (draft-tree expansion) -----------------------------------------------------------
// One CTA per row of logits [R, V] (fp32): max and sum of exponentials, then the k largest logits (ties: lower
// index) from per-thread lists merged by warps and then by warp 0. Outputs log-probabilities
// max(logit - logsumexp, floor) and indices mapped to target ids (index + d2t[index] when a draft vocabulary map is
// given). Replaces log_softmax + clamp + topk + gather in every expansion step of the dynamic tree.
constexpr int kTopThreads = 512;
constexpr int kMaxTopK = 16;

struct Cand {
  float v;
  int i;
};

__device__ __forceinline__ bool better(const Cand& a, const Cand& b) { return a.v > b.v || (a.v == b.v && a.i < b.i); }

// Sorted (descending) candidate list of K entries kept in registers: insertion bubbles the new candidate down with
// unrolled compare-and-swaps, and popping the head shifts the list (no dynamic indexing, so no local memory).
template <int K>
__device__ __forceinline__ void list_insert(Cand (&m)[K], Cand c) {
  if (!better(c, m[K - 1])) return;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (better(c, m[j])) {
      const Cand t = m[j];
      m[j] = c;
      c = t;
    }
  }
}

template <int K>
__device__ __forceinline__ void list_pop(Cand (&m)[K]) {
#pragma unroll
  for (int j = 0; j < K - 1; ++j) m[j] = m[j + 1];
  m[K - 1] = Cand{-INFINITY, 0x7fffffff};
}

// k rounds of the best head among the 32 lanes' sorted lists; lane 0 receives the k winners in order
template <int K>
__device__ __forceinline__ void warp_merge(Cand (&m)[K], int k, Cand* out) {
  for (int r = 0; r < k; ++r) {
    const Cand c = m[0];
    Cand best = c;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const Cand o{__shfl_xor_sync(0xffffffffu, best.v, off), __shfl_xor_sync(0xffffffffu, best.i, off)};
      if (better(o, best)) best = o;
    }
    if (c.i == best.i && c.v == best.v) list_pop(m);
    if ((threadIdx.x & 31) == 0) out[r] = best;
  }
}

template <int K>
__global__ void __launch_bounds__(kTopThreads) topk_logp_kernel(const float* __restrict__ logits,
                                                               const int64_t* __restrict__ d2t, float* __restrict__ vals,
                                                               int64_t* __restrict__ ids, int V, int k, float floor_v) {
  pdl_trigger();
  pdl_wait();
  const float* row = logits + static_cast<size_t>(blockIdx.x) * V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float red[32];
  __shared__ Cand wl[kTopThreads / 32][K];
  // one pass: the thread's running max with a rescaled sum of exponentials, and its own top-K
  Cand mine[K];
#pragma unroll
  for (int j = 0; j < K; ++j) mine[j] = Cand{-INFINITY, 0x7fffffff};
  float mx = -INFINITY, se = 0.f;
  for (int i = tid; i < V; i += kTopThreads) {
    const float x = __ldg(row + i);
    if (x > mx) {
      se = se * __expf(mx - x) + 1.f;
      mx = x;
    } else if (x != -INFINITY) {  // a -inf logit adds nothing (and exp(-inf - -inf) would be NaN)
      se += __expf(x - mx);
    }
    list_insert(mine, Cand{x, i});
  }
  // block log-sum-exp: warp-level then block-level (max, rescaled sum)
  float wmx = warp_max(mx);
  float wse = warp_sum(mx == -INFINITY ? 0.f : se * __expf(mx - wmx));
  if (lane == 0) {
    red[warp] = wmx;
    red[16 + warp] = wse;
  }
  warp_merge(mine, k, wl[warp]);
  __syncthreads();
  if (warp == 0) {
    const float m_l = lane < kTopThreads / 32 ? red[lane] : -INFINITY;
    const float bmx = warp_max(m_l);
    const float s_l = lane < kTopThreads / 32 && m_l != -INFINITY ? red[16 + lane] * __expf(m_l - bmx) : 0.f;
    const float lse = bmx + __logf(warp_sum(s_l));
    // lane l holds warp l's sorted list (16 lists of k)
    Cand lst[K];
#pragma unroll
    for (int j = 0; j < K; ++j) lst[j] = (lane < kTopThreads / 32 && j < k) ? wl[lane][j] : Cand{-INFINITY, 0x7fffffff};
    Cand win{-INFINITY, 0};
    for (int r = 0; r < k; ++r) {
      const Cand c = lst[0];
      Cand best = c;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const Cand o{__shfl_xor_sync(0xffffffffu, best.v, off), __shfl_xor_sync(0xffffffffu, best.i, off)};
        if (better(o, best)) best = o;
      }
      if (c.i == best.i && c.v == best.v) list_pop(lst);
      if (lane == r) win = best;  // lane r keeps the r-th winner
    }
    if (lane < k) {  // all k id-map loads in flight at once
      const size_t o = static_cast<size_t>(blockIdx.x) * k + lane;
      vals[o] = fmaxf(win.v - lse, floor_v);
      ids[o] = d2t != nullptr ? win.i + d2t[win.i] : win.i;
    }
  }
}

// ---- split variant: rows too few to fill the GPU ------------------------------------------------------------------
// Grid (rows, S): CTA (r, s) scans chunk s of row r for its max, rescaled sum of exponentials and top-k, and writes
// them to the workspace; the last CTA of a row to finish (a per-row arrival counter, reset by that CTA for the next
// launch) merges the S partial results into the row's log-sum-exp and top-k. Same outputs as topk_logp_kernel: the
// candidates are compared by (value, index) everywhere, so the merged top-k is the row's top-k.
constexpr int kSplitThreads = 256;

template <int K>
__global__ void __launch_bounds__(kSplitThreads) topk_logp_split_kernel(
    const float* __restrict__ logits, const int64_t* __restrict__ d2t, float* __restrict__ vals,
    int64_t* __restrict__ ids, Cand* __restrict__ ws_cands, float2* __restrict__ ws_stats, int* __restrict__ counters,
    int V, int k, int chunk, float floor_v) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x, s = blockIdx.y, S = gridDim.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kWarps = kSplitThreads / 32;
  __shared__ float red[2 * kWarps];
  __shared__ Cand wl[kWarps][K];
  __shared__ int is_last;
  const float* row = logits + static_cast<size_t>(r) * V;
  const int lo = s * chunk, hi = min(V, lo + chunk);
  Cand mine[K];
#pragma unroll
  for (int j = 0; j < K; ++j) mine[j] = Cand{-INFINITY, 0x7fffffff};
  float mx = -INFINITY, se = 0.f;
  for (int i = lo + tid; i < hi; i += kSplitThreads) {
    const float x = __ldg(row + i);
    if (x > mx) {
      se = se * __expf(mx - x) + 1.f;
      mx = x;
    } else if (x != -INFINITY) {
      se += __expf(x - mx);
    }
    list_insert(mine, Cand{x, i});
  }
  float wmx = warp_max(mx);
  float wse = warp_sum(mx == -INFINITY ? 0.f : se * __expf(mx - wmx));
  if (lane == 0) {
    red[warp] = wmx;
    red[kWarps + warp] = wse;
  }
  warp_merge(mine, k, wl[warp]);
  __syncthreads();
  Cand* out_c = ws_cands + (static_cast<size_t>(r) * S + s) * K;
  if (warp == 0) {
    const float m_l = lane < kWarps ? red[lane] : -INFINITY;
    const float bmx = warp_max(m_l);
    const float s_l = lane < kWarps && m_l != -INFINITY ? red[kWarps + lane] * __expf(m_l - bmx) : 0.f;
    const float bse = warp_sum(s_l);
    Cand lst[K];
#pragma unroll
    for (int j = 0; j < K; ++j) lst[j] = (lane < kWarps && j < k) ? wl[lane][j] : Cand{-INFINITY, 0x7fffffff};
    warp_merge(lst, k, out_c);
    if (lane == 0) ws_stats[static_cast<size_t>(r) * S + s] = make_float2(bmx, bse);
    __threadfence();
    __syncwarp();
    if (lane == 0) {
      const int prev = atomicAdd(&counters[r], 1);
      is_last = prev == S - 1;
      if (is_last) counters[r] = 0;  // ready for the next launch
    }
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // ---- merge the row's S partial results ----
  const Cand* row_c = ws_cands + static_cast<size_t>(r) * S * K;
  const float2* row_s = ws_stats + static_cast<size_t>(r) * S;
#pragma unroll
  for (int j = 0; j < K; ++j) mine[j] = Cand{-INFINITY, 0x7fffffff};
  // the other CTAs' results are read from L2 (ld.global.cg): this SM's L1 may not have seen their stores
  for (int i = tid; i < S * k; i += kSplitThreads) {
    const Cand* src = row_c + (i / k) * K + i % k;
    list_insert(mine, Cand{__ldcg(&src->v), __ldcg(&src->i)});
  }
  float m2 = -INFINITY;
  for (int i = tid; i < S; i += kSplitThreads) m2 = fmaxf(m2, __ldcg(&row_s[i].x));
  m2 = warp_max(m2);
  if (lane == 0) red[warp] = m2;
  __syncthreads();
  float rmx = lane < kWarps ? red[lane] : -INFINITY;
  rmx = warp_max(rmx);
  float s2 = 0.f;
  for (int i = tid; i < S; i += kSplitThreads) {
    const float2 st = __ldcg(&row_s[i]);
    if (st.x != -INFINITY) s2 += st.y * __expf(st.x - rmx);
  }
  s2 = warp_sum(s2);
  __syncthreads();
  if (lane == 0) red[kWarps + warp] = s2;
  warp_merge(mine, k, wl[warp]);
  __syncthreads();
  if (warp == 0) {
    const float lse = rmx + __logf(warp_sum(lane < kWarps ? red[kWarps + lane] : 0.f));
    Cand lst[K];
#pragma unroll
    for (int j = 0; j < K; ++j) lst[j] = (lane < kWarps && j < k) ? wl[lane][j] : Cand{-INFINITY, 0x7fffffff};
    Cand win{-INFINITY, 0};
    for (int q = 0; q < k; ++q) {
      const Cand c = lst[0];
      Cand best = c;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const Cand o{__shfl_xor_sync(0xffffffffu, best.v, off), __shfl_xor_sync(0xffffffffu, best.i, off)};
        if (better(o, best)) best = o;
      }
      if (c.i == best.i && c.v == best.v) list_pop(lst);
      if (lane == q) win = best;
    }
    if (lane < k) {
      const size_t o = static_cast<size_t>(r) * k + lane;
      vals[o] = fmaxf(win.v - lse, floor_v);
      ids[o] = d2t != nullptr ? win.i + d2t[win.i] : win.i;
    }
  }
}

}  // namespace

// Chunks per row for the split top-k: enough CTAs for two per SM, each chunk at least 512 logits, at most 64.
int topk_splits(int rows, int V, int num_sms) {
  if (rows <= 0 || rows >= num_sms) return 1;
  const int want = (2 * num_sms + rows - 1) / rows;
  return std::max(1, std::min(std::min(want, 64), V / 512));
}

size_t topk_workspace_bytes(int rows, int splits) {
  return static_cast<size_t>(rows) * splits * (kMaxTopK * sizeof(Cand) + sizeof(float2));
}

int launch_sample(const float* probs, const float* u, int64_t* out, int rows, int V, cudaStream_t stream) {
  if (rows == 0) return 0;
  launch_pdl(sample_kernel, dim3(rows), dim3(kThreads), 0, stream, probs, u, out, V);
  return 0;
}

int launch_rejection(const float* p, const float* q, const int64_t* drafts, const float* u_acc, const float* u_draw,
                     int* n_acc, int64_t* out, int B, int k, int V, cudaStream_t stream) {
  if (B == 0) return 0;
  launch_pdl(rejection_kernel, dim3(B), dim3(kThreads), 0, stream, p, q, drafts, u_acc, u_draw, n_acc, out, k, V);
  return 0;
}

int launch_topk_logp(const float* logits, const int64_t* d2t, float* vals, int64_t* ids, int rows, int V, int k,
                     float floor_v, cudaStream_t stream, int splits, void* workspace, int* counters) {
  if (k < 1 || k > kMaxTopK || k > V) return -1;
  if (rows == 0) return 0;
  if (splits > 1) {
    if (workspace == nullptr || counters == nullptr) return -2;
    Cand* wc = static_cast<Cand*>(workspace);
    float2* wsst = reinterpret_cast<float2*>(wc + static_cast<size_t>(rows) * splits * kMaxTopK);
    const int chunk = (V + splits - 1) / splits;
    const dim3 grid(rows, splits);
    if (k <= 4) {
      launch_pdl(topk_logp_split_kernel<4>, grid, dim3(kSplitThreads), 0, stream, logits, d2t, vals, ids, wc, wsst,
                 counters, V, k, chunk, floor_v);
    } else if (k <= 8) {
      launch_pdl(topk_logp_split_kernel<8>, grid, dim3(kSplitThreads), 0, stream, logits, d2t, vals, ids, wc, wsst,
                 counters, V, k, chunk, floor_v);
    } else {
      launch_pdl(topk_logp_split_kernel<16>, grid, dim3(kSplitThreads), 0, stream, logits, d2t, vals, ids, wc, wsst,
                 counters, V, k, chunk, floor_v);
    }
    return 0;
  }
  if (k <= 4) {
    launch_pdl(topk_logp_kernel<4>, dim3(rows), dim3(kTopThreads), 0, stream, logits, d2t, vals, ids, V, k, floor_v);
  } else if (k <= 8) {
    launch_pdl(topk_logp_kernel<8>, dim3(rows), dim3(kTopThreads), 0, stream, logits, d2t, vals, ids, V, k, floor_v);
  } else {
    launch_pdl(topk_logp_kernel<16>, dim3(rows), dim3(kTopThreads), 0, stream, logits, d2t, vals, ids, V, k,
               floor_v);
  }
  return 0;
}

}  // namespace ecz
