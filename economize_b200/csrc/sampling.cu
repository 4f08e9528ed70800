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

__global__ void __launch_bounds__(kTopThreads) topk_logp_kernel(const float* __restrict__ logits,
                                                               const int64_t* __restrict__ d2t, float* __restrict__ vals,
                                                               int64_t* __restrict__ ids, int V, int k, float floor_v) {
  pdl_trigger();
  pdl_wait();
  const float* row = logits + static_cast<size_t>(blockIdx.x) * V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float red[32];
  __shared__ Cand wl[kTopThreads / 32][kMaxTopK];
  // max
  float mx = -INFINITY;
  for (int i = tid; i < V; i += kTopThreads) mx = fmaxf(mx, row[i]);
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (warp == 0) {
    float t = lane < kTopThreads / 32 ? red[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  // sum of exponentials and the thread's own top-k (sorted, descending)
  Cand mine[kMaxTopK];
  for (int j = 0; j < k; ++j) mine[j] = {-INFINITY, 0x7fffffff};
  float se = 0.f;
  for (int i = tid; i < V; i += kTopThreads) {
    const float x = row[i];
    se += __expf(x - mx);
    Cand c{x, i};
    if (better(c, mine[k - 1])) {
      int j = k - 1;
      while (j > 0 && better(c, mine[j - 1])) {
        mine[j] = mine[j - 1];
        --j;
      }
      mine[j] = c;
    }
  }
  se = warp_sum(se);
  if (lane == 0) red[warp] = se;
  // warp merge: k rounds of the best head among the 32 lanes' lists
  int head = 0;
  for (int r = 0; r < k; ++r) {
    Cand c = head < k ? mine[head] : Cand{-INFINITY, 0x7fffffff};
    Cand best = c;
    for (int off = 16; off > 0; off >>= 1) {
      Cand o{__shfl_xor_sync(0xffffffffu, best.v, off), __shfl_xor_sync(0xffffffffu, best.i, off)};
      if (better(o, best)) best = o;
    }
    if (head < k && c.i == best.i && c.v == best.v) ++head;
    if (lane == 0) wl[warp][r] = best;
  }
  __syncthreads();
  if (warp == 0) {
    float tot = lane < kTopThreads / 32 ? red[lane] : 0.f;
    tot = warp_sum(tot);
    const float lse = mx + __logf(tot);
    int h = 0;  // lane l merges list l (16 lists of k)
    for (int r = 0; r < k; ++r) {
      Cand c = (lane < kTopThreads / 32 && h < k) ? wl[lane][h] : Cand{-INFINITY, 0x7fffffff};
      Cand best = c;
      for (int off = 16; off > 0; off >>= 1) {
        Cand o{__shfl_xor_sync(0xffffffffu, best.v, off), __shfl_xor_sync(0xffffffffu, best.i, off)};
        if (better(o, best)) best = o;
      }
      if (lane < kTopThreads / 32 && h < k && c.i == best.i && c.v == best.v) ++h;
      if (lane == 0) {
        const size_t o = static_cast<size_t>(blockIdx.x) * k + r;
        vals[o] = fmaxf(best.v - lse, floor_v);
        ids[o] = d2t != nullptr ? best.i + d2t[best.i] : best.i;
      }
    }
  }
}

}  // namespace

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
                     float floor_v, cudaStream_t stream) {
  if (k < 1 || k > kMaxTopK || k > V) return -1;
  if (rows == 0) return 0;
  launch_pdl(topk_logp_kernel, dim3(rows), dim3(kTopThreads), 0, stream, logits, d2t, vals, ids, V, k, floor_v);
  return 0;
}

}  // namespace ecz
