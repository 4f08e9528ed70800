// Prompt-lookup drafting on the device: for every row, find an earlier occurrence of the history's last n tokens
// (n from max_n down to min_n, the first n that matches wins) and propose the k tokens that followed it. The
// search runs over every start position in parallel; `earliest` picks the first occurrence, otherwise the last.
// Rows without a match (or proposals running past the history) get -1, which the verifier never accepts.
#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

__global__ void __launch_bounds__(256) ngram_kernel(const int64_t* __restrict__ history, const int* __restrict__ len,
                                                    int64_t* __restrict__ drafts, int cap, int k, int min_n,
                                                    int max_n, int earliest) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  const int64_t* h = history + static_cast<size_t>(b) * cap;
  const int n_hist = min(len[b], cap);
  __shared__ int best;
  __shared__ int found_n;
  if (threadIdx.x == 0) found_n = 0;
  __syncthreads();
  for (int n = max_n; n >= min_n; --n) {
    if (n_hist <= n) continue;
    if (threadIdx.x == 0) best = earliest ? 0x7fffffff : -1;
    __syncthreads();
    // candidate start i: history[i .. i + n) == history[n_hist - n .. n_hist), with i + n < n_hist
    for (int i = threadIdx.x; i + n < n_hist; i += blockDim.x) {
      bool eq = true;
      for (int j = 0; j < n && eq; ++j) eq = h[i + j] == h[n_hist - n + j];
      if (eq) {
        if (earliest) atomicMin(&best, i);
        else atomicMax(&best, i);
      }
    }
    __syncthreads();
    const int hit = best;
    __syncthreads();
    if (hit >= 0 && hit != 0x7fffffff) {
      if (threadIdx.x == 0) { best = hit; found_n = n; }
      __syncthreads();
      break;
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    int64_t tok = -1;
    if (found_n > 0) {
      const int src = best + found_n + j;
      if (src < n_hist) tok = h[src];
    }
    drafts[static_cast<size_t>(b) * k + j] = tok;
  }
}

}  // namespace

int launch_ngram(const int64_t* history, const int* len, int64_t* drafts, int B, int cap, int k, int min_n, int max_n,
                 bool earliest, cudaStream_t stream) {
  if (B == 0) return 0;
  launch_pdl(ngram_kernel, dim3(B), dim3(256), 0, stream, history, len, drafts, cap, k, min_n, max_n,
             earliest ? 1 : 0);
  return 0;
}

}  // namespace ecz
