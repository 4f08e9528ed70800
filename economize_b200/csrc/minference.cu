// MInference vertical-slash pattern -> per-KV-head key bitmap (economize attention/_minference_kernels.py:13-66
// converts the same pattern into block ranges and columns for its sparse prefill kernel; here the pattern becomes the
// keep bitmap that the tcgen05 attention kernel ANDs into its visibility rule and uses to skip hidden key chunks).
//
// For one query chunk of t queries starting at position `base`, key j is kept by
//   * a vertical column: j is one of the `nv` column indices of its (row, KV head);
//   * a slash diagonal of offset o (o = query position - key position): j lies in [base - o, base + t - o), the keys
//     the diagonal crosses for the chunk's queries;
// and only keys below `limit` (the chunk's first position: earlier keys only) are kept.
//
// One CTA of 256 threads per (row, KV head). The bitmap of that head (S / 32 words) is built in shared memory: columns
// are set with shared-memory atomicOr, then every thread owns words and ORs in the bits of every diagonal's range
// (offsets are read through L1; ns is at most a few thousand), and the words are written out with the `limit` cut.
#include "common.cuh"
#include "launchers.h"

namespace ecz {

constexpr int kVsMaxWords = 8192;  // S <= 262144 keys per head: 32 KB of shared memory

__global__ void __launch_bounds__(256) vs_keep_kernel(const int64_t* __restrict__ cols, int nv,
                                                      const int64_t* __restrict__ offsets, int ns, int base, int t,
                                                      int limit, int words, uint32_t* __restrict__ keep) {
  extern __shared__ uint32_t vs_words[];
  pdl_trigger();
  pdl_wait();
  const int bh = blockIdx.x;
  for (int w = threadIdx.x; w < words; w += blockDim.x) vs_words[w] = 0u;
  __syncthreads();
  const int S = words * 32;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const int64_t j = cols[static_cast<size_t>(bh) * nv + i];
    if (j >= 0 && j < S) atomicOr(&vs_words[j >> 5], 1u << (j & 31));
  }
  __syncthreads();
  const int64_t* off = offsets + static_cast<size_t>(bh) * ns;
  for (int w = threadIdx.x; w < words; w += blockDim.x) {
    const int lo_w = w * 32, hi_w = lo_w + 32;
    uint32_t bits = vs_words[w];
    for (int k = 0; k < ns; ++k) {
      const int64_t o = __ldg(off + k);
      const int64_t lo = static_cast<int64_t>(base) - o, hi = lo + t;
      if (hi <= lo_w || lo >= hi_w) continue;
      const int a = static_cast<int>(lo > lo_w ? lo - lo_w : 0);
      const int b = static_cast<int>(hi < hi_w ? hi - lo_w : 32);
      const uint32_t upto_b = b == 32 ? 0xffffffffu : ((1u << b) - 1u);
      bits |= upto_b & ~((1u << a) - 1u);
    }
    // keys at or past `limit` are not kept
    if (hi_w > limit) bits &= limit <= lo_w ? 0u : ((1u << (limit - lo_w)) - 1u);
    keep[static_cast<size_t>(bh) * words + w] = bits;
  }
}

int launch_vs_keep(const int64_t* cols, int nv, const int64_t* offsets, int ns, int base, int t, int limit, int rows,
                   int S, uint32_t* keep, cudaStream_t stream) {
  if (S % 32 != 0 || S / 32 > kVsMaxWords || rows < 1 || nv < 0 || ns < 0 || t < 0) return -1;
  const int words = S / 32;
  const cudaError_t err = launch_pdl(vs_keep_kernel, dim3(rows), dim3(256), static_cast<size_t>(words) * 4, stream,
                                     cols, nv, offsets, ns, base, t, limit, words, keep);
  return err == cudaSuccess ? 0 : -3;
}

}  // namespace ecz
