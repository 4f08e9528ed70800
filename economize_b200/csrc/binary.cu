// Binary (sign) matrix products for LittleBit factors: out[m, n] = sum_k s[n, k] x[m, k] with s in {+1, -1} packed
// 32 per 32-bit word along k (bit set = -1). One warp per output row n: lane j reads x[m, 32 w + j] (coalesced) and
// bit j of the row's word w (a broadcast), accumulates +-x, and the warp sums its lanes at the end.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

template <int MT>
__global__ void __launch_bounds__(256) sign_matvec_kernel(const uint32_t* __restrict__ bits, const float* __restrict__ x,
                                                          float* __restrict__ out, int M, int N, int K, int words) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (n >= N) return;
  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.f;
  const uint32_t* row = bits + static_cast<long>(n) * words;
  for (int w = 0; w < words; ++w) {
    const uint32_t word = __ldg(row + w);
    const int k = w * 32 + lane;
    const float sgn = (word >> lane) & 1u ? -1.f : 1.f;
    if (k < K) {
#pragma unroll
      for (int m = 0; m < MT; ++m)
        if (m < M) acc[m] = fmaf(sgn, __ldg(x + static_cast<long>(m) * K + k), acc[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const float s = warp_sum(acc[m]);
    if (lane == 0 && m < M) out[static_cast<long>(m) * N + n] = s;
  }
}

template <int MT>
void run_sign(const uint32_t* bits, const float* x, float* out, int M, int N, int K, cudaStream_t stream) {
  const int words = (K + 31) / 32;
  launch_pdl(sign_matvec_kernel<MT>, dim3((N + 7) / 8), dim3(256), 0, stream, bits, x, out, M, N, K, words);
}

}  // namespace

int launch_sign_matvec(const uint32_t* bits, const float* x, float* out, int M, int N, int K, cudaStream_t stream) {
  if (M < 1 || M > 16 || N < 1 || K < 1) return -1;
  if (M == 1) run_sign<1>(bits, x, out, M, N, K, stream);
  else if (M <= 4) run_sign<4>(bits, x, out, M, N, K, stream);
  else run_sign<16>(bits, x, out, M, N, K, stream);
  return 0;
}

}  // namespace ecz
