// Block-scaled fp8 GEMM on tcgen05 (kind::f8f6f4): Y[M, N] = (sx * X8)[M, K] . (sw * W8)[N, K]^T with e4m3
// operands, one fp32 weight scale per 128 x 128 block and one activation scale per token and 128-wide K block (the
// DeepSeek-V3 / "1x128 activation, 128x128 weight" format; economize reaches fp8 only through torch's row-wise
// _scaled_mm, src/economize/techniques/quant/backends.py:1-40).
//
// Because the scales change every 128 K-elements, the tensor cores accumulate one K-block at a time into one of two
// TMEM buffers and four epilogue warps promote it: acc[j] += D[j] * sw[kb] * sx[token j, kb] in registers, while
// the tensor cores already run the next K-block into the other buffer.
//
//   warp 0      TMA: weight tile [128 x 128 B], activation tile [BN x 128 B], the block's activation scales
//   warp 1      UMMA: 4 x kind::f8f6f4 (K = 32) per K-block into TMEM buffer kb % 2
//   warps 2-5   promotion (TMEM lane = output feature), then the epilogue (bf16 Y or fp32 split-K partials)
//
// act_quant_kernel quantises bf16 activations: per token and K-block, scale = max|x| / 448, codes = e4m3(x / scale).
#include <algorithm>

#include <cuda_fp8.h>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 128;  // fp8 elements per stage = one scale block = one 128-byte swizzle row
constexpr int kABytes = kBM * kBK;
constexpr int kThreads = 192;

template <int BN>
struct Fp8Cfg {
  static constexpr int kOcc = BN <= 64 ? 2 : 1;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kScaleBytes = ((BN * 4 + 127) / 128) * 128;
  static constexpr int kStageBytes = kABytes + kBBytes + kScaleBytes;
  static constexpr int kStages = std::min(8, ((kOcc == 1 ? 200 : 100) * 1024) / kStageBytes);
  static constexpr int kTmemCols = 2 * (BN < 32 ? 32 : BN);  // two accumulator buffers
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
  return (1u << 4)                                 // D format: f32
         | (0u << 7)                               // A format: e4m3
         | (0u << 10)                              // B format: e4m3
         | (static_cast<uint32_t>(n >> 3) << 17)   // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);  // M >> 4
}

__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int BN>
__global__ void __launch_bounds__(kThreads, Fp8Cfg<BN>::kOcc)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_sx, const float* __restrict__ sw, bf16* __restrict__ y,
                    float* __restrict__ ws, int M, int N, int K, int kb_per_split, unsigned* status) {
  using Cfg = Fp8Cfg<BN>;
  constexpr int S = Cfg::kStages;
  constexpr int kCols = BN < 32 ? 32 : BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = smem + S * kABytes;
  float* s_tiles = reinterpret_cast<float*>(smem + S * (kABytes + Cfg::kBBytes));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;     // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBM, m0 = blockIdx.y * BN, split = blockIdx.z;
  const int total_kb = K / kBK;
  const int kb0 = split * kb_per_split;
  const int nkb = max(0, min(kb_per_split, total_kb - kb0));
  constexpr uint32_t kStageTx = kABytes + Cfg::kBBytes + BN * 4;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);  // the MMA commit and the four promotion warps (done with the stage's scales)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_sx);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  float acc[kCols];
#pragma unroll
  for (int j = 0; j < kCols; ++j) acc[j] = 0.f;

  if (nkb > 0 && warp == 0 && lane == 0) {
    const int pre = nkb < S ? nkb : S;
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(&full[kb], kStageTx);
      tma_load_2d(a_tiles + kb * kABytes, &tm_w, &full[kb], (kb0 + kb) * kBK, n0);
    }
    pdl_wait();
    for (int kb = 0; kb < pre; ++kb) {
      tma_load_2d(b_tiles + kb * Cfg::kBBytes, &tm_x, &full[kb], (kb0 + kb) * kBK, m0);
      tma_load_2d(reinterpret_cast<uint8_t*>(s_tiles) + kb * Cfg::kScaleBytes, &tm_sx, &full[kb], m0, kb0 + kb);
    }
    for (int kb = pre; kb < nkb; ++kb) {
      const int s = kb % S;
      if (!mbar_wait(&empty[s], ((kb / S) & 1u) ^ 1u, status, kStatusWaitEmpty, abort_flag)) break;
      mbar_arrive_expect_tx(&full[s], kStageTx);
      const int k = (kb0 + kb) * kBK;
      tma_load_2d(a_tiles + s * kABytes, &tm_w, &full[s], k, n0);
      tma_load_2d(b_tiles + s * Cfg::kBBytes, &tm_x, &full[s], k, m0);
      tma_load_2d(reinterpret_cast<uint8_t*>(s_tiles) + s * Cfg::kScaleBytes, &tm_sx, &full[s], m0, kb0 + kb);
    }
  } else if (nkb > 0 && warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_e4m3_f32(kBM, BN);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S, b = kb & 1;
      if (!mbar_wait(&full[s], (kb / S) & 1u, status, kStatusWaitFull, abort_flag)) break;
      if (!mbar_wait(&acc_empty[b], ((kb >> 1) & 1u) ^ 1u, status, kStatusWaitEmpty, abort_flag)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(a_tiles + s * kABytes);
      const uint32_t b_addr = smem_u32(b_tiles + s * Cfg::kBBytes);
#pragma unroll
      for (int kk = 0; kk < kBK / 32; ++kk) {
        umma_f8(tmem + b * kCols, desc_kmajor_sw128(a_addr + kk * 32), desc_kmajor_sw128(b_addr + kk * 32), idesc,
                kk != 0 ? 1u : 0u);
      }
      umma_commit(&acc_full[b]);
      umma_commit(&empty[s]);
    }
  } else if (nkb > 0 && warp >= 2) {
    // ---- promotion: warp w reads TMEM lanes 32 (w % 4) .. (output features) ----
    const int quarter = warp & 3;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int n_blk = n0 / kBM;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S, b = kb & 1;
      if (!mbar_wait(&acc_full[b], (kb >> 1) & 1u, status, kStatusWaitAccum, abort_flag)) break;
      // the stage's activation scales were written by TMA: acquire them through the stage's own barrier
      if (!mbar_wait(&full[s], (kb / S) & 1u, status, kStatusWaitFull, abort_flag)) break;
      tc_fence_after();
      const float wscale = sw[static_cast<size_t>(n_blk) * total_kb + kb0 + kb];
      const float* sx = s_tiles + s * (Cfg::kScaleBytes / 4);
#pragma unroll
      for (int c = 0; c < kCols; c += 16) {
        float v[16];
        tmem_ld16(lane_base + b * kCols + c, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[c + j] = fmaf(v[j], wscale * sx[c + j], acc[c + j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc_empty[b]);
        mbar_arrive(&empty[s]);
      }
    }
  }
  __syncwarp();
  pdl_wait();
  __syncthreads();
  const bool ok = nkb > 0 && !*abort_flag;
  if (ok && warp >= 2) {
    const int n = n0 + (warp & 3) * 32 + lane;
    if (n < N) {
#pragma unroll
      for (int j = 0; j < kCols; ++j) {
        const int m = m0 + j;
        if (j < BN && m < M) {
          if (ws == nullptr) y[static_cast<size_t>(m) * N + n] = __float2bfloat16(acc[j]);
          else ws[(static_cast<size_t>(split) * M + m) * N + n] = acc[j];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

__global__ void __launch_bounds__(256) fp8_reduce_kernel(const float* __restrict__ ws, bf16* __restrict__ y,
                                                         long total, int splits) {
  pdl_trigger();
  pdl_wait();
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    float a = ws[i];
    for (int s = 1; s < splits; ++s) a += ws[s * total + i];
    y[i] = __float2bfloat16(a);
  }
}

// one warp per (token, K-block): 128 values, 4 per lane
__global__ void __launch_bounds__(256) act_quant_kernel(const bf16* __restrict__ x, uint8_t* __restrict__ q,
                                                        float* __restrict__ sx, int M, int K, int sx_stride) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int blocks = K / kBK;
  if (warp >= M * blocks) return;
  const int m = warp / blocks, kb = warp % blocks;
  const size_t off = static_cast<size_t>(m) * K + kb * kBK + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(x + off);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  const float amax = warp_max(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y))));
  const float scale = amax > 0.f ? amax / 448.f : 1.f;
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(__fdiv_rn(a.x, scale), __fdiv_rn(a.y, scale)),
                                                           __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(__fdiv_rn(b.x, scale), __fdiv_rn(b.y, scale)),
                                                           __NV_SATFINITE, __NV_E4M3);
  *reinterpret_cast<uint32_t*>(q + off) = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  if (lane == 0) sx[static_cast<size_t>(kb) * sx_stride + m] = scale;
}

template <int BN>
int run_fp8(const CUtensorMap& tm_w, const CUtensorMap& tm_x, const CUtensorMap& tm_sx, const float* sw, void* y,
            float* ws, int M, int N, int K, int splits, unsigned* status, cudaStream_t stream) {
  using Cfg = Fp8Cfg<BN>;
  set_max_smem(gemm_fp8_kernel<BN>, Cfg::kSmem);
  const int total_kb = K / kBK;
  const int kbps = (total_kb + splits - 1) / splits;
  splits = (total_kb + kbps - 1) / kbps;
  dim3 grid((N + kBM - 1) / kBM, (M + BN - 1) / BN, splits);
  launch_pdl(gemm_fp8_kernel<BN>, grid, dim3(kThreads), Cfg::kSmem, stream, tm_w, tm_x, tm_sx, sw,
             static_cast<bf16*>(y), splits > 1 ? ws : nullptr, M, N, K, kbps, status);
  if (splits > 1) {
    const long total = static_cast<long>(M) * N;
    const int blocks = static_cast<int>(std::min<long>((total + 255) / 256, 148L * 8));
    launch_pdl(fp8_reduce_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, stream, static_cast<const float*>(ws),
               static_cast<bf16*>(y), total, splits);
  }
  return 0;
}

}  // namespace

int fp8_block_n(int M) { return M <= 32 ? 32 : (M <= 64 ? 64 : 128); }

int launch_act_quant_fp8(const void* x, void* q, float* sx, int M, int K, int sx_stride, cudaStream_t stream) {
  if (K % kBK != 0 || sx_stride < M) return -1;
  const long warps = static_cast<long>(M) * (K / kBK);
  launch_pdl(act_quant_kernel, dim3(static_cast<unsigned>((warps * 32 + 255) / 256)), dim3(256), 0, stream,
             static_cast<const bf16*>(x), static_cast<uint8_t*>(q), sx, M, K, sx_stride);
  return 0;
}

int launch_gemm_fp8(const CUtensorMap* tm_w, const CUtensorMap* tm_x, const CUtensorMap* tm_sx, const float* sw,
                    void* y, float* ws, int M, int N, int K, int splits, unsigned* status, cudaStream_t stream) {
  if (K % kBK != 0 || N % kBM != 0 || splits < 1) return -1;
  switch (fp8_block_n(M)) {
    case 32: return run_fp8<32>(*tm_w, *tm_x, *tm_sx, sw, y, ws, M, N, K, splits, status, stream);
    case 64: return run_fp8<64>(*tm_w, *tm_x, *tm_sx, sw, y, ws, M, N, K, splits, status, stream);
    default: return run_fp8<128>(*tm_w, *tm_x, *tm_sx, sw, y, ws, M, N, K, splits, status, stream);
  }
}

}  // namespace ecz
