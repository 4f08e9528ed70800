// Weight-only quantized GEMM on tcgen05: Y[M, N] = X[M, K] . dequant(W)[N, K]^T with bf16 activations and int4,
// int8 or fp8-e4m3 weights carrying one bf16 scale (and for int4 one zero point) per output feature and group of
// `group` consecutive K. This is the W4A16 / W8A16 path of GPTQ, AWQ and round-to-nearest checkpoints (the roles
// of economize's Marlin / Machete / Triton weight-only GEMMs, src/economize/techniques/quant/marlin.py:267-486,
// machete.py:112-222, _triton_gemm_kernels.py:10-56).
//
// Decode is bound by the weight stream, so the kernel keeps the bf16 GEMM's swapped operands (weights on the UMMA M
// side, tokens on N) and inserts a dequantisation stage between TMA and the tensor core:
//
//   warp 0      TMA: packed weight tile [128 x 64 K], this group's scales (and zeros) and the activation tile
//   warps 2-9   half a weight row per thread: unpack, subtract the zero, multiply by the scale (bf16x2 arithmetic,
//               bit-exact with bf16((q - z) * s)), store the 128 x 64 bf16 tile in the 128-byte-swizzled K-major
//               layout tcgen05 reads, fence the generic->async proxy and arrive on the stage's barrier
//   warp 1      UMMA issue (4 x K=16 per stage) from the converted tile and the activation tile
//   warps 2-5   epilogue: TMEM -> bf16 Y; with split K the CTAs of a cluster sum their partials over DSMEM
//
// Packed layouts (written by economize_b200.ops.quant):
//   int4  uint8 [N, K/2]; each 32-bit word holds 8 consecutive k as nibbles in the order k0 k2 k4 k6 k1 k3 k5 k7,
//         so the pair (k_2i, k_2i+1) is (word >> 4i) & 0x000F000F. Values are unsigned codes 0..15.
//   int8  uint8 [N, K]; each word holds 4 consecutive k in the byte order k0 k2 k1 k3, stored as q + 128.
//   fp8   uint8 [N, K] e4m3 codes in natural order.
//   sp24  2:4 sparse bf16 weights (no scales): the kept values [N, K / 2] and their positions [N / 2, K / 4] bytes
//         (per row and 64-wide K-block 8 bytes, 4 bits per group of 4: the two kept positions; rows 2p and 2p + 1
//         share a 16-byte line). The expansion to dense bf16 happens in shared memory, so a decode pass streams 56 %
//         of the dense bytes.
//   mxfp4 / nvfp4  uint8 [N, K/2] FP4 E2M1 codes, k = 2b in the low and 2b + 1 in the high nibble of byte b; the
//         scale group is 32 K (MX) or 16 K (NV), so a stage carries 2 or 4 scale rows and each 8-K chunk picks its
//         group's scale. The stored bf16 scale is the effective one (MX: the E8M0 power of two; NV: the e4m3 group
//         scale times the power-of-two inverse global scale), exact in bf16. (economize's fp4 grids,
//         src/economize/techniques/quant/fp4.py:1-60; Blackwell W4A16: the codes stream at 4.25 / 4.5 bits.)
// scales bf16 [K/group, N]; zeros (int4) bf16 [K/group, N] holding 128 + z, so that (128 + q) - (128 + z) = q - z.
#include <algorithm>

#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kConvBytes = kBM * kBK * 2;  // one bf16 weight tile
constexpr int kDeqWarps = 8;  // two threads per weight row, each converting half of the 64-wide K-block
constexpr int kThreads = 64 + 32 * kDeqWarps;

template <int FMT>
struct WqFmt {
  static constexpr bool kFp4 = FMT == kWqMxfp4 || FMT == kWqNvfp4;
  // int4 / fp4: 32 B of codes per row and K-block; int8/fp8: 64 B; 2:4 sparse: the 32 kept bf16 values (64 B)
  static constexpr int kRawRowBytes = FMT == kWqInt4 || kFp4 ? kBK / 2 : FMT == kWqInt2 ? kBK / 4 : kBK;
  static constexpr int kRawBytes = kBM * kRawRowBytes;
  static constexpr bool kZeros = FMT == kWqInt4 || FMT == kWqInt2;
  // scale rows per K-block: fp4 formats have a scale per 32 (MX) or 16 (NV) K, the others one per >= 64 K
  static constexpr int kScaleRows = FMT == kWqMxfp4 ? kBK / 32 : FMT == kWqNvfp4 ? kBK / 16 : 1;
  // per-stage side data: bf16 scales [kScaleRows][128 rows], or the 2:4 positions (8 B per row)
  static constexpr int kSideBytes = FMT == kWqSp24 ? kBM * 8 : kBM * 2 * kScaleRows;
};

template <int FMT, int BN>
struct WqCfg {
  static constexpr int kOcc = BN <= 64 ? 2 : 1;
  static constexpr int kXBytes = BN * kBK * 2;
  static constexpr int kLoadBytes = kXBytes + WqFmt<FMT>::kRawBytes + WqFmt<FMT>::kSideBytes + kBM * 2;
  static constexpr int kBudget = (kOcc == 1 ? 200 : 100) * 1024;
  // converted-tile ring: three deep for decode tiles (the dequant -> MMA -> release round trip bounds a stage),
  // two for wide token tiles whose activation stages need the room
  static constexpr int kConvStages = BN <= 64 ? 3 : 2;
  static constexpr int kStages = std::min(8, (kBudget - kConvStages * kConvBytes) / kLoadBytes);
  static_assert(kStages >= 2, "the load ring needs two stages");
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  // layout: conv ring | X ring | raw ring | scale ring | zero ring | barriers
  static constexpr int kXOff = kConvStages * kConvBytes;
  static constexpr int kRawOff = kXOff + kStages * kXBytes;
  static constexpr int kScaleOff = kRawOff + kStages * WqFmt<FMT>::kRawBytes;
  static constexpr int kZeroOff = kScaleOff + kStages * WqFmt<FMT>::kSideBytes;
  static constexpr int kBarOff = kZeroOff + kStages * kBM * 2;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static_assert(BN * kBM * 4 <= kBarOff, "the fp32 partial tile must fit the rings");
};

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf2(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }

// 128 + nibble pair as bf16x2 (exact: 128..143 needs 8 significant bits)
__device__ __forceinline__ __nv_bfloat162 nib_pair(uint32_t w, int shift) {
  return bits_bf2(((w >> shift) & 0x000F000Fu) | 0x43004300u);
}

// Dequantise one 8-element chunk (k = 8j .. 8j+7) of a weight row, given the row's packed words, into 4 bf16x2
// words.
template <int FMT>
__device__ __forceinline__ uint4 dequant_chunk(const uint32_t* w, int j, __nv_bfloat162 s2, __nv_bfloat162 z2) {
  uint32_t out[4];
  if constexpr (FMT == kWqInt4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = bf2_bits(__hmul2(__hsub2(nib_pair(w[j], 4 * i), z2), s2));
  } else if constexpr (FMT == kWqInt2) {
    // a word holds 16 codes: bits 2m of the low half = k_2m, of the high half = k_2m+1 (m = 0..7); chunk j is the
    // low (j even) or high (j odd) eight of them
    const uint32_t word = w[j >> 1];
    const int base = (j & 1) * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 q = bits_bf2(((word >> (base + 2 * i)) & 0x00030003u) | 0x43004300u);  // 128 + code
      out[i] = bf2_bits(__hmul2(__hsub2(q, z2), s2));
    }
  } else if constexpr (FMT == kWqInt8) {
    const __nv_bfloat162 c136 = bits_bf2(0x43084308u);  // 136 = 128 + 8
    const __nv_bfloat162 c128 = bits_bf2(0x43004300u);
    const __nv_bfloat162 c16 = bits_bf2(0x41804180u);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int p = 0; p < 2; ++p) {  // pair (k0, k1) in bytes 0 / 2, pair (k2, k3) in bytes 1 / 3
        const uint32_t word = w[2 * j + h];
        const __nv_bfloat162 lo = __hsub2(nib_pair(word, 8 * p), c128);      // low nibble
        const __nv_bfloat162 hi = __hsub2(nib_pair(word, 8 * p + 4), c136);  // high nibble - 8
        const __nv_bfloat162 q = __hfma2(hi, c16, lo);                       // exact: |q| <= 128
        out[2 * h + p] = bf2_bits(__hmul2(q, s2));
      }
    }
  } else if constexpr (FMT == kWqMxfp4 || FMT == kWqNvfp4) {
    // byte i of word j holds k = 8j + 2i (low nibble) and 8j + 2i + 1 (high nibble) as FP4 E2M1 codes
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_fp4x2_storage_t pair = static_cast<__nv_fp4x2_storage_t>((w[j] >> (8 * i)) & 0xFFu);
      const __half2 hv = __half2(__nv_cvt_fp4x2_to_halfraw2(pair, __NV_E2M1));
      const __nv_bfloat162 b = __float22bfloat162_rn(__half22float2(hv));  // exact: E2M1 values fit bf16
      out[i] = bf2_bits(__hmul2(b, s2));
    }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const uint32_t word = w[2 * j + h];
        const __nv_fp8x2_storage_t pair = static_cast<__nv_fp8x2_storage_t>((word >> (16 * p)) & 0xFFFFu);
        const __half2 hv = __half2(__nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3));
        const __nv_bfloat162 b = __float22bfloat162_rn(__half22float2(hv));  // exact: e4m3 values fit bf16
        out[2 * h + p] = bf2_bits(__hmul2(b, s2));
      }
    }
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// 2:4 sparse: chunk j of a row holds groups 2j and 2j + 1 (4 K-positions each); group g keeps values
// w[2g], w[2g + 1] at positions (meta >> 4g) & 3 and (meta >> (4g + 2)) & 3, the other two positions are zero.
__device__ __forceinline__ uint4 expand_sp24(const uint32_t* w, uint64_t meta, int j) {
  uint32_t out[4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int g = 2 * j + h;
    const uint32_t pair = w[g];  // two bf16 values
    const uint32_t m = static_cast<uint32_t>(meta >> (4 * g)) & 0xFu;
    const uint32_t i0 = m & 3u, i1 = (m >> 2) & 3u;
    uint16_t slot[4] = {0, 0, 0, 0};
    slot[i0] = static_cast<uint16_t>(pair & 0xFFFFu);
    slot[i1] = static_cast<uint16_t>(pair >> 16);
    out[2 * h] = slot[0] | (static_cast<uint32_t>(slot[1]) << 16);
    out[2 * h + 1] = slot[2] | (static_cast<uint32_t>(slot[3]) << 16);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

template <int FMT, int BN>
__global__ void __launch_bounds__(kThreads, WqCfg<FMT, BN>::kOcc)
    gemm_wq_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                   const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_x,
                   bf16* __restrict__ y, int M, int N, int K, int group, int kb_per_split, unsigned* status) {
  using Cfg = WqCfg<FMT, BN>;
  using F = WqFmt<FMT>;
  constexpr int S = Cfg::kStages;
  constexpr int kConvStages = Cfg::kConvStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* conv = smem;
  uint8_t* xs = smem + Cfg::kXOff;
  uint8_t* raw = smem + Cfg::kRawOff;
  bf16* scales = reinterpret_cast<bf16*>(smem + Cfg::kScaleOff);
  bf16* zeros = reinterpret_cast<bf16*>(smem + Cfg::kZeroOff);
  float* partial = reinterpret_cast<float*>(smem);  // [BN][128] fp32 after the pipeline drained
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* empty = full + S;
  uint64_t* conv_full = empty + S;
  uint64_t* conv_empty = conv_full + kConvStages;
  uint64_t* accum = conv_empty + kConvStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBM, m0 = blockIdx.y * BN;
  const int splits = static_cast<int>(gridDim.z);
  const uint32_t rank = splits > 1 ? cluster_ctarank() : 0u;
  const int total_kb = K / kBK;
  const int kb0 = static_cast<int>(blockIdx.z) * kb_per_split;
  const int nkb = max(0, min(kb_per_split, total_kb - kb0));
  constexpr uint32_t kStageTx = Cfg::kXBytes + F::kRawBytes + F::kSideBytes + (F::kZeros ? kBM * 2 : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int c = 0; c < kConvStages; ++c) {
      mbar_init(&conv_full[c], kDeqWarps);  // one arrival per dequantising warp
      mbar_init(&conv_empty[c], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_s);
    if (F::kZeros) tma_prefetch_desc(&tm_z);
    tma_prefetch_desc(&tm_x);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (nkb > 0 && warp == 0 && lane == 0) {
    // ---- TMA producer: weights and their scales first (independent of the previous kernel), then activations ----
    const int pre = nkb < S ? nkb : S;
    auto load_w = [&](int s, int kb) {
      const int k = (kb0 + kb) * kBK;
      if constexpr (FMT == kWqSp24) {
        tma_load_2d(raw + s * F::kRawBytes, &tm_w, &full[s], k / 2, n0);  // bf16 values [N, K / 2]
        tma_load_2d(reinterpret_cast<uint8_t*>(scales) + s * F::kSideBytes, &tm_s, &full[s], (k / kBK) * 16,
                    n0 / 2);  // positions [N / 2, K / 4] bytes: a row pair's 16 B per K-block
        return;
      }
      tma_load_2d(raw + s * F::kRawBytes, &tm_w, &full[s], k * F::kRawRowBytes / kBK, n0);
      // fp4: the kScaleRows scale rows of this K-block (group = kBK / kScaleRows); else the one row k / group
      tma_load_2d(reinterpret_cast<uint8_t*>(scales) + s * F::kSideBytes, &tm_s, &full[s], n0,
                  F::kScaleRows > 1 ? k / kBK * F::kScaleRows : k / group);
      if (F::kZeros) tma_load_2d(zeros + s * kBM, &tm_z, &full[s], n0, k / group);
    };
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(&full[kb], kStageTx);
      load_w(kb, kb);
    }
    pdl_wait();
    for (int kb = 0; kb < pre; ++kb) tma_load_2d(xs + kb * Cfg::kXBytes, &tm_x, &full[kb], (kb0 + kb) * kBK, m0);
    for (int kb = pre; kb < nkb; ++kb) {
      const int s = kb % S;
      if (!mbar_wait(&empty[s], ((kb / S) & 1u) ^ 1u, status, kStatusWaitEmpty, abort_flag)) break;
      mbar_arrive_expect_tx(&full[s], kStageTx);
      load_w(s, kb);
      tma_load_2d(xs + s * Cfg::kXBytes, &tm_x, &full[s], (kb0 + kb) * kBK, m0);
    }
  } else if (nkb > 0 && warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S, c = kb % kConvStages;
      if (!mbar_wait(&conv_full[c], (kb / kConvStages) & 1u, status, kStatusWaitFull, abort_flag)) break;
      if (!mbar_wait(&full[s], (kb / S) & 1u, status, kStatusWaitFull, abort_flag)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(conv + c * kConvBytes);
      const uint32_t b_addr = smem_u32(xs + s * Cfg::kXBytes);
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        umma_bf16(tmem, desc_kmajor_sw128(a_addr + kk * 32), desc_kmajor_sw128(b_addr + kk * 32), idesc,
                  (kb | kk) != 0 ? 1u : 0u);
      }
      umma_commit(&empty[s]);
      umma_commit(&conv_empty[c]);
    }
    umma_commit(accum);
  } else if (nkb > 0 && warp >= 2) {
    // ---- dequantisation: thread t converts chunks 4h .. 4h + 3 (h = t / 128, warp-uniform) of weight row t % 128
    const int row = (threadIdx.x - 64) & (kBM - 1);
    const int half = (threadIdx.x - 64) / kBM;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S, c = kb % kConvStages;
      if (!mbar_wait(&full[s], (kb / S) & 1u, status, kStatusWaitFull, abort_flag)) break;
      if (!mbar_wait(&conv_empty[c], ((kb / kConvStages) & 1u) ^ 1u, status, kStatusWaitEmpty, abort_flag)) break;
      uint64_t meta = 0;
      bf16 sc = __float2bfloat16(1.f);
      if constexpr (FMT == kWqSp24) {
        meta = *reinterpret_cast<const uint64_t*>(reinterpret_cast<const uint8_t*>(scales) + s * F::kSideBytes +
                                                  (row >> 1) * 16 + (row & 1) * 8);
      } else if constexpr (F::kScaleRows == 1) {
        sc = scales[s * kBM + row];
      }
      const __nv_bfloat162 s2 = __halves2bfloat162(sc, sc);
      __nv_bfloat162 z2 = __halves2bfloat162(__float2bfloat16(0.f), __float2bfloat16(0.f));
      if (F::kZeros) {
        const bf16 zc = zeros[s * kBM + row];
        z2 = __halves2bfloat162(zc, zc);
      }
      const uint4* raw_row = reinterpret_cast<const uint4*>(raw + s * F::kRawBytes + row * F::kRawRowBytes);
      uint32_t words[F::kRawRowBytes / 4];
      constexpr int kVecs = F::kRawRowBytes / 16;
#pragma unroll
      for (int i = 0; i < kVecs; ++i) {
        if (kVecs > 1 && i * 2 / kVecs != half) continue;  // only this half's codes (int2 rows are one vector)
        const uint4 v = raw_row[i];
        words[4 * i] = v.x; words[4 * i + 1] = v.y; words[4 * i + 2] = v.z; words[4 * i + 3] = v.w;
      }
      uint8_t* dst_row = conv + c * kConvBytes + row * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if ((j >> 2) != half) continue;  // uniform per warp; j stays a compile-time index into `words`
        uint4 v;
        if constexpr (FMT == kWqSp24) {
          v = expand_sp24(words, meta, j);
        } else if constexpr (F::kScaleRows > 1) {  // fp4: the scale of the group holding k = 8j .. 8j + 7
          const bf16 sj = scales[s * (F::kSideBytes / 2) + (j * F::kScaleRows / 8) * kBM + row];
          v = dequant_chunk<FMT>(words, j, __halves2bfloat162(sj, sj), z2);
        } else {
          v = dequant_chunk<FMT>(words, j, s2, z2);
        }
        *reinterpret_cast<uint4*>(dst_row + ((j ^ (row & 7)) << 4)) = v;
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv_full[c]);
    }
  }
  __syncwarp();
  if (nkb > 0 && warp >= 2) mbar_wait(accum, 0, status, kStatusWaitAccum, abort_flag);
  pdl_wait();
  __syncthreads();
  tc_fence_after();
  const bool ok = nkb > 0 && !*abort_flag;
  const bool epi = warp >= 2 && warp < 6;  // the epilogue warps: one per TMEM lane quarter
  const int quarter = warp & 3;  // TMEM lanes 32 * (warp % 4) .. + 31 belong to this warp
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
  const int feat = quarter * 32 + lane;
  if (splits == 1) {
    if (ok && epi) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(lane_base + c, v);
        const int n = n0 + feat;
        if (n < N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c + j;
            if (m < M) y[static_cast<size_t>(m) * N + n] = __float2bfloat16(v[j]);
          }
        }
      }
    }
  } else {
    if (epi) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(lane_base + c, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) partial[(c + j) * kBM + feat] = ok ? v[j] : 0.f;
      }
    }
    cluster_sync();
    if (epi) {
      const int t = threadIdx.x - 64;
      const int cg = t & 31, rp = t >> 5;
      const int n = n0 + cg * 4;
      const uint32_t base_addr = smem_u32(partial);
      for (int i = rp;; i += 4) {
        const int j = static_cast<int>(rank) + splits * i;
        const int m = m0 + j;
        if (j >= BN || m >= M) break;
        const uint32_t addr = base_addr + (j * kBM + cg * 4) * 4;
        float4 acc = ld_dsmem_v4(addr, 0);
        for (int r = 1; r < splits; ++r) {
          const float4 v = ld_dsmem_v4(addr, r);
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        if (n < N && ok) {
          __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
          __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
          *reinterpret_cast<uint2*>(y + static_cast<size_t>(m) * N + n) = make_uint2(bf2_bits(lo), bf2_bits(hi));
        }
      }
    }
    cluster_sync();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

template <int FMT, int BN>
int run_wq(const WqMaps& maps, void* y, int M, int N, int K, int group, int splits, unsigned* status,
           cudaStream_t stream) {
  using Cfg = WqCfg<FMT, BN>;
  set_max_smem(gemm_wq_kernel<FMT, BN>, Cfg::kSmem);
  const int total_kb = K / kBK;
  const int kbps = (total_kb + splits - 1) / splits;
  splits = (total_kb + kbps - 1) / kbps;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + kBM - 1) / kBM, (M + BN - 1) / BN, splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = splits;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, gemm_wq_kernel<FMT, BN>, *maps.w, *maps.s,
                                             *(maps.z != nullptr ? maps.z : maps.s), *maps.x, static_cast<bf16*>(y),
                                             M, N, K, group, kbps, status);
  return err == cudaSuccess ? 0 : -2;
}

template <int FMT>
int run_wq_bn(const WqMaps& maps, void* y, int M, int N, int K, int group, int splits, unsigned* status,
              cudaStream_t stream) {
  switch (gemm_block_n(M)) {
    case 32: return run_wq<FMT, 32>(maps, y, M, N, K, group, splits, status, stream);
    case 64: return run_wq<FMT, 64>(maps, y, M, N, K, group, splits, status, stream);
    case 128: return run_wq<FMT, 128>(maps, y, M, N, K, group, splits, status, stream);
    default: return run_wq<FMT, 256>(maps, y, M, N, K, group, splits, status, stream);
  }
}

}  // namespace

// Split rule: like the bf16 kernel's, over the weight bytes this format streams (int4 moves a quarter of them).
int gemm_wq_splits(int M, int N, int K, int fmt, int num_sms) {
  const int slots = gemm_block_n(M) <= 64 ? 2 * num_sms : num_sms;
  const int tiles = ((N + kBM - 1) / kBM) * ((M + gemm_block_n(M) - 1) / gemm_block_n(M));
  const int kb = K / kBK;
  // at least 8 K-blocks (512 K) per CTA (16 for int2): below that the prologue dominates
  const int min_kb = fmt == kWqInt2 ? 16 : 8;
  int splits = std::max(1, std::min(slots / std::max(1, tiles), kb / min_kb));
  return std::min(8, splits);
}

int launch_gemm_wq(const WqMaps& maps, void* y, int M, int N, int K, int group, int fmt, int splits,
                   unsigned* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return 0;
  const int fp4_group = fmt == kWqMxfp4 ? 32 : fmt == kWqNvfp4 ? 16 : 0;
  if (fp4_group ? group != fp4_group : group % kBK != 0) return -1;
  if (K % kBK != 0 || K % group != 0 || N % 8 != 0 || splits < 1 || splits > 8) return -1;
  switch (fmt) {
    case kWqInt4: return run_wq_bn<kWqInt4>(maps, y, M, N, K, group, splits, status, stream);
    case kWqInt8: return run_wq_bn<kWqInt8>(maps, y, M, N, K, group, splits, status, stream);
    case kWqFp8: return run_wq_bn<kWqFp8>(maps, y, M, N, K, group, splits, status, stream);
    case kWqSp24: return run_wq_bn<kWqSp24>(maps, y, M, N, K, K, splits, status, stream);
    case kWqInt2: return run_wq_bn<kWqInt2>(maps, y, M, N, K, group, splits, status, stream);
    case kWqMxfp4: return run_wq_bn<kWqMxfp4>(maps, y, M, N, K, group, splits, status, stream);
    case kWqNvfp4: return run_wq_bn<kWqNvfp4>(maps, y, M, N, K, group, splits, status, stream);
    default: return -1;
  }
}

}  // namespace ecz
