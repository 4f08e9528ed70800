// Sparse mixture-of-experts MLP on the tensor cores: routing, token permutation, grouped expert GEMMs and the
// weighted combine (Mixtral-style top-k routing; economize runs Hugging Face's MoE modules,
// src/economize/techniques/draft_model/technique.py:54-70).
//
//   moe_route_kernel    one CTA: per token softmax over the router logits, top-k experts, weights renormalised
//                       over the k chosen (fp32); per expert the tokens in token order (deterministic positions),
//                       expert offsets (exclusive scan) for the grouped GEMMs
//   moe_gather_kernel   x_sorted[pos[t, j]] = x[t]
//   gemm_grouped_kernel swap-AB tcgen05 GEMM over all experts at once: CTA (n-tile, m-tile, expert) computes
//                       rows offsets[e] + m-tile of x_sorted against expert e's weight rows; tiles beyond an
//                       expert's token count exit after reading the offsets
//   moe_combine_kernel  out[t] = sum_j w[t, j] * y[pos[t, j]] (fp32 accumulation in j order, bf16 out)
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kMaxExperts = 64;
constexpr int kMaxTopK = 8;

// ---- routing ---------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) moe_route_kernel(const bf16* __restrict__ logits, int T, int E, int k,
                                                         int* __restrict__ ids, float* __restrict__ weights,
                                                         int* __restrict__ pos, int* __restrict__ offsets) {
  pdl_trigger();
  pdl_wait();
  __shared__ int counts[kMaxExperts];
  __shared__ int base[kMaxExperts + 1];
  if (threadIdx.x < kMaxExperts) counts[threadIdx.x] = 0;
  __syncthreads();
  // phase 1: top-k per token (thread per token)
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const bf16* row = logits + static_cast<size_t>(t) * E;
    float mx = -INFINITY;
    for (int e = 0; e < E; ++e) mx = fmaxf(mx, __bfloat162float(row[e]));
    float denom = 0.f;
    for (int e = 0; e < E; ++e) denom += __expf(__bfloat162float(row[e]) - mx);
    int chosen[kMaxTopK];
    float prob[kMaxTopK];
    float sel = 0.f;
    for (int j = 0; j < k; ++j) {
      int best = -1;
      float bv = -INFINITY;
      for (int e = 0; e < E; ++e) {
        bool used = false;
        for (int i = 0; i < j; ++i) used |= chosen[i] == e;
        const float v = __bfloat162float(row[e]);
        if (!used && v > bv) {  // ties: the lower expert id
          bv = v;
          best = e;
        }
      }
      chosen[j] = best;
      prob[j] = __expf(bv - mx) / denom;
      sel += prob[j];
    }
    for (int j = 0; j < k; ++j) {
      ids[t * k + j] = chosen[j];
      weights[t * k + j] = prob[j] / sel;
      atomicAdd(&counts[chosen[j]], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    base[0] = 0;
    for (int e = 0; e < E; ++e) base[e + 1] = base[e] + counts[e];
    for (int e = 0; e <= E; ++e) offsets[e] = base[e];
  }
  __syncthreads();
  // phase 2: deterministic positions (token order within an expert): warp e scans the (t, j) list
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pairs = T * k;
  for (int e = warp; e < E; e += blockDim.x / 32) {
    int running = base[e];
    for (int i0 = 0; i0 < pairs; i0 += 32) {
      const int i = i0 + lane;
      const bool hit = i < pairs && ids[i] == e;
      const unsigned mask = __ballot_sync(0xffffffffu, hit);
      if (hit) pos[i] = running + __popc(mask & ((1u << lane) - 1u));
      running += __popc(mask);
    }
  }
}

__global__ void __launch_bounds__(256) moe_gather_kernel(const bf16* __restrict__ x, const int* __restrict__ pos,
                                                         bf16* __restrict__ xs, int T, int k, int H) {
  pdl_trigger();
  pdl_wait();
  const int pair = blockIdx.x;  // t * k + j
  const int t = pair / k;
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H);
  uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<size_t>(pos[pair]) * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}

__global__ void __launch_bounds__(256) moe_combine_kernel(const bf16* __restrict__ y, const int* __restrict__ pos,
                                                          const float* __restrict__ w, bf16* __restrict__ out, int k,
                                                          int H) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < H / 2; c += blockDim.x) {
    float2 acc = make_float2(0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const float wt = w[t * k + j];
      const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(y + static_cast<size_t>(pos[t * k + j]) * H)[c];
      acc.x += wt * __bfloat162float(v.x);
      acc.y += wt * __bfloat162float(v.y);
    }
    reinterpret_cast<__nv_bfloat162*>(out + static_cast<size_t>(t) * H)[c] = __floats2bfloat162_rn(acc.x, acc.y);
  }
}

// ---- grouped GEMM ----------------------------------------------------------------------------------------------
template <int BN>
struct GroupedCfg {
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = std::min(8, (100 * 1024) / kStageBytes);
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

template <int BN>
__global__ void __launch_bounds__(128, 2)
    gemm_grouped_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                        bf16* __restrict__ y, const int* __restrict__ seg_start, const int* __restrict__ seg_end,
                        const int* __restrict__ seg_expert, int N, int K, unsigned* status) {
  using Cfg = GroupedCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = smem + S * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  pdl_trigger();
  pdl_wait();  // the segments come from the routing (or expert-parallel dispatch) kernel
  const int g = blockIdx.z;  // segment: rows [seg_start[g], seg_end[g]) use expert seg_expert[g] (default g)
  const int e = seg_expert != nullptr ? seg_expert[g] : g;
  const int row_end = seg_end[g];
  const int m0 = seg_start[g] + blockIdx.y * BN;
  if (m0 >= row_end) return;  // uniform: the whole CTA leaves before any shared state exists
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_local = blockIdx.x * kBM;
  const int n_row = e * N + n_local;  // row of the stacked [E * N, K] weights
  const int nkb = K / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S;
      if (kb >= S && !mbar_wait(&empty[s], ((kb / S) & 1u) ^ 1u, status, kStatusWaitEmpty, abort_flag)) break;
      mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
      tma_load_2d(a_tiles + s * kABytes, &tm_w, &full[s], kb * kBK, n_row);
      tma_load_2d(b_tiles + s * Cfg::kBBytes, &tm_x, &full[s], kb * kBK, m0);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S;
      if (!mbar_wait(&full[s], (kb / S) & 1u, status, kStatusWaitFull, abort_flag)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(a_tiles + s * kABytes);
      const uint32_t b_addr = smem_u32(b_tiles + s * Cfg::kBBytes);
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        umma_bf16(tmem, desc_kmajor_sw128(a_addr + kk * 32), desc_kmajor_sw128(b_addr + kk * 32), idesc,
                  (kb | kk) != 0 ? 1u : 0u);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(accum);
  }
  __syncwarp();
  mbar_wait(accum, 0, status, kStatusWaitAccum, abort_flag);
  __syncthreads();
  tc_fence_after();
  const bool ok = !*abort_flag;
  const int n = n_local + warp * 32 + lane;
  if (ok) {  // warp-uniform: tcgen05.ld is a warp-collective load; only the stores are masked per lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      tmem_ld16(lane_base + c, v);
      if (n < N) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c + j;
          if (m < row_end) y[static_cast<size_t>(m) * N + n] = __float2bfloat16(v[j]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

template <int BN>
int run_grouped(const CUtensorMap& tm_w, const CUtensorMap& tm_x, void* y, const int* seg_start, const int* seg_end,
                const int* seg_expert, int G, int max_rows, int N, int K, unsigned* status, cudaStream_t stream) {
  using Cfg = GroupedCfg<BN>;
  set_max_smem(gemm_grouped_kernel<BN>, Cfg::kSmem);
  dim3 grid((N + kBM - 1) / kBM, (max_rows + BN - 1) / BN, G);
  launch_pdl(gemm_grouped_kernel<BN>, grid, dim3(128), Cfg::kSmem, stream, tm_w, tm_x, static_cast<bf16*>(y),
             seg_start, seg_end, seg_expert, N, K, status);
  return 0;
}

}  // namespace

int launch_moe_route(const void* logits, int T, int E, int k, int* ids, float* weights, int* pos, int* offsets,
                     cudaStream_t stream) {
  if (E > kMaxExperts || k > kMaxTopK || k > E || T < 1) return -1;
  launch_pdl(moe_route_kernel, dim3(1), dim3(1024), 0, stream, static_cast<const bf16*>(logits), T, E, k, ids,
             weights, pos, offsets);
  return 0;
}

int launch_moe_gather(const void* x, const int* pos, void* xs, int T, int k, int H, cudaStream_t stream) {
  if (H % 8 != 0) return -1;
  launch_pdl(moe_gather_kernel, dim3(T * k), dim3(256), 0, stream, static_cast<const bf16*>(x), pos,
             static_cast<bf16*>(xs), T, k, H);
  return 0;
}

int launch_moe_combine(const void* y, const int* pos, const float* w, void* out, int T, int k, int H,
                       cudaStream_t stream) {
  if (H % 2 != 0) return -1;
  launch_pdl(moe_combine_kernel, dim3(T), dim3(256), 0, stream, static_cast<const bf16*>(y), pos, w,
             static_cast<bf16*>(out), k, H);
  return 0;
}

// Rows per expert are unknown on the host: the grid covers `max_rows` (every routed row in one expert) and CTAs
// past an expert's count exit. The tile width follows the average rows per expert.
int grouped_block_n(int rows, int E) {
  const int avg = (rows + E - 1) / E;
  return avg <= 32 ? 32 : (avg <= 64 ? 64 : 128);
}

int launch_gemm_grouped(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, const int* offsets, int E,
                        int rows, int N, int K, unsigned* status, cudaStream_t stream) {
  if (K % kBK != 0 || N % 8 != 0 || rows < 1) return -1;
  switch (grouped_block_n(rows, E)) {
    case 32: return run_grouped<32>(*tm_w, *tm_x, y, offsets, offsets + 1, nullptr, E, rows, N, K, status, stream);
    case 64: return run_grouped<64>(*tm_w, *tm_x, y, offsets, offsets + 1, nullptr, E, rows, N, K, status, stream);
    default: return run_grouped<128>(*tm_w, *tm_x, y, offsets, offsets + 1, nullptr, E, rows, N, K, status, stream);
  }
}

// Segments (start, end, expert) instead of expert offsets: rows of one segment use one expert's weights; at most
// `max_rows` rows per segment.
int launch_gemm_segments(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, const int* seg_start,
                         const int* seg_end, const int* seg_expert, int G, int max_rows, int N, int K,
                         unsigned* status, cudaStream_t stream) {
  if (K % kBK != 0 || N % 8 != 0 || max_rows < 1 || G < 1) return -1;
  switch (grouped_block_n(max_rows, G)) {
    case 32: return run_grouped<32>(*tm_w, *tm_x, y, seg_start, seg_end, seg_expert, G, max_rows, N, K, status, stream);
    case 64: return run_grouped<64>(*tm_w, *tm_x, y, seg_start, seg_end, seg_expert, G, max_rows, N, K, status, stream);
    default:
      return run_grouped<128>(*tm_w, *tm_x, y, seg_start, seg_end, seg_expert, G, max_rows, N, K, status, stream);
  }
}

}  // namespace ecz
