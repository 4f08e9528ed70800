// Activation-sparse GEMVs for decoding steps (at most 16 rows): the weight rows or columns that the sparsified
// activations do not need are never read from HBM.
//
//   colsparse_gemv_kernel  y = sparsify(x) @ W^T with W stored transposed (W^T [K, N], row-major): only the rows
//                          k of W^T whose input column is kept by some row of x are streamed (TEAL: |x| > t; with
//                          t = 0 the exact zeros of a CATS / Deja Vu down-projection input are skipped).
//                          Each CTA compacts the kept columns of 128-wide chunks of its K range into shared memory;
//                          every quarter-warp then streams one 128-byte segment of a kept W^T row (8 lanes x 16 B)
//                          so one warp has eight rows of 64 columns in flight per step. Split-K partials are summed
//                          in split order by the last CTA of each column tile (deterministic).
//   glu_rows_kernel        h = (g * 1[keep]) * up(x) of a gated MLP whose [gate; up] weight is row-major [2F, H]:
//                          only the up rows (CATS: gate given densely, keep = |silu(gate)| > t) or the gate and up
//                          rows (Deja Vu: keep given by the predictor) of kept channels are read.
//
// The CUDA cores do the arithmetic: at <= 16 rows these products are bound by the weight bytes, which the sparsity
// reduces, not by the tensor cores.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

__device__ __forceinline__ uint4 ldg_stream(const bf16* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// the comparison |x| > t of a bf16 tensor with a 0-dim fp32 threshold happens in bf16
__device__ __forceinline__ float threshold_of(const float* thr) {
  return thr != nullptr ? __bfloat162float(__float2bfloat16(*thr)) : 0.f;
}

constexpr int kCsChunk = 128;   // K columns compacted per step (= threads of the CTA)
constexpr int kCsTile = 256;    // output columns per CTA (4 warps x 64)

template <int MT>
__global__ void __launch_bounds__(128) colsparse_gemv_kernel(const bf16* __restrict__ x, int ldx,
                                                             const bf16* __restrict__ wt, const float* thr,
                                                             bf16* __restrict__ out, float* __restrict__ ws,
                                                             int* __restrict__ counters, int M, int N, int K, int kc) {
  pdl_trigger();
  pdl_wait();
  __shared__ int act_k[kCsChunk];
  __shared__ float act_x[MT][kCsChunk];
  __shared__ int warp_cnt[4];
  __shared__ int is_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * kCsTile + warp * 64 + (lane & 7) * 8;  // this lane's 8 output columns
  const int q = lane >> 3;                                            // which kept row of each group of 4
  const bool col_ok = n0 < N;
  const int split = blockIdx.y;
  const int k_begin = split * kc, k_end = min(K, k_begin + kc);
  const float t = threshold_of(thr);
  float acc[MT][8];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[m][c] = 0.f;

  for (int c0 = k_begin; c0 < k_end; c0 += kCsChunk) {
    // ---- compact the kept columns of this chunk (any row keeps it); dropped entries of kept columns are 0 ----
    const int k = c0 + tid;
    float xv[MT];
    bool any = false;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      xv[m] = 0.f;
      if (m < M && k < k_end) {
        const float v = __bfloat162float(x[static_cast<long>(m) * ldx + k]);
        if (fabsf(v) > t) {
          xv[m] = v;
          any = true;
        }
      }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, any);
    if (lane == 0) warp_cnt[warp] = __popc(bal);
    __syncthreads();
    int base = 0;
    for (int w = 0; w < warp; ++w) base += warp_cnt[w];
    const int total = warp_cnt[0] + warp_cnt[1] + warp_cnt[2] + warp_cnt[3];
    if (any) {
      const int j = base + __popc(bal & ((1u << lane) - 1u));
      act_k[j] = k;
#pragma unroll
      for (int m = 0; m < MT; ++m) act_x[m][j] = xv[m];
    }
    __syncthreads();
    // ---- stream the kept rows of W^T: quarter-warp q takes kept rows q, q + 4, ...; 8 rows in flight ----
    if (col_ok) {
      int j = q;
      for (; j + 28 < total; j += 32) {
        uint4 w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) w[u] = ldg_stream(wt + static_cast<long>(act_k[j + 4 * u]) * N + n0);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float f[8];
          unpack8(w[u], f);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const float a = act_x[m][j + 4 * u];
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[m][c] = fmaf(a, f[c], acc[m][c]);
          }
        }
      }
      for (; j < total; j += 4) {
        float f[8];
        unpack8(ldg_stream(wt + static_cast<long>(act_k[j]) * N + n0), f);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const float a = act_x[m][j];
#pragma unroll
          for (int c = 0; c < 8; ++c) acc[m][c] = fmaf(a, f[c], acc[m][c]);
        }
      }
    }
    __syncthreads();  // the next chunk overwrites act_k / act_x
  }
  // ---- sum the four quarter-warps (fixed order: deterministic) ----
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      acc[m][c] += __shfl_xor_sync(0xffffffffu, acc[m][c], 8);
      acc[m][c] += __shfl_xor_sync(0xffffffffu, acc[m][c], 16);
    }
  if (gridDim.y == 1) {
    if (q == 0 && col_ok) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m >= M) break;
        uint4 o;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(acc[m][2 * i], acc[m][2 * i + 1]);
        *reinterpret_cast<uint4*>(out + static_cast<long>(m) * N + n0) = o;
      }
    }
    return;
  }
  if (q == 0 && col_ok) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m >= M) break;
      float4* dst = reinterpret_cast<float4*>(ws + (static_cast<long>(split) * M + m) * N + n0);
      dst[0] = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
      dst[1] = make_float4(acc[m][4], acc[m][5], acc[m][6], acc[m][7]);
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(&counters[blockIdx.x], 1) == static_cast<int>(gridDim.y) - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // the last CTA of this column tile: out = sum of the splits' partials in split order
  const int col = blockIdx.x * kCsTile + tid * 2;
  if (col < N) {
    for (int m = 0; m < M; ++m) {
      float2 s = make_float2(0.f, 0.f);
      for (int sp = 0; sp < static_cast<int>(gridDim.y); ++sp) {
        const float2 v = __ldcg(reinterpret_cast<const float2*>(ws + (static_cast<long>(sp) * M + m) * N + col));
        s.x += v.x;
        s.y += v.y;
      }
      *reinterpret_cast<__nv_bfloat162*>(out + static_cast<long>(m) * N + col) = __floats2bfloat162_rn(s.x, s.y);
    }
  }
  if (tid == 0) counters[blockIdx.x] = 0;
}

constexpr int kGluChannels = 32;  // channels per CTA (one per lane of warp 0 in the selection step)

__device__ __forceinline__ float silu_bf16(float v) { return bf16r(v / (1.f + expf(-v))); }

__device__ __forceinline__ float dot8(const uint4& a, const uint4& b) {
  float fa[8], fb[8];
  unpack8(a, fa);
  unpack8(b, fb);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s = fmaf(fa[i], fb[i], s);
  return s;
}

// DEJAVU: keep [M, F] (uint8) is given and the gate rows of kept channels are computed here too; otherwise (CATS)
// gate_pre [M, F] (row stride ld_gate) is the dense gate output and keep = |silu(gate)| > t.
template <int MT, bool DEJAVU>
__global__ void __launch_bounds__(128) glu_rows_kernel(const bf16* __restrict__ x, int ldx, const bf16* __restrict__ w,
                                                       const bf16* __restrict__ gate_pre, int ld_gate,
                                                       const uint8_t* __restrict__ keep_in, const float* thr,
                                                       bf16* __restrict__ h, int M, int F, int H) {
  pdl_trigger();
  pdl_wait();
  constexpr int R = DEJAVU ? 4 : 2;  // weight rows per group of two channels: (gate, gate,) up, up
  __shared__ float g_s[MT][kGluChannels];
  __shared__ int act_c[kGluChannels];
  __shared__ unsigned act_bits[kGluChannels];
  __shared__ int n_act;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int f0 = blockIdx.x * kGluChannels;
  if (warp == 0) {
    const int f = f0 + lane;
    unsigned bits = 0;
    if (f < F) {
      const float t = threshold_of(thr);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m >= M) break;
        if (DEJAVU) {
          if (keep_in[static_cast<long>(m) * F + f] != 0) bits |= 1u << m;
        } else {
          const float g = silu_bf16(__bfloat162float(gate_pre[static_cast<long>(m) * ld_gate + f]));
          g_s[m][lane] = g;
          if (fabsf(g) > t) bits |= 1u << m;
        }
      }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, bits != 0);
    if (bits != 0) {
      const int j = __popc(bal & ((1u << lane) - 1u));
      act_c[j] = lane;
      act_bits[j] = bits;
    } else if (f < F) {
      for (int m = 0; m < M; ++m) h[static_cast<long>(m) * F + f] = __float2bfloat16(0.f);
    }
    if (lane == 0) n_act = __popc(bal);
  }
  __syncthreads();
  const int groups = (n_act + 1) / 2;
  const int chunks = H / 8;
  for (int gi = warp; gi < groups; gi += 4) {
    int rows[R];
    const int ja = 2 * gi, jb = min(2 * gi + 1, n_act - 1);  // an odd last group computes its channel twice
    const int fa = f0 + act_c[ja], fb = f0 + act_c[jb];
    if (DEJAVU) {
      rows[0] = fa;
      rows[1] = fb;
      rows[2] = F + fa;
      rows[3] = F + fb;
    } else {
      rows[0] = F + fa;
      rows[1] = F + fb;
    }
    float acc[R][MT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;
    for (int p0 = lane; p0 < chunks; p0 += 32 * 4) {
      uint4 wv[4][R];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int p = p0 + 32 * u;
#pragma unroll
        for (int r = 0; r < R; ++r)
          wv[u][r] = p < chunks ? ldg_stream(w + static_cast<long>(rows[r]) * H + p * 8) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int p = p0 + 32 * u;
        if (p >= chunks) break;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m >= M) break;
          const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + static_cast<long>(m) * ldx + p * 8));
#pragma unroll
          for (int r = 0; r < R; ++r) acc[r][m] += dot8(wv[u][r], xv);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], o);
    // every lane holds the sums; lane (c * MT + m) % 32 writes h[m, channel c]
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int j = c == 0 ? ja : jb;
      const int f = c == 0 ? fa : fb;
      const unsigned bits = act_bits[j];
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m >= M || lane != (c * MT + m) % 32) continue;
        float g;
        if (DEJAVU) {
          g = silu_bf16(bf16r(acc[c][m]));
        } else {
          g = g_s[m][act_c[j]];
        }
        const float u = bf16r(acc[R - 2 + c][m]);
        h[static_cast<long>(m) * F + f] = __float2bfloat16(((bits >> m) & 1u) ? g * u : 0.f);
      }
    }
  }
}

template <int MT>
void run_colsparse(const bf16* x, int ldx, const bf16* wt, const float* thr, bf16* out, float* ws, int* counters,
                   int M, int N, int K, int splits, int kc, cudaStream_t stream) {
  const dim3 grid((N + kCsTile - 1) / kCsTile, splits);
  launch_pdl(colsparse_gemv_kernel<MT>, grid, dim3(128), 0, stream, x, ldx, wt, thr, out, ws, counters, M, N, K, kc);
}

template <int MT>
void run_glu(const bf16* x, int ldx, const bf16* w, const bf16* gate_pre, int ld_gate, const uint8_t* keep,
             const float* thr, bf16* h, int M, int F, int H, cudaStream_t stream) {
  const dim3 grid((F + kGluChannels - 1) / kGluChannels);
  if (keep != nullptr) {
    launch_pdl(glu_rows_kernel<MT, true>, grid, dim3(128), 0, stream, x, ldx, w, gate_pre, ld_gate, keep, thr, h, M,
               F, H);
  } else {
    launch_pdl(glu_rows_kernel<MT, false>, grid, dim3(128), 0, stream, x, ldx, w, gate_pre, ld_gate, keep, thr, h,
               M, F, H);
  }
}

}  // namespace

// K chunk per CTA (a multiple of 128) for about 8 CTAs per SM; the split count is ceil(K / chunk).
int colsparse_chunk(int M, int N, int K, int num_sms) {
  const int tiles = (N + kCsTile - 1) / kCsTile;
  const int target = num_sms * (M <= 4 ? 8 : 4);
  const int splits = std::max(1, std::min((target + tiles - 1) / tiles, (K + kCsChunk - 1) / kCsChunk));
  const int kc = (K + splits - 1) / splits;
  return (kc + kCsChunk - 1) / kCsChunk * kCsChunk;
}

int launch_colsparse_gemv(const void* x, int ldx, const void* wt, const float* thr, void* out, float* ws,
                          int* counters, int M, int N, int K, int kc, cudaStream_t stream) {
  if (M < 1 || M > 16 || N % 8 != 0 || kc % kCsChunk != 0 || (N + kCsTile - 1) / kCsTile > 8192) return -1;
  const int splits = (K + kc - 1) / kc;
  if (splits > 1 && (ws == nullptr || counters == nullptr)) return -2;
  auto xb = static_cast<const bf16*>(x);
  auto wb = static_cast<const bf16*>(wt);
  auto ob = static_cast<bf16*>(out);
  if (M == 1) run_colsparse<1>(xb, ldx, wb, thr, ob, ws, counters, M, N, K, splits, kc, stream);
  else if (M == 2) run_colsparse<2>(xb, ldx, wb, thr, ob, ws, counters, M, N, K, splits, kc, stream);
  else if (M <= 4) run_colsparse<4>(xb, ldx, wb, thr, ob, ws, counters, M, N, K, splits, kc, stream);
  else if (M <= 8) run_colsparse<8>(xb, ldx, wb, thr, ob, ws, counters, M, N, K, splits, kc, stream);
  else run_colsparse<16>(xb, ldx, wb, thr, ob, ws, counters, M, N, K, splits, kc, stream);
  return 0;
}

int launch_glu_rows(const void* x, int ldx, const void* w, const void* gate_pre, int ld_gate, const uint8_t* keep,
                    const float* thr, void* h, int M, int F, int H, cudaStream_t stream) {
  if (M < 1 || M > 16 || H % 8 != 0 || ldx % 8 != 0 || (gate_pre == nullptr && keep == nullptr)) return -1;
  auto xb = static_cast<const bf16*>(x);
  auto wb = static_cast<const bf16*>(w);
  auto gb = static_cast<const bf16*>(gate_pre);
  auto hb = static_cast<bf16*>(h);
  if (M == 1) run_glu<1>(xb, ldx, wb, gb, ld_gate, keep, thr, hb, M, F, H, stream);
  else if (M == 2) run_glu<2>(xb, ldx, wb, gb, ld_gate, keep, thr, hb, M, F, H, stream);
  else if (M <= 4) run_glu<4>(xb, ldx, wb, gb, ld_gate, keep, thr, hb, M, F, H, stream);
  else if (M <= 8) run_glu<8>(xb, ldx, wb, gb, ld_gate, keep, thr, hb, M, F, H, stream);
  else run_glu<16>(xb, ldx, wb, gb, ld_gate, keep, thr, hb, M, F, H, stream);
  return 0;
}

}  // namespace ecz
