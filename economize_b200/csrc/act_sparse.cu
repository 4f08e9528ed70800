// Activation-sparse GEMVs for decoding steps (at most 16 rows): the weight rows or columns that the sparsified
// activations do not need are never read from HBM.
//
//   colsparse_gemv_kernel  y = sparsify(x) @ W^T with W stored transposed (W^T [K, N], row-major): only the rows
//                          k of W^T whose input column is kept by some row of x are streamed (TEAL: |x| > t; with
//                          t = 0 the exact zeros of a CATS / Deja Vu down-projection input are skipped).
//                          Each CTA compacts the kept columns of its K range chunk by chunk into shared memory;
//                          every quarter-warp then streams one 128-byte segment of a kept W^T row (8 lanes x 16 B),
//                          eight rows in flight. K-groups of warps split each chunk and are summed in shared memory;
//                          the split-K partials of a column tile are summed in split order by its last CTA, so the
//                          result is deterministic.
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

constexpr int kCsTile = 256;   // output columns per CTA (4 warps x 64)
constexpr int kCsChunk = 128;  // K columns compacted per step (one per thread)
constexpr int kCsCluster = 8;  // CTAs of one column tile whose partials are summed through DSMEM

// grid (column tiles, CS * G), cluster (1, CS): CTA (tile, split) streams the kept rows of its K range; the CS
// CTAs of a cluster sum their partial tiles through distributed shared memory in rank order, and with G > 1 the
// tile's last cluster sums the G cluster partials in order (deterministic; no fp32 atomics).
template <int MT>
__global__ void __launch_bounds__(128, MT <= 4 ? 8 : 2) colsparse_gemv_kernel(const bf16* __restrict__ x, int ldx,
                                                             const bf16* __restrict__ wt, const float* thr,
                                                             bf16* __restrict__ out, float* __restrict__ ws,
                                                             int* __restrict__ counters, int M, int N, int K, int kc) {
  pdl_trigger();
  pdl_wait();
  __shared__ int act_k[kCsChunk];
  __shared__ float act_x[MT][kCsChunk];
  __shared__ __align__(16) float part[MT][kCsTile];
  __shared__ int warp_cnt[4];
  __shared__ int is_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * kCsTile + warp * 64 + (lane & 7) * 8;  // this lane's 8 output columns
  const int q = lane >> 3;                                            // which kept row of each group of 4
  const bool col_ok = n0 < N;
  const int split = blockIdx.y;
  const int k_begin = min(K, split * kc), k_end = min(K, k_begin + kc);
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
  // ---- sum the four quarter-warps (fixed order) into this CTA's partial tile ----
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      acc[m][c] += __shfl_xor_sync(0xffffffffu, acc[m][c], 8);
      acc[m][c] += __shfl_xor_sync(0xffffffffu, acc[m][c], 16);
    }
  if (q == 0) {
    const int cin = warp * 64 + (lane & 7) * 8;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float4* dst = reinterpret_cast<float4*>(&part[m][cin]);
      dst[0] = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
      dst[1] = make_float4(acc[m][4], acc[m][5], acc[m][6], acc[m][7]);
    }
  }
  // ---- cluster: rank r sums columns [r * 256 / CS, (r + 1) * 256 / CS) over the CS CTAs in rank order ----
  const int CS = min(static_cast<int>(gridDim.y), kCsCluster);
  const int G = gridDim.y / CS;
  const int rank = static_cast<int>(cluster_ctarank());
  cluster_sync();
  const int span = (kCsTile / CS) & ~3;  // 16-byte aligned slices; the last rank also takes the remainder
  const int c_lo = rank * span, c_hi = rank == CS - 1 ? kCsTile : c_lo + span;
  const int g = split / CS;
  for (int i = tid; i < M * ((c_hi - c_lo + 3) / 4); i += 128) {
    const int per = (c_hi - c_lo + 3) / 4;
    const int m = i / per, c = c_lo + (i % per) * 4;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    const uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(&part[m][c]));
    for (int r = 0; r < CS; ++r) {
      const float4 v = ld_dsmem_v4(local, r);
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
    }
    const int col = blockIdx.x * kCsTile + c;
    if (col >= N) continue;
    if (G == 1) {
      __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(out + static_cast<long>(m) * N + col);
      o[0] = __floats2bfloat162_rn(sum.x, sum.y);
      o[1] = __floats2bfloat162_rn(sum.z, sum.w);
    } else {
      *reinterpret_cast<float4*>(ws + (static_cast<long>(g) * M + m) * N + col) = sum;
    }
  }
  cluster_sync();  // the peers' partial tiles stay alive until every rank has read them
  if (G == 1) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(&counters[blockIdx.x], 1) == static_cast<int>(gridDim.y) - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // the tile's last CTA: out = sum of the G cluster partials in order (all loads in flight at once)
  for (int i = tid; i < M * (kCsTile / 4); i += 128) {
    const int m = i / (kCsTile / 4), c = (i % (kCsTile / 4)) * 4;
    const int col = blockIdx.x * kCsTile + c;
    if (col >= N) continue;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int g0 = 0; g0 < G; g0 += 8) {  // eight cluster partials in flight
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (g0 + u < G)
          v[u] = __ldcg(reinterpret_cast<const float4*>(ws + (static_cast<long>(g0 + u) * M + m) * N + col));
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (g0 + u < G) {
          sum.x += v[u].x;
          sum.y += v[u].y;
          sum.z += v[u].z;
          sum.w += v[u].w;
        }
    }
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(out + static_cast<long>(m) * N + col);
    o[0] = __floats2bfloat162_rn(sum.x, sum.y);
    o[1] = __floats2bfloat162_rn(sum.z, sum.w);
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
  const int cs = std::min(splits, kCsCluster);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + kCsTile - 1) / kCsTile, splits);
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = cs;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, colsparse_gemv_kernel<MT>, x, ldx, wt, thr, out, ws, counters, M, N, K, kc);
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

// Split count: about 8 CTAs per SM in one wave, as CS CTAs per cluster (CS <= 8) times G <= 16 cluster groups; the
// K range per CTA is a multiple of 128 (CTAs past the end of K contribute zeros).
int colsparse_splits(int M, int N, int K, int num_sms) {
  const int tiles = (N + kCsTile - 1) / kCsTile;
  const int target = num_sms * (M <= 4 ? 8 : 4);
  int want = std::max(1, std::min((target + tiles - 1) / tiles, (K + kCsChunk - 1) / kCsChunk));
  if (want <= kCsCluster) return want;
  const int groups = std::min(16, (want + kCsCluster - 1) / kCsCluster);
  return groups * kCsCluster;
}

int launch_colsparse_gemv(const void* x, int ldx, const void* wt, const float* thr, void* out, float* ws,
                          int* counters, int M, int N, int K, int splits, cudaStream_t stream) {
  if (M < 1 || M > 16 || N % 8 != 0 || splits < 1 || (N + kCsTile - 1) / kCsTile > 8192) return -1;
  if (splits > kCsCluster && (splits % kCsCluster != 0 || splits / kCsCluster > 16)) return -1;
  if (splits > kCsCluster && (ws == nullptr || counters == nullptr)) return -2;
  int kc = (K + splits - 1) / splits;
  kc = (kc + kCsChunk - 1) / kCsChunk * kCsChunk;
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
