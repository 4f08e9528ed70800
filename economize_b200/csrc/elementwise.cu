// Memory-bound fused kernels of the decoder block and of the speculative-decoding cycle:
//   * rmsnorm_kernel      fused residual add + RMSNorm (one CTA per token row, 16-byte vector loads)
//   * rope_store_kernel   optional per-head RMSNorm (QK-norm families) + rotary embedding of q and k, and the
//                         KV-cache write of k and v (one warp per token x head)
//   * glu_kernel          SwiGLU / GeGLU / clamped SwiGLU activation of a fused [gate; up] projection
//   * argmax_kernel       first index of the row maximum (one CTA per row)
//   * greedy_accept_kernel longest accepted path of a verified draft tree (one warp per row)
//   * kv_compact_kernel   moves the accepted path's K/V to consecutive slots in all layers at once
//
// Rounding follows Hugging Face's Llama modules where it matters for greedy identity: the residual sum and the
// normalized value are rounded to bf16 before the weight multiply, and the rotary products are rounded per term.
#include <cuda_fp8.h>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

// Split-K partials: a GEMM may leave `splits` fp32 partial products [splits][elems] instead of its bf16 output; the
// consuming kernel sums them in split order and rounds to bf16, which is exactly the value the GEMM's own reduction
// would have stored. These load 8 (2) consecutive values of element offset `off` either way.
struct Parts {
  const float* p = nullptr;
  int splits = 0;
  long stride = 0;  // elements between consecutive partials
};

constexpr int kMaxParts = 8;  // the split-K GEMM feeding a consumer never splits wider

__device__ __forceinline__ uint4 load8(const bf16* x, const Parts& parts, size_t off) {
  if (parts.p == nullptr) return *reinterpret_cast<const uint4*>(x + off);
  // issue every partial's loads before the (ordered) sum
  float4 c[kMaxParts], d[kMaxParts];
#pragma unroll
  for (int s = 0; s < kMaxParts; ++s) {
    if (s < parts.splits) {
      c[s] = __ldcg(reinterpret_cast<const float4*>(parts.p + s * parts.stride + off));
      d[s] = __ldcg(reinterpret_cast<const float4*>(parts.p + s * parts.stride + off + 4));
    }
  }
  float4 a = c[0], b = d[0];
#pragma unroll
  for (int s = 1; s < kMaxParts; ++s) {
    if (s < parts.splits) {
      a.x += c[s].x; a.y += c[s].y; a.z += c[s].z; a.w += c[s].w;
      b.x += d[s].x; b.y += d[s].y; b.z += d[s].z; b.w += d[s].w;
    }
  }
  __nv_bfloat162 h[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                         __floats2bfloat162_rn(b.x, b.y), __floats2bfloat162_rn(b.z, b.w)};
  return *reinterpret_cast<uint4*>(h);
}

__device__ __forceinline__ __nv_bfloat162 load2(const bf16* x, const Parts& parts, size_t off) {
  if (parts.p == nullptr) return *reinterpret_cast<const __nv_bfloat162*>(x + off);
  float2 c[kMaxParts];
#pragma unroll
  for (int s = 0; s < kMaxParts; ++s) {
    if (s < parts.splits) c[s] = __ldcg(reinterpret_cast<const float2*>(parts.p + s * parts.stride + off));
  }
  float2 a = c[0];
#pragma unroll
  for (int s = 1; s < kMaxParts; ++s) {
    if (s < parts.splits) { a.x += c[s].x; a.y += c[s].y; }
  }
  return __floats2bfloat162_rn(a.x, a.y);
}

// ---------------------------------------------------------------------------------------------------------------
// RMSNorm
// ---------------------------------------------------------------------------------------------------------------
template <int kMaxVec>
__global__ void __launch_bounds__(512) rmsnorm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ resid,
                                                      const bf16* __restrict__ w, bf16* __restrict__ out,
                                                      bf16* __restrict__ resid_out, int hidden, float eps,
                                                      Parts parts) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int nvec = hidden / 8;
  const uint4* rv = resid ? reinterpret_cast<const uint4*>(resid + static_cast<size_t>(row) * hidden) : nullptr;
  uint4* ro = reinterpret_cast<uint4*>(resid_out + static_cast<size_t>(row) * hidden);
  float vals[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      uint4 a = load8(x, parts, static_cast<size_t>(row) * hidden + v * 8);
      const bf16* ap = reinterpret_cast<const bf16*>(&a);
      uint4 s;
      bf16* sp = reinterpret_cast<bf16*>(&s);
      if (rv) {
        uint4 b = rv[v];
        const bf16* bp = reinterpret_cast<const bf16*>(&b);
#pragma unroll
        for (int j = 0; j < 8; ++j) sp[j] = __float2bfloat16(__bfloat162float(ap[j]) + __bfloat162float(bp[j]));
      } else {
        s = a;
      }
      ro[v] = s;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float f = __bfloat162float(sp[j]);
        vals[i][j] = f;
        ss += f * f;
      }
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / static_cast<float>(hidden) + eps);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  uint4* ov = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * hidden);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      uint4 ww = wv[v];
      const bf16* wp = reinterpret_cast<const bf16*>(&ww);
      uint4 o;
      bf16* op = reinterpret_cast<bf16*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) op[j] = __float2bfloat16(__bfloat162float(wp[j]) * bf16r(vals[i][j] * inv));
      ov[v] = o;
    }
  }
}

int launch_rmsnorm(const void* x, const void* resid, const void* w, void* out, void* resid_out, int rows, int hidden,
                   float eps, cudaStream_t stream, const float* x_parts, int splits) {
  const Parts parts{x_parts, splits, static_cast<long>(rows) * hidden};
  if (hidden % 8 != 0 || hidden > 256 * 8 * 8) return -1;
  const int nvec = hidden / 8;
  // partial sums cost several loads per vector: one vector per thread up to 512 threads
  const int cap = x_parts != nullptr ? 512 : 256;
  int threads = nvec < cap ? ((nvec + 31) / 32) * 32 : cap;
  const int per = (nvec + threads - 1) / threads;
  auto args = [&](auto kernel) {
    launch_pdl(kernel, dim3(rows), dim3(threads), 0, stream, static_cast<const bf16*>(x),
               static_cast<const bf16*>(resid), static_cast<const bf16*>(w), static_cast<bf16*>(out),
               static_cast<bf16*>(resid_out), hidden, eps, parts);
  };
  if (per <= 1) args(rmsnorm_kernel<1>);
  else if (per <= 2) args(rmsnorm_kernel<2>);
  else if (per <= 4) args(rmsnorm_kernel<4>);
  else args(rmsnorm_kernel<8>);
  return 0;
}

// ---------------------------------------------------------------------------------------------------------------
// Rotary embedding + KV-cache store (+ optional per-head RMSNorm of q and k)
// ---------------------------------------------------------------------------------------------------------------
// qkv [B*T, (H + 2 Hkv) * D]; q_out [B*T, H, D]; caches [B, Hkv, S, D]; token (b, t) writes slot
// kv_len[b] + q_offset + t when q_offset + t < n_new[b]. One warp per (token, head slot), head slot in
// [0, H + Hkv): q heads first, then kv heads (k rotated and stored with its v).
template <int D>
__global__ void __launch_bounds__(256) rope_store_kernel(
    const bf16* __restrict__ qkv, const int* __restrict__ positions, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, bf16* __restrict__ q_out, bf16* __restrict__ k_cache,
    bf16* __restrict__ v_cache, const int* __restrict__ kv_len, const int* __restrict__ n_new,
    const bf16* __restrict__ q_norm, const bf16* __restrict__ k_norm, float eps, int tokens, int T, int H, int Hkv,
    int S, int q_offset, const float* __restrict__ k_scale, const float* __restrict__ v_scale, Parts parts,
    KVPages pages, int table_rows, unsigned* status) {
  pdl_trigger();
  pdl_wait();
  // each active lane owns E consecutive elements (whole bf16 pairs) of each half of the head: D = 64 uses 16 lanes
  constexpr int E = D / 64 < 2 ? 2 : D / 64;
  constexpr int kLanes = D / (2 * E);
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int slots = H + Hkv;
  if (warp >= tokens * slots) return;
  const int token = warp / slots;
  const int head = warp % slots;
  const int b = token / T, t = token % T;
  const bool is_q = head < H;
  const int width = (H + 2 * Hkv) * D;
  const size_t src = static_cast<size_t>(token) * width + (is_q ? head * D : H * D + (head - H) * D);
  // lane owns elements [E * lane, E * lane + E) of the first half and their partners in the second half
  const bool active = lane < kLanes;
  const int i0 = E * (active ? lane : 0);
  float x[E], y[E];
#pragma unroll
  for (int e = 0; e < E; e += 2) {
    const __nv_bfloat162 lo = load2(qkv, parts, src + i0 + e);
    const __nv_bfloat162 hi = load2(qkv, parts, src + i0 + e + D / 2);
    x[e] = __bfloat162float(lo.x); x[e + 1] = __bfloat162float(lo.y);
    y[e] = __bfloat162float(hi.x); y[e + 1] = __bfloat162float(hi.y);
  }
  const bf16* nw = is_q ? q_norm : k_norm;
  if (nw != nullptr) {
    float part = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) part += x[e] * x[e] + y[e] * y[e];
    const float inv = rsqrtf(warp_sum(active ? part : 0.f) / D + eps);  // every lane joins the shuffle
#pragma unroll
    for (int e = 0; e < E; ++e) {
      x[e] = bf16r(__bfloat162float(nw[i0 + e]) * bf16r(x[e] * inv));
      y[e] = bf16r(__bfloat162float(nw[i0 + e + D / 2]) * bf16r(y[e] * inv));
    }
  }
  if (!active) return;
  int pos = positions[token];
  if (pos < 0 || pos >= table_rows) {  // a position past the rotary tables: report it, never read past them
    if (lane == 0 && status != nullptr) atomicOr(status, kStatusBadIndex);
    pos = min(max(pos, 0), table_rows - 1);
  }
  const float* cp = cos_t + static_cast<size_t>(pos) * (D / 2) + i0;
  const float* sp = sin_t + static_cast<size_t>(pos) * (D / 2) + i0;
  // out = x * cos + rotate_half(x) * sin, each product rounded to bf16 (HF computes it in the input dtype)
  float ra[E], rb[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float c = bf16r(cp[e]), sn = bf16r(sp[e]);
    ra[e] = bf16r(bf16r(x[e] * c) + bf16r(-y[e] * sn));
    rb[e] = bf16r(bf16r(y[e] * c) + bf16r(x[e] * sn));
  }
  if (is_q) {
    bf16* dst = q_out + (static_cast<size_t>(token) * H + head) * D;
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      *reinterpret_cast<__nv_bfloat162*>(dst + i0 + e) = __floats2bfloat162_rn(ra[e], ra[e + 1]);
      *reinterpret_cast<__nv_bfloat162*>(dst + i0 + e + D / 2) = __floats2bfloat162_rn(rb[e], rb[e + 1]);
    }
    return;
  }
  const int j = q_offset + t;
  if (j >= n_new[b]) return;
  const int kvh = head - H;
  if (kv_len[b] + j >= S) {  // a slot past the cache: report it, never write past the cache
    if (lane == 0 && status != nullptr) atomicOr(status, kStatusBadIndex);
    return;
  }
  const size_t off = kv_row(pages, b, Hkv, kvh, S, kv_len[b] + j) * D;
  const size_t vsrc = static_cast<size_t>(token) * width + (H + Hkv) * D + kvh * D;
  if (k_scale != nullptr) {
    // fp8 cache: e4m3 codes of value / scale (quotient rounded to fp32 first, then to e4m3 with saturation)
    const float sk = k_scale[kvh], sv = v_scale[kvh];
    uint8_t* kc = reinterpret_cast<uint8_t*>(k_cache) + off;
    uint8_t* vc = reinterpret_cast<uint8_t*>(v_cache) + off;
    auto put = [](uint8_t* dst, float a, float b2) {
      *reinterpret_cast<__nv_fp8x2_storage_t*>(dst) =
          __nv_cvt_float2_to_fp8x2(make_float2(a, b2), __NV_SATFINITE, __NV_E4M3);
    };
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      put(kc + i0 + e, __fdiv_rn(ra[e], sk), __fdiv_rn(ra[e + 1], sk));
      put(kc + i0 + e + D / 2, __fdiv_rn(rb[e], sk), __fdiv_rn(rb[e + 1], sk));
      const __nv_bfloat162 va = load2(qkv, parts, vsrc + i0 + e);
      const __nv_bfloat162 vb = load2(qkv, parts, vsrc + i0 + e + D / 2);
      put(vc + i0 + e, __fdiv_rn(__bfloat162float(va.x), sv), __fdiv_rn(__bfloat162float(va.y), sv));
      put(vc + i0 + e + D / 2, __fdiv_rn(__bfloat162float(vb.x), sv), __fdiv_rn(__bfloat162float(vb.y), sv));
    }
    return;
  }
#pragma unroll
  for (int e = 0; e < E; e += 2) {
    *reinterpret_cast<__nv_bfloat162*>(k_cache + off + i0 + e) = __floats2bfloat162_rn(ra[e], ra[e + 1]);
    *reinterpret_cast<__nv_bfloat162*>(k_cache + off + i0 + e + D / 2) = __floats2bfloat162_rn(rb[e], rb[e + 1]);
    *reinterpret_cast<__nv_bfloat162*>(v_cache + off + i0 + e) = load2(qkv, parts, vsrc + i0 + e);
    *reinterpret_cast<__nv_bfloat162*>(v_cache + off + i0 + e + D / 2) = load2(qkv, parts, vsrc + i0 + e + D / 2);
  }
}

int launch_rope_store(const void* qkv, const int* positions, const float* cos_t, const float* sin_t, void* q_out,
                      void* k_cache, void* v_cache, const int* kv_len, const int* n_new, const void* q_norm,
                      const void* k_norm, float eps, int B, int T, int H, int Hkv, int D, int S, int q_offset,
                      cudaStream_t stream, const float* k_scale, const float* v_scale, const float* qkv_parts,
                      int splits, const KVPages& pages, int table_rows, unsigned* status) {
  if ((D != 64 && D != 128 && D != 256) || table_rows < 1) return -1;
  const Parts parts{qkv_parts, splits, static_cast<long>(B) * T * (H + 2 * Hkv) * D};
  const long warps = static_cast<long>(B) * T * (H + Hkv);
  const int blocks = static_cast<int>((warps * 32 + 255) / 256);
  auto kernel = D == 64 ? rope_store_kernel<64> : D == 128 ? rope_store_kernel<128> : rope_store_kernel<256>;
  launch_pdl(kernel, dim3(blocks), dim3(256), 0, stream, static_cast<const bf16*>(qkv), positions, cos_t,
             sin_t, static_cast<bf16*>(q_out), static_cast<bf16*>(k_cache), static_cast<bf16*>(v_cache), kv_len,
             n_new, static_cast<const bf16*>(q_norm), static_cast<const bf16*>(k_norm), eps, B * T, T, H, Hkv, S,
             q_offset, k_scale, v_scale, parts, pages, table_rows, status);
  return 0;
}

// ---------------------------------------------------------------------------------------------------------------
// act(gate) * up: SiLU (SwiGLU), the tanh approximation of GELU (GeGLU, Gemma's gelu_pytorch_tanh), or gpt-oss's
// clamped SwiGLU: g = min(gate, limit), (clamp(up, -limit, limit) + 1) * g * sigmoid(1.702 g)
// ---------------------------------------------------------------------------------------------------------------
template <int kAct>
__device__ __forceinline__ float glu_act(float x, float limit) {
  if constexpr (kAct == 0) {
    return x / (1.f + expf(-x));
  } else if constexpr (kAct == 1) {  // 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3)))
    const float inner = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
    return 0.5f * x * (1.f + tanhf(inner));
  } else {
    const float g = fminf(x, limit);
    return g / (1.f + expf(-1.702f * g));
  }
}

template <int kAct>
__device__ __forceinline__ float glu_up(float u, float limit) {
  if constexpr (kAct == 2) {
    return fminf(fmaxf(u, -limit), limit) + 1.f;
  } else {
    return u;
  }
}

template <int kAct>
__global__ void __launch_bounds__(256) glu_kernel(const bf16* __restrict__ gu, bf16* __restrict__ out, int rows,
                                                  int F, Parts parts, float limit) {
  pdl_trigger();
  pdl_wait();
  const long total = static_cast<long>(rows) * (F / 8);
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long r = i / (F / 8), c = i % (F / 8);
    const uint4 g = load8(gu, parts, static_cast<size_t>(r) * 2 * F + c * 8);
    const uint4 u = load8(gu, parts, static_cast<size_t>(r) * 2 * F + F + c * 8);
    const bf16* gp = reinterpret_cast<const bf16*>(&g);
    const bf16* up = reinterpret_cast<const bf16*>(&u);
    uint4 o;
    bf16* op = reinterpret_cast<bf16*>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float s = bf16r(glu_act<kAct>(__bfloat162float(gp[j]), limit));
      op[j] = __float2bfloat16(s * glu_up<kAct>(__bfloat162float(up[j]), limit));
    }
    reinterpret_cast<uint4*>(out + r * F)[c] = o;
  }
}

int launch_glu(const void* gu, void* out, int rows, int F, cudaStream_t stream, const float* gu_parts, int splits,
               int act, float limit) {
  if (F % 8 != 0 || act < 0 || act > 2) return -1;
  const Parts parts{gu_parts, splits, static_cast<long>(rows) * 2 * F};
  const long total = static_cast<long>(rows) * (F / 8);
  int blocks = static_cast<int>(std::min<long>((total + 255) / 256, 148L * 16));
  if (blocks < 1) blocks = 1;
  launch_pdl(act == 0 ? glu_kernel<0> : act == 1 ? glu_kernel<1> : glu_kernel<2>, dim3(blocks), dim3(256), 0, stream,
             static_cast<const bf16*>(gu), static_cast<bf16*>(out), rows, F, parts, limit);
  return 0;
}

int launch_silu_mul(const void* gu, void* out, int rows, int F, cudaStream_t stream, const float* gu_parts,
                    int splits) {
  return launch_glu(gu, out, rows, F, stream, gu_parts, splits, 0);
}

// ---------------------------------------------------------------------------------------------------------------
// Block Walsh-Hadamard transform along the last dimension (QuaRot's online rotation of the down projection's input):
// y[r, k*b : (k+1)*b] = x[r, k*b : (k+1)*b] H_b / sqrt(b) with H_b the Sylvester matrix, b a power of two in
// [8, kMaxHadamard]. kGlu = true computes x as act(gate) * up of a fused [gate; up] projection first (the producing
// kernel of the rotated activation, so the activation never goes through HBM unrotated); its bf16 rounding is that of
// glu_kernel, so the fused result equals glu followed by the plain transform bit for bit.
//
// One CTA of 256 threads per (row, block): each thread loads 8 consecutive elements (16-byte loads), applies the
// butterflies of half-width 1, 2 and 4 in registers, and stores them to shared memory (b fp32 values); the butterflies
// of half-width 8 .. b/2 then run in shared memory, one __syncthreads() per stage; the result is scaled and stored with
// 16-byte stores. The transform is memory bound (b x 2 bytes in and out per CTA); stages run in the order h = 1, 2, 4,
// ..., b/2, the order of the fp32 host reference.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kMaxHadamard = 8192;  // 32 KB of fp32 shared memory: below the 48 KB default, no attribute needed

template <int kAct, bool kGlu>
__global__ void __launch_bounds__(256) hadamard_kernel(const bf16* __restrict__ in, bf16* __restrict__ out, int F,
                                                       int block, int blocks_per_row, Parts parts, float limit,
                                                       float scale) {
  extern __shared__ float hsh[];
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x / blocks_per_row;
  const int base = (blockIdx.x % blocks_per_row) * block;
  const int groups = block / 8;
  for (int g = threadIdx.x; g < groups; g += blockDim.x) {
    float v[8];
    if constexpr (kGlu) {
      const size_t off = static_cast<size_t>(r) * 2 * F + base + g * 8;
      const uint4 gv = load8(in, parts, off);
      const uint4 uv = load8(in, parts, off + F);
      const bf16* gp = reinterpret_cast<const bf16*>(&gv);
      const bf16* up = reinterpret_cast<const bf16*>(&uv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float a = bf16r(glu_act<kAct>(__bfloat162float(gp[j]), limit));
        v[j] = bf16r(a * glu_up<kAct>(__bfloat162float(up[j]), limit));
      }
    } else {
      const uint4 xv = *reinterpret_cast<const uint4*>(in + static_cast<size_t>(r) * F + base + g * 8);
      const bf16* xp = reinterpret_cast<const bf16*>(&xv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(xp[j]);
    }
#pragma unroll
    for (int h = 1; h < 8; h <<= 1) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if ((j & h) == 0) {
          const float a = v[j], b = v[j + h];
          v[j] = a + b;
          v[j + h] = a - b;
        }
      }
    }
    float4* dst = reinterpret_cast<float4*>(hsh + g * 8);
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
  __syncthreads();
  for (int h = 8; h < block; h <<= 1) {
    for (int t = threadIdx.x; t < block / 2; t += blockDim.x) {
      const int i = ((t & ~(h - 1)) << 1) | (t & (h - 1));
      const float a = hsh[i], b = hsh[i + h];
      hsh[i] = a + b;
      hsh[i + h] = a - b;
    }
    __syncthreads();
  }
  for (int g = threadIdx.x; g < groups; g += blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(hsh + g * 8)[0];
    const float4 b = reinterpret_cast<const float4*>(hsh + g * 8)[1];
    uint4 o;
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&o);
    op[0] = __floats2bfloat162_rn(a.x * scale, a.y * scale);
    op[1] = __floats2bfloat162_rn(a.z * scale, a.w * scale);
    op[2] = __floats2bfloat162_rn(b.x * scale, b.y * scale);
    op[3] = __floats2bfloat162_rn(b.z * scale, b.w * scale);
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(r) * F + base + g * 8) = o;
  }
}

int launch_hadamard(const void* x, void* out, int rows, int F, int block, cudaStream_t stream, int glu_act_kind,
                    const float* gu_parts, int splits, float limit) {
  if (block < 8 || block > kMaxHadamard || (block & (block - 1)) != 0 || F % block != 0 || rows < 1) return -1;
  if (glu_act_kind < -1 || glu_act_kind > 2) return -1;
  const long ctas = static_cast<long>(rows) * (F / block);
  if (ctas > 0x7fffffffL) return -1;
  const Parts parts{gu_parts, splits, static_cast<long>(rows) * 2 * F};
  const size_t smem = static_cast<size_t>(block) * sizeof(float);
  const float scale = rsqrtf(static_cast<float>(block));
  auto kernel = glu_act_kind < 0    ? hadamard_kernel<0, false>
                : glu_act_kind == 0 ? hadamard_kernel<0, true>
                : glu_act_kind == 1 ? hadamard_kernel<1, true>
                                    : hadamard_kernel<2, true>;
  const cudaError_t err = launch_pdl(kernel, dim3(static_cast<unsigned>(ctas)), dim3(256), smem, stream,
                                     static_cast<const bf16*>(x), static_cast<bf16*>(out), F, block, F / block, parts,
                                     limit, scale);
  return err == cudaSuccess ? 0 : -3;
}

// ---------------------------------------------------------------------------------------------------------------
// Row argmax (first maximal index), bf16 or fp32 input
// ---------------------------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<bf16>(bf16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }

// Two stages: every CTA scans one slice of a row with 16-byte loads and writes its (max, first index); a second
// kernel reduces the slices of each row. Ties resolve to the smallest index in both stages.
__device__ __forceinline__ void argmax_merge(float& best, int& idx, float ob, int oi) {
  if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
}

__device__ __forceinline__ void block_argmax(float& best, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_merge(best, idx, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, idx, o));
  __shared__ float sb[32];
  __shared__ int si[32];
  if ((threadIdx.x & 31) == 0) { sb[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = idx; }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    best = threadIdx.x < nw ? sb[threadIdx.x] : -INFINITY;
    idx = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      argmax_merge(best, idx, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, idx, o));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) argmax_slice_kernel(const T* __restrict__ x, float* __restrict__ part_v,
                                                           int* __restrict__ part_i, int V, int slice) {
  pdl_trigger();
  pdl_wait();
  constexpr int kVec = 16 / sizeof(T);
  const int row = blockIdx.y, s = blockIdx.x;
  const T* base = x + static_cast<size_t>(row) * V;
  const int lo = s * slice, hi = min(V, lo + slice);
  float best = -INFINITY;
  int idx = 0x7fffffff;
  const bool aligned = (V % kVec == 0) && (lo % kVec == 0);
  if (aligned) {
    for (int v = lo / kVec + threadIdx.x; v < hi / kVec; v += blockDim.x) {
      const uint4 raw = reinterpret_cast<const uint4*>(base)[v];
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int j = 0; j < kVec; ++j) argmax_merge(best, idx, to_f<T>(e[j]), v * kVec + j);
    }
  } else {
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) argmax_merge(best, idx, to_f<T>(base[i]), i);
  }
  block_argmax(best, idx);
  if (threadIdx.x == 0) {
    part_v[row * gridDim.x + s] = best;
    part_i[row * gridDim.x + s] = idx;
  }
}

__global__ void __launch_bounds__(32) argmax_finish_kernel(const float* __restrict__ part_v,
                                                           const int* __restrict__ part_i, int64_t* __restrict__ out,
                                                           int slices) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int s = threadIdx.x; s < slices; s += 32) argmax_merge(best, idx, part_v[row * slices + s], part_i[row * slices + s]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_merge(best, idx, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, idx, o));
  if (threadIdx.x == 0) out[row] = idx == 0x7fffffff ? 0 : idx;
}

int argmax_slices(int rows, int V) {
  // enough CTAs to cover the SMs a few times, slices of at least 4096 entries
  int slices = std::max(1, std::min((V + 4095) / 4096, (4 * 148 + rows - 1) / std::max(rows, 1)));
  return std::min(slices, 32);
}

int launch_argmax(const void* x, bool is_bf16, int64_t* out, float* part_v, int* part_i, int rows, int V,
                  cudaStream_t stream) {
  if (rows == 0) return 0;
  const int slices = argmax_slices(rows, V);
  int slice = (V + slices - 1) / slices;
  slice = (slice + 7) / 8 * 8;
  dim3 grid(slices, rows);
  if (is_bf16) {
    launch_pdl(argmax_slice_kernel<bf16>, grid, dim3(256), 0, stream, static_cast<const bf16*>(x), part_v, part_i, V,
               slice);
  } else {
    launch_pdl(argmax_slice_kernel<float>, grid, dim3(256), 0, stream, static_cast<const float*>(x), part_v, part_i,
               V, slice);
  }
  launch_pdl(argmax_finish_kernel, dim3(rows), dim3(32), 0, stream, part_v, part_i, out, slices);
  return 0;
}

// ---------------------------------------------------------------------------------------------------------------
// Greedy acceptance of a draft tree (chains are trees with parent t-1)
// ---------------------------------------------------------------------------------------------------------------
// One warp per row; T <= 64 nodes. Node t (t >= 1) is accepted when its parent is and tokens[t] == pred[parent].
// The deepest accepted node (first on ties) ends the path. Outputs n_acc [B], path [B, T] (node of the i-th path
// position, padded with the last node) and out [B, T] (path tokens after the root, then the bonus pred[last]).
__global__ void greedy_accept_kernel(const int64_t* __restrict__ tokens, const int64_t* __restrict__ parents,
                                     const int64_t* __restrict__ pred, const uint8_t* __restrict__ ok,
                                     int* __restrict__ n_acc, int* __restrict__ path, int64_t* __restrict__ out,
                                     int T) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  const int lane = threadIdx.x;
  __shared__ int acc[64], depth[64], par[64];
  const int64_t* tk = tokens + static_cast<size_t>(b) * T;
  const int64_t* pa = parents + static_cast<size_t>(b) * T;
  const int64_t* pr = pred + static_cast<size_t>(b) * T;
  for (int t = lane; t < T; t += 32) par[t] = t == 0 ? -1 : static_cast<int>(pa[t]);
  __syncwarp();
  if (lane == 0) {
    acc[0] = 1;
    depth[0] = 0;
    int best = 0, best_depth = 0;
    for (int t = 1; t < T; ++t) {
      const int p = par[t];
      const bool match = ok != nullptr ? ok[static_cast<size_t>(b) * T + t] != 0 : tk[t] == pr[p];
      const bool good = p >= 0 && p < t && acc[p] && match;
      acc[t] = good;
      depth[t] = (p >= 0 && p < t) ? depth[p] + 1 : 0;
      if (good && depth[t] > best_depth) { best_depth = depth[t]; best = t; }
    }
    n_acc[b] = best_depth;
    int node = best;
    for (int i = best_depth; i >= 0; --i) {  // walk up from the last node
      path[static_cast<size_t>(b) * T + i] = node;
      if (i >= 1) out[static_cast<size_t>(b) * T + i - 1] = tk[node];
      node = i > 0 ? par[node] : 0;
    }
    for (int i = best_depth + 1; i < T; ++i) path[static_cast<size_t>(b) * T + i] = best;
    out[static_cast<size_t>(b) * T + best_depth] = pr[best];
    for (int i = best_depth + 1; i < T; ++i) out[static_cast<size_t>(b) * T + i] = 0;
  }
}

int launch_greedy_accept(const int64_t* tokens, const int64_t* parents, const int64_t* pred, const uint8_t* ok,
                         int* n_acc, int* path, int64_t* out, int B, int T, cudaStream_t stream) {
  if (T > 64) return -1;
  launch_pdl(greedy_accept_kernel, dim3(B), dim3(32), 0, stream, tokens, parents, pred, ok, n_acc, path, out, T);
  return 0;
}

// ---------------------------------------------------------------------------------------------------------------
// KV compaction after a tree pass: cache [L*2, B, Hkv, S, D]; slot kv_len + path[i] -> kv_len + i, i <= n_acc.
// One CTA per (layer*2 + kv, b, kv head); every thread reads its 16-byte chunk first, then all write, so
// overlapping source/destination slots of one path never race.
// ---------------------------------------------------------------------------------------------------------------
// Every (path position, 16-byte vector) pair of a row is read into registers before any is written (a source slot
// may be another position's destination); a thread owns up to kCompactPer pairs, so rows of up to 64 vectors (D = 256
// bf16) move 64 path positions deep in one 1024-thread block.
constexpr int kCompactPer = 4;

__global__ void kv_compact_kernel(uint8_t* __restrict__ cache, const int* __restrict__ kv_len,
                                  const int* __restrict__ path, const int* __restrict__ n_acc, int B, int Hkv, int S,
                                  int row_bytes, int T, int max_depth, KVLayout layout) {
  pdl_trigger();
  pdl_wait();
  const int layer = blockIdx.x >> 1, kv = blockIdx.x & 1;
  const int b = blockIdx.y, h = blockIdx.z;
  const int n = n_acc[b];
  const int vecs = row_bytes / 16;
  const int pairs = max_depth * vecs;
  const int start = kv_len[b];
  auto row = [&](int slot) { return cache + kv_layer_row(layout, layer, kv, b, Hkv, h, S, slot) * row_bytes; };
  uint4 v[kCompactPer];
  int dst[kCompactPer];
#pragma unroll
  for (int u = 0; u < kCompactPer; ++u) {
    const int pr = threadIdx.x + u * blockDim.x;
    const int i = pr / vecs + 1;  // path position (the root at 0 never moves)
    dst[u] = -1;
    if (pr < pairs && i <= n && i < T) {
      const int src = path[static_cast<size_t>(b) * T + i];
      if (start + src >= S || start + i >= S || src < 0) continue;  // never move past the cache
      if (src != i) {
        v[u] = reinterpret_cast<const uint4*>(row(start + src))[pr % vecs];
        dst[u] = i;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < kCompactPer; ++u) {
    if (dst[u] >= 0) {
      const int pr = threadIdx.x + u * blockDim.x;
      reinterpret_cast<uint4*>(row(start + dst[u]))[pr % vecs] = v[u];
    }
  }
}

// Rows of `row_bytes` bytes (D * element size: bf16 and fp8 caches alike).
int launch_kv_compact(void* cache, const int* kv_len, const int* path, const int* n_acc, int L, int B, int Hkv,
                      int S, int row_bytes, int T, int max_depth, cudaStream_t stream, const KVLayout& layout) {
  if (row_bytes % 16 || max_depth < 1) return -1;
  const int pairs = max_depth * (row_bytes / 16);
  const int threads = std::min(1024, ((pairs + 31) / 32) * 32);
  if (pairs > threads * kCompactPer) return -1;
  dim3 grid(2 * L, B, Hkv);
  launch_pdl(kv_compact_kernel, grid, dim3(threads), 0, stream, static_cast<uint8_t*>(cache), kv_len, path, n_acc,
             B, Hkv, S, row_bytes, T, max_depth, layout);
  return 0;
}

}  // namespace ecz
