// Tree-masked / causal attention over the slot KV cache on the 5th-generation tensor cores.
//
// Replaces economize's Triton split-K decode kernel (src/economize/attention/_decode_kernels.py:110-226) and its
// sdpa prefill path. One CTA handles 128 "packed" query rows of one (sequence b, KV head): row p is query token
// t = p / G of query head kvh * G + p % G (G = H / H_kv), so a GQA group's heads share every K/V tile. The CTA walks
// 128-key chunks of the cache:
//
//   TMA   K, V chunk [128 keys, 128 dims] (two 64-wide 128B-swizzled boxes each), double-buffered
//   UMMA  S = Q . K^T  (M = 128 rows, N = 128 keys, K = 128 dims) into TMEM columns [0, 128)
//   regs  thread r (TMEM lane r) reads its score row, applies the scale and the visibility rule, updates the
//         running max / sum, and writes P = exp(s - max) as bf16 into a swizzled shared tile
//   UMMA  PV = P . V  (N = 128 dims, V read MN-major) into TMEM columns [128, 256)
//   regs  O = O * exp(max_old - max_new) + PV
//
// Visibility of slot s for query token t of row b: s < kv_len[b] (committed prefix), or j = s - kv_len[b] < n_new[b]
// and (bit j of mask[b, t], or j <= q_offset + t without a mask). The key range may be split over `splits` CTAs,
// whose (O, max, sum) partials a merge kernel combines in log-sum-exp form (the split-K merge of the reference).
//
// Exact-tail mode (tail_w > 0, decode and verification passes): a query at position p takes the keys at positions
// below p - tail_w from the tensor-core walk above, by absolute slot (they are committed keys at slot = position in
// every pass), and the keys at positions [p - tail_w, p] in the merge kernel, one at a time in position order on the
// CUDA cores: committed slots first, then the query's own new keys (its ancestors and itself) in depth order. How a
// key enters the sum then depends only on the query's and the key's positions, never on where a draft tree put the
// key or how many queries share the pass, so a verification pass computes every accepted token's attention bit for
// bit as a one-token pass at the same position does (greedy speculative decoding reproduces plain decoding exactly)
// as long as the tree is at most tail_w deep.
//
// Options (AttnOpts): tanh soft-capping of the scores (Gemma-2: s -> cap * tanh(s / cap), applied to the scaled
// natural-log score), attention sinks (gpt-oss: one learned logit per query head that joins every row's softmax
// denominator and contributes no value), and sliding windows (Mistral / Gemma-2/3 / OLMo-3 local layers: a query at
// position p sees keys at positions > p - window). With a window the CTA walks only the chunks its rows can see,
// and the key split is planned over the window's span with split boundaries at absolute multiples of the chunks per
// split, so passes of different widths still reduce a row's keys in the same groups.
//
// Head dimension 256 (Gemma): Q [128, 256] and one stage each of K and V [128, 256] fill the shared memory (the row
// partials share the P tile), so K of the next chunk streams while P . V runs and V while the next S runs; the
// accumulator uses TMEM columns [128, 384) of a 512-column allocation.
//
// Pipelined walk (bf16 caches without KIVI codes at head dimension 64 / 128, the PIPE instantiation): the scores
// are double-buffered in TMEM (columns [0, 128) and [128, 256)) and the output accumulates in TMEM (columns from
// 256), so the tensor cores compute S of chunk i + 1 while the threads run chunk i's softmax, and P . V of chunk i
// accumulates into O without a per-chunk read of the accumulator. The running maximum is rescaled lazily: a row keeps
// its reference maximum until a chunk raises it by more than kLazyLog2 (P then stays below 2^kLazyLog2), and only
// then are its O columns read, scaled and written back (the per-row decision keeps a row's arithmetic independent
// of the other rows, which the exact-tail guarantee needs). K and V stream on their own barriers: K of chunk i + 2
// loads as soon as S of chunk i has read its stage, V of chunk i + 1 as soon as P . V of chunk i - 1 has.
//
// fp8 caches (e4m3 codes with one static scale per KV head, K = s_k * K8, V = s_v * V8): TMA brings the raw
// [128 keys, 128 B] code tiles into a double-buffered staging ring, all threads convert them to bf16 (exact: every
// e4m3 value is a bf16 value) in the swizzled layout the UMMAs read, and the scales are applied outside the tensor
// cores: s_k multiplies the softmax scale, s_v the output. This reads half the bytes of a bf16 cache (the
// reference's fp8_kv decode path decodes the codes in registers, src/economize/attention/_decode_kernels.py:17).
#include <algorithm>
#include <cstdlib>

#include <cuda_fp8.h>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

constexpr int kRows = 128;
constexpr int kKeys = 128;
constexpr int kDim = 128;
constexpr int kAtom = kRows * 128;          // bytes of one 64-column swizzled half tile (128 rows x 128 B)
constexpr int kTile = 2 * kAtom;            // a 128 x 128 bf16 tile
constexpr int kSmem = 6 * kTile + 1024 + 64 + 4 * 128 * 4;  // Q, P, 2 x K, 2 x V, barriers, row partials
// the same layout for head dimension D (Q [128, D], P [128, 128], two stages of K and V [128, D])
__host__ __device__ constexpr int attn_smem_bytes(int D) {
  return D == 256 ? kRows * D * 2 + kTile + 2 * kKeys * D * 2 + 1024 + 64  // one K/V stage; partials in the P tile
                  : kRows * D * 2 + kTile + 4 * kKeys * D * 2 + 1024 + 64 + 4 * 128 * 4;
}
// The pipelined walk keeps Q and P in TMEM: the shared memory holds kPipeStages rings of K and V chunks, the
// barriers (128 B) and the row partials.
__host__ __device__ constexpr int pipe_stages(int D) { return D == 64 ? 6 : 3; }
__host__ __device__ constexpr int attn_pipe_smem_bytes(int D) {
  return 2 * pipe_stages(D) * kKeys * D * 2 + 1024 + 128 + 4 * 128 * 4;
}
static_assert(attn_pipe_smem_bytes(128) <= 232448 && attn_pipe_smem_bytes(64) <= 232448, "pipelined rings fit");
static_assert(attn_smem_bytes(256) <= 232448, "the D = 256 layout must fit 227 KB");
static_assert(attn_smem_bytes(128) == kSmem, "the D = 128 layout is the reference footprint");
constexpr int kRawTile = kKeys * kDim;                        // one fp8 code tile (128 keys x 128 B)
// fp8: Q, P, converted K, converted V, then 2 stages x (raw K, raw V): the same 6 x kTile
static_assert(4 * kTile + 4 * kRawTile == 6 * kTile, "fp8 layout must fit the bf16 footprint");

__device__ __forceinline__ void store_row_swizzled(uint8_t* tile, int r, int chunk, uint4 v) {
  // chunk in [0, 16): 16-byte chunk of a 256-byte row; chunks 0-7 in the first half tile, 8-15 in the second
  uint8_t* atom = tile + (chunk >> 3) * kAtom;
  const int c = chunk & 7;
  *reinterpret_cast<uint4*>(atom + r * 128 + ((c ^ (r & 7)) << 4)) = v;
}

// Convert one 128 x 128 e4m3 code tile (row-major, 128 B rows) into the bf16 swizzled two-atom tile; thread t of
// 512 converts 32 codes of row t / 4.
__device__ __forceinline__ void convert_fp8_tile(const uint8_t* raw, uint8_t* tile, int tid) {
  const int row = tid >> 2, part = tid & 3;
  const uint4* src = reinterpret_cast<const uint4*>(raw + row * kDim + part * 32);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 v = src[h];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int u = 0; u < 2; ++u) {  // 8 codes -> one 16-byte chunk of 8 bf16
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t word = w[2 * u + k / 2];
        const __nv_fp8x2_storage_t pair = static_cast<__nv_fp8x2_storage_t>((word >> (16 * (k & 1))) & 0xFFFFu);
        const __half2 hv = __half2(__nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3));
        __nv_bfloat162 bv = __float22bfloat162_rn(__half22float2(hv));
        o[k] = *reinterpret_cast<uint32_t*>(&bv);
      }
      store_row_swizzled(tile, row, part * 4 + h * 2 + u, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}


// ---- KIVI (2- or 4-bit) chunks ------------------------------------------------------------------------------------
// A quantized 128-key chunk of one (layer, row, KV head) is stored contiguously (kivi_chunk_bytes): key codes
// (token-major, 128 channels x bits), per-channel key scales and zeros (bf16, group = the chunk's 128 tokens), value
// codes (token-major), per-token value scales and zeros for groups of 32 channels. Dequantisation is
// bf16(code * scale + zero) with the product and the sum rounded separately in fp32.
__host__ __device__ constexpr int kivi_code_bytes(int bits) { return kKeys * kDim * bits / 8; }
__host__ __device__ constexpr int kivi_chunk_bytes(int bits) {
  return 2 * kivi_code_bytes(bits) + 2 * kDim * 2 + 2 * kKeys * (kDim / 32) * 2;
}

// Thread tid of 512 fills row tid / 4, channels [32 (tid % 4), + 32) of the K and V tiles of a quantized chunk.
__device__ __forceinline__ void dequant_kivi_tile(const uint8_t* chunk, int bits, uint8_t* k_tile, uint8_t* v_tile,
                                                  int tid) {
  const int row = tid >> 2, part = tid & 3;
  const int code_row = kDim * bits / 8;  // bytes per token
  const uint8_t* kc = chunk;
  const bf16* ks = reinterpret_cast<const bf16*>(chunk + kivi_code_bytes(bits));
  const bf16* kz = ks + kDim;
  const uint8_t* vc = chunk + kivi_code_bytes(bits) + 2 * kDim * 2;
  const bf16* vs = reinterpret_cast<const bf16*>(vc + kivi_code_bytes(bits));
  const bf16* vz = vs + kKeys * (kDim / 32);
  const float vscale = __bfloat162float(vs[row * 4 + part]), vzero = __bfloat162float(vz[row * 4 + part]);
  const int mask = (1 << bits) - 1;
#pragma unroll
  for (int u = 0; u < 4; ++u) {  // 8 channels per 16-byte chunk of the swizzled tile
    const int ch0 = part * 32 + u * 8;
    uint32_t kw, vw;  // the 8 codes of channels ch0 .. ch0 + 7
    if (bits == 2) {
      kw = *reinterpret_cast<const uint16_t*>(kc + row * code_row + ch0 / 4);
      vw = *reinterpret_cast<const uint16_t*>(vc + row * code_row + ch0 / 4);
    } else {
      kw = *reinterpret_cast<const uint32_t*>(kc + row * code_row + ch0 / 2);
      vw = *reinterpret_cast<const uint32_t*>(vc + row * code_row + ch0 / 2);
    }
    uint32_t ko[4], vo[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      float kv[2], vv[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int ch = ch0 + e + h;
        const float kcode = static_cast<float>((kw >> ((e + h) * bits)) & mask);
        const float vcode = static_cast<float>((vw >> ((e + h) * bits)) & mask);
        kv[h] = __fadd_rn(__fmul_rn(kcode, __bfloat162float(ks[ch])), __bfloat162float(kz[ch]));
        vv[h] = __fadd_rn(__fmul_rn(vcode, vscale), vzero);
      }
      __nv_bfloat162 k2 = __floats2bfloat162_rn(kv[0], kv[1]), v2 = __floats2bfloat162_rn(vv[0], vv[1]);
      ko[e / 2] = *reinterpret_cast<uint32_t*>(&k2);
      vo[e / 2] = *reinterpret_cast<uint32_t*>(&v2);
    }
    store_row_swizzled(k_tile, row, part * 4 + u, make_uint4(ko[0], ko[1], ko[2], ko[3]));
    store_row_swizzled(v_tile, row, part * 4 + u, make_uint4(vo[0], vo[1], vo[2], vo[3]));
  }
}

// Visibility of the 32 slots [s0, s0 + 32) for one query row, bit i = slot s0 + i.
__device__ __forceinline__ uint32_t visible32(int s0, int base, int nn, bool use_mask, uint64_t bits, int causal_lim,
                                              bool row_valid) {
  if (!row_valid) return 0u;
  const int pre = min(max(base - s0, 0), 32);  // committed prefix
  uint32_t vis = pre >= 32 ? 0xffffffffu : ((1u << pre) - 1u);
  const int j0 = s0 - base;  // new-region index of slot s0
  const int lim = use_mask ? min(nn, 64) : min(nn, causal_lim);
  const int hi = min(lim - j0, 32);  // bits i < hi have j < lim
  const int lo = max(-j0, 0);        // bits i >= lo have j >= 0
  if (hi > lo) {
    uint32_t range = (hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u)) & ~(lo >= 32 ? 0xffffffffu : ((1u << lo) - 1u));
    uint32_t sel = 0xffffffffu;
    if (use_mask) {
      const uint64_t w = j0 >= 0 ? (j0 < 64 ? (bits >> j0) : 0ull) : (-j0 < 64 ? (bits << (-j0)) : 0ull);
      sel = static_cast<uint32_t>(w);
    }
    vis |= range & sel;
  }
  return vis;
}

// Bits i of the 32 slots [s0, s0 + 32) with s0 + i >= lo (the sliding window's first visible slot).
__device__ __forceinline__ uint32_t at_or_above(int s0, int lo) {
  const long k = static_cast<long>(lo) - s0;
  return k <= 0 ? 0xffffffffu : (k >= 32 ? 0u : ~((1u << k) - 1u));
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Combine the split partials of packed row r of tile `tile`: out = sum_s O_s 2^(m_s - M) / sum_s l_s 2^(m_s - M).
// One warp per row, lane l owns columns E l .. E l + E - 1 (E = D / 32).
template <int D>
__device__ __forceinline__ void merge_row(const float* __restrict__ ws_o, const float* __restrict__ ws_ml,
                                          bf16* __restrict__ out, int tile, int r, int lane, int T, int H, int Hkv,
                                          int m_tiles, int splits, float* __restrict__ lse_out,
                                          const float* __restrict__ sinks) {
  const int m_tile = tile % m_tiles, bh = tile / m_tiles;
  const int b = bh / Hkv, kvh = bh % Hkv;
  const int G = H / Hkv;
  const int p = m_tile * kRows + r;
  const int t = p / G;
  if (t >= T) return;
  const int head = kvh * G + p % G;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) {
    const size_t slot = (static_cast<size_t>(tile) * splits + s) * kRows + r;
    if (ws_ml[slot * 2 + 1] > 0.f) mx = fmaxf(mx, ws_ml[slot * 2]);
  }
  const float sink2 = sinks != nullptr ? sinks[head] * 1.4426950408889634f : -INFINITY;
  mx = fmaxf(mx, sink2);  // a sink logit joins the denominator only
  constexpr int E = D / 32;
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  float denom = 0.f;
  for (int s = 0; s < splits; ++s) {
    const size_t slot = (static_cast<size_t>(tile) * splits + s) * kRows + r;
    const float l = ws_ml[slot * 2 + 1];
    if (!(l > 0.f)) continue;
    const float w = exp2f(ws_ml[slot * 2] - mx);
    const float* v = ws_o + slot * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] += v[e] * w;
    denom += l * w;
  }
  if (sinks != nullptr) denom += exp2f(sink2 - mx);
  const float inv = denom > 0.f ? 1.f / denom : 0.f;
  if (lse_out != nullptr && lane == 0)
    lse_out[(static_cast<size_t>(b) * T + t) * H + head] = denom > 0.f ? mx + __log2f(denom) : -INFINITY;
  bf16* dst = out + ((static_cast<size_t>(b) * T + t) * H + head) * D + lane * E;
#pragma unroll
  for (int e = 0; e < E; e += 2)
    *reinterpret_cast<__nv_bfloat162*>(dst + e) = __floats2bfloat162_rn(acc[e] * inv, acc[e + 1] * inv);
}

// 16 warps: warp w reads TMEM lanes 32 * (w % 4) .. (its rows) and owns score / output columns
// [32 * (w / 4), 32 * (w / 4) + 32) of them (quarter q).
constexpr int kThreads = 512;

// a row's reference maximum moves when a chunk raises it by more than this (log2 units; P < 2^kLazyLog2)
constexpr float kLazyLog2 = 8.f;

template <bool FP8, int D = 128, bool PIPE = false>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const bf16* __restrict__ q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, bf16* __restrict__ out, float* __restrict__ ws_o,
                   float* __restrict__ ws_ml, const int* __restrict__ kv_len, const int* __restrict__ n_new,
                   const int64_t* __restrict__ mask, int T, int H, int Hkv, int S, float scale_log2, int q_offset,
                   int chunks_per_split, int m_tiles, unsigned* status, unsigned long long* trace,
                   const float* __restrict__ k_scale, const float* __restrict__ v_scale,
                   const uint32_t* __restrict__ keep, float* __restrict__ lse_out,
                   const uint8_t* __restrict__ kivi, const int* __restrict__ kivi_chunks, int kivi_bits, int tail_w,
                   AttnOpts opts, KVPages pages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  static_assert(D == 64 || D == 128 || D == 256, "head dimensions 64, 128 and 256");
  static_assert(!FP8 || D == 128, "fp8 caches at head dimension 128");
  static_assert(!PIPE || (!FP8 && D <= 128), "the pipelined walk reads bf16 caches at head dimension 64 / 128");
  constexpr bool kSingle = D == 256;       // one K/V stage (see the file comment)
  constexpr int kQTile = kRows * D * 2;    // Q [128 rows, D]
  constexpr int kKVTile = kKeys * D * 2;   // one K or V chunk [128 keys, D]
  constexpr int kDQ = D / 4;               // output columns per quarter of the CTA
  constexpr int kAtoms = D / 64;           // 64-column swizzled atoms per row
  constexpr int kStages = kSingle ? 1 : 2;
  constexpr uint32_t kTmemCols = (kSingle || PIPE) ? 512 : 256;
  constexpr int kRing = pipe_stages(D);  // PIPE: depth of the K and V rings
  uint8_t* q_tile = smem;
  uint8_t* p_tile = smem + kQTile;
  // bf16: kStages stages of K and V tiles; fp8: one converted K and V tile, then two stages of raw codes;
  // PIPE: kRing stages of K, then kRing of V, from the start (Q and P live in TMEM)
  uint8_t* k_tiles = PIPE ? smem : p_tile + kTile;
  uint8_t* v_tiles = PIPE ? smem + kRing * kKVTile : FP8 ? k_tiles + kTile : k_tiles + kStages * kKVTile;
  uint8_t* raw = smem + 4 * kTile;  // fp8 stage s: raw K at s * 2 * kRawTile, raw V after it
  // kv_full[s]: stage s of K and V (kSingle: [0] = K, [1] = V; PIPE: K of ring stage s, v_full[s] its V)
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(PIPE ? smem + 2 * kRing * kKVTile
                                                       : p_tile + kTile + 2 * kStages * kKVTile);
  uint64_t* v_full = kv_full + kRing;
  uint64_t* bar_s = PIPE ? kv_full + 2 * kRing : kv_full + 2;  // PIPE: one per score buffer
  uint64_t* bar_pv = PIPE ? bar_s + 2 : bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_pv + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [4][128] row partials (kSingle: inside the P tile, free whenever the partials are in use)
  float* red = kSingle ? reinterpret_cast<float*>(p_tile)
                       : reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(kv_full) + (PIPE ? 128 : 64));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, quarter = warp >> 2;
  const int r = quad * 32 + lane;  // this thread's row (TMEM lane)
  unsigned long long* stamp = (trace != nullptr && tid == 0)
                                  ? trace + (static_cast<size_t>(blockIdx.y) * gridDim.x + blockIdx.x) * 16
                                  : nullptr;
  if (stamp) stamp[0] = global_timer_ns();
  pdl_trigger();
  pdl_wait();
  const int m_tile = blockIdx.x % m_tiles;
  const int bh = blockIdx.x / m_tiles;
  const int b = bh / Hkv, kvh = bh % Hkv;
  const int split = blockIdx.y;
  const int G = H / Hkv;

  const int p = m_tile * kRows + r;
  const int t = p / G;
  const int head = kvh * G + p % G;
  const bool row_valid = t < T;
  const int base = kv_len[b];
  const int nn = n_new[b];
  const bool use_mask = mask != nullptr;
  const uint64_t bits = (row_valid && use_mask) ? static_cast<uint64_t>(mask[static_cast<size_t>(b) * T + t]) : 0ull;
  const int causal_lim = q_offset + t + 1;
  // the query's position minus the committed length (tree depth, or its index among the new tokens)
  const int qdepth = use_mask ? max(0, __popcll(bits) - 1) : (q_offset + t);
  const int wlo = (opts.window > 0 && row_valid) ? base + qdepth - opts.window + 1 : INT_MIN;  // first visible slot

  const int t_last = min(T - 1, ((m_tile + 1) * kRows - 1) / G);
  const bool tail = tail_w > 0;
  // exact-tail mode: this row's tensor-core keys are the committed slots below its position minus tail_w
  int tc_lim = 0;
  if (tail && row_valid) tc_lim = max(0, min(base, base + qdepth - tail_w));
  int visible_end = tail ? base : use_mask ? base + nn : base + min(nn, q_offset + t_last + 1);
  visible_end = min(visible_end, S);
  const int n_chunks = (visible_end + kKeys - 1) / kKeys;
  // with a window, split groups start at the group of the first chunk any row of the tile can see
  int g0 = 0;
  if (opts.window > 0) {
    const int t_first = min(T - 1, (m_tile * kRows) / G);
    const int pos_min = base + (use_mask ? 0 : q_offset + t_first);
    g0 = (max(0, pos_min - opts.window + 1) / kKeys) / chunks_per_split;
  }
  const int c0 = (g0 + split) * chunks_per_split;
  const int c1 = min(n_chunks, c0 + chunks_per_split);
  if (!index_ok(base >= 0 && nn >= 0 && base <= S, tid == 0 ? status : nullptr)) return;  // bounds-checked builds

  const int q_chunks = (!FP8 && kivi != nullptr) ? kivi_chunks[b] : 0;  // chunks [0, q_chunks) are KIVI-coded
  auto issue_kv = [&](int c, int s) {
    const int y = static_cast<int>(kv_row(pages, b, Hkv, kvh, S, c * kKeys));
    if (c < q_chunks) {  // filled by the threads at its turn; the stage barrier completes without bytes
      mbar_arrive(&kv_full[s]);
      return;
    }
    if constexpr (FP8) {
      mbar_arrive_expect_tx(&kv_full[s], 2 * kRawTile);
      tma_load_2d(raw + s * 2 * kRawTile, &tm_k, &kv_full[s], 0, y);
      tma_load_2d(raw + s * 2 * kRawTile + kRawTile, &tm_v, &kv_full[s], 0, y);
    } else {
      mbar_arrive_expect_tx(&kv_full[s], 2 * kAtoms * kAtom);
#pragma unroll
      for (int a = 0; a < kAtoms; ++a) {
        tma_load_2d(k_tiles + s * kKVTile + a * kAtom, &tm_k, &kv_full[s], 64 * a, y);
        tma_load_2d(v_tiles + s * kKVTile + a * kAtom, &tm_v, &kv_full[s], 64 * a, y);
      }
    }
  };
  // kSingle: K and V of chunk c into the single stage, each on its own barrier
  auto issue_one = [&](int c, bool is_v) {
    const int y = static_cast<int>(kv_row(pages, b, Hkv, kvh, S, c * kKeys));
    uint64_t* bar = &kv_full[is_v ? 1 : 0];
    uint8_t* dst = is_v ? v_tiles : k_tiles;
    mbar_arrive_expect_tx(bar, kAtoms * kAtom);
#pragma unroll
    for (int a = 0; a < kAtoms; ++a) tma_load_2d(dst + a * kAtom, is_v ? &tm_v : &tm_k, bar, 64 * a, y);
  };
  // PIPE: K or V of chunk c into stage st, each on its own barrier
  auto issue_half = [&](int c, int st, bool is_v) {
    const int y = static_cast<int>(kv_row(pages, b, Hkv, kvh, S, c * kKeys));
    uint64_t* bar = is_v ? &v_full[st] : &kv_full[st];
    uint8_t* dst = (is_v ? v_tiles : k_tiles) + st * kKVTile;
    mbar_arrive_expect_tx(bar, kAtoms * kAtom);
#pragma unroll
    for (int a = 0; a < kAtoms; ++a) tma_load_2d(dst + a * kAtom, is_v ? &tm_v : &tm_k, bar, 64 * a, y);
  };
  // Chunks whose committed keys are all hidden by the keep bitmap (and that hold no new key) are skipped: the
  // CTA walks the active chunks only, every thread computing the same sequence from the bitmap.
  auto active = [&](int c) -> bool {
    if (keep == nullptr || (c + 1) * kKeys > base) return true;
    const uint32_t* kw = keep + (static_cast<size_t>(b) * Hkv + kvh) * (S / 32) + c * (kKeys / 32);
    return (kw[0] | kw[1] | kw[2] | kw[3]) != 0u;
  };
  auto next_active = [&](int c) -> int {
    while (c < c1 && !active(c)) ++c;
    return c;
  };
  if constexpr (FP8) scale_log2 *= k_scale[kvh];  // S = s_k * (Q . K8^T)
  // soft-cap: s2 = cap log2(e) tanh(raw * scale / cap) (scale_log2 = scale log2(e))
  const bool capped = opts.softcap > 0.f;
  const float cap_in = capped ? scale_log2 / (1.4426950408889634f * opts.softcap) : 0.f;
  const float cap_out = capped ? opts.softcap * 1.4426950408889634f : 0.f;
  if (tid == 0) {
    mbar_init(&kv_full[0], 1);
    mbar_init(&kv_full[1], 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_pv, 1);
    if constexpr (PIPE) {
      for (int st = 0; st < kRing; ++st) {
        mbar_init(&kv_full[st], 1);
        mbar_init(&v_full[st], 1);
      }
      mbar_init(bar_s + 1, 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
    // the first active K/V chunks stream while the CTA allocates TMEM and stages Q
    const int a0 = next_active(c0);
    if constexpr (PIPE) {  // the first kRing chunks fill both rings
      int a = a0;
      for (int j = 0; j < kRing && a < c1; ++j) {
        issue_half(a, j, false);
        issue_half(a, j, true);
        a = next_active(a + 1);
      }
    } else if constexpr (kSingle) {
      if (a0 < c1) {
        issue_one(a0, false);
        issue_one(a0, true);
      }
    } else {
      const int a1 = a0 < c1 ? next_active(a0 + 1) : c1;
      if (a0 < c1) issue_kv(a0, 0);
      if (a1 < c1) issue_kv(a1, 1);
    }
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);

  if constexpr (PIPE) {
    // Q row r, dimensions [quarter * D / 4, + D / 4) -> TMEM lane r, packed two per column from column 256 + D
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tq = *tmem_slot + 256 + D + quarter * (D / 8) + (static_cast<uint32_t>(quad * 32) << 16);
    const uint4* src = reinterpret_cast<const uint4*>(q + (static_cast<size_t>(b) * T + t) * H * D +
                                                      static_cast<size_t>(head) * D);
    uint32_t w[D / 8];
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      const uint4 v = row_valid ? src[quarter * (D / 32) + c] : make_uint4(0, 0, 0, 0);
      w[4 * c] = v.x;
      w[4 * c + 1] = v.y;
      w[4 * c + 2] = v.z;
      w[4 * c + 3] = v.w;
    }
    if constexpr (D == 128) tmem_st_u32x16(tq, w);
    else tmem_st_u32x8(tq, w);
    tmem_wait_st();
  } else {
    // Q row r, 16-byte chunks [quarter * D / 32, + D / 32) -> swizzled K-major tile (zeros for padding rows)
    const uint4* src = reinterpret_cast<const uint4*>(q + (static_cast<size_t>(b) * T + t) * H * D +
                                                      static_cast<size_t>(head) * D);
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      const int chunk = quarter * (D / 32) + c;
      store_row_swizzled(q_tile, r, chunk, row_valid ? src[chunk] : make_uint4(0, 0, 0, 0));
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (stamp) stamp[1] = global_timer_ns();
  const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t col0 = quarter * 32;        // this quarter's score columns
  const uint32_t ocol0 = quarter * kDQ;      // this quarter's output columns
  const uint32_t tmem_s = tmem + col0, tmem_pv = tmem + 128 + ocol0;

  float o[kDQ];
#pragma unroll
  for (int d = 0; d < kDQ; ++d) o[d] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  constexpr uint32_t idesc_s = idesc_bf16_f32(kRows, kKeys);
  constexpr uint32_t idesc_pv = idesc_bf16_f32(kRows, D, /*b_mn_major=*/true);
  bool ok = true;
  if constexpr (PIPE) {
    const uint32_t tmem_o = tmem + 256 + ocol0;
    const uint32_t tmem_q = tmem + 256 + D, tmem_p = tmem + 256 + D + D / 2;  // Q and P, two bf16 per column
    // warps whose 32 rows are all padding (decode: T * G rows of the 128) skip the softmax and the O updates: their
    // rows' P and O are never read back (an MMA row depends only on its own row of P)
    const bool live = m_tile * kRows + quad * 32 < T * G;
    // S of the chunk in K stage kst into score buffer sb (A = Q from TMEM), signalled on bar_s[sb]
    auto issue_s = [&](int sb, int kst) {
      tc_fence_after();
      const uint32_t ka = smem_u32(k_tiles + kst * kKVTile);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
        umma_bf16_ta(tmem + 128 * sb, tmem_q + kk * 8, desc_kmajor_sw128(ka + off), idesc_s, kk != 0);
      }
      umma_commit(&bar_s[sb]);
    };
    int c = next_active(c0);
    int c_next = c < c1 ? next_active(c + 1) : c1;
    // thread 0's ring cursors: sequence index and chunk of the next K / V load (the prologue issued kRing of each)
    int kq = 0, vq = 0, k_id = c, v_id = c, pv_done = -1;
    if (tid == 0) {
      while (kq < kRing && k_id < c1) {
        k_id = next_active(k_id + 1);
        ++kq;
      }
      vq = kq;
      v_id = k_id;
      if (c < c1) {
        ok = mbar_wait(&kv_full[0], 0, status, kStatusWaitFull, abort_flag);
        if (ok) issue_s(0, 0);
      }
    }
    // V of sequence index j may load into stage j % kRing once P . V of j - kRing has completed
    auto refill_v = [&]() {
      while (vq <= pv_done + kRing && v_id < c1) {
        issue_half(v_id, vq % kRing, true);
        v_id = next_active(v_id + 1);
        ++vq;
      }
    };
    int i = 0;
    for (; c < c1; ++i) {
      const int sb = i & 1;
      unsigned long long* fine = (stamp != nullptr && i == 2) ? stamp + 8 : nullptr;  // chunk 2, in SM cycles
      if (fine) fine[0] = clock64();
      ok = mbar_wait(&bar_s[sb], (i >> 1) & 1, status, kStatusWaitAccum, abort_flag);
      if (!ok) break;
      __syncwarp();
      tc_fence_after();
      if (stamp && i == 0) stamp[2] = global_timer_ns();
      if (fine) fine[1] = clock64();
      if (tid == 0) {
        while (kq <= i + kRing && k_id < c1) {  // S of chunk i has read its K stage
          issue_half(k_id, kq % kRing, false);
          k_id = next_active(k_id + 1);
          ++kq;
        }
        if (c_next < c1) {  // S of chunk i + 1 runs during this chunk's softmax
          const int kst = (i + 1) % kRing;
          ok = mbar_wait(&kv_full[kst], ((i + 1) / kRing) & 1, status, kStatusWaitFull, abort_flag);
          if (ok) issue_s(sb ^ 1, kst);
        }
        if (i > 0 && pv_done < i - 1 && mbar_try_wait(bar_pv, (i - 1) & 1)) pv_done = i - 1;
        refill_v();
      }
      __syncwarp();
      if (fine) fine[2] = clock64();

      float sc[32];
      if (live) tmem_ld32(tmem + 128 * sb + col0 + lane_off, sc);
      if (stamp && i == 0) stamp[3] = global_timer_ns();
      const int s0 = c * kKeys + col0;
      // Every row computes p = 2^(fma(s, scale log2(e), -m)) from its raw scores s and the maximum of its visible
      // raw scores times the scale (equal to the maximum of the scaled ones), so whether a warp takes the
      // all-visible fast path (no per-key tests) never changes a row's bits. Soft-capped scores are transformed
      // first (cap log2(e) tanh(s scale / cap)) and then enter with a unit scale.
      uint32_t vis = 0u;
      float qmax = -INFINITY;
      bool full = false;
      const float sl = capped ? 1.f : scale_log2;
      if (live) {
        vis = tail ? visible32(s0, tc_lim, 0, false, 0ull, 0, row_valid)
                   : visible32(s0, base, nn, use_mask, bits, causal_lim, row_valid);
        if (keep != nullptr) {  // evicted committed slots are invisible (new slots are never evicted)
          const uint32_t kw = keep[(static_cast<size_t>(b) * Hkv + kvh) * (S / 32) + s0 / 32];
          const int pre = min(max(base - s0, 0), 32);
          const uint32_t committed = pre >= 32 ? 0xffffffffu : ((1u << pre) - 1u);
          vis &= kw | ~committed;
        }
        if (opts.window > 0) vis &= at_or_above(s0, wlo);
        if (capped) {
#pragma unroll
          for (int j = 0; j < 32; ++j) sc[j] = cap_out * tanhf(sc[j] * cap_in);
        }
        full = __all_sync(0xffffffffu, vis == 0xffffffffu);
        float mx = -INFINITY;
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; ++j) mx = fmaxf(mx, sc[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if ((vis >> j) & 1u) mx = fmaxf(mx, sc[j]);
        }
        qmax = mx * sl;
        red[quarter * kRows + r] = qmax;
      }
      __syncthreads();
      if (fine) fine[3] = clock64();
      float alpha = 1.f, csum = 0.f;
      uint32_t packed[16];
      if (live) {
        const float cmax = fmaxf(fmaxf(red[r], red[kRows + r]), fmaxf(red[2 * kRows + r], red[3 * kRows + r]));
        // lazy rescaling: the reference maximum moves only when this chunk exceeds it by more than kLazyLog2
        if (cmax > m_run + kLazyLog2 || (m_run == -INFINITY && cmax != -INFINITY)) {
          alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - cmax);
          m_run = cmax;
        }
        const float nm = -m_run;
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float p0 = fast_exp2(fmaf(sc[j], sl, nm)), p1 = fast_exp2(fmaf(sc[j + 1], sl, nm));
            __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
            csum += p0 + p1;
            packed[j / 2] = *reinterpret_cast<uint32_t*>(&h2);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float p0 = ((vis >> j) & 1u) ? fast_exp2(fmaf(sc[j], sl, nm)) : 0.f;
            const float p1 = ((vis >> (j + 1)) & 1u) ? fast_exp2(fmaf(sc[j + 1], sl, nm)) : 0.f;
            __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
            csum += p0 + p1;
            packed[j / 2] = *reinterpret_cast<uint32_t*>(&h2);
          }
        }
      }
      l_run = l_run * alpha + csum;
      if (i > 0) {  // P . V of chunk i - 1 has finished with the P tile and the accumulator
        ok = mbar_wait(bar_pv, (i - 1) & 1, status, kStatusWaitAccum, abort_flag);
        if (!ok) break;
        __syncwarp();
        tc_fence_after();
        if (fine) fine[4] = clock64();
        if (tid == 0) {
          pv_done = i - 1;
          refill_v();
        }
        if (live && __any_sync(0xffffffffu, alpha != 1.f)) {  // rows whose maximum moved: O *= alpha (others x 1)
#pragma unroll
          for (int c16 = 0; c16 < kDQ; c16 += 16) {
            float ov[16];
            tmem_ld16(tmem_o + lane_off + c16, ov);
#pragma unroll
            for (int d = 0; d < 16; ++d) ov[d] *= alpha;
            tmem_st16(tmem_o + lane_off + c16, ov);
          }
        }
      }
      if (live) {  // this row's 32 probabilities: 16 columns of P from column 16 * quarter
        tmem_st_u32x16(tmem_p + quarter * 16 + lane_off, packed);
        tmem_wait_st();
      }
      if (stamp && i == 0) stamp[4] = global_timer_ns();
      if (fine) fine[5] = clock64();
      tc_fence_before();
      __syncthreads();
      if (fine) fine[6] = clock64();
      if (tid == 0) {
        const int vst = i % kRing;
        ok = mbar_wait(&v_full[vst], (i / kRing) & 1, status, kStatusWaitFull, abort_flag);
        if (ok) {
          tc_fence_after();
          const uint32_t va = smem_u32(v_tiles + vst * kKVTile);
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk)
            umma_bf16_ta(tmem + 256, tmem_p + kk * 8, desc_mnmajor_sw128(va + kk * 2048, kAtom), idesc_pv,
                         i > 0 || kk != 0);
          umma_commit(bar_pv);
        }
      }
      __syncwarp();
      if (stamp && i == 0) stamp[5] = global_timer_ns();
      if (fine) fine[7] = clock64();
      c = c_next;
      c_next = c_next < c1 ? next_active(c_next + 1) : c1;
    }
    // the last P . V, then the accumulator into registers for the epilogue
    if (ok && i > 0 && mbar_wait(bar_pv, (i - 1) & 1, status, kStatusWaitAccum, abort_flag)) {
      __syncwarp();
      tc_fence_after();
      if (live) {
#pragma unroll
        for (int c16 = 0; c16 < kDQ; c16 += 16) tmem_ld16(tmem_o + lane_off + c16, o + c16);
      }
    }
  } else {

    int c = next_active(c0);
    int c_next = c < c1 ? next_active(c + 1) : c1;
    for (int i = 0; c < c1 && ok; ++i) {
      const int c_after = c_next < c1 ? next_active(c_next + 1) : c1;  // the chunk two ahead (prefetched below)
      const int s = kSingle ? 0 : (i & 1);
      const uint32_t kv_phase = kSingle ? (i & 1) : ((i >> 1) & 1);
      const uint32_t ph = i & 1;
      ok = mbar_wait(&kv_full[s], kv_phase, status, kStatusWaitFull, abort_flag);
      if (!ok) break;
      if (stamp && i == 0) stamp[2] = global_timer_ns();
      if constexpr (FP8) {  // the previous chunk's S MMA has completed: the converted K tile is free
        convert_fp8_tile(raw + s * 2 * kRawTile, k_tiles, tid);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
      } else if constexpr (!kSingle) {
        if (c < q_chunks) {  // stage s was last read by chunk c - 2, whose MMAs have completed
          const size_t chunk_id = (static_cast<size_t>(b) * Hkv + kvh) * (S / kKeys) + c;
          dequant_kivi_tile(kivi + chunk_id * kivi_chunk_bytes(kivi_bits), kivi_bits, k_tiles + s * kKVTile,
                            v_tiles + s * kKVTile, tid);
          fence_async_smem();
          tc_fence_before();
          __syncthreads();
        }
      }
      if (tid == 0) {
        tc_fence_after();
        const uint32_t qa = smem_u32(q_tile), ka = smem_u32(k_tiles + (FP8 ? 0 : s * kKVTile));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
          umma_bf16(tmem, desc_kmajor_sw128(qa + off), desc_kmajor_sw128(ka + off), idesc_s, kk != 0);
        }
        umma_commit(bar_s);
      }
      __syncwarp();
      if constexpr (FP8) {  // V converts while the S MMA runs (the previous PV MMA has completed)
        convert_fp8_tile(raw + s * 2 * kRawTile + kRawTile, v_tiles, tid);
        fence_async_smem();
      }
      ok = mbar_wait(bar_s, ph, status, kStatusWaitAccum, abort_flag);
      if (!ok) break;
      __syncwarp();
      tc_fence_after();
      if constexpr (kSingle) {  // the S MMA has read K: the next chunk's K streams during this chunk's softmax and PV
        if (tid == 0 && c_next < c1) issue_one(c_next, false);
      }
      if (stamp && i == 0) stamp[3] = global_timer_ns();

      // this thread's 32 scores of the chunk
      float sc[32];
      tmem_ld16(tmem_s + lane_off, sc);
      tmem_ld16(tmem_s + lane_off + 16, sc + 16);
      const int s0 = c * kKeys + col0;
      uint32_t vis = tail ? visible32(s0, tc_lim, 0, false, 0ull, 0, row_valid)
                          : visible32(s0, base, nn, use_mask, bits, causal_lim, row_valid);
      if (keep != nullptr) {  // evicted committed slots are invisible (new slots are never evicted)
        const uint32_t kw = keep[(static_cast<size_t>(b) * Hkv + kvh) * (S / 32) + s0 / 32];
        const int pre = min(max(base - s0, 0), 32);
        const uint32_t committed = pre >= 32 ? 0xffffffffu : ((1u << pre) - 1u);
        vis &= kw | ~committed;
      }
      if (opts.window > 0) vis &= at_or_above(s0, wlo);
      float qmax = -INFINITY;
      if (capped) {
#pragma unroll
        for (int j = 0; j < 32; ++j) sc[j] = cap_out * tanhf(sc[j] * cap_in);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) sc[j] *= scale_log2;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if ((vis >> j) & 1u) qmax = fmaxf(qmax, sc[j]);
      red[quarter * kRows + r] = qmax;
      __syncthreads();
      const float cmax = fmaxf(fmaxf(red[r], red[kRows + r]), fmaxf(red[2 * kRows + r], red[3 * kRows + r]));
      if constexpr (kSingle) __syncthreads();  // every thread has read the partials before P overwrites them
      const float m_new = fmaxf(m_run, cmax);
      const float alpha = m_new == -INFINITY ? 1.f : fast_exp2(m_run - m_new);
      float csum = 0.f;
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float p0 = ((vis >> j) & 1u) ? fast_exp2(sc[j] - m_new) : 0.f;
        const float p1 = ((vis >> (j + 1)) & 1u) ? fast_exp2(sc[j + 1] - m_new) : 0.f;
        __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
        csum += __bfloat162float(h2.x) + __bfloat162float(h2.y);  // the sum of what P . V multiplies
        packed[j / 2] = *reinterpret_cast<uint32_t*>(&h2);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        store_row_swizzled(p_tile, r, quarter * 4 + u,
                           make_uint4(packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]));
      }
      l_run = l_run * alpha + csum;
      m_run = m_new;
      if (stamp && i == 0) stamp[4] = global_timer_ns();
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if constexpr (FP8) {  // every thread has converted stage s: its raw codes may be overwritten
        if (tid == 0 && c_after < c1) issue_kv(c_after, s);
      }
      if constexpr (kSingle) {
        ok = mbar_wait(&kv_full[1], ph, status, kStatusWaitFull, abort_flag);
        if (!ok) break;
      }
      if (tid == 0) {
        tc_fence_after();
        const uint32_t pa = smem_u32(p_tile), va = smem_u32(v_tiles + (FP8 ? 0 : s * kKVTile));
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * kAtom + (kk & 3) * 32;
          umma_bf16(tmem + 128, desc_kmajor_sw128(pa + a_off), desc_mnmajor_sw128(va + kk * 2048, kAtom), idesc_pv,
                    kk != 0);
        }
        umma_commit(bar_pv);
      }
      __syncwarp();
      ok = mbar_wait(bar_pv, ph, status, kStatusWaitAccum, abort_flag);
      if (!ok) break;
      __syncwarp();
      tc_fence_after();
      if (stamp && i == 0) stamp[5] = global_timer_ns();
      if constexpr (kSingle) {  // the PV MMA has read V: the next chunk's V streams during its S and softmax
        if (tid == 0 && c_next < c1) issue_one(c_next, true);
      } else if constexpr (!FP8) {
        if (tid == 0 && c_after < c1) issue_kv(c_after, s);  // both MMAs reading stage s are done
      }
      __syncwarp();
#pragma unroll
      for (int c16 = 0; c16 < kDQ; c16 += 16) {  // 16 columns at a time keeps D = 256 within the register budget
        float pv[16];
        tmem_ld16(tmem_pv + lane_off + c16, pv);
#pragma unroll
        for (int d = 0; d < 16; ++d) o[c16 + d] = o[c16 + d] * alpha + pv[d];
      }
      c = c_next;
      c_next = c_after;
    }
  }
  if (stamp) stamp[6] = global_timer_ns();
  tc_fence_before();
  __syncthreads();
  const bool failed = *abort_flag != 0;
  // row sum over the four quarters
  red[quarter * kRows + r] = l_run;
  __syncthreads();
  const float l_tot = red[r] + red[kRows + r] + red[2 * kRows + r] + red[3 * kRows + r];
  if constexpr (FP8) {  // O = s_v * (P . V8)
    const float sv = v_scale[kvh];
#pragma unroll
    for (int d = 0; d < kDQ; ++d) o[d] *= sv;
  }

  if (!failed && row_valid) {
    if (gridDim.y == 1 && !tail) {
      // a sink logit joins the denominator: rescale to the larger of the row maximum and the sink
      float m_fin = m_run, l_fin = l_tot, fac = 1.f;
      if (opts.sinks != nullptr) {
        const float s2 = opts.sinks[head] * 1.4426950408889634f;
        m_fin = fmaxf(m_run, s2);
        fac = exp2f(m_run - m_fin);
        l_fin = l_tot * fac + exp2f(s2 - m_fin);
      }
      if (lse_out != nullptr && quarter == 0)  // log2-domain log-sum-exp of the row's scaled scores
        lse_out[(static_cast<size_t>(b) * T + t) * H + head] = l_fin > 0.f ? m_fin + __log2f(l_fin) : -INFINITY;
      const float inv = l_fin > 0.f ? fac / l_fin : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(out + ((static_cast<size_t>(b) * T + t) * H + head) * D + ocol0);
#pragma unroll
      for (int c = 0; c < kDQ / 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          __nv_bfloat162 h2 = __floats2bfloat162_rn(o[c * 8 + 2 * u] * inv, o[c * 8 + 2 * u + 1] * inv);
          w[u] = *reinterpret_cast<uint32_t*>(&h2);
        }
        dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
      const size_t slot = (static_cast<size_t>(blockIdx.x) * gridDim.y + split) * kRows + r;
      float4* dst = reinterpret_cast<float4*>(ws_o + slot * D + ocol0);
#pragma unroll
      for (int c = 0; c < kDQ / 4; ++c) dst[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
      if (quarter == 0) {
        ws_ml[slot * 2] = m_run;
        ws_ml[slot * 2 + 1] = l_tot;
      }
    }
  }
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
  if (stamp) stamp[7] = global_timer_ns();
}

// Merge of the split partials, one warp per packed row (a launch of its own: one warp per row keeps the chains of
// dependent loads short, where a last-arriving CTA merging all 128 rows was measured 3x slower).
template <int D>
__global__ void __launch_bounds__(128) attn_merge_kernel(const float* __restrict__ ws_o,
                                                         const float* __restrict__ ws_ml, bf16* __restrict__ out,
                                                         int T, int H, int Hkv, int m_tiles, int splits,
                                                         float* __restrict__ lse_out,
                                                         const float* __restrict__ sinks) {
  pdl_trigger();
  pdl_wait();
  merge_row<D>(ws_o, ws_ml, out, blockIdx.x, blockIdx.y * 4 + (threadIdx.x >> 5), threadIdx.x & 31, T, H, Hkv, m_tiles,
            splits, lse_out, sinks);
}

// Exact-tail merge: one warp per packed row combines the tensor-core partials of every split with the row's tail
// keys (positions [p - tail_w, p]), which it attends itself in position order. Lane l owns dimensions E l .. E l + E
// - 1 (E = D / 32); a score is the lane products summed in a fixed order and then over the warp by a butterfly, so
// every lane holds the same value, and it is computed the same way in both passes over the tail (max, then weights).
template <int E>
__device__ __forceinline__ void load_kv(const uint8_t* base, size_t row, int lane, bool fp8, float* v) {
  if (fp8) {  // e4m3 codes (head dimension 128, E = 4)
    const uint32_t w = *reinterpret_cast<const uint32_t*>(base + row * (32 * E) + lane * E);
    const __half2 lo = __half2(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w & 0xFFFFu), __NV_E4M3));
    const __half2 hi = __half2(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w >> 16), __NV_E4M3));
    const float2 a = __half22float2(lo), b = __half22float2(hi);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    return;
  }
  const __nv_bfloat162* src = reinterpret_cast<const __nv_bfloat162*>(base + (row * (32 * E) + lane * E) * 2);
#pragma unroll
  for (int e = 0; e < E; e += 2) {
    const float2 f = __bfloat1622float2(src[e / 2]);
    v[e] = f.x;
    v[e + 1] = f.y;
  }
}

constexpr int kTailKeysMax = 128;  // committed tail (tail_w <= 64) + new keys (at most 64)
constexpr int kTailBatch = 8;      // keys whose loads are issued together

// Shared memory of the tail merge: the K rows, then the V rows, of the slots [start, end) the CTA's four rows need
// (at most tail_w committed slots below the shallowest row's position and the pass's 64 new slots).
__host__ __device__ constexpr int tail_stage_bytes(int D, bool fp8, int tail_w) {
  return 2 * (tail_w + 64) * (fp8 ? D : 2 * D);
}

template <int D>
__global__ void __launch_bounds__(128) attn_merge_tail_kernel(
    const float* __restrict__ ws_o, const float* __restrict__ ws_ml, bf16* __restrict__ out, int T, int H, int Hkv,
    int m_tiles, int splits, float* __restrict__ lse_out, const bf16* __restrict__ q,
    const uint8_t* __restrict__ k_cache, const uint8_t* __restrict__ v_cache, const int* __restrict__ kv_len,
    const int* __restrict__ n_new, const int64_t* __restrict__ mask, int S, float scale_log2, int q_offset,
    int tail_w, const float* __restrict__ k_scale, const float* __restrict__ v_scale,
    const uint32_t* __restrict__ keep, float softcap, const float* __restrict__ sinks, KVPages pages,
    unsigned* status) {
  extern __shared__ __align__(16) uint8_t tail_stage[];  // K rows, then V rows, of slots [start, end)
  __shared__ int s_row[4][kTailKeysMax];    // staged row of each of this warp's tail keys, in position order
  __shared__ float s_sc[4][kTailKeysMax];   // their scaled scores
  __shared__ int s_lo[4], s_hi[4];
  pdl_trigger();
  pdl_wait();
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, r = blockIdx.y * 4 + wid;
  const int m_tile = tile % m_tiles, bh = tile / m_tiles;
  const int b = bh / Hkv, kvh = bh % Hkv;
  const int G = H / Hkv;
  const int p = m_tile * kRows + r;
  const int t = p / G;
  const bool valid = t < T;
  const int head = kvh * G + p % G;
  const bool fp8 = k_scale != nullptr;
  const float sl = fp8 ? scale_log2 * k_scale[kvh] : scale_log2;
  const float sv = fp8 ? v_scale[kvh] : 1.f;
  const float cap_in = softcap > 0.f ? sl / (1.4426950408889634f * softcap) : 0.f;
  const float cap_out = softcap > 0.f ? softcap * 1.4426950408889634f : 0.f;
  const int base = kv_len[b], nn = n_new[b];
  const bool use_mask = mask != nullptr;
  const uint64_t bits = (use_mask && valid) ? static_cast<uint64_t>(mask[static_cast<size_t>(b) * T + t]) : 0ull;
  const int depth = max(0, use_mask ? (__popcll(bits) - 1) : (q_offset + t));  // a row seeing no new key: 0
  const int lo = max(0, base + depth - tail_w);
  constexpr int E = D / 32;
  const int n_end = min(nn, use_mask ? 64 : q_offset + t + 1);

  // The four rows' slots [start, end) are staged once with 16-byte loads that are all in flight together (the
  // rows of one token share them: a GQA group's heads are consecutive packed rows).
  if (lane == 0) {
    s_lo[wid] = valid ? min(lo, base) : INT_MAX;
    s_hi[wid] = valid ? base + max(n_end, 0) : INT_MIN;
  }
  __syncthreads();
  const int start = min(min(s_lo[0], s_lo[1]), min(s_lo[2], s_lo[3]));
  const int end = max(max(s_hi[0], s_hi[1]), max(s_hi[2], s_hi[3]));
  int rows = end > start ? end - start : 0;
  // never stage past the buffer (a range this wide cannot come from kv_len / n_new of a valid pass); bounds-checked
  // builds also report slots outside the cache
  if (rows > tail_w + 64) rows = 0;
  if (!index_ok(start >= 0 && end <= S, threadIdx.x == 0 ? status : nullptr)) rows = 0;
  const int rb = fp8 ? D : 2 * D;  // bytes of one cache row
  uint8_t* k_stage = tail_stage;
  uint8_t* v_stage = tail_stage + (tail_w + 64) * rb;
  {
    const int per_row = rb / 16;
    for (int i = threadIdx.x; i < rows * per_row; i += blockDim.x) {
      const int row = i / per_row, c = i - row * per_row;
      const size_t src = kv_row(pages, b, Hkv, kvh, S, start + row) * rb + c * 16;
      const uint4 kx = __ldg(reinterpret_cast<const uint4*>(k_cache + src));
      const uint4 vx = __ldg(reinterpret_cast<const uint4*>(v_cache + src));
      *reinterpret_cast<uint4*>(k_stage + row * rb + c * 16) = kx;
      *reinterpret_cast<uint4*>(v_stage + row * rb + c * 16) = vx;
    }
  }
  __syncthreads();
  if (!valid) return;
  // this row's split partials: O of split sp, then its (max, sum)
  auto part_o = [&](int sp) { return ws_o + ((static_cast<size_t>(tile) * splits + sp) * kRows + r) * D; };
  auto part_ml = [&](int sp) { return ws_ml + ((static_cast<size_t>(tile) * splits + sp) * kRows + r) * 2; };

  float qv[E];
  load_kv<E>(reinterpret_cast<const uint8_t*>(q), (static_cast<size_t>(b) * T + t) * H + head, lane, false, qv);

  // the tail keys in position order: committed slots [lo, base) the keep bitmap shows, then the row's own new keys
  // (ancestors and itself, in depth order), compacted with warp ballots
  int n_keys = 0;
  for (int s0 = lo; s0 < base; s0 += 32) {
    const int s = s0 + lane;
    bool vis = s < base;
    if (vis && keep != nullptr)
      vis = (keep[(static_cast<size_t>(b) * Hkv + kvh) * (S / 32) + s / 32] >> (s & 31)) & 1u;
    const unsigned ballot = __ballot_sync(0xffffffffu, vis);
    if (vis) s_row[wid][n_keys + __popc(ballot & ((1u << lane) - 1u))] = s - start;
    n_keys += __popc(ballot);
  }
  for (int j0 = 0; j0 < n_end; j0 += 32) {
    const int j = j0 + lane;
    const bool vis = j < n_end && (use_mask ? ((bits >> j) & 1ull) != 0ull : j <= q_offset + t);
    const unsigned ballot = __ballot_sync(0xffffffffu, vis);
    if (vis) s_row[wid][n_keys + __popc(ballot & ((1u << lane) - 1u))] = base + j - start;
    n_keys += __popc(ballot);
  }
  if (rows == 0) n_keys = 0;  // a failed bounds check staged nothing
  __syncwarp();

  // scores of kTailBatch keys at a time: each lane's partial dot products, then one butterfly that reduces the
  // eight sums together (after the xor-16, -8 and -4 steps a lane keeps the key of its lane bits 4..2, and each step
  // adds the same pairs warp_sum adds, so every score has warp_sum's bits)
  static_assert(kTailBatch == 8, "the transposed reduction sums eight keys");
  float mx = -INFINITY;
  for (int sp = 0; sp < splits; ++sp) {
    const float* ml = part_ml(sp);
    if (ml[1] > 0.f) mx = fmaxf(mx, ml[0]);
  }
  const float sink2 = sinks != nullptr ? sinks[head] * 1.4426950408889634f : -INFINITY;
  mx = fmaxf(mx, sink2);
  float kmx = -INFINITY;  // the tail keys' maximum (one lane per key of each batch)
  for (int i0 = 0; i0 < n_keys; i0 += kTailBatch) {
    float d[kTailBatch];
#pragma unroll
    for (int u = 0; u < kTailBatch; ++u) {
      d[u] = 0.f;
      if (i0 + u < n_keys) {
        float kv[E];
        load_kv<E>(k_stage, s_row[wid][i0 + u], lane, fp8, kv);
        float x = qv[0] * kv[0];
#pragma unroll
        for (int e = 1; e < E; ++e) x = fmaf(qv[e], kv[e], x);
        d[u] = x;
      }
    }
    float h4[4], h2[2];
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float mine = b4 ? d[j + 4] : d[j], theirs = b4 ? d[j] : d[j + 4];
      h4[j] = mine + __shfl_xor_sync(0xffffffffu, theirs, 16);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float mine = b3 ? h4[j + 2] : h4[j], theirs = b3 ? h4[j] : h4[j + 2];
      h2[j] = mine + __shfl_xor_sync(0xffffffffu, theirs, 8);
    }
    float raw;
    {
      const float mine = b2 ? h2[1] : h2[0], theirs = b2 ? h2[0] : h2[1];
      raw = mine + __shfl_xor_sync(0xffffffffu, theirs, 4);
    }
    raw += __shfl_xor_sync(0xffffffffu, raw, 2);
    raw += __shfl_xor_sync(0xffffffffu, raw, 1);
    const int u = lane >> 2;  // this lane's key of the batch
    if (i0 + u < n_keys) {
      const float sc = cap_out > 0.f ? cap_out * tanhf(raw * cap_in) : raw * sl;
      if ((lane & 3) == 0) s_sc[wid][i0 + u] = sc;
      kmx = fmaxf(kmx, sc);
    }
  }
  mx = fmaxf(mx, warp_max(kmx));
  __syncwarp();

  // the splits' partials, then the tail keys in position order
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  float denom = 0.f;
  for (int sp = 0; sp < splits; ++sp) {
    const float* ml = part_ml(sp);
    const float l = ml[1];
    if (!(l > 0.f)) continue;
    const float w = exp2f(ml[0] - mx);
    const float* v = part_o(sp) + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] += v[e] * w;
    denom += l * w;
  }
  for (int i0 = 0; i0 < n_keys; i0 += kTailBatch) {
    float vv[kTailBatch][E];
#pragma unroll
    for (int u = 0; u < kTailBatch; ++u)
      if (i0 + u < n_keys) load_kv<E>(v_stage, s_row[wid][i0 + u], lane, fp8, vv[u]);
#pragma unroll
    for (int u = 0; u < kTailBatch; ++u) {
      if (i0 + u < n_keys) {
        const float w = exp2f(s_sc[wid][i0 + u] - mx);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] += (vv[u][e] * sv) * w;
        denom += w;
      }
    }
  }
  if (sinks != nullptr) denom += exp2f(sink2 - mx);

  const float inv = denom > 0.f ? 1.f / denom : 0.f;
  if (lse_out != nullptr && lane == 0)
    lse_out[(static_cast<size_t>(b) * T + t) * H + head] = denom > 0.f ? mx + __log2f(denom) : -INFINITY;
  bf16* dst = out + ((static_cast<size_t>(b) * T + t) * H + head) * D + lane * E;
#pragma unroll
  for (int e = 0; e < E; e += 2)
    *reinterpret_cast<__nv_bfloat162*>(dst + e) = __floats2bfloat162_rn(acc[e] * inv, acc[e + 1] * inv);
}

// ---- attention scores for KV eviction (H2O / SnapKV / PyramidKV) -------------------------------------------------
// scores[b, kvh, s] += sum over the query rows of KV head kvh (the GQA group's heads x the pass's tokens) of the
// normalised attention probability exp2(S * scale_log2 - lse2[row]), for every visible slot s. One CTA per (packed
// 128-row tile, 128-key chunk): S = Q K^T on the tensor cores into TMEM, probabilities in registers, column sums
// through shared memory, one atomic add per key and tile. lse2 comes from a pass of attn_tc_kernel with lse_out.
constexpr int kScoreSmem = 2 * kTile + kRows * kKeys * 4 + 1024 + 64;

__global__ void __launch_bounds__(kThreads, 1)
    attn_scores_kernel(const bf16* __restrict__ q, const __grid_constant__ CUtensorMap tm_k,
                       const float* __restrict__ lse2, float* __restrict__ scores, const int* __restrict__ kv_len,
                       const int* __restrict__ n_new, const int64_t* __restrict__ mask, int T, int H, int Hkv, int S,
                       float scale_log2, int q_offset, int m_tiles, unsigned* status, KVPages pages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_tile = smem;
  uint8_t* k_tile = smem + kTile;
  float* colbuf = reinterpret_cast<float*>(smem + 2 * kTile);  // [128 rows][128 keys]
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + 2 * kTile + kRows * kKeys * 4);
  uint64_t* bar_s = kv_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, quarter = warp >> 2;
  const int r = quad * 32 + lane;
  const int m_tile = blockIdx.x % m_tiles, bh = blockIdx.x / m_tiles;
  const int b = bh / Hkv, kvh = bh % Hkv;
  const int G = H / Hkv;
  const int p = m_tile * kRows + r;
  const int t = p / G, head = kvh * G + p % G;
  const bool row_valid = t < T;
  const int base = kv_len[b], nn = n_new[b];
  const int c = blockIdx.y;  // key chunk
  const int end = base + nn;
  if (c * kKeys >= end) return;  // uniform: the whole CTA leaves
  const bool use_mask = mask != nullptr;
  const uint64_t bits = (row_valid && use_mask) ? static_cast<uint64_t>(mask[static_cast<size_t>(b) * T + t]) : 0ull;
  const float l2 = row_valid ? lse2[(static_cast<size_t>(b) * T + t) * H + head] : 0.f;

  if (tid == 0) {
    mbar_init(kv_full, 1);
    mbar_init(bar_s, 1);
    *abort_flag = 0;
    fence_mbar_init();
    mbar_arrive_expect_tx(kv_full, 2 * kAtom);
    const int y = static_cast<int>(kv_row(pages, b, Hkv, kvh, S, c * kKeys));
    tma_load_2d(k_tile, &tm_k, kv_full, 0, y);
    tma_load_2d(k_tile + kAtom, &tm_k, kv_full, 64, y);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, 128);
  {
    const uint4* src = reinterpret_cast<const uint4*>(q + (static_cast<size_t>(b) * T + t) * H * kDim +
                                                      static_cast<size_t>(head) * kDim);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int chunk = quarter * 4 + u;
      store_row_swizzled(q_tile, r, chunk, row_valid ? src[chunk] : make_uint4(0, 0, 0, 0));
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = mbar_wait(kv_full, 0, status, kStatusWaitFull, abort_flag);
  if (ok && tid == 0) {
    tc_fence_after();
    constexpr uint32_t idesc = idesc_bf16_f32(kRows, kKeys);
    const uint32_t qa = smem_u32(q_tile), ka = smem_u32(k_tile);
#pragma unroll
    for (int kk = 0; kk < kDim / 16; ++kk) {
      const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
      umma_bf16(tmem, desc_kmajor_sw128(qa + off), desc_kmajor_sw128(ka + off), idesc, kk != 0);
    }
    umma_commit(bar_s);
  }
  __syncwarp();
  ok = ok && mbar_wait(bar_s, 0, status, kStatusWaitAccum, abort_flag);
  __syncthreads();
  ok = !*abort_flag;
  tc_fence_after();
  const uint32_t col0 = quarter * 32;
  if (ok) {
    float sc[32];
    tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + col0, sc);
    tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + col0 + 16, sc + 16);
    const uint32_t vis = visible32(c * kKeys + col0, base, nn, use_mask, bits, q_offset + t + 1, row_valid);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      colbuf[r * kKeys + col0 + j] = ((vis >> j) & 1u) ? fast_exp2(sc[j] * scale_log2 - l2) : 0.f;
  }
  __syncthreads();
  if (ok && tid < kKeys) {
    float acc = 0.f;
    for (int row = 0; row < kRows; ++row) acc += colbuf[row * kKeys + tid];
    const int slot = c * kKeys + tid;
    if (slot < end && acc != 0.f) atomicAdd(scores + (static_cast<size_t>(b) * Hkv + kvh) * S + slot, acc);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ---- KIVI quantisation of committed chunks ------------------------------------------------------------------------
// CTA (layer, row * H_kv + head, i) quantises chunk qc = chunks[row] + i of the bf16 cache when it lies at least
// `residual` slots behind the row's committed length (its tokens can no longer move). 128 threads: thread d owns
// key channel d (per-channel scales over the chunk's tokens), then thread t owns token t (per-token value scales).
__global__ void __launch_bounds__(128) kivi_quantize_kernel(const bf16* __restrict__ cache, uint8_t* __restrict__ kivi,
                                                            const int* __restrict__ kv_len,
                                                            const int* __restrict__ chunks, int B, int Hkv, int S,
                                                            int bits, int residual, KVLayout layout) {
  pdl_trigger();
  pdl_wait();
  const int layer = blockIdx.x, bh = blockIdx.y, b = bh / Hkv;
  const int c = chunks[b] + static_cast<int>(blockIdx.z);
  if ((c + 1) * kKeys + residual > kv_len[b]) return;
  if (!index_ok(c >= 0 && (c + 1) * kKeys <= S, nullptr)) return;
  __shared__ uint8_t codes[kKeys][kDim + 4];
  const int tid = threadIdx.x;
  const float levels = static_cast<float>((1 << bits) - 1);
  const int kvh = bh % Hkv;
  const bf16* K = cache + kv_layer_row(layout, layer, 0, b, Hkv, kvh, S, c * kKeys) * kDim;
  const bf16* V = cache + kv_layer_row(layout, layer, 1, b, Hkv, kvh, S, c * kKeys) * kDim;
  uint8_t* out = kivi + ((static_cast<size_t>(layer) * B * Hkv + bh) * (S / kKeys) + c) * kivi_chunk_bytes(bits);
  bf16* ks = reinterpret_cast<bf16*>(out + kivi_code_bytes(bits));
  bf16* kz = ks + kDim;
  uint8_t* vc = out + kivi_code_bytes(bits) + 2 * kDim * 2;
  bf16* vs = reinterpret_cast<bf16*>(vc + kivi_code_bytes(bits));
  bf16* vz = vs + kKeys * (kDim / 32);
  // keys: channel tid over the chunk's 128 tokens
  {
    float lo = INFINITY, hi = -INFINITY;
    for (int t = 0; t < kKeys; ++t) {
      const float x = __bfloat162float(K[t * kDim + tid]);
      lo = fminf(lo, x);
      hi = fmaxf(hi, x);
    }
    const bf16 sb = __float2bfloat16((hi - lo) / levels), zb = __float2bfloat16(lo);
    const float sc = __bfloat162float(sb) > 0.f ? __bfloat162float(sb) : 1.f, z = __bfloat162float(zb);
    ks[tid] = __float2bfloat16(sc);
    kz[tid] = zb;
    for (int t = 0; t < kKeys; ++t) {
      const float x = __bfloat162float(K[t * kDim + tid]);
      codes[t][tid] = static_cast<uint8_t>(fminf(fmaxf(rintf(__fdiv_rn(x - z, sc)), 0.f), levels));
    }
  }
  __syncthreads();
  {  // pack token tid's key codes: 8 (2-bit) or 2 (4-bit) codes per byte ... as words of 8 codes
    const int per_word = bits == 2 ? 8 : 8;
    for (int ch0 = 0; ch0 < kDim; ch0 += per_word) {
      uint32_t w = 0;
      for (int e = 0; e < 8; ++e) w |= static_cast<uint32_t>(codes[tid][ch0 + e]) << (e * bits);
      if (bits == 2) *reinterpret_cast<uint16_t*>(out + tid * (kDim * 2 / 8) + ch0 / 4) = static_cast<uint16_t>(w);
      else *reinterpret_cast<uint32_t*>(out + tid * (kDim * 4 / 8) + ch0 / 2) = w;
    }
  }
  // values: token tid, groups of 32 channels
  const bf16* vrow = V + static_cast<size_t>(tid) * kDim;
  for (int g = 0; g < kDim / 32; ++g) {
    float lo = INFINITY, hi = -INFINITY;
    for (int d = 0; d < 32; ++d) {
      const float x = __bfloat162float(vrow[g * 32 + d]);
      lo = fminf(lo, x);
      hi = fmaxf(hi, x);
    }
    const bf16 sb = __float2bfloat16((hi - lo) / levels), zb = __float2bfloat16(lo);
    const float sc = __bfloat162float(sb) > 0.f ? __bfloat162float(sb) : 1.f, z = __bfloat162float(zb);
    vs[tid * 4 + g] = __float2bfloat16(sc);
    vz[tid * 4 + g] = zb;
    for (int d0 = 0; d0 < 32; d0 += 8) {
      uint32_t w = 0;
      for (int e = 0; e < 8; ++e) {
        const float x = __bfloat162float(vrow[g * 32 + d0 + e]);
        w |= static_cast<uint32_t>(fminf(fmaxf(rintf(__fdiv_rn(x - z, sc)), 0.f), levels)) << (e * bits);
      }
      const int ch0 = g * 32 + d0;
      if (bits == 2) *reinterpret_cast<uint16_t*>(vc + tid * (kDim * 2 / 8) + ch0 / 4) = static_cast<uint16_t>(w);
      else *reinterpret_cast<uint32_t*>(vc + tid * (kDim * 4 / 8) + ch0 / 2) = w;
    }
  }
}

__global__ void kivi_advance_kernel(const int* __restrict__ kv_len, int* __restrict__ chunks, int B, int max_new,
                                    int residual) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int ready = max(0, (kv_len[b] - residual) / kKeys);
  chunks[b] = max(chunks[b], min(ready, chunks[b] + max_new));
}

}  // namespace

// The split over keys depends on the batch, the KV heads and the cache size only (not on the number of query
// tokens), so a one-token pass and a verification pass reduce a row's keys in the same order.
// With a sliding window the split covers the window's span (the chunks one tile's rows can see: the window, up to
// 128 positions of rows, and one chunk of misalignment) plus one group, because the CTAs start at the absolute
// group of their first visible chunk.
AttnPlan attention_plan(int B, int T, int H, int Hkv, int S, int num_sms, bool tail, int D, int window) {
  AttnPlan plan;
  const int G = H / Hkv;
  plan.m_tiles = (T * G + kRows - 1) / kRows;
  const int total_chunks = (S + kKeys - 1) / kKeys;
  const int span = window > 0 ? std::min(total_chunks, (window + 2 * kKeys - 1) / kKeys + 1) : total_chunks;
  const int heads = B * Hkv;
  int splits = 1;
  // one wave of splits per (row, KV head) for a decode pass; the split count never depends on T, so a tree pass and
  // a one-token pass reduce a row's keys in the same groups (the exact-tail guarantee)
  if (heads < num_sms) splits = std::min(span, std::max(1, num_sms / heads));
  plan.chunks_per_split = (span + splits - 1) / splits;
  plan.splits = (span + plan.chunks_per_split - 1) / plan.chunks_per_split;
  if (span < total_chunks)
    plan.splits = std::min(plan.splits + 1, (total_chunks + plan.chunks_per_split - 1) / plan.chunks_per_split);
  const long ctas = static_cast<long>(heads) * plan.m_tiles;
  plan.ws_floats = (plan.splits > 1 || tail) ? ctas * plan.splits * kRows * (D + 2) : 0;
  plan.tail = tail;
  return plan;
}

int launch_attention(const void* q, const CUtensorMap* tm_k, const CUtensorMap* tm_v, void* out, float* ws,
                     const int* kv_len, const int* n_new, const int64_t* mask, int B, int T, int H, int Hkv, int D,
                     int S, float scale, int q_offset, const AttnPlan& plan, unsigned* status, cudaStream_t stream,
                     unsigned long long* trace, const float* k_scale, const float* v_scale, const uint32_t* keep,
                     float* lse_out, const uint8_t* kivi, const int* kivi_chunks, int kivi_bits, int tail_w,
                     const void* k_cache, const void* v_cache, const AttnOpts& opts, const KVPages& pages) {
  if (kivi != nullptr && (k_scale != nullptr || (kivi_bits != 2 && kivi_bits != 4))) return -1;
  if (tail_w < 0 || tail_w > 64 || (tail_w > 0 && (!plan.tail || k_cache == nullptr || v_cache == nullptr)))
    return -1;
  if ((D != 64 && D != 128 && D != 256) || H % Hkv != 0) return -1;
  if (opts.softcap < 0.f || opts.window < 0) return -1;
  // a window must cover a tree (up to 64 new keys) and the exact tail: those keys are never filtered
  if (opts.window > 0 && ((mask != nullptr && opts.window <= 64) || (tail_w > 0 && opts.window <= tail_w)))
    return -2;
  if (mask != nullptr && T > 64) return -1;
  const bool fp8 = k_scale != nullptr;
  if (fp8 && v_scale == nullptr) return -1;
  if (D != 128 && (fp8 || kivi != nullptr)) return -1;  // fp8 and KIVI caches at head dimension 128
  const int ctas = B * Hkv * plan.m_tiles;
  const bool staged = plan.splits > 1 || tail_w > 0;  // partials go through the workspace and a merge
  float* ws_o = staged ? ws : nullptr;
  float* ws_ml = staged ? ws + static_cast<size_t>(ctas) * plan.splits * kRows * D : nullptr;
  dim3 grid(ctas, plan.splits);
  const float sl2 = scale * 1.4426950408889634f;
  cudaError_t launch_err = cudaSuccess;  // a refused launch (e.g. a shared-memory request) returns -3
  auto note = [&](cudaError_t e) {
    if (e != cudaSuccess && launch_err == cudaSuccess) launch_err = e;
  };
  auto run = [&](auto kernel, int smem) {
    note(set_max_smem(kernel, smem));
    note(launch_pdl(kernel, grid, dim3(kThreads), smem, stream, static_cast<const bf16*>(q), *tm_k, *tm_v,
               static_cast<bf16*>(out), ws_o, ws_ml, kv_len, n_new, mask, T, H, Hkv, S, sl2, q_offset,
               plan.chunks_per_split, plan.m_tiles, status, trace, k_scale, v_scale, keep, lse_out, kivi, kivi_chunks,
               kivi_bits, tail_w, opts, pages));
  };
  // bf16 caches without KIVI codes take the pipelined walk (ECZ_ATTN_PIPE=0 selects the serial one, for comparison)
  static const bool pipe_env = [] {
    const char* v = std::getenv("ECZ_ATTN_PIPE");
    return v == nullptr || v[0] != '0';
  }();
  const bool pipe = pipe_env && kivi == nullptr;
  if (D == 64) {
    if (pipe) run(attn_tc_kernel<false, 64, true>, attn_pipe_smem_bytes(64));
    else run(attn_tc_kernel<false, 64>, attn_smem_bytes(64));
  } else if (D == 256) {
    run(attn_tc_kernel<false, 256>, attn_smem_bytes(256));
  } else if (fp8) {
    run(attn_tc_kernel<true, 128>, kSmem);
  } else if (pipe) {
    run(attn_tc_kernel<false, 128, true>, attn_pipe_smem_bytes(128));
  } else {
    run(attn_tc_kernel<false, 128>, kSmem);
  }
  dim3 mgrid(ctas, kRows / 4);
  if (tail_w > 0) {
    auto merge = D == 64 ? attn_merge_tail_kernel<64> : D == 256 ? attn_merge_tail_kernel<256>
                                                                 : attn_merge_tail_kernel<128>;
    const int stage = tail_stage_bytes(D, fp8, tail_w);
    if (stage > 48 * 1024) note(set_max_smem(merge, stage));
    note(launch_pdl(merge, mgrid, dim3(128), stage, stream, static_cast<const float*>(ws_o),
                    static_cast<const float*>(ws_ml), static_cast<bf16*>(out), T, H, Hkv, plan.m_tiles, plan.splits,
                    lse_out, static_cast<const bf16*>(q), static_cast<const uint8_t*>(k_cache),
                    static_cast<const uint8_t*>(v_cache), kv_len, n_new, mask, S, sl2, q_offset, tail_w, k_scale,
                    v_scale, keep, opts.softcap, opts.sinks, pages, status));
  } else if (plan.splits > 1) {
    auto merge = D == 64 ? attn_merge_kernel<64> : D == 256 ? attn_merge_kernel<256> : attn_merge_kernel<128>;
    note(launch_pdl(merge, mgrid, dim3(128), 0, stream, static_cast<const float*>(ws_o),
                    static_cast<const float*>(ws_ml), static_cast<bf16*>(out), T, H, Hkv, plan.m_tiles,
                    plan.splits, lse_out, opts.sinks));
  }
  return launch_err == cudaSuccess ? 0 : -3;
}

int launch_attention_scores(const void* q, const CUtensorMap* tm_k, const float* lse2, float* scores,
                            const int* kv_len, const int* n_new, const int64_t* mask, int B, int T, int H, int Hkv,
                            int D, int S, float scale, int q_offset, unsigned* status, cudaStream_t stream,
                            const KVPages& pages) {
  if (D != kDim || H % Hkv != 0 || (mask != nullptr && T > 64)) return -1;
  set_max_smem(attn_scores_kernel, kScoreSmem);
  const int G = H / Hkv;
  const int m_tiles = (T * G + kRows - 1) / kRows;
  dim3 grid(B * Hkv * m_tiles, (S + kKeys - 1) / kKeys);
  launch_pdl(attn_scores_kernel, grid, dim3(kThreads), kScoreSmem, stream, static_cast<const bf16*>(q), *tm_k, lse2,
             scores, kv_len, n_new, mask, T, H, Hkv, S, scale * 1.4426950408889634f, q_offset, m_tiles, status,
             pages);
  return 0;
}

int kivi_chunk_size(int bits) { return kivi_chunk_bytes(bits); }

int launch_kivi_quantize(const void* cache, void* kivi, const int* kv_len, int* chunks, int L, int B, int Hkv, int S,
                         int D, int bits, int residual, int max_new, cudaStream_t stream, const KVLayout& layout) {
  if (D != kDim || S % kKeys != 0 || (bits != 2 && bits != 4) || max_new < 1) return -1;
  launch_pdl(kivi_quantize_kernel, dim3(L, B * Hkv, max_new), dim3(kKeys), 0, stream,
             static_cast<const bf16*>(cache), static_cast<uint8_t*>(kivi), kv_len, static_cast<const int*>(chunks), B,
             Hkv, S, bits, residual, layout);
  launch_pdl(kivi_advance_kernel, dim3((B + 127) / 128), dim3(128), 0, stream, kv_len, chunks, B, max_new, residual);
  return 0;
}

}  // namespace ecz
