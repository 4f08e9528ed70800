// tcgen05 / TMA GEMM for the decoder's projections: Y[M, N] = X[M, K] . W[N, K]^T (bf16 in, fp32 accumulate).
//
// Decode passes have few token rows (a verified draft tree is ~61 rows per sequence) and large weights, so the
// kernel swaps the operands: the UMMA "A" operand is a 128-row tile of W (128 output features on the 128 TMEM
// lanes) and the "B" operand a BN-row tile of X (tokens on the UMMA N side, BN in {32, 64, 128, 256}). The
// accumulator D[n, m] lives in TMEM (BN fp32 columns); the epilogue reads it with tcgen05.ld and writes Y[m, n].
//
// Pipeline: one elected TMA thread streams (W, X) K-slices of 64 elements (128-byte swizzled rows) into a ring of
// `STAGES` shared-memory stages guarded by full/empty mbarriers; one elected MMA thread issues 4 UMMAs (K = 16
// each) per stage and releases the stage with tcgen05.commit; the accumulator barrier wakes the epilogue.
//
// When the tile grid cannot fill the 148 SMs, K is split over `splits` CTAs per tile, each writing fp32 partials
// to a workspace that a second kernel sums (and rounds to bf16). Every wait is bounded (common.cuh).
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

constexpr int kBM = 128;  // W rows per tile (UMMA M)
constexpr int kBK = 64;   // K elements per stage (one 128-byte swizzle row)
constexpr int kABytes = kBM * kBK * 2;

// kOcc CTAs share an SM: the stage ring is sized so that they fit its 228 KB of shared memory.
template <int BN, int kOcc = 1>
struct GemmCfg {
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = std::min(8, ((kOcc == 1 ? 200 : 100) * 1024) / kStageBytes);
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// Skinny tiles (BN <= 64) run two CTAs per SM in the split kernels, so one CTA's prologue and epilogue overlap
// the other's weight stream.
template <int BN>
constexpr int split_occupancy() { return BN <= 64 ? 2 : 1; }

// Push mode (tensor-parallel row-parallel projections): output tiles go straight into slot `rank` of every peer's
// receive buffer (bf16 [rows, N], parity `parity`), and the last tile writer of the grid announces the arrival to
// every peer, as the push kernel of comm.cu does.
__device__ __forceinline__ bf16* peer_slot(const PeerOut& peer, int p) {
  return reinterpret_cast<bf16*>(static_cast<uint8_t*>(peer.ptrs.ptr[p]) + peer.control_bytes) +
         (static_cast<long>(peer.parity) * peer.world + peer.rank) * peer.slot_elems;
}

__device__ __forceinline__ void push_signal(const PeerOut& peer, bool wrote, unsigned writers_total, int parity) {
  // every CTA that stored a tile counts itself; the last one signals the peers (writers_total = tiles). The CTA
  // barrier orders all threads' stores before thread 0's system-scope fence.
  __syncthreads();
  if (threadIdx.x == 0 && wrote) {
    __threadfence_system();
    unsigned* own = reinterpret_cast<unsigned*>(peer.ptrs.ptr[peer.rank]);
    const unsigned done = atomicAdd(own + kSpPushDone, 1u);  // push_done of the control block
    if (done == writers_total - 1) {
      own[kSpPushDone] = 0;
      __threadfence_system();
      for (int p = 0; p < peer.world; ++p)
        atomicAdd_system(static_cast<unsigned*>(peer.ptrs.ptr[p]) + kSpRsArrive + parity, 1u);
    }
  }
}

// Mode-1 (reduce-scatter) destination of output element (m, n): the owner rank's partial slot of this rank.
__device__ __forceinline__ bf16* scatter_dst(const PeerOut& peer, int parity, int m, int n, int N) {
  const int owner = m / peer.shard_rows;
  const int local = m - owner * peer.shard_rows;
  bf16* base = reinterpret_cast<bf16*>(static_cast<uint8_t*>(peer.ptrs.ptr[owner]) + peer.data_off);
  return base + ((static_cast<size_t>(parity) * peer.world + peer.rank) * peer.shard_max + local) *
                    static_cast<size_t>(N) + n;
}

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The all-gather wait of an AG -> GEMM consumer (one thread): returns the round's parity. On timeout the status
// records kStatusWaitPeer and the GEMM proceeds on whatever the buffer holds (its copies then complete normally).
__device__ __forceinline__ int ag_wait(const AgWait& ag, unsigned* status) {
  const int par = static_cast<int>(ag.ctrl[kSpAgRound] & 1u);
  const unsigned* flag = ag.ctrl + kSpAgArrive + par;
  if (ld_acquire_sys_u32(flag) < static_cast<unsigned>(ag.world)) {
    const unsigned long long start = global_timer_ns();
    while (ld_acquire_sys_u32(flag) < static_cast<unsigned>(ag.world)) {
      if (global_timer_ns() - start > kWaitLimitNs) {
        atomicOr(status, kStatusWaitPeer);
        break;
      }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");  // the peers' stores become visible to TMA reads
  return par;
}

// The last CTA of an AG -> GEMM consumer resets the round's arrival count and advances the round.
__device__ __forceinline__ void ag_release(const AgWait& ag, int par, unsigned ctas) {
  __threadfence();
  if (atomicAdd(ag.ctrl + kSpAgDone, 1u) == ctas - 1) {
    ag.ctrl[kSpAgDone] = 0;
    ag.ctrl[kSpAgArrive + par] = 0;
    ag.ctrl[kSpAgRound] += 1u;
    __threadfence();
  }
}

template <int BN, int OCC = 1>
__global__ void __launch_bounds__(128, OCC)
    gemm_swapab_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                       bf16* __restrict__ y, float* __restrict__ ws, int* __restrict__ counters, int M, int N,
                       int K, int kb_per_split, unsigned* status, PeerOut peer, AgWait ag,
                       const __grid_constant__ CUtensorMap tm_x1) {
  using Cfg = GemmCfg<BN, OCC>;
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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBM, m0 = blockIdx.y * BN, split = blockIdx.z;
  const int total_kb = (K + kBK - 1) / kBK;
  const int kb0 = split * kb_per_split;
  const int nkb = std::min(kb_per_split, total_kb - kb0);

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

  int ag_par = 0;
  if (nkb > 0 && warp == 0 && lane == 0) {
    // ---- TMA producer ----
    // The weights do not depend on the previous kernel: the first ring of weight tiles is requested before
    // griddepcontrol.wait, so it streams while the predecessor finishes; activations follow after the wait (and,
    // for an all-gather -> GEMM, after every rank's rows arrived in this round's half of the buffer).
    const int pre = nkb < S ? nkb : S;
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(&full[kb], Cfg::kStageBytes);
      tma_load_2d(a_tiles + kb * kABytes, &tm_w, &full[kb], (kb0 + kb) * kBK, n0);
    }
    pdl_wait();
    if (ag.ctrl != nullptr) ag_par = ag_wait(ag, status);
    const CUtensorMap* mx = ag_par ? &tm_x1 : &tm_x;
    for (int kb = 0; kb < pre; ++kb) tma_load_2d(b_tiles + kb * Cfg::kBBytes, mx, &full[kb], (kb0 + kb) * kBK, m0);
    for (int kb = pre; kb < nkb; ++kb) {
      const int s = kb % S;
      const uint32_t use = kb / S;
      if (!mbar_wait(&empty[s], (use & 1u) ^ 1u, status, kStatusWaitEmpty, abort_flag)) break;
      mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
      const int kx = (kb0 + kb) * kBK;
      tma_load_2d(a_tiles + s * kABytes, &tm_w, &full[s], kx, n0);
      tma_load_2d(b_tiles + s * Cfg::kBBytes, mx, &full[s], kx, m0);
    }
  } else if (nkb > 0 && warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S;
      const uint32_t use = kb / S;
      if (!mbar_wait(&full[s], use & 1u, status, kStatusWaitFull, abort_flag)) break;
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
    umma_commit(accum);  // also on abort, so the epilogue's wait ends
  }
  __syncwarp();

  // ---- epilogue: warp w owns TMEM lanes 32w..32w+31 = output features n0 + 32w + lane ----
  if (nkb > 0) mbar_wait(accum, 0, status, kStatusWaitAccum, abort_flag);
  pdl_wait();       // no global write before the predecessor grid has completed
  __syncthreads();  // a failed wait set abort_flag; the decision below is uniform across the CTA
  tc_fence_after();
  const bool ok = nkb > 0 && !*abort_flag;
  const int n = n0 + warp * 32 + lane;
  if (ok) {
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      tmem_ld16(lane_base + c, v);
      if (n < N) {
        if (ws == nullptr) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c + j;
            if (m < M) {
              const bf16 o = __float2bfloat16(v[j]);
              if (peer.world == 0) {
                y[static_cast<size_t>(m) * N + n] = o;
              } else {
                for (int p = 0; p < peer.world; ++p) peer_slot(peer, p)[static_cast<size_t>(m) * N + n] = o;
              }
            }
          }
        } else {
          float* part = ws + static_cast<size_t>(split) * M * N;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c + j;
            if (m < M) part[static_cast<size_t>(m) * N + n] = v[j];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
  bool wrote = ok && ws == nullptr;  // this CTA stored its output tile (split-K: only the tile's last CTA does)
  if (ok && ws != nullptr && counters != nullptr) {
    // In-kernel split-K reduction: the last CTA of this output tile (counted with a self-resetting atomic) sums
    // the partials of all splits in split order, so the result does not depend on which CTA finishes last.
    __shared__ int last;
    __threadfence();
    __syncthreads();
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    if (threadIdx.x == 0) last = atomicAdd(&counters[tile], 1) == static_cast<int>(gridDim.z) - 1;
    __syncthreads();
    if (last) {
      __threadfence();
      // thread t sums 4 consecutive columns (group t % 32) of rows m0 + t / 32, + 4, + 8, ...; four rows' loads of
      // every split are issued before they are summed, in split order
      const int cg = threadIdx.x & 31, rp = threadIdx.x >> 5;
      const int col = n0 + cg * 4;
      const int nsplit = static_cast<int>(gridDim.z);
      const int m_end = min(M, m0 + BN);
      if (col < N) {
        for (int mb = m0 + rp; mb < m_end; mb += 16) {
          float4 acc[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int sp = 0; sp < nsplit; ++sp) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int m = mb + 4 * u;
              v[u] = m < m_end ? __ldcg(reinterpret_cast<const float4*>(ws + (static_cast<size_t>(sp) * M + m) * N + col))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              acc[u].x += v[u].x; acc[u].y += v[u].y; acc[u].z += v[u].z; acc[u].w += v[u].w;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int m = mb + 4 * u;
            if (m < m_end) {
              __nv_bfloat162 lo = __floats2bfloat162_rn(acc[u].x, acc[u].y);
              __nv_bfloat162 hi = __floats2bfloat162_rn(acc[u].z, acc[u].w);
              uint2 packed;
              packed.x = *reinterpret_cast<uint32_t*>(&lo);
              packed.y = *reinterpret_cast<uint32_t*>(&hi);
              if (peer.world == 0) {
                *reinterpret_cast<uint2*>(y + static_cast<size_t>(m) * N + col) = packed;
              } else {
                for (int p = 0; p < peer.world; ++p)
                  *reinterpret_cast<uint2*>(peer_slot(peer, p) + static_cast<size_t>(m) * N + col) = packed;
              }
            }
          }
        }
      }
      if (threadIdx.x == 0) counters[tile] = 0;
    }
    wrote = last;
  }
  if (peer.world > 0 && ok) push_signal(peer, wrote, gridDim.x * gridDim.y, peer.parity);
  if (ag.ctrl != nullptr && threadIdx.x == 0) {  // the last CTA closes the all-gather round (see ag_release)
    const int par = nkb > 0 ? ag_par : static_cast<int>(ag.ctrl[kSpAgRound] & 1u);
    ag_release(ag, par, gridDim.x * gridDim.y * gridDim.z);
  }
}

__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws, bf16* __restrict__ y,
                                                             long total, int splits) {
  pdl_trigger();
  pdl_wait();
  for (long i = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) * 4; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x * 4) {
    float4 acc = *reinterpret_cast<const float4*>(ws + i);
    for (int s = 1; s < splits; ++s) {
      const float4 p = *reinterpret_cast<const float4*>(ws + static_cast<size_t>(s) * total + i);
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(y + i) = packed;
  }
}

// flags: bit 0 = two CTAs per SM for skinny tiles, bit 1 = leave the fp32 partials in ws (no reduction)
template <int BN>
int run_gemm(const CUtensorMap& tm_w, const CUtensorMap& tm_x, void* y, float* ws, int* counters, int M, int N,
             int K, int splits, unsigned* status, cudaStream_t stream, const PeerOut& peer, int flags = 0,
             const AgWait& ag = AgWait{}, const CUtensorMap* tm_x1 = nullptr) {
  const CUtensorMap& x1 = tm_x1 != nullptr ? *tm_x1 : tm_x;
  constexpr int kOcc2 = split_occupancy<BN>();
  const bool occ2 = (flags & 1) != 0 && kOcc2 == 2;
  set_max_smem(gemm_swapab_kernel<BN, 1>, GemmCfg<BN, 1>::kSmem);
  set_max_smem(gemm_swapab_kernel<BN, kOcc2>, GemmCfg<BN, kOcc2>::kSmem);
  const int total_kb = (K + kBK - 1) / kBK;
  const int kbps = (total_kb + splits - 1) / splits;
  splits = (total_kb + kbps - 1) / kbps;  // no empty split
  dim3 grid((N + kBM - 1) / kBM, (M + BN - 1) / BN, splits);
  if (occ2) {
    launch_pdl(gemm_swapab_kernel<BN, kOcc2>, grid, dim3(128), GemmCfg<BN, kOcc2>::kSmem, stream, tm_w, tm_x,
               static_cast<bf16*>(y), splits > 1 ? ws : nullptr, splits > 1 ? counters : nullptr, M, N, K, kbps,
               status, peer, ag, x1);
  } else {
    launch_pdl(gemm_swapab_kernel<BN, 1>, grid, dim3(128), GemmCfg<BN, 1>::kSmem, stream, tm_w, tm_x,
               static_cast<bf16*>(y), splits > 1 ? ws : nullptr, splits > 1 ? counters : nullptr, M, N, K, kbps,
               status, peer, ag, x1);
  }
  if (splits > 1 && counters == nullptr && (flags & 2) == 0) {
    const long total = static_cast<long>(M) * N;
    const int blocks = static_cast<int>(std::min<long>((total / 4 + 255) / 256, 148L * 8));
    launch_pdl(splitk_reduce_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, stream,
               static_cast<const float*>(ws), static_cast<bf16*>(y), total, splits);
  }
  return 0;
}

// ---------------------------------------------------------------------------------------------------------------
// Cluster split-K GEMM (the main path when the tiles cannot cover the SMs)
// ---------------------------------------------------------------------------------------------------------------
// The `splits` K-slices of one output tile form a thread-block cluster (1 x 1 x splits). Every CTA runs the
// TMA/UMMA pipeline over its K-slice, parks its fp32 partial [BN rows][128 features] in its own shared memory (the
// drained stage ring), and after a cluster barrier reduces rows r = rank, rank + splits, ... by reading all partials
// over DSMEM in split order (deterministic, independent of scheduling). No global workspace is touched.

template <int BN>
__global__ void __launch_bounds__(128, split_occupancy<BN>())
    gemm_cluster_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                        bf16* __restrict__ y, int M, int N, int K, int kb_per_split, unsigned* status, PeerOut peer,
                        AgWait ag, const __grid_constant__ CUtensorMap tm_x1) {
  using Cfg = GemmCfg<BN, split_occupancy<BN>()>;
  constexpr int S = Cfg::kStages;
  static_assert(BN * kBM * 4 <= S * Cfg::kStageBytes, "the partial tile must fit the stage ring");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = smem + S * kABytes;
  float* partial = reinterpret_cast<float*>(smem);  // reused after the pipeline drained: [BN][128] fp32
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBM, m0 = blockIdx.y * BN;
  const int splits = static_cast<int>(gridDim.z);
  const uint32_t rank = splits > 1 ? cluster_ctarank() : 0u;
  const int total_kb = (K + kBK - 1) / kBK;
  const int kb0 = static_cast<int>(blockIdx.z) * kb_per_split;
  const int nkb = max(0, min(kb_per_split, total_kb - kb0));

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

  int ag_par = 0;
  if (nkb > 0 && warp == 0 && lane == 0) {
    const int pre = nkb < S ? nkb : S;
    for (int kb = 0; kb < pre; ++kb) {  // weights first: they do not depend on the previous kernel
      mbar_arrive_expect_tx(&full[kb], Cfg::kStageBytes);
      tma_load_2d(a_tiles + kb * kABytes, &tm_w, &full[kb], (kb0 + kb) * kBK, n0);
    }
    pdl_wait();
    if (ag.ctrl != nullptr) ag_par = ag_wait(ag, status);  // all-gather -> GEMM: the rows of every rank arrived
    const CUtensorMap* mx = ag_par ? &tm_x1 : &tm_x;
    for (int kb = 0; kb < pre; ++kb) tma_load_2d(b_tiles + kb * Cfg::kBBytes, mx, &full[kb], (kb0 + kb) * kBK, m0);
    for (int kb = pre; kb < nkb; ++kb) {
      const int s = kb % S;
      const uint32_t use = kb / S;
      if (!mbar_wait(&empty[s], (use & 1u) ^ 1u, status, kStatusWaitEmpty, abort_flag)) break;
      mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
      const int kx = (kb0 + kb) * kBK;
      tma_load_2d(a_tiles + s * kABytes, &tm_w, &full[s], kx, n0);
      tma_load_2d(b_tiles + s * Cfg::kBBytes, mx, &full[s], kx, m0);
    }
  } else if (nkb > 0 && warp == 1 && lane == 0) {
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
  if (nkb > 0) mbar_wait(accum, 0, status, kStatusWaitAccum, abort_flag);
  pdl_wait();
  __syncthreads();
  tc_fence_after();
  const bool ok = nkb > 0 && !*abort_flag;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const int feat = warp * 32 + lane;  // this thread's TMEM lane = output feature n0 + feat
  // reduce-scatter round parity: this rank's own round counter (its predecessor grids have completed)
  const int rs_par = peer.mode == 1 ? static_cast<int>(static_cast<const unsigned*>(peer.ptrs.ptr[peer.rank])[kSpRsRound] & 1u)
                                    : peer.parity;
  if (splits == 1) {
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(lane_base + c, v);
        const int n = n0 + feat;
        if (n < N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c + j;
            if (m >= M) continue;
            const bf16 o = __float2bfloat16(v[j]);
            if (peer.world == 0) y[static_cast<size_t>(m) * N + n] = o;
            else if (peer.mode == 1) *scatter_dst(peer, rs_par, m, n, N) = o;
            else for (int p = 0; p < peer.world; ++p) peer_slot(peer, p)[static_cast<size_t>(m) * N + n] = o;
          }
        }
      }
    }
  } else {
    // park the partial (zeros after a failure, so the reduction still runs on every CTA of the cluster)
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      tmem_ld16(lane_base + c, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) partial[(c + j) * kBM + feat] = ok ? v[j] : 0.f;
    }
    cluster_sync();  // every partial of the tile is in place
    // this CTA reduces rows j = rank + splits * i; thread t sums features [4 (t % 32), + 4) of rows i = t / 32 + 4k
    const int cg = threadIdx.x & 31, rp = threadIdx.x >> 5;
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
        uint2 packed;
        packed.x = *reinterpret_cast<uint32_t*>(&lo);
        packed.y = *reinterpret_cast<uint32_t*>(&hi);
        if (peer.world == 0) {
          *reinterpret_cast<uint2*>(y + static_cast<size_t>(m) * N + n) = packed;
        } else if (peer.mode == 1) {
          *reinterpret_cast<uint2*>(scatter_dst(peer, rs_par, m, n, N)) = packed;
        } else {
          for (int p = 0; p < peer.world; ++p)
            *reinterpret_cast<uint2*>(peer_slot(peer, p) + static_cast<size_t>(m) * N + n) = packed;
        }
      }
    }
    cluster_sync();  // no CTA leaves while another still reads its shared memory
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
  if (peer.world > 0 && ok) push_signal(peer, true, gridDim.x * gridDim.y * gridDim.z, rs_par);
  if (ag.ctrl != nullptr && threadIdx.x == 0) {
    // every CTA's producer has waited (it is this thread): the last one closes the round. ag_par was set by this
    // thread's wait; CTAs without K work read the round's parity themselves.
    const int par = nkb > 0 ? ag_par : static_cast<int>(ag.ctrl[kSpAgRound] & 1u);
    ag_release(ag, par, gridDim.x * gridDim.y * gridDim.z);
  }
}

template <int BN>
int run_gemm_cluster(const CUtensorMap& tm_w, const CUtensorMap& tm_x, void* y, int M, int N, int K, int splits,
                     unsigned* status, cudaStream_t stream, const PeerOut& peer, const AgWait& ag,
                     const CUtensorMap& tm_x1) {
  using Cfg = GemmCfg<BN, split_occupancy<BN>()>;
  set_max_smem(gemm_cluster_kernel<BN>, Cfg::kSmem);
  const int total_kb = (K + kBK - 1) / kBK;
  const int kbps = (total_kb + splits - 1) / splits;
  splits = (total_kb + kbps - 1) / kbps;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + kBM - 1) / kBM, (M + BN - 1) / BN, splits);
  cfg.blockDim = dim3(128);
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
  const cudaError_t err = cudaLaunchKernelEx(&cfg, gemm_cluster_kernel<BN>, tm_w, tm_x, static_cast<bf16*>(y), M, N,
                                             K, kbps, status, peer, ag, tm_x1);
  return err == cudaSuccess ? 0 : -2;
}

// ---------------------------------------------------------------------------------------------------------------
// Persistent stream-K GEMM (the main path)
// ---------------------------------------------------------------------------------------------------------------
// Work = tiles x K-blocks "units" (tile-major). CTA c of C owns units [c*U/C, (c+1)*U/C); each maximal run of its
// units inside one tile is a segment. Warp 0 streams (W, X) stages, warp 1 issues UMMAs into one of two TMEM
// accumulators, warps 2-5 drain the other. A segment that covers its whole tile is written as bf16 directly;
// otherwise its fp32 partial goes to slot 2c (first tile of the CTA) or 2c+1 (last tile), and the tile's last
// contributor (counted on counters[c_lo]) sums the contributors' partials in CTA order.
struct StreamK {
  int units, ctas, kb, n_tiles;
  __device__ __forceinline__ int start(int c) const { return static_cast<int>((static_cast<long long>(c) * units) / ctas); }
  __device__ __forceinline__ int cta_of(int u) const {
    return static_cast<int>(((static_cast<long long>(u) + 1) * ctas + units - 1) / units) - 1;
  }
};

template <int BN>
__global__ void __launch_bounds__(192, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                           bf16* __restrict__ y, float* __restrict__ ws, int* __restrict__ counters, int M, int N,
                           int K, unsigned* status) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  constexpr int kAccCols = BN;
  constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = smem + S * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;   // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = const_cast<int*>(reinterpret_cast<volatile int*>(tmem_slot + 2));

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (N + kBM - 1) / kBM;
  const int m_tiles = (M + BN - 1) / BN;
  StreamK sk;
  sk.kb = (K + kBK - 1) / kBK;
  sk.units = n_tiles * m_tiles * sk.kb;
  sk.ctas = gridDim.x;
  sk.n_tiles = n_tiles;
  const int c = blockIdx.x;
  const int u_begin = sk.start(c), u_end = sk.start(c + 1);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer: walks every unit of this CTA in order ----
    const int n_units = u_end - u_begin;
    const int pre = n_units < S ? n_units : S;
    for (int g = 0; g < pre; ++g) {  // weight tiles of the first ring before waiting on the predecessor
      const int u = u_begin + g, t = u / sk.kb, kb = u % sk.kb;
      mbar_arrive_expect_tx(&full[g], Cfg::kStageBytes);
      tma_load_2d(a_tiles + g * kABytes, &tm_w, &full[g], kb * kBK, (t % n_tiles) * kBM);
    }
    pdl_wait();
    for (int g = 0; g < pre; ++g) {
      const int u = u_begin + g, t = u / sk.kb, kb = u % sk.kb;
      tma_load_2d(b_tiles + g * Cfg::kBBytes, &tm_x, &full[g], kb * kBK, (t / n_tiles) * BN);
    }
    for (int g = pre; g < n_units; ++g) {
      const int st = g % S;
      const uint32_t use = g / S;
      if (!mbar_wait(&empty[st], (use & 1u) ^ 1u, status, kStatusWaitEmpty, abort_flag)) break;
      const int u = u_begin + g, t = u / sk.kb, kb = u % sk.kb;
      mbar_arrive_expect_tx(&full[st], Cfg::kStageBytes);
      tma_load_2d(a_tiles + st * kABytes, &tm_w, &full[st], kb * kBK, (t % n_tiles) * kBM);
      tma_load_2d(b_tiles + st * Cfg::kBBytes, &tm_x, &full[st], kb * kBK, (t / n_tiles) * BN);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN);
    int g = 0, seg = 0;
    bool good = true;
    for (int u = u_begin; u < u_end && good; ++seg) {
      const int t = u / sk.kb;
      const int seg_end = min(u_end, (t + 1) * sk.kb);
      const int buf = seg & 1;
      if (!mbar_wait(&acc_empty[buf], ((seg >> 1) & 1) ^ 1, status, kStatusWaitAccum, abort_flag)) break;
      tc_fence_after();
      const uint32_t acc = tmem + buf * kAccCols;
      const int seg_start = u;
      for (; u < seg_end; ++u, ++g) {
        const int st = g % S;
        if (!mbar_wait(&full[st], (g / S) & 1u, status, kStatusWaitFull, abort_flag)) { good = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(a_tiles + st * kABytes);
        const uint32_t b_addr = smem_u32(b_tiles + st * Cfg::kBBytes);
        const bool first = u == seg_start;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          umma_bf16(acc, desc_kmajor_sw128(a_addr + kk * 32), desc_kmajor_sw128(b_addr + kk * 32), idesc,
                    (first && kk == 0) ? 0u : 1u);
        }
        umma_commit(&empty[st]);
      }
      umma_commit(&acc_full[buf]);  // also after a failure, so the epilogue's wait ends
    }
  } else if (warp >= 2) {
    // ---- epilogue: warp w drains TMEM lanes 32 * (w % 4) .. (output features) ----
    const int quad = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const int et = threadIdx.x - 64;  // 0..127
    pdl_wait();  // no global write before the predecessor grid completed
    int seg = 0;
    for (int u = u_begin; u < u_end; ++seg) {
      const int t = u / sk.kb;
      const int seg_begin = u;
      const int seg_end = min(u_end, (t + 1) * sk.kb);
      u = seg_end;
      const int buf = seg & 1;
      mbar_wait(&acc_full[buf], (seg >> 1) & 1, status, kStatusWaitAccum, abort_flag);  // sets abort_flag on failure
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the decision below is uniform over the epilogue warps
      tc_fence_after();
      const int n0 = (t % n_tiles) * kBM, m0 = (t / n_tiles) * BN;
      const int n = n0 + quad * 32 + lane;
      const bool whole = seg_begin == t * sk.kb && seg_end == (t + 1) * sk.kb;
      const bool live = !*abort_flag;
      float* part = nullptr;
      if (!whole) part = ws + (static_cast<size_t>(2 * c + (t == u_begin / sk.kb ? 0 : 1)) * BN) * kBM;
      const uint32_t acc = tmem + buf * kAccCols;
#pragma unroll 1
      for (int cc = 0; cc < BN; cc += 16) {
        float v[16];
        tmem_ld16(acc + lane_base + cc, v);
        if (!live) continue;
        if (whole) {
          if (n < N) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = m0 + cc + j;
              if (m < M) y[static_cast<size_t>(m) * N + n] = __float2bfloat16(v[j]);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) part[(cc + j) * kBM + quad * 32 + lane] = v[j];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);  // this warp's reads of the accumulator are done
      if (whole || !live) continue;
      // ---- stream-K fixup: the tile's last contributor sums all partials in CTA order ----
      const int c_lo = sk.cta_of(t * sk.kb), c_hi = sk.cta_of((t + 1) * sk.kb - 1);
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps
      if (et == 0) *last_flag = atomicAdd(&counters[c_lo], 1) == c_hi - c_lo;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*last_flag) {
        __threadfence();
        const int cg = et & 31, rp = et >> 5;  // 4 features (cg) x rows rp, rp + 4, ...
        const int col = n0 + cg * 4;
        const int m_end = min(M, m0 + BN);
        if (col < N) {
          for (int mb = m0 + rp; mb < m_end; mb += 16) {
            float4 accv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) accv[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int cc2 = c_lo; cc2 <= c_hi; ++cc2) {
              const int first_tile = sk.start(cc2) / sk.kb;
              const float* src = ws + (static_cast<size_t>(2 * cc2 + (t == first_tile ? 0 : 1)) * BN) * kBM;
              float4 vv[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int m = mb + 4 * q;
                vv[q] = m < m_end ? __ldcg(reinterpret_cast<const float4*>(src + (m - m0) * kBM + cg * 4))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                accv[q].x += vv[q].x; accv[q].y += vv[q].y; accv[q].z += vv[q].z; accv[q].w += vv[q].w;
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int m = mb + 4 * q;
              if (m < m_end) {
                __nv_bfloat162 lo = __floats2bfloat162_rn(accv[q].x, accv[q].y);
                __nv_bfloat162 hi = __floats2bfloat162_rn(accv[q].z, accv[q].w);
                uint2 packed;
                packed.x = *reinterpret_cast<uint32_t*>(&lo);
                packed.y = *reinterpret_cast<uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(y + static_cast<size_t>(m) * N + col) = packed;
              }
            }
          }
        }
        if (et == 0) counters[c_lo] = 0;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // last_flag is reused by the next segment
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

template <int BN>
int run_gemm_persistent(const CUtensorMap& tm_w, const CUtensorMap& tm_x, void* y, float* ws, int* counters, int M,
                        int N, int K, int ctas, unsigned* status, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  set_max_smem(gemm_persistent_kernel<BN>, Cfg::kSmem);
  launch_pdl(gemm_persistent_kernel<BN>, dim3(ctas), dim3(192), Cfg::kSmem, stream, tm_w, tm_x,
             static_cast<bf16*>(y), ws, counters, M, N, K, status);
  return 0;
}

}  // namespace

int gemm_block_n(int M) {
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

// Split count from the weight shape (and, for large M, the token tiles): enough CTAs to cover the SMs, at least
// 4 K-slices per split. Depends on M only through the number of token tiles, so every decode pass of up to
// 256 rows reduces each output in the same order.
int gemm_splits(int M, int N, int K, int num_sms) {
  const int bn = gemm_block_n(M);
  const int m_tiles = (M + bn - 1) / bn;
  const int tiles = ((N + kBM - 1) / kBM) * m_tiles;
  const int total_kb = (K + kBK - 1) / kBK;
  if (tiles >= num_sms) return 1;
  int splits = num_sms / tiles;
  splits = std::min(splits, total_kb / 4);
  return std::max(1, std::min(splits, 16));
}

template <int BN>
int cluster_capacity_bn(int splits);

// Split count of the cluster split-K kernel: the gemm_splits rule over the CTA slots (two per SM for skinny
// tiles), capped at 8 CTAs per (portable) cluster, then lowered until every tile's cluster is resident at once
// (the hardware places clusters inside GPCs, so a tile grid larger than the resident clusters runs in waves).
// Identical for every M up to 64 rows (the 64-row configuration's capacity stands for both skinny tile widths), so
// one-token and verification passes reduce K the same way.
int gemm_cluster_splits(int M, int N, int K, int num_sms) {
  const int bn = gemm_block_n(M);
  const int slots = bn <= 64 ? 2 * num_sms : num_sms;
  int splits = std::min(8, gemm_splits(M, N, K, slots));
  const int tiles = ((N + kBM - 1) / kBM) * ((M + bn - 1) / bn);
  while (splits > 1) {
    const int cap = bn <= 64 ? cluster_capacity_bn<64>(splits)
                  : bn == 128 ? cluster_capacity_bn<128>(splits) : cluster_capacity_bn<256>(splits);
    if (tiles <= cap) break;
    --splits;
  }
  return splits;
}

// How many clusters of `splits` CTAs of the BN-wide cluster kernel can be resident at once (the hardware packs
// clusters inside GPCs, so this is far below SMs * CTAs-per-SM / splits for large clusters).
template <int BN>
int cluster_capacity_bn(int splits) {
  using Cfg = GemmCfg<BN, split_occupancy<BN>()>;
  static std::mutex mu;
  static int cache[64][9] = {};  // per device (the occupancy query reads the device's own attributes)
  if (splits < 1 || splits > 8) return 0;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 1;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device][splits] == 0) {
    set_max_smem(gemm_cluster_kernel<BN>, Cfg::kSmem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, 1, splits);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = splits;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_cluster_kernel<BN>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 1;
    }
    cache[device][splits] = std::max(1, n);
  }
  return cache[device][splits];
}

int gemm_cluster_capacity(int M, int splits) {
  switch (gemm_block_n(M)) {
    case 32: return cluster_capacity_bn<32>(splits);
    case 64: return cluster_capacity_bn<64>(splits);
    case 128: return cluster_capacity_bn<128>(splits);
    default: return cluster_capacity_bn<256>(splits);
  }
}

int launch_gemm_cluster(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, int M, int N, int K, int splits,
                        unsigned* status, cudaStream_t stream, const PeerOut* peer, const AgWait* ag,
                        const CUtensorMap* tm_x1) {
  if (K % 8 != 0 || N % 4 != 0 || splits < 1 || splits > 8) return -1;
  const PeerOut none{};
  const PeerOut& pe = peer != nullptr ? *peer : none;
  if (pe.mode == 1 && (pe.shard_rows < 1 || pe.shard_max < pe.shard_rows || pe.world < 1 ||
                       (M + pe.shard_rows - 1) / pe.shard_rows > pe.world)) return -1;
  const AgWait no_wait{};
  const AgWait& aw = ag != nullptr ? *ag : no_wait;
  const CUtensorMap& x1 = tm_x1 != nullptr ? *tm_x1 : *tm_x;
  switch (gemm_block_n(M)) {
    case 32: return run_gemm_cluster<32>(*tm_w, *tm_x, y, M, N, K, splits, status, stream, pe, aw, x1);
    case 64: return run_gemm_cluster<64>(*tm_w, *tm_x, y, M, N, K, splits, status, stream, pe, aw, x1);
    case 128: return run_gemm_cluster<128>(*tm_w, *tm_x, y, M, N, K, splits, status, stream, pe, aw, x1);
    default: return run_gemm_cluster<256>(*tm_w, *tm_x, y, M, N, K, splits, status, stream, pe, aw, x1);
  }
}

int gemm_persistent_ctas(int M, int N, int K, int num_sms) {
  const int bn = gemm_block_n(M);
  const long units = static_cast<long>((N + kBM - 1) / kBM) * ((M + bn - 1) / bn) * ((K + kBK - 1) / kBK);
  return static_cast<int>(std::min<long>(num_sms, units));
}

long gemm_persistent_ws_floats(int M, int N, int K, int num_sms) {
  return 2L * gemm_persistent_ctas(M, N, K, num_sms) * gemm_block_n(M) * kBM;
}

int launch_gemm_persistent(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, float* ws, int* counters, int M,
                           int N, int K, int num_sms, unsigned* status, cudaStream_t stream) {
  if (K % 8 != 0 || N % 4 != 0 || counters == nullptr || ws == nullptr) return -1;
  const int ctas = gemm_persistent_ctas(M, N, K, num_sms);
  switch (gemm_block_n(M)) {
    case 32: return run_gemm_persistent<32>(*tm_w, *tm_x, y, ws, counters, M, N, K, ctas, status, stream);
    case 64: return run_gemm_persistent<64>(*tm_w, *tm_x, y, ws, counters, M, N, K, ctas, status, stream);
    case 128: return run_gemm_persistent<128>(*tm_w, *tm_x, y, ws, counters, M, N, K, ctas, status, stream);
    default: return run_gemm_persistent<256>(*tm_w, *tm_x, y, ws, counters, M, N, K, ctas, status, stream);
  }
}

int launch_gemm_bf16(const CUtensorMap* tm_w, const CUtensorMap* tm_x, void* y, float* ws, int M, int N, int K,
                     int splits, unsigned* status, cudaStream_t stream, int* counters, const PeerOut* peer,
                     int flags, const AgWait* ag, const CUtensorMap* tm_x1) {
  if (K % 8 != 0 || N % 4 != 0) return -1;
  if (splits > 1 && counters == nullptr && peer != nullptr && peer->world > 0) return -1;  // push needs the fused reduce
  const PeerOut none{};
  const PeerOut& pe = peer != nullptr ? *peer : none;
  const AgWait none_ag{};
  const AgWait& aw = ag != nullptr ? *ag : none_ag;
  switch (gemm_block_n(M)) {
    case 32: return run_gemm<32>(*tm_w, *tm_x, y, ws, counters, M, N, K, splits, status, stream, pe, flags, aw, tm_x1);
    case 64: return run_gemm<64>(*tm_w, *tm_x, y, ws, counters, M, N, K, splits, status, stream, pe, flags, aw, tm_x1);
    case 128:
      return run_gemm<128>(*tm_w, *tm_x, y, ws, counters, M, N, K, splits, status, stream, pe, flags, aw, tm_x1);
    default:
      return run_gemm<256>(*tm_w, *tm_x, y, ws, counters, M, N, K, splits, status, stream, pe, flags, aw, tm_x1);
  }
}

}  // namespace ecz

// ---------------------------------------------------------------------------------------------------------------
// Allocation-free entry point (see noalloc.h): the split-K partials live in a file-scope device array.
// ---------------------------------------------------------------------------------------------------------------
#include <cstdio>
#include <mutex>

#include "noalloc.h"

namespace {

// fp32 split-K partials, then one status word for the bounded waits.
static __device__ __align__(256) float g_noalloc_scratch[ECZ_NOALLOC_SCRATCH_FLOATS + 64];

float* noalloc_scratch_for_current_device(int device) {
  static std::mutex mu;
  static float* addr[64] = {};
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess) {
      std::fprintf(stderr, "ecz_linear_bf16_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", device,
                   cudaGetErrorString(err));
      return nullptr;
    }
    addr[device] = static_cast<float*>(p);
  }
  return addr[device];
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int ecz_linear_bf16_noalloc(const void* x, const void* w, void* y,
                                                                               int M, int N, int K, void* stream) {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) {
    std::fprintf(stderr, "ecz_linear_bf16_noalloc: no current CUDA device\n");
    return -5;
  }
  if (M <= 0 || N <= 0 || K <= 0 || K % 8 != 0 || N % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(w) & 15u) ||
      (reinterpret_cast<uintptr_t>(y) & 15u)) {
    std::fprintf(stderr, "ecz_linear_bf16_noalloc: bad shape or alignment (M=%d N=%d K=%d; K %% 8 and N %% 4 must "
                 "be 0, pointers 16-byte aligned)\n", M, N, K);
    return -1;
  }
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int splits = ecz::gemm_splits(M, N, K, sms > 0 ? sms : 148);
  if (splits > 1 && static_cast<size_t>(splits) * M * N > ECZ_NOALLOC_SCRATCH_FLOATS) {
    std::fprintf(stderr, "ecz_linear_bf16_noalloc: %d x %d x %d split-K partials need %zu floats, more than the "
                 "%u-float scratch array\n", splits, M, N, static_cast<size_t>(splits) * M * N,
                 ECZ_NOALLOC_SCRATCH_FLOATS);
    return -2;
  }
  float* scratch = noalloc_scratch_for_current_device(device);
  if (scratch == nullptr) return -4;
  unsigned* status = reinterpret_cast<unsigned*>(scratch + ECZ_NOALLOC_SCRATCH_FLOATS);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t clear = cudaMemsetAsync(status, 0, sizeof(unsigned), s);  // every call starts with a clear word
  if (clear != cudaSuccess) {
    std::fprintf(stderr, "ecz_linear_bf16_noalloc: clearing the status word failed: %s\n", cudaGetErrorString(clear));
    return -6;
  }
  CUtensorMap tm_w, tm_x;
  if (ecz::make_tmap_2d_bf16(&tm_w, w, N, K, K, 128) != 0 ||
      ecz::make_tmap_2d_bf16(&tm_x, x, M, K, K, ecz::gemm_block_n(M)) != 0) {
    std::fprintf(stderr, "ecz_linear_bf16_noalloc: cuTensorMapEncodeTiled failed\n");
    return -3;
  }
  if (ecz::launch_gemm_bf16(&tm_w, &tm_x, y, splits > 1 ? scratch : nullptr, M, N, K, splits, status, s) != 0) {
    return -1;
  }
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    std::fprintf(stderr, "ecz_linear_bf16_noalloc: launch failed: %s\n", cudaGetErrorString(err));
    return -6;
  }
  return 0;
}

extern "C" __attribute__((visibility("default"))) int ecz_linear_bf16_noalloc_status(unsigned* status_out) {
  int device = -1;
  if (status_out == nullptr) return -1;
  if (cudaGetDevice(&device) != cudaSuccess) return -5;
  float* scratch = noalloc_scratch_for_current_device(device);
  if (scratch == nullptr) return -4;
  // a synchronous 4-byte copy into the caller's host memory (pageable: no allocation on either side)
  const cudaError_t err = cudaMemcpy(status_out, scratch + ECZ_NOALLOC_SCRATCH_FLOATS, sizeof(unsigned),
                                     cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) {
    std::fprintf(stderr, "ecz_linear_bf16_noalloc_status: reading the status word failed: %s\n",
                 cudaGetErrorString(err));
    return -6;
  }
  return 0;
}

namespace {

// One thread waits on an mbarrier that nothing completes, bounded by `limit_ns`: the wait runs out, records
// kStatusWaitFull in the status word and the kernel returns. No copy or MMA is in flight when it gives up.
__global__ void noalloc_wait_selftest_kernel(unsigned* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    ecz::mbar_init(&bar, 1);
    ecz::fence_mbar_init();
    ecz::mbar_wait(&bar, 0, status, ecz::kStatusWaitFull, nullptr, limit_ns);
  }
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int ecz_noalloc_wait_selftest(unsigned long long limit_ns,
                                                                                 void* stream) {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return -5;
  if (limit_ns == 0 || limit_ns > 1000000000ull) return -1;
  float* scratch = noalloc_scratch_for_current_device(device);
  if (scratch == nullptr) return -4;
  unsigned* status = reinterpret_cast<unsigned*>(scratch + ECZ_NOALLOC_SCRATCH_FLOATS);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(status, 0, sizeof(unsigned), s) != cudaSuccess) return -6;
  noalloc_wait_selftest_kernel<<<1, 32, 0, s>>>(status, limit_ns);
  return cudaGetLastError() == cudaSuccess ? 0 : -6;
}
