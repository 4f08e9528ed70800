// Sequence-parallel tensor parallelism over NVLink peer memory: the collective halves of the fused
// GEMM -> reduce-scatter and all-gather -> GEMM pair of every transformer sublayer.
//
// Between sublayers the residual stream is split by token: rank r owns rows [r * s, (r + 1) * s) of the pass's M
// rows (s = ceil(M / P); the last ranks may own fewer or none). A sublayer runs as
//
//   AG -> GEMM   the column-parallel projection (QKV, gate/up) waits until every rank's normed rows of the round
//                arrived in this rank's all-gather buffer, then streams X from local memory (gemm_tc.cu, AgWait)
//   ...          attention / SwiGLU on this rank's heads / features, all M rows
//   GEMM -> RS   the row-parallel projection (O, down) stores each output row straight into the partial slot of
//                the row's owner (gemm_tc.cu, PeerOut mode 1) and signals every rank once
//   reduce       here: the owner sums the P partials of its rows in rank order, adds its residual rows, applies
//                the next RMSNorm and pushes the normed rows into every rank's all-gather buffer (the all-gather),
//                optionally the residual rows too (block outputs a drafter reads), and signals every rank once
//
// so each row crosses NVLink twice per sublayer (to its owner as a partial, from its owner as a normed row) instead
// of P - 1 times as a full all-reduce would move it. One IPC buffer per rank:
//
//   [control words][reduce-scatter partials [2][P][s_max][H]][all-gather rows [2][M_max][H]][captures [C][M_max][H]]
//
// Rounds alternate between two parities per kind; the round counters are device words that the consumers advance,
// so every launch derives its parity on the device and a captured CUDA graph replays correctly. A rank writes round
// k + 2 of a kind into a peer only after a chain of data dependencies through that peer's later kernels, so a slot is
// never overwritten while it is read. Every wait is bounded by the global timer and records kStatusWaitPeer.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

constexpr int kRowsPerCta = 1;  // one row per CTA: a boundary of M rows runs M / P CTAs in parallel

__device__ __forceinline__ unsigned ld_acquire_sys32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait (one thread) until *flag >= target.
__device__ __forceinline__ bool wait_count(const unsigned* flag, unsigned target, unsigned* status) {
  if (ld_acquire_sys32(flag) >= target) return true;
  const unsigned long long start = global_timer_ns();
  while (ld_acquire_sys32(flag) < target) {
    if (global_timer_ns() - start > kWaitLimitNs) {
      atomicOr(status, kStatusWaitPeer);
      return false;
    }
  }
  return true;
}

struct SpArgs {
  PeerPtrs peers;
  int world, rank, hidden, max_rows, shard_max;
  long rs_off, ag_off, cap_off;
};

__device__ __forceinline__ unsigned* ctrl_of(const SpArgs& a, int p) { return static_cast<unsigned*>(a.peers.ptr[p]); }

__device__ __forceinline__ bf16* region(const SpArgs& a, int p, long off) {
  return reinterpret_cast<bf16*>(static_cast<uint8_t*>(a.peers.ptr[p]) + off);
}

__global__ void __launch_bounds__(256) sp_reduce_norm_kernel(SpArgs a, int partials, const bf16* __restrict__ resid,
                                                             bf16* __restrict__ resid_out, const bf16* __restrict__ w,
                                                             int rows, int row0, float eps, int cap_slot,
                                                             unsigned* status) {
  pdl_trigger();
  pdl_wait();
  unsigned* own = ctrl_of(a, a.rank);
  const int rs_par = static_cast<int>(own[kSpRsRound] & 1u);
  const int ag_par = static_cast<int>(own[kSpAgRound] & 1u);
  __shared__ float red_s[32];
  if (partials && threadIdx.x == 0) wait_count(own + kSpRsArrive + rs_par, static_cast<unsigned>(a.world), status);
  __syncthreads();
  __threadfence();
  const int H = a.hidden, nvec = H / 8;
  const bf16* slots = region(a, a.rank, a.rs_off) + static_cast<size_t>(rs_par) * a.world * a.shard_max * H;
  for (int r = blockIdx.x * kRowsPerCta; r < min(rows, (blockIdx.x + 1) * kRowsPerCta); ++r) {
    float ss = 0.f;
    // pass 1: the partials summed in rank order and rounded to bf16 (an all-reduce of bf16 tensors), plus the
    // residual; the new residual row is written and its square sum accumulated
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      if (partials) {
        for (int p = 0; p < a.world; ++p) {
          const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(slots + (static_cast<size_t>(p) * a.shard_max + r) * H) + v);
          const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(e[j]);
        }
      }
      const uint4 rr = reinterpret_cast<const uint4*>(resid + static_cast<size_t>(r) * H)[v];
      const bf16* re = reinterpret_cast<const bf16*>(&rr);
      uint4 so;
      bf16* se = reinterpret_cast<bf16*>(&so);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float s = partials ? bf16r(bf16r(acc[j]) + __bfloat162float(re[j])) : __bfloat162float(re[j]);
        se[j] = __float2bfloat16(s);
        ss += s * s;
      }
      reinterpret_cast<uint4*>(resid_out + static_cast<size_t>(r) * H)[v] = so;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < (blockDim.x >> 5) ? red_s[threadIdx.x] : 0.f;
      t = warp_sum(t);
      if (threadIdx.x == 0) red_s[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red_s[0] / static_cast<float>(H) + eps);
    __syncthreads();
    // pass 2: normalise and push the row (and the residual row of a captured block) to every rank
    const size_t grow = static_cast<size_t>(row0 + r);
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      const uint4 so = reinterpret_cast<const uint4*>(resid_out + static_cast<size_t>(r) * H)[v];
      const uint4 ww = reinterpret_cast<const uint4*>(w)[v];
      const bf16* se = reinterpret_cast<const bf16*>(&so);
      const bf16* we = reinterpret_cast<const bf16*>(&ww);
      uint4 o;
      bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        oe[j] = __float2bfloat16(__bfloat162float(we[j]) * bf16r(__bfloat162float(se[j]) * inv));
      for (int p = 0; p < a.world; ++p) {
        bf16* ag = region(a, p, a.ag_off) + (static_cast<size_t>(ag_par) * a.max_rows + grow) * H;
        reinterpret_cast<uint4*>(ag)[v] = o;
        if (cap_slot >= 0) {
          bf16* cap = region(a, p, a.cap_off) + (static_cast<size_t>(cap_slot) * a.max_rows + grow) * H;
          reinterpret_cast<uint4*>(cap)[v] = so;
        }
      }
    }
  }
  __syncthreads();  // every thread's stores precede thread 0's system-scope fence
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(own + kSpReduceDone, 1u) == gridDim.x - 1) {  // the last CTA closes both rounds
      own[kSpReduceDone] = 0;
      if (partials) {
        own[kSpRsArrive + rs_par] = 0;
        own[kSpRsRound] += 1u;
      }
      __threadfence_system();
      for (int p = 0; p < a.world; ++p) atomicAdd_system(ctrl_of(a, p) + kSpAgArrive + ag_par, 1u);
    }
  }
}

// An all-gather consumer that copies the round's rows [0, rows) into `out` (the final hidden states of a pass).
__global__ void __launch_bounds__(256) sp_fetch_kernel(SpArgs a, bf16* __restrict__ out, int rows, unsigned* status) {
  pdl_trigger();
  pdl_wait();
  unsigned* own = ctrl_of(a, a.rank);
  const int par = static_cast<int>(own[kSpAgRound] & 1u);
  if (threadIdx.x == 0) wait_count(own + kSpAgArrive + par, static_cast<unsigned>(a.world), status);
  __syncthreads();
  __threadfence();
  const bf16* src = region(a, a.rank, a.ag_off) + static_cast<size_t>(par) * a.max_rows * a.hidden;
  const long vecs = static_cast<long>(rows) * a.hidden / 8;
  for (long v = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; v < vecs;
       v += static_cast<long>(gridDim.x) * blockDim.x)
    reinterpret_cast<uint4*>(out)[v] = __ldcg(reinterpret_cast<const uint4*>(src) + v);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(own + kSpAgDone, 1u) == gridDim.x - 1) {
      own[kSpAgDone] = 0;
      own[kSpAgArrive + par] = 0;
      own[kSpAgRound] += 1u;
      __threadfence();
    }
  }
}

SpArgs args_of(const PeerPtrs& peers, const SpLayout& L) {
  SpArgs a;
  a.peers = peers;
  a.world = L.world;
  a.rank = L.rank;
  a.hidden = L.hidden;
  a.max_rows = L.max_rows;
  a.shard_max = L.shard_max;
  a.rs_off = L.rs_off;
  a.ag_off = L.ag_off;
  a.cap_off = L.cap_off;
  return a;
}

long align256(long x) { return (x + 255) / 256 * 256; }

}  // namespace

SpLayout sp_layout(int world, int rank, int hidden, int max_rows, int n_cap) {
  SpLayout L;
  L.world = world;
  L.rank = rank;
  L.hidden = hidden;
  L.max_rows = max_rows;
  L.shard_max = world > 0 ? (max_rows + world - 1) / world : 0;
  L.n_cap = n_cap;
  L.rs_off = kSpControlBytes;
  L.ag_off = align256(L.rs_off + 2L * world * L.shard_max * hidden * 2);
  L.cap_off = align256(L.ag_off + 2L * max_rows * hidden * 2);
  L.bytes = align256(L.cap_off + static_cast<long>(n_cap) * max_rows * hidden * 2);
  return L;
}

int launch_sp_reduce_norm(const PeerPtrs& peers, const SpLayout& L, bool partials, const void* resid_in,
                          void* resid_out, const void* w, int rows, int row0, float eps, int cap_slot,
                          unsigned* status, cudaStream_t stream) {
  if (L.world < 1 || L.world > kMaxPeers || L.hidden % 8 != 0 || rows < 0 || rows > L.shard_max ||
      row0 < 0 || row0 + rows > L.max_rows || cap_slot >= L.n_cap || (rows > 0 && (resid_in == nullptr || w == nullptr)))
    return -1;
  const int ctas = std::max(1, (rows + kRowsPerCta - 1) / kRowsPerCta);
  launch_pdl(sp_reduce_norm_kernel, dim3(ctas), dim3(256), 0, stream, args_of(peers, L), partials ? 1 : 0,
             static_cast<const bf16*>(resid_in), static_cast<bf16*>(resid_out), static_cast<const bf16*>(w), rows,
             row0, eps, cap_slot, status);
  return 0;
}

int launch_sp_fetch(const PeerPtrs& peers, const SpLayout& L, void* out, int rows, unsigned* status,
                    cudaStream_t stream) {
  if (L.world < 1 || rows < 0 || rows > L.max_rows || L.hidden % 8 != 0) return -1;
  const long vecs = static_cast<long>(rows) * L.hidden / 8;
  const int ctas = static_cast<int>(std::max<long>(1, std::min<long>((vecs + 255) / 256, 64)));
  launch_pdl(sp_fetch_kernel, dim3(ctas), dim3(256), 0, stream, args_of(peers, L), static_cast<bf16*>(out), rows,
             status);
  return 0;
}

}  // namespace ecz
