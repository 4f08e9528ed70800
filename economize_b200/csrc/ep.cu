// Expert-parallel MoE over NVLink peer memory: the all-to-all dispatch and combine are done by kernels that store
// the routed rows straight into the peers' IPC-mapped symmetric buffers (no NCCL call, no host synchronisation).
//
// Rank r owns experts [r E_l, (r + 1) E_l). Per MoE call:
//   ep_dispatch_kernel   the rows of the local expert-ordered activations xs whose expert lives on rank d are
//                        stored into d's recv[r] (with their source row in d's meta[r]) and the per-expert counts
//                        into d's counts[r]; the launch's last CTA fences at system scope and bumps every rank's
//                        dispatch counter
//   ep_segments_kernel   waits (bounded) until every rank dispatched this call, turns the counts into grouped-GEMM
//                        segments (source-major: segment (s, e) = the rows of local expert e sent by rank s)
//   grouped GEMMs        gate/up and down over the segments (moe.cu, on local memory only)
//   ep_combine_kernel    every output row goes back into its source rank's ret buffer at the row's source
//                        position; then the combine counters of all ranks are bumped the same way
//   ep_finish_kernel     waits until every rank returned its rows and sums each token's weighted expert outputs
//
// One buffer set suffices. Rank r dispatches call k + 1 only after its finish of call k, which needed every rank's
// combine of call k, which each rank issues after its segments and GEMMs of call k have read counts, meta and recv.
// A peer writes r's ret for call k + 1 only after its segments of k + 1 saw r's dispatch of k + 1, i.e. after r's
// finish of k read ret. By induction over calls no counter can reach call k's target with arrivals of call k + 1.
// Every wait is bounded by the global timer (status kStatusWaitPeer); after a timeout the kernels move no rows.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

struct EpControl {
  unsigned dispatched;  // dispatch arrivals (bumped by every rank once per call)
  unsigned combined;    // combine arrivals
  unsigned d_epoch;     // calls whose dispatch this rank consumed
  unsigned c_epoch;     // calls whose combine this rank consumed
  unsigned done[4];     // CTA counters of the current dispatch / combine / finish launch
  unsigned pad[56];
};
static_assert(sizeof(EpControl) == 256, "control block is 256 bytes");

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint8_t* ep_base(const PeerPtrs& peers, int p) { return static_cast<uint8_t*>(peers.ptr[p]); }
__device__ __forceinline__ EpControl* ctl(const PeerPtrs& peers, int p) {
  return reinterpret_cast<EpControl*>(ep_base(peers, p));
}
__device__ __forceinline__ int* counts_of(uint8_t* base, const EpLayout& L, int src) {
  return reinterpret_cast<int*>(base + L.counts_off) + src * L.experts_local;
}
__device__ __forceinline__ int* meta_of(uint8_t* base, const EpLayout& L, int src) {
  return reinterpret_cast<int*>(base + L.meta_off) + static_cast<long>(src) * L.cap;
}
__device__ __forceinline__ bf16* recv_of(uint8_t* base, const EpLayout& L, int src) {
  return reinterpret_cast<bf16*>(base + L.recv_off) + static_cast<long>(src) * L.cap * L.hidden;
}
__device__ __forceinline__ bf16* ret_of(uint8_t* base, const EpLayout& L) {
  return reinterpret_cast<bf16*>(base + L.ret_off);
}

// Every thread fences its peer stores at system scope; the launch's last CTA then bumps counter `which`
// (0 dispatched, 1 combined) of every rank.
__device__ __forceinline__ void signal_all(const PeerPtrs& peers, const EpLayout& L, int rank, int which) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    EpControl* own = ctl(peers, rank);
    const unsigned done = atomicAdd(&own->done[which], 1u);
    if (done == gridDim.x * gridDim.y - 1) {
      own->done[which] = 0;
      __threadfence_system();
      for (int p = 0; p < L.world; ++p) {
        EpControl* c = ctl(peers, p);
        atomicAdd_system(which == 0 ? &c->dispatched : &c->combined, 1u);
      }
    }
  }
}

__device__ __forceinline__ bool wait_count(const unsigned* counter, unsigned target, unsigned* status) {
  const unsigned long long start = global_timer_ns();
  while (ld_acquire_sys(counter) < target) {
    if (*reinterpret_cast<volatile unsigned*>(status) & kStatusWaitPeer) return false;  // another CTA gave up
    if (global_timer_ns() - start > kWaitLimitNs) {
      atomicOr(status, kStatusWaitPeer);
      return false;
    }
  }
  return true;
}

// grid (row blocks, world): CTA (i, d) copies rows [offsets[d E_l], offsets[(d + 1) E_l]) of xs to rank d, four
// rows per CTA per step (64 threads x 16 B per row)
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const bf16* __restrict__ xs, const int* __restrict__ offsets,
                                                          PeerPtrs peers, EpLayout L, int rank) {
  pdl_trigger();
  pdl_wait();
  const int d = blockIdx.y;
  const int start = offsets[d * L.experts_local], end = offsets[(d + 1) * L.experts_local];
  uint8_t* peer = ep_base(peers, d);
  if (blockIdx.x == 0 && threadIdx.x < L.experts_local) {
    const int e = d * L.experts_local + threadIdx.x;
    counts_of(peer, L, rank)[threadIdx.x] = offsets[e + 1] - offsets[e];
  }
  bf16* dst = recv_of(peer, L, rank);
  int* meta = meta_of(peer, L, rank);
  const int vecs = L.hidden / 8;
  for (int row = start + blockIdx.x * 4 + (threadIdx.x >> 6); row < end; row += gridDim.x * 4) {
    const int i = row - start;
    if (i >= L.cap) break;  // the host sizes cap so that this never drops a row
    const uint4* src = reinterpret_cast<const uint4*>(xs + static_cast<long>(row) * L.hidden);
    uint4* out = reinterpret_cast<uint4*>(dst + static_cast<long>(i) * L.hidden);
    for (int v = threadIdx.x & 63; v < vecs; v += 64) out[v] = src[v];
    if ((threadIdx.x & 63) == 0) meta[i] = row;
  }
  signal_all(peers, L, rank, 0);
}

// one CTA: wait for every rank's dispatch, then the segments (start, end, expert) of the received rows
__global__ void __launch_bounds__(128) ep_segments_kernel(PeerPtrs peers, EpLayout L, int rank,
                                                          int* __restrict__ seg_start, int* __restrict__ seg_end,
                                                          int* __restrict__ seg_expert, unsigned* status) {
  pdl_trigger();
  pdl_wait();
  EpControl* own = ctl(peers, rank);
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const unsigned epoch = own->d_epoch;
    ok = wait_count(&own->dispatched, static_cast<unsigned>(L.world) * (epoch + 1u), status);
    own->d_epoch = epoch + 1u;
  }
  __syncthreads();
  const int g = threadIdx.x;
  if (g < L.world * L.experts_local) {
    const int s = g / L.experts_local, e = g % L.experts_local;
    int lo = 0, n = 0;
    if (ok) {
      const int* cnt = counts_of(ep_base(peers, rank), L, s);
      for (int j = 0; j < e; ++j) lo += cnt[j];
      lo = min(max(lo, 0), L.cap);
      n = min(max(cnt[e], 0), L.cap - lo);
    }
    seg_start[g] = s * L.cap + lo;
    seg_end[g] = s * L.cap + lo + n;
    seg_expert[g] = e;
  }
}

// grid (row blocks, world): the rows received from source s go back to s's ret buffer at their source rows
__global__ void __launch_bounds__(256) ep_combine_kernel(const bf16* __restrict__ y, const int* __restrict__ seg_start,
                                                         const int* __restrict__ seg_end, PeerPtrs peers, EpLayout L,
                                                         int rank) {
  pdl_trigger();
  pdl_wait();
  const int s = blockIdx.y;
  const int n = seg_end[(s + 1) * L.experts_local - 1] - s * L.cap;  // rows received from s (0 after a timeout)
  const int* meta = meta_of(ep_base(peers, rank), L, s);
  bf16* ret = ret_of(ep_base(peers, s), L);
  const int vecs = L.hidden / 8;
  for (int i = blockIdx.x * 4 + (threadIdx.x >> 6); i < n; i += gridDim.x * 4) {
    const int dst_row = meta[i];
    if (dst_row < 0 || dst_row >= L.ret_rows) continue;
    const uint4* src = reinterpret_cast<const uint4*>(y + (static_cast<long>(s) * L.cap + i) * L.hidden);
    uint4* out = reinterpret_cast<uint4*>(ret + static_cast<long>(dst_row) * L.hidden);
    for (int v = threadIdx.x & 63; v < vecs; v += 64) out[v] = src[v];
  }
  signal_all(peers, L, rank, 1);
}

// one CTA per token (at least one): wait until every rank returned its rows, then out[t] = sum_j w[t, j] * ret[pos[t, j]] (fp32)
__global__ void __launch_bounds__(256) ep_finish_kernel(PeerPtrs peers, EpLayout L, int rank,
                                                        const int* __restrict__ pos, const float* __restrict__ w,
                                                        bf16* __restrict__ out, int tokens, int k,
                                                        unsigned* status) {
  pdl_trigger();
  pdl_wait();
  EpControl* own = ctl(peers, rank);
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const unsigned epoch = own->c_epoch;  // advanced only after every CTA of this launch read it (below)
    ok = wait_count(&own->combined, static_cast<unsigned>(L.world) * (epoch + 1u), status);
  }
  __syncthreads();
  const int t = blockIdx.x;
  const bf16* ret = ret_of(ep_base(peers, rank), L);
  for (int c = threadIdx.x; t < tokens && c < L.hidden / 2; c += blockDim.x) {
    float2 acc = make_float2(0.f, 0.f);
    if (ok) {
      for (int j = 0; j < k; ++j) {
        const float wt = w[t * k + j];
        const long row = pos[t * k + j];
        const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(ret + row * L.hidden)[c];
        acc.x += wt * __bfloat162float(v.x);
        acc.y += wt * __bfloat162float(v.y);
      }
    }
    reinterpret_cast<__nv_bfloat162*>(out + static_cast<long>(t) * L.hidden)[c] = __floats2bfloat162_rn(acc.x, acc.y);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned done = atomicAdd(&own->done[2], 1u);
    if (done == gridDim.x - 1) {
      own->done[2] = 0;
      own->c_epoch = own->c_epoch + 1u;
    }
  }
}

}  // namespace

EpLayout ep_layout(int world, int experts_local, int cap, int hidden, int ret_rows) {
  EpLayout L;
  L.world = world;
  L.experts_local = experts_local;
  L.cap = cap;
  L.hidden = hidden;
  L.ret_rows = ret_rows;
  auto up = [](long v) { return (v + 255) / 256 * 256; };
  long off = sizeof(EpControl);
  L.counts_off = off;
  off = up(off + 4L * world * experts_local);
  L.meta_off = off;
  off = up(off + 4L * world * cap);
  L.recv_off = off;
  off = up(off + 2L * world * cap * hidden);
  L.ret_off = off;
  off = up(off + 2L * ret_rows * hidden);
  L.bytes = off;
  return L;
}

int launch_ep_dispatch(const void* xs, const int* offsets, const PeerPtrs& peers, const EpLayout& L, int rank,
                       int rows, cudaStream_t stream) {
  if (L.hidden % 8 != 0 || L.world < 1 || L.world > kMaxPeers || L.experts_local > 256) return -1;
  const int blocks = std::max(1, std::min((rows / L.world + 3) / 4, 64));
  launch_pdl(ep_dispatch_kernel, dim3(blocks, L.world), dim3(256), 0, stream, static_cast<const bf16*>(xs), offsets,
             peers, L, rank);
  return 0;
}

int launch_ep_segments(const PeerPtrs& peers, const EpLayout& L, int rank, int* seg_start, int* seg_end,
                       int* seg_expert, unsigned* status, cudaStream_t stream) {
  if (L.world * L.experts_local > 128) return -1;
  launch_pdl(ep_segments_kernel, dim3(1), dim3(128), 0, stream, peers, L, rank, seg_start, seg_end, seg_expert,
             status);
  return 0;
}

int launch_ep_combine(const void* y, const int* seg_start, const int* seg_end, const PeerPtrs& peers,
                      const EpLayout& L, int rank, cudaStream_t stream) {
  const int blocks = std::max(1, std::min((L.cap + 3) / 4, 64));
  launch_pdl(ep_combine_kernel, dim3(blocks, L.world), dim3(256), 0, stream, static_cast<const bf16*>(y), seg_start,
             seg_end, peers, L, rank);
  return 0;
}

int launch_ep_finish(const PeerPtrs& peers, const EpLayout& L, int rank, const int* pos, const float* w, void* out,
                     int tokens, int k, unsigned* status, cudaStream_t stream) {
  if (tokens < 0 || L.hidden % 2 != 0) return -1;
  // with no tokens one CTA still takes part in the call's epoch (the peers counted this rank's combine)
  launch_pdl(ep_finish_kernel, dim3(std::max(tokens, 1)), dim3(256), 0, stream, peers, L, rank, pos, w,
             static_cast<bf16*>(out), tokens, k, status);
  return 0;
}

}  // namespace ecz
