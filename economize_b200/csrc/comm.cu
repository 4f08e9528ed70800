// Fused all-reduce + residual add + RMSNorm over NVLink peer memory (tensor-parallel row-parallel outputs).
//
// Every rank owns one IPC-exported buffer: a control block (arrival counters and epochs) followed by
// data[2 parities][P slots][slot_elems] bf16. All-reduce number k uses parity k % 2. A rank's push kernel stores its
// partial [rows, hidden] into slot `rank` of every peer's data[parity] with 16-byte P2P stores, fences at system
// scope, and its last CTA adds 1 to every peer's arrival counter[parity] (system-scope atomics over NVLink). The
// consumer kernel on each rank waits (bounded by the global timer) until counter[parity] reaches P * (epoch + 1),
// then sums the P slots of its rows in rank order in fp32 (every rank gets bit-identical sums), adds the residual and
// applies RMSNorm. Parities alternate, and a rank pushes all-reduce k + 2 only after every rank consumed k + 1,
// which it could only do after consuming k, so a slot is never overwritten while it is read.
#include <cstdio>

#include "common.cuh"
#include "launchers.h"

namespace ecz {

namespace {

struct Control {
  unsigned arrivals[2];   // written by peers
  unsigned epoch[2];      // all-reduces of each parity this rank has consumed
  unsigned push_done;     // CTAs of the current push that finished
  unsigned reduce_done;   // CTAs of the current consumer that finished
  unsigned pad[58];
};
static_assert(sizeof(Control) == 256, "control block is 256 bytes");

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) push_kernel(const bf16* __restrict__ src, long elems, PeerPtrs peers,
                                                   int rank, int world, int parity, long slot_elems) {
  pdl_trigger();
  pdl_wait();
  const long vecs = elems / 8;
  for (int p = 0; p < world; ++p) {
    uint8_t* base = static_cast<uint8_t*>(peers.ptr[p]) + sizeof(Control);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(base) +
                                          (static_cast<long>(parity) * world + rank) * slot_elems);
    for (long v = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; v < vecs;
         v += static_cast<long>(gridDim.x) * blockDim.x) {
      dst[v] = reinterpret_cast<const uint4*>(src)[v];
    }
  }
  __syncthreads();  // the CTA's stores are ordered before thread 0's system-scope fence and signal
  if (threadIdx.x == 0) {
    __threadfence_system();
    Control* own = static_cast<Control*>(peers.ptr[rank]);
    const unsigned done = atomicAdd(&own->push_done, 1u);
    if (done == gridDim.x - 1) {  // the last CTA of this push announces it to every rank
      own->push_done = 0;
      __threadfence_system();
      for (int p = 0; p < world; ++p) atomicAdd_system(&static_cast<Control*>(peers.ptr[p])->arrivals[parity], 1u);
    }
  }
}

// One CTA per row block of 4 rows: waits for every rank's partial, sums slots in rank order, adds the residual,
// writes resid_out and the RMSNorm output.
__global__ void __launch_bounds__(256) reduce_rmsnorm_kernel(PeerPtrs peers, int rank, int world, int parity,
                                                             long slot_elems, const bf16* __restrict__ resid,
                                                             const bf16* __restrict__ w, bf16* __restrict__ out,
                                                             bf16* __restrict__ resid_out, int rows, int hidden,
                                                             float eps, unsigned* status) {
  pdl_trigger();
  pdl_wait();
  Control* own = static_cast<Control*>(peers.ptr[rank]);
  __shared__ int ok;
  __shared__ unsigned epoch;
  if (threadIdx.x == 0) {
    epoch = own->epoch[parity];
    const unsigned target = static_cast<unsigned>(world) * (epoch + 1u);
    const unsigned long long start = global_timer_ns();
    int good = 1;
    while (ld_acquire_sys(&own->arrivals[parity]) < target) {
      if (global_timer_ns() - start > kWaitLimitNs) {
        atomicOr(status, kStatusWaitPeer);
        good = 0;
        break;
      }
    }
    ok = good;
  }
  __syncthreads();
  __threadfence();
  if (ok) {
    const bf16* data = reinterpret_cast<const bf16*>(static_cast<uint8_t*>(peers.ptr[rank]) + sizeof(Control)) +
                       static_cast<long>(parity) * world * slot_elems;
    const int nvec = hidden / 8;
    for (int r = blockIdx.x * 4; r < min(rows, blockIdx.x * 4 + 4); ++r) {
      float ss = 0.f;
      // pass 1: sum ranks + residual, write resid_out, accumulate the square sum
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int p = 0; p < world; ++p) {
          const uint4 raw = reinterpret_cast<const uint4*>(data + static_cast<long>(p) * slot_elems +
                                                           static_cast<long>(r) * hidden)[v];
          const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(e[j]);
        }
        // the reduced partial is rounded to bf16 (what an all-reduce of bf16 tensors returns), then added
        uint4 rr = make_uint4(0, 0, 0, 0);
        if (resid != nullptr) rr = reinterpret_cast<const uint4*>(resid + static_cast<long>(r) * hidden)[v];
        const bf16* re = reinterpret_cast<const bf16*>(&rr);
        uint4 so;
        bf16* se = reinterpret_cast<bf16*>(&so);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float red = bf16r(acc[j]);
          const float s = resid != nullptr ? bf16r(red + __bfloat162float(re[j])) : red;
          se[j] = __float2bfloat16(s);
          ss += s * s;
        }
        reinterpret_cast<uint4*>(resid_out + static_cast<long>(r) * hidden)[v] = so;
      }
      __shared__ float red_s[32];
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red_s[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red_s[0] = t;
      }
      __syncthreads();
      const float inv = rsqrtf(red_s[0] / static_cast<float>(hidden) + eps);
      __syncthreads();
      // pass 2: normalize (re-reading the residual row just written: it is in L1/L2)
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        const uint4 so = reinterpret_cast<const uint4*>(resid_out + static_cast<long>(r) * hidden)[v];
        const uint4 ww = reinterpret_cast<const uint4*>(w)[v];
        const bf16* se = reinterpret_cast<const bf16*>(&so);
        const bf16* we = reinterpret_cast<const bf16*>(&ww);
        uint4 o;
        bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
        for (int j = 0; j < 8; ++j) oe[j] = __float2bfloat16(__bfloat162float(we[j]) * bf16r(__bfloat162float(se[j]) * inv));
        reinterpret_cast<uint4*>(out + static_cast<long>(r) * hidden)[v] = o;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned done = atomicAdd(&own->reduce_done, 1u);
    if (done == gridDim.x - 1) {  // every CTA has waited: this all-reduce of the parity is consumed
      own->reduce_done = 0;
      own->epoch[parity] = epoch + 1u;
    }
  }
}

}  // namespace

size_t symm_control_bytes() { return sizeof(Control); }

int launch_push(const void* src, long elems, const PeerPtrs& peers, int rank, int world, int parity, long slot_elems,
                int num_sms, cudaStream_t stream) {
  if (elems % 8 != 0 || elems > slot_elems || world > kMaxPeers) return -1;
  const long vecs = elems / 8;
  const int blocks = static_cast<int>(std::min<long>((vecs + 255) / 256, 4L * num_sms));
  launch_pdl(push_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, stream, static_cast<const bf16*>(src), elems,
             peers, rank, world, parity, slot_elems);
  return 0;
}

int launch_reduce_rmsnorm(const PeerPtrs& peers, int rank, int world, int parity, long slot_elems, const void* resid,
                          const void* w, void* out, void* resid_out, int rows, int hidden, float eps,
                          unsigned* status, cudaStream_t stream) {
  if (hidden % 8 != 0 || static_cast<long>(rows) * hidden > slot_elems) return -1;
  launch_pdl(reduce_rmsnorm_kernel, dim3((rows + 3) / 4), dim3(256), 0, stream, peers, rank, world, parity,
             slot_elems, static_cast<const bf16*>(resid), static_cast<const bf16*>(w), static_cast<bf16*>(out),
             static_cast<bf16*>(resid_out), rows, hidden, eps, status);
  return 0;
}

}  // namespace ecz
