// Shared device helpers of the economize_b200 sm_100a kernels: bounded mbarrier waits, TMA loads, tcgen05
// (TMEM allocation, UMMA issue/commit, TMEM loads) and small numeric utilities.
//
// Every wait on an mbarrier or a flag is bounded by the global timer: after `kWaitLimitNs` the waiting thread
// records a code in the caller's status word and returns false, so a broken pipeline ends the kernel with an error
// status the host reads instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <utility>

#include "launchers.h"  // KVPages, KVLayout

namespace ecz {

using bf16 = __nv_bfloat16;

// Status codes (bit flags) written to the per-device status word.
enum StatusCode : unsigned {
  kStatusOk = 0u,
  kStatusWaitFull = 1u,       // consumer gave up waiting for a TMA stage
  kStatusWaitEmpty = 2u,      // producer gave up waiting for a free stage
  kStatusWaitAccum = 4u,      // epilogue gave up waiting for the accumulator
  kStatusWaitPeer = 8u,       // a fused collective gave up waiting for a peer's flag
  kStatusBadShape = 16u,      // a launch saw a shape it cannot handle (kernel returned without work)
  kStatusBadIndex = 32u,      // an index argument lay outside its table (the kernel clamped it and reported it)
};

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier --------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase of parity `parity` of `bar` completed. Returns false (and sets `code` in *status) when the
// wait exceeds `limit_ns` (kWaitLimitNs by default) or when *abort became non-zero (another role of the CTA gave up
// already).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* status, unsigned code,
                                          volatile int* abort, unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u) {
      if (abort != nullptr && *abort) return false;
      if (global_timer_ns() - start > limit_ns) {
        if (status != nullptr) atomicOr(status, code);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
}

// ---- TMA -------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of the box at (x = inner coordinate, y = outer coordinate) into shared memory, completing on `bar`.
// x must be a multiple of 16 bytes / element size (callers pass multiples of 64 bf16 elements).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---- tcgen05 ---------------------------------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32); the whole warp executes it. The base address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored with the 128-byte swizzle (rows of 64 bf16,
// 8-row groups 1024 bytes apart): start >> 4 in bits [0,14), LBO (unused for this layout, 16 B) in [16,30),
// SBO = 1024 B in [32,46), descriptor version 1 in [46,48), layout type SWIZZLE_128B (2) in [61,64).
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Descriptor of an MN-major operand stored as rows of 64 bf16 along MN with the 128-byte swizzle (the layout a TMA
// box {64 (MN), rows (K)} with SWIZZLE_128B produces): LBO = byte distance between consecutive 64-element MN
// blocks, SBO = 1024 B between consecutive 8-row K groups.
__device__ __forceinline__ uint64_t desc_mnmajor_sw128(uint32_t smem_addr, uint32_t mn_block_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((mn_block_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor of kind::f16 with bf16 A and B, fp32 accumulation, shape M x N, both operands K-major
// unless `b_mn_major` (bit 16).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n, bool b_mn_major = false) {
  return (1u << 4)                                   // D format: f32
         | (1u << 7)                                 // A format: bf16
         | (1u << 10)                                // B format: bf16
         | ((b_mn_major ? 1u : 0u) << 16)            // B major
         | (static_cast<uint32_t>(n >> 3) << 17)     // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);    // M >> 4
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same MMA with A read from tensor memory: row m of A in TMEM lane m, its K elements packed two per 32-bit column
// from column `a_tmem` (16 bf16 per MMA: 8 columns), B from shared memory.
__device__ __forceinline__ void umma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Load 16 consecutive fp32 columns of this thread's TMEM lane (32x32b shape: warp w of a warpgroup reads lanes
// 32w..32w+31, so `taddr` carries the lane base in bits [16,32)).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive fp32 columns of this thread's TMEM lane (the 32x32b shape of tmem_ld16), and wait for it.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Store 8 / 16 consecutive 32-bit words into this thread's TMEM lane (no wait: callers wait once for a batch).
__device__ __forceinline__ void tmem_st_u32x8(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_u32x16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Load 32 consecutive fp32 columns of this thread's TMEM lane with one wait (two x16 loads in flight).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr + 16));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Generic-proxy writes to shared memory become visible to the async proxy (tcgen05.mma, TMA store) after this.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- thread-block clusters ----------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 16-byte load from CTA `rank`'s shared memory at the address `local_addr` has in this CTA. Not volatile: the
// partials are immutable between the two cluster barriers, so the compiler may batch these loads.
__device__ __forceinline__ float4 ld_dsmem_v4(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float4 v;
  asm("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(remote));
  return v;
}

// ---- programmatic dependent launch ---------------------------------------------------------------------------
// Kernels launched with launch_pdl may start while the previous kernel of the stream is still running. Each kernel
// lets its own dependents start early (pdl_trigger) and waits for its predecessor (pdl_wait) before it reads the
// predecessor's outputs or writes any global memory. Both are no-ops without a programmatic dependency.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

bool pdl_enabled();

// Raise a kernel's dynamic shared-memory limit on the CURRENT device. The attribute belongs to the (kernel, device)
// pair, so a process that launches on several GPUs must set it on each; this records the largest size set for each
// pair (under a lock, so host threads may launch concurrently) and sets it again only for a larger request.
inline cudaError_t set_max_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // the largest size set per (kernel, device)
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find({kernel, device});
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess) done[{kernel, device}] = bytes;
  return err;
}

template <typename... KArgs>
inline cudaError_t set_max_smem(void (*kernel)(KArgs...), int bytes) {
  return set_max_smem(reinterpret_cast<const void*>(kernel), bytes);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- bounds-checked builds ---------------------------------------------------------------------------------------
// Built with -DECZ_CHECK (ECZ_CHECK=1 python setup.py build_ext --inplace: the module economize_b200._C_check, loaded
// when the environment has ECZ_CHECK=1), kernels check the indices they read from device memory before those
// address memory; a bad one sets kStatusBadIndex in the device status word and the access is skipped. Nothing
// traps, so the context stays usable and the host reads the flag (ops.require().status). Regular builds compile
// the checks away.
#ifdef ECZ_CHECK
constexpr bool kCheckedBuild = true;
#else
constexpr bool kCheckedBuild = false;
#endif

__device__ __forceinline__ bool index_ok(bool in_range, unsigned* status) {
  if (!kCheckedBuild || in_range) return true;
  if (status != nullptr) atomicOr(status, kStatusBadIndex);
  return false;
}

// ---- KV cache addressing ----------------------------------------------------------------------------------------
// Where the K (or V) row of (sequence b, KV head kvh, logical slot s) lives. Contiguous caches [B, Hkv, S, D]: row
// (b Hkv + kvh) S + s. Paged caches: logical chunk s / 128 of sequence b sits in page table[b * max_chunks + s / 128]
// of a pool whose pages start page_rows rows apart and hold the KV heads' 128-slot blocks one after another (a pool
// [P, 2, Hkv, 128, D] of K and V pages has page_rows = 2 Hkv 128 from either base). A ring cache of a sliding-window
// layer is a page table that maps chunk c to the row's page c mod R.
__device__ __forceinline__ size_t kv_row(const KVPages& pg, int b, int Hkv, int kvh, int S, int s) {
  if (pg.table == nullptr) return (static_cast<size_t>(b) * Hkv + kvh) * S + s;
  const int page = pg.table[static_cast<size_t>(b) * pg.max_chunks + (s >> 7)];
  return static_cast<size_t>(page) * pg.page_rows + static_cast<size_t>(kvh) * 128 + (s & 127);
}

// Every layer of a cache (kernels that touch all layers at once: KV compaction, KIVI coding). The K row of
// (layer l, sequence b, head kvh, slot s) is l layer_rows + kv_row(l's pages, ...), its V row v_rows further.
// Contiguous [L, 2, B, Hkv, S, D]: layer_rows = 2 B Hkv S, v_rows = B Hkv S, no table. Paged pool [P, 2, Hkv, 128,
// D] with tables [L, B, C]: layer_rows = 0 (pages are global), v_rows = Hkv 128, table_stride = B C.
__device__ __forceinline__ size_t kv_layer_row(const KVLayout& L, int layer, int kv, int b, int Hkv, int kvh, int S,
                                               int s) {
  KVPages pg = L.pages;
  if (pg.table != nullptr) pg.table += static_cast<size_t>(layer) * L.table_stride;
  return static_cast<size_t>(layer) * L.layer_rows + static_cast<size_t>(kv) * L.v_rows +
         kv_row(pg, b, Hkv, kvh, S, s);
}

// ---- numerics --------------------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

}  // namespace ecz
