// Allocation-free C entry point of the tcgen05 GEMM (Y = X . W^T, bf16).
//
// This entry point has no counterpart in the reference (economize ships no native code); it is an addition of this
// library for callers that cannot allocate GPU memory: plugins hosted by a runtime that owns all device memory and
// forbids raw cudaMalloc calls, code that runs on a latency-critical path where a synchronizing cudaMalloc/cudaFree
// would stall every stream of the device, and C programs that do not link PyTorch's caching allocator.
//
// The split-K partial sums that ecz_linear_bf16 otherwise takes from the caching allocator live here in one
// file-scope device array of ECZ_NOALLOC_SCRATCH_FLOATS fp32 values (16 MiB, plus a status word), which every GPU
// that loads the library holds until the process exits.
//
//   int ecz_linear_bf16_noalloc(const void* x, const void* w, void* y, int M, int N, int K, void* stream);
//
//   x  [M, K] bf16, row-major, 16-byte aligned      w [N, K] bf16, row-major, 16-byte aligned
//   y  [M, N] bf16 output                            stream: a cudaStream_t (nullptr = legacy default stream)
//   K must be a multiple of 8 and N a multiple of 4. The call is asynchronous on `stream`.
//
// Returns 0 when the kernels were launched; a negative code (with a message on stderr) otherwise:
//   -1  bad shape or alignment          -2  the split-K partials (splits * M * N floats) exceed the scratch array
//   -3  a TMA descriptor failed          -4  the scratch array's device address could not be obtained
//   -5  no current CUDA device           -6  the launch failed
//
// The first call on a device sets that device up (it looks up the array's device address with
// cudaGetSymbolAddress and records it), so make the first call on each device before any stream capture. Every call
// shares the one array per device and leaves its contents behind: calls whose work overlaps on the GPU (other
// streams, other host threads) race on it and must be serialized by the caller.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define ECZ_NOALLOC_SCRATCH_FLOATS (4u << 20)

int ecz_linear_bf16_noalloc(const void* x, const void* w, void* y, int M, int N, int K, void* stream);

#ifdef __cplusplus
}
#endif
