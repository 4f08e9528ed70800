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
//   -5  no current CUDA device           -6  a launch or the clearing of the status word failed
//
// A return of 0 means the work was queued, not that it succeeded. Every wait inside the kernels is bounded; a wait
// that gives up records a bit in the status word of the scratch array (1: a tile load, 2: a free stage, 4: the
// accumulator) and the kernel returns without writing its tile, so y is undefined after such a call. Read the word
// with ecz_linear_bf16_noalloc_status once the call's stream has been synchronized; each call clears it first.
//
//   int ecz_linear_bf16_noalloc_status(unsigned* status_out);
//     *status_out = the status word of the current device's scratch array (0: every wait of the last call on this
//     device completed). A synchronous 4-byte device-to-host copy; returns 0, or -1/-4/-5/-6 as above.
//
//   int ecz_noalloc_wait_selftest(unsigned long long limit_ns, void* stream);
//     Clears the status word and launches one thread that waits at most limit_ns (1 ns .. 1 s) on a barrier that
//     nothing completes, so the wait runs out and records 1 in the word: a check of the status path that needs no
//     fault. Returns 0 when launched.
//
// The first call on a device sets that device up (it looks up the array's device address with
// cudaGetSymbolAddress and records it), so make the first call on each device before any stream capture. The
// recorded address belongs to the device's current context: after cudaDeviceReset (or any other teardown of the
// primary context) the library must be reloaded before these entry points are used on that device again. Every call
// shares the one array per device and leaves its contents behind: calls whose work overlaps on the GPU (other
// streams, other host threads) race on it and must be serialized by the caller.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define ECZ_NOALLOC_SCRATCH_FLOATS (4u << 20)

int ecz_linear_bf16_noalloc(const void* x, const void* w, void* y, int M, int N, int K, void* stream);
int ecz_linear_bf16_noalloc_status(unsigned* status_out);
int ecz_noalloc_wait_selftest(unsigned long long limit_ns, void* stream);

#ifdef __cplusplus
}
#endif
