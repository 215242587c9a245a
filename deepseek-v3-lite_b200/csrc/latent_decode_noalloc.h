// Allocation-free entry point for the absorbed-MLA decode step.
//
// This entry point has no counterpart in the reference implementation; it is
// an addition of this library for callers that cannot allocate device
// memory while they run -- for example an inference server that replays a
// captured CUDA graph or runs under a fixed memory budget, or a host program
// written in C that has no caching allocator at hand.  The ordinary entry
// point (`latent_decode` in the Python module) takes a caller-provided
// scratch tensor; this one keeps its scratch in a fixed-size device array
// inside the library instead.
//
// Contract:
//   * the caller passes inputs and outputs (device pointers) and a stream;
//   * scratch is the file-scope device array in latent_decode_noalloc.cu of
//     DSV3_NOALLOC_SCRATCH_FLOATS floats (16 MiB); every GPU that loads the
//     library holds it until the process exits;
//   * the call returns DSV3_NOALLOC_TOO_LARGE (and launches nothing) when
//     B * H * ceil(max_len / 256) * (R + 2) exceeds that size;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture;
//   * all calls share the one array, so calls whose kernels overlap on the
//     GPU (different streams, no ordering between them) race on it;
//   * the looked-up address is cached per device for the life of the
//     process; calls after a cudaDeviceReset are not supported;
//   * lens[b] must not exceed max_len: cache rows past
//     ceil(max_len / 256) * 256 are not read (the result is then computed
//     over a truncated cache, silently; no out-of-bounds access occurs);
//   * a row with lens[b] == 0 yields zeros;
//   * the return value reports argument errors and the status of this
//     call's own kernel launches (asynchronous faults surface later, as for
//     any CUDA launch);
//   * no cudaMalloc / cudaFree or allocating library routine is called.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSV3_NOALLOC_OK 0
#define DSV3_NOALLOC_TOO_LARGE 1
#define DSV3_NOALLOC_BAD_ARGS 2
#define DSV3_NOALLOC_CUDA_ERROR 3

// q_lat [B, H, R] bf16, q_pe [B, H, dr] bf16, kv [B, *, R] bf16 with batch
// stride kv_batch_stride elements, pe [B, *, dr] bf16 with batch stride
// pe_batch_stride, lens [B] int32 (valid cache rows per batch row, each
// <= max_len) -> out [B, H, R] bf16 = softmax(scale * (q_lat.kv + q_pe.pe)) kv.
int dsv3_latent_decode_noalloc(const void* q_lat, const void* q_pe, const void* kv, const void* pe,
                               const int* lens, int B, int H, int R, int dr, long long kv_batch_stride,
                               long long pe_batch_stride, int max_len, float scale, void* out,
                               cudaStream_t stream);

#ifdef __cplusplus
}
#endif
