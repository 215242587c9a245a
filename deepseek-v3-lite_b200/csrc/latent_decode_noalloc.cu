// Allocation-free absorbed-MLA decode (see latent_decode_noalloc.h for the
// contract).  It calls the same launcher as the torch entry point
// `latent_decode` (latent_decode.cuh: the tensor-core kernel where the sizes
// fit, else the per-warp kernel, then the merge), so both run the same
// kernels on the same inputs; only the split-K partials live in a fixed
// file-scope device array instead of a caller tensor.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "latent_decode_noalloc.h"

#define DSV3_NOALLOC_SCRATCH_FLOATS (4 * 1024 * 1024)
#define DSV3_NOALLOC_MAX_DEVICES 64

namespace dsv3 {
namespace {
typedef __nv_bfloat16 bf16;
#include "latent_decode.cuh"
}  // namespace
}  // namespace dsv3

// Split-K partials (max, sum, partial output) of the most recent call.
static __device__ __align__(256) float g_decode_scratch[DSV3_NOALLOC_SCRATCH_FLOATS];

// Device address of g_decode_scratch per device, looked up once per device and
// kept for the life of the process.  A cudaDeviceReset (or any other
// destruction of the device's primary context) invalidates it; this library
// does not support calls after such a reset.
static std::atomic<float*> g_scratch_addr[DSV3_NOALLOC_MAX_DEVICES];

static float* scratch_for_current_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= DSV3_NOALLOC_MAX_DEVICES) {
    *err = DSV3_NOALLOC_CUDA_ERROR;
    return nullptr;
  }
  float* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (p) return p;
  void* addr = nullptr;
  // The host-side symbol is only a stand-in; the kernels need the device address.
  if (cudaGetSymbolAddress(&addr, g_decode_scratch) != cudaSuccess || addr == nullptr) {
    *err = DSV3_NOALLOC_CUDA_ERROR;
    return nullptr;
  }
  g_scratch_addr[dev].store(static_cast<float*>(addr), std::memory_order_release);
  return static_cast<float*>(addr);
}

extern "C" __attribute__((visibility("default"))) int dsv3_latent_decode_noalloc(
    const void* q_lat, const void* q_pe, const void* kv, const void* pe, const int* lens, int B, int H, int R, int dr,
    long long kv_batch_stride, long long pe_batch_stride, int max_len, float scale, void* out, cudaStream_t stream) {
  if (!q_lat || !q_pe || !kv || !pe || !lens || !out || B <= 0 || H <= 0 || R <= 0 || R > 1024 || dr < 0 ||
      dr > 128 || max_len <= 0)
    return DSV3_NOALLOC_BAD_ARGS;
  if (dsv3::latent_decode_scratch_floats(B, H, R, max_len) > DSV3_NOALLOC_SCRATCH_FLOATS) return DSV3_NOALLOC_TOO_LARGE;
  int err = DSV3_NOALLOC_OK;
  float* scratch = scratch_for_current_device(&err);
  if (!scratch) return err;
  dsv3::LatentDecodeArgs a{};
  a.q_lat = static_cast<const __nv_bfloat16*>(q_lat);
  a.q_pe = static_cast<const __nv_bfloat16*>(q_pe);
  a.kv = static_cast<const __nv_bfloat16*>(kv);
  a.pe = static_cast<const __nv_bfloat16*>(pe);
  a.lens = lens;
  a.B = B;
  a.H = H;
  a.R = R;
  a.dr = dr;
  a.kv_bs = (long)kv_batch_stride;
  a.pe_bs = (long)pe_batch_stride;
  a.qpb = 1;
  a.max_len = max_len;
  a.scale = scale;
  a.scratch = scratch;
  a.out = static_cast<__nv_bfloat16*>(out);
  // the launches' own status (not cudaGetLastError, which would also report,
  // and clear, an unrelated earlier error of this thread)
  return dsv3::launch_latent_decode(a, stream) == cudaSuccess ? DSV3_NOALLOC_OK : DSV3_NOALLOC_CUDA_ERROR;
}
