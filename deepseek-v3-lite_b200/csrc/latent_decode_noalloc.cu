// Allocation-free absorbed-MLA decode (see latent_decode_noalloc.h for the
// contract).  Same kernels as the torch entry point; the split-K partials
// live in a fixed file-scope device array instead of a caller tensor.
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

// Device address of g_decode_scratch per device, looked up once per device.
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
  const int chunk = 256;
  const int nsplit = (max_len + chunk - 1) / chunk;
  const long long need = (long long)B * H * nsplit * (2 + R);
  if (need > DSV3_NOALLOC_SCRATCH_FLOATS) return DSV3_NOALLOC_TOO_LARGE;
  int err = DSV3_NOALLOC_OK;
  float* scratch = scratch_for_current_device(&err);
  if (!scratch) return err;
  float* pm = scratch;
  float* pl = pm + (long long)B * H * nsplit;
  float* po = pl + (long long)B * H * nsplit;
  const int warps = B * H * nsplit;
  dsv3::latent_decode_split_kernel<<<(warps + 3) / 4, 128, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(q_lat), static_cast<const __nv_bfloat16*>(q_pe), static_cast<const __nv_bfloat16*>(kv),
      static_cast<const __nv_bfloat16*>(pe), lens, H, R, dr, (long)kv_batch_stride, (long)pe_batch_stride, 1, chunk, nsplit,
      B * H, scale, pm, pl, po);
  dsv3::latent_decode_merge_kernel<<<B * H, 128, 0, stream>>>(pm, pl, po, nsplit, R, B * H, static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? DSV3_NOALLOC_OK : DSV3_NOALLOC_CUDA_ERROR;
}
