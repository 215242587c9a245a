// Host-side TMA tensor-map construction shared by the GEMM and attention
// launchers (driver entry point fetched once through the runtime).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <mutex>

namespace dsv3 {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map (bf16 unless `dtype` says otherwise), 128-byte swizzle, zero fill out of bounds.  dims[0] is the
// contiguous dimension; strides are in bytes for dims[1..rank-1].
inline CUtensorMap make_map(const void* ptr, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                            const uint32_t* box, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B,
                            CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA base address must be 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i)
    TORCH_CHECK(strides_bytes[i] % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  CUresult r = encode_fn()(&m, dtype, rank, const_cast<void*>(ptr), d, s, b, e,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", int(r));
  return m;
}

}  // namespace dsv3
