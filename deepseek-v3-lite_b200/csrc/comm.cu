// Symmetric memory for one-process-per-GPU jobs on one NVSwitch box.
//
// Every rank cudaMalloc's one region of the same size, exports it with a CUDA
// IPC handle and opens every peer's handle; the peer base addresses then go
// to the kernels (by value) so a kernel can store straight into another GPU's
// region over NVLink.  Sub-allocation happens in Python with an identical bump
// sequence on every rank, so an offset means the same buffer everywhere.
//
// No counterpart in the reference, which is single-device.
#include <torch/extension.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <cstring>
#include <string>

namespace dsv3 {

namespace {

// (pointer, 64-byte IPC handle) of a fresh zeroed region on the current device.
pybind11::tuple symm_alloc(int64_t nbytes) {
  TORCH_CHECK(nbytes > 0, "symm_alloc: size must be positive");
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)nbytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  std::string bytes(reinterpret_cast<const char*>(&h), sizeof(h));
  return pybind11::make_tuple((int64_t)(uintptr_t)p, pybind11::bytes(bytes));
}

int64_t symm_open(const std::string& handle) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "symm_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return (int64_t)(uintptr_t)p;
}

void symm_close(int64_t peer_ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle((void*)(uintptr_t)peer_ptr)); }

void symm_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree((void*)(uintptr_t)ptr)); }

// A uint8 tensor aliasing [ptr, ptr + nbytes) of this rank's region (no ownership).
at::Tensor symm_view(int64_t ptr, int64_t nbytes, int64_t device) {
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, (int)device);
  return torch::from_blob((void*)(uintptr_t)ptr, {nbytes}, [](void*) {}, opts);
}

}  // namespace

void register_comm(pybind11::module_& m) {
  m.def("symm_alloc", &symm_alloc, "allocate a zeroed IPC-exportable region: (ptr, handle bytes)");
  m.def("symm_open", &symm_open, "map a peer's region from its IPC handle; returns the local address");
  m.def("symm_close", &symm_close, "unmap a peer region");
  m.def("symm_free", &symm_free, "free this rank's region");
  m.def("symm_view", &symm_view, "uint8 tensor view of a region (no ownership)");
}

}  // namespace dsv3
