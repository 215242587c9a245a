// Fused optimizer kernels over flat fp32 parameter / gradient buffers:
//   grad_sqsum   deterministic two-level sum of squares (global gradient norm);
//   clip_coef    min(1, max_norm / (norm + 1e-6)) on the device (no host sync);
//   adamw_flat   decoupled-weight-decay AdamW (same update rule as
//                torch.optim.AdamW) that also refreshes the bf16 shadow
//                weights the GEMMs read, and applies the clip coefficient.
// Elements [0, n_decay) of a buffer get weight decay, the rest do not.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "adamw.cuh"
#include "common.cuh"

namespace dsv3 {

namespace {

constexpr int kSqBlocks = 1024;

__global__ void sqsum_kernel(const float* __restrict__ g, long n, float* __restrict__ partial) {
  __shared__ float s[32];
  float acc = 0.f;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = g[i];
    acc += v * v;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? s[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
  }
}

__global__ void sum_partials_kernel(const float* __restrict__ partial, int n, float* __restrict__ out) {
  __shared__ float s[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? s[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) *out = v;
  }
}

__global__ void clip_coef_kernel(const float* __restrict__ sqsum, float max_norm, float* __restrict__ norm,
                                 float* __restrict__ coef) {
  const float nrm = sqrtf(*sqsum);
  *norm = nrm;
  *coef = fminf(1.0f, max_norm / (nrm + 1e-6f));
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ shadow, long n, long n_decay,
                             float lr, float beta1, float beta2, float eps, float wd, float bc1, float bc2_sqrt,
                             const float* __restrict__ coef_ptr) {
  const float coef = coef_ptr ? *coef_ptr : 1.0f;
  const AdamHyper h{lr, beta1, beta2, eps, wd, bc1, bc2_sqrt};
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float pi = p[i], mi = m[i], vi = v[i];
    adamw_elem(pi, mi, vi, g[i] * coef, i < n_decay, h);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (shadow) shadow[i] = __float2bfloat16(pi);
  }
}

int grid_for(long n) { return (int)std::min<long>(4 * 148 * 8, (n + 255) / 256); }

}  // namespace

// Adds the sum of squares of each tensor (fp32, contiguous) into out[0].
void grad_sqsum(const std::vector<at::Tensor>& grads, at::Tensor& scratch, at::Tensor& out) {
  TORCH_CHECK(scratch.numel() >= kSqBlocks * (long)std::max<size_t>(1, grads.size()), "grad_sqsum: scratch too small");
  auto st = at::cuda::getCurrentCUDAStream();
  int used = 0;
  for (const auto& t : grads) {
    TORCH_CHECK(t.is_contiguous() && t.scalar_type() == at::kFloat, "grad_sqsum: contiguous fp32");
    if (t.numel() == 0) continue;
    sqsum_kernel<<<kSqBlocks, 256, 0, st>>>(t.data_ptr<float>(), t.numel(), scratch.data_ptr<float>() + used);
    used += kSqBlocks;
  }
  if (used == 0) {
    C10_CUDA_CHECK(cudaMemsetAsync(out.data_ptr<float>(), 0, sizeof(float), st));
    return;
  }
  sum_partials_kernel<<<1, 1024, 0, st>>>(scratch.data_ptr<float>(), used, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void clip_coef(const at::Tensor& sqsum, double max_norm, at::Tensor& norm, at::Tensor& coef) {
  clip_coef_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(sqsum.data_ptr<float>(), (float)max_norm,
                                                                   norm.data_ptr<float>(), coef.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_flat(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, c10::optional<at::Tensor> shadow,
                int64_t n_decay, double lr, double beta1, double beta2, double eps, double wd, int64_t step,
                c10::optional<at::Tensor> coef) {
  const long n = p.numel();
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw: contiguous");
  TORCH_CHECK(g.numel() == n && m.numel() == n && v.numel() == n, "adamw: sizes");
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(p.device());
  const float bc1 = 1.0f - (float)std::pow(beta1, (double)step);
  const float bc2s = (float)std::sqrt(1.0 - std::pow(beta2, (double)step));
  __nv_bfloat16* sh = nullptr;
  if (shadow) {
    TORCH_CHECK(shadow->numel() == n && shadow->is_contiguous(), "adamw: shadow size");
    sh = reinterpret_cast<__nv_bfloat16*>(shadow->data_ptr());
  }
  adamw_kernel<<<grid_for(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(p.data_ptr<float>(), g.data_ptr<float>(),
      m.data_ptr<float>(), v.data_ptr<float>(), sh, n, n_decay, (float)lr, (float)beta1, (float)beta2, (float)eps,
      (float)wd, bc1, bc2s, coef ? coef->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_optim(pybind11::module_& m) {
  m.def("grad_sqsum", &grad_sqsum, "deterministic sum of squares of fp32 buffers");
  m.def("clip_coef", &clip_coef, "global-norm clip coefficient on the device");
  m.def("adamw_flat", &adamw_flat, "fused AdamW over a flat buffer (+ bf16 shadow refresh)");
}

}  // namespace dsv3
