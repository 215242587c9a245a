// Data-parallel optimizer step over NVLink peer memory (one kernel chain,
// no NCCL): the flat fp32 gradient / fp32 master / bf16 shadow buffers of
// every rank live in a symmetric heap (csrc/comm.cu) and rank r owns the
// contiguous shard [lo_r, hi_r) of each buffer.
//
//   dp_barrier   every rank raises a flag on every peer and waits (bounded)
//                for all peers' flags of the phase (grads complete, norms
//                written, shards written);
//   dp_reduce    reduce-scatter fused with the averaging scale and the
//                squared-norm partial: the shard's gradient is the mean of
//                the peers' gradients, read with 16-byte P2P loads, written
//                into this rank's own buffer;
//   dp_norm      all-gather of the per-rank squared norms through peer
//                stores, then the global clip coefficient (same value on
//                every rank);
//   dp_update    AdamW on the shard (fp32 moments of this rank's shard only:
//                the moment buffers hold [lo, hi) and nothing else)
//                fused with the all-gather: the updated fp32 master and its
//                bf16 shadow are stored straight into every peer's buffers.
//
// Ordering needs no extra credits: a rank zeroes its gradients for the next
// step only after the "shards written" barrier, which every peer raises after
// its reduce (the last reader of this rank's gradients) has finished.
//
// No counterpart in the reference (single device).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include "adamw.cuh"
#include "common.cuh"
#include "status.h"

namespace dsv3 {

namespace {

constexpr int kMaxRanks = 8;
constexpr int kDpPhases = 4;

struct DpArgs {
  unsigned long long peer[kMaxRanks];
  long long off_flags;   // uint32 [kDpPhases][kMaxRanks]
  long long off_norms;   // f32 [kMaxRanks] squared-norm partials (written by every peer)
  int me, R;
  unsigned long long budget_ns;
};

template <typename T>
__device__ __forceinline__ T* at_rank(const DpArgs& a, int r, long long off) {
  return reinterpret_cast<T*>(a.peer[r] + off);
}

__device__ __forceinline__ void remote_signal(uint32_t* flag) {
  asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(flag) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool wait_count(const uint32_t* flag, uint32_t target, unsigned long long budget, unsigned int* status) {
  const uint64_t t0 = globaltimer_ns();
  while ((int)(load_acquire_sys(flag) - target) < 0) {
    if (globaltimer_ns() - t0 > budget) {
      record_error(status, DSV3_ERR_WAIT_PEER);
      return false;
    }
    __nanosleep(128);
  }
  return true;
}

// Lane p signals peer p and waits for peer p's signal.
__global__ void dp_barrier_kernel(DpArgs a, int phase, uint32_t* expect, unsigned int* status) {
  const int p = threadIdx.x;
  if (p < a.R) {
    __threadfence_system();  // everything this rank wrote before (earlier kernels) is visible first
    remote_signal(at_rank<uint32_t>(a, p, a.off_flags) + phase * kMaxRanks + a.me);
    const uint32_t target = expect[phase * kMaxRanks + p] + 1u;
    wait_count(at_rank<uint32_t>(a, a.me, a.off_flags) + phase * kMaxRanks + p, target, a.budget_ns, status);
    expect[phase * kMaxRanks + p] = target;
  }
}

// Mean over ranks of the shard [lo, hi) (float4 granularity), into this rank's
// own buffer; adds the shard's sum of squares into *sq.
__global__ void __launch_bounds__(256) dp_reduce_kernel(DpArgs a, long long off_grad, long long lo4, long long hi4,
                                                        float scale, float* sq) {
  __shared__ float red[8];
  float acc = 0.f;
  float4* own = at_rank<float4>(a, a.me, off_grad);
  for (long long i = lo4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < hi4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < a.R; ++p) {
      const float4 v = __ldcg(at_rank<const float4>(a, p, off_grad) + i);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    s.x *= scale;
    s.y *= scale;
    s.z *= scale;
    s.w *= scale;
    own[i] = s;
    acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(sq, t);
  }
}

// All-gather of the squared-norm partials (lane p stores ours into peer p and
// waits for peer p's), then the clip coefficient from the global norm.
__global__ void dp_norm_kernel(DpArgs a, const float* sq, uint32_t* expect, float max_norm, float* norm_out,
                               float* coef_out, unsigned int* status) {
  const int p = threadIdx.x;
  __shared__ int ok;
  if (p == 0) ok = 1;
  __syncthreads();
  if (p < a.R) {
    at_rank<float>(a, p, a.off_norms)[a.me] = *sq;
    __threadfence_system();
    remote_signal(at_rank<uint32_t>(a, p, a.off_flags) + 1 * kMaxRanks + a.me);
    const uint32_t target = expect[1 * kMaxRanks + p] + 1u;
    if (!wait_count(at_rank<uint32_t>(a, a.me, a.off_flags) + 1 * kMaxRanks + p, target, a.budget_ns, status)) ok = 0;
    expect[1 * kMaxRanks + p] = target;
  }
  __syncthreads();
  if (p == 0) {
    const volatile float* n = at_rank<float>(a, a.me, a.off_norms);
    float tot = 0.f;
    for (int r = 0; r < a.R; ++r) tot += n[r];   // same order on every rank: same coefficient
    const float nrm = sqrtf(tot);
    *norm_out = nrm;
    *coef_out = ok ? fminf(1.0f, max_norm / (nrm + 1e-6f)) : 0.0f;   // a failed exchange skips the update
  }
}

// AdamW on the shard [lo, hi) (4 elements per thread step); the new master and
// shadow go to every rank's buffers (this rank's own included).
__global__ void __launch_bounds__(256) dp_update_kernel(DpArgs a, long long off_master, long long off_grad,
                                                        long long off_shadow, float* __restrict__ m,
                                                        float* __restrict__ v, long long lo4, long long hi4,
                                                        long long n_decay, AdamHyper h, const float* coef_ptr) {
  const float coef = *coef_ptr;
  const float4* g4 = at_rank<const float4>(a, a.me, off_grad);
  const float4* p4 = at_rank<const float4>(a, a.me, off_master);
  for (long long i = lo4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < hi4;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 g = g4[i];
    float4 p = p4[i];
    float4 mm = reinterpret_cast<float4*>(m)[i - lo4], vv = reinterpret_cast<float4*>(v)[i - lo4];
    const long long e = 4 * i;
    adamw_elem(p.x, mm.x, vv.x, g.x * coef, e < n_decay, h);
    adamw_elem(p.y, mm.y, vv.y, g.y * coef, e + 1 < n_decay, h);
    adamw_elem(p.z, mm.z, vv.z, g.z * coef, e + 2 < n_decay, h);
    adamw_elem(p.w, mm.w, vv.w, g.w * coef, e + 3 < n_decay, h);
    reinterpret_cast<float4*>(m)[i - lo4] = mm;
    reinterpret_cast<float4*>(v)[i - lo4] = vv;
    const uint2 sh = make_uint2(pack_bf16x2(p.x, p.y), pack_bf16x2(p.z, p.w));
    for (int r = 0; r < a.R; ++r) {
      at_rank<float4>(a, r, off_master)[i] = p;
      at_rank<uint2>(a, r, off_shadow)[i] = sh;
    }
  }
}

DpArgs make_args(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, int64_t me,
                 int64_t budget_ns) {
  TORCH_CHECK(peers.size() >= 1 && peers.size() <= kMaxRanks, "dp: 1..8 ranks");
  TORCH_CHECK(offs.size() == 2, "dp: offs = [flags, norms]");
  DpArgs a{};
  a.R = (int)peers.size();
  for (int r = 0; r < a.R; ++r) a.peer[r] = (unsigned long long)peers[r];
  a.off_flags = offs[0];
  a.off_norms = offs[1];
  a.me = (int)me;
  a.budget_ns = (unsigned long long)budget_ns;
  TORCH_CHECK(a.me >= 0 && a.me < a.R, "dp: rank out of range");
  return a;
}

int grid_for(long long n4) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (int)std::max<long long>(1, std::min<long long>(4LL * sms, (n4 + 255) / 256));
}

}  // namespace

void dp_barrier(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, int64_t me, int64_t budget_ns,
                int64_t phase, at::Tensor& expect) {
  const DpArgs a = make_args(peers, offs, me, budget_ns);
  TORCH_CHECK(phase >= 0 && phase < kDpPhases, "dp_barrier: bad phase");
  const at::cuda::CUDAGuard guard(expect.device());
  dp_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(a, (int)phase,
                                                                     reinterpret_cast<uint32_t*>(expect.data_ptr()),
                                                                     status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_reduce(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, int64_t me, int64_t budget_ns,
               int64_t off_grad, int64_t lo, int64_t hi, double scale, at::Tensor& sq) {
  const DpArgs a = make_args(peers, offs, me, budget_ns);
  TORCH_CHECK(lo % 4 == 0 && hi % 4 == 0 && off_grad % 16 == 0, "dp_reduce: 16-byte aligned shard");
  if (hi <= lo) return;
  const at::cuda::CUDAGuard guard(sq.device());
  dp_reduce_kernel<<<grid_for((hi - lo) / 4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(a, off_grad, lo / 4, hi / 4,
                                                                                         (float)scale,
                                                                                         sq.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_norm(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, int64_t me, int64_t budget_ns,
             const at::Tensor& sq, at::Tensor& expect, double max_norm, at::Tensor& norm, at::Tensor& coef) {
  const DpArgs a = make_args(peers, offs, me, budget_ns);
  const at::cuda::CUDAGuard guard(sq.device());
  dp_norm_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(a, sq.data_ptr<float>(),
                                                                  reinterpret_cast<uint32_t*>(expect.data_ptr()),
                                                                  (float)max_norm, norm.data_ptr<float>(),
                                                                  coef.data_ptr<float>(), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_update(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, int64_t me, int64_t budget_ns,
               int64_t off_master, int64_t off_grad, int64_t off_shadow, at::Tensor& m, at::Tensor& v, int64_t lo,
               int64_t hi, int64_t n_decay, double lr, double beta1, double beta2, double eps, double wd,
               int64_t step, const at::Tensor& coef) {
  const DpArgs a = make_args(peers, offs, me, budget_ns);
  TORCH_CHECK(lo % 4 == 0 && hi % 4 == 0 && off_master % 16 == 0 && off_grad % 16 == 0 && off_shadow % 8 == 0,
              "dp_update: aligned shard");
  TORCH_CHECK(m.is_contiguous() && v.is_contiguous() && m.numel() == hi - lo && v.numel() == hi - lo,
              "dp_update: moments must hold exactly the shard [lo, hi)");
  if (hi <= lo) return;
  const AdamHyper h{(float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd,
                    1.0f - (float)std::pow(beta1, (double)step), (float)std::sqrt(1.0 - std::pow(beta2, (double)step))};
  const at::cuda::CUDAGuard guard(m.device());
  dp_update_kernel<<<grid_for((hi - lo) / 4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      a, off_master, off_grad, off_shadow, m.data_ptr<float>(), v.data_ptr<float>(), lo / 4, hi / 4, n_decay, h,
      coef.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_dp(pybind11::module_& m) {
  m.def("dp_barrier", &dp_barrier, "bounded all-rank barrier over peer flags");
  m.def("dp_reduce", &dp_reduce, "reduce-scatter (mean) of a gradient shard over P2P loads, with its squared norm");
  m.def("dp_norm", &dp_norm, "all-gather of squared-norm partials and the global clip coefficient");
  m.def("dp_update", &dp_update, "AdamW on this rank's shard fused with the all-gather of master and shadow");
}

}  // namespace dsv3
