// DeepSeekMoE routing and token movement on one GPU:
//   router_topk     sigmoid scores, bias-shifted top-k, normalised weights and
//                   per-expert counts (one warp per token, fp32 throughout);
//   permute_plan    per-expert row ranges padded to 256 rows (one CTA-pair GEMM tile),
//                   the tile -> expert map used by the grouped GEMMs;
//   permute_scatter destination row of every (token, slot) assignment;
//   gather_rows     expert-sorted copy of the activations (zero padding rows);
//   combine_fwd     out[t] += sum_j w[t,j] * y[row(t,j)]   (fp32 residual);
//   combine_bwd     dy[row] = w * dout[t], dw[t,j] = <dout[t], y[row]>;
//   unpermute_bwd   dx[t] += sum_j dx_sorted[row(t,j)];
//   router_bwd      gradient of the normalised sigmoid weights w.r.t. logits.
// Nothing here synchronises with the host: counts stay on the device and the
// grouped GEMMs skip tiles whose expert id is negative.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "status.h"

namespace dsv3 {

namespace {

constexpr int kMaxExpertsPerLane = 8;  // E <= 256
constexpr int kGroupRows = 256;        // expert row ranges: multiples of one CTA-pair GEMM tile

// Sigmoid + bias top-k routing, one warp per token (TPW tokens per warp in
// turn).  NL experts per lane (E <= 32 * NL) keeps the arg-max loops fully
// unrolled over live registers only.  Per-expert counts are histogrammed in
// shared memory and added to the global counts once per CTA.
template <int NL>
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, long ldl,
                                                          const float* __restrict__ bias, int T, int E, int k,
                                                          float route_scale, int* __restrict__ idx,
                                                          float* __restrict__ w, float* __restrict__ s_sel,
                                                          int* __restrict__ counts, int tpw) {
  __shared__ int hist[32 * NL];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  float bias_l[NL];
#pragma unroll
  for (int i = 0; i < NL; ++i) bias_l[i] = lane + 32 * i < E ? bias[lane + 32 * i] : 0.f;
  for (int tt = 0; tt < tpw; ++tt) {
    const int t = warp_global * tpw + tt;
    if (t >= T) break;
    float sc[NL], bsc[NL];
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        const float s = 1.0f / (1.0f + __expf(-logits[(size_t)t * ldl + e]));
        sc[i] = s;
        bsc[i] = s + bias_l[i];
      } else {
        sc[i] = 0.f;
        bsc[i] = -INFINITY;
      }
    }
    float total = 0.f, my_s = 0.f;
    int my_e = 0;
    for (int j = 0; j < k; ++j) {
      // warp arg-max over the biased scores; ties go to the lower expert id
      float bv = -INFINITY;
      int be = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < NL; ++i) {
        const int e = lane + 32 * i;
        if (e < E && (bsc[i] > bv || (bsc[i] == bv && e < be))) {
          bv = bsc[i];
          be = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ov > bv || (ov == bv && oe < be)) {
          bv = ov;
          be = oe;
        }
      }
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < NL; ++i)
        if (lane + 32 * i == be) {
          s = sc[i];
          bsc[i] = -INFINITY;
        }
      s = __shfl_sync(0xffffffffu, s, be & 31);
      if (lane == j) {
        my_s = s;
        my_e = be;
      }
      total += s;
    }
    if (lane < k) {
      idx[(size_t)t * k + lane] = my_e;
      s_sel[(size_t)t * k + lane] = my_s;
      w[(size_t)t * k + lane] = my_s / fmaxf(total, 1e-10f) * route_scale;
      atomicAdd(&hist[my_e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (hist[e]) atomicAdd(&counts[e], hist[e]);
}

// Single block.  row_off[e] = sum_{e'<e} pad256(counts[e']); tile_group[i] =
// expert owning 128-row tile i (or -1); cursor zeroed; src[0..P) = -1.
__global__ void permute_plan_kernel(const int* __restrict__ counts, int E, int* __restrict__ row_off,
                                    int* __restrict__ tile_group, int max_tiles, int* __restrict__ cursor,
                                    int* __restrict__ src, int P, int src_tail_only) {
  extern __shared__ int off_s[];  // E + 1
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      off_s[e] = acc;
      acc += (counts[e] + kGroupRows - 1) / kGroupRows * kGroupRows;
    }
    off_s[E] = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) row_off[e] = off_s[e];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cursor[e] = 0;
  for (int i = threadIdx.x; i < max_tiles; i += blockDim.x) {
    const int row = i * 128;
    int g = -1;
    if (row < off_s[E]) {
      int lo = 0, hi = E - 1;  // last e with off_s[e] <= row
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off_s[mid] <= row) lo = mid;
        else hi = mid - 1;
      }
      g = lo;
    }
    tile_group[i] = g;
  }
  // src = -1 everywhere, or (permute_gather writes the expert ranges) only
  // past the last expert's range
  for (int i = (src_tail_only ? off_s[E] : 0) + threadIdx.x; i < P; i += blockDim.x) src[i] = -1;
}

// Permutation fused with the gather.  A chunk CTA takes kPgThreads / k
// consecutive tokens: each (token, slot) counts itself into its expert in
// shared memory, one thread per expert reserves the chunk's rows of that
// expert with a single global atomicAdd on the cursor, and each token row is
// then read once and stored to its k destination rows.  The first E CTAs zero
// the padding rows [row_off[e] + counts[e], row_off[e + 1]) of expert e and set
// their src to -1.  Replaces permute_scatter + gather_rows (and permute_plan's
// src initialisation).  Row order inside an expert's range depends on the
// order in which chunks reserve; src / dst describe whichever order results.
constexpr int kPgThreads = 256;
constexpr int kPgUnroll = 4;  // 16-byte loads in flight per lane

__global__ void __launch_bounds__(kPgThreads) permute_gather_kernel(const int* __restrict__ idx, int n_assign,
                                                                    int k, const int* __restrict__ counts,
                                                                    const int* __restrict__ row_off, int* cursor,
                                                                    const __nv_bfloat16* __restrict__ x, long ldx,
                                                                    int D, int* __restrict__ src,
                                                                    int* __restrict__ dst,
                                                                    __nv_bfloat16* __restrict__ out, long ldo, int E,
                                                                    int P, unsigned int* status) {
  __shared__ int s_cnt[kMaxExpertsPerLane * 32];
  __shared__ int s_pos[kPgThreads];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int D8 = D >> 3;
  if ((int)blockIdx.x < E) {  // padding rows of expert blockIdx.x
    const int e = blockIdx.x;
    const int r0 = row_off[e] + counts[e], r1 = min(row_off[e + 1], P);
    for (int r = r0 + warp; r < r1; r += kPgThreads / 32) {
      uint4* o = reinterpret_cast<uint4*>(out + (size_t)r * ldo);
      for (int c = lane; c < D8; c += 32) o[c] = make_uint4(0, 0, 0, 0);
      if (lane == 0) src[r] = -1;
    }
    return;
  }
  const int tpb = kPgThreads / k;
  const int tok0 = (blockIdx.x - E) * tpb;
  const int a0 = tok0 * k;
  const int na = min(tpb * k, n_assign - a0);
  for (int e = t; e < E; e += kPgThreads) s_cnt[e] = 0;
  __syncthreads();
  int e = -1, rank = 0;
  if (t < na) {
    e = idx[a0 + t];
    if (e >= 0 && e < E) {
      rank = atomicAdd(&s_cnt[e], 1);
    } else {
      record_error(status, DSV3_ERR_BOUNDS);
      e = -1;
    }
  }
  __syncthreads();
  for (int j = t; j < E; j += kPgThreads) {
    const int c = s_cnt[j];
    s_cnt[j] = c ? atomicAdd(&cursor[j], c) : 0;  // this chunk's first row of expert j
  }
  __syncthreads();
  if (t < na) {
    int pos = -1;
    if (e >= 0) {
      pos = row_off[e] + s_cnt[e] + rank;
      if (pos >= row_off[e + 1] || pos >= P) {
        record_error(status, DSV3_ERR_BOUNDS);
        pos = -1;
      } else {
        src[pos] = a0 + t;
        dst[a0 + t] = pos;
      }
    }
    s_pos[t] = pos;
  }
  __syncthreads();
  const int ntok = na / k;
  for (int i = warp; i < ntok; i += kPgThreads / 32) {
    const uint4* sr = reinterpret_cast<const uint4*>(x + (size_t)(tok0 + i) * ldx);
    for (int c0 = lane; c0 < D8; c0 += 32 * kPgUnroll) {
      uint4 v[kPgUnroll];
#pragma unroll
      for (int u = 0; u < kPgUnroll; ++u)
        if (c0 + 32 * u < D8) v[u] = __ldg(sr + c0 + 32 * u);
      for (int j = 0; j < k; ++j) {
        const int pos = s_pos[i * k + j];
        if (pos < 0) continue;
        uint4* o = reinterpret_cast<uint4*>(out + (size_t)pos * ldo);
#pragma unroll
        for (int u = 0; u < kPgUnroll; ++u)
          if (c0 + 32 * u < D8) o[c0 + 32 * u] = v[u];
      }
    }
  }
}

__global__ void permute_scatter_kernel(const int* __restrict__ idx, int n_assign, const int* __restrict__ row_off,
                                       int* __restrict__ cursor, int* __restrict__ src, int* __restrict__ dst,
                                       int E, int P, unsigned int* status) {
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= n_assign) return;
  const int e = idx[a];
  DSV3_CHECK(e >= 0 && e < E, status, return)
  const int pos = row_off[e] + atomicAdd(&cursor[e], 1);
  DSV3_CHECK(pos < P, status, return)
  src[pos] = a;
  dst[a] = pos;
}

// One warp per sorted row: copy token row (a / k) of x, or zeros for padding.
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, long ldx, const int* __restrict__ src,
                                   int P, int k, int D, __nv_bfloat16* __restrict__ out, long ldo, int T,
                                   unsigned int* status) {
  const int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p >= P) return;
  const int a = src[p];
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)p * ldo);
  if (a < 0) {
    for (int c = lane; c < D / 8; c += 32) o[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  DSV3_CHECK(a / k < T, status, return)
  const uint4* s = reinterpret_cast<const uint4*>(x + (size_t)(a / k) * ldx);
  for (int c = lane; c < D / 8; c += 32) o[c] = s[c];
}

// out[t] (fp32) += sum_j w[t,j] * y[dst[t,j]]
__global__ void combine_fwd_kernel(const __nv_bfloat16* __restrict__ y, long ldy, const int* __restrict__ dst,
                                   const float* __restrict__ w, int T, int k, int D, float* __restrict__ out,
                                   long ldo, int P, unsigned int* status) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float* o = out + (size_t)t * ldo;
  for (int c = lane * 8; c < D; c += 256) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int row = dst[(size_t)t * k + j];
      DSV3_CHECK(row >= 0 && row < P, status, continue)
      const float wj = w[(size_t)t * k + j];
      const uint4 v = *reinterpret_cast<const uint4*>(y + (size_t)row * ldy + c);
      const uint16_t* h = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += wj * bf16_bits_to_float(h[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; i += 4) {
      float4 cur = *reinterpret_cast<float4*>(o + c + i);
      cur.x += acc[i];
      cur.y += acc[i + 1];
      cur.z += acc[i + 2];
      cur.w += acc[i + 3];
      *reinterpret_cast<float4*>(o + c + i) = cur;
    }
  }
}

// Row-parallel: dy[p] = w[a] * dout[a/k], dw[a] = <dout[a/k], y[p]>; padding rows -> 0.
__global__ void combine_bwd_kernel(const __nv_bfloat16* __restrict__ dout, long ldd, const __nv_bfloat16* __restrict__ y,
                                   long ldy, const int* __restrict__ src, const float* __restrict__ w, int P, int k,
                                   int D, __nv_bfloat16* __restrict__ dy, long lddy, float* __restrict__ dw) {
  const int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p >= P) return;
  const int a = src[p];
  uint4* o = reinterpret_cast<uint4*>(dy + (size_t)p * lddy);
  if (a < 0) {
    for (int c = lane; c < D / 8; c += 32) o[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const float wa = w[a];
  const uint4* g = reinterpret_cast<const uint4*>(dout + (size_t)(a / k) * ldd);
  const uint4* yr = reinterpret_cast<const uint4*>(y + (size_t)p * ldy);
  float dot = 0.f;
  for (int c = lane; c < D / 8; c += 32) {
    const uint4 gv = g[c], yv = yr[c];
    const uint16_t* gh = reinterpret_cast<const uint16_t*>(&gv);
    const uint16_t* yh = reinterpret_cast<const uint16_t*>(&yv);
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const float g0 = bf16_bits_to_float(gh[i]), g1 = bf16_bits_to_float(gh[i + 1]);
      dot += g0 * bf16_bits_to_float(yh[i]) + g1 * bf16_bits_to_float(yh[i + 1]);
      pk[i / 2] = pack_bf16x2(g0 * wa, g1 * wa);
    }
    o[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
  dot = warp_sum(dot);
  if (lane == 0) dw[a] = dot;
}

// dx[t] (fp32) += sum_j dxs[dst[t,j]]
__global__ void unpermute_bwd_kernel(const __nv_bfloat16* __restrict__ dxs, long ldx, const int* __restrict__ dst,
                                     int T, int k, int D, float* __restrict__ out, long ldo, int P,
                                     unsigned int* status) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float* o = out + (size_t)t * ldo;
  for (int c = lane * 8; c < D; c += 256) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int row = dst[(size_t)t * k + j];
      DSV3_CHECK(row >= 0 && row < P, status, continue)
      const uint4 v = *reinterpret_cast<const uint4*>(dxs + (size_t)row * ldx + c);
      const uint16_t* h = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += bf16_bits_to_float(h[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; i += 4) {
      float4 cur = *reinterpret_cast<float4*>(o + c + i);
      cur.x += acc[i];
      cur.y += acc[i + 1];
      cur.z += acc[i + 2];
      cur.w += acc[i + 3];
      *reinterpret_cast<float4*>(o + c + i) = cur;
    }
  }
}

// w_j = rs * s_j / S (S = sum of the k selected scores).  dL/ds_j =
// rs * (dw_j - sum_i dw_i w_i / rs) / S; dlogit_j = dL/ds_j * s_j (1 - s_j).
// Unselected experts get zero (the bias only selects; it carries no gradient).
__global__ void router_bwd_kernel(const float* __restrict__ dw, const float* __restrict__ s_sel,
                                  const int* __restrict__ idx, int T, int k, int Ep, float rs,
                                  __nv_bfloat16* __restrict__ dlogits, long ldd) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  __nv_bfloat16* row = dlogits + (size_t)t * ldd;
  for (int e = 0; e < Ep; ++e) row[e] = __float2bfloat16(0.f);
  float S = 0.f, dot = 0.f;
  for (int j = 0; j < k; ++j) {
    S += s_sel[(size_t)t * k + j];
    dot += dw[(size_t)t * k + j] * s_sel[(size_t)t * k + j];
  }
  S = fmaxf(S, 1e-10f);
  for (int j = 0; j < k; ++j) {
    const float s = s_sel[(size_t)t * k + j];
    const float ds = rs * (dw[(size_t)t * k + j] / S - dot / (S * S));
    row[idx[(size_t)t * k + j]] = __float2bfloat16(ds * s * (1.f - s));
  }
}

int nblk(long n, int per) { return (int)((n + per - 1) / per); }
const __nv_bfloat16* cbf(const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
__nv_bfloat16* bf(at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

}  // namespace

void router_topk(const at::Tensor& logits, const at::Tensor& bias, int64_t E, int64_t k, double route_scale,
                 at::Tensor& idx, at::Tensor& w, at::Tensor& s_sel, at::Tensor& counts) {
  const int T = logits.size(0);
  TORCH_CHECK(E <= 32 * kMaxExpertsPerLane && k <= 8 && k <= E, "router_topk: E <= 256, k <= 8");
  const at::cuda::CUDAGuard guard(logits.device());
  constexpr int kTpw = 8;   // tokens per warp: 64 per CTA of 8 warps
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = nblk(T, 8 * kTpw);
#define DSV3_ROUTER(NL_)                                                                                     \
  router_topk_kernel<NL_><<<grid, 256, 0, st>>>(logits.data_ptr<float>(), logits.stride(0),                \
      bias.data_ptr<float>(), T, E, k, (float)route_scale, idx.data_ptr<int>(), w.data_ptr<float>(),       \
      s_sel.data_ptr<float>(), counts.data_ptr<int>(), kTpw)
  if (E <= 32) DSV3_ROUTER(1);
  else if (E <= 64) DSV3_ROUTER(2);
  else if (E <= 128) DSV3_ROUTER(4);
  else DSV3_ROUTER(8);
#undef DSV3_ROUTER
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void permute_plan(const at::Tensor& counts, at::Tensor& row_off, at::Tensor& tile_group, at::Tensor& cursor,
                  at::Tensor& src, bool src_tail_only) {
  const int E = counts.numel();
  const at::cuda::CUDAGuard guard(counts.device());
  permute_plan_kernel<<<1, 1024, (E + 1) * sizeof(int), at::cuda::getCurrentCUDAStream()>>>(counts.data_ptr<int>(),
      E, row_off.data_ptr<int>(), tile_group.data_ptr<int>(), tile_group.numel(), cursor.data_ptr<int>(),
      src.data_ptr<int>(), src.numel(), src_tail_only ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void permute_scatter(const at::Tensor& idx, const at::Tensor& row_off, at::Tensor& cursor, at::Tensor& src,
                     at::Tensor& dst) {
  const int n = idx.numel();
  const at::cuda::CUDAGuard guard(idx.device());
  permute_scatter_kernel<<<nblk(n, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(idx.data_ptr<int>(), n,
      row_off.data_ptr<int>(), cursor.data_ptr<int>(), src.data_ptr<int>(), dst.data_ptr<int>(),
      (int)cursor.numel(), (int)src.numel(), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void permute_gather(const at::Tensor& idx, const at::Tensor& counts, const at::Tensor& row_off, at::Tensor& cursor,
                    const at::Tensor& x, at::Tensor& src, at::Tensor& dst, at::Tensor& out) {
  const int n = idx.numel(), E = counts.numel(), P = out.size(0), D = x.size(1);
  const int k = n / std::max<int64_t>(1, x.size(0));
  TORCH_CHECK(n == x.size(0) * k && dst.numel() == n && src.numel() >= P, "permute_gather: idx [T, k], src [P]");
  TORCH_CHECK(D % 8 == 0 && x.stride(0) % 8 == 0 && out.stride(0) % 8 == 0 && out.size(1) == D,
              "permute_gather: 16-byte rows");
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(k >= 1 && k <= kPgThreads && E <= kMaxExpertsPerLane * 32, "permute_gather: k <= 256, E <= 256");
  const int tpb = kPgThreads / k;
  const int grid = E + nblk(x.size(0), tpb);
  permute_gather_kernel<<<grid, kPgThreads, 0, at::cuda::getCurrentCUDAStream()>>>(idx.data_ptr<int>(), n, k,
      counts.data_ptr<int>(), row_off.data_ptr<int>(), cursor.data_ptr<int>(), cbf(x), x.stride(0), D,
      src.data_ptr<int>(), dst.data_ptr<int>(), bf(out), out.stride(0), E, P, status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gather_rows(const at::Tensor& x, const at::Tensor& src, int64_t k, at::Tensor& out) {
  const int P = out.size(0), D = x.size(1);
  TORCH_CHECK(D % 8 == 0 && x.stride(0) % 8 == 0 && out.stride(0) % 8 == 0, "gather_rows: 16-byte rows");
  const at::cuda::CUDAGuard guard(x.device());
  gather_rows_kernel<<<nblk(P, 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(cbf(x), x.stride(0),
      src.data_ptr<int>(), P, k, D, bf(out), out.stride(0), (int)x.size(0), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void combine_fwd(const at::Tensor& y, const at::Tensor& dst, const at::Tensor& w, at::Tensor& out) {
  const int T = dst.size(0), k = dst.size(1), D = y.size(1);
  TORCH_CHECK(D % 8 == 0 && out.scalar_type() == at::kFloat, "combine_fwd: D % 8, fp32 out");
  const at::cuda::CUDAGuard guard(y.device());
  combine_fwd_kernel<<<nblk(T, 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(cbf(y), y.stride(0),
      dst.data_ptr<int>(), w.data_ptr<float>(), T, k, D, out.data_ptr<float>(), out.stride(0), (int)y.size(0),
      status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void combine_bwd(const at::Tensor& dout, const at::Tensor& y, const at::Tensor& src, const at::Tensor& w, int64_t k,
                 at::Tensor& dy, at::Tensor& dw) {
  const int P = y.size(0), D = y.size(1);
  const at::cuda::CUDAGuard guard(y.device());
  combine_bwd_kernel<<<nblk(P, 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(cbf(dout), dout.stride(0), cbf(y),
      y.stride(0), src.data_ptr<int>(), w.data_ptr<float>(), P, k, D, bf(dy), dy.stride(0), dw.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void unpermute_bwd(const at::Tensor& dxs, const at::Tensor& dst, at::Tensor& out) {
  const int T = dst.size(0), k = dst.size(1), D = dxs.size(1);
  const at::cuda::CUDAGuard guard(dxs.device());
  unpermute_bwd_kernel<<<nblk(T, 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(cbf(dxs), dxs.stride(0),
      dst.data_ptr<int>(), T, k, D, out.data_ptr<float>(), out.stride(0), (int)dxs.size(0), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void router_bwd(const at::Tensor& dw, const at::Tensor& s_sel, const at::Tensor& idx, double route_scale,
                at::Tensor& dlogits) {
  const int T = idx.size(0), k = idx.size(1), Ep = dlogits.size(1);
  const at::cuda::CUDAGuard guard(dw.device());
  router_bwd_kernel<<<nblk(T, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(dw.data_ptr<float>(),
      s_sel.data_ptr<float>(), idx.data_ptr<int>(), T, k, Ep, (float)route_scale, bf(dlogits), dlogits.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_moe(pybind11::module_& m) {
  m.def("router_topk", &router_topk, "sigmoid + bias top-k routing with per-expert counts");
  m.def("permute_plan", &permute_plan, "256-row padded expert ranges and the tile->expert map",
        pybind11::arg("counts"), pybind11::arg("row_off"), pybind11::arg("tile_group"), pybind11::arg("cursor"),
        pybind11::arg("src"), pybind11::arg("src_tail_only") = false);
  m.def("permute_scatter", &permute_scatter, "destination row of each (token, slot)");
  m.def("permute_gather", &permute_gather,
        "expert-sorted slots of every (token, slot) fused with the copy of its row; padding rows zeroed");
  m.def("gather_rows", &gather_rows, "expert-sorted activation rows (padding rows zeroed)");
  m.def("combine_fwd", &combine_fwd, "weighted sum of expert outputs into the fp32 residual");
  m.def("combine_bwd", &combine_bwd, "gradients of the weighted combine");
  m.def("unpermute_bwd", &unpermute_bwd, "sum expert-input gradients back to tokens");
  m.def("router_bwd", &router_bwd, "router logit gradients");
}

}  // namespace dsv3
