// Memory-bound kernels of the training step: RMSNorm forward/backward (fp32
// residual stream in, bf16 GEMM operand out), decoupled RoPE, MLA Q/K/V
// packing for the attention kernels, token embedding, dtype casts and the
// cross-entropy finalisation.  One warp per row throughout; rows are
// processed with 16-byte vector accesses where the width allows.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "status.h"

namespace dsv3 {

namespace {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

constexpr int kMaxPerLane = 64;  // supports rows up to 2048 wide

// ------------------------------------------------------------------ RMSNorm
template <typename TIn>
__global__ void rmsnorm_fwd_kernel(const TIn* __restrict__ x, long ldx, const float* __restrict__ w, float eps,
                                   __nv_bfloat16* __restrict__ y, long ldy, float* __restrict__ rstd, int T, int D) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const TIn* xr = x + (size_t)row * ldx;
  float v[kMaxPerLane];
  float ss = 0.f;
  int n = 0;
  for (int c = lane; c < D; c += 32, ++n) {
    v[n] = ld_f(xr + c);
    ss += v[n] * v[n];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  __nv_bfloat16* yr = y + (size_t)row * ldy;
  n = 0;
  for (int c = lane; c < D; c += 32, ++n) yr[c] = __float2bfloat16(v[n] * r * w[c]);
  if (lane == 0 && rstd) rstd[row] = r;
}

// dx = r * (w*dy - xhat * mean(xhat * w * dy)),  xhat = x * r;  dw += sum_rows dy * xhat.
// dx is either accumulated into an fp32 buffer (residual stream gradient;
// then `dx_copy` optionally receives a bf16 copy of the updated sum) or
// stored as bf16.
template <typename TIn, typename TDy>
__global__ void rmsnorm_bwd_kernel(const TDy* __restrict__ dy, long lddy, const TIn* __restrict__ x, long ldx,
                                   const float* __restrict__ w, const float* __restrict__ rstd,
                                   float* __restrict__ dx_acc, long ldacc, __nv_bfloat16* __restrict__ dx_out,
                                   long ldout, __nv_bfloat16* __restrict__ dx_copy, long ldcopy,
                                   float* __restrict__ dw, int T, int D, int rows_per_block) {
  extern __shared__ float dw_s[];
  const int warps = blockDim.x >> 5;
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < D; c += blockDim.x) dw_s[c] = 0.f;
  __syncthreads();
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(T, r0 + rows_per_block);
  float dwl[kMaxPerLane];
  for (int i = 0; i < kMaxPerLane; ++i) dwl[i] = 0.f;
  for (int row = r0 + wid; row < r1; row += warps) {
    const float r = rstd[row];
    float xh[kMaxPerLane], g[kMaxPerLane];
    float dot = 0.f;
    int n = 0;
    for (int c = lane; c < D; c += 32, ++n) {
      xh[n] = ld_f(x + (size_t)row * ldx + c) * r;
      const float gy = ld_f(dy + (size_t)row * lddy + c);
      g[n] = gy * w[c];
      dot += xh[n] * g[n];
      dwl[n] += gy * xh[n];
    }
    dot = warp_sum(dot) / D;
    n = 0;
    for (int c = lane; c < D; c += 32, ++n) {
      const float d = r * (g[n] - xh[n] * dot);
      if (dx_acc) {
        float* p = dx_acc + (size_t)row * ldacc + c;
        const float s = *p + d;
        *p = s;
        if (dx_copy) dx_copy[(size_t)row * ldcopy + c] = __float2bfloat16(s);
      } else {
        dx_out[(size_t)row * ldout + c] = __float2bfloat16(d);
      }
    }
  }
  int n = 0;
  for (int c = lane; c < D; c += 32, ++n) atomicAdd(&dw_s[c], dwl[n]);
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(&dw[c], dw_s[c]);
}

// --------------------------------------------------------------------- RoPE
// Rotate pairs (x[2i], x[2i+1]) of a [T, H, ...] bf16 tensor in place, at
// column offset `off` of each head.  Position of token t is pos[t] when given,
// else (t % seqlen) + start.  `inverse` rotates by -theta (backward pass).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, long ld_tok, long ld_head, int off, int T, int H,
                            int half, const float* __restrict__ cosv, const float* __restrict__ sinv,
                            const int* __restrict__ pos, int seqlen, int start, int inverse) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long total = (long)T * H * half;
  if (idx >= total) return;
  const int i = idx % half;
  const int h = (idx / half) % H;
  const int t = idx / ((long)half * H);
  const int p = pos ? pos[t] : (t % seqlen) + start;
  const float c = cosv[(size_t)p * half + i];
  const float s = inverse ? -sinv[(size_t)p * half + i] : sinv[(size_t)p * half + i];
  __nv_bfloat16* e = x + (size_t)t * ld_tok + (size_t)h * ld_head + off + 2 * i;
  const float a = __bfloat162float(e[0]), b = __bfloat162float(e[1]);
  e[0] = __float2bfloat16(a * c - b * s);
  e[1] = __float2bfloat16(a * s + b * c);
}

// ------------------------------------------------------------ MLA packing
// Build the attention operands of the materialised formulation from the
// projection outputs of T = B*S tokens:
//   q   [T, H, dn + dr]      (q_nope | q_pe, q_pe not yet rotated)
//   kvb [T, H, dn + dv]      (k_nope | v)
//   kpe [T, dr] (stride ldk) (shared RoPE key, not yet rotated)
// into Q, K [B, H, S, DP] (DP >= dn + dr, zero padded) and V [B, H, S, dv],
// rotating q_pe / k_pe on the way (RoPE in fp32, rounded to bf16 once).
__global__ void mla_pack_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kvb,
                                const __nv_bfloat16* __restrict__ kpe, long ldk, __nv_bfloat16* __restrict__ Q,
                                __nv_bfloat16* __restrict__ K, __nv_bfloat16* __restrict__ V, int B, int S, int H,
                                int dn, int dr, int dv, int DP, const float* __restrict__ cosv,
                                const float* __restrict__ sinv, int start) {
  const int t = blockIdx.x;       // token
  const int h = blockIdx.y;       // head
  const int b = t / S, s = t % S;
  const int p = s + start;
  const size_t o_qk = (((size_t)b * H + h) * S + s) * DP;
  const size_t o_v = (((size_t)b * H + h) * S + s) * dv;
  const __nv_bfloat16* qs = q + ((size_t)t * H + h) * (dn + dr);
  const __nv_bfloat16* ks = kvb + ((size_t)t * H + h) * (dn + dv);
  for (int c = threadIdx.x; c < DP; c += blockDim.x) {
    __nv_bfloat16 qv, kv;
    if (c < dn) {
      qv = qs[c];
      kv = ks[c];
    } else if (c < dn + dr) {
      const int j = c - dn, i = j >> 1;
      const float cs = cosv[(size_t)p * (dr / 2) + i], sn = sinv[(size_t)p * (dr / 2) + i];
      const float qa = __bfloat162float(qs[dn + 2 * i]), qb = __bfloat162float(qs[dn + 2 * i + 1]);
      const float ka = __bfloat162float(kpe[(size_t)t * ldk + 2 * i]), kb = __bfloat162float(kpe[(size_t)t * ldk + 2 * i + 1]);
      qv = __float2bfloat16((j & 1) ? qa * sn + qb * cs : qa * cs - qb * sn);
      kv = __float2bfloat16((j & 1) ? ka * sn + kb * cs : ka * cs - kb * sn);
    } else {
      qv = __float2bfloat16(0.f);
      kv = qv;
    }
    Q[o_qk + c] = qv;
    K[o_qk + c] = kv;
  }
  for (int c = threadIdx.x; c < dv; c += blockDim.x) V[o_v + c] = ks[dn + c];
}

// Inverse of the packing for the gradients.  dQ, dK are fp32 [B,H,S,DP]; dV
// bf16 or fp32 [B,H,S,dv].  Writes dq [T,H,dn+dr] and dkvb [T,H,dn+dv] (bf16)
// and dkpe [T, dr] (bf16, summed over heads) with the RoPE rotation undone.
template <typename TV>
__global__ void mla_unpack_kernel(const float* __restrict__ dQ, const float* __restrict__ dK,
                                  const TV* __restrict__ dV, __nv_bfloat16* __restrict__ dq,
                                  __nv_bfloat16* __restrict__ dkvb, __nv_bfloat16* __restrict__ dkpe, long ldk, int B,
                                  int S, int H, int dn, int dr, int dv, int DP, const float* __restrict__ cosv,
                                  const float* __restrict__ sinv, int start) {
  const int t = blockIdx.x;
  const int b = t / S, s = t % S;
  const int p = s + start;
  extern __shared__ float kpe_acc[];  // [dr]
  for (int c = threadIdx.x; c < dr; c += blockDim.x) kpe_acc[c] = 0.f;
  __syncthreads();
  for (int h = 0; h < H; ++h) {
    const size_t o_qk = (((size_t)b * H + h) * S + s) * DP;
    const size_t o_v = (((size_t)b * H + h) * S + s) * dv;
    __nv_bfloat16* dqs = dq + ((size_t)t * H + h) * (dn + dr);
    __nv_bfloat16* dks = dkvb + ((size_t)t * H + h) * (dn + dv);
    for (int c = threadIdx.x; c < dn; c += blockDim.x) {
      dqs[c] = __float2bfloat16(dQ[o_qk + c]);
      dks[c] = __float2bfloat16(dK[o_qk + c]);
    }
    for (int i = threadIdx.x; i < dr / 2; i += blockDim.x) {
      const float cs = cosv[(size_t)p * (dr / 2) + i], sn = sinv[(size_t)p * (dr / 2) + i];
      const float qa = dQ[o_qk + dn + 2 * i], qb = dQ[o_qk + dn + 2 * i + 1];
      dqs[dn + 2 * i] = __float2bfloat16(qa * cs + qb * sn);
      dqs[dn + 2 * i + 1] = __float2bfloat16(-qa * sn + qb * cs);
      const float ka = dK[o_qk + dn + 2 * i], kb = dK[o_qk + dn + 2 * i + 1];
      kpe_acc[2 * i] += ka * cs + kb * sn;
      kpe_acc[2 * i + 1] += -ka * sn + kb * cs;
    }
    for (int c = threadIdx.x; c < dv; c += blockDim.x) dks[dn + c] = __float2bfloat16(ld_f(dV + o_v + c));
  }
  __syncthreads();
  for (int c = threadIdx.x; c < dr; c += blockDim.x) dkpe[(size_t)t * ldk + c] = __float2bfloat16(kpe_acc[c]);
}

// ---------------------------------------------------------------- embedding
// Token ids come from user data: an id outside [0, V) is reported through the
// status word (DSV3_ERR_BOUNDS) and its row is zero / skipped, never read.
__global__ void embedding_fwd_kernel(const long* __restrict__ tok, const float* __restrict__ w,
                                     float* __restrict__ out, int T, int D, long V, unsigned int* status) {
  const int row = blockIdx.x;
  const long id = tok[row];
  float4* dst = reinterpret_cast<float4*>(out + (size_t)row * D);
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) record_error(status, DSV3_ERR_BOUNDS);
    for (int c = threadIdx.x; c < D / 4; c += blockDim.x) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  const float4* src = reinterpret_cast<const float4*>(w + (size_t)id * D);
  for (int c = threadIdx.x; c < D / 4; c += blockDim.x) dst[c] = src[c];
}

__global__ void embedding_bwd_kernel(const long* __restrict__ tok, const float* __restrict__ g,
                                     float* __restrict__ dw, int T, int D, long V, unsigned int* status) {
  const int row = blockIdx.x;
  const long id = tok[row];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) record_error(status, DSV3_ERR_BOUNDS);
    return;
  }
  float* dst = dw + (size_t)id * D;
  const float* src = g + (size_t)row * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(dst + c, src[c]);
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ a, __nv_bfloat16* __restrict__ b, long n) {
  const long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(a + i);
    uint2 o;
    o.x = pack_bf16x2(v.x, v.y);
    o.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(b + i) = o;
  } else {
    for (long j = i; j < n; ++j) b[j] = __float2bfloat16(a[j]);
  }
}

// ---------------------------------------------------------- cross-entropy
// Combine the per-tile (max, sum-exp) partials into lse and per-row loss.
__global__ void ce_rows_kernel(const float* __restrict__ pmax, const float* __restrict__ psum,
                               const float* __restrict__ tgt_logit, const long* __restrict__ tgt, int T, int nt,
                               float* __restrict__ lse, float* __restrict__ loss) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  float m = -INFINITY;
  for (int i = lane; i < nt; i += 32) m = fmaxf(m, pmax[(size_t)row * nt + i]);
  m = warp_max(m);
  float s = 0.f;
  for (int i = lane; i < nt; i += 32) {
    const float pm = pmax[(size_t)row * nt + i];
    if (pm != -INFINITY) s += psum[(size_t)row * nt + i] * __expf(pm - m);
  }
  s = warp_sum(s);
  if (lane == 0) {
    const float l = m + logf(s);
    lse[row] = l;
    loss[row] = tgt[row] >= 0 ? l - tgt_logit[row] : 0.f;
  }
}

// Deterministic per-segment mean of the row losses (rows [seg_start[i],
// seg_start[i+1]) with targets != -100).  Writes loss[i] = mean and the
// backward row scale  weight[i] * grad_scale / count_i  (0 for ignored rows).
// Segment means of the row losses (main, MTP depths) in two grid-wide
// passes: ce_seg_sum_kernel adds every row block's per-segment (sum, count)
// into acc[nseg][2]; ce_seg_scale_kernel writes each row's gradient scale
// (segment weight * grad_scale / count for rows with a target) and block 0
// the segment losses.
__global__ void ce_seg_sum_kernel(const float* __restrict__ loss_rows, const long* __restrict__ tgt,
                                  const int* __restrict__ seg_start, int nseg, int rows,
                                  float* __restrict__ acc) {
  __shared__ float ssum[32], scnt[32];
  const int r0 = blockIdx.x * blockDim.x * 4;
  const int r1 = min(rows, r0 + (int)blockDim.x * 4);
  for (int sgi = 0; sgi < nseg; ++sgi) {
    const int a = max(seg_start[sgi], r0), b = min(seg_start[sgi + 1], r1);
    if (a >= b) continue;                       // uniform across the block
    float sum = 0.f, cnt = 0.f;
    for (int r = a + threadIdx.x; r < b; r += blockDim.x)
      if (tgt[r] >= 0) {
        sum += loss_rows[r];
        cnt += 1.f;
      }
    sum = warp_sum(sum);
    cnt = warp_sum(cnt);
    if ((threadIdx.x & 31) == 0) {
      ssum[threadIdx.x >> 5] = sum;
      scnt[threadIdx.x >> 5] = cnt;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      float s2 = threadIdx.x < (blockDim.x >> 5) ? ssum[threadIdx.x] : 0.f;
      float c2 = threadIdx.x < (blockDim.x >> 5) ? scnt[threadIdx.x] : 0.f;
      s2 = warp_sum(s2);
      c2 = warp_sum(c2);
      if (threadIdx.x == 0) {
        atomicAdd(&acc[2 * sgi], s2);
        atomicAdd(&acc[2 * sgi + 1], c2);
      }
    }
    __syncthreads();
  }
}

__global__ void ce_seg_scale_kernel(const long* __restrict__ tgt, const int* __restrict__ seg_start,
                                    const float* __restrict__ seg_weight, int nseg, int rows, float grad_scale,
                                    const float* __restrict__ acc, float* __restrict__ loss_out,
                                    float* __restrict__ row_scale) {
  if (blockIdx.x == 0 && threadIdx.x < nseg) {
    const float c = acc[2 * threadIdx.x + 1];
    loss_out[threadIdx.x] = c > 0.f ? acc[2 * threadIdx.x] / c : 0.f;
  }
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    int sgi = 0;
    while (sgi + 1 < nseg && r >= seg_start[sgi + 1]) ++sgi;
    const float c = acc[2 * sgi + 1];
    row_scale[r] = (tgt[r] >= 0 && c > 0.f) ? seg_weight[sgi] * grad_scale / c : 0.f;
  }
}

// ---------------------------------------------------- generic head packing
// dst[b*H + h, s, 0:hd] = src[(b*S + s), col0 + h*hd + (0:hd)], zero-padded to DP.
__global__ void heads_pack_kernel(const __nv_bfloat16* __restrict__ src, long ld, int col0, int H, int hd, int S,
                                  int DP, __nv_bfloat16* __restrict__ dst) {
  const int t = blockIdx.x, h = blockIdx.y;
  const int b = t / S, s = t % S;
  __nv_bfloat16* d = dst + (((size_t)b * H + h) * S + s) * DP;
  const __nv_bfloat16* r = src + (size_t)t * ld + col0 + (size_t)h * hd;
  for (int c = threadIdx.x; c < DP; c += blockDim.x) d[c] = c < hd ? r[c] : __float2bfloat16(0.f);
}

// Inverse for gradients: dst[(b*S + s), col0 + h*hd + c] = bf16(src[b*H + h, s, c]) (c < hd).
__global__ void heads_unpack_kernel(const float* __restrict__ src, int H, int hd, int S, int DP,
                                    __nv_bfloat16* __restrict__ dst, long ld, int col0) {
  const int t = blockIdx.x, h = blockIdx.y;
  const int b = t / S, s = t % S;
  const float* r = src + (((size_t)b * H + h) * S + s) * DP;
  __nv_bfloat16* d = dst + (size_t)t * ld + col0 + (size_t)h * hd;
  for (int c = threadIdx.x; c < hd; c += blockDim.x) d[c] = __float2bfloat16(r[c]);
}

// 16-byte versions: one thread per 8-element chunk; consecutive threads take
// consecutive chunks of a head row, then consecutive tokens of the same head,
// so a warp reads 128-byte row pieces and writes contiguous [S, DP] rows.
// Need hd, DP, ld and col0 multiples of 8 and 16-byte aligned bases.
__global__ void heads_pack_v(const __nv_bfloat16* __restrict__ src, long ld, int col0, int H, int hd, int S, int DP,
                             __nv_bfloat16* __restrict__ dst, long T) {
  const int chunks = DP / 8;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * H * chunks) return;
  const int j = (int)(idx % chunks);
  const long t = (idx / chunks) % T;
  const int h = (int)(idx / (chunks * T));
  const long b = t / S, s = t % S;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (8 * j < hd) v = *reinterpret_cast<const uint4*>(src + t * ld + col0 + (size_t)h * hd + 8 * j);
  *reinterpret_cast<uint4*>(dst + ((b * H + h) * S + s) * DP + 8 * j) = v;
}

__global__ void heads_unpack_v(const float* __restrict__ src, int H, int hd, int S, int DP,
                               __nv_bfloat16* __restrict__ dst, long ld, int col0, long T) {
  const int chunks = hd / 8;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * H * chunks) return;
  const int j = (int)(idx % chunks);
  const long t = (idx / chunks) % T;
  const int h = (int)(idx / (chunks * T));
  const long b = t / S, s = t % S;
  const float4* r = reinterpret_cast<const float4*>(src + ((b * H + h) * S + s) * DP + 8 * j);
  const float4 x = r[0], y = r[1];
  *reinterpret_cast<uint4*>(dst + t * ld + col0 + (size_t)h * hd + 8 * j) =
      make_uint4(pack_bf16x2(x.x, x.y), pack_bf16x2(x.z, x.w), pack_bf16x2(y.x, y.y), pack_bf16x2(y.z, y.w));
}

// ---------------------------------------------- RMSNorm, width-specialised
// PAIRS = D / 64: each lane owns PAIRS column pairs (2 * (lane + 32 i)), so a
// warp reads 256 contiguous bytes of fp32 (128 of bf16) per step.
template <typename T>
__device__ __forceinline__ float2 ld2(const T* p);
template <>
__device__ __forceinline__ float2 ld2<float>(const float* p) { return *reinterpret_cast<const float2*>(p); }
template <>
__device__ __forceinline__ float2 ld2<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

template <typename TIn, int PAIRS>
__global__ void rmsnorm_fwd_v(const TIn* __restrict__ x, long ldx, const float* __restrict__ w, float eps,
                              __nv_bfloat16* __restrict__ y, long ldy, float* __restrict__ rstd, int T) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  constexpr int D = 64 * PAIRS;
  float2 v[PAIRS];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PAIRS; ++i) {
    v[i] = ld2(x + (size_t)row * ldx + 2 * (lane + 32 * i));
    ss += v[i].x * v[i].x + v[i].y * v[i].y;
  }
  const float r = rsqrtf(warp_sum(ss) / D + eps);
#pragma unroll
  for (int i = 0; i < PAIRS; ++i) {
    const int c = 2 * (lane + 32 * i);
    const float2 wv = *reinterpret_cast<const float2*>(w + c);
    *reinterpret_cast<uint32_t*>(y + (size_t)row * ldy + c) = pack_bf16x2(v[i].x * r * wv.x, v[i].y * r * wv.y);
  }
  if (lane == 0 && rstd) rstd[row] = r;
}

template <typename TIn, typename TDy, int PAIRS>
__global__ void rmsnorm_bwd_v(const TDy* __restrict__ dy, long lddy, const TIn* __restrict__ x, long ldx,
                              const float* __restrict__ w, const float* __restrict__ rstd, float* __restrict__ dx_acc,
                              long ldacc, __nv_bfloat16* __restrict__ dx_out, long ldout,
                              __nv_bfloat16* __restrict__ dx_copy, long ldcopy, float* __restrict__ dw, int T,
                              int rows_per_block) {
  constexpr int D = 64 * PAIRS;
  __shared__ float dw_s[D];
  const int warps = blockDim.x >> 5;
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < D; c += blockDim.x) dw_s[c] = 0.f;
  __syncthreads();
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(T, r0 + rows_per_block);
  float2 dwl[PAIRS], wv[PAIRS];
#pragma unroll
  for (int i = 0; i < PAIRS; ++i) {
    dwl[i] = make_float2(0.f, 0.f);
    wv[i] = *reinterpret_cast<const float2*>(w + 2 * (lane + 32 * i));
  }
  for (int row = r0 + wid; row < r1; row += warps) {
    const float r = rstd[row];
    float2 xh[PAIRS], g[PAIRS], av[PAIRS];
    float dot = 0.f;
    if (dx_acc) {
      // the accumulator is read with x and dy: one memory round trip per row
#pragma unroll
      for (int i = 0; i < PAIRS; ++i)
        av[i] = *reinterpret_cast<const float2*>(dx_acc + (size_t)row * ldacc + 2 * (lane + 32 * i));
    }
#pragma unroll
    for (int i = 0; i < PAIRS; ++i) {
      const int c = 2 * (lane + 32 * i);
      const float2 xv = ld2(x + (size_t)row * ldx + c);
      const float2 gy = ld2(dy + (size_t)row * lddy + c);
      xh[i] = make_float2(xv.x * r, xv.y * r);
      g[i] = make_float2(gy.x * wv[i].x, gy.y * wv[i].y);
      dot += xh[i].x * g[i].x + xh[i].y * g[i].y;
      dwl[i].x += gy.x * xh[i].x;
      dwl[i].y += gy.y * xh[i].y;
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int i = 0; i < PAIRS; ++i) {
      const int c = 2 * (lane + 32 * i);
      const float d0 = r * (g[i].x - xh[i].x * dot), d1 = r * (g[i].y - xh[i].y * dot);
      if (dx_acc) {
        float2* p = reinterpret_cast<float2*>(dx_acc + (size_t)row * ldacc + c);
        float2 sv = av[i];
        sv.x += d0;
        sv.y += d1;
        *p = sv;
        if (dx_copy) *reinterpret_cast<uint32_t*>(dx_copy + (size_t)row * ldcopy + c) = pack_bf16x2(sv.x, sv.y);
      } else {
        *reinterpret_cast<uint32_t*>(dx_out + (size_t)row * ldout + c) = pack_bf16x2(d0, d1);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PAIRS; ++i) {
    atomicAdd(&dw_s[2 * (lane + 32 * i)], dwl[i].x);
    atomicAdd(&dw_s[2 * (lane + 32 * i) + 1], dwl[i].y);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(&dw[c], dw_s[c]);
}

// ------------------------------------- MoE input gradient + RMSNorm backward
// The gradient at a MoE layer's normalised input has three parts: the shared
// experts' (fp32, optional), the routed experts' rows un-permuted from the
// expert-sorted buffer (bf16, one row per (token, slot)), and the router
// logits' (dlog[t, :E] @ W_gate, K = E).  One warp per token row sums them in
// registers and runs the RMSNorm backward on the sum:
//   g = dsh[t] + sum_j dxs[dst[t, j]] + sum_e dlog[t, e] W_gate[e]
//   dres[t] += rstd (g w - x_hat <x_hat, g w> / D),  dres_b[t] = bf16(dres[t]),
//   dw += g * x_hat.
// Replaces unpermute_bwd, the router data-gradient GEMM and rmsnorm_bwd (three
// fp32 round trips of the [T, D] gradient).  W_gate (as fp32) and the norm
// weight sit in shared memory; lanes broadcast the row's router-logit
// gradients by shuffle.  All of a row's loads are issued before the first use.
constexpr int kMoeNormMaxK = 8;   // routed slots per token the fused kernel unrolls

template <int PAIRS>
__global__ void __launch_bounds__(256, 1) moe_norm_bwd_v(
    const __nv_bfloat16* __restrict__ dxs, long ldxs, const int* __restrict__ dst, int k, int P,
    const float* __restrict__ dsh, long ldsh, const __nv_bfloat16* __restrict__ dlog, long ldl,
    const __nv_bfloat16* __restrict__ wg, int E, const float* __restrict__ x, long ldx, const float* __restrict__ w,
    const float* __restrict__ rstd, float* __restrict__ dres, long ldr, __nv_bfloat16* __restrict__ dres_b, long ldb,
    float* __restrict__ dw, int T, int rows_per_block, unsigned int* status) {
  constexpr int D = 64 * PAIRS;
  extern __shared__ __align__(16) uint8_t moe_norm_smem[];
  float* dw_s = reinterpret_cast<float*>(moe_norm_smem);                                           // [D]
  float* w_s = dw_s + D;                                                                            // [D]
  float2* wg_s = reinterpret_cast<float2*>(moe_norm_smem + 2 * D * sizeof(float));                  // [E][D / 2]
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    dw_s[c] = 0.f;
    w_s[c] = w[c];
  }
  for (int i = threadIdx.x; i < E * (D / 2); i += blockDim.x)
    wg_s[i] = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(wg)[i]);
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(T, r0 + rows_per_block);
  float2 dwl[PAIRS];
#pragma unroll
  for (int i = 0; i < PAIRS; ++i) dwl[i] = make_float2(0.f, 0.f);
  for (int row = r0 + wid; row < r1; row += warps) {
    // every load of the row is issued before any is consumed: the k slot
    // indices (lane j holds slot j), the router gradients (lane e holds e),
    // the shared part, x, the accumulated residual gradient, then the k rows
    const int myp = (k > 0 && lane < k) ? dst[(size_t)row * k + lane] : 0;
    const float al0 = lane < E ? __bfloat162float(dlog[(size_t)row * ldl + lane]) : 0.f;
    float2 g[PAIRS], xv[PAIRS], av[PAIRS];
#pragma unroll
    for (int i = 0; i < PAIRS; ++i) {
      const int c = 2 * (lane + 32 * i);
      g[i] = dsh ? *reinterpret_cast<const float2*>(dsh + (size_t)row * ldsh + c) : make_float2(0.f, 0.f);
      xv[i] = *reinterpret_cast<const float2*>(x + (size_t)row * ldx + c);
      av[i] = *reinterpret_cast<const float2*>(dres + (size_t)row * ldr + c);
    }
#pragma unroll
    for (int j = 0; j < kMoeNormMaxK; ++j) {
      if (j < k) {
        const int p = __shfl_sync(0xffffffffu, myp, j);
        if (p >= 0 && p < P) {
#pragma unroll
          for (int i = 0; i < PAIRS; ++i) {
            const float2 v = ld2(dxs + (size_t)p * ldxs + 2 * (lane + 32 * i));
            g[i].x += v.x;
            g[i].y += v.y;
          }
        } else if (lane == 0) {
          record_error(status, DSV3_ERR_BOUNDS);
        }
      }
    }
    for (int e0 = 0; e0 < E; e0 += 32) {
      const float al = e0 == 0 ? al0 : (e0 + lane < E ? __bfloat162float(dlog[(size_t)row * ldl + e0 + lane]) : 0.f);
      const int ne = min(32, E - e0);
      for (int e = 0; e < ne; ++e) {
        const float a = __shfl_sync(0xffffffffu, al, e);
        const float2* wr = wg_s + (size_t)(e0 + e) * (D / 2);
#pragma unroll
        for (int i = 0; i < PAIRS; ++i) {
          const float2 f = wr[lane + 32 * i];
          g[i].x = fmaf(a, f.x, g[i].x);
          g[i].y = fmaf(a, f.y, g[i].y);
        }
      }
    }
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < PAIRS; ++i) {
      xv[i].x *= r;   // x_hat
      xv[i].y *= r;
      const float2 wv = *reinterpret_cast<const float2*>(w_s + 2 * (lane + 32 * i));
      dot += xv[i].x * g[i].x * wv.x + xv[i].y * g[i].y * wv.y;
      dwl[i].x += g[i].x * xv[i].x;
      dwl[i].y += g[i].y * xv[i].y;
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int i = 0; i < PAIRS; ++i) {
      const int c = 2 * (lane + 32 * i);
      const float2 wv = *reinterpret_cast<const float2*>(w_s + c);
      float2 sv = av[i];
      sv.x += r * (g[i].x * wv.x - xv[i].x * dot);
      sv.y += r * (g[i].y * wv.y - xv[i].y * dot);
      *reinterpret_cast<float2*>(dres + (size_t)row * ldr + c) = sv;
      *reinterpret_cast<uint32_t*>(dres_b + (size_t)row * ldb + c) = pack_bf16x2(sv.x, sv.y);
    }
  }
#pragma unroll
  for (int i = 0; i < PAIRS; ++i) {
    atomicAdd(&dw_s[2 * (lane + 32 * i)], dwl[i].x);
    atomicAdd(&dw_s[2 * (lane + 32 * i) + 1], dwl[i].y);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(&dw[c], dw_s[c]);
}

// -------------------------------------------------- vectorised MLA packing
// One block per token; each thread moves one 8-element (16-byte) chunk of Q,
// K or V for one head.  Requires dn, dr, dv, DP to be multiples of 8.
__global__ void mla_pack_v(const __nv_bfloat16* __restrict__ q, long ldq, const __nv_bfloat16* __restrict__ kvb,
                           const __nv_bfloat16* __restrict__ kpe, long ldk, __nv_bfloat16* __restrict__ Q,
                           __nv_bfloat16* __restrict__ K, __nv_bfloat16* __restrict__ V, int S, int H, int dn, int dr,
                           int dv, int DP, const float* __restrict__ cosv, const float* __restrict__ sinv, int start) {
  const int t = blockIdx.x, b = t / S, s = t % S, p = s + start;
  const int qk_chunks = DP / 8, v_chunks = dv / 8;
  const int per_head = qk_chunks + v_chunks;
  for (int idx = threadIdx.x; idx < H * per_head; idx += blockDim.x) {
    const int h = idx / per_head, j = idx % per_head;
    if (j >= qk_chunks) {
      const int c = (j - qk_chunks) * 8;
      *reinterpret_cast<uint4*>(V + (((size_t)b * H + h) * S + s) * dv + c) =
          *reinterpret_cast<const uint4*>(kvb + ((size_t)t * H + h) * (dn + dv) + dn + c);
      continue;
    }
    const int c = j * 8;
    const size_t o = (((size_t)b * H + h) * S + s) * DP + c;
    uint4 qv, kv;
    if (c + 8 <= dn) {
      qv = *reinterpret_cast<const uint4*>(q + (size_t)t * ldq + (size_t)h * (dn + dr) + c);
      kv = *reinterpret_cast<const uint4*>(kvb + ((size_t)t * H + h) * (dn + dv) + c);
    } else if (c >= dn + dr) {
      qv = make_uint4(0, 0, 0, 0);
      kv = qv;
    } else {
      const uint4 qr = *reinterpret_cast<const uint4*>(q + (size_t)t * ldq + (size_t)h * (dn + dr) + c);
      const uint4 kr = *reinterpret_cast<const uint4*>(kpe + (size_t)t * ldk + (c - dn));
      const __nv_bfloat162* qh = reinterpret_cast<const __nv_bfloat162*>(&qr);
      const __nv_bfloat162* kh = reinterpret_cast<const __nv_bfloat162*>(&kr);
      uint32_t qo[4], ko[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = (c - dn) / 2 + e;
        const float cs = cosv[(size_t)p * (dr / 2) + i], sn = sinv[(size_t)p * (dr / 2) + i];
        const float2 a = __bfloat1622float2(qh[e]), k2 = __bfloat1622float2(kh[e]);
        qo[e] = pack_bf16x2(a.x * cs - a.y * sn, a.x * sn + a.y * cs);
        ko[e] = pack_bf16x2(k2.x * cs - k2.y * sn, k2.x * sn + k2.y * cs);
      }
      qv = make_uint4(qo[0], qo[1], qo[2], qo[3]);
      kv = make_uint4(ko[0], ko[1], ko[2], ko[3]);
    }
    *reinterpret_cast<uint4*>(Q + o) = qv;
    *reinterpret_cast<uint4*>(K + o) = kv;
  }
}

// Attention gradients back to the projection outputs (inverse of mla_pack),
// one CTA per (batch row, TB consecutive positions).  For each head the TB
// positions' rows of dQ / dK / dV are adjacent in memory, so consecutive
// threads read consecutive 32-byte chunks: nope / v chunks go to dq and dkvb
// as bf16; each decoupled-RoPE chunk of a position is handled by one thread
// that walks the heads, applies the inverse rotation to dq and sums the
// rotated dK over heads into the shared k_pe gradient in registers.
template <int TB>
__global__ void __launch_bounds__(256) mla_unpack_blk(const float* __restrict__ dQ, const float* __restrict__ dK,
                                                      const float* __restrict__ dV, __nv_bfloat16* __restrict__ dq,
                                                      long lddq, __nv_bfloat16* __restrict__ dkvb,
                                                      __nv_bfloat16* __restrict__ dkpe, long ldk, int S, int H, int dn,
                                                      int dr, int dv, int DP, const float* __restrict__ cosv,
                                                      const float* __restrict__ sinv, int start) {
  const int b = blockIdx.y, s0 = blockIdx.x * TB;
  const int nn = dn / 8, nv = dv / 8, nr = dr / 8, per = nn + nv;
  const int main_items = H * TB * per, rope_items = TB * nr;
  for (int idx = threadIdx.x; idx < main_items + rope_items; idx += blockDim.x) {
    if (idx < main_items) {
      const int h = idx / (TB * per), rem = idx - h * (TB * per), i = rem / per, j = rem - i * per;
      const int s = s0 + i;
      if (s >= S) continue;
      const size_t t = (size_t)b * S + s, row = ((size_t)b * H + h) * S + s;
      if (j < nn) {
        const int c = j * 8;
        const float4* q4 = reinterpret_cast<const float4*>(dQ + row * DP + c);
        const float4* k4 = reinterpret_cast<const float4*>(dK + row * DP + c);
        const float4 qa = q4[0], qb = q4[1], ka = k4[0], kb = k4[1];
        *reinterpret_cast<uint4*>(dq + t * lddq + (size_t)h * (dn + dr) + c) =
            make_uint4(pack_bf16x2(qa.x, qa.y), pack_bf16x2(qa.z, qa.w), pack_bf16x2(qb.x, qb.y), pack_bf16x2(qb.z, qb.w));
        *reinterpret_cast<uint4*>(dkvb + (t * H + h) * (dn + dv) + c) =
            make_uint4(pack_bf16x2(ka.x, ka.y), pack_bf16x2(ka.z, ka.w), pack_bf16x2(kb.x, kb.y), pack_bf16x2(kb.z, kb.w));
      } else {
        const int c = (j - nn) * 8;
        const float4* v4 = reinterpret_cast<const float4*>(dV + row * dv + c);
        const float4 a = v4[0], bb = v4[1];
        *reinterpret_cast<uint4*>(dkvb + (t * H + h) * (dn + dv) + dn + c) =
            make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(bb.x, bb.y), pack_bf16x2(bb.z, bb.w));
      }
    } else {
      const int r = idx - main_items, i = r / nr, k = r - i * nr;
      const int s = s0 + i;
      if (s >= S) continue;
      const size_t t = (size_t)b * S + s;
      const int p = s + start, c = dn + k * 8;
      float cs[4], sn[4], acc[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        cs[e] = cosv[(size_t)p * (dr / 2) + k * 4 + e];
        sn[e] = sinv[(size_t)p * (dr / 2) + k * 4 + e];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      for (int h = 0; h < H; ++h) {
        const size_t row = ((size_t)b * H + h) * S + s;
        float qv[8], kv[8];
        *reinterpret_cast<float4*>(qv) = reinterpret_cast<const float4*>(dQ + row * DP + c)[0];
        *reinterpret_cast<float4*>(qv + 4) = reinterpret_cast<const float4*>(dQ + row * DP + c)[1];
        *reinterpret_cast<float4*>(kv) = reinterpret_cast<const float4*>(dK + row * DP + c)[0];
        *reinterpret_cast<float4*>(kv + 4) = reinterpret_cast<const float4*>(dK + row * DP + c)[1];
        uint32_t qo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          qo[e] = pack_bf16x2(qv[2 * e] * cs[e] + qv[2 * e + 1] * sn[e], -qv[2 * e] * sn[e] + qv[2 * e + 1] * cs[e]);
          acc[2 * e] += kv[2 * e] * cs[e] + kv[2 * e + 1] * sn[e];
          acc[2 * e + 1] += -kv[2 * e] * sn[e] + kv[2 * e + 1] * cs[e];
        }
        *reinterpret_cast<uint4*>(dq + t * lddq + (size_t)h * (dn + dr) + c) = make_uint4(qo[0], qo[1], qo[2], qo[3]);
      }
      *reinterpret_cast<uint4*>(dkpe + t * ldk + k * 8) =
          make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                     pack_bf16x2(acc[6], acc[7]));
    }
  }
}

int blocks_for(long n, int per) { return (int)((n + per - 1) / per); }

}  // namespace

#define DSV3_PAIRS_LIST(X) X(1) X(2) X(3) X(4) X(6) X(8) X(12) X(16) X(24) X(32)

void rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, double eps, at::Tensor& y, at::Tensor& rstd) {
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && y.stride(1) == 1, "rmsnorm_fwd: 2-D row-major views");
  const int T = x.size(0), D = x.size(1);
  TORCH_CHECK(D <= 32 * kMaxPerLane, "rmsnorm_fwd: row too wide");
  const at::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  float* r = rstd.defined() && rstd.numel() ? rstd.data_ptr<float>() : nullptr;
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  const bool f = x.scalar_type() == at::kFloat;
  const bool vec_ok = D % 64 == 0 && x.stride(0) % 2 == 0 && y.stride(0) % 2 == 0;
#define DSV3_FWD_CASE(P)                                                                                        \
  if (vec_ok && D == 64 * P) {                                                                                 \
    if (f) rmsnorm_fwd_v<float, P><<<blocks_for(T, 8), 256, 0, st>>>(x.data_ptr<float>(), x.stride(0),        \
        w.data_ptr<float>(), (float)eps, yp, y.stride(0), r, T);                                               \
    else rmsnorm_fwd_v<__nv_bfloat16, P><<<blocks_for(T, 8), 256, 0, st>>>(                                    \
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), w.data_ptr<float>(), (float)eps, yp,  \
        y.stride(0), r, T);                                                                                    \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                            \
    return;                                                                                                    \
  }
  DSV3_PAIRS_LIST(DSV3_FWD_CASE)
#undef DSV3_FWD_CASE
  if (f)
    rmsnorm_fwd_kernel<float><<<blocks_for(T, 8), 256, 0, st>>>(x.data_ptr<float>(), x.stride(0), w.data_ptr<float>(),
        (float)eps, yp, y.stride(0), r, T, D);
  else
    rmsnorm_fwd_kernel<__nv_bfloat16><<<blocks_for(T, 8), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), w.data_ptr<float>(), (float)eps, yp,
        y.stride(0), r, T, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                 c10::optional<at::Tensor> dx_acc, c10::optional<at::Tensor> dx_out, c10::optional<at::Tensor> dx_copy,
                 at::Tensor& dw) {
  const int T = x.size(0), D = x.size(1);
  TORCH_CHECK(D <= 32 * kMaxPerLane, "rmsnorm_bwd: row too wide");
  TORCH_CHECK(dx_acc.has_value() != dx_out.has_value(), "rmsnorm_bwd: exactly one of dx_acc / dx_out");
  const at::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int rows_per_block = 64;
  float* acc = dx_acc ? dx_acc->data_ptr<float>() : nullptr;
  long ldacc = dx_acc ? dx_acc->stride(0) : 0;
  auto* out = dx_out ? reinterpret_cast<__nv_bfloat16*>(dx_out->data_ptr()) : nullptr;
  long ldout = dx_out ? dx_out->stride(0) : 0;
  auto* cp = dx_copy ? reinterpret_cast<__nv_bfloat16*>(dx_copy->data_ptr()) : nullptr;
  long ldcp = dx_copy ? dx_copy->stride(0) : 0;
  const int grid = blocks_for(T, rows_per_block);
  const size_t smem = D * sizeof(float);
  const bool vec_ok = D % 64 == 0 && x.stride(0) % 2 == 0 && dy.stride(0) % 2 == 0 && ldacc % 2 == 0 &&
                      ldout % 2 == 0 && ldcp % 2 == 0;
#define DSV3_BWD_V(TIN, TDY, P)                                                                                  \
  rmsnorm_bwd_v<TIN, TDY, P><<<grid, 256, 0, st>>>(reinterpret_cast<const TDY*>(dy.data_ptr()), dy.stride(0),     \
      reinterpret_cast<const TIN*>(x.data_ptr()), x.stride(0), w.data_ptr<float>(), rstd.data_ptr<float>(), acc,  \
      ldacc, out, ldout, cp, ldcp, dw.data_ptr<float>(), T, rows_per_block)
#define DSV3_BWD_CASE(P)                                                                                         \
  if (vec_ok && D == 64 * P) {                                                                                  \
    const bool xf_ = x.scalar_type() == at::kFloat, df_ = dy.scalar_type() == at::kFloat;                       \
    if (xf_ && df_) DSV3_BWD_V(float, float, P);                                                                 \
    else if (xf_) DSV3_BWD_V(float, __nv_bfloat16, P);                                                           \
    else if (df_) DSV3_BWD_V(__nv_bfloat16, float, P);                                                           \
    else DSV3_BWD_V(__nv_bfloat16, __nv_bfloat16, P);                                                            \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                             \
    return;                                                                                                     \
  }
  DSV3_PAIRS_LIST(DSV3_BWD_CASE)
#undef DSV3_BWD_CASE
#undef DSV3_BWD_V
#define DSV3_NORM_BWD(TIN, TDY)                                                                                   \
  rmsnorm_bwd_kernel<TIN, TDY><<<grid, 256, smem, st>>>(                                                          \
      reinterpret_cast<const TDY*>(dy.data_ptr()), dy.stride(0), reinterpret_cast<const TIN*>(x.data_ptr()),      \
      x.stride(0), w.data_ptr<float>(), rstd.data_ptr<float>(), acc, ldacc, out, ldout, cp, ldcp,                 \
      dw.data_ptr<float>(), T, D, rows_per_block)
  const bool xf = x.scalar_type() == at::kFloat, df = dy.scalar_type() == at::kFloat;
  if (xf && df) DSV3_NORM_BWD(float, float);
  else if (xf) DSV3_NORM_BWD(float, __nv_bfloat16);
  else if (df) DSV3_NORM_BWD(__nv_bfloat16, float);
  else DSV3_NORM_BWD(__nv_bfloat16, __nv_bfloat16);
#undef DSV3_NORM_BWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Shared memory the fused MoE-gradient + norm backward needs (W_gate staged as bf16).
int64_t moe_norm_bwd_smem(int64_t E, int64_t D) { return D * 8 + E * D * 4; }

void moe_norm_bwd(c10::optional<at::Tensor> dxs, c10::optional<at::Tensor> dst, c10::optional<at::Tensor> dsh,
                  const at::Tensor& dlog, const at::Tensor& wg, const at::Tensor& x, const at::Tensor& w,
                  const at::Tensor& rstd, at::Tensor& dres, at::Tensor& dres_b, at::Tensor& dw) {
  const int T = x.size(0), D = x.size(1), E = wg.size(0);
  TORCH_CHECK(x.scalar_type() == at::kFloat && dres.scalar_type() == at::kFloat && w.scalar_type() == at::kFloat &&
              dw.scalar_type() == at::kFloat && rstd.scalar_type() == at::kFloat, "moe_norm_bwd: fp32 x / dres / w / dw");
  TORCH_CHECK(dres_b.scalar_type() == at::kBFloat16 && dlog.scalar_type() == at::kBFloat16 &&
              wg.scalar_type() == at::kBFloat16 && wg.is_contiguous() && wg.size(1) == D,
              "moe_norm_bwd: bf16 dres_b / dlog, contiguous bf16 W_gate [E, D]");
  TORCH_CHECK(dlog.size(0) == T && dlog.size(1) >= E && dlog.stride(1) == 1, "moe_norm_bwd: dlog [T, >= E]");
  TORCH_CHECK(dxs.has_value() == dst.has_value(), "moe_norm_bwd: dxs and dst together");
  const int k = dst ? (int)dst->size(1) : 0;
  TORCH_CHECK(k <= kMoeNormMaxK, "moe_norm_bwd: at most ", kMoeNormMaxK, " routed slots per token");
  const int P = dxs ? (int)dxs->size(0) : 0;
  if (dxs) {
    TORCH_CHECK(dxs->scalar_type() == at::kBFloat16 && dxs->size(1) == D && dxs->stride(1) == 1 &&
                dxs->stride(0) % 2 == 0, "moe_norm_bwd: bf16 dxs [P, D]");
    TORCH_CHECK(dst->scalar_type() == at::kInt && dst->is_contiguous() && dst->size(0) == T, "moe_norm_bwd: dst [T, k]");
  }
  if (dsh) TORCH_CHECK(dsh->scalar_type() == at::kFloat && dsh->size(0) == T && dsh->size(1) == D &&
                       dsh->stride(1) == 1 && dsh->stride(0) % 2 == 0, "moe_norm_bwd: fp32 dsh [T, D]");
  TORCH_CHECK(x.stride(1) == 1 && dres.stride(1) == 1 && dres_b.stride(1) == 1 && x.stride(0) % 2 == 0 &&
              dres.stride(0) % 2 == 0 && dres_b.stride(0) % 2 == 0, "moe_norm_bwd: row-major, even row strides");
  const size_t smem = (size_t)moe_norm_bwd_smem(E, D);
  TORCH_CHECK(smem <= 200 * 1024, "moe_norm_bwd: W_gate too large for shared memory");
  const at::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  if (T == 0) return;
  // one CTA per SM (W_gate is staged once per SM), 8 rows per CTA at least
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  }
  const int rows_per_block = std::max(8, blocks_for(T, sms));
  const int grid = blocks_for(T, rows_per_block);
#define DSV3_MNB(P_)                                                                                               \
  if (D == 64 * P_) {                                                                                              \
    auto kern = moe_norm_bwd_v<P_>;                                                                                \
    if (smem > 48 * 1024) C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                                              (int)smem));                                         \
    kern<<<grid, 256, smem, st>>>(dxs ? reinterpret_cast<const __nv_bfloat16*>(dxs->data_ptr()) : nullptr,       \
        dxs ? dxs->stride(0) : 0, dst ? dst->data_ptr<int>() : nullptr, k, P,                                      \
        dsh ? dsh->data_ptr<float>() : nullptr, dsh ? dsh->stride(0) : 0,                                          \
        reinterpret_cast<const __nv_bfloat16*>(dlog.data_ptr()), dlog.stride(0),                                   \
        reinterpret_cast<const __nv_bfloat16*>(wg.data_ptr()), E, x.data_ptr<float>(), x.stride(0),                \
        w.data_ptr<float>(), rstd.data_ptr<float>(), dres.data_ptr<float>(), dres.stride(0),                       \
        reinterpret_cast<__nv_bfloat16*>(dres_b.data_ptr()), dres_b.stride(0), dw.data_ptr<float>(), T,           \
        rows_per_block, status_ptr());                                                                             \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                                \
    return;                                                                                                        \
  }
  DSV3_PAIRS_LIST(DSV3_MNB)
#undef DSV3_MNB
  TORCH_CHECK(false, "moe_norm_bwd: D must be 64 x one of 1, 2, 3, 4, 6, 8, 12, 16, 24, 32");
}

void rope_inplace(at::Tensor& x, int64_t off, int64_t half, const at::Tensor& cosv, const at::Tensor& sinv,
                  c10::optional<at::Tensor> pos, int64_t seqlen, int64_t start, bool inverse) {
  // x: [T, H, W] bf16 view (any strides on T / H, unit on W)
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1 && x.scalar_type() == at::kBFloat16, "rope_inplace: [T,H,W] bf16");
  const int T = x.size(0), H = x.size(1);
  const at::cuda::CUDAGuard guard(x.device());
  const long total = (long)T * H * half;
  rope_kernel<<<blocks_for(total, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0), x.stride(1), off, T, H, half,
      cosv.data_ptr<float>(), sinv.data_ptr<float>(), pos ? pos->data_ptr<int>() : nullptr, seqlen, start,
      inverse ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mla_pack(const at::Tensor& q, const at::Tensor& kvb, const at::Tensor& kpe, at::Tensor& Q, at::Tensor& K,
              at::Tensor& V, int64_t B, int64_t S, int64_t H, int64_t dn, int64_t dr, int64_t dv,
              const at::Tensor& cosv, const at::Tensor& sinv, int64_t start) {
  const int DP = Q.size(-1);
  const at::cuda::CUDAGuard guard(q.device());
  if (dn % 8 == 0 && dr % 8 == 0 && dv % 8 == 0 && DP % 8 == 0 && kpe.stride(0) % 8 == 0 && q.stride(0) % 8 == 0) {
    mla_pack_v<<<B * S, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(kvb.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(kpe.data_ptr()), kpe.stride(0),
        reinterpret_cast<__nv_bfloat16*>(Q.data_ptr()), reinterpret_cast<__nv_bfloat16*>(K.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(V.data_ptr()), S, H, dn, dr, dv, DP, cosv.data_ptr<float>(),
        sinv.data_ptr<float>(), start);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  TORCH_CHECK(q.stride(0) == H * (dn + dr), "mla_pack: strided q needs 8-element aligned head dims");
  dim3 grid(B * S, H);
  mla_pack_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(kvb.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(kpe.data_ptr()), kpe.stride(0),
      reinterpret_cast<__nv_bfloat16*>(Q.data_ptr()), reinterpret_cast<__nv_bfloat16*>(K.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(V.data_ptr()), B, S, H, dn, dr, dv, DP, cosv.data_ptr<float>(),
      sinv.data_ptr<float>(), start);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mla_unpack(const at::Tensor& dQ, const at::Tensor& dK, const at::Tensor& dV, at::Tensor& dq, at::Tensor& dkvb,
                at::Tensor& dkpe, int64_t B, int64_t S, int64_t H, int64_t dn, int64_t dr, int64_t dv,
                const at::Tensor& cosv, const at::Tensor& sinv, int64_t start) {
  const int DP = dQ.size(-1);
  const at::cuda::CUDAGuard guard(dQ.device());
  auto st = at::cuda::getCurrentCUDAStream();
  auto* dqp = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  auto* dkp = reinterpret_cast<__nv_bfloat16*>(dkvb.data_ptr());
  auto* dpe = reinterpret_cast<__nv_bfloat16*>(dkpe.data_ptr());
  if (dV.scalar_type() == at::kFloat && dn % 8 == 0 && dr % 8 == 0 && dv % 8 == 0 && DP % 8 == 0 &&
      dkpe.stride(0) % 8 == 0 && dq.stride(0) % 8 == 0) {
    constexpr int TB = 16;
    mla_unpack_blk<TB><<<dim3((S + TB - 1) / TB, B), 256, 0, st>>>(dQ.data_ptr<float>(), dK.data_ptr<float>(),
        dV.data_ptr<float>(), dqp, dq.stride(0), dkp, dpe, dkpe.stride(0), S, H, dn, dr, dv, DP, cosv.data_ptr<float>(),
        sinv.data_ptr<float>(), start);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  if (dV.scalar_type() == at::kFloat)
    mla_unpack_kernel<float><<<B * S, 64, dr * sizeof(float), st>>>(dQ.data_ptr<float>(), dK.data_ptr<float>(),
        dV.data_ptr<float>(), dqp, dkp, dpe, dkpe.stride(0), B, S, H, dn, dr, dv, DP, cosv.data_ptr<float>(),
        sinv.data_ptr<float>(), start);
  else
    mla_unpack_kernel<__nv_bfloat16><<<B * S, 64, dr * sizeof(float), st>>>(dQ.data_ptr<float>(),
        dK.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(dV.data_ptr()), dqp, dkp, dpe, dkpe.stride(0),
        B, S, H, dn, dr, dv, DP, cosv.data_ptr<float>(), sinv.data_ptr<float>(), start);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_fwd(const at::Tensor& tok, const at::Tensor& w, at::Tensor& out) {
  const int T = tok.numel(), D = w.size(1);
  TORCH_CHECK(D % 4 == 0 && tok.scalar_type() == at::kLong, "embedding_fwd: D % 4 == 0, int64 ids");
  TORCH_CHECK(tok.is_contiguous() && w.is_contiguous() && out.is_contiguous(), "embedding_fwd: contiguous tensors");
  const at::cuda::CUDAGuard guard(w.device());
  embedding_fwd_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream()>>>(tok.data_ptr<int64_t>(),
      w.data_ptr<float>(), out.data_ptr<float>(), T, D, w.size(0), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_bwd(const at::Tensor& tok, const at::Tensor& g, at::Tensor& dw) {
  const int T = tok.numel(), D = dw.size(1);
  TORCH_CHECK(tok.is_contiguous() && g.is_contiguous() && dw.is_contiguous(), "embedding_bwd: contiguous tensors");
  const at::cuda::CUDAGuard guard(dw.device());
  embedding_bwd_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream()>>>(tok.data_ptr<int64_t>(),
      g.data_ptr<float>(), dw.data_ptr<float>(), T, D, dw.size(0), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void cast_f32_bf16(const at::Tensor& a, at::Tensor& b) {
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && a.numel() == b.numel(), "cast: contiguous, same size");
  const long n = a.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(a.device());
  cast_f32_bf16_kernel<<<blocks_for(n, 1024), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      a.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(b.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_rows(const at::Tensor& pmax, const at::Tensor& psum, const at::Tensor& tl, const at::Tensor& tgt,
             at::Tensor& lse, at::Tensor& loss) {
  const int T = pmax.size(0), nt = pmax.size(1);
  TORCH_CHECK(tgt.is_contiguous() && pmax.is_contiguous() && psum.is_contiguous(), "ce_rows: contiguous tensors");
  const at::cuda::CUDAGuard guard(pmax.device());
  ce_rows_kernel<<<blocks_for(T, 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(pmax.data_ptr<float>(),
      psum.data_ptr<float>(), tl.data_ptr<float>(), tgt.data_ptr<int64_t>(), T, nt, lse.data_ptr<float>(),
      loss.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_reduce(const at::Tensor& loss_rows, const at::Tensor& tgt, const at::Tensor& seg_start,
               const at::Tensor& seg_weight, double grad_scale, at::Tensor& loss_out, at::Tensor& row_scale) {
  const at::cuda::CUDAGuard guard(loss_rows.device());
  const int nseg = seg_start.numel() - 1, rows = loss_rows.numel();
  auto st = at::cuda::getCurrentCUDAStream();
  at::Tensor acc = at::zeros({2 * nseg}, loss_rows.options());
  ce_seg_sum_kernel<<<std::max(1, (rows + 1023) / 1024), 256, 0, st>>>(loss_rows.data_ptr<float>(),
      tgt.data_ptr<int64_t>(), seg_start.data_ptr<int>(), nseg, rows, acc.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  ce_seg_scale_kernel<<<std::max(1, std::min(1024, (rows + 255) / 256)), 256, 0, st>>>(tgt.data_ptr<int64_t>(),
      seg_start.data_ptr<int>(), seg_weight.data_ptr<float>(), nseg, rows, (float)grad_scale, acc.data_ptr<float>(),
      loss_out.data_ptr<float>(), row_scale.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void heads_pack(const at::Tensor& src, int64_t col0, int64_t H, int64_t hd, int64_t S, at::Tensor& dst) {
  const int T = src.size(0), DP = dst.size(-1);
  const at::cuda::CUDAGuard guard(src.device());
  const bool vec = hd % 8 == 0 && DP % 8 == 0 && src.stride(0) % 8 == 0 && col0 % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(src.data_ptr()) | reinterpret_cast<uintptr_t>(dst.data_ptr())) & 15) == 0;
  if (vec) {
    const long total = (long)T * H * (DP / 8);
    if (total == 0) return;
    heads_pack_v<<<(int)((total + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), src.stride(0), (int)col0, (int)H, (int)hd, (int)S, DP,
        reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), (long)T);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  heads_pack_kernel<<<dim3(T, H), 64, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), src.stride(0), col0, H, hd, S, DP,
      reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void heads_unpack(const at::Tensor& src, int64_t H, int64_t hd, int64_t S, at::Tensor& dst, int64_t col0) {
  const int T = dst.size(0), DP = src.size(-1);
  const at::cuda::CUDAGuard guard(src.device());
  const bool vec = hd % 8 == 0 && DP % 4 == 0 && dst.stride(0) % 8 == 0 && col0 % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(src.data_ptr()) | reinterpret_cast<uintptr_t>(dst.data_ptr())) & 15) == 0;
  if (vec) {
    const long total = (long)T * H * (hd / 8);
    if (total == 0) return;
    heads_unpack_v<<<(int)((total + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        src.data_ptr<float>(), (int)H, (int)hd, (int)S, DP, reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()),
        dst.stride(0), (int)col0, (long)T);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  heads_unpack_kernel<<<dim3(T, H), 64, 0, at::cuda::getCurrentCUDAStream()>>>(src.data_ptr<float>(), H, hd, S, DP,
      reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), dst.stride(0), col0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_elementwise(pybind11::module_& m) {
  m.def("heads_pack", &heads_pack, "[T, ld] head slices -> [B*H, S, DP] (zero padded)");
  m.def("heads_unpack", &heads_unpack, "gradient of heads_pack (fp32 -> bf16 strided)");
  m.def("rmsnorm_fwd", &rmsnorm_fwd, "y(bf16) = rmsnorm(x) * w; stores 1/rms per row");
  m.def("rmsnorm_bwd", &rmsnorm_bwd, "RMSNorm backward (dx accumulate or store, dw +=)");
  m.def("moe_norm_bwd", &moe_norm_bwd,
        "MoE input gradient (shared + un-permuted routed + router rows) fused with the RMSNorm backward");
  m.def("moe_norm_bwd_smem", &moe_norm_bwd_smem, "shared memory bytes moe_norm_bwd needs for E experts of width D");
  m.def("rope_inplace", &rope_inplace, "rotate interleaved pairs in place (optionally inverse)");
  m.def("mla_pack", &mla_pack, "MLA Q/K/V packing with RoPE for the attention kernels");
  m.def("mla_unpack", &mla_unpack, "gradient of mla_pack");
  m.def("embedding_fwd", &embedding_fwd, "fp32 row gather");
  m.def("embedding_bwd", &embedding_bwd, "fp32 scatter-add into the embedding gradient");
  m.def("cast_f32_bf16", &cast_f32_bf16, "fp32 -> bf16");
  m.def("ce_rows", &ce_rows, "log-sum-exp and per-row loss from the fused head partials");
  m.def("ce_reduce", &ce_reduce, "per-segment mean loss and backward row scales");
}

}  // namespace dsv3
