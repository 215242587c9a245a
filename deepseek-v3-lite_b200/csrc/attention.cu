// MLA attention kernels.
//
// fa_fwd / fa_bwd: causal (global-position) flash attention over the
// materialised formulation: Q, K [BH, S, DQK] (DQK = dn + dr rounded up to a
// multiple of 16, zero padded), V [BH, S, DV].  Online softmax in the log2
// domain; the forward stores L = m + log2(l) per query row, the backward
// recomputes P from it (FlashAttention-2 schedule: one CTA per 64-key block,
// dK/dV in registers, dQ accumulated with fp32 atomics).  These use the
// warp-level mma.sync bf16 tensor-core path.
//
// latent_decode: absorbed-formulation decode over the latent cache with a
// per-row cache length, split over the sequence (split-K) with a second
// combine pass -- the decode step reads each cached latent row once per head
// group instead of materialising K/V.
#include <torch/extension.h>

#include <cstdlib>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attention_sm100.cuh"
#include "attention_bwd_wide.cuh"
#include "common.cuh"
#include "status.h"
#include "tma_host.h"

namespace dsv3 {

namespace {

typedef __nv_bfloat16 bf16;

#include "mma_sync.cuh"

constexpr int BM = 64;
constexpr int BN = 64;

// Copy a [rows x D] bf16 tile (row stride D in global) into smem with row
// stride SD, zero-filling rows >= valid_rows.
template <int D, int SD>
__device__ __forceinline__ void load_tile_async(bf16* s, const bf16* g, int rows, int valid_rows, int tid, int nthr) {
  constexpr int CH = D / 8;
  for (int c = tid; c < rows * CH; c += nthr) {
    const int r = c / CH, cc = (c % CH) * 8;
    const bool ok = r < valid_rows;
    cp_async16(s + r * SD + cc, g + (size_t)(ok ? r : 0) * D + cc, ok);
  }
}

// Same as load_tile_async with an explicit global row stride (elements).
template <int D, int SD>
__device__ __forceinline__ void load_tile_strided(bf16* s, const bf16* g, long ld, int rows, int valid_rows, int tid,
                                                  int nthr) {
  constexpr int CH = D / 8;
  for (int c = tid; c < rows * CH; c += nthr) {
    const int r = c / CH, cc = (c % CH) * 8;
    const bool ok = r < valid_rows;
    cp_async16(s + r * SD + cc, g + (size_t)(ok ? r : 0) * ld + cc, ok);
  }
}

template <int DQK, int DV>
__global__ void __launch_bounds__(128) fa_fwd_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K,
                                                     const bf16* __restrict__ V, bf16* __restrict__ O,
                                                     float* __restrict__ L, int Sq, int Sk, int q_off,
                                                     float scale_log2, int causal, int H) {
  constexpr int QS = DQK + 8, VS = DV + 8;
  extern __shared__ __align__(16) uint8_t fa_smem[];
  bf16* sQ = reinterpret_cast<bf16*>(fa_smem);
  bf16* sK = sQ + BM * QS;
  bf16* sV = sK + 2 * BN * QS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, m0 = blockIdx.x * BM;
  const bf16* Qb = Q + (size_t)bh * Sq * DQK;
  const bf16* Kb = K + (size_t)bh * Sk * DQK;
  const bf16* Vb = V + (size_t)bh * Sk * DV;

  load_tile_async<DQK, QS>(sQ, Qb + (size_t)m0 * DQK, BM, Sq - m0, tid, 128);
  const int n_end = causal ? min(Sk, q_off + m0 + BM) : Sk;
  const int nblocks = (n_end + BN - 1) / BN;
  if (nblocks > 0) {
    load_tile_async<DQK, QS>(sK, Kb, BN, Sk, tid, 128);
    load_tile_async<DV, VS>(sV, Vb, BN, Sk, tid, 128);
  }
  cp_async_commit();

  float o[DV / 8][4];
#pragma unroll
  for (int i = 0; i < DV / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int g = lane >> 2, tig = lane & 3;
  const int qrow0 = m0 + warp * 16 + g;  // rows qrow0 and qrow0 + 8

  for (int nb = 0; nb < nblocks; ++nb) {
    const int st = nb & 1;
    if (nb + 1 < nblocks) {
      const int n1 = (nb + 1) * BN;
      load_tile_async<DQK, QS>(sK + (st ^ 1) * BN * QS, Kb + (size_t)n1 * DQK, BN, Sk - n1, tid, 128);
      load_tile_async<DV, VS>(sV + (st ^ 1) * BN * VS, Vb + (size_t)n1 * DV, BN, Sk - n1, tid, 128);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const bf16* k_s = sK + st * BN * QS;
    const bf16* v_s = sV + st * BN * VS;

    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DQK / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, sQ + (warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * QS + kk * 16 + 8 * (lane >> 4));
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        ldsm_x4(b, k_s + (np * 16 + (lane & 7) + 8 * (lane >> 4)) * QS + kk * 16 + 8 * ((lane >> 3) & 1));
        mma16816(s[2 * np], a, b[0], b[1]);
        mma16816(s[2 * np + 1], a, b[2], b[3]);
      }
    }
    // scale + mask, then online softmax per row (rows g and g + 8 of the warp)
    const int n0 = nb * BN;
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = n0 + j * 8 + 2 * tig + (e & 1);
        const int qr = qrow0 + (e >> 1) * 8;
        float v = s[j][e] * scale_log2;
        if (col >= Sk || (causal && col > q_off + qr)) v = -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) corr[r] = mx[r] == -INFINITY ? 1.f : exp2f(mrow[r] - mx[r]);
    uint32_t pa[4][4];  // P as A fragments, 4 k16 chunks over the 64 keys
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = mx[e >> 1];
        p[e] = m == -INFINITY ? 0.f : exp2f(s[j][e] - m);
        rs[e >> 1] += p[e];
      }
      pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(p[0], p[1]);
      pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(p[2], p[3]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      lrow[r] = lrow[r] * corr[r] + rs[r];
      mrow[r] = mx[r];
    }
#pragma unroll
    for (int i = 0; i < DV / 8; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    // O += P V   (A fragment order: a0 = rows g / k lo, a1 = rows g+8 / k lo, a2, a3 = k hi)
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t a[4] = {pa[kc][0], pa[kc][1], pa[kc][2], pa[kc][3]};
#pragma unroll
      for (int dp = 0; dp < DV / 16; ++dp) {
        uint32_t b[4];
        ldsm_x4_t(b, v_s + (kc * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * VS + dp * 16 + 8 * (lane >> 4));
        mma16816(o[2 * dp], a, b[0], b[1]);
        mma16816(o[2 * dp + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // O is token-major: [B, Sq, H, DV]
  bf16* Ob = O + ((size_t)(bh / H) * Sq * H + (bh % H)) * DV;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qr = qrow0 + r * 8;
    if (qr >= Sq) continue;
    const float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
#pragma unroll
    for (int i = 0; i < DV / 8; ++i) {
      const int col = i * 8 + 2 * tig;
      *reinterpret_cast<uint32_t*>(Ob + (size_t)qr * H * DV + col) = pack_bf16x2(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
    }
    if (tig == 0) L[(size_t)bh * Sq + qr] = lrow[r] > 0.f ? mrow[r] + log2f(lrow[r]) : -INFINITY;
  }
}

// delta[row] = sum_d dO[row, d] * O[row, d]
// O / dO token-major [B, S, H, DV]; row r = (b*S + s)*H + h; delta is [B*H, S].
// DV / 8 lanes share a row (one 16-byte load of each tensor per lane), so a
// warp's loads cover 32 * 16 consecutive bytes; the partial dots are summed
// over the row's lanes by shuffles.
template <int DV>
__global__ void __launch_bounds__(256) fa_bwd_pre_kernel(const bf16* __restrict__ O, const bf16* __restrict__ dO,
                                                         float* __restrict__ delta, long rows, int S, int H) {
  constexpr int LPR = DV / 8;                       // lanes per row
  static_assert(DV % 8 == 0 && LPR <= 32 && (32 % LPR) == 0, "fa_bwd_pre: DV / 8 divides 32");
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long r = t / LPR;
  const int j = (int)(t % LPR);
  float acc = 0.f;
  if (r < rows) {
    const uint4 a = reinterpret_cast<const uint4*>(O + r * DV)[j];
    const uint4 d = reinterpret_cast<const uint4*>(dO + r * DV)[j];
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&d);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __bfloat1622float2(a2[i]), y = __bfloat1622float2(d2[i]);
      acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
    }
  }
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (r < rows && j == 0) {
    const long h = r % H, bs = r / H, b = bs / S, s = bs % S;
    delta[(b * H + h) * S + s] = acc;
  }
}

template <int DQK, int DV>
__global__ void __launch_bounds__(128) fa_bwd_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K,
                                                     const bf16* __restrict__ V, const bf16* __restrict__ dO,
                                                     const float* __restrict__ L, const float* __restrict__ delta,
                                                     float* __restrict__ dQ, float* __restrict__ dK,
                                                     float* __restrict__ dV, int Sq, int Sk, int q_off,
                                                     float scale_log2, float scale, int causal, int H) {
  constexpr int QS = DQK + 8, VS = DV + 8, PS = BM + 8;
  extern __shared__ __align__(16) uint8_t fa_smem[];
  bf16* sK = reinterpret_cast<bf16*>(fa_smem);
  bf16* sV = sK + BN * QS;
  bf16* sQ = sV + BN * VS;
  bf16* sdO = sQ + BM * QS;
  bf16* sdS = sdO + BM * VS;  // dS^T [keys][queries]
  float* sL = reinterpret_cast<float*>(sdS + BN * PS);
  float* sD = sL + BM;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int bh = blockIdx.y, n0 = blockIdx.x * BN;
  const bf16* Qb = Q + (size_t)bh * Sq * DQK;
  const bf16* Kb = K + (size_t)bh * Sk * DQK;
  const bf16* Vb = V + (size_t)bh * Sk * DV;
  const bf16* dOb = dO + ((size_t)(bh / H) * Sq * H + (bh % H)) * DV;  // token-major, row stride H*DV

  load_tile_async<DQK, QS>(sK, Kb + (size_t)n0 * DQK, BN, Sk - n0, tid, 128);
  load_tile_async<DV, VS>(sV, Vb + (size_t)n0 * DV, BN, Sk - n0, tid, 128);
  cp_async_commit();

  float dk[DQK / 8][4], dv[DV / 8][4];
#pragma unroll
  for (int i = 0; i < DQK / 8; ++i) dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
#pragma unroll
  for (int i = 0; i < DV / 8; ++i) dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;

  // first query block that can see key n0: q_off + q >= n0
  const int qstart = causal ? max(0, (n0 - q_off) / BM * BM) : 0;
  const int key0 = n0 + warp * 16 + g;  // this thread's keys: key0, key0 + 8
  for (int m0 = qstart; m0 < Sq; m0 += BM) {
    load_tile_async<DQK, QS>(sQ, Qb + (size_t)m0 * DQK, BM, Sq - m0, tid, 128);
    load_tile_strided<DV, VS>(sdO, dOb + (size_t)m0 * H * DV, (long)H * DV, BM, Sq - m0, tid, 128);
    cp_async_commit();
    for (int i = tid; i < BM; i += 128) {
      const bool ok = m0 + i < Sq;
      sL[i] = ok ? L[(size_t)bh * Sq + m0 + i] : 0.f;
      sD[i] = ok ? delta[(size_t)bh * Sq + m0 + i] : 0.f;
    }
    cp_async_wait<0>();
    __syncthreads();

    // S^T = K Q^T  (16 keys x 64 queries per warp)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DQK / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, sK + (warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * QS + kk * 16 + 8 * (lane >> 4));
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        ldsm_x4(b, sQ + (np * 16 + (lane & 7) + 8 * (lane >> 4)) * QS + kk * 16 + 8 * ((lane >> 3) & 1));
        mma16816(s[2 * np], a, b[0], b[1]);
        mma16816(s[2 * np + 1], a, b[2], b[3]);
      }
    }
    // dP^T = V dO^T
    float dp[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) dp[j][0] = dp[j][1] = dp[j][2] = dp[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DV / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, sV + (warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * VS + kk * 16 + 8 * (lane >> 4));
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        ldsm_x4(b, sdO + (np * 16 + (lane & 7) + 8 * (lane >> 4)) * VS + kk * 16 + 8 * ((lane >> 3) & 1));
        mma16816(dp[2 * np], a, b[0], b[1]);
        mma16816(dp[2 * np + 1], a, b[2], b[3]);
      }
    }
    // P^T, dS^T (register fragments reused as A operands)
    uint32_t pa[4][4], dsa[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p[4], ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = m0 + j * 8 + 2 * tig + (e & 1);
        const int key = key0 + (e >> 1) * 8;
        const int qi = j * 8 + 2 * tig + (e & 1);
        const bool valid = q < Sq && key < Sk && !(causal && key > q_off + q);
        p[e] = valid ? exp2f(s[j][e] * scale_log2 - sL[qi]) : 0.f;
        ds[e] = p[e] * (dp[j][e] - sD[qi]);
      }
      pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(p[0], p[1]);
      pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(p[2], p[3]);
      dsa[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(ds[0], ds[1]);
      dsa[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(ds[2], ds[3]);
      // stash dS^T for the dQ product
      bf16* row0 = sdS + (warp * 16 + g) * PS + j * 8 + 2 * tig;
      bf16* row1 = row0 + 8 * PS;
      *reinterpret_cast<uint32_t*>(row0) = pack_bf16x2(ds[0], ds[1]);
      *reinterpret_cast<uint32_t*>(row1) = pack_bf16x2(ds[2], ds[3]);
    }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t a[4] = {pa[kc][0], pa[kc][1], pa[kc][2], pa[kc][3]};
#pragma unroll
      for (int d2 = 0; d2 < DV / 16; ++d2) {
        uint32_t b[4];
        ldsm_x4_t(b, sdO + (kc * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * VS + d2 * 16 + 8 * (lane >> 4));
        mma16816(dv[2 * d2], a, b[0], b[1]);
        mma16816(dv[2 * d2 + 1], a, b[2], b[3]);
      }
      uint32_t a2[4] = {dsa[kc][0], dsa[kc][1], dsa[kc][2], dsa[kc][3]};
#pragma unroll
      for (int d2 = 0; d2 < DQK / 16; ++d2) {
        uint32_t b[4];
        ldsm_x4_t(b, sQ + (kc * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * QS + d2 * 16 + 8 * (lane >> 4));
        mma16816(dk[2 * d2], a2, b[0], b[1]);
        mma16816(dk[2 * d2 + 1], a2, b[2], b[3]);
      }
    }
    __syncthreads();
    // dQ[q, :] += sum_keys dS[q, key] K[key, :]   (warp: 16 queries)
    {
      float dq[DQK / 8][4];
#pragma unroll
      for (int i = 0; i < DQK / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kc = 0; kc < 4; ++kc) {
        uint32_t a[4];
        ldsm_x4_t(a, sdS + (kc * 16 + (lane & 7) + 8 * (lane >> 4)) * PS + warp * 16 + 8 * ((lane >> 3) & 1));
#pragma unroll
        for (int d2 = 0; d2 < DQK / 16; ++d2) {
          uint32_t b[4];
          ldsm_x4_t(b, sK + (kc * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * QS + d2 * 16 + 8 * (lane >> 4));
          mma16816(dq[2 * d2], a, b[0], b[1]);
          mma16816(dq[2 * d2 + 1], a, b[2], b[3]);
        }
      }
      float* dQb = dQ + (size_t)bh * Sq * DQK;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int q = m0 + warp * 16 + g + r * 8;
        if (q >= Sq) continue;
#pragma unroll
        for (int i = 0; i < DQK / 8; ++i) {
          atomicAdd(dQb + (size_t)q * DQK + i * 8 + 2 * tig, dq[i][2 * r] * scale);
          atomicAdd(dQb + (size_t)q * DQK + i * 8 + 2 * tig + 1, dq[i][2 * r + 1] * scale);
        }
      }
    }
    __syncthreads();
  }
  float* dKb = dK + (size_t)bh * Sk * DQK;
  float* dVb = dV + (size_t)bh * Sk * DV;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = key0 + r * 8;
    if (key >= Sk) continue;
#pragma unroll
    for (int i = 0; i < DQK / 8; ++i) {
      dKb[(size_t)key * DQK + i * 8 + 2 * tig] = dk[i][2 * r] * scale;
      dKb[(size_t)key * DQK + i * 8 + 2 * tig + 1] = dk[i][2 * r + 1] * scale;
    }
#pragma unroll
    for (int i = 0; i < DV / 8; ++i) {
      dVb[(size_t)key * DV + i * 8 + 2 * tig] = dv[i][2 * r];
      dVb[(size_t)key * DV + i * 8 + 2 * tig + 1] = dv[i][2 * r + 1];
    }
  }
}

#include "latent_decode.cuh"

template <int DQK, int DV>
size_t fwd_smem() {
  return (size_t)(BM * (DQK + 8) + 2 * BN * (DQK + 8) + 2 * BN * (DV + 8)) * 2;
}
template <int DQK, int DV>
size_t bwd_smem() {
  return (size_t)(BN * (DQK + 8) + BN * (DV + 8) + BM * (DQK + 8) + BM * (DV + 8) + BN * (BM + 8)) * 2 +
         2 * BM * sizeof(float);
}

template <int DQK, int DV>
void run_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse, int q_off,
             double scale, bool causal, int H) {
  const int BH = q.size(0), Sq = q.size(1), Sk = k.size(1);
  auto kern = fa_fwd_kernel<DQK, DV>;
  const size_t smem = fwd_smem<DQK, DV>();
  static bool cfg = false;
  if (!cfg) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cfg = true;
  }
  dim3 grid((Sq + BM - 1) / BM, BH);
  kern<<<grid, 128, smem, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
      reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<bf16*>(o.data_ptr()), lse.data_ptr<float>(), Sq,
      Sk, q_off, (float)(scale * 1.4426950408889634), causal ? 1 : 0, H);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int DV>
void launch_bwd_pre(const at::Tensor& o, const at::Tensor& dout, at::Tensor& delta, long rows, int Sq, int H,
                    cudaStream_t st) {
  TORCH_CHECK(((reinterpret_cast<uintptr_t>(o.data_ptr()) | reinterpret_cast<uintptr_t>(dout.data_ptr())) & 15) == 0,
              "flash_bwd: O and dO must be 16-byte aligned");
  fa_bwd_pre_kernel<DV><<<(int)((rows * (DV / 8) + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const bf16*>(o.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
      delta.data_ptr<float>(), rows, Sq, H);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int DQK, int DV>
void run_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
             const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq, at::Tensor& dk,
             at::Tensor& dv, int q_off, double scale, bool causal, int H) {
  const int BH = q.size(0), Sq = q.size(1), Sk = k.size(1);
  auto st = at::cuda::getCurrentCUDAStream();
  const long rows = (long)BH * Sq;
  launch_bwd_pre<DV>(o, dout, delta, rows, Sq, H, st);
  auto kern = fa_bwd_kernel<DQK, DV>;
  const size_t smem = bwd_smem<DQK, DV>();
  static bool cfg = false;
  if (!cfg) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cfg = true;
  }
  dim3 grid((Sk + BN - 1) / BN, BH);
  kern<<<grid, 128, smem, st>>>(reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
      reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
      lse.data_ptr<float>(), delta.data_ptr<float>(), dq.data_ptr<float>(), dk.data_ptr<float>(),
      dv.data_ptr<float>(), Sq, Sk, q_off, (float)(scale * 1.4426950408889634), (float)scale, causal ? 1 : 0, H);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


// Causal tcgen05 kernels take, instead of a plain 1, the number of (batch,
// head) rows per tile-order group: tiles run heaviest first within a group,
// and a group's K/V (or Q/dO) rows, about 64 MB at most, stay in L2 while
// its CTAs run.  0 = not causal.
inline int causal_groups(bool causal, int BH, long rows, int dqk, int dv) {
  if (!causal) return 0;
  const long per_bh = std::max(1L, rows * (long)(dqk + dv) * 2);
  const long g = (64L << 20) / per_bh;
  return (int)std::max(1L, std::min((long)BH, g));
}

template <int NA, int NB, int DV>
void run_fwd_sm100(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                   int q_off, double scale, bool causal, int H) {
  const int BH = q.size(0), Sq = q.size(1), Sk = k.size(1), DP = q.size(2);
  using Cfg = FaCfg<NA, NB, DV>;
  auto mk = [](const at::Tensor& t, int S, int D, uint32_t box0, CUtensorMapSwizzle swz) {
    uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)t.size(0)};
    uint64_t st[2] = {(uint64_t)D * 2, (uint64_t)S * D * 2};
    uint32_t box[3] = {box0, 128, 1};
    return make_map(t.data_ptr(), 3, dims, st, box, swz);
  };
  CUtensorMap qa = mk(q, Sq, DP, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap ka = mk(k, Sk, DP, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap qb = NB ? mk(q, Sq, DP, 16, CU_TENSOR_MAP_SWIZZLE_32B) : qa;
  CUtensorMap kb = NB ? mk(k, Sk, DP, 16, CU_TENSOR_MAP_SWIZZLE_32B) : ka;
  CUtensorMap vm = mk(v, Sk, DV, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  // two query tiles per CTA (independent softmax chains) for qk <= 80, v 64;
  // DSV3_FA_FWD_2Q=0 selects the one-tile kernel
  if constexpr (Fa2Cfg<NA, NB, DV>::FITS) {
    static const bool two_q = [] {
      const char* e = getenv("DSV3_FA_FWD_2Q");
      return !(e != nullptr && e[0] == '0');
    }();
    if (two_q) {
      using C2 = Fa2Cfg<NA, NB, DV>;
      auto k2 = fa_fwd2q_sm100_kernel<NA, NB, DV>;
      static bool cfg2 = false;
      if (!cfg2) {
        C10_CUDA_CHECK(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, C2::SMEM));
        cfg2 = true;
      }
      k2<<<dim3((Sq + 255) / 256, BH), 320, C2::SMEM, at::cuda::getCurrentCUDAStream()>>>(qa, qb, ka, kb, vm,
          reinterpret_cast<bf16*>(o.data_ptr()), lse.data_ptr<float>(), Sq, Sk, H, q_off,
          (float)(scale * 1.4426950408889634), causal_groups(causal, BH, Sk, (int)q.size(2), DV), status_ptr());
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      return;
    }
  }
  // two softmax warpgroups per CTA where the exchange buffer fits
  // (DSV3_FA_FWD_WG=1: one)
  constexpr int WG2 = Cfg::XR_B > 0 ? 2 : 1;
  static const int wg = [] {
    const char* e = getenv("DSV3_FA_FWD_WG");
    return (e != nullptr && e[0] == '1') ? 1 : WG2;
  }();
  auto kern = wg == 2 ? fa_fwd_sm100_kernel<NA, NB, DV, WG2> : fa_fwd_sm100_kernel<NA, NB, DV, 1>;
  static bool cfg = false;
  if (!cfg) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(fa_fwd_sm100_kernel<NA, NB, DV, 1>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    C10_CUDA_CHECK(cudaFuncSetAttribute(fa_fwd_sm100_kernel<NA, NB, DV, WG2>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    cfg = true;
  }
  dim3 grid((Sq + 127) / 128, BH);
  kern<<<grid, 64 + 128 * wg, Cfg::SMEM, at::cuda::getCurrentCUDAStream()>>>(qa, qb, ka, kb, vm,
      reinterpret_cast<bf16*>(o.data_ptr()), lse.data_ptr<float>(), Sq, Sk, H, q_off,
      (float)(scale * 1.4426950408889634), causal_groups(causal, BH, Sk, (int)q.size(2), DV), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int NA, int NB, int DV>
void run_bwd_sm100(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                   const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq, at::Tensor& dk,
                   at::Tensor& dv, int q_off, double scale, bool causal, int H) {
  const int BH = q.size(0), Sq = q.size(1), Sk = k.size(1), DP = q.size(2);
  const int B = BH / H;
  auto st = at::cuda::getCurrentCUDAStream();
  const long rows = (long)BH * Sq;
  launch_bwd_pre<DV>(o, dout, delta, rows, Sq, H, st);
  using Cfg = FabCfg<NA, NB, DV>;
  auto mk = [](const at::Tensor& t, int S, int D, uint32_t box0, CUtensorMapSwizzle swz) {
    uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)t.size(0)};
    uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)S * D * 2};
    uint32_t box[3] = {box0, 128, 1};
    return make_map(t.data_ptr(), 3, dims, strides, box, swz);
  };
  CUtensorMap qa = mk(q, Sq, DP, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap ka = mk(k, Sk, DP, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap qb = NB ? mk(q, Sq, DP, 16, CU_TENSOR_MAP_SWIZZLE_32B) : qa;
  CUtensorMap kb = NB ? mk(k, Sk, DP, 16, CU_TENSOR_MAP_SWIZZLE_32B) : ka;
  CUtensorMap vm = mk(v, Sk, DV, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  // dO is token-major [B, Sq, H, DV]
  uint64_t ddims[4] = {(uint64_t)DV, (uint64_t)H, (uint64_t)Sq, (uint64_t)B};
  uint64_t dstr[3] = {(uint64_t)DV * 2, (uint64_t)H * DV * 2, (uint64_t)Sq * H * DV * 2};
  uint32_t dbox[4] = {64, 1, 128, 1};
  CUtensorMap dom = make_map(dout.data_ptr(), 4, ddims, dstr, dbox, CU_TENSOR_MAP_SWIZZLE_128B);
  // DSV3_FA_BWD_DRAIN=1: four dedicated dQ-drain warps (measured 4% slower
  // on the 412M shapes than draining from the softmax warps, which is the
  // default)
  static const int drain = [] {
    const char* e = getenv("DSV3_FA_BWD_DRAIN");
    return (e != nullptr && e[0] == '1') ? 1 : 0;
  }();
  auto kern = drain ? fa_bwd_sm100_kernel<NA, NB, DV, 1> : fa_bwd_sm100_kernel<NA, NB, DV, 0>;
  static bool cfg = false;
  if (!cfg) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(fa_bwd_sm100_kernel<NA, NB, DV, 0>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    C10_CUDA_CHECK(cudaFuncSetAttribute(fa_bwd_sm100_kernel<NA, NB, DV, 1>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    cfg = true;
  }
  dim3 grid((Sk + 127) / 128, BH);
  kern<<<grid, 320 + 128 * drain, Cfg::SMEM, st>>>(qa, qb, ka, kb, vm, dom, lse.data_ptr<float>(), delta.data_ptr<float>(),
      dq.data_ptr<float>(), dk.data_ptr<float>(), dv.data_ptr<float>(), Sq, Sk, H, q_off,
      (float)(scale * 1.4426950408889634), (float)scale, causal_groups(causal, BH, Sq, (int)q.size(2), DV), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Two-kernel tcgen05 backward (qk 64 * NA + 16 * NB, v DV): dK / dV per key
// tile over 64-query sub-tiles, then dQ per query tile (attention_bwd_wide.cuh).
template <int NA, int NB, int DV>
void run_bwd_sm100_wide(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                        const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq,
                        at::Tensor& dk, at::Tensor& dv, int q_off, double scale, bool causal, int H) {
  const int BH = q.size(0), Sq = q.size(1), Sk = k.size(1), DP = q.size(2);
  TORCH_CHECK(DP == NA * 64 + NB * 16 && v.size(2) == DV, "flash backward (two-kernel): head dims");
  const int B = BH / H;
  auto st = at::cuda::getCurrentCUDAStream();
  const long rows = (long)BH * Sq;
  launch_bwd_pre<DV>(o, dout, delta, rows, Sq, H, st);
  // [b*h, S, D] bf16 with `box_rows`-row boxes: 64 columns in 128B swizzle
  // (or the 16-column block in 32B swizzle)
  auto mk = [](const at::Tensor& t, int S, int D, uint32_t box_rows, bool narrow = false) {
    uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)t.size(0)};
    uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)S * D * 2};
    uint32_t box[3] = {narrow ? 16u : 64u, box_rows, 1};
    return make_map(t.data_ptr(), 3, dims, strides, box,
                    narrow ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_128B);
  };
  // dO is token-major [B, Sq, H, DV]
  auto mk_do = [&](uint32_t box_rows) {
    uint64_t ddims[4] = {(uint64_t)DV, (uint64_t)H, (uint64_t)Sq, (uint64_t)B};
    uint64_t dstr[3] = {(uint64_t)DV * 2, (uint64_t)H * DV * 2, (uint64_t)Sq * H * DV * 2};
    uint32_t dbox[4] = {64, 1, box_rows, 1};
    return make_map(dout.data_ptr(), 4, ddims, dstr, dbox, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  const CUtensorMap q64 = mk(q, Sq, DP, 64), q128 = mk(q, Sq, DP, 128), k128 = mk(k, Sk, DP, 128);
  const CUtensorMap q64b = NB ? mk(q, Sq, DP, 64, true) : q64, q128b = NB ? mk(q, Sq, DP, 128, true) : q128;
  const CUtensorMap k128b = NB ? mk(k, Sk, DP, 128, true) : k128;
  const CUtensorMap v128 = mk(v, Sk, DV, 128), do64 = mk_do(64), do128 = mk_do(128);
  const float sl2 = (float)(scale * 1.4426950408889634), sc = (float)scale;
  using Ckv = FabKvCfg<NA, NB, DV>;
  using Cq = FabQCfg<NA, NB, DV>;
  auto kkv = fa_bwd_kv_sm100_kernel<NA, NB, DV>;
  auto kq = fa_bwd_dq_sm100_kernel<NA, NB, DV>;
  static bool cfg = false;
  if (!cfg) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kkv, cudaFuncAttributeMaxDynamicSharedMemorySize, Ckv::SMEM));
    C10_CUDA_CHECK(cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, Cq::SMEM));
    cfg = true;
  }
  kkv<<<dim3((Sk + 127) / 128, BH), 320, Ckv::SMEM, st>>>(q64, q64b, k128, k128b, v128, do64, lse.data_ptr<float>(),
      delta.data_ptr<float>(), dk.data_ptr<float>(), dv.data_ptr<float>(), Sq, Sk, H, q_off, sl2, sc,
      causal_groups(causal, BH, Sq, (int)q.size(2), DV), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  kq<<<dim3((Sq + 127) / 128, BH), 320, Cq::SMEM, st>>>(q128, q128b, k128, k128b, v128, do128, lse.data_ptr<float>(),
      delta.data_ptr<float>(), dq.data_ptr<float>(), Sq, Sk, H, q_off, sl2, sc, causal_groups(causal, BH, Sk, (int)q.size(2), DV), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// The wide-head tcgen05 backward is opt-in (DSV3_FA_BWD_WIDE=1) until it has
// been validated on the GPU; flash_bwd otherwise keeps the mma.sync kernel
// for qk 128 / 192.
// The two-kernel tcgen05 backward serves qk 128 / 192 with v 128 (validated
// against fp32 on B200: dQ / dK / dV within 3e-2); DSV3_FA_BWD_WIDE=0 falls
// back to the warp-level mma.sync kernel for those head dims.
bool wide_bwd_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("DSV3_FA_BWD_WIDE");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

#define DSV3_FA_DISPATCH(DQK_, DV_, CALL)                                                          \
  if (dqk == DQK_ && dvv == DV_) {                                                                 \
    CALL;                                                                                          \
    return;                                                                                        \
  }

}  // namespace

// q, k: [B*H, S, DQK] bf16; v: [B*H, Sk, DV]; o: token-major [B, Sq, H, DV] bf16;
// lse: [B*H, Sq] fp32 (log2 domain).
void flash_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
               int64_t q_off, double scale, bool causal, int64_t H) {
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && o.is_contiguous(), "flash_fwd: contiguous");
  const at::cuda::CUDAGuard guard(q.device());
  const int dqk = q.size(2), dvv = v.size(2);
  // tcgen05 kernels where the head dims map onto 64/16-element swizzle blocks
  DSV3_FA_DISPATCH(80, 64, (run_fwd_sm100<1, 1, 64>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(64, 64, (run_fwd_sm100<1, 0, 64>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(128, 128, (run_fwd_sm100<2, 0, 128>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(192, 128, (run_fwd_sm100<3, 0, 128>(q, k, v, o, lse, q_off, scale, causal, H)))
  // warp-level mma.sync kernels for the remaining shapes
  DSV3_FA_DISPATCH(32, 16, (run_fwd<32, 16>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(16, 16, (run_fwd<16, 16>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(32, 32, (run_fwd<32, 32>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(192, 128, (run_fwd<192, 128>(q, k, v, o, lse, q_off, scale, causal, H)))
  TORCH_CHECK(false, "flash_fwd: unsupported head dims ", dqk, "/", dvv);
}

void flash_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
               const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq, at::Tensor& dk,
               at::Tensor& dv, int64_t q_off, double scale, bool causal, int64_t H) {
  const at::cuda::CUDAGuard guard(q.device());
  const int dqk = q.size(2), dvv = v.size(2);
  DSV3_FA_DISPATCH(80, 64, (run_bwd_sm100<1, 1, 64>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(64, 64, (run_bwd_sm100<1, 0, 64>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  if (wide_bwd_enabled()) {
    DSV3_FA_DISPATCH(192, 128, (run_bwd_sm100_wide<3, 0, 128>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale,
                                                           causal, H)))
    DSV3_FA_DISPATCH(128, 128, (run_bwd_sm100_wide<2, 0, 128>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale,
                                                           causal, H)))
  }
  DSV3_FA_DISPATCH(32, 16, (run_bwd<32, 16>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(16, 16, (run_bwd<16, 16>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(32, 32, (run_bwd<32, 32>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(64, 64, (run_bwd<64, 64>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(128, 128, (run_bwd<128, 128>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(192, 128, (run_bwd<192, 128>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  TORCH_CHECK(false, "flash_bwd: unsupported head dims ", dqk, "/", dvv);
}


// q_lat [B, H, R], q_pe [B, H, dr], kv [B, S, R] (batch stride kv.stride(0)),
// pe [B, S, dr], lens [B] int32 -> out [B, H, R] bf16.
// Query rows may outnumber cache rows: row b reads cache batch b / qpb, where
// qpb = q_lat.size(0) / kv.size(0) (1 for plain decode, S for a chunk of S
// queries per sequence).
void latent_decode(const at::Tensor& q_lat, const at::Tensor& q_pe, const at::Tensor& kv, const at::Tensor& pe,
                   const at::Tensor& lens, double scale, int64_t max_len, at::Tensor& scratch, at::Tensor& out,
                   int64_t qpb) {
  const int B = q_lat.size(0), H = q_lat.size(1), R = q_lat.size(2), dr = q_pe.size(2);
  TORCH_CHECK(R <= 1024 && dr <= 128, "latent_decode: R <= 1024, dr <= 128");
  const at::cuda::CUDAGuard guard(q_lat.device());
  const long long need = latent_decode_scratch_floats(B, H, R, (int)max_len);
  TORCH_CHECK(scratch.numel() >= need && scratch.scalar_type() == at::kFloat, "latent_decode: scratch too small (need ",
              need, " floats)");
  TORCH_CHECK(kv.stride(1) == R && pe.stride(1) == dr && kv.stride(2) == 1 && pe.stride(2) == 1,
              "latent_decode: cache rows must be contiguous");
  LatentDecodeArgs a{};
  a.q_lat = reinterpret_cast<const bf16*>(q_lat.data_ptr());
  a.q_pe = reinterpret_cast<const bf16*>(q_pe.data_ptr());
  a.kv = reinterpret_cast<const bf16*>(kv.data_ptr());
  a.pe = reinterpret_cast<const bf16*>(pe.data_ptr());
  a.lens = lens.data_ptr<int>();
  a.B = B;
  a.H = H;
  a.R = R;
  a.dr = dr;
  a.kv_bs = kv.stride(0);
  a.pe_bs = pe.stride(0);
  a.qpb = (int)std::max<int64_t>(1, qpb);
  a.max_len = (int)max_len;
  a.scale = (float)scale;
  a.scratch = scratch.data_ptr<float>();
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.cache_rows = std::min(kv.size(1), pe.size(1));
  a.cache_batches = (int)std::min(kv.size(0), pe.size(0));
  a.status = status_ptr();
  C10_CUDA_CHECK(launch_latent_decode(a, at::cuda::getCurrentCUDAStream()));
}

// Query (mode < 0) or set which kernel latent_decode runs where the sizes
// fit: 1 = tcgen05, 0 = warp-level mma.sync, 2 = by latent rank (default).
// Returns the previous mode.
int64_t decode_tc(int64_t mode) {
  const int prev = latent_tc_mode();
  if (mode >= 0) latent_tc_mode() = mode > 2 ? 2 : (int)mode;
  return prev;
}

// The tcgen05 forward (attention_sm100.cuh).  Same contract as flash_fwd.
void flash_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                  int64_t q_off, double scale, bool causal, int64_t H) {
  const at::cuda::CUDAGuard guard(q.device());
  const int dqk = q.size(2), dvv = v.size(2);
  DSV3_FA_DISPATCH(80, 64, (run_fwd_sm100<1, 1, 64>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(64, 64, (run_fwd_sm100<1, 0, 64>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(128, 128, (run_fwd_sm100<2, 0, 128>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(192, 128, (run_fwd_sm100<3, 0, 128>(q, k, v, o, lse, q_off, scale, causal, H)))
  TORCH_CHECK(false, "flash_fwd_tc: unsupported head dims");
}

// The warp-level (mma.sync) backward, kept callable for comparison tests.
void flash_bwd_mma(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                   const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq, at::Tensor& dk,
                   at::Tensor& dv, int64_t q_off, double scale, bool causal, int64_t H) {
  const at::cuda::CUDAGuard guard(q.device());
  const int dqk = q.size(2), dvv = v.size(2);
  DSV3_FA_DISPATCH(80, 64, (run_bwd<80, 64>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(64, 64, (run_bwd<64, 64>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale, causal, H)))
  TORCH_CHECK(false, "flash_bwd_mma: unsupported head dims");
}

// The two-kernel tcgen05 backward for qk 128 / 192 with v 128 (and the 412M
// head dims 80 / 64 for comparison with the single-kernel backward), callable
// directly; flash_bwd selects it for qk 128 / 192 only with
// DSV3_FA_BWD_WIDE=1.  dq is overwritten, not accumulated.
void flash_bwd_wide(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                    const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq, at::Tensor& dk,
                    at::Tensor& dv, int64_t q_off, double scale, bool causal, int64_t H) {
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && dout.is_contiguous(),
              "flash_bwd_wide: contiguous inputs");
  const at::cuda::CUDAGuard guard(q.device());
  const int dqk = q.size(2), dvv = v.size(2);
  DSV3_FA_DISPATCH(192, 128, (run_bwd_sm100_wide<3, 0, 128>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale,
                                                         causal, H)))
  DSV3_FA_DISPATCH(128, 128, (run_bwd_sm100_wide<2, 0, 128>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale,
                                                         causal, H)))
  DSV3_FA_DISPATCH(80, 64, (run_bwd_sm100_wide<1, 1, 64>(q, k, v, o, dout, lse, delta, dq, dk, dv, q_off, scale,
                                                        causal, H)))
  TORCH_CHECK(false, "flash_bwd_wide: unsupported head dims ", dqk, "/", dvv);
}

// The warp-level (mma.sync) forward, kept callable for comparison tests.
void flash_fwd_mma(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                   int64_t q_off, double scale, bool causal, int64_t H) {
  const at::cuda::CUDAGuard guard(q.device());
  const int dqk = q.size(2), dvv = v.size(2);
  DSV3_FA_DISPATCH(80, 64, (run_fwd<80, 64>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(64, 64, (run_fwd<64, 64>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(128, 128, (run_fwd<128, 128>(q, k, v, o, lse, q_off, scale, causal, H)))
  DSV3_FA_DISPATCH(192, 128, (run_fwd<192, 128>(q, k, v, o, lse, q_off, scale, causal, H)))
  TORCH_CHECK(false, "flash_fwd_mma: unsupported head dims");
}

void register_attention(pybind11::module_& m) {
  m.def("flash_fwd_mma", &flash_fwd_mma, "warp-level mma.sync flash attention forward");
  m.def("flash_fwd_tc", &flash_fwd_tc, "tcgen05 flash attention forward");
  m.def("flash_bwd_mma", &flash_bwd_mma, "warp-level mma.sync flash attention backward");
  m.def("flash_bwd_wide", &flash_bwd_wide, "two-kernel tcgen05 flash attention backward (qk 192/128/80)");
  m.def("flash_fwd", &flash_fwd, "causal flash attention forward (stores log2-domain LSE)");
  m.def("flash_bwd", &flash_bwd, "flash attention backward (dQ fp32 accumulated, dK/dV fp32)");
  m.def("latent_decode", &latent_decode, "absorbed MLA decode over the latent cache (split-K)", pybind11::arg("q_lat"),
        pybind11::arg("q_pe"), pybind11::arg("kv"), pybind11::arg("pe"), pybind11::arg("lens"), pybind11::arg("scale"),
        pybind11::arg("max_len"), pybind11::arg("scratch"), pybind11::arg("out"), pybind11::arg("qpb") = 1);
  m.def("decode_tc", &decode_tc, "query (-1) or set the latent-decode kernel (0 mma.sync, 1 tcgen05, 2 by rank); returns the previous mode");
}

}  // namespace dsv3
