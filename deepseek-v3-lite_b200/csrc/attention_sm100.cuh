// Flash-attention forward on the 5th-generation tensor cores (tcgen05).
//
// One CTA per (128-query tile, batch*head).  Warp 0 streams K and V tiles of
// 128 keys with TMA (lane 0: Q once, then K; lane 1: V; separate rings so K_{j+1}
// streams in while V_j is in use), warp 1 issues the MMAs from one thread,
// and WG softmax warpgroups own the query rows: with WG = 1 warps 2-5 take a
// whole row of S per thread; with WG = 2 warps 2-5 take key columns 0-63 and
// warps 6-9 columns 64-127 of the same rows (two softmax warps per SM
// sub-partition, half the registers and exponentials per thread), and the
// two halves of a row agree on its running max through shared memory and a
// bounded mbarrier per 32-row quarter:
//
//   S_j   = Q K_j^T          tcgen05.mma, M=128, N=128, fp32 in TMEM (2 buffers)
//   P_j   = exp2(S_j * c - m) softmax threads: tcgen05.ld a whole row of S,
//                            row max / sum in registers (no shuffles), P
//                            written to shared memory in the 128B-swizzled
//                            K-major layout the next MMA reads
//   O    += P_j V_j          tcgen05.mma, M=128, N=DV, V read MN-major
//
// S_{j+1} is issued while the softmax threads work on S_j.  The running max is
// only moved (and O in TMEM rescaled through tcgen05.ld/st) when it grows by
// more than 2^8; otherwise P is computed against the stale max, which keeps P
// below 256 and leaves the final O / l exact.
//
// Head dimension DQK = 64 * NA + 16 * NB: NA 128B-swizzled blocks of 64 plus
// an optional 32B-swizzled block of 16 (so 72 = 48 + 24 pads only to 80).
// Output O is token-major [B, S, H, DV]; L[bh, q] = m + log2(l) (log2 domain),
// the same contract as the mma.sync kernels it replaces.
#pragma once

#include "common.cuh"

namespace dsv3 {

template <int NA, int NB, int DV>
struct FaCfg {
  static constexpr int QA_B = NA * 16384;
  static constexpr int QB_B = NB * 4096;
  static constexpr int Q_B = QA_B + QB_B;
  static constexpr int K_B = Q_B;
  static constexpr int V_B = (DV / 64) * 16384;
  // K and V rings (separate barriers, so K_{j+1} streams in while V_j is
  // still in use); one stage each for wide heads (DQK 192) to fit smem
  static constexpr int ST = NA >= 3 ? 1 : 2;
  static constexpr int P_B = 32768;
  static constexpr int OFF_K = Q_B;
  static constexpr int OFF_V = OFF_K + ST * K_B;
  static constexpr int OFF_P = OFF_V + ST * V_B;
  static constexpr int OFF_BAR = OFF_P + 2 * P_B;
  // row-max / row-sum exchange [2][2][128] f32 of the two-warpgroup softmax,
  // where it fits next to the rings (not at qk 128 / v 128)
  static constexpr int XR_B = OFF_BAR + 256 + 2048 + 1024 <= 232448 ? 2048 : 0;
  static constexpr int OFF_XR = OFF_BAR + 256;
  static constexpr int SMEM = OFF_XR + XR_B + 1024;
};

// Causal grids: `causal` (nonzero) is the number of (batch, head) rows per
// group.  Groups run one after another; inside a group tiles run heaviest
// first across its rows (longest-processing-time order, so each group ends
// on its shortest CTAs) while the group's K/V (or Q/dO) rows stay in L2.
// Linear block L: group g = L / (G * T), then tile rank r / rows_g (0 =
// heaviest) and row g * G + r % rows_g.  Non-causal grids keep
// (blockIdx.x, blockIdx.y).
__device__ __forceinline__ void fa_tile_order(int causal, bool heavy_last_index, int& tile, int& bh) {
  tile = blockIdx.x;
  bh = blockIdx.y;
  if (causal > 0) {
    const int T = gridDim.x, BH = gridDim.y, G = causal;
    const int L = blockIdx.x + blockIdx.y * T;
    const int g = L / (G * T), r = L - g * G * T;
    const int rows = min(G, BH - g * G);
    const int rank = r / rows;
    tile = heavy_last_index ? T - 1 - rank : rank;
    bh = g * G + r % rows;
  }
}

template <int NA, int NB, int DV, int WG = 1>
__global__ void __launch_bounds__(64 + 128 * WG, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQa, const __grid_constant__ CUtensorMap tmQb,
                        const __grid_constant__ CUtensorMap tmKa, const __grid_constant__ CUtensorMap tmKb,
                        const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O,
                        float* __restrict__ L, int Sq, int Sk, int H, int q_off, float scale_log2, int causal,
                        unsigned int* status) {
  using C = FaCfg<NA, NB, DV>;
  static_assert(DV % 64 == 0 && DV <= 128, "DV must be 64 or 128");
  static_assert(WG == 1 || C::XR_B > 0, "two softmax warpgroups need the exchange buffer");
  extern __shared__ __align__(1024) uint8_t fa_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint8_t* sP = smem + C::OFF_P;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;    // [ST]
  uint64_t* k_empty = bar + 3;   // [ST]
  uint64_t* v_full = bar + 5;    // [ST]
  uint64_t* v_empty = bar + 7;   // [ST]
  uint64_t* s_full = bar + 9;    // [2]
  uint64_t* s_free = bar + 11;   // [2]
  uint64_t* p_full = bar + 13;   // [2]
  uint64_t* pv_done = bar + 15;  // [2]
  uint64_t* drain = bar + 17;
  uint64_t* xchg = bar + 18;     // [4] row-max exchange between the two halves of a row quarter (WG = 2)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xr = reinterpret_cast<float*>(smem + C::OFF_XR);   // [2 parities][2 halves][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int q_tile, bh;
  fa_tile_order(causal, true, q_tile, bh);   // later query tiles see more keys
  const int m0 = q_tile * 128;
  int n_blocks = (Sk + 127) / 128;
  if (causal) n_blocks = min(n_blocks, (q_off + m0 + 128 + 127) / 128);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128 * WG);
      mbar_init(&p_full[i], 128 * WG);
      mbar_init(&pv_done[i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&xchg[i], 64);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ producer: Q and K
      mbar_arrive_expect_tx(q_full, C::Q_B);
#pragma unroll
      for (int a = 0; a < NA; ++a) tma_load_3d(sQ + a * 16384, &tmQa, q_full, a * 64, m0, bh);
      if (NB) tma_load_3d(sQ + C::QA_B, &tmQb, q_full, NA * 64, m0, bh);
      uint32_t issued = 0, last_phase = 0;
      for (int j = 0; j < n_blocks; ++j) {
        const int st = j % C::ST;
        const uint32_t ph = (j / C::ST) & 1;
        if (!mbar_wait_bounded(&k_empty[st], ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&k_full[st], C::K_B);
        uint8_t* k = sK + st * C::K_B;
#pragma unroll
        for (int a = 0; a < NA; ++a) tma_load_3d(k + a * 16384, &tmKa, &k_full[st], a * 64, j * 128, bh);
        if (NB) tma_load_3d(k + C::QA_B, &tmKb, &k_full[st], NA * 64, j * 128, bh);
        issued |= 1u << st;
        last_phase = (last_phase & ~(1u << st)) | (ph << st);
      }
      mbar_wait_bounded(q_full, 0, nullptr, status, DSV3_ERR_WAIT_FULL);
      for (int st = 0; st < C::ST; ++st)
        if (issued & (1u << st)) mbar_wait_bounded(&k_full[st], (last_phase >> st) & 1u, nullptr, status, DSV3_ERR_WAIT_FULL);
    } else if (lane == 1) {
      // ------------------------------------------------------ producer: V
      uint32_t issued = 0, last_phase = 0;
      for (int j = 0; j < n_blocks; ++j) {
        const int st = j % C::ST;
        const uint32_t ph = (j / C::ST) & 1;
        if (!mbar_wait_bounded(&v_empty[st], ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&v_full[st], C::V_B);
        uint8_t* v = sV + st * C::V_B;
#pragma unroll
        for (int d = 0; d < DV / 64; ++d) tma_load_3d(v + d * 16384, &tmV, &v_full[st], d * 64, j * 128, bh);
        issued |= 1u << st;
        last_phase = (last_phase & ~(1u << st)) | (ph << st);
      }
      for (int st = 0; st < C::ST; ++st)
        if (issued & (1u << st)) mbar_wait_bounded(&v_full[st], (last_phase >> st) & 1u, nullptr, status, DSV3_ERR_WAIT_FULL);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      constexpr uint32_t IDS = idesc_bf16_f32(128, 128, 0, 0);
      constexpr uint32_t IDO = idesc_bf16_f32(128, DV, 0, 1);
      const uint32_t tO = tmem + 256;
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, status, DSV3_ERR_WAIT_FULL);
      bool any = false;
      for (int j = 0; ok && j <= n_blocks; ++j) {
        if (j < n_blocks) {
          const int st = j % C::ST, sb = j & 1;
          if (!mbar_wait_bounded(&k_full[st], (j / C::ST) & 1, abort_flag, status, DSV3_ERR_WAIT_FULL)) break;
          if (j >= 2 && !mbar_wait_bounded(&s_free[sb], ((j - 2) >> 1) & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM))
            break;
          tc_fence_after();
          const uint32_t q = smem_u32(sQ), k = smem_u32(sK + st * C::K_B);
          uint32_t acc = 0;
#pragma unroll
          for (int a = 0; a < NA; ++a)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              umma_bf16(tmem + sb * 128, smem_desc_sw128(q + a * 16384 + kk * 32, 16, 1024),
                        smem_desc_sw128(k + a * 16384 + kk * 32, 16, 1024), IDS, acc);
              acc = 1;
            }
          if (NB) umma_bf16(tmem + sb * 128, smem_desc_sw32(q + C::QA_B, 256), smem_desc_sw32(k + C::QA_B, 256), IDS, acc);
          umma_commit(&s_full[sb]);
          umma_commit(&k_empty[st]);   // K_j is free once S_j is computed
          any = true;
        }
        if (j >= 1) {
          const int pj = j - 1, pb = pj & 1;
          if (!mbar_wait_bounded(&p_full[pb], (pj >> 1) & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM)) break;
          if (!mbar_wait_bounded(&v_full[pj % C::ST], (pj / C::ST) & 1, abort_flag, status, DSV3_ERR_WAIT_FULL)) break;
          tc_fence_after();
          const uint32_t p = smem_u32(sP + pb * C::P_B), v = smem_u32(sV + (pj % C::ST) * C::V_B);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tO, smem_desc_sw128(p + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                      smem_desc_sw128(v + kk * 2048, 16384, 1024), IDO, (pj > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&pv_done[pb]);
          umma_commit(&v_empty[pj % C::ST]);
        }
      }
      if (any) {
        umma_commit(drain);
        mbar_wait_bounded(drain, 0, nullptr, status, DSV3_ERR_WAIT_TMEM);
      }
    }
  } else {
    // ----------------------------------------------- softmax / epilogue
    // WG = 1: one thread per query row, all 128 key columns of S.
    // WG = 2: half h of the row's key columns (64 * h ..), O columns DV/2 * h ..
    constexpr int NC = 128 / WG;                       // key columns per thread
    constexpr int OC = DV / WG;                        // O columns per thread
    const int quarter = warp & 3;
    const int half = WG == 2 ? (warp - 2) >> 2 : 0;
    const int row = quarter * 32 + lane;
    const int qrow = m0 + row;
    const int qpos = q_off + qrow;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tO = tmem + lane_base + 256 + half * OC;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_blocks && ok; ++j) {
      const int sb = j & 1;
      // Waits are made warp-uniform: the TMEM loads/stores below are
      // warp-collective and must never run with part of the warp gone.
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[sb], (j >> 1) & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[NC];
      {
        uint32_t raw[NC / 16][16];
#pragma unroll
        for (int c = 0; c < NC / 16; ++c) tmem_ld16(tmem + lane_base + sb * 128 + half * NC + c * 16, raw[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < NC / 16; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) s[c * 16 + e] = __uint_as_float(raw[c][e]);
      }
      tc_fence_before();
      mbar_arrive(&s_free[sb]);
      const int n0 = j * 128 + half * NC;
      // keys < lim are visible to this row (causal by global position, and < Sk)
      const int lim = causal ? min(Sk, qpos + 1) - n0 : Sk - n0;
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const float v = c < lim ? s[c] * scale_log2 : -INFINITY;
        s[c] = v;
        mx4[c & 3] = fmaxf(mx4[c & 3], v);
      }
      float rmax = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      if constexpr (WG == 2) {
        // the other half's maximum of this row (double-buffered by tile parity)
        xr[((j & 1) * 2 + half) * 128 + row] = rmax;
        mbar_arrive(&xchg[quarter]);
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&xchg[quarter], j & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
          ok = false;
          break;
        }
        rmax = fmaxf(rmax, xr[((j & 1) * 2 + (half ^ 1)) * 128 + row]);
      }
      const float m_new = fmaxf(m_used, rmax);
      if (j == 0) {
        m_used = m_new;
      } else if (__any_sync(0xffffffffu, m_new > m_used + 8.0f)) {
        // Some row of this warp moved its max by more than 2^8: rescale the
        // warp's rows of O (warp-uniform; rows that did not move get a factor
        // <= 1 as well, which is always valid; both halves of a row see the
        // same maxima and decide alike).  O must not be read before PV_{j-1}
        // has finished writing it.
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, status,
                                                        DSV3_ERR_WAIT_TMEM))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float corr = m_used == -INFINITY ? 0.f : ex2_approx(m_used - m_new);
        l *= corr;
#pragma unroll
        for (int d = 0; d < OC / 16; ++d) {
          uint32_t r[16];
          tmem_ld16(tO + d * 16, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * corr);
          tmem_st16(tO + d * 16, r);
        }
        tmem_st_wait();
        m_used = m_new;
      }
      // The P buffer being written was last read by PV_{j-2}.
      if (j >= 2 &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(&pv_done[sb], ((j - 2) >> 1) & 1, abort_flag, status,
                                                     DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      // this thread's key columns are 16-byte chunks [NC/8 * half, ..) of the row, 64 keys per 16 KB block
      uint8_t* prow = sP + sb * C::P_B + row * 128;
      // m_used == -inf only if every key so far is masked; then s is -inf too and 2^(s - 0) = 0.
      const float msub = m_used == -INFINITY ? 0.f : m_used;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < NC / 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = ex2_approx(s[c * 8 + 2 * e] - msub);
          const float p1 = ex2_approx(s[c * 8 + 2 * e + 1] - msub);
          rs4[e] += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
        const int gc = half * (NC / 8) + c;            // chunk index within the row
        const int blk = gc >> 3, cc = gc & 7;
        *reinterpret_cast<uint4*>(prow + blk * 16384 + ((cc ^ (row & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      const float rs = (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      l += rs;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    if constexpr (WG == 2) {
      // row sum = both halves' sums (one more exchange phase)
      if (ok && n_blocks > 0) {
        xr[((n_blocks & 1) * 2 + half) * 128 + row] = l;
        mbar_arrive(&xchg[quarter]);
        if (__all_sync(0xffffffffu, mbar_wait_bounded(&xchg[quarter], n_blocks & 1, abort_flag, status,
                                                       DSV3_ERR_WAIT_TMEM)))
          l += xr[((n_blocks & 1) * 2 + (half ^ 1)) * 128 + row];
        else
          ok = false;
      }
    }
    if (ok && n_blocks > 0 &&
        __all_sync(0xffffffffu, mbar_wait_bounded(&pv_done[(n_blocks - 1) & 1], ((n_blocks - 1) >> 1) & 1, abort_flag,
                                                  status, DSV3_ERR_WAIT_TMEM))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int b = bh / H, h = bh % H;
      __nv_bfloat16* orow = O + (((size_t)b * Sq + qrow) * H + h) * DV + half * OC;
#pragma unroll
      for (int d = 0; d < OC / 16; ++d) {
        uint32_t r[16];
        tmem_ld16(tO + d * 16, r);
        tmem_ld_wait();
        if (qrow < Sq) {
          uint32_t pk[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) pk[e] = pack_bf16x2(__uint_as_float(r[2 * e]) * inv, __uint_as_float(r[2 * e + 1]) * inv);
          reinterpret_cast<uint4*>(orow + d * 16)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          reinterpret_cast<uint4*>(orow + d * 16)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      if (qrow < Sq && half == 0) L[(size_t)bh * Sq + qrow] = l > 0.f ? m_used + log2f(l) : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace dsv3

namespace dsv3 {

// ----------------------------------------------------------------------------
// Forward with two query tiles per CTA (qk up to 80, v 64).  Tiles A (rows
// m0..m0+127) and B (m0+128..m0+255) of the same head share every K / V tile
// brought in by TMA; warps 2-5 run tile A's softmax and warps 6-9 tile B's,
// two independent chains, so while one waits on its TMEM loads or barriers
// the other issues.  TMEM: S_A, S_B (128 columns each, one buffer per tile:
// S_t(j+1) is written once the tile's softmax holds S_t(j) in registers),
// O_A, O_B (DV each).  P_A, P_B: one 32 KB shared tile each (P_t(j) is
// written once PV_t(j-1) has read P_t(j-1)).  The MMA thread issues, per KV
// tile j, S_A(j) and S_B(j), then PV_A(j-1) and PV_B(j-1).  Under the causal
// mask tile B sees one more KV tile than A.
// ----------------------------------------------------------------------------
template <int NA, int NB, int DV>
struct Fa2Cfg {
  static constexpr int Q_B = NA * 16384 + NB * 4096;
  static constexpr int K_B = Q_B;
  static constexpr int V_B = (DV / 64) * 16384;
  static constexpr int P_B = 32768;
  static constexpr int OFF_K = 2 * Q_B;
  static constexpr int OFF_V = OFF_K + 2 * K_B;
  static constexpr int OFF_P = OFF_V + 2 * V_B;
  static constexpr int OFF_BAR = OFF_P + 2 * P_B;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr bool FITS = SMEM <= 232448 && DV == 64 && NA == 1;
};

template <int NA, int NB, int DV>
__global__ void __launch_bounds__(320, 1)
    fa_fwd2q_sm100_kernel(const __grid_constant__ CUtensorMap tmQa, const __grid_constant__ CUtensorMap tmQb,
                          const __grid_constant__ CUtensorMap tmKa, const __grid_constant__ CUtensorMap tmKb,
                          const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O,
                          float* __restrict__ L, int Sq, int Sk, int H, int q_off, float scale_log2, int causal,
                          unsigned int* status) {
  using C = Fa2Cfg<NA, NB, DV>;
  static_assert(C::FITS, "two-tile forward: qk <= 80, v 64");
  extern __shared__ __align__(1024) uint8_t fa2_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa2_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint8_t* sP = smem + C::OFF_P;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;    // [2]
  uint64_t* k_empty = bar + 3;   // [2]
  uint64_t* v_full = bar + 5;    // [2]
  uint64_t* v_empty = bar + 7;   // [2]
  uint64_t* s_full = bar + 9;    // [tile]
  uint64_t* s_free = bar + 11;   // [tile]
  uint64_t* p_full = bar + 13;   // [tile]
  uint64_t* pv_done = bar + 15;  // [tile]
  uint64_t* drain = bar + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int q_tile, bh;
  fa_tile_order(causal, true, q_tile, bh);   // later query tiles see more keys
  const int m0 = q_tile * 256;
  const int nk = (Sk + 127) / 128;
  // KV tiles each query tile attends to (0 when the tile lies past Sq)
  int nt[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int mt = m0 + 128 * t;
    nt[t] = mt >= Sq ? 0 : (causal ? min(nk, (q_off + mt + 128 + 127) / 128) : nk);
  }
  const int n_all = max(nt[0], nt[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------- producer: Q_A, Q_B, then K
      const int nq = nt[1] > 0 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, nq * C::Q_B);
      for (int t = 0; t < nq; ++t) {
#pragma unroll
        for (int a = 0; a < NA; ++a) tma_load_3d(smem + t * C::Q_B + a * 16384, &tmQa, q_full, a * 64, m0 + 128 * t, bh);
        if (NB) tma_load_3d(smem + t * C::Q_B + NA * 16384, &tmQb, q_full, NA * 64, m0 + 128 * t, bh);
      }
      uint32_t issued = 0, last_phase = 0;
      for (int j = 0; j < n_all; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_bounded(&k_empty[st], ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&k_full[st], C::K_B);
        uint8_t* k = sK + st * C::K_B;
#pragma unroll
        for (int a = 0; a < NA; ++a) tma_load_3d(k + a * 16384, &tmKa, &k_full[st], a * 64, j * 128, bh);
        if (NB) tma_load_3d(k + NA * 16384, &tmKb, &k_full[st], NA * 64, j * 128, bh);
        issued |= 1u << st;
        last_phase = (last_phase & ~(1u << st)) | (ph << st);
      }
      mbar_wait_bounded(q_full, 0, nullptr, status, DSV3_ERR_WAIT_FULL);
      for (int st = 0; st < 2; ++st)
        if (issued & (1u << st)) mbar_wait_bounded(&k_full[st], (last_phase >> st) & 1u, nullptr, status, DSV3_ERR_WAIT_FULL);
    } else if (lane == 1) {
      // -------------------------------------------------------- producer: V
      uint32_t issued = 0, last_phase = 0;
      for (int j = 0; j < n_all; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_bounded(&v_empty[st], ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&v_full[st], C::V_B);
        uint8_t* v = sV + st * C::V_B;
#pragma unroll
        for (int d = 0; d < DV / 64; ++d) tma_load_3d(v + d * 16384, &tmV, &v_full[st], d * 64, j * 128, bh);
        issued |= 1u << st;
        last_phase = (last_phase & ~(1u << st)) | (ph << st);
      }
      for (int st = 0; st < 2; ++st)
        if (issued & (1u << st)) mbar_wait_bounded(&v_full[st], (last_phase >> st) & 1u, nullptr, status, DSV3_ERR_WAIT_FULL);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      constexpr uint32_t IDS = idesc_bf16_f32(128, 128, 0, 0);
      constexpr uint32_t IDO = idesc_bf16_f32(128, DV, 0, 1);
      bool ok = n_all > 0 && mbar_wait_bounded(q_full, 0, abort_flag, status, DSV3_ERR_WAIT_FULL);
      bool any = false;
      for (int j = 0; ok && j <= n_all; ++j) {
        if (j < n_all) {
          const int st = j & 1;
          if (!mbar_wait_bounded(&k_full[st], (j >> 1) & 1, abort_flag, status, DSV3_ERR_WAIT_FULL)) break;
          const uint32_t k = smem_u32(sK + st * C::K_B);
          for (int t = 0; t < 2 && ok; ++t) {
            if (j >= nt[t]) continue;
            // the tile's only S buffer is free once its softmax loaded S_t(j-1)
            if (j >= 1 && !mbar_wait_bounded(&s_free[t], (j - 1) & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t q = smem_u32(smem + t * C::Q_B);
            uint32_t acc = 0;
#pragma unroll
            for (int a = 0; a < NA; ++a)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                umma_bf16(tmem + t * 128, smem_desc_sw128(q + a * 16384 + kk * 32, 16, 1024),
                          smem_desc_sw128(k + a * 16384 + kk * 32, 16, 1024), IDS, acc);
                acc = 1;
              }
            if (NB) umma_bf16(tmem + t * 128, smem_desc_sw32(q + NA * 16384, 256), smem_desc_sw32(k + NA * 16384, 256),
                              IDS, acc);
            umma_commit(&s_full[t]);
            any = true;
          }
          if (!ok) break;
          umma_commit(&k_empty[st]);   // K_j is free once every S of tile j is computed
        }
        if (j >= 1) {
          const int pj = j - 1, vs = pj & 1;
          if (!mbar_wait_bounded(&v_full[vs], (pj >> 1) & 1, abort_flag, status, DSV3_ERR_WAIT_FULL)) break;
          const uint32_t v = smem_u32(sV + vs * C::V_B);
          for (int t = 0; t < 2 && ok; ++t) {
            if (pj >= nt[t]) continue;
            if (!mbar_wait_bounded(&p_full[t], pj & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t pp = smem_u32(sP + t * C::P_B);
            const uint32_t tO = tmem + 256 + t * DV;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_bf16(tO, smem_desc_sw128(pp + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                        smem_desc_sw128(v + kk * 2048, 16384, 1024), IDO, (pj > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&pv_done[t]);
          }
          if (!ok) break;
          umma_commit(&v_empty[vs]);
        }
      }
      if (any) {
        umma_commit(drain);
        mbar_wait_bounded(drain, 0, nullptr, status, DSV3_ERR_WAIT_TMEM);
      }
    }
  } else {
    // ---------------------------------------- softmax / epilogue of tile t
    const int t = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qrow = m0 + 128 * t + row;
    const int qpos = q_off + qrow;
    const int n_blocks = nt[t];
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_base + t * 128;
    const uint32_t tO = tmem + lane_base + 256 + t * DV;
    uint8_t* prow = sP + t * C::P_B + row * 128;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_blocks && ok; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[t], j & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
      {
        uint32_t raw[8][16];
#pragma unroll
        for (int c = 0; c < 8; ++c) tmem_ld16(tS + c * 16, raw[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 8; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) s[c * 16 + e] = __uint_as_float(raw[c][e]);
      }
      tc_fence_before();
      mbar_arrive(&s_free[t]);
      const int n0 = j * 128;
      const int lim = causal ? min(Sk, qpos + 1) - n0 : Sk - n0;
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        const float v = c < lim ? s[c] * scale_log2 : -INFINITY;
        s[c] = v;
        mx4[c & 3] = fmaxf(mx4[c & 3], v);
      }
      const float rmax = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      const float m_new = fmaxf(m_used, rmax);
      // PV_t(j-1) must have read P_t(j-1) (single buffer) and written O_t
      // before this tile rescales O_t or overwrites P_t.
      if (j >= 1 && !__all_sync(0xffffffffu, mbar_wait_bounded(&pv_done[t], (j - 1) & 1, abort_flag, status,
                                                                DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      if (j == 0) {
        m_used = m_new;
      } else if (__any_sync(0xffffffffu, m_new > m_used + 8.0f)) {
        tc_fence_after();
        const float corr = m_used == -INFINITY ? 0.f : ex2_approx(m_used - m_new);
        l *= corr;
#pragma unroll
        for (int d = 0; d < DV / 16; ++d) {
          uint32_t r[16];
          tmem_ld16(tO + d * 16, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * corr);
          tmem_st16(tO + d * 16, r);
        }
        tmem_st_wait();
        m_used = m_new;
      }
      const float msub = m_used == -INFINITY ? 0.f : m_used;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = ex2_approx(s[c * 8 + 2 * e] - msub);
          const float p1 = ex2_approx(s[c * 8 + 2 * e + 1] - msub);
          rs4[e] += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
        const int blk = c >> 3, cc = c & 7;
        *reinterpret_cast<uint4*>(prow + blk * 16384 + ((cc ^ (row & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (ok && n_blocks > 0 &&
        __all_sync(0xffffffffu, mbar_wait_bounded(&pv_done[t], (n_blocks - 1) & 1, abort_flag, status,
                                                  DSV3_ERR_WAIT_TMEM))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int b = bh / H, h = bh % H;
      __nv_bfloat16* orow = O + (((size_t)b * Sq + qrow) * H + h) * DV;
#pragma unroll
      for (int d = 0; d < DV / 16; ++d) {
        uint32_t r[16];
        tmem_ld16(tO + d * 16, r);
        tmem_ld_wait();
        if (qrow < Sq) {
          uint32_t pk[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) pk[e] = pack_bf16x2(__uint_as_float(r[2 * e]) * inv, __uint_as_float(r[2 * e + 1]) * inv);
          reinterpret_cast<uint4*>(orow + d * 16)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          reinterpret_cast<uint4*>(orow + d * 16)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      if (qrow < Sq) L[(size_t)bh * Sq + qrow] = l > 0.f ? m_used + log2f(l) : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------
// Flash-attention backward on tcgen05.  One CTA per (128-key tile, b*h); it
// walks the query tiles that can see its keys (causal) and keeps dK / dV for
// its keys in TMEM:
//
//   S^T  = K Q_i^T      dP^T = V dO_i^T                  (TMEM, 128 x 128 each)
//   P^T  = exp2(S^T c - L[q]),  dS^T = P^T (dP^T - delta[q])   (softmax warps,
//          one key row per thread, written to smem as bf16 K-major tiles)
//   dV  += P^T dO_i     dK += dS^T Q_i                   (TMEM accumulators)
//   dQ_i = dS K          -> TMEM, drained with fp32 vector reductions into
//                           the global dQ: by the softmax warps after they
//                           hand tile i+1 to the MMA warp (DRAIN = 0), or by
//                           four dedicated drain warps that run beside the
//                           softmax of the next tile (DRAIN = 1)
//
// Q_i / K are used both K-major (for S^T) and MN-major (for dK / dQ): a
// 128-row tile of 64 (or 16) head-dim columns in 128B (32B) swizzle is the
// canonical layout of either role.  TMEM: S^T 128 + dP^T 128 + dV DV +
// dK DQK + dQ DQK columns (<= 512 for DQK = 80, DV = 64).
// ----------------------------------------------------------------------------
template <int NA, int NB, int DV>
struct FabCfg {
  static constexpr int DQK = NA * 64 + NB * 16;
  static constexpr int T_B = NA * 16384 + NB * 4096;  // one 128-row Q or K tile
  static constexpr int V_B = (DV / 64) * 16384;       // one 128-row V or dO tile
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + T_B;
  static constexpr int OFF_Q = OFF_V + V_B;             // 2 stages
  static constexpr int OFF_DO = OFF_Q + 2 * T_B;        // 2 stages
  static constexpr int OFF_P = OFF_DO + 2 * V_B;        // P^T [128 keys][128 q]
  static constexpr int OFF_DS = OFF_P + 32768;          // dS^T
  static constexpr int OFF_LD = OFF_DS + 32768;         // L / delta, 2 buffers x 2 x 128 floats
  static constexpr int OFF_BAR = OFF_LD + 2048;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr int DQKP = (DQK + 31) / 32 * 32;   // TMEM regions start on 32-column boundaries
  static constexpr int C_S = 0, C_DP = 128, C_DV = 256, C_DK = 256 + DV, C_DQ = 256 + DV + DQKP;
  static_assert(C_DQ + DQKP <= 512, "TMEM budget");
};

template <int NA, int NB, int DV, int DRAIN = 0>
__global__ void __launch_bounds__(320 + 128 * DRAIN, 1)
    fa_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQa, const __grid_constant__ CUtensorMap tmQb,
                        const __grid_constant__ CUtensorMap tmKa, const __grid_constant__ CUtensorMap tmKb,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                        const float* __restrict__ L, const float* __restrict__ delta, float* __restrict__ dQ,
                        float* __restrict__ dK, float* __restrict__ dVo, int Sq, int Sk, int H, int q_off,
                        float scale_log2, float scale, int causal, unsigned int* status) {
  using C = FabCfg<NA, NB, DV>;
  constexpr int DQK = C::DQK;
  extern __shared__ __align__(1024) uint8_t fab_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fab_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* kv_full = bar;        // K, V loaded
  uint64_t* qd_full = bar + 1;    // [2] Q_i, dO_i loaded
  uint64_t* qd_empty = bar + 3;   // [2]
  uint64_t* s_full = bar + 5;     // S^T, dP^T ready
  uint64_t* s_free = bar + 6;     // softmax has them in registers
  uint64_t* p_full = bar + 7;     // P^T, dS^T written
  uint64_t* p_free = bar + 8;     // MMAs reading P^T, dS^T done
  uint64_t* dq_full = bar + 9;
  uint64_t* dq_free = bar + 10;
  uint64_t* acc_done = bar + 11;  // final dK, dV in TMEM
  uint64_t* ld_ready = bar + 12;  // L / delta of the query tile staged
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sLD = reinterpret_cast<float*>(smem + C::OFF_LD);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int k_tile, bh;
  fa_tile_order(causal, false, k_tile, bh);  // earlier key tiles are seen by more queries
  const int n0 = k_tile * 128;
  const int b = bh / H, h = bh % H;
  const int qstart = causal ? max(0, (n0 - q_off) / 128) : 0;
  const int nq = (Sq + 127) / 128;
  const int iters = max(0, nq - qstart);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(p_full, 256);
    mbar_init(p_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, DRAIN ? 128 : 256);
    mbar_init(acc_done, 1);
    mbar_init(ld_ready, 128);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // -------------------------------------------------------- producer
      mbar_arrive_expect_tx(kv_full, C::T_B + C::V_B);
#pragma unroll
      for (int a = 0; a < NA; ++a) tma_load_3d(smem + C::OFF_K + a * 16384, &tmKa, kv_full, a * 64, n0, bh);
      if (NB) tma_load_3d(smem + C::OFF_K + NA * 16384, &tmKb, kv_full, NA * 64, n0, bh);
#pragma unroll
      for (int d = 0; d < DV / 64; ++d) tma_load_3d(smem + C::OFF_V + d * 16384, &tmV, kv_full, d * 64, n0, bh);
      uint32_t issued = 0, last_phase = 0;
      for (int it = 0; it < iters; ++it) {
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        const int q0 = (qstart + it) * 128;
        if (!mbar_wait_bounded(&qd_empty[st], ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&qd_full[st], C::T_B + C::V_B);
        uint8_t* q = smem + C::OFF_Q + st * C::T_B;
        uint8_t* o = smem + C::OFF_DO + st * C::V_B;
#pragma unroll
        for (int a = 0; a < NA; ++a) tma_load_3d(q + a * 16384, &tmQa, &qd_full[st], a * 64, q0, bh);
        if (NB) tma_load_3d(q + NA * 16384, &tmQb, &qd_full[st], NA * 64, q0, bh);
#pragma unroll
        for (int d = 0; d < DV / 64; ++d) tma_load_4d(o + d * 16384, &tmdO, &qd_full[st], d * 64, h, q0, b);
        issued |= 1u << st;
        last_phase = (last_phase & ~(1u << st)) | (ph << st);
      }
      mbar_wait_bounded(kv_full, 0, nullptr, status, DSV3_ERR_WAIT_FULL);
      for (int st = 0; st < 2; ++st)
        if (issued & (1u << st)) mbar_wait_bounded(&qd_full[st], (last_phase >> st) & 1u, nullptr, status, DSV3_ERR_WAIT_FULL);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------- MMA issuer
      // Per query tile i: S^T_i, dP^T_i (as soon as the compute warps hold
      // tile i-1's in registers), then dV, dK once P^T_i / dS^T_i are in
      // shared memory, then dQ_i once dQ_{i-1} has been drained.
      constexpr uint32_t I_S = idesc_bf16_f32(128, 128, 0, 0);       // S^T, dP^T
      constexpr uint32_t I_DV = idesc_bf16_f32(128, DV, 0, 1);       // dV += P^T dO
      constexpr uint32_t I_A64 = idesc_bf16_f32(128, 64, 0, 1);      // dK (SW128 part)
      constexpr uint32_t I_A16 = idesc_bf16_f32(128, 16, 0, 1);      // dK (SW32 part)
      constexpr uint32_t I_Q64 = idesc_bf16_f32(128, 64, 1, 1);      // dQ (A = dS, MN-major)
      constexpr uint32_t I_Q16 = idesc_bf16_f32(128, 16, 1, 1);
      const uint32_t k_s = smem_u32(smem + C::OFF_K), v_s = smem_u32(smem + C::OFF_V);
      const uint32_t p_s = smem_u32(smem + C::OFF_P), ds_s = smem_u32(smem + C::OFF_DS);
      auto issue_s_dp = [&](int it) {
        const int st = it & 1;
        const uint32_t q_s = smem_u32(smem + C::OFF_Q + st * C::T_B), o_s = smem_u32(smem + C::OFF_DO + st * C::V_B);
        // S^T = K Q^T
        uint32_t acc = 0;
#pragma unroll
        for (int a = 0; a < NA; ++a)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_bf16(tmem + C::C_S, smem_desc_sw128(k_s + a * 16384 + kk * 32, 16, 1024),
                      smem_desc_sw128(q_s + a * 16384 + kk * 32, 16, 1024), I_S, acc);
            acc = 1;
          }
        if (NB) umma_bf16(tmem + C::C_S, smem_desc_sw32(k_s + NA * 16384, 256), smem_desc_sw32(q_s + NA * 16384, 256), I_S, 1);
        // dP^T = V dO^T
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk)
          umma_bf16(tmem + C::C_DP, smem_desc_sw128(v_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                    smem_desc_sw128(o_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), I_S, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
      };
      bool ok = mbar_wait_bounded(kv_full, 0, abort_flag, status, DSV3_ERR_WAIT_FULL);
      bool any = false;
      if (ok && iters > 0) {
        ok = mbar_wait_bounded(&qd_full[0], 0, abort_flag, status, DSV3_ERR_WAIT_FULL);
        if (ok) {
          tc_fence_after();
          issue_s_dp(0);
          any = true;
        }
      }
      for (int it = 0; ok && it < iters; ++it) {
        const int st = it & 1;
        const uint32_t ph = it & 1;
        if (it + 1 < iters) {
          // S / dP TMEM is free once the compute warps loaded tile it
          if (!mbar_wait_bounded(s_free, ph, abort_flag, status, DSV3_ERR_WAIT_TMEM)) break;
          if (!mbar_wait_bounded(&qd_full[st ^ 1], ((it + 1) >> 1) & 1, abort_flag, status, DSV3_ERR_WAIT_FULL)) break;
          tc_fence_after();
          issue_s_dp(it + 1);
        }
        if (!mbar_wait_bounded(p_full, ph, abort_flag, status, DSV3_ERR_WAIT_TMEM)) break;
        tc_fence_after();
        const uint32_t q_s = smem_u32(smem + C::OFF_Q + st * C::T_B), o_s = smem_u32(smem + C::OFF_DO + st * C::V_B);
        // dV += P^T dO  (K = the 128 queries, 16 per step)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tmem + C::C_DV, smem_desc_sw128(p_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                    smem_desc_sw128(o_s + kk * 2048, 16384, 1024), I_DV, (it > 0 || kk > 0) ? 1u : 0u);
        // dK += dS^T Q   (Q read MN-major: 64-wide SW128 blocks, then the 16-wide SW32 block)
#pragma unroll
        for (int a = 0; a < NA; ++a)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tmem + C::C_DK + a * 64, smem_desc_sw128(ds_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                      smem_desc_sw128(q_s + a * 16384 + kk * 2048, 16384, 1024), I_A64, (it > 0 || kk > 0) ? 1u : 0u);
        if (NB)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tmem + C::C_DK + NA * 64, smem_desc_sw128(ds_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                      smem_desc_sw32(q_s + NA * 16384 + kk * 512, 256), I_A16, (it > 0 || kk > 0) ? 1u : 0u);
        // dQ = dS K (A = dS^T read MN-major; K = the 128 keys) once dQ_{it-1} left TMEM
        if (it > 0 && !mbar_wait_bounded(dq_free, ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_TMEM)) break;
        tc_fence_after();
#pragma unroll
        for (int a = 0; a < NA; ++a)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tmem + C::C_DQ + a * 64, smem_desc_sw128(ds_s + kk * 2048, 16384, 1024),
                      smem_desc_sw128(k_s + a * 16384 + kk * 2048, 16384, 1024), I_Q64, kk > 0 ? 1u : 0u);
        if (NB)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tmem + C::C_DQ + NA * 64, smem_desc_sw128(ds_s + kk * 2048, 16384, 1024),
                      smem_desc_sw32(k_s + NA * 16384 + kk * 512, 256), I_Q16, kk > 0 ? 1u : 0u);
        umma_commit(dq_full);
        umma_commit(p_free);
        umma_commit(&qd_empty[st]);
      }
      if (any) {
        umma_commit(acc_done);
        mbar_wait_bounded(acc_done, 0, nullptr, status, DSV3_ERR_WAIT_TMEM);
      }
    }
  } else if (DRAIN && warp >= 10) {
    // ------------------------------------------- dQ drain (warps 10-13)
    // One query row of dQ_i per thread (TMEM lane = query row), all DQK
    // columns, fp32 vector reductions into the global dQ; then dq_free lets
    // the MMA warp write dQ_{i+1}.
    const int quarter = warp & 3;
    const int qr = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    for (int it = 0; it < iters; ++it) {
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(dq_full, it & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM))) break;
      tc_fence_after();
      const int q = (qstart + it) * 128 + qr;
      float* dqr = dQ + ((size_t)bh * Sq + q) * DQK;
#pragma unroll
      for (int c = 0; c < DQK / 16; ++c) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + C::C_DQ + c * 16, r);
        tmem_ld_wait();
        if (q < Sq)
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dqr + c * 16 + e),
                         "f"(__uint_as_float(r[e]) * scale), "f"(__uint_as_float(r[e + 1]) * scale),
                         "f"(__uint_as_float(r[e + 2]) * scale), "f"(__uint_as_float(r[e + 3]) * scale)
                         : "memory");
      }
      tc_fence_before();
      mbar_arrive(dq_free);
    }
  } else {
    // ---------------------------------------------- compute (key rows)
    // Warps 2-5 and 6-9 share each key row (same TMEM lane quarter): the
    // first group takes query columns 0-63 of S^T / dP^T, the second 64-127.
    // Without drain warps they drain dQ_{i-1} (each group half of its
    // columns) with fp32 vector reductions after handing tile i over.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int kr = quarter * 32 + lane;
    const int key = n0 + kr;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    constexpr int NDQ = DQK / 16;                  // 16-column chunks of dQ / dK
    const int dq_c0 = half ? (NDQ + 1) / 2 : 0, dq_c1 = half ? NDQ : (NDQ + 1) / 2;
    auto drain_dq = [&](int it) {
      const int q = (qstart + it) * 128 + kr;      // TMEM lane = query row of the dQ tile
      float* dqr = dQ + ((size_t)bh * Sq + q) * DQK;
      for (int c = dq_c0; c < dq_c1; ++c) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + C::C_DQ + c * 16, r);
        tmem_ld_wait();
        if (q < Sq)
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dqr + c * 16 + e),
                         "f"(__uint_as_float(r[e]) * scale), "f"(__uint_as_float(r[e + 1]) * scale),
                         "f"(__uint_as_float(r[e + 2]) * scale), "f"(__uint_as_float(r[e + 3]) * scale)
                         : "memory");
      }
      tc_fence_before();
      mbar_arrive(dq_free);
    };
    // L / delta of the next query tile are fetched into registers one tile
    // ahead, so their global-load latency overlaps the current tile.
    float nL = 0.f, nD = 0.f;
    auto fetch_ld = [&](int it) {
      const int q = (qstart + it) * 128 + kr;
      nL = q < Sq ? __ldg(L + (size_t)bh * Sq + q) : 0.f;
      nD = q < Sq ? __ldg(delta + (size_t)bh * Sq + q) : 0.f;
    };
    if (half == 0 && iters > 0) fetch_ld(0);
    bool ok = true;
    for (int it = 0; it < iters && ok; ++it) {
      const uint32_t ph = it & 1;
      const int q0 = (qstart + it) * 128;
      float* Lb = sLD + (it & 1) * 256;
      float* Db = Lb + 128;
      if (half == 0) {
        Lb[kr] = nL;
        Db[kr] = nD;
        mbar_arrive(ld_ready);
        if (it + 1 < iters) fetch_ld(it + 1);
      }
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(ld_ready, ph, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(s_full, ph, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // keys >= lim[q] are masked: key <= q_off + q  <=>  q >= key - q_off
      const int qmin = causal ? key - q_off : -0x7fffffff;
      // tiles fully inside the sequences and the causal band skip the per-element mask
      const bool all_valid = q0 + 128 <= Sq && key < Sk && q0 + half * 64 >= qmin;
      uint8_t* prow = smem + C::OFF_P + half * 16384 + kr * 128;
      uint8_t* dsrow = smem + C::OFF_DS + half * 16384 + kr * 128;
      const float4* L4 = reinterpret_cast<const float4*>(Lb + half * 64);
      const float4* D4 = reinterpret_cast<const float4*>(Db + half * 64);
      // The half's 64 query columns are read from TMEM in NP passes (two
      // passes of 32 with the drain warps, whose threads have fewer registers).
      constexpr int NP = DRAIN ? 2 : 1, PC = 64 / NP;
      bool pass_ok = true;
#pragma unroll
      for (int pass = 0; pass < NP; ++pass) {
        uint32_t sr[PC / 16][16], dr[PC / 16][16];
#pragma unroll
        for (int c = 0; c < PC / 16; ++c) {
          tmem_ld16(tmem + lane_base + C::C_S + half * 64 + pass * PC + c * 16, sr[c]);
          tmem_ld16(tmem + lane_base + C::C_DP + half * 64 + pass * PC + c * 16, dr[c]);
        }
        tmem_ld_wait();
        if (pass == NP - 1) {
          tc_fence_before();
          mbar_arrive(s_free);
        }
        // P^T / dS^T of tile it-1 must have been consumed before they are overwritten
        if (pass == 0 && it > 0 &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(p_free, ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
          pass_ok = false;
          break;
        }
#pragma unroll
        for (int cc = 0; cc < PC / 8; ++cc) {
          const int c = pass * (PC / 8) + cc;              // 8-column chunk within the half
          uint32_t pk[4], dk[4];
          const float4 la = L4[2 * c], lb = L4[2 * c + 1], da = D4[2 * c], db = D4[2 * c + 1];
          const float lv[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
          const float dl[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float pv[2], dv2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int col = cc * 8 + 2 * e + u;            // within this pass
              const int q = q0 + half * 64 + pass * PC + col;
              const float s = __uint_as_float(sr[col >> 4][col & 15]);
              const float dp = __uint_as_float(dr[col >> 4][col & 15]);
              float p = ex2_approx(s * scale_log2 - lv[2 * e + u]);
              if (!all_valid && !(q < Sq && key < Sk && q >= qmin)) p = 0.f;
              pv[u] = p;
              dv2[u] = p * (dp - dl[2 * e + u]);
            }
            pk[e] = pack_bf16x2(pv[0], pv[1]);
            dk[e] = pack_bf16x2(dv2[0], dv2[1]);
          }
          const int sw = (c ^ (kr & 7)) << 4;
          *reinterpret_cast<uint4*>(prow + sw) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(dsrow + sw) = make_uint4(dk[0], dk[1], dk[2], dk[3]);
        }
      }
      if (!pass_ok) {
        ok = false;
        break;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
      // dQ_{it-1} finished with the MMAs that released P^T / dS^T above
      if (!DRAIN && it > 0) {
        tc_fence_after();
        drain_dq(it - 1);
      }
    }
    // last dQ tile, then final dK, dV for this thread's key row (its half of the columns)
    if (ok && iters > 0 &&
        __all_sync(0xffffffffu, mbar_wait_bounded(acc_done, 0, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
      tc_fence_after();
      if (!DRAIN) drain_dq(iters - 1);
      float* dkr = dK + ((size_t)bh * Sk + key) * DQK;
      float* dvr = dVo + ((size_t)bh * Sk + key) * DV;
      // every TMEM read of this thread's dK / dV columns is issued before the
      // one wait (the CTA's last work: no serial load-wait-store chain)
      constexpr int KC = (NDQ + 1) / 2, VC = DV / 32;
      uint32_t rk[KC][16], rv[VC][16];
#pragma unroll
      for (int j = 0; j < KC; ++j)
        if (dq_c0 + j < dq_c1) tmem_ld16(tmem + lane_base + C::C_DK + (dq_c0 + j) * 16, rk[j]);
#pragma unroll
      for (int j = 0; j < VC; ++j) tmem_ld16(tmem + lane_base + C::C_DV + (half * VC + j) * 16, rv[j]);
      tmem_ld_wait();
      if (key < Sk) {
#pragma unroll
        for (int j = 0; j < KC; ++j)
          if (dq_c0 + j < dq_c1)
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              *reinterpret_cast<float4*>(dkr + (dq_c0 + j) * 16 + e) =
                  make_float4(__uint_as_float(rk[j][e]) * scale, __uint_as_float(rk[j][e + 1]) * scale,
                              __uint_as_float(rk[j][e + 2]) * scale, __uint_as_float(rk[j][e + 3]) * scale);
#pragma unroll
        for (int j = 0; j < VC; ++j)
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4*>(dvr + (half * VC + j) * 16 + e) =
                make_float4(__uint_as_float(rv[j][e]), __uint_as_float(rv[j][e + 1]), __uint_as_float(rv[j][e + 2]),
                            __uint_as_float(rv[j][e + 3]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace dsv3
