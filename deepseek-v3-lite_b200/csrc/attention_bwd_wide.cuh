// Flash-attention backward on tcgen05 as two kernels, for heads of
// qk = 64 * NA + 16 * NB (NA 128B-swizzled blocks of 64, an optional
// 32B-swizzled block of 16) and v = DV.  The single-kernel backward
// (attention_sm100.cuh) keeps S^T, dP^T, dV, dK and dQ in TMEM; at qk 192 /
// v 128 that is 768 columns, more than the 512 a CTA can hold.  The work is
// split in two kernels that each fit (columns given for qk 192 / v 128):
//
//   fa_bwd_kv_sm100_kernel   one CTA per (128-key tile, b*h), walking 64-query
//                            sub-tiles:  S^T = K Q^T, dP^T = V dO^T  (64 + 64
//                            columns), P^T / dS^T as bf16 tiles in shared
//                            memory (double-buffered, so the softmax of the
//                            next sub-tile overlaps the dV / dK MMAs of this
//                            one), dV += P^T dO, dK += dS^T Q  (128 + 192
//                            columns).  448 columns in all.
//   fa_bwd_dq_sm100_kernel   one CTA per (128-query tile, b*h), walking the
//                            key tiles it can see:  S = Q K^T, dP = dO V^T
//                            (128 + 128 columns), dS = P (dP - delta) as a
//                            bf16 tile in shared memory, dQ += dS K in TMEM
//                            (192 columns), stored once at the end (no
//                            atomics, dQ need not be zeroed).
//
// The dQ kernel recomputes S and dP: 7 GEMM passes instead of 5, all on the
// tensor cores.  Both use the contracts of the single-kernel backward: L in
// the log2 domain (m + log2 l of the scaled scores), delta = rowsum(dO * O),
// Q / K [b*h, S, qk], V [b*h, Sk, v], dO token-major [B, Sq, H, v]; dK, dV, dQ
// fp32 in the layouts of Q / K / V.  Every wait is bounded; a wait that runs
// out records a status code and the CTA stops issuing, drains what it has in
// flight and frees its TMEM.
#pragma once

#include "common.cuh"

namespace dsv3 {

template <int NA, int NB, int DV>
struct FabKvCfg {
  static constexpr int DQK = NA * 64 + NB * 16;
  static constexpr int K_B = NA * 16384 + NB * 4096;  // K tile: 128 keys x DQK
  static constexpr int V_B = (DV / 64) * 16384;       // V tile: 128 keys x DV
  static constexpr int QS_B = NA * 8192 + NB * 2048;  // Q sub-tile: 64 queries x DQK
  static constexpr int OS_B = (DV / 64) * 8192;  // dO sub-tile: 64 queries x DV
  static constexpr int PT_B = 16384;             // P^T or dS^T: 128 keys x 64 queries, bf16
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + K_B;
  static constexpr int OFF_Q = OFF_V + V_B;        // 2 stages
  static constexpr int OFF_DO = OFF_Q + 2 * QS_B;  // 2 stages
  static constexpr int OFF_P = OFF_DO + 2 * OS_B;  // 2 buffers
  static constexpr int OFF_DS = OFF_P + 2 * PT_B;  // 2 buffers
  static constexpr int OFF_LD = OFF_DS + 2 * PT_B; // L / delta: 2 buffers x 2 x 64 floats
  static constexpr int OFF_BAR = OFF_LD + 1024;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr int DQKP = (DQK + 31) / 32 * 32;  // TMEM regions start on 32-column boundaries
  static constexpr int C_S = 0, C_DP = 64, C_DV = 128, C_DK = 128 + DV;
  static_assert(DV % 64 == 0 && DV <= 128, "DV must be 64 or 128");
  static_assert(C_DK + DQKP <= 512, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
};

template <int NA, int NB, int DV>
__global__ void __launch_bounds__(320, 1)
    fa_bwd_kv_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmQb,
                           const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmKb,
                           const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                           const float* __restrict__ L, const float* __restrict__ delta, float* __restrict__ dK,
                           float* __restrict__ dVo, int Sq, int Sk, int H, int q_off, float scale_log2, float scale,
                           int causal, unsigned int* status) {
  using C = FabKvCfg<NA, NB, DV>;
  constexpr int DQK = C::DQK;
  extern __shared__ __align__(1024) uint8_t fkv_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fkv_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* kv_full = bar;        // K, V loaded
  uint64_t* qd_full = bar + 1;    // [2] Q / dO sub-tile loaded
  uint64_t* qd_empty = bar + 3;   // [2]
  uint64_t* s_full = bar + 5;     // S^T, dP^T ready
  uint64_t* s_free = bar + 6;     // compute warps hold them in registers
  uint64_t* p_full = bar + 7;     // [2] P^T, dS^T written
  uint64_t* p_free = bar + 9;     // [2] dV / dK MMAs done reading them
  uint64_t* acc_done = bar + 11;  // final dK, dV in TMEM
  uint64_t* ld_ready = bar + 12;  // L / delta of the sub-tile staged
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sLD = reinterpret_cast<float*>(smem + C::OFF_LD);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int k_tile, bh;
  fa_tile_order(causal, false, k_tile, bh);  // earlier key tiles are seen by more queries
  const int n0 = k_tile * 128;
  const int b = bh / H, h = bh % H;
  // first 64-query sub-tile with a query that sees key n0 (key <= q + q_off)
  const int qstart = causal ? max(0, (n0 - q_off) / 64) : 0;
  const int nq = (Sq + 63) / 64;
  const int iters = max(0, nq - qstart);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(acc_done, 1);
    mbar_init(ld_ready, 64);
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
      mbar_arrive_expect_tx(kv_full, C::K_B + C::V_B);
#pragma unroll
      for (int a = 0; a < NA; ++a) tma_load_3d(smem + C::OFF_K + a * 16384, &tmK, kv_full, a * 64, n0, bh);
      if (NB) tma_load_3d(smem + C::OFF_K + NA * 16384, &tmKb, kv_full, NA * 64, n0, bh);
#pragma unroll
      for (int d = 0; d < DV / 64; ++d) tma_load_3d(smem + C::OFF_V + d * 16384, &tmV, kv_full, d * 64, n0, bh);
      uint32_t issued = 0, last_phase = 0;
      for (int it = 0; it < iters; ++it) {
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        const int q0 = (qstart + it) * 64;
        if (!mbar_wait_bounded(&qd_empty[st], ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&qd_full[st], C::QS_B + C::OS_B);
        uint8_t* q = smem + C::OFF_Q + st * C::QS_B;
        uint8_t* o = smem + C::OFF_DO + st * C::OS_B;
#pragma unroll
        for (int a = 0; a < NA; ++a) tma_load_3d(q + a * 8192, &tmQ, &qd_full[st], a * 64, q0, bh);
        if (NB) tma_load_3d(q + NA * 8192, &tmQb, &qd_full[st], NA * 64, q0, bh);
#pragma unroll
        for (int d = 0; d < DV / 64; ++d) tma_load_4d(o + d * 8192, &tmdO, &qd_full[st], d * 64, h, q0, b);
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
      constexpr uint32_t I_S = idesc_bf16_f32(128, 64, 0, 0);    // S^T, dP^T: N = the 64 queries
      constexpr uint32_t I_MN = idesc_bf16_f32(128, 64, 0, 1);   // dV, dK: 64-column chunks, B MN-major
      constexpr uint32_t I_MN16 = idesc_bf16_f32(128, 16, 0, 1); // dK: the 16-column block
      const uint32_t k_s = smem_u32(smem + C::OFF_K), v_s = smem_u32(smem + C::OFF_V);
      auto issue_s_dp = [&](int it) {
        const int st = it & 1;
        const uint32_t q_s = smem_u32(smem + C::OFF_Q + st * C::QS_B), o_s = smem_u32(smem + C::OFF_DO + st * C::OS_B);
        // S^T = K Q^T  (K = the DQK head dims, 16 per step)
        uint32_t acc = 0;
#pragma unroll
        for (int a = 0; a < NA; ++a)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_bf16(tmem + C::C_S, smem_desc_sw128(k_s + a * 16384 + kk * 32, 16, 1024),
                      smem_desc_sw128(q_s + a * 8192 + kk * 32, 16, 1024), I_S, acc);
            acc = 1;
          }
        if (NB) umma_bf16(tmem + C::C_S, smem_desc_sw32(k_s + NA * 16384, 256), smem_desc_sw32(q_s + NA * 8192, 256), I_S, 1);
        // dP^T = V dO^T
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk)
          umma_bf16(tmem + C::C_DP, smem_desc_sw128(v_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                    smem_desc_sw128(o_s + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), I_S, kk > 0 ? 1u : 0u);
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
        const int st = it & 1, pb = it & 1;
        if (it + 1 < iters) {
          // S / dP TMEM is free once the compute warps loaded sub-tile it
          if (!mbar_wait_bounded(s_free, it & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM)) break;
          if (!mbar_wait_bounded(&qd_full[st ^ 1], ((it + 1) >> 1) & 1, abort_flag, status, DSV3_ERR_WAIT_FULL)) break;
          tc_fence_after();
          issue_s_dp(it + 1);
        }
        if (!mbar_wait_bounded(&p_full[pb], (it >> 1) & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM)) break;
        tc_fence_after();
        const uint32_t q_s = smem_u32(smem + C::OFF_Q + st * C::QS_B), o_s = smem_u32(smem + C::OFF_DO + st * C::OS_B);
        const uint32_t p_s = smem_u32(smem + C::OFF_P + pb * C::PT_B);
        const uint32_t ds_s = smem_u32(smem + C::OFF_DS + pb * C::PT_B);
        // dV += P^T dO   (K = the 64 queries, 16 per step; dO read MN-major)
#pragma unroll
        for (int d = 0; d < DV / 64; ++d)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + C::C_DV + d * 64, smem_desc_sw128(p_s + kk * 32, 16, 1024),
                      smem_desc_sw128(o_s + d * 8192 + kk * 2048, 8192, 1024), I_MN, (it > 0 || kk > 0) ? 1u : 0u);
        // dK += dS^T Q   (Q read MN-major)
#pragma unroll
        for (int a = 0; a < NA; ++a)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + C::C_DK + a * 64, smem_desc_sw128(ds_s + kk * 32, 16, 1024),
                      smem_desc_sw128(q_s + a * 8192 + kk * 2048, 8192, 1024), I_MN, (it > 0 || kk > 0) ? 1u : 0u);
        if (NB)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + C::C_DK + NA * 64, smem_desc_sw128(ds_s + kk * 32, 16, 1024),
                      smem_desc_sw32(q_s + NA * 8192 + kk * 512, 256), I_MN16, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&p_free[pb]);
        umma_commit(&qd_empty[st]);
      }
      if (any) {
        umma_commit(acc_done);
        mbar_wait_bounded(acc_done, 0, nullptr, status, DSV3_ERR_WAIT_TMEM);
      }
    }
  } else {
    // ---------------------------------------------- compute (key rows)
    // Warps 2-5 and 6-9 share each key row (same TMEM lane quarter): the
    // first group takes query columns 0-31 of the sub-tile, the second 32-63.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int kr = quarter * 32 + lane;
    const int key = n0 + kr;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    // L / delta of the next sub-tile are fetched one sub-tile ahead by the
    // 64 threads of warps 2-3 (one query each)
    const bool stager = half == 0 && kr < 64;
    float nL = 0.f, nD = 0.f;
    auto fetch_ld = [&](int it) {
      const int q = (qstart + it) * 64 + kr;
      nL = q < Sq ? __ldg(L + (size_t)bh * Sq + q) : 0.f;
      nD = q < Sq ? __ldg(delta + (size_t)bh * Sq + q) : 0.f;
    };
    if (stager && iters > 0) fetch_ld(0);
    bool ok = true;
    for (int it = 0; it < iters && ok; ++it) {
      const int pb = it & 1;
      const int q0 = (qstart + it) * 64;
      float* Lb = sLD + (it & 1) * 128;
      float* Db = Lb + 64;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(s_full, it & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      // S(it) issued means every compute thread loaded S(it-1), so it finished
      // sub-tile it-2, the last reader of this L / delta buffer
      if (stager) {
        Lb[kr] = nL;
        Db[kr] = nD;
        mbar_arrive(ld_ready);
        if (it + 1 < iters) fetch_ld(it + 1);
      }
      tc_fence_after();
      uint32_t sr[2][16], dr[2][16];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld16(tmem + lane_base + C::C_S + half * 32 + c * 16, sr[c]);
        tmem_ld16(tmem + lane_base + C::C_DP + half * 32 + c * 16, dr[c]);
      }
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(s_free);
      // P^T / dS^T buffer pb was last read by the MMAs of sub-tile it-2
      if (it >= 2 &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(&p_free[pb], ((it >> 1) & 1) ^ 1u, abort_flag, status,
                                                     DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(ld_ready, it & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      // key <= q_off + q  <=>  q >= key - q_off
      const int qmin = causal ? key - q_off : -0x7fffffff;
      const bool all_valid = q0 + 64 <= Sq && key < Sk && q0 + half * 32 >= qmin;
      uint8_t* prow = smem + C::OFF_P + pb * C::PT_B + kr * 128;
      uint8_t* dsrow = smem + C::OFF_DS + pb * C::PT_B + kr * 128;
      const float4* L4 = reinterpret_cast<const float4*>(Lb + half * 32);
      const float4* D4 = reinterpret_cast<const float4*>(Db + half * 32);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[4], dk[4];
        const float4 la = L4[2 * c], lb = L4[2 * c + 1], da = D4[2 * c], db = D4[2 * c + 1];
        const float lv[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
        const float dl[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float pv[2], dv2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = c * 8 + 2 * e + u;   // within this half
            const int q = q0 + half * 32 + col;
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
        // 16-byte chunk (half * 4 + c) of the key row, 128B swizzle
        const int sw = ((half * 4 + c) ^ (kr & 7)) << 4;
        *reinterpret_cast<uint4*>(prow + sw) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(dsrow + sw) = make_uint4(dk[0], dk[1], dk[2], dk[3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[pb]);
    }
    // final dK, dV of this thread's key row (its half of the columns)
    if (ok && iters > 0 &&
        __all_sync(0xffffffffu, mbar_wait_bounded(acc_done, 0, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
      tc_fence_after();
      constexpr int NDK = DQK / 16;
      const int c0 = half ? NDK / 2 : 0, c1 = half ? NDK : NDK / 2;
      float* dkr = dK + ((size_t)bh * Sk + key) * DQK;
      float* dvr = dVo + ((size_t)bh * Sk + key) * DV;
      for (int c = c0; c < c1; ++c) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + C::C_DK + c * 16, r);
        tmem_ld_wait();
        if (key < Sk)
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4*>(dkr + c * 16 + e) =
                make_float4(__uint_as_float(r[e]) * scale, __uint_as_float(r[e + 1]) * scale,
                            __uint_as_float(r[e + 2]) * scale, __uint_as_float(r[e + 3]) * scale);
      }
      for (int c = half * (DV / 32); c < (half + 1) * (DV / 32); ++c) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + C::C_DV + c * 16, r);
        tmem_ld_wait();
        if (key < Sk)
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4*>(dvr + c * 16 + e) = make_float4(
                __uint_as_float(r[e]), __uint_as_float(r[e + 1]), __uint_as_float(r[e + 2]), __uint_as_float(r[e + 3]));
      }
    } else if (iters == 0 && key < Sk) {
      // no query sees these keys: their gradients are zero
      constexpr int NDK = DQK / 16;
      const int c0 = half ? NDK / 2 : 0, c1 = half ? NDK : NDK / 2;
      for (int c = c0 * 16; c < c1 * 16; ++c) dK[((size_t)bh * Sk + key) * DQK + c] = 0.f;
      for (int c = half * (DV / 2); c < (half + 1) * (DV / 2); ++c) dVo[((size_t)bh * Sk + key) * DV + c] = 0.f;
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

template <int NA, int NB, int DV>
struct FabQCfg {
  static constexpr int DQK = NA * 64 + NB * 16;
  static constexpr int Q_B = NA * 16384 + NB * 4096;  // Q tile: 128 queries x DQK
  static constexpr int O_B = (DV / 64) * 16384;       // dO tile: 128 queries x DV
  static constexpr int K_B = NA * 16384 + NB * 4096;  // K tile: 128 keys x DQK
  static constexpr int V_B = (DV / 64) * 16384;  // V tile: 128 keys x DV
  static constexpr int S_B = 32768;              // dS [128 queries][128 keys] bf16
  // two K stages where they fit (qk 128), one at qk 192
  static constexpr int KST = (Q_B + O_B + 2 * K_B + V_B + S_B + 256 + 1024 <= 232448) ? 2 : 1;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_O = OFF_Q + Q_B;
  static constexpr int OFF_K = OFF_O + O_B;
  static constexpr int OFF_V = OFF_K + KST * K_B;
  static constexpr int OFF_S = OFF_V + V_B;
  static constexpr int OFF_BAR = OFF_S + S_B;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr int DQKP = (DQK + 31) / 32 * 32;
  static constexpr int C_S = 0, C_DP = 128, C_DQ = 256;
  static_assert(DV % 64 == 0 && DV <= 128, "DV must be 64 or 128");
  static_assert(C_DQ + DQKP <= 512, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
};

template <int NA, int NB, int DV>
__global__ void __launch_bounds__(320, 1)
    fa_bwd_dq_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmQb,
                           const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmKb,
                           const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                           const float* __restrict__ L, const float* __restrict__ delta, float* __restrict__ dQ,
                           int Sq, int Sk, int H, int q_off, float scale_log2, float scale, int causal,
                           unsigned int* status) {
  using C = FabQCfg<NA, NB, DV>;
  constexpr int DQK = C::DQK;
  constexpr int KST = C::KST;
  extern __shared__ __align__(1024) uint8_t fdq_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fdq_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bar;        // Q, dO loaded
  uint64_t* k_full = bar + 1;    // [2]
  uint64_t* k_empty = bar + 3;   // [2]
  uint64_t* v_full = bar + 5;
  uint64_t* v_empty = bar + 6;
  uint64_t* s_full = bar + 7;    // S, dP ready
  uint64_t* s_free = bar + 8;    // compute warps hold them in registers
  uint64_t* p_full = bar + 9;    // dS written
  uint64_t* p_free = bar + 10;   // dQ MMA done reading dS
  uint64_t* dq_done = bar + 11;  // final dQ in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int q_tile, bh;
  fa_tile_order(causal, true, q_tile, bh);   // later query tiles see more keys
  const int m0 = q_tile * 128;
  const int b = bh / H, h = bh % H;
  int n_blocks = (Sk + 127) / 128;
  if (causal) n_blocks = min(n_blocks, (q_off + m0 + 128 + 127) / 128);
  n_blocks = max(n_blocks, 0);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(p_full, 256);
    mbar_init(p_free, 1);
    mbar_init(dq_done, 1);
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
      // ---------------------------------------- producer: Q, dO, then K
      mbar_arrive_expect_tx(q_full, C::Q_B + C::O_B);
#pragma unroll
      for (int a = 0; a < NA; ++a) tma_load_3d(smem + C::OFF_Q + a * 16384, &tmQ, q_full, a * 64, m0, bh);
      if (NB) tma_load_3d(smem + C::OFF_Q + NA * 16384, &tmQb, q_full, NA * 64, m0, bh);
#pragma unroll
      for (int d = 0; d < DV / 64; ++d) tma_load_4d(smem + C::OFF_O + d * 16384, &tmdO, q_full, d * 64, h, m0, b);
      uint32_t issued = 0, last_phase = 0;
      for (int j = 0; j < n_blocks; ++j) {
        const int st = j % KST;
        const uint32_t ph = (j / KST) & 1;
        if (!mbar_wait_bounded(&k_empty[st], ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&k_full[st], C::K_B);
        uint8_t* k = smem + C::OFF_K + st * C::K_B;
#pragma unroll
        for (int a = 0; a < NA; ++a) tma_load_3d(k + a * 16384, &tmK, &k_full[st], a * 64, j * 128, bh);
        if (NB) tma_load_3d(k + NA * 16384, &tmKb, &k_full[st], NA * 64, j * 128, bh);
        issued |= 1u << st;
        last_phase = (last_phase & ~(1u << st)) | (ph << st);
      }
      mbar_wait_bounded(q_full, 0, nullptr, status, DSV3_ERR_WAIT_FULL);
      for (int st = 0; st < KST; ++st)
        if (issued & (1u << st)) mbar_wait_bounded(&k_full[st], (last_phase >> st) & 1u, nullptr, status, DSV3_ERR_WAIT_FULL);
    } else if (lane == 1) {
      // ------------------------------------------------------ producer: V
      int issued = 0;
      for (int j = 0; j < n_blocks; ++j) {
        if (!mbar_wait_bounded(v_empty, (j & 1) ^ 1u, abort_flag, status, DSV3_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(v_full, C::V_B);
#pragma unroll
        for (int d = 0; d < DV / 64; ++d) tma_load_3d(smem + C::OFF_V + d * 16384, &tmV, v_full, d * 64, j * 128, bh);
        issued = j + 1;
      }
      if (issued > 0) mbar_wait_bounded(v_full, (issued - 1) & 1, nullptr, status, DSV3_ERR_WAIT_FULL);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------- MMA issuer
      constexpr uint32_t I_S = idesc_bf16_f32(128, 128, 0, 0);   // S, dP
      constexpr uint32_t I_Q = idesc_bf16_f32(128, 64, 0, 1);    // dQ: 64-column chunks, K read MN-major
      constexpr uint32_t I_Q16 = idesc_bf16_f32(128, 16, 0, 1);  // dQ: the 16-column block
      const uint32_t q_s = smem_u32(smem + C::OFF_Q), o_s = smem_u32(smem + C::OFF_O);
      const uint32_t v_s = smem_u32(smem + C::OFF_V), ds_s = smem_u32(smem + C::OFF_S);
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, status, DSV3_ERR_WAIT_FULL);
      bool any = false;
      for (int j = 0; ok && j < n_blocks; ++j) {
        const int st = j % KST;
        const uint32_t k_s = smem_u32(smem + C::OFF_K + st * C::K_B);
        if (!mbar_wait_bounded(&k_full[st], (j / KST) & 1, abort_flag, status, DSV3_ERR_WAIT_FULL)) break;
        if (!mbar_wait_bounded(v_full, j & 1, abort_flag, status, DSV3_ERR_WAIT_FULL)) break;
        // S / dP TMEM is free once the compute warps loaded tile j-1
        if (j > 0 && !mbar_wait_bounded(s_free, (j - 1) & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM)) break;
        tc_fence_after();
        // S = Q K^T
        uint32_t acc = 0;
#pragma unroll
        for (int a = 0; a < NA; ++a)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_bf16(tmem + C::C_S, smem_desc_sw128(q_s + a * 16384 + kk * 32, 16, 1024),
                      smem_desc_sw128(k_s + a * 16384 + kk * 32, 16, 1024), I_S, acc);
            acc = 1;
          }
        if (NB) umma_bf16(tmem + C::C_S, smem_desc_sw32(q_s + NA * 16384, 256), smem_desc_sw32(k_s + NA * 16384, 256), I_S, 1);
        // dP = dO V^T
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk)
          umma_bf16(tmem + C::C_DP, smem_desc_sw128(o_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                    smem_desc_sw128(v_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), I_S, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
        umma_commit(v_empty);   // V_j is free once dP_j is computed
        any = true;
        if (!mbar_wait_bounded(p_full, j & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM)) break;
        tc_fence_after();
        // dQ += dS K   (K = the 128 keys, 16 per step; K read MN-major)
#pragma unroll
        for (int a = 0; a < NA; ++a)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tmem + C::C_DQ + a * 64, smem_desc_sw128(ds_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                      smem_desc_sw128(k_s + a * 16384 + kk * 2048, 16384, 1024), I_Q, (j > 0 || kk > 0) ? 1u : 0u);
        if (NB)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tmem + C::C_DQ + NA * 64, smem_desc_sw128(ds_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                      smem_desc_sw32(k_s + NA * 16384 + kk * 512, 256), I_Q16, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(p_free);
        umma_commit(&k_empty[st]);
      }
      if (any) {
        umma_commit(dq_done);
        mbar_wait_bounded(dq_done, 0, nullptr, status, DSV3_ERR_WAIT_TMEM);
      }
    }
  } else {
    // -------------------------------------------- compute (query rows)
    // Warps 2-5 and 6-9 share each query row (same TMEM lane quarter): the
    // first group takes key columns 0-63 of the tile, the second 64-127.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int q = m0 + row;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float Lq = q < Sq ? __ldg(L + (size_t)bh * Sq + q) : 0.f;
    const float Dq = q < Sq ? __ldg(delta + (size_t)bh * Sq + q) : 0.f;
    const int kmax = causal ? min(Sk - 1, q + q_off) : Sk - 1;   // last key this row sees
    bool ok = true;
    for (int j = 0; j < n_blocks && ok; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(s_full, j & 1, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[4][16], dr[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld16(tmem + lane_base + C::C_S + half * 64 + c * 16, sr[c]);
        tmem_ld16(tmem + lane_base + C::C_DP + half * 64 + c * 16, dr[c]);
      }
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(s_free);
      // the dS tile was last read by the dQ MMAs of tile j-1
      if (j > 0 && !__all_sync(0xffffffffu, mbar_wait_bounded(p_free, (j - 1) & 1, abort_flag, status,
                                                                DSV3_ERR_WAIT_TMEM))) {
        ok = false;
        break;
      }
      const int k0 = j * 128 + half * 64;
      const bool all_valid = q < Sq && k0 + 63 <= kmax;
      uint8_t* srow = smem + C::OFF_S + half * 16384 + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t dk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float d2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = c * 8 + 2 * e + u;   // within this half
            const float s = __uint_as_float(sr[col >> 4][col & 15]);
            const float dp = __uint_as_float(dr[col >> 4][col & 15]);
            float p = ex2_approx(s * scale_log2 - Lq);
            if (!all_valid && !(q < Sq && k0 + col <= kmax)) p = 0.f;
            d2[u] = p * (dp - Dq);
          }
          dk[e] = pack_bf16x2(d2[0], d2[1]);
        }
        *reinterpret_cast<uint4*>(srow + ((c ^ (row & 7)) << 4)) = make_uint4(dk[0], dk[1], dk[2], dk[3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    constexpr int NDQ = DQK / 16;
    const int c0 = half ? NDQ / 2 : 0, c1 = half ? NDQ : NDQ / 2;
    float* dqr = dQ + ((size_t)bh * Sq + q) * DQK;
    if (ok && n_blocks > 0 &&
        __all_sync(0xffffffffu, mbar_wait_bounded(dq_done, 0, abort_flag, status, DSV3_ERR_WAIT_TMEM))) {
      tc_fence_after();
      for (int c = c0; c < c1; ++c) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + C::C_DQ + c * 16, r);
        tmem_ld_wait();
        if (q < Sq)
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4*>(dqr + c * 16 + e) =
                make_float4(__uint_as_float(r[e]) * scale, __uint_as_float(r[e + 1]) * scale,
                            __uint_as_float(r[e + 2]) * scale, __uint_as_float(r[e + 3]) * scale);
      }
    } else if (n_blocks == 0 && q < Sq) {
      for (int c = c0 * 16; c < c1 * 16; ++c) dqr[c] = 0.f;
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
