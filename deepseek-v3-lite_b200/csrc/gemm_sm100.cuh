// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[m, n] = sum_k A[m, k] * B[n, k]        (bf16 in, fp32 accumulate in TMEM)
//
// One CTA per SM loops over output tiles of 128 x BN.  Warp 0 is the TMA
// producer, warp 1 issues tcgen05.mma from one elected thread and owns the
// TMEM allocation, warps 2-5 run the epilogue (TMEM -> registers -> global).
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the MMAs of tile i+1.  Shared memory holds a ring of
// STAGES (A, B) K-blocks of 64 elements, 128-byte swizzled.
//
// Operands may be K-major (reduction dimension contiguous) or MN-major
// (output dimension contiguous); together that covers the forward (x W^T),
// data-gradient (dY W) and weight-gradient (dY^T X) products without any
// transpose copies.  Three schedules:
//   Dense     - one problem, optional split-K (weight gradients);
//   GroupedM  - rows are expert-sorted and padded to 128 per expert; a device
//               array maps each 128-row tile to its expert (B is per expert);
//   GroupedK  - per-expert weight gradients: the reduction runs over the
//               expert's padded row range, read from a device offset array.
// Epilogues are fused: bf16 store, fp32 accumulate (residual stream, weight
// gradients), SwiGLU forward/backward, and the two halves of the LM-head
// cross-entropy (online log-sum-exp partials; softmax-minus-one-hot grads).
#pragma once

#include "common.cuh"

namespace dsv3 {

enum class Sched : int { Dense = 0, GroupedM = 1, GroupedK = 2 };
enum class Epi : int {
  StoreBF16 = 0,     // out (bf16) = acc
  AddF32 = 1,        // out (fp32) += acc
  AtomicAddF32 = 2,  // out (fp32) += acc, atomically (split-K)
  SwigluFwd = 3,     // h = silu(g) * u, gu = [g | u]
  SwigluBwd = 4,     // dgu from dh = acc and the saved gu
  CeFwd = 5,         // per-row (max, sum-exp) partials + target logit
  CeBwd = 6,         // (softmax - onehot) * scale, bf16
  StoreF32 = 7,      // out (fp32) = acc
  ResidF32 = 8,      // out (fp32) = aux (fp32) + acc   (out-of-place residual add)
  ScatterBF16 = 9,   // out (bf16) = acc, and each row also stored into its home rank's
                     // combine inbox over peer memory (expert-parallel combine)
  CeBwdTma = 10,     // CeBwd, each warp's 32 x 64 output boxes staged in shared memory
                     // (128-byte swizzle) and written by TMA stores; columns N .. N rounded
                     // up to 8 receive zeros
  // fp32 outputs through shared memory: each warp's 32 x 32 fp32 boxes go out
  // by TMA (N a multiple of 4; the output map is 3-D [groups][rows][N])
  StoreF32Tma = 11,  // out = acc (TMA store)
  AddF32Tma = 12,    // out += acc (TMA reduce-add, atomic per element: also split-K)
  ResidF32Tma = 13,  // out = aux + acc (aux read by the epilogue, TMA store)
  StoreBF16Tma = 14, // out (bf16) = acc through 32 x 64 bf16 boxes (N a multiple of 8)
  SwigluFwdTma = 15, // SwigluFwd with h (map C) and the gate / up pair (map D, [rows][2][I]) by TMA
  SwigluBwdTma = 16  // SwigluBwd with dg / du (map C, [rows][2][I]) by TMA
};

// Epilogues that stage their output in shared memory and write it with TMA.
constexpr bool epi_tma(Epi E) {
  return E == Epi::CeBwdTma || E == Epi::StoreF32Tma || E == Epi::AddF32Tma || E == Epi::ResidF32Tma ||
         E == Epi::StoreBF16Tma || E == Epi::SwigluFwdTma || E == Epi::SwigluBwdTma;
}

constexpr float kLog2e = 1.4426950408889634f;   // log2(e)
constexpr int kEpiWarps = 8;                 // two warpgroups drain TMEM
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
// ScatterBF16 stages each warp's 32 rows x 64 columns (bf16) in shared memory
// so its stores to other ranks go out as 128-byte row segments
constexpr int kScatterStageBytes = kEpiWarps * 32 * 128;

// CeBwdTma: two 32 x 64 bf16 boxes (4 KB each) per epilogue warp, 1024-byte
// aligned after the barrier block
constexpr int kTmaBoxBytes = 32 * 128;
constexpr int kTmaStageBytes = kEpiWarps * 2 * kTmaBoxBytes;

// SwigluFwdTma: three boxes per warp (h, g, u of one 64-column half tile)
constexpr int kSwigluStageBytes = kEpiWarps * 3 * kTmaBoxBytes;

template <Epi E>
constexpr int epi_smem_bytes() {
  return E == Epi::ScatterBF16 ? kScatterStageBytes
                               : (E == Epi::SwigluFwdTma ? 1024 + kSwigluStageBytes
                                                         : (epi_tma(E) ? 1024 + kTmaStageBytes : 0));
}

struct GemmArgs {
  int M;                 // valid output rows (per group for GroupedK)
  int N;                 // valid output columns
  int K;                 // reduction length (Dense / GroupedM)
  int m_tiles, n_tiles, k_splits, groups;
  int num_tiles;
  int kb_per_split;      // Dense: K-blocks per split
  int panel_rows;        // Dense: > 0 walks the tiles in panels of this many rows, rows fastest
                         // inside a panel (a B operand larger than L2 is then streamed once per
                         // panel while the panel's A rows stay in L2); 0: columns fastest
  const int* tile_group;     // GroupedM: expert of each 128-row tile (< 0: unused tile)
  int tile_rows;             // GroupedM: expert ranges are multiples of this (128 or 256; 256 allows CTA pairs)
  const int* group_row_off;  // GroupedK: [groups + 1] padded row offsets (multiples of 128)
  void* out;             // primary output
  long ldo;
  long out_group_stride; // GroupedK: elements between consecutive experts' outputs
  void* out2;            // SwigluFwd: pre-activations [M, 2I]
  long ldo2;
  const void* aux;       // SwigluBwd: pre-activations [M, 2I]
  long ld_aux;
  int inter;             // SwiGLU: I (the up half starts at column I of out2 / aux)
  const long* targets;   // CE: target id per row (-100 = ignored)
  float* part_max;       // CeFwd: [M, n_tiles]
  float* part_sum;       // CeFwd: [M, n_tiles]
  float* tgt_logit;      // CeFwd: [M]
  const float* lse;      // CeBwd: [M]
  const float* row_scale;// CeBwd: [M]
  unsigned int* status;  // device status word (bounded-wait failures)
  // ScatterBF16: row r goes to rank origin[r] / scatter_tk, slot origin[r] % scatter_tk
  // of the inbox at heap offset scatter_off (rows of N bf16); the last CTA to
  // finish raises flag [scatter_phase][scatter_me] on every rank.
  const unsigned long long* peer_base;   // heap base of every rank (device array)
  const int* origin;
  const float* scatter_extra;            // optional: one float per row, stored to scatter_extra_off[slot]
  long long scatter_extra_off;
  long long scatter_off;
  long long flags_off;
  int scatter_tk, scatter_me, scatter_ranks, scatter_phase;
  unsigned int* done_ctr;
};

// CG = 2: a CTA pair shares one 256-row tile (each CTA: 128 rows of A and
// BN/2 rows of B in its own shared memory), which halves the B traffic per
// MMA and leaves room for more pipeline stages.
template <int BN, int CG = 1, Epi E = Epi::StoreBF16>
struct GemmCfg {
  static constexpr int BM = 128;            // accumulator rows per CTA
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / CG) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // the TMA-store staging (64 KB) takes one (pair) or one more (single) stage
  static constexpr int STAGES = E == Epi::SwigluFwdTma ? (CG == 2 ? 4 : 2)
                                : (epi_tma(E) ? (CG == 2 ? 5 : 3) : (CG == 2 ? 6 : (BN >= 256 ? 4 : 6)));
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;
};

struct TileInfo {
  int m0, n0, g, kb0, kb1, n_tile;
  bool run;
};

template <Sched S>
__device__ __forceinline__ TileInfo decode_tile(int t, const GemmArgs& a, int BN_, int BM_ = 128) {
  TileInfo ti;
  int n, m, outer;
  if (S == Sched::Dense && a.panel_rows > 0) {
    const int mn = a.m_tiles * a.n_tiles;
    outer = t / mn;
    int r = t - outer * mn;
    const int pt = max(1, a.panel_rows / BM_);           // m-tiles per panel
    const int p = r / (pt * a.n_tiles);
    r -= p * pt * a.n_tiles;
    const int pm = min(pt, a.m_tiles - p * pt);           // the last panel may be shorter
    n = r / pm;
    m = p * pt + (r - n * pm);
  } else {
    n = t % a.n_tiles;
    const int rest = t / a.n_tiles;
    m = rest % a.m_tiles;
    outer = rest / a.m_tiles;
  }
  ti.n_tile = n;
  ti.n0 = n * BN_;
  ti.m0 = m * BM_;
  ti.g = 0;
  ti.run = true;
  if constexpr (S == Sched::Dense) {
    int total = (a.K + 63) / 64;
    ti.kb0 = outer * a.kb_per_split;
    ti.kb1 = min(total, ti.kb0 + a.kb_per_split);
  } else if constexpr (S == Sched::GroupedM) {
    ti.g = a.tile_group[m * (BM_ / 128)];   // a pair tile's two halves belong to one expert
    ti.kb0 = 0;
    ti.kb1 = (a.K + 63) / 64;
    ti.run = ti.g >= 0;
  } else {
    // outer = group * k_splits + split; the group's row range (known only on
    // the device) is cut into k_splits equal chunks of 64-row blocks.
    const int splits = a.k_splits;
    ti.g = outer / splits;
    const int sp = outer - ti.g * splits;
    const int lo = a.group_row_off[ti.g] / 64, hi = a.group_row_off[ti.g + 1] / 64;
    const int chunk = (hi - lo + splits - 1) / splits;
    ti.kb0 = lo + sp * chunk;
    ti.kb1 = min(hi, ti.kb0 + chunk);
  }
  ti.run = ti.run && (ti.kb1 > ti.kb0);
  return ti;
}

// B_SWIGLU: B is read as two 128-row halves (gate rows, up rows) of a 4-D
// tensor map [G][2][I][K]; BN must be 256 and the epilogue pairs column c of
// the gate half with column c of the up half.
template <int BN, int A_MN, int B_MN, Sched S, Epi E, bool B_SWIGLU, int CG>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                      GemmArgs args) {
  using C = GemmCfg<BN, CG, E>;
  constexpr bool kTmaOut = epi_tma(E);
  static_assert(!B_SWIGLU || (BN == 256 && !B_MN), "SwiGLU B layout needs BN=256, K-major");
  // CTA pairs: BN 256, or BN 128 with an MN-major B (each CTA then loads one
  // 64-column box of B)
  static_assert(CG == 1 || (CG == 2 && (BN == 256 || (BN == 128 && B_MN))), "CTA pairs: BN=256, or BN=128 with MN-major B");
  constexpr int BMT = 128 * CG;                   // rows of one (pair) tile
  const uint32_t cta = CG == 2 ? cluster_ctarank() : 0u;
  const bool leader = cta == 0;
  const int tile0 = CG == 2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstep = CG == 2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint4* scatter_stage = reinterpret_cast<uint4*>(smem + C::STAGES * C::STAGE_BYTES + C::BAR_BYTES);
  uint8_t* tma_stage = smem + C::STAGES * C::STAGE_BYTES + 1024;   // CeBwdTma boxes (1024-byte aligned)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  static_assert(BN % 32 == 0, "BN must split into two 16-column-aligned halves");

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps * CG);   // one arrival per epilogue warp of the pair
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (kTmaOut) tma_prefetch_desc(&tmC);
    if constexpr (E == Epi::SwigluFwdTma) tma_prefetch_desc(&tmD);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();   // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, last_phase = 0;
      for (int t = tile0; t < args.num_tiles && !*abort_flag; t += tstep) {
        TileInfo ti = decode_tile<S>(t, args, B_SWIGLU ? 128 : BN, BMT);
        if (!ti.run) continue;
        for (int kb = ti.kb0; kb < ti.kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, args.status, DSV3_ERR_WAIT_EMPTY)) break;
          uint8_t* sA = smem + stage * C::STAGE_BYTES;
          uint8_t* sB = sA + C::A_BYTES;
          const int k0 = kb * 64;
          // GroupedK walks global rows of A and B; their maps have no group axis.
          const int bg = (S == Sched::GroupedK) ? 0 : ti.g;
          if constexpr (CG == 2) {
            // Both CTAs' copies complete on the even CTA's barrier, which
            // expects the bytes of the whole pair.
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            const uint32_t fb = cluster_map(smem_u32(&full[stage]), 0);
            const int ma = ti.m0 + (int)cta * 128;
            if constexpr (A_MN) {
              tma_load_2d_pair(sA, &tmA, fb, ma, k0);
              tma_load_2d_pair(sA + 8192, &tmA, fb, ma + 64, k0);
            } else {
              tma_load_2d_pair(sA, &tmA, fb, k0, ma);
            }
            if constexpr (B_SWIGLU) {
              tma_load_4d_pair(sB, &tmB, fb, k0, ti.n0, (int)cta, bg);   // CTA 0: gate rows, CTA 1: up rows
            } else if constexpr (B_MN) {
              tma_load_3d_pair(sB, &tmB, fb, ti.n0 + (int)cta * (BN / 2), k0, bg);
              if constexpr (BN / 2 > 64) tma_load_3d_pair(sB + 8192, &tmB, fb, ti.n0 + (int)cta * (BN / 2) + 64, k0, bg);
            } else {
              tma_load_3d_pair(sB, &tmB, fb, k0, ti.n0 + (int)cta * 128, bg);
            }
          } else {
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          if constexpr (A_MN) {
            tma_load_2d(sA, &tmA, &full[stage], ti.m0, k0);
            tma_load_2d(sA + 8192, &tmA, &full[stage], ti.m0 + 64, k0);
          } else {
            tma_load_2d(sA, &tmA, &full[stage], k0, ti.m0);
          }
          if constexpr (B_SWIGLU) {
            tma_load_4d(sB, &tmB, &full[stage], k0, ti.n0, 0, bg);
            tma_load_4d(sB + 16384, &tmB, &full[stage], k0, ti.n0, 1, bg);
          } else if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_3d(sB + j * 8192, &tmB, &full[stage], ti.n0 + 64 * j, k0, bg);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j) tma_load_3d(sB + j * 16384, &tmB, &full[stage], k0, ti.n0 + 128 * j, bg);
          }
          }
          issued_mask |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every issued copy must land before the CTA may exit (the odd CTA of a
      // pair sees that through the MMA's release of the stage).
      for (int s = 0; s < C::STAGES; ++s)
        if (issued_mask & (1u << s)) {
          if (leader) mbar_wait_bounded(&full[s], (last_phase >> s) & 1u, nullptr, args.status, DSV3_ERR_WAIT_FULL);
          else mbar_wait_bounded(&empty[s], (last_phase >> s) & 1u, nullptr, args.status, DSV3_ERR_WAIT_EMPTY);
        }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t IDESC = idesc_bf16_f32(BMT, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool issued_any = false;
      for (int t = tile0; t < args.num_tiles && !*abort_flag; t += tstep) {
        TileInfo ti = decode_tile<S>(t, args, B_SWIGLU ? 128 : BN, BMT);
        if (!ti.run) continue;
        const int buf = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&tempty[buf], aphase ^ 1u, abort_flag, args.status, DSV3_ERR_WAIT_TMEM)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        bool ok = true;
        for (int kb = ti.kb0; kb < ti.kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, args.status, DSV3_ERR_WAIT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t b_base = a_base + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = A_MN ? smem_desc_sw128(a_base + k * 2048, 8192, 1024)
                                     : smem_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(b_base + k * 2048, 8192, 1024)
                                     : smem_desc_sw128(b_base + k * 32, 16, 1024);
            if constexpr (CG == 2) umma_bf16_pair(d_tmem, ad, bd, IDESC, (kb > ti.kb0 || k > 0) ? 1u : 0u);
            else umma_bf16(d_tmem, ad, bd, IDESC, (kb > ti.kb0 || k > 0) ? 1u : 0u);
          }
          issued_any = true;
          if constexpr (CG == 2) umma_commit_pair_both(&empty[stage], 0x3);
          else umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (CG == 2) umma_commit_pair_both(&tfull[buf], 0x3);
        else umma_commit(&tfull[buf]);
        ++local;
      }
      // Drain: make sure no MMA still writes TMEM when it is freed.
      if (issued_any) {
        if constexpr (CG == 2) umma_commit_pair(drain);
        else umma_commit(drain);
        mbar_wait_bounded(drain, 0, nullptr, args.status, DSV3_ERR_WAIT_TMEM);
      }
    }
  } else {
    // --------------------------------------------------------- epilogue
    const int quarter = warp & 3;              // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;          // which half of the tile's columns
    const int r_in_tile = quarter * 32 + lane;
    constexpr int HALF = BN / 2;
    int local = 0;
    int tma_box = 0;                           // CeBwdTma: boxes this warp has stored (buffer = parity)
    (void)tma_box;
    for (int t = tile0; t < args.num_tiles && !*abort_flag; t += tstep) {
      TileInfo ti = decode_tile<S>(t, args, B_SWIGLU ? 128 : BN, BMT);
      if (!ti.run) continue;
      ti.m0 += (int)cta * 128;                  // this CTA's rows of the pair tile
      const int buf = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&tfull[buf], aphase, abort_flag, args.status, DSV3_ERR_WAIT_TMEM)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
      const int row = ti.m0 + r_in_tile;
      const bool row_ok = row < args.M;
      uint32_t r[16];

      if constexpr (E == Epi::StoreBF16Tma) {
        // Two 32-column TMEM steps = one 32 x 64 bf16 box (lane = row, 8
        // 16-byte chunks, chunk j at j ^ (row & 7)); two boxes per warp alternate.
        uint8_t* box_row = tma_stage + (warp - 2) * 2 * kTmaBoxBytes + lane * 128;
        const int box_y = ti.m0 + quarter * 32;
#pragma unroll 1
        for (int c4 = half * HALF; c4 < (half + 1) * HALF; c4 += 64) {
          uint8_t* brow = box_row + (tma_box & 1) * kTmaBoxBytes;
          if (lane == 0) bulk_wait_group_read<1>();   // the store that last used this buffer has read it
          __syncwarp();
#pragma unroll 1
          for (int c2 = c4; c2 < c4 + 64; c2 += 32) {
            uint32_t rr[2][16];
            __syncwarp();
            tmem_ld16(tbase + c2, rr[0]);
            tmem_ld16(tbase + c2 + 16, rr[1]);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              uint32_t pk[8];
#pragma unroll
              for (int j = 0; j < 16; j += 2)
                pk[j / 2] = pack_bf16x2(__uint_as_float(rr[q][j]), __uint_as_float(rr[q][j + 1]));
              const int ch = ((c2 - c4) + 16 * q) >> 3;
              *reinterpret_cast<uint4*>(brow + ((ch ^ (lane & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              *reinterpret_cast<uint4*>(brow + (((ch + 1) ^ (lane & 7)) << 4)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (ti.n0 + c4 < args.N && box_y < args.M) tma_store_3d(&tmC, brow - lane * 128, ti.n0 + c4, box_y, 0);
            bulk_commit_group();
          }
          ++tma_box;
        }
      } else
      if constexpr (E == Epi::StoreF32Tma || E == Epi::AddF32Tma || E == Epi::ResidF32Tma) {
        // One 32-column TMEM step = one 32 x 32 fp32 box: lane = row of the
        // warp's 32 rows, its 32 values as 8 16-byte chunks, chunk j at
        // j ^ (row & 7) (128-byte swizzle); two boxes per warp alternate.
        uint8_t* box_row = tma_stage + (warp - 2) * 2 * kTmaBoxBytes + lane * 128;
        const int box_y = ti.m0 + quarter * 32;
        const int gz = (S == Sched::GroupedK) ? ti.g : 0;
        const float* aux_row = nullptr;
        if constexpr (E == Epi::ResidF32Tma)
          aux_row = reinterpret_cast<const float*>(args.aux) + (size_t)(row_ok ? row : 0) * args.ld_aux;
#pragma unroll 1
        for (int c2 = half * HALF; c2 < (half + 1) * HALF; c2 += 32) {
          const int col = ti.n0 + c2;
          uint8_t* brow = box_row + (tma_box & 1) * kTmaBoxBytes;
          float4 av[8];
          if constexpr (E == Epi::ResidF32Tma) {   // the residual's 32 values, requested before the TMEM wait
#pragma unroll
            for (int j = 0; j < 8; ++j)
              av[j] = (row_ok && col + 4 * j < args.N) ? reinterpret_cast<const float4*>(aux_row + col)[j]
                                                        : make_float4(0.f, 0.f, 0.f, 0.f);
          }
          uint32_t rr[2][16];
          __syncwarp();
          tmem_ld16(tbase + c2, rr[0]);
          tmem_ld16(tbase + c2 + 16, rr[1]);
          if (lane == 0) bulk_wait_group_read<1>();   // the store that last used this buffer has read it
          __syncwarp();
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 v = make_float4(__uint_as_float(rr[j >> 2][(j & 3) * 4]), __uint_as_float(rr[j >> 2][(j & 3) * 4 + 1]),
                                   __uint_as_float(rr[j >> 2][(j & 3) * 4 + 2]),
                                   __uint_as_float(rr[j >> 2][(j & 3) * 4 + 3]));
            if constexpr (E == Epi::ResidF32Tma) {
              v.x += av[j].x;
              v.y += av[j].y;
              v.z += av[j].z;
              v.w += av[j].w;
            }
            *reinterpret_cast<float4*>(brow + ((j ^ (lane & 7)) << 4)) = v;
          }
          fence_proxy_async_smem();   // this lane's box row is visible to the TMA engine
          __syncwarp();
          if (lane == 0) {
            if (col < args.N && box_y < args.M) {
              if constexpr (E == Epi::AddF32Tma) tma_reduce_add_3d(&tmC, brow - lane * 128, col, box_y, gz);
              else tma_store_3d(&tmC, brow - lane * 128, col, box_y, gz);
            }
            bulk_commit_group();
          }
          ++tma_box;
        }
      } else
      if constexpr (E == Epi::StoreBF16 || E == Epi::AddF32 || E == Epi::AtomicAddF32 || E == Epi::StoreF32 ||
                    E == Epi::ResidF32 || E == Epi::ScatterBF16) {
        char* base = reinterpret_cast<char*>(args.out);
        __nv_bfloat16* remote = nullptr;   // ScatterBF16: this row in its home rank's inbox
        if constexpr (E == Epi::ScatterBF16) {
          const int o = row_ok ? args.origin[row] : -1;
          if (o >= 0) {
            const int src = o / args.scatter_tk, slot = o - src * args.scatter_tk;
            if (src < args.scatter_ranks) {
              remote = reinterpret_cast<__nv_bfloat16*>(args.peer_base[src] + args.scatter_off) + (size_t)slot * args.N;
              if (args.scatter_extra != nullptr && ti.n0 == 0 && half == 0)   // once per row
                reinterpret_cast<float*>(args.peer_base[src] + args.scatter_extra_off)[slot] = args.scatter_extra[row];
            }
          }
        }
        if constexpr (S == Sched::GroupedK)
          base += (size_t)ti.g * args.out_group_stride * (E == Epi::StoreBF16 ? 2 : 4);
        static_assert(HALF % 32 == 0, "epilogue drains 32 columns per TMEM wait");
        // ScatterBF16 with N a multiple of 64: this warp's rows are staged 64
        // columns at a time and stored to the home ranks as 128-byte row
        // segments (a warp instruction covers 8 rows x 64 bytes, two
        // instructions a row's 128 bytes) instead of 16-byte pieces per row.
        uint4* stage = scatter_stage + (warp - 2) * 256;   // [32 rows][8 x 16 B]
        const bool staged = E == Epi::ScatterBF16 && (args.N % 64) == 0;
#pragma unroll 1
        for (int c2 = half * HALF; c2 < (half + 1) * HALF; c2 += 32) {
          uint32_t rr[2][16];   // two TMEM loads in flight per wait
          __syncwarp();
          tmem_ld16(tbase + c2, rr[0]);
          tmem_ld16(tbase + c2 + 16, rr[1]);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 2; ++q) {
          const uint32_t (&r)[16] = rr[q];
          const int c = c2 + 16 * q;
          const int col = ti.n0 + c;
          if (!row_ok || col >= args.N) continue;
          const bool full16 = col + 16 <= args.N;
          if constexpr (E == Epi::StoreBF16 || E == Epi::ScatterBF16) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(base) + (size_t)row * args.ldo + col;
            if (full16) {
              uint4 v0, v1;
              v0.x = pack_bf16x2(__uint_as_float(r[0]), __uint_as_float(r[1]));
              v0.y = pack_bf16x2(__uint_as_float(r[2]), __uint_as_float(r[3]));
              v0.z = pack_bf16x2(__uint_as_float(r[4]), __uint_as_float(r[5]));
              v0.w = pack_bf16x2(__uint_as_float(r[6]), __uint_as_float(r[7]));
              v1.x = pack_bf16x2(__uint_as_float(r[8]), __uint_as_float(r[9]));
              v1.y = pack_bf16x2(__uint_as_float(r[10]), __uint_as_float(r[11]));
              v1.z = pack_bf16x2(__uint_as_float(r[12]), __uint_as_float(r[13]));
              v1.w = pack_bf16x2(__uint_as_float(r[14]), __uint_as_float(r[15]));
              reinterpret_cast<uint4*>(o)[0] = v0;
              reinterpret_cast<uint4*>(o)[1] = v1;
              if constexpr (E == Epi::ScatterBF16) {
                if (staged) {
                  const int slot = ((c2 & 63) >> 3) + 2 * q;          // 16-byte unit of the row's 64 columns
                  stage[lane * 8 + slot] = v0;
                  stage[lane * 8 + slot + 1] = v1;
                } else if (remote != nullptr) {
                  reinterpret_cast<uint4*>(remote + col)[0] = v0;
                  reinterpret_cast<uint4*>(remote + col)[1] = v1;
                }
              }
            } else {
              for (int j = 0; j < 16 && col + j < args.N; ++j) {
                o[j] = __float2bfloat16(__uint_as_float(r[j]));
                if constexpr (E == Epi::ScatterBF16) {
                  if (remote != nullptr) remote[col + j] = o[j];
                }
              }
            }
          } else if constexpr (E == Epi::AddF32 || E == Epi::ResidF32) {
            float* o = reinterpret_cast<float*>(base) + (size_t)row * args.ldo + col;
            const float* src = E == Epi::AddF32 ? o : reinterpret_cast<const float*>(args.aux) + (size_t)row * args.ld_aux + col;
            if (full16) {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                float4 v = *reinterpret_cast<const float4*>(src + j);
                v.x += __uint_as_float(r[j]);
                v.y += __uint_as_float(r[j + 1]);
                v.z += __uint_as_float(r[j + 2]);
                v.w += __uint_as_float(r[j + 3]);
                *reinterpret_cast<float4*>(o + j) = v;
              }
            } else {
              for (int j = 0; j < 16 && col + j < args.N; ++j) o[j] = src[j] + __uint_as_float(r[j]);
            }
          } else if constexpr (E == Epi::StoreF32) {
            float* o = reinterpret_cast<float*>(base) + (size_t)row * args.ldo + col;
            if (full16) {
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4*>(o + j) =
                    make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                __uint_as_float(r[j + 3]));
            } else {
              for (int j = 0; j < 16 && col + j < args.N; ++j) o[j] = __uint_as_float(r[j]);
            }
          } else {
            float* o = reinterpret_cast<float*>(base) + (size_t)row * args.ldo + col;
            if (full16 && (args.ldo & 3) == 0) {
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(o + j), "f"(__uint_as_float(r[j])),
                             "f"(__uint_as_float(r[j + 1])), "f"(__uint_as_float(r[j + 2])),
                             "f"(__uint_as_float(r[j + 3]))
                             : "memory");
            } else {
              for (int j = 0; j < 16; ++j)
                if (col + j < args.N) atomicAdd(o + j, __uint_as_float(r[j]));
            }
          }
          }
          if constexpr (E == Epi::ScatterBF16) {
            // after every second 32-column step: 64 staged columns of 32 rows
            // go out, lanes 4i..4i+3 covering one row's 64 bytes per instruction
            const int cbase = ti.n0 + (c2 & ~63);
            if (staged && (c2 & 63) == 32 && cbase < args.N) {
              __syncwarp();
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int u = i * 32 + lane, rr = u >> 3, qq = u & 7;
                const unsigned long long rp =
                    __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(remote), rr);
                if (rp != 0ull) reinterpret_cast<uint4*>(rp)[(cbase >> 3) + qq] = stage[u];
              }
              __syncwarp();
            }
          }
        }
      } else if constexpr (E == Epi::SwigluFwd || E == Epi::SwigluFwdTma) {
        // TMEM columns [0,128): gate, [128,256): up, for I-columns n0 .. n0+127.
        // SwigluFwdTma: this warp's 64 columns of h, g and u go to three
        // 32 x 64 boxes (lane = row, chunk j at j ^ (row & 7)), then TMA.
        constexpr bool kT = E == Epi::SwigluFwdTma;
        __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(args.out);
        __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(args.out2);
        uint8_t* hbox = tma_stage + (warp - 2) * 3 * kTmaBoxBytes + lane * 128;
        if constexpr (kT) {
          if (lane == 0) bulk_wait_group_read<0>();   // the previous tile's stores have read the boxes
          __syncwarp();
        }
        uint32_t u[16];
#pragma unroll 1
        for (int c = half * 64; c < half * 64 + 64; c += 16) {
          __syncwarp();
          tmem_ld16(tbase + c, r);
          tmem_ld16(tbase + 128 + c, u);
          tmem_ld_wait();
          const int col = ti.n0 + c;
          if (!kT && (!row_ok || col >= args.N)) continue;
          const int nv = min(16, args.N - col);
          uint32_t hp[8], gp[8], up[8];
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            // Round the pre-activations to bf16 first so forward and backward
            // see identical gate/up values.
            const float g0 = __bfloat162float(__float2bfloat16(__uint_as_float(r[j])));
            const float g1 = __bfloat162float(__float2bfloat16(__uint_as_float(r[j + 1])));
            const float u0 = __bfloat162float(__float2bfloat16(__uint_as_float(u[j])));
            const float u1 = __bfloat162float(__float2bfloat16(__uint_as_float(u[j + 1])));
            hp[j / 2] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
            gp[j / 2] = pack_bf16x2(g0, g1);
            up[j / 2] = pack_bf16x2(u0, u1);
          }
          if constexpr (kT) {
            const int ch = (c - half * 64) >> 3;
            const int o0 = (ch ^ (lane & 7)) << 4, o1 = ((ch + 1) ^ (lane & 7)) << 4;
            *reinterpret_cast<uint4*>(hbox + o0) = make_uint4(hp[0], hp[1], hp[2], hp[3]);
            *reinterpret_cast<uint4*>(hbox + o1) = make_uint4(hp[4], hp[5], hp[6], hp[7]);
            *reinterpret_cast<uint4*>(hbox + kTmaBoxBytes + o0) = make_uint4(gp[0], gp[1], gp[2], gp[3]);
            *reinterpret_cast<uint4*>(hbox + kTmaBoxBytes + o1) = make_uint4(gp[4], gp[5], gp[6], gp[7]);
            *reinterpret_cast<uint4*>(hbox + 2 * kTmaBoxBytes + o0) = make_uint4(up[0], up[1], up[2], up[3]);
            *reinterpret_cast<uint4*>(hbox + 2 * kTmaBoxBytes + o1) = make_uint4(up[4], up[5], up[6], up[7]);
            continue;
          }
          __nv_bfloat16* ho = h + (size_t)row * args.ldo + col;
          __nv_bfloat16* go = gu + (size_t)row * args.ldo2 + col;
          __nv_bfloat16* uo = gu + (size_t)row * args.ldo2 + args.inter + col;
          if (nv == 16) {
            reinterpret_cast<uint4*>(ho)[0] = make_uint4(hp[0], hp[1], hp[2], hp[3]);
            reinterpret_cast<uint4*>(ho)[1] = make_uint4(hp[4], hp[5], hp[6], hp[7]);
            reinterpret_cast<uint4*>(go)[0] = make_uint4(gp[0], gp[1], gp[2], gp[3]);
            reinterpret_cast<uint4*>(go)[1] = make_uint4(gp[4], gp[5], gp[6], gp[7]);
            reinterpret_cast<uint4*>(uo)[0] = make_uint4(up[0], up[1], up[2], up[3]);
            reinterpret_cast<uint4*>(uo)[1] = make_uint4(up[4], up[5], up[6], up[7]);
          } else {
            const uint16_t* hs = reinterpret_cast<const uint16_t*>(hp);
            const uint16_t* gs = reinterpret_cast<const uint16_t*>(gp);
            const uint16_t* us = reinterpret_cast<const uint16_t*>(up);
            for (int j = 0; j < nv; ++j) {
              reinterpret_cast<uint16_t*>(ho)[j] = hs[j];
              reinterpret_cast<uint16_t*>(go)[j] = gs[j];
              reinterpret_cast<uint16_t*>(uo)[j] = us[j];
            }
          }
        }
        if constexpr (kT) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int col = ti.n0 + half * 64, y = ti.m0 + quarter * 32;
            if (col < args.N && y < args.M) {
              tma_store_3d(&tmC, hbox, col, y, 0);                        // h [rows][I]
              tma_store_3d(&tmD, hbox + kTmaBoxBytes, col, 0, y);         // gate half of [rows][2][I]
              tma_store_3d(&tmD, hbox + 2 * kTmaBoxBytes, col, 1, y);     // up half
            }
            bulk_commit_group();
          }
        }
      } else if constexpr (E == Epi::SwigluBwd || E == Epi::SwigluBwdTma) {
        // Accumulator = dh for I-columns n0 .. n0+BN-1.  out = dgu [M, 2I].
        // SwigluBwdTma: each 64 columns of dg and du go to two 32 x 64 boxes
        // of this warp (lane = row, chunk j at j ^ (row & 7)), then TMA.
        constexpr bool kT = E == Epi::SwigluBwdTma;
        const __nv_bfloat16* gu = reinterpret_cast<const __nv_bfloat16*>(args.aux);
        __nv_bfloat16* dgu = reinterpret_cast<__nv_bfloat16*>(args.out);
        uint8_t* gbox = tma_stage + (warp - 2) * 2 * kTmaBoxBytes + lane * 128;
#pragma unroll 1
        for (int c2 = half * HALF; c2 < (half + 1) * HALF; c2 += 32) {
          uint32_t rr[2][16];
          uint16_t gvv[2][16], uvv[2][16];
          if constexpr (kT) {
            if (((c2 - half * HALF) & 63) == 0) {
              if (lane == 0) bulk_wait_group_read<0>();   // the boxes' previous stores have read them
            }
          }
          __syncwarp();
          tmem_ld16(tbase + c2, rr[0]);
          tmem_ld16(tbase + c2 + 16, rr[1]);
          // the saved gate / up values of both 16-column groups are requested
          // before any is used
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int col = ti.n0 + c2 + 16 * q;
            if (!row_ok || col >= args.N) continue;
            const int nv = min(16, args.N - col);
            const uint16_t* gsrc = reinterpret_cast<const uint16_t*>(gu + (size_t)row * args.ld_aux + col);
            const uint16_t* usrc = reinterpret_cast<const uint16_t*>(gu + (size_t)row * args.ld_aux + args.inter + col);
            if (nv == 16) {
              *reinterpret_cast<uint4*>(gvv[q]) = reinterpret_cast<const uint4*>(gsrc)[0];
              *reinterpret_cast<uint4*>(gvv[q] + 8) = reinterpret_cast<const uint4*>(gsrc)[1];
              *reinterpret_cast<uint4*>(uvv[q]) = reinterpret_cast<const uint4*>(usrc)[0];
              *reinterpret_cast<uint4*>(uvv[q] + 8) = reinterpret_cast<const uint4*>(usrc)[1];
            } else {
              for (int j = 0; j < 16; ++j) {
                gvv[q][j] = j < nv ? gsrc[j] : 0;
                uvv[q][j] = j < nv ? usrc[j] : 0;
              }
            }
          }
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 2; ++q) {
          const uint32_t (&r)[16] = rr[q];
          const uint16_t (&gv)[16] = gvv[q];
          const uint16_t (&uv)[16] = uvv[q];
          const int c = c2 + 16 * q;
          const int col = ti.n0 + c;
          if (!row_ok || col >= args.N) continue;
          const int nv = min(16, args.N - col);
          uint32_t dg[8], du[8];
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            float o[2][2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const float g = bf16_bits_to_float(gv[j + q]);
              const float u = bf16_bits_to_float(uv[j + q]);
              const float dh = __uint_as_float(r[j + q]);
              const float s = 1.0f / (1.0f + __expf(-g));
              o[0][q] = dh * u * s * (1.0f + g * (1.0f - s));
              o[1][q] = dh * g * s;
            }
            dg[j / 2] = pack_bf16x2(o[0][0], o[0][1]);
            du[j / 2] = pack_bf16x2(o[1][0], o[1][1]);
          }
          if constexpr (kT) {
            const int ch = ((c - half * HALF) & 63) >> 3;
            const int o0 = (ch ^ (lane & 7)) << 4, o1 = ((ch + 1) ^ (lane & 7)) << 4;
            *reinterpret_cast<uint4*>(gbox + o0) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
            *reinterpret_cast<uint4*>(gbox + o1) = make_uint4(dg[4], dg[5], dg[6], dg[7]);
            *reinterpret_cast<uint4*>(gbox + kTmaBoxBytes + o0) = make_uint4(du[0], du[1], du[2], du[3]);
            *reinterpret_cast<uint4*>(gbox + kTmaBoxBytes + o1) = make_uint4(du[4], du[5], du[6], du[7]);
            continue;
          }
          __nv_bfloat16* go = dgu + (size_t)row * args.ldo + col;
          __nv_bfloat16* uo = dgu + (size_t)row * args.ldo + args.inter + col;
          if (nv == 16) {
            reinterpret_cast<uint4*>(go)[0] = make_uint4(dg[0], dg[1], dg[2], dg[3]);
            reinterpret_cast<uint4*>(go)[1] = make_uint4(dg[4], dg[5], dg[6], dg[7]);
            reinterpret_cast<uint4*>(uo)[0] = make_uint4(du[0], du[1], du[2], du[3]);
            reinterpret_cast<uint4*>(uo)[1] = make_uint4(du[4], du[5], du[6], du[7]);
          } else {
            const uint16_t* gs = reinterpret_cast<const uint16_t*>(dg);
            const uint16_t* us = reinterpret_cast<const uint16_t*>(du);
            for (int j = 0; j < nv; ++j) {
              reinterpret_cast<uint16_t*>(go)[j] = gs[j];
              reinterpret_cast<uint16_t*>(uo)[j] = us[j];
            }
          }
          }
          if constexpr (kT) {
            if (((c2 + 32 - half * HALF) & 63) == 0) {   // a 64-column pair of boxes is complete
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                const int col = ti.n0 + (c2 & ~63), y = ti.m0 + quarter * 32;
                if (col < args.N && y < args.M) {
                  tma_store_3d(&tmC, gbox, col, 0, y);                  // dg half of [rows][2][I]
                  tma_store_3d(&tmC, gbox + kTmaBoxBytes, col, 1, y);   // du half
                }
                bulk_commit_group();
              }
            }
          }
        }
      } else if constexpr (E == Epi::CeFwd) {
        const long tgt = row_ok ? args.targets[row] : -1;
        float run_max = -INFINITY, run_sum = 0.0f;
#pragma unroll 1
        for (int c2 = half * HALF; c2 < (half + 1) * HALF; c2 += 32) {
          uint32_t rr[2][16];
          __syncwarp();
          tmem_ld16(tbase + c2, rr[0]);
          tmem_ld16(tbase + c2 + 16, rr[1]);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 2; ++q) {
          const uint32_t (&r)[16] = rr[q];
          const int col = ti.n0 + c2 + 16 * q;
          // exp(x - m) = 2^(x log2(e) - m log2(e)): one FFMA and one ex2 per
          // element; column bounds are only checked in the vocabulary's last tile
          const bool full = col + 16 <= args.N;
          float cmax = -INFINITY;
          if (full) {
#pragma unroll
            for (int j = 0; j < 16; ++j) cmax = fmaxf(cmax, __uint_as_float(r[j]));
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (col + j < args.N) cmax = fmaxf(cmax, __uint_as_float(r[j]));
          }
          if (cmax == -INFINITY) continue;
          const float nm = fmaxf(run_max, cmax);
          const float nml = nm * kLog2e;
          float s = run_sum * ex2_approx((run_max - nm) * kLog2e);
          if (full) {
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 16; ++j) s4[j & 3] += ex2_approx(fmaf(__uint_as_float(r[j]), kLog2e, -nml));
            s += (s4[0] + s4[1]) + (s4[2] + s4[3]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (col + j < args.N) s += ex2_approx(fmaf(__uint_as_float(r[j]), kLog2e, -nml));
          }
          run_sum = s;
          run_max = nm;
          if (tgt >= col && tgt < col + 16 && tgt < args.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (col + j == tgt && row_ok) args.tgt_logit[row] = __uint_as_float(r[j]);
          }
          }
        }
        if (row_ok) {  // two partials per (row, tile): one per column half
          args.part_max[(size_t)row * 2 * args.n_tiles + 2 * ti.n_tile + half] = run_max;
          args.part_sum[(size_t)row * 2 * args.n_tiles + 2 * ti.n_tile + half] = run_sum;
        }
      } else if constexpr (E == Epi::CeBwd || E == Epi::CeBwdTma) {
        const long tgt = row_ok ? args.targets[row] : -1;
        const float l = row_ok ? args.lse[row] : 0.0f;
        const float sc = row_ok ? args.row_scale[row] : 0.0f;
        const float ll = l * kLog2e;
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(args.out) + (size_t)row * args.ldo;
        // CeBwdTma: lane = row of this warp's 32-row box; the 16-byte chunk j
        // of a 64-column box row sits at chunk j ^ (row & 7) (128-byte swizzle)
        uint8_t* box_row = tma_stage + (warp - 2) * 2 * kTmaBoxBytes + lane * 128;
        const int box_y = ti.m0 + quarter * 32;
#pragma unroll 1
        for (int c4 = half * HALF; c4 < (half + 1) * HALF; c4 += 64) {
          uint8_t* brow = box_row + (tma_box & 1) * kTmaBoxBytes;
          if constexpr (kTmaOut) {
            if (lane == 0) bulk_wait_group_read<1>();   // the store that last used this buffer has read it
            __syncwarp();
          }
#pragma unroll 1
          for (int c2 = c4; c2 < c4 + 64; c2 += 32) {
          uint32_t rr[2][16];
          __syncwarp();
          tmem_ld16(tbase + c2, rr[0]);
          tmem_ld16(tbase + c2 + 16, rr[1]);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 2; ++q) {
          const uint32_t (&r)[16] = rr[q];
          const int col = ti.n0 + c2 + 16 * q;
          // out-of-range rows / columns of a TMA box are clipped by the store
          if (!kTmaOut && (!row_ok || col >= args.N)) continue;
          // softmax row (2^(x log2(e) - lse log2(e))) times the row scale; the
          // target column's "- 1" is applied to the one chunk that holds it
          float pv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) pv[j] = ex2_approx(fmaf(__uint_as_float(r[j]), kLog2e, -ll)) * sc;
          if (tgt >= col && tgt < col + 16) {
            const int tj = (int)(tgt - col);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (j == tj) pv[j] -= sc;
          }
          if (kTmaOut && col + 16 > args.N) {
            // the store clips the box at 16-byte granularity: columns N .. N
            // rounded up to 8 are written too, as zeros
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (col + j >= args.N) pv[j] = 0.0f;
          }
          uint32_t pk[8];
#pragma unroll
          for (int j = 0; j < 16; j += 2) pk[j / 2] = pack_bf16x2(pv[j], pv[j + 1]);
          if constexpr (kTmaOut) {
            const int ch = ((c2 - c4) + 16 * q) >> 3;   // first of this group's two 16-byte chunks
            *reinterpret_cast<uint4*>(brow + ((ch ^ (lane & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            *reinterpret_cast<uint4*>(brow + (((ch + 1) ^ (lane & 7)) << 4)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          } else if (col + 16 <= args.N) {
            reinterpret_cast<uint4*>(o + col)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            reinterpret_cast<uint4*>(o + col)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          } else {
            const uint16_t* ps = reinterpret_cast<const uint16_t*>(pk);
            for (int j = 0; col + j < args.N; ++j) reinterpret_cast<uint16_t*>(o + col)[j] = ps[j];
          }
          }
          }
          if constexpr (kTmaOut) {
            fence_proxy_async_smem();   // this lane's box row is visible to the TMA engine
            __syncwarp();
            if (lane == 0) {
              if (ti.n0 + c4 < args.N && box_y < args.M)
                tma_store_2d(&tmC, box_row + (tma_box & 1) * kTmaBoxBytes, ti.n0 + c4, box_y);
              bulk_commit_group();
            }
            ++tma_box;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {   // this warp's TMEM reads are done: release the buffer (on the even CTA)
        if constexpr (CG == 2) mbar_arrive_cluster(cluster_map(smem_u32(&tempty[buf]), 0));
        else mbar_arrive(&tempty[buf]);
      }
      ++local;
    }
    if constexpr (kTmaOut) {
      if (lane == 0) bulk_wait_group_all();   // this warp's stores are done before the CTA's shared memory goes
    }
  }

  if constexpr (E == Epi::ScatterBF16) __threadfence_system();   // this CTA's peer stores before the signal
  tc_fence_before();
  __syncthreads();
  if constexpr (E == Epi::ScatterBF16) {
    if (threadIdx.x == 0) {
      // the last CTA of the grid tells every rank that all rows have landed
      const unsigned int prev = atomicAdd(args.done_ctr, 1u);
      if (prev == gridDim.x - 1) {
        *args.done_ctr = 0u;
        __threadfence_system();
        for (int p = 0; p < args.scatter_ranks; ++p) {
          uint32_t* flag = reinterpret_cast<uint32_t*>(args.peer_base[p] + args.flags_off) +
                           args.scatter_phase * 8 + args.scatter_me;
          asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(flag) : "memory");
        }
      }
    }
  }
  if constexpr (CG == 2) cluster_sync();   // the peer no longer touches this CTA's barriers or TMEM
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (CG == 2) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace dsv3
