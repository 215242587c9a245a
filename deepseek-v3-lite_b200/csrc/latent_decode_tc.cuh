// tcgen05 absorbed-MLA decode over the latent cache (sm_100a).  Included by
// latent_decode.cuh inside each user's anonymous namespace.
//
// Work item = (query row b, group of 16 heads, split of 256 cache rows);
// persistent CTAs (two per SM) walk items.  Per 128-row tile of the cache
// (latent R columns + rope columns, cache batch b / qpb):
//
//   S^T [128 rows x 16 heads]  = K [128 x (R + 64)] . Q^T           (TMEM cols 0..15)
//   softmax over the 128 rows of each head column (4 warps, one row each)
//   O^T [R x 16] += V^T [R x 128] . P^T [128 x 16]                  (TMEM, 16 cols per 128 latent)
//
// The tile is staged by TMA as 64-column chunks of 128 rows (16 KB, 128-byte
// swizzle) through a ring of kLtcSlots slots.  Per tile the ring carries the
// S pass (latent chunks 0 .. NCL-1, the rope chunk zero-filled past dr, and
// one empty use so the next pass starts on an even slot), then the PV pass
// (latent chunks 0 .. NCL-1 again, read MN-major in adjacent slot pairs 2m,
// 2m+1 as the A operand of output block m).  The PV pass re-reads the tile's
// latent part a few microseconds after the S pass brought it in, so it comes
// from L2, not DRAM; in exchange the ring is small enough for two CTAs per SM,
// and loads run ahead of the tensor core through both passes and across
// tiles.  Chunks wholly past R are empty uses (no copy, no S MMA; the PV rows
// they feed are latent dims past R, which are discarded).
//
// Warp roles: 0 = TMA producer, 1 = MMA issuer (owns TMEM), 2..5 = softmax /
// epilogue (warp w reads TMEM lanes 32 * (w % 4) ..; the four warps meet at a
// shared-counter barrier with a time budget, never at an unbounded one).  The running max is
// kept per head and only moved (with a rescale of O^T and the row sums) when
// a tile's max exceeds it by more than 2^8, so most tiles never touch O^T.
// Partials (max in natural-log units, sum, O) use the split-K layout of the
// merge kernel.  Every wait is bounded (status word + abort flag).

constexpr int kLtcThreads = 192;          // producer, MMA, 4 softmax warps
constexpr int kLtcChunk = 128 * 128;      // one 64-column x 128-row bf16 chunk (bytes)
constexpr int kLtcQChunk = 16 * 128;      // 16 heads x 64 columns (bytes)
constexpr int kLtcSlots = 4;              // ring slots (even: PV pairs sit in slots 2i, 2i+1)

template <int NCL>
struct LtcCfg {
  static constexpr int NCH = NCL + 1;                    // + the rope chunk
  static constexpr int USES = 2 * NCL + 2;               // ring uses per tile: S pass (NCL + 2), PV pass (NCL)
  static constexpr int OFF_Q = kLtcSlots * kLtcChunk;
  static constexpr int OFF_P = OFF_Q + NCH * kLtcQChunk;  // P: two [16][64] K-major chunks
  static constexpr int OFF_RED = OFF_P + 2 * kLtcQChunk;  // [2][4][16] floats + [4][16] floats
  static constexpr int OFF_BAR = OFF_RED + (2 * 4 * 16 + 4 * 16) * 4;
  static constexpr int NBAR = 2 * kLtcSlots + 6;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;   // + TMEM slot, abort flag, sync counter; slack
  static constexpr int TMEM_COLS = 128;                  // S^T at 0, O^T block m at 32 + 16 m
};

// Barrier of the four softmax warps with a time budget (a hardware named
// barrier cannot give up): lane 0 of each warp counts itself in and spins on
// the shared counter.  `epoch` is this thread's count of passed barriers.
// Returns false (abort flag raised) if the others do not arrive in time.
__device__ __forceinline__ bool ltc_sync(unsigned int* ctr, unsigned int& epoch, volatile int* abort_flag,
                                         unsigned int* status) {
  __syncwarp();
  int ok = 1;
  ++epoch;
  if ((threadIdx.x & 31) == 0) {
    __threadfence_block();
    atomicAdd(ctr, 1u);
    const unsigned int target = 4u * epoch;
    volatile unsigned int* vc = ctr;
    if (*vc < target) {
      const uint64_t t0 = globaltimer_ns();
      while (*vc < target) {
        if (*abort_flag || globaltimer_ns() - t0 > DSV3_WAIT_BUDGET_NS) {
          record_error(status, DSV3_ERR_WAIT_FULL);
          *abort_flag = 1;
          ok = 0;
          break;
        }
      }
    }
    __threadfence_block();
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int NCL>
__global__ void __launch_bounds__(kLtcThreads, 2) latent_decode_tc_kernel(
    const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_pe,
    const bf16* __restrict__ q_lat, const bf16* __restrict__ q_pe, const int* __restrict__ lens, int B, int H, int R,
    int dr, int qpb, int nsplit, float scale_log2, float* __restrict__ part_m, float* __restrict__ part_l,
    float* __restrict__ part_o, unsigned int* status) {
  using C = LtcCfg<NCL>;
  constexpr int NCH = C::NCH;
  constexpr int NMB = NCL / 2;                            // 128-wide output blocks
  extern __shared__ __align__(1024) uint8_t ltc_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ltc_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);       // [2][4][16] tile maxima
  float* red_l = red + 2 * 4 * 16;                                // [4][16] row sums
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + kLtcSlots;
  uint64_t* s_full = empty + kLtcSlots;
  uint64_t* p_full = s_full + 1;
  uint64_t* pv_done = p_full + 1;
  uint64_t* q_ready = pv_done + 1;
  uint64_t* o_free = q_ready + 1;
  uint64_t* drain = o_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  unsigned int* sync_ctr = reinterpret_cast<unsigned int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HG = (H + 15) / 16;
  const int items = B * HG * nsplit;

  if (threadIdx.x == 0) {
    for (int c = 0; c < kLtcSlots; ++c) {
      mbar_init(&full[c], 1);
      mbar_init(&empty[c], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(q_ready, 4);
    mbar_init(o_free, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    *sync_ctr = 0u;
    fence_barrier_init();
    tma_prefetch_desc(&tm_kv);
    tma_prefetch_desc(&tm_pe);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // item -> (b, head group, split, first row, rows, tiles); every role derives the same
  auto decode_item = [&](int it, int& b, int& hg, int& split, int& r0, int& r1, int& nt) {
    split = it % nsplit;
    const int rest = it / nsplit;
    hg = rest % HG;
    b = rest / HG;
    const int len = lens[b];
    r0 = split * 256;
    r1 = min(len, r0 + 256);
    nt = r1 > r0 ? (r1 - r0 + 127) / 128 : 0;
  };

  // ring use v of a tile: 0 .. NCL-1 S-pass latent chunk v, NCL the rope
  // chunk, NCL + 1 empty, NCL + 2 .. 2 NCL + 1 PV-pass latent chunk
  // v - NCL - 2; a latent chunk wholly past R is an empty use
  auto use_chunk = [&](int v) { return v < NCL ? v : (v == NCL ? NCL : (v == NCL + 1 ? -1 : v - NCL - 2)); };
  auto use_loads = [&](int v) {
    const int c = use_chunk(v);
    return c == NCL || (c >= 0 && 64 * c < R);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t g = 0;           // ring uses so far: slot g % kLtcSlots, phase (g / kLtcSlots) & 1
      uint32_t last_phase = 0;  // per slot: phase its latest use completes
      bool ok = true;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        int b, hg, split, r0, r1, nt;
        decode_item(it, b, hg, split, r0, r1, nt);
        const int cb = b / qpb;
        for (int t = 0; t < nt && ok; ++t) {
          const int row = r0 + 128 * t;
          for (int v = 0; v < C::USES; ++v, ++g) {
            const int slot = g % kLtcSlots;
            const uint32_t ph = (g / kLtcSlots) & 1u;
            if (!mbar_wait_bounded(&empty[slot], ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_EMPTY)) {
              ok = false;
              break;
            }
            const int c = use_chunk(v);
            if (use_loads(v)) {
              mbar_arrive_expect_tx(&full[slot], kLtcChunk);
              if (c < NCL) tma_load_3d(smem + slot * kLtcChunk, &tm_kv, &full[slot], 64 * c, row, cb);
              else tma_load_3d(smem + slot * kLtcChunk, &tm_pe, &full[slot], 0, row, cb);
            } else {
              mbar_arrive(&full[slot]);   // an empty use completes its phase at once
            }
            last_phase = (last_phase & ~(1u << slot)) | (ph << slot);
          }
        }
      }
      // every issued copy lands before the CTA may exit
      const uint32_t used = g < (uint32_t)kLtcSlots ? g : (uint32_t)kLtcSlots;
      for (uint32_t sl = 0; sl < used; ++sl)
        mbar_wait_bounded(&full[sl], (last_phase >> sl) & 1u, nullptr, status, DSV3_ERR_WAIT_FULL);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t I_S = idesc_bf16_f32(128, 16, 0, 0);    // S^T = K Q^T
      constexpr uint32_t I_O = idesc_bf16_f32(128, 16, 1, 0);    // O^T += V^T P^T (V^T read MN-major)
      const uint32_t base = smem_u32(smem);
      const uint32_t q_s = base + C::OFF_Q, p_s = base + C::OFF_P;
      uint32_t g = 0, tiles = 0, items_done = 0;
      bool ok = true, issued_any = false;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        int b, hg, split, r0, r1, nt;
        decode_item(it, b, hg, split, r0, r1, nt);
        if (nt == 0) continue;
        if (!mbar_wait_bounded(q_ready, items_done & 1u, abort_flag, status, DSV3_ERR_WAIT_FULL)) break;
        tc_fence_after();
        for (int t = 0; t < nt; ++t, ++tiles) {
          const uint32_t ph = tiles & 1u;
          // S pass: S^T += chunk . Q^T(chunk), each slot released by the commit after its MMAs
          uint32_t acc = 0;
          for (int v = 0; v < NCL + 2; ++v, ++g) {
            const int slot = g % kLtcSlots;
            if (!mbar_wait_bounded(&full[slot], (g / kLtcSlots) & 1u, abort_flag, status, DSV3_ERR_WAIT_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const int c = use_chunk(v);
            if (use_loads(v)) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                umma_bf16(tmem, smem_desc_sw128(base + slot * kLtcChunk + kk * 32, 16, 1024),
                          smem_desc_sw128(q_s + c * kLtcQChunk + kk * 32, 16, 1024), I_S, acc);
                acc = 1;
              }
              issued_any = true;
            }
            umma_commit(&empty[slot]);
          }
          if (!ok) break;
          umma_commit(s_full);
          if (!mbar_wait_bounded(p_full, ph, abort_flag, status, DSV3_ERR_WAIT_FULL)) {
            ok = false;
            break;
          }
          if (t == 0 && items_done > 0) {   // the previous item's O^T has been read out
            if (!mbar_wait_bounded(o_free, (items_done - 1) & 1u, abort_flag, status, DSV3_ERR_WAIT_TMEM)) {
              ok = false;
              break;
            }
          }
          tc_fence_after();
          // PV pass: output block m reads latent chunks 2m, 2m+1 from slots s, s+1
#pragma unroll 1
          for (int m = 0; m < NMB && ok; ++m, g += 2) {
            const int slot = g % kLtcSlots;   // even
            const uint32_t sph = (g / kLtcSlots) & 1u;
            if (!mbar_wait_bounded(&full[slot], sph, abort_flag, status, DSV3_ERR_WAIT_FULL) ||
                !mbar_wait_bounded(&full[slot + 1], sph, abort_flag, status, DSV3_ERR_WAIT_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              umma_bf16(tmem + 32 + 16 * m,
                        smem_desc_sw128(base + slot * kLtcChunk + kk * 2048, kLtcChunk, 1024),
                        smem_desc_sw128(p_s + (kk >> 2) * kLtcQChunk + (kk & 3) * 32, 16, 1024), I_O,
                        (t > 0 || kk > 0) ? 1u : 0u);
            }
            issued_any = true;
            umma_commit(&empty[slot]);
            umma_commit(&empty[slot + 1]);
          }
          if (!ok) break;
          umma_commit(pv_done);
        }
        ++items_done;
      }
      // no MMA may still write TMEM when it is freed
      if (issued_any) {
        umma_commit(drain);
        mbar_wait_bounded(drain, 0, nullptr, status, DSV3_ERR_WAIT_TMEM);
      }
    }
  } else {
    // ---------------------------------------------------- softmax / epilogue
    const int quarter = warp & 3;
    const int sw = warp - 2;                       // softmax warp 0..3
    const int tid = threadIdx.x - 64;              // 0..127 (plain loads / stores)
    const int trow = quarter * 32 + lane;          // TMEM lane = tile row (S^T) / latent dim (O^T)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    unsigned int epoch = 0;
    uint8_t* q_sm = smem + C::OFF_Q;
    uint8_t* p_sm = smem + C::OFF_P;
    uint32_t tiles = 0, items_done = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      int b, hg, split, r0, r1, nt;
      decode_item(it, b, hg, split, r0, r1, nt);
      const int h0 = hg * 16;
      if (nt == 0) {   // nothing of this row's cache in this split (the merge skips its O)
        if (tid < 16 && h0 + tid < H) {
          part_m[(size_t)(b * H + h0 + tid) * nsplit + split] = -INFINITY;
          part_l[(size_t)(b * H + h0 + tid) * nsplit + split] = 0.f;
        }
        continue;
      }
      // queries of the 16 heads as NCH chunks of [16][64] (128-byte swizzle;
      // zeros past H, past R and past dr): thread tid moves 16-byte unit
      // tid % 8 of head tid / 8 in every chunk, all loads issued before the
      // first store
      {
        const int h = tid >> 3, j = tid & 7;
        const bool hv = h0 + h < H;
        const size_t qrow = (size_t)b * H + h0 + h;
        uint4 v[NCH];
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          v[c] = make_uint4(0, 0, 0, 0);
          if (hv) {
            if (c < NCL) {
              if (64 * c + 8 * j < R) v[c] = *reinterpret_cast<const uint4*>(q_lat + qrow * R + 64 * c + 8 * j);
            } else if (8 * j < dr) {
              v[c] = *reinterpret_cast<const uint4*>(q_pe + qrow * dr + 8 * j);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < NCH; ++c)
          *reinterpret_cast<uint4*>(q_sm + c * kLtcQChunk + h * 128 + ((j ^ (h & 7)) << 4)) = v[c];
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);

      float m_use[16], l_part[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        m_use[h] = -INFINITY;
        l_part[h] = 0.f;
      }
      for (int t = 0; t < nt; ++t, ++tiles) {
        const uint32_t ph = tiles & 1u;
        if (!mbar_wait_bounded(s_full, ph, abort_flag, status, DSV3_ERR_WAIT_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[16];
        tmem_ld16(tmem + lane_base, sr);
        tmem_ld_wait();
        const int row = r0 + 128 * t + trow;
        const bool live = row < r1;
        float s[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) s[h] = live ? __uint_as_float(sr[h]) * scale_log2 : -INFINITY;
        // per-head maxima of the tile: warp butterflies, then across the 4 warps
        float* rt = red + (tiles & 1u) * 64;
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          float v = s[h];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
          if (lane == h) rt[sw * 16 + h] = v;
        }
        if (!ltc_sync(sync_ctr, epoch, abort_flag, status)) {
          ok = false;
          break;
        }
        bool any_move = false;
        float corr[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float tmax = fmaxf(fmaxf(rt[h], rt[16 + h]), fmaxf(rt[32 + h], rt[48 + h]));
          corr[h] = 1.f;
          // move the reference max only when this tile exceeds it by 2^8
          if (tmax > m_use[h] + 8.f) {
            corr[h] = m_use[h] == -INFINITY ? 0.f : ex2_approx(m_use[h] - tmax);
            m_use[h] = tmax;
            any_move = true;
          }
        }
        // P and O^T of the previous tile are no longer in use by the tensor core
        if (t > 0 && !mbar_wait_bounded(pv_done, ph ^ 1u, abort_flag, status, DSV3_ERR_WAIT_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (any_move) {
#pragma unroll
          for (int h = 0; h < 16; ++h) l_part[h] *= corr[h];
          if (t > 0) {   // the first tile of an item overwrites O^T
#pragma unroll 1
            for (int m = 0; m < NMB; ++m) {
              uint32_t o[16];
              tmem_ld16(tmem + lane_base + 32 + 16 * m, o);
              tmem_ld_wait();
#pragma unroll
              for (int h = 0; h < 16; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * corr[h]);
              tmem_st16(tmem + lane_base + 32 + 16 * m, o);
            }
            tmem_st_wait();
          }
        }
        // p = 2^(s - m); P^T as [16 heads][128 rows] K-major (two 64-row chunks)
        uint8_t* pc = p_sm + (trow >> 6) * kLtcQChunk;
        const int k = trow & 63;
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float p = live ? ex2_approx(s[h] - m_use[h]) : 0.f;
          l_part[h] += p;
          *reinterpret_cast<__nv_bfloat16*>(pc + h * 128 + (((k >> 3) ^ (h & 7)) << 4) + (k & 7) * 2) =
              __float2bfloat16(p);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      if (!ok) break;
      // ---- item epilogue: row sums, maxima, O^T -> partials
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float v = warp_sum(l_part[h]);
        if (lane == h) red_l[sw * 16 + h] = v;
      }
      if (!mbar_wait_bounded(pv_done, (tiles - 1) & 1u, abort_flag, status, DSV3_ERR_WAIT_TMEM)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (!ltc_sync(sync_ctr, epoch, abort_flag, status)) {
        ok = false;
        break;
      }
      constexpr float kLn2 = 0.69314718055994531f;
      if (tid < 16 && h0 + tid < H) {
        float mv = 0.f;   // every thread holds the same maxima; pick head `tid` without dynamic indexing
#pragma unroll
        for (int h = 0; h < 16; ++h)
          if (h == tid) mv = m_use[h];
        const size_t pi = (size_t)(b * H + h0 + tid) * nsplit + split;
        part_m[pi] = mv * kLn2;
        part_l[pi] = red_l[tid] + red_l[16 + tid] + red_l[32 + tid] + red_l[48 + tid];
      }
#pragma unroll 1
      for (int m = 0; m < NMB; ++m) {
        uint32_t o[16];
        tmem_ld16(tmem + lane_base + 32 + 16 * m, o);
        tmem_ld_wait();
        const int col = 128 * m + trow;    // latent dim of this lane
        if (col < R) {
#pragma unroll
          for (int h = 0; h < 16; ++h)
            if (h0 + h < H) part_o[((size_t)(b * H + h0 + h) * nsplit + split) * R + col] = __uint_as_float(o[h]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
      if (!ltc_sync(sync_ctr, epoch, abort_flag, status)) break;   // red_l is rewritten by the next item
      ++items_done;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// -------------------------------------------------------------- host side
typedef CUresult (*LtcEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline LtcEncodeFn ltc_encode_fn() {
  static LtcEncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (LtcEncodeFn) nullptr;
    return reinterpret_cast<LtcEncodeFn>(p);
  }();
  return fn;
}

// 3-D bf16 map [batches][rows][cols] with row stride `cols` elements, box
// 64 columns x 128 rows, 128-byte swizzle, zero fill out of bounds.
inline bool ltc_map(CUtensorMap* m, const void* ptr, int cols, long rows, long batches, long batch_stride) {
  LtcEncodeFn fn = ltc_encode_fn();
  if (fn == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || (cols * 2) % 16 != 0 ||
      (batch_stride * 2) % 16 != 0)
    return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batches};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)batch_stride * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline int ltc_num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}
