// Split-K absorbed-MLA decode kernels over the latent cache, shared by the
// torch entry point (attention.cu) and the allocation-free C entry point
// (latent_decode_noalloc.cu).  Device code only; included inside an
// anonymous namespace by each user.
#pragma once
#include "common.cuh"
#include "mma_sync.cuh"
#include "latent_decode_tc.cuh"

// Absorbed decode: per (batch row b, head h): scores over cache rows
// [0, len_b) = q_lat . kv + q_pe . pe, softmax, out = sum p * kv (latent R).
// Split-K over the sequence: split s handles rows [s*chunk, (s+1)*chunk) and
// writes (max, sum, partial out); a second kernel merges the splits.
// One warp per (b, h, split); R <= 1024.
__global__ void latent_decode_split_kernel(const bf16* __restrict__ q_lat, const bf16* __restrict__ q_pe,
                                           const bf16* __restrict__ kv, const bf16* __restrict__ pe,
                                           const int* __restrict__ lens, int H, int R, int dr, long kv_bs, long pe_bs,
                                           int qpb, int chunk, int nsplit, int BH, float scale,
                                           float* __restrict__ part_m,
                                           float* __restrict__ part_l, float* __restrict__ part_o) {
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int split = warp_global % nsplit;
  const int bh = warp_global / nsplit;
  // query row b (its own causal length lens[b]) reads cache batch b / qpb
  const int b = bh / H, h = bh % H;
  if (bh >= BH) return;
  const int cb = b / qpb;
  const int len = lens[b];
  const int r0 = split * chunk, r1 = min(len, r0 + chunk);
  float ql[32], qp[4];  // R <= 1024 (32 per lane), dr <= 128
  for (int i = 0; i < 32; ++i) ql[i] = (lane + 32 * i < R) ? __bfloat162float(q_lat[((size_t)b * H + h) * R + lane + 32 * i]) : 0.f;
  for (int i = 0; i < 4; ++i) qp[i] = (lane + 32 * i < dr) ? __bfloat162float(q_pe[((size_t)b * H + h) * dr + lane + 32 * i]) : 0.f;
  float m = -INFINITY, l = 0.f;
  float acc[32];
  for (int i = 0; i < 32; ++i) acc[i] = 0.f;
  for (int r = r0; r < r1; ++r) {
    const bf16* kr = kv + (size_t)cb * kv_bs + (size_t)r * R;
    const bf16* pr = pe + (size_t)cb * pe_bs + (size_t)r * dr;
    float kvv[32];
    float dot = 0.f;
    for (int i = 0; i < 32; ++i) {
      kvv[i] = (lane + 32 * i < R) ? __bfloat162float(kr[lane + 32 * i]) : 0.f;
      dot += ql[i] * kvv[i];
    }
    for (int i = 0; i < 4; ++i) dot += (lane + 32 * i < dr) ? qp[i] * __bfloat162float(pr[lane + 32 * i]) : 0.f;
    dot = warp_sum(dot) * scale;
    const float nm = fmaxf(m, dot);
    const float c = __expf(m - nm), p = __expf(dot - nm);
    l = l * c + p;
    for (int i = 0; i < 32; ++i) acc[i] = acc[i] * c + p * kvv[i];
    m = nm;
  }
  const size_t pi = (size_t)bh * nsplit + split;
  if (lane == 0) {
    part_m[pi] = m;
    part_l[pi] = l;
  }
  for (int i = 0; i < 32; ++i)
    if (lane + 32 * i < R) part_o[pi * R + lane + 32 * i] = acc[i];
}

__global__ void latent_decode_merge_kernel(const float* __restrict__ part_m, const float* __restrict__ part_l,
                                           const float* __restrict__ part_o, int nsplit, int R, int BH,
                                           bf16* __restrict__ out) {
  const int bh = blockIdx.x;
  if (bh >= BH) return;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_m[(size_t)bh * nsplit + s]);
  float Lsum = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float ms = part_m[(size_t)bh * nsplit + s];
    if (ms != -INFINITY) Lsum += part_l[(size_t)bh * nsplit + s] * __expf(ms - M);
  }
  for (int c = threadIdx.x; c < R; c += blockDim.x) {
    float v = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float ms = part_m[(size_t)bh * nsplit + s];
      if (ms != -INFINITY) v += part_o[((size_t)bh * nsplit + s) * R + c] * __expf(ms - M);
    }
    out[(size_t)bh * R + c] = __float2bfloat16(Lsum > 0.f ? v / Lsum : 0.f);
  }
}


// Tensor-core absorbed decode (warp-level mma.sync m16n8k16).  One CTA per
// (query row b, group of 16 heads, split of `chunk` cache rows).  Each 64-row
// tile of the cache (R latent + DRP zero-padded rope columns) is staged in
// shared memory once (cp.async, double-buffered) and serves all 16 heads:
//   S[16 x 64]  = Q[16 x (R + DRP)] . K^T      warp w: cache rows w*64/NW ..
//   row max / sum of the tile across the NW warps through shared memory
//   O[16 x R]  += P[16 x 64] . V[64 x R]       warp w: output columns w*R/NW ..
// V is the latent part of the same tile, so every cache byte is read once
// per 16 heads.  With 8 warps each warp takes 8 cache rows and runs the two
// halves of the score reduction as independent MMA chains.  Partials (max in
// natural-log units, sum, O) have the layout the merge kernel above expects.
template <int R, int DRP, int NW, int TK = 64>
__global__ void __launch_bounds__(32 * NW) latent_decode_mma_kernel(
    const bf16* __restrict__ q_lat, const bf16* __restrict__ q_pe, const bf16* __restrict__ kv,
    const bf16* __restrict__ pe, const int* __restrict__ lens, int H, int dr, long kv_bs, long pe_bs, int qpb,
    int chunk, int nsplit, float scale_log2, float* __restrict__ part_m, float* __restrict__ part_l,
    float* __restrict__ part_o) {
  constexpr int DK = R + DRP, KS = DK + 8, PS = TK + 8, RW = R / NW, KPW = TK / NW, NT = 32 * NW;
  static_assert(DRP % 16 == 0 && RW % 16 == 0 && (KPW == 8 || KPW == 16), "latent decode tiling");
  extern __shared__ __align__(16) uint8_t ld_smem[];
  bf16* sQ = reinterpret_cast<bf16*>(ld_smem);           // [16][KS]
  bf16* sK = sQ + 16 * KS;                                // [2][TK][KS]
  bf16* sP = sK + 2 * TK * KS;                            // [16][PS]
  float* red = reinterpret_cast<float*>(sP + 16 * PS);    // [2][NW][16]: tile row max, tile row sum
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int split = blockIdx.x, h0 = blockIdx.y * 16, b = blockIdx.z;
  const int cb = b / qpb;
  const int len = lens[b];
  const int r0 = split * chunk, r1 = min(len, r0 + chunk);
  const bf16* kvb = kv + (size_t)cb * kv_bs;
  const bf16* peb = pe + (size_t)cb * pe_bs;
  const int drc = dr / 8;                                 // 16-byte chunks of a rope row

  if (r0 >= r1) {  // nothing of this row's cache in this split
    for (int i = tid; i < 16 * R; i += NT) {
      const int h = h0 + i / R;
      if (h < H) part_o[((size_t)(b * H + h) * nsplit + split) * R + i % R] = 0.f;
    }
    if (tid < 16 && h0 + tid < H) {
      part_m[(size_t)(b * H + h0 + tid) * nsplit + split] = -INFINITY;
      part_l[(size_t)(b * H + h0 + tid) * nsplit + split] = 0.f;
    }
    return;
  }

  // queries of the 16 heads (zeros past H and past dr)
  for (int c = tid; c < 16 * (DK / 8); c += NT) {
    const int i = c / (DK / 8), cc = c % (DK / 8), h = h0 + i;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h < H) {
      if (cc < R / 8) v = *reinterpret_cast<const uint4*>(q_lat + ((size_t)b * H + h) * R + cc * 8);
      else if (cc - R / 8 < drc) v = *reinterpret_cast<const uint4*>(q_pe + ((size_t)b * H + h) * dr + (cc - R / 8) * 8);
    }
    *reinterpret_cast<uint4*>(sQ + i * KS + cc * 8) = v;
  }
  auto load_tile = [&](int t, int st) {
    bf16* dst = sK + st * TK * KS;
    const int base = r0 + t * TK;
    for (int c = tid; c < TK * (DK / 8); c += NT) {
      const int i = c / (DK / 8), cc = c % (DK / 8), r = base + i;
      const bool row_ok = r < r1;
      if (cc < R / 8) {
        cp_async16(dst + i * KS + cc * 8, kvb + (size_t)(row_ok ? r : r0) * R + cc * 8, row_ok);
      } else {
        const int pc = cc - R / 8;
        const bool ok = row_ok && pc < drc;
        cp_async16(dst + i * KS + cc * 8, peb + (size_t)(ok ? r : r0) * dr + (ok ? pc : 0) * 8, ok);
      }
    }
  };

  const int ntiles = (r1 - r0 + TK - 1) / TK;
  load_tile(0, 0);
  cp_async_commit();
  float o[RW / 8][4];
#pragma unroll
  for (int n = 0; n < RW / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  constexpr int NS = KPW / 8;                             // 8-key score tiles per warp

  for (int t = 0; t < ntiles; ++t) {
    const int st = t & 1;
    if (t + 1 < ntiles) load_tile(t + 1, st ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const bf16* ks = sK + st * TK * KS;
    float s[NS][4];
#pragma unroll
    for (int j = 0; j < NS; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    if constexpr (KPW == 16) {
#pragma unroll 4
      for (int kk = 0; kk < DK / 16; ++kk) {
        uint32_t a[4], bb[4];
        ldsm_x4(a, sQ + ((lane & 7) + 8 * ((lane >> 3) & 1)) * KS + kk * 16 + 8 * (lane >> 4));
        ldsm_x4(bb, ks + (warp * 16 + (lane & 7) + 8 * (lane >> 4)) * KS + kk * 16 + 8 * ((lane >> 3) & 1));
        mma16816(s[0], a, bb[0], bb[1]);
        mma16816(s[NS - 1], a, bb[2], bb[3]);
      }
    } else {
      // 8 cache rows per warp: one B load covers two k-steps, accumulated in
      // two independent chains (even / odd k-steps) that are added at the end.
      float s2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int kk = 0; kk < DK / 16; kk += 2) {
        uint32_t a0[4], a1[4], bb[4];
        ldsm_x4(bb, ks + (warp * 8 + (lane & 7)) * KS + kk * 16 + 8 * (lane >> 3));
        ldsm_x4(a0, sQ + ((lane & 7) + 8 * ((lane >> 3) & 1)) * KS + kk * 16 + 8 * (lane >> 4));
        mma16816(s[0], a0, bb[0], bb[1]);
        if (kk + 1 < DK / 16) {
          ldsm_x4(a1, sQ + ((lane & 7) + 8 * ((lane >> 3) & 1)) * KS + (kk + 1) * 16 + 8 * (lane >> 4));
          mma16816(s2, a1, bb[2], bb[3]);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) s[0][e] += s2[e];
    }
    // scale + mask rows past the cache length; this warp's row maxima
    const int kbase = r0 + t * TK + warp * KPW;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < NS; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = kbase + j * 8 + 2 * tig + (e & 1);
        const float v = col < r1 ? s[j][e] * scale_log2 : -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    if (tig == 0) {
      red[warp * 16 + g] = mx[0];
      red[warp * 16 + g + 8] = mx[1];
    }
    __syncthreads();
    float m_new[2], corr[2], msub[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = g + 8 * r;
      float tmax = red[row];
#pragma unroll
      for (int w = 1; w < NW; ++w) tmax = fmaxf(tmax, red[w * 16 + row]);
      m_new[r] = fmaxf(m_run[r], tmax);
      msub[r] = m_new[r] == -INFINITY ? 0.f : m_new[r];
      corr[r] = m_run[r] == -INFINITY ? 0.f : exp2f(m_run[r] - m_new[r]);
    }
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const float p0 = exp2f(s[j][0] - msub[0]), p1 = exp2f(s[j][1] - msub[0]);
      const float p2 = exp2f(s[j][2] - msub[1]), p3 = exp2f(s[j][3] - msub[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int col = warp * KPW + j * 8 + 2 * tig;
      *reinterpret_cast<uint32_t*>(sP + g * PS + col) = pack_bf16x2(p0, p1);
      *reinterpret_cast<uint32_t*>(sP + (g + 8) * PS + col) = pack_bf16x2(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
    }
    if (tig == 0) {
      red[NW * 16 + warp * 16 + g] = rs[0];
      red[NW * 16 + warp * 16 + g + 8] = rs[1];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = g + 8 * r;
      float tsum = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) tsum += red[NW * 16 + w * 16 + row];
      l_run[r] = l_run[r] * corr[r] + tsum;
      m_run[r] = m_new[r];
    }
#pragma unroll
    for (int n = 0; n < RW / 8; ++n) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
    // O[:, warp's columns] += P . V  (V = the latent columns of the tile)
#pragma unroll
    for (int kc = 0; kc < TK / 16; ++kc) {
      uint32_t a[4];
      ldsm_x4(a, sP + ((lane & 7) + 8 * ((lane >> 3) & 1)) * PS + kc * 16 + 8 * (lane >> 4));
#pragma unroll
      for (int dp = 0; dp < RW / 16; ++dp) {
        uint32_t bb[4];
        ldsm_x4_t(bb, ks + (kc * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * KS + warp * RW + dp * 16 + 8 * (lane >> 4));
        mma16816(o[2 * dp], a, bb[0], bb[1]);
        mma16816(o[2 * dp + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  constexpr float kLn2 = 0.69314718055994531f;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int h = h0 + g + 8 * r;
    if (h >= H) continue;
    const size_t pi = (size_t)(b * H + h) * nsplit + split;
    if (warp == 0 && tig == 0) {
      part_m[pi] = m_run[r] * kLn2;
      part_l[pi] = l_run[r];
    }
    float* po = part_o + pi * R + warp * RW;
#pragma unroll
    for (int n = 0; n < RW / 8; ++n)
      *reinterpret_cast<float2*>(po + n * 8 + 2 * tig) = make_float2(o[n][2 * r], o[n][2 * r + 1]);
  }
}

// ---------------------------------------------------------------------------
// Host-side launcher shared by both entry points (no torch types): picks the
// tensor-core kernel when the sizes fit one of its instantiations, else the
// per-warp kernel, then the merge.  Scratch layout: part_m [B*H*nsplit],
// part_l [B*H*nsplit], part_o [B*H*nsplit*R] (fp32).  Returns the first
// launch error (each launch goes through cudaLaunchKernelEx, whose return
// value is that launch's own status).
struct LatentDecodeArgs {
  const bf16* q_lat;
  const bf16* q_pe;
  const bf16* kv;
  const bf16* pe;
  const int* lens;
  int B, H, R, dr;
  long kv_bs, pe_bs;   // batch strides of the caches (elements)
  int qpb;             // query rows per cache batch row
  int max_len;
  float scale;
  float* scratch;
  bf16* out;
  long cache_rows;          // rows per cache batch (0: kv_bs / R)
  int cache_batches;        // cache batch rows (0: ceil(B / qpb))
  unsigned int* status;     // device status word for bounded-wait failures (may be null)
};

// DSV3_DECODE_TILE=64 selects the one-CTA-per-SM 64-row tiles for R 512.
inline bool latent_small_tiles() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("DSV3_DECODE_TILE");
    v = (e != nullptr && e[0] == '6') ? 0 : 1;
  }
  return v == 1;
}

inline int latent_decode_nsplit(int max_len) { return max_len < 1 ? 1 : (max_len + 255) / 256; }

inline long long latent_decode_scratch_floats(int B, int H, int R, int max_len) {
  return (long long)B * H * latent_decode_nsplit(max_len) * (2 + R);
}

template <typename Kern, typename... Args>
inline cudaError_t launch_ex(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Which kernel latent_decode runs where the tcgen05 one fits: mode 1 =
// tcgen05 (latent_decode_tc.cuh), 0 = the warp-level mma.sync kernel, 2 =
// automatic (the default): tcgen05 for a latent rank of 384 or more, where it
// is faster (measured on the MLA decode case, R 512: 120 us against 149 us),
// mma.sync below (R 192: 41 us against 39 us).  DSV3_DECODE_TC=0/1 sets the
// initial mode.
inline int& latent_tc_mode() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("DSV3_DECODE_TC");
    v = e == nullptr ? 2 : (e[0] == '1' ? 1 : (e[0] == '0' ? 0 : 2));
  }
  return v;
}

inline bool latent_tc_enabled(int R) {
  const int v = latent_tc_mode();
  return v == 1 || (v == 2 && R >= 384);
}

// tcgen05 kernel for NCL latent chunks of 64 columns (NCL / 2 output blocks
// of 128).  Sets *done = false (and launches nothing) when a tensor map
// cannot describe the caches.
template <int NCL>
inline cudaError_t launch_latent_tc(const LatentDecodeArgs& a, int nsplit, float* pm, float* pl, float* po,
                                    cudaStream_t st, bool* done) {
  *done = false;
  const long rows = a.cache_rows > 0 ? a.cache_rows : a.kv_bs / a.R;
  const long prow = a.cache_rows > 0 ? a.cache_rows : a.pe_bs / a.dr;
  const long nb = a.cache_batches > 0 ? a.cache_batches : (a.B + a.qpb - 1) / a.qpb;
  CUtensorMap tkv, tpe;
  if (rows < 1 || prow < 1 || !ltc_map(&tkv, a.kv, a.R, rows, nb, a.kv_bs) || !ltc_map(&tpe, a.pe, a.dr, prow, nb, a.pe_bs))
    return cudaSuccess;
  auto kern = latent_decode_tc_kernel<NCL>;
  constexpr int smem = LtcCfg<NCL>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const int items = a.B * ((a.H + 15) / 16) * nsplit;
  const int ctas = 2 * ltc_num_sms();   // two persistent CTAs per SM
  const int grid = items < ctas ? items : ctas;
  *done = true;
  return launch_ex(kern, dim3(grid), dim3(kLtcThreads), (size_t)smem, st, tkv, tpe, a.q_lat, a.q_pe, a.lens, a.B,
                   a.H, a.R, a.dr, a.qpb, nsplit, (float)(a.scale * 1.4426950408889634), pm, pl, po, a.status);
}

template <int R, int DRP, int NW, int TK = 64>
inline cudaError_t launch_latent_mma(const LatentDecodeArgs& a, int nsplit, float* pm, float* pl, float* po,
                                     cudaStream_t st) {
  constexpr int KS = R + DRP + 8;
  constexpr size_t smem = (size_t)(16 * KS + 2 * TK * KS + 16 * (TK + 8)) * 2 + 2 * NW * 16 * 4;
  auto kern = latent_decode_mma_kernel<R, DRP, NW, TK>;
  // the shared-memory opt-in is per device: set it on every call (cheap, host only)
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_ex(kern, dim3(nsplit, (a.H + 15) / 16, a.B), dim3(32 * NW), smem, st, a.q_lat, a.q_pe, a.kv, a.pe,
                   a.lens, a.H, a.dr, a.kv_bs, a.pe_bs, a.qpb, 256, nsplit, (float)(a.scale * 1.4426950408889634),
                   pm, pl, po);
}

inline cudaError_t launch_latent_decode(const LatentDecodeArgs& a, cudaStream_t st) {
  const int nsplit = latent_decode_nsplit(a.max_len);
  float* pm = a.scratch;
  float* pl = pm + (long long)a.B * a.H * nsplit;
  float* po = pl + (long long)a.B * a.H * nsplit;
  cudaError_t e = cudaErrorNotSupported;
  // tcgen05 kernel: R a multiple of 64 up to 512, rope width a multiple of 8
  // up to 64, 16-byte aligned rows and batches
  const bool tc_ok = latent_tc_enabled(a.R) && a.R % 64 == 0 && a.R <= 512 && a.dr % 8 == 0 && a.dr > 0 &&
                     a.dr <= 64 && a.kv_bs % 8 == 0 && a.pe_bs % 8 == 0 && a.B > 0 &&
                     (reinterpret_cast<uintptr_t>(a.q_lat) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.q_pe) & 15) == 0;
  if (tc_ok) {
    bool done = false;
    const int ncl = (a.R + 127) / 128 * 2;
    if (ncl == 2) e = launch_latent_tc<2>(a, nsplit, pm, pl, po, st, &done);
    else if (ncl == 4) e = launch_latent_tc<4>(a, nsplit, pm, pl, po, st, &done);
    else if (ncl == 6) e = launch_latent_tc<6>(a, nsplit, pm, pl, po, st, &done);
    else e = launch_latent_tc<8>(a, nsplit, pm, pl, po, st, &done);
    if (e != cudaSuccess) return e;
    if (!done) e = cudaErrorNotSupported;
  }
  const int drp = (a.dr + 15) / 16 * 16;
  // warp-level tensor-core kernel where the tcgen05 one did not launch
  const bool mma_ok = e == cudaErrorNotSupported && a.dr % 8 == 0 && a.dr <= 64 && a.kv_bs % 8 == 0 &&
                      a.pe_bs % 8 == 0;
#define DSV3_LD_CASE(R_, DRP_, NW_) \
  if (mma_ok && a.R == R_ && drp == DRP_) e = launch_latent_mma<R_, DRP_, NW_>(a, nsplit, pm, pl, po, st);
  // R 512: 32-row cache tiles and 4 warps keep shared memory at ~95 KB, so two
  // CTAs share an SM and one's loads overlap the other's synchronisation
  if (mma_ok && a.R == 512 && drp == 64 && latent_small_tiles())
    e = launch_latent_mma<512, 64, 4, 32>(a, nsplit, pm, pl, po, st);
  else DSV3_LD_CASE(512, 64, 8)
  DSV3_LD_CASE(192, 32, 4)
  DSV3_LD_CASE(128, 32, 8)
  DSV3_LD_CASE(64, 16, 4)
#undef DSV3_LD_CASE
  if (e == cudaErrorNotSupported) {
    const int warps = a.B * a.H * nsplit;
    e = launch_ex(latent_decode_split_kernel, dim3((warps + 3) / 4), dim3(128), 0, st, a.q_lat, a.q_pe, a.kv, a.pe,
                  a.lens, a.H, a.R, a.dr, a.kv_bs, a.pe_bs, a.qpb, 256, nsplit, a.B * a.H, a.scale, pm, pl, po);
  }
  if (e != cudaSuccess) return e;
  return launch_ex(latent_decode_merge_kernel, dim3(a.B * a.H), dim3(128), 0, st, (const float*)pm, (const float*)pl,
                   (const float*)po, nsplit, a.R, a.B * a.H, a.out);
}
