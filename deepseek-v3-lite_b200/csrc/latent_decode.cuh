// Split-K absorbed-MLA decode kernels over the latent cache, shared by the
// torch entry point (attention.cu) and the allocation-free C entry point
// (latent_decode_noalloc.cu).  Device code only; included inside an
// anonymous namespace by each user.
#pragma once
#include "common.cuh"

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

