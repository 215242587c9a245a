// Expert-parallel MoE token movement over NVLink / NVSwitch peer memory.
//
// Ranks of one box share a symmetric heap (csrc/comm.cu): the same offsets in
// every rank's region, every region mapped into every peer.  Two receive
// layouts:
//
//   owner     routed experts are split into contiguous ranges, rank d owning
//             [d*E/R, (d+1)*E/R), and receives every row routed to them (the
//             layout when each rank holds only its own experts' weights);
//   balanced  (expert weights replicated) the rows of all ranks, in expert
//             order with each expert's range padded to 256, form one global
//             sequence of P rows; rank d receives the contiguous share
//             [d*chunk, (d+1)*chunk), chunk = P / R rounded up to 256.  Every
//             rank then runs the same number of expert rows whatever the
//             routing, an expert's rows may be split between two ranks, and
//             each rank adds its rows' part of the expert weight gradients
//             (the data-parallel gradient sum completes them).
//
// Per MoE layer and micro-batch:
//
//   ep_plan        (1 CTA) all-gathers the per-expert routing counts by P2P
//                  stores + a signal, waits for every rank's counts and
//                  derives, identically on every rank, the receive layout:
//                  on rank d, local expert l owns rows [row_off[l],
//                  row_off[l+1]) (256-row padded), inside which source s
//                  writes its rows from  send_base[e] = row_off[l] +
//                  sum_{s'<s} count[s'][e];  plus the tile -> expert map of the
//                  grouped GEMMs.
//   ep_dispatch    one warp per (token, slot): 16-byte stores of the token's
//                  activation row straight into the owner's receive slot,
//                  with the row's origin (source rank, slot) and gate weight;
//                  zeroes this rank's own padding rows; the last CTA raises
//                  every peer's flag.
//   ep_wait        bounded spin until every peer's flag of a phase arrived.
//   ep_send_back   one warp per received row: stores an expert-output (or
//                  input-gradient) row into the home rank's combine inbox at
//                  the token's slot (plus one float per row in backward).
//   ep_dispatch_bwd the output-gradient rows take the forward routes.
//   ep_bwd_prep    on the expert side: dy = w * dout and dw = <dout, y> per row.
//
// Flags are monotonic counters, one per (phase, source rank) in the receiver's
// region; a sender adds 1 with release semantics after a system fence, a
// waiter keeps its own expected count in local memory, so CUDA-graph replays
// need no host-side sequence numbers.  Every wait is bounded: on timeout the
// kernel records DSV3_ERR_WAIT_PEER in the status word and returns.
// Buffer reuse is ordered by the data flow itself: a rank writes a peer's
// inbox for layer L+1 only after that peer's signal for a later phase that it
// raises after consuming layer L (the count exchange in forward, the combine
// in backward).
//
// No counterpart in the reference, which keeps every expert on one device
// (its DeepSeekMoE gathers rows locally: models/moe.py:108-132).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include "common.cuh"
#include "status.h"

namespace dsv3 {

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxExperts = 256;
enum Phase { PH_COUNTS = 0, PH_DISPATCH = 1, PH_COMBINE = 2, PH_BWD_DISPATCH = 3, PH_BWD_COMBINE = 4, kPhases = 5 };

struct EpArgs {
  unsigned long long peer[kMaxRanks];  // heap base of every rank (peer[me] is this rank's own)
  long long off_flags;                 // uint32 [kPhases][kMaxRanks]   incoming signal counters
  long long off_counts;                // int32  [2][kMaxRanks][E]       routing-count inbox (parity)
  long long off_comb;                  // bf16   [T*k][D]                combine inbox (home side)
  long long off_dw;                    // f32    [T*k]                   gate-weight gradient inbox
  long long off_bwd;                   // bf16   [cap][D]                output-gradient receive rows
  long long off_xs;                    // bf16   [cap][D]  this layer's receive rows
  long long off_origin;                // int32  [cap]     source rank * T*k + slot, -1 on padding
  long long off_w;                     // f32    [cap]     gate weight of the row
  int me, R, E, k, T, D, cap;
  int bal;                             // 1: balanced layout, 0: owner layout
  unsigned long long budget_ns;
};

template <typename T>
__device__ __forceinline__ T* at_rank(const EpArgs& a, int r, long long off) {
  return reinterpret_cast<T*>(a.peer[r] + off);
}

__host__ __device__ __forceinline__ int first_expert(int d, int E, int R) { return (int)(((long long)d * E) / R); }

__device__ __forceinline__ int owner_of(int e, int E, int R) {
  int d = R - 1;
  while (d > 0 && first_expert(d, E, R) > e) --d;
  return d;
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

// After this CTA's stores: the last CTA of the grid raises flag `phase` of
// this rank on every peer (release, after a system-scope fence).
__device__ void grid_done_signal(const EpArgs& a, int phase, unsigned int* done) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      *done = 0u;  // ready for the next launch (stream order)
      __threadfence_system();
      for (int p = 0; p < a.R; ++p) remote_signal(at_rank<uint32_t>(a, p, a.off_flags) + phase * kMaxRanks + a.me);
    }
  }
}

// Copy one D-element bf16 row with the warp's lanes (16-byte chunks): every
// load of the lane is issued before the first store, so a lane keeps up to
// eight 16-byte chunks in flight (rows up to 2048 elements in one pass).
__device__ __forceinline__ void copy_row(const __nv_bfloat16* __restrict__ src, __nv_bfloat16* dst, int D8, int lane) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int base = 0; base < D8; base += 256) {
    uint4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = base + lane + 32 * i;
      if (c < D8) v[i] = s[c];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = base + lane + 32 * i;
      if (c < D8) d[c] = v[i];
    }
  }
}

__global__ void __launch_bounds__(1024) ep_plan_kernel(EpArgs a, const int* __restrict__ counts, uint32_t* expect,
                                                       uint32_t* sendcnt, int* __restrict__ cnt_all,
                                                       int* __restrict__ send_base, int* __restrict__ row_off,
                                                       int* __restrict__ recv_cnt, int* __restrict__ tile_group,
                                                       int max_tiles, int* __restrict__ cursor,
                                                       int* __restrict__ bal_info, unsigned int* status) {
  __shared__ int s_cnt[kMaxRanks * kMaxExperts];
  __shared__ int s_off[kMaxExperts + 1];
  __shared__ int s_start[kMaxExperts + 1];
  __shared__ int s_tot[kMaxExperts];
  __shared__ int s_chunk;
  __shared__ int s_abort;
  const int tid = threadIdx.x, R = a.R, E = a.E;
  if (tid == 0) s_abort = 0;
  const int par = (int)(sendcnt[0] & 1u);
  // 1. my counts -> inbox[par][me][:] of every rank (myself included)
  for (int i = tid; i < R * E; i += blockDim.x) {
    const int p = i / E, e = i - p * E;
    at_rank<int>(a, p, a.off_counts)[(par * kMaxRanks + a.me) * E + e] = counts[e];
  }
  for (int e = tid; e < E; e += blockDim.x) cursor[e] = 0;
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    sendcnt[0] += 1u;
    for (int p = 0; p < R; ++p) remote_signal(at_rank<uint32_t>(a, p, a.off_flags) + PH_COUNTS * kMaxRanks + a.me);
  }
  // 2. every rank's counts arrived
  if (tid < R) {
    const uint32_t target = expect[PH_COUNTS * kMaxRanks + tid] + 1u;
    const uint32_t* f = at_rank<uint32_t>(a, a.me, a.off_flags) + PH_COUNTS * kMaxRanks + tid;
    if (!wait_count(f, target, a.budget_ns, status)) s_abort = 1;
    expect[PH_COUNTS * kMaxRanks + tid] = target;
  }
  __syncthreads();
  const volatile int* inbox = at_rank<int>(a, a.me, a.off_counts) + par * kMaxRanks * E;
  for (int i = tid; i < R * E; i += blockDim.x) {
    const int v = s_abort ? 0 : inbox[i];  // after a timeout the plan is empty
    s_cnt[i] = v;
    cnt_all[i] = v;
  }
  __syncthreads();
  // 3. layout of every rank's receive slot (each rank computes all of them)
  if (a.bal) {
    // balanced: global expert-ordered sequence cut into R equal shares
    for (int e = tid; e < E; e += blockDim.x) {
      int tot = 0;
      for (int s = 0; s < R; ++s) tot += s_cnt[s * E + e];
      s_tot[e] = tot;
    }
    __syncthreads();
    if (tid == 0) {
      int acc = 0;
      for (int e = 0; e < E; ++e) {
        s_start[e] = acc;
        acc += (s_tot[e] + 255) / 256 * 256;
      }
      s_start[E] = acc;
      s_chunk = max(256, ((acc + R - 1) / R + 255) / 256 * 256);
    }
    __syncthreads();
    const int chunk = s_chunk, lo = a.me * chunk;
    const int used = max(0, min(chunk, s_start[E] - lo));
    for (int e = tid; e < E; e += blockDim.x) {
      int pre = 0;
      for (int s = 0; s < a.me; ++s) pre += s_cnt[s * E + e];
      send_base[e] = s_start[e] + pre;                       // global position of my first row of e
      s_off[e] = min(max(s_start[e] - lo, 0), used);
      recv_cnt[e] = min(max(s_start[e] + s_tot[e] - lo, 0), used) - s_off[e];   // real rows of e in my share
    }
    if (tid == 0) {
      s_off[E] = used;
      bal_info[0] = chunk;
      bal_info[1] = used;
      if (chunk > a.cap) record_error(status, DSV3_ERR_BOUNDS);   // receive capacity exceeded
    }
    __syncthreads();
    for (int i = tid; i <= E; i += blockDim.x) row_off[i] = s_off[i];
    for (int i = tid; i < max_tiles; i += blockDim.x) {
      const int row = i * 128;
      int g = -1;
      if (row < used) {
        int l = 0, h = E - 1;  // last e with s_off[e] <= row: the expert whose rows hold `row`
        while (l < h) {
          const int mid = (l + h + 1) >> 1;
          if (s_off[mid] <= row) l = mid;
          else h = mid - 1;
        }
        g = l;
      }
      tile_group[i] = g;
    }
    return;
  }
  const int e_lo = first_expert(a.me, E, R), Eloc = first_expert(a.me + 1, E, R) - e_lo;
  if (tid < R) {
    const int d = tid, e0 = first_expert(d, E, R), e1 = first_expert(d + 1, E, R);
    int seg = 0;
    for (int e = e0; e < e1; ++e) {
      int tot = 0, pre = 0;
      for (int s = 0; s < R; ++s) {
        const int c = s_cnt[s * E + e];
        tot += c;
        if (s < a.me) pre += c;
      }
      send_base[e] = seg + pre;
      if (d == a.me) {
        s_off[e - e0] = min(seg, a.cap);
        recv_cnt[e - e0] = tot;
      }
      seg += (tot + 255) / 256 * 256;   // 256-row ranges: the grouped GEMMs may pair CTAs
    }
    if (d == a.me) {
      s_off[e1 - e0] = min(seg, a.cap);
      if (seg > a.cap) record_error(status, DSV3_ERR_BOUNDS);  // receive capacity exceeded
    }
  }
  __syncthreads();
  for (int i = tid; i <= Eloc; i += blockDim.x) row_off[i] = s_off[i];
  const int used = s_off[Eloc];
  for (int i = tid; i < max_tiles; i += blockDim.x) {
    const int row = i * 128;
    int g = -1;
    if (row < used) {
      int lo = 0, hi = Eloc - 1;  // last l with s_off[l] <= row
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_off[mid] <= row) lo = mid;
        else hi = mid - 1;
      }
      g = lo;
    }
    tile_group[i] = g;
  }
}

__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpArgs a, const __nv_bfloat16* __restrict__ x, long ldx,
                                                          const int* __restrict__ idx, const float* __restrict__ w,
                                                          const int* __restrict__ send_base, int* cursor,
                                                          int* __restrict__ route, const int* __restrict__ row_off,
                                                          const int* __restrict__ recv_cnt, int Eloc,
                                                          const int* __restrict__ bal_info, unsigned int* done,
                                                          unsigned int* status) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
  const int TK = a.T * a.k, D8 = a.D / 8;
  const int chunk = a.bal ? bal_info[0] : 0;
  for (int i = warp; i < TK; i += nwarps) {
    int row = 0, d = 0;
    if (lane == 0) {
      const int e = idx[i];
      if (a.bal) {
        const int gp = send_base[e] + atomicAdd(&cursor[e], 1);   // global position in expert order
        d = gp / chunk;
        row = gp - d * chunk;
        if (d >= a.R) {
          record_error(status, DSV3_ERR_BOUNDS);
          d = 0;
          row = a.cap;
        }
      } else {
        d = owner_of(e, a.E, a.R);
        row = send_base[e] + atomicAdd(&cursor[e], 1);
      }
      if (row >= a.cap) {
        record_error(status, DSV3_ERR_BOUNDS);
        row = -1;
      }
      route[i] = row;
      route[TK + i] = d;
      if (row >= 0) {
        at_rank<int>(a, d, a.off_origin)[row] = a.me * TK + i;
        at_rank<float>(a, d, a.off_w)[row] = w[i];
      }
    }
    row = __shfl_sync(0xffffffffu, row, 0);
    d = __shfl_sync(0xffffffffu, d, 0);
    if (row < 0) continue;
    copy_row(x + (size_t)(i / a.k) * ldx, at_rank<__nv_bfloat16>(a, d, a.off_xs) + (size_t)row * a.D, D8, lane);
  }
  // this rank's own padding rows: zero activations, no origin
  __nv_bfloat16* xs = at_rank<__nv_bfloat16>(a, a.me, a.off_xs);
  int* origin = at_rank<int>(a, a.me, a.off_origin);
  float* wrow = at_rank<float>(a, a.me, a.off_w);
  for (int p = warp; p < Eloc * 256; p += nwarps) {
    const int l = p >> 8, j = p & 255;
    const int r = row_off[l] + recv_cnt[l] + j;
    if (r < row_off[l + 1]) {
      uint4* o = reinterpret_cast<uint4*>(xs + (size_t)r * a.D);
      for (int c = lane; c < D8; c += 32) o[c] = make_uint4(0, 0, 0, 0);
      if (lane == 0) {
        origin[r] = -1;
        wrow[r] = 0.f;
      }
    }
  }
  grid_done_signal(a, PH_DISPATCH, done);
}

__global__ void __launch_bounds__(256) ep_dispatch_bwd_kernel(EpArgs a, const __nv_bfloat16* __restrict__ g, long ldg,
                                                              const int* __restrict__ route, unsigned int* done) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
  const int TK = a.T * a.k, D8 = a.D / 8;
  for (int i = warp; i < TK; i += nwarps) {
    const int row = route[i], d = route[TK + i];
    if (row < 0) continue;
    copy_row(g + (size_t)(i / a.k) * ldg, at_rank<__nv_bfloat16>(a, d, a.off_bwd) + (size_t)row * a.D, D8, lane);
  }
  grid_done_signal(a, PH_BWD_DISPATCH, done);
}

__global__ void ep_wait_kernel(EpArgs a, int phase, uint32_t* expect, unsigned int* status) {
  const int p = threadIdx.x;
  if (p < a.R) {
    const uint32_t target = expect[phase * kMaxRanks + p] + 1u;
    wait_count(at_rank<uint32_t>(a, a.me, a.off_flags) + phase * kMaxRanks + p, target, a.budget_ns, status);
    expect[phase * kMaxRanks + p] = target;
  }
}

__global__ void __launch_bounds__(256) ep_send_back_kernel(EpArgs a, int phase, const __nv_bfloat16* __restrict__ rows,
                                                           long ldr, const float* __restrict__ extra,
                                                           const int* __restrict__ row_off, int Eloc,
                                                           unsigned int* done, unsigned int* status) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
  const int TK = a.T * a.k, D8 = a.D / 8;
  const int used = row_off[Eloc];
  const int* origin = at_rank<int>(a, a.me, a.off_origin);
  for (int r = warp; r < used; r += nwarps) {
    const int o = origin[r];
    if (o < 0) continue;
    const int s = o / TK, i = o - s * TK;
    if (s >= a.R) {  // only after a failed exchange left stale metadata
      if (lane == 0) record_error(status, DSV3_ERR_BOUNDS);
      continue;
    }
    copy_row(rows + (size_t)r * ldr, at_rank<__nv_bfloat16>(a, s, a.off_comb) + (size_t)i * a.D, D8, lane);
    if (extra != nullptr && lane == 0) at_rank<float>(a, s, a.off_dw)[i] = extra[r];
  }
  grid_done_signal(a, phase, done);
}

// Expert side of the combine backward: dy[r] = w[r] * dout[r], dw[r] = <dout[r], y[r]>.
__global__ void __launch_bounds__(256) ep_bwd_prep_kernel(EpArgs a, const __nv_bfloat16* __restrict__ y, long ldy,
                                                          const int* __restrict__ row_off, int Eloc,
                                                          __nv_bfloat16* __restrict__ dy, long lddy,
                                                          float* __restrict__ dw) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
  const int D8 = a.D / 8;
  const int used = row_off[Eloc];
  const int* origin = at_rank<int>(a, a.me, a.off_origin);
  const float* wrow = at_rank<float>(a, a.me, a.off_w);
  const __nv_bfloat16* g = at_rank<__nv_bfloat16>(a, a.me, a.off_bwd);
  for (int r = warp; r < used; r += nwarps) {
    uint4* o = reinterpret_cast<uint4*>(dy + (size_t)r * lddy);
    if (origin[r] < 0) {
      for (int c = lane; c < D8; c += 32) o[c] = make_uint4(0, 0, 0, 0);
      if (lane == 0) dw[r] = 0.f;
      continue;
    }
    const float wr = wrow[r];
    const uint4* gr = reinterpret_cast<const uint4*>(g + (size_t)r * a.D);
    const uint4* yr = reinterpret_cast<const uint4*>(y + (size_t)r * ldy);
    float dot = 0.f;
    for (int c = lane; c < D8; c += 32) {
      const uint4 gv = gr[c], yv = yr[c];
      const uint16_t* gh = reinterpret_cast<const uint16_t*>(&gv);
      const uint16_t* yh = reinterpret_cast<const uint16_t*>(&yv);
      uint32_t pk[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const float g0 = bf16_bits_to_float(gh[i]), g1 = bf16_bits_to_float(gh[i + 1]);
        dot += g0 * bf16_bits_to_float(yh[i]) + g1 * bf16_bits_to_float(yh[i + 1]);
        pk[i / 2] = pack_bf16x2(g0 * wr, g1 * wr);
      }
      o[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[r] = dot;
  }
}

// ---------------------------------------------------------------- host side

int sm_count() {
  int dev = 0, n = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

// peers: heap base per rank; offs: [flags, counts, comb, dw, bwd, xs, origin, w];
// dims: [me, R, E, k, T, D, cap, budget_ns(, balanced)]
EpArgs make_args(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, const std::vector<int64_t>& dims) {
  TORCH_CHECK(offs.size() == 8 && (dims.size() == 8 || dims.size() == 9), "ep: offs has 8 entries, dims 8 or 9");
  EpArgs a{};
  const int R = (int)dims[1];
  TORCH_CHECK(R >= 1 && R <= kMaxRanks && (int)peers.size() == R, "ep: 1..8 ranks, one heap base per rank");
  for (int r = 0; r < R; ++r) a.peer[r] = (unsigned long long)peers[r];
  a.off_flags = offs[0];
  a.off_counts = offs[1];
  a.off_comb = offs[2];
  a.off_dw = offs[3];
  a.off_bwd = offs[4];
  a.off_xs = offs[5];
  a.off_origin = offs[6];
  a.off_w = offs[7];
  for (int i = 0; i < 8; ++i) TORCH_CHECK(offs[i] % 16 == 0, "ep: heap offsets must be 16-byte aligned");
  a.me = (int)dims[0];
  a.R = R;
  a.E = (int)dims[2];
  a.k = (int)dims[3];
  a.T = (int)dims[4];
  a.D = (int)dims[5];
  a.cap = (int)dims[6];
  a.budget_ns = (unsigned long long)dims[7];
  a.bal = dims.size() == 9 ? (int)(dims[8] != 0) : 0;
  TORCH_CHECK(a.me >= 0 && a.me < R, "ep: rank out of range");
  TORCH_CHECK(a.E >= R && a.E <= kMaxExperts, "ep: R <= E <= 256");
  TORCH_CHECK(a.D % 8 == 0 && a.cap % 256 == 0, "ep: D % 8 == 0, capacity a multiple of 256");
  TORCH_CHECK((long long)R * a.T * a.k < (1ll << 31), "ep: R*T*k must fit int32");
  return a;
}

// weight groups of the receive layout: this rank's experts (owner) or all experts (balanced)
int local_experts(const EpArgs& a) {
  return a.bal ? a.E : first_expert(a.me + 1, a.E, a.R) - first_expert(a.me, a.E, a.R);
}

const int* bal_ptr(const EpArgs& a, const c10::optional<at::Tensor>& bal_info) {
  if (!a.bal) return nullptr;
  TORCH_CHECK(bal_info.has_value() && bal_info->scalar_type() == at::kInt && bal_info->numel() >= 2,
              "ep: the balanced layout needs bal_info (int32 [>= 2])");
  return bal_info->data_ptr<int>();
}

const __nv_bfloat16* cbf(const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
__nv_bfloat16* bf(at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
uint32_t* u32(at::Tensor& t) { return reinterpret_cast<uint32_t*>(t.data_ptr()); }

int copy_grid(long rows) {
  const long want = (rows + 7) / 8;
  return (int)std::max(1L, std::min(want, (long)sm_count() * 8));
}

}  // namespace

void ep_plan(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, const std::vector<int64_t>& dims,
             const at::Tensor& counts, at::Tensor& expect, at::Tensor& sendcnt, at::Tensor& cnt_all,
             at::Tensor& send_base, at::Tensor& row_off, at::Tensor& recv_cnt, at::Tensor& tile_group,
             at::Tensor& cursor, const c10::optional<at::Tensor>& bal_info) {
  const EpArgs a = make_args(peers, offs, dims);
  const int* bal = bal_ptr(a, bal_info);
  const int Eloc = local_experts(a);
  TORCH_CHECK(counts.numel() == a.E && cnt_all.numel() == a.R * a.E && send_base.numel() == a.E &&
                  row_off.numel() == Eloc + 1 && recv_cnt.numel() == Eloc && cursor.numel() == a.E,
              "ep_plan: buffer sizes");
  TORCH_CHECK(tile_group.numel() * 128 >= a.cap, "ep_plan: tile_group must cover the capacity");
  const at::cuda::CUDAGuard guard(counts.device());
  ep_plan_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(a, counts.data_ptr<int>(), u32(expect),
      u32(sendcnt), cnt_all.data_ptr<int>(), send_base.data_ptr<int>(), row_off.data_ptr<int>(),
      recv_cnt.data_ptr<int>(), tile_group.data_ptr<int>(), (int)tile_group.numel(), cursor.data_ptr<int>(),
      const_cast<int*>(bal), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_dispatch(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, const std::vector<int64_t>& dims,
                 const at::Tensor& x, const at::Tensor& idx, const at::Tensor& w, const at::Tensor& send_base,
                 at::Tensor& cursor, at::Tensor& route, const at::Tensor& row_off, const at::Tensor& recv_cnt,
                 at::Tensor& done, const c10::optional<at::Tensor>& bal_info) {
  const EpArgs a = make_args(peers, offs, dims);
  const int* bal = bal_ptr(a, bal_info);
  TORCH_CHECK(x.size(0) == a.T && x.size(1) == a.D && x.stride(1) == 1 && x.stride(0) % 8 == 0,
              "ep_dispatch: x [T, D] with 16-byte rows");
  TORCH_CHECK(idx.numel() == (long)a.T * a.k && w.numel() == idx.numel() && route.numel() == 2 * idx.numel(),
              "ep_dispatch: idx / w [T, k], route [2, T*k]");
  const at::cuda::CUDAGuard guard(x.device());
  ep_dispatch_kernel<<<copy_grid((long)a.T * a.k), 256, 0, at::cuda::getCurrentCUDAStream()>>>(a, cbf(x), x.stride(0),
      idx.data_ptr<int>(), w.data_ptr<float>(), send_base.data_ptr<int>(), cursor.data_ptr<int>(),
      route.data_ptr<int>(), row_off.data_ptr<int>(), recv_cnt.data_ptr<int>(), local_experts(a), bal, u32(done),
      status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_dispatch_bwd(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs,
                     const std::vector<int64_t>& dims, const at::Tensor& g, const at::Tensor& route, at::Tensor& done) {
  const EpArgs a = make_args(peers, offs, dims);
  TORCH_CHECK(g.size(0) == a.T && g.size(1) == a.D && g.stride(1) == 1 && g.stride(0) % 8 == 0,
              "ep_dispatch_bwd: g [T, D] with 16-byte rows");
  const at::cuda::CUDAGuard guard(g.device());
  ep_dispatch_bwd_kernel<<<copy_grid((long)a.T * a.k), 256, 0, at::cuda::getCurrentCUDAStream()>>>(a, cbf(g),
      g.stride(0), route.data_ptr<int>(), u32(done));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_wait(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, const std::vector<int64_t>& dims,
             int64_t phase, at::Tensor& expect) {
  const EpArgs a = make_args(peers, offs, dims);
  TORCH_CHECK(phase >= 0 && phase < kPhases, "ep_wait: bad phase");
  const at::cuda::CUDAGuard guard(expect.device());
  ep_wait_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(a, (int)phase, u32(expect), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_send_back(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, const std::vector<int64_t>& dims,
                  int64_t phase, const at::Tensor& rows, const c10::optional<at::Tensor>& extra,
                  const at::Tensor& row_off, at::Tensor& done) {
  const EpArgs a = make_args(peers, offs, dims);
  TORCH_CHECK(phase == PH_COMBINE || phase == PH_BWD_COMBINE, "ep_send_back: combine phases only");
  TORCH_CHECK(rows.size(0) >= a.cap && rows.size(1) == a.D && rows.stride(1) == 1 && rows.stride(0) % 8 == 0,
              "ep_send_back: rows [cap, D] with 16-byte rows");
  const float* ex = extra.has_value() ? extra->data_ptr<float>() : nullptr;
  const at::cuda::CUDAGuard guard(rows.device());
  ep_send_back_kernel<<<copy_grid(a.cap), 256, 0, at::cuda::getCurrentCUDAStream()>>>(a, (int)phase, cbf(rows),
      rows.stride(0), ex, row_off.data_ptr<int>(), local_experts(a), u32(done), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_bwd_prep(const std::vector<int64_t>& peers, const std::vector<int64_t>& offs, const std::vector<int64_t>& dims,
                 const at::Tensor& y, const at::Tensor& row_off, at::Tensor& dy, at::Tensor& dw) {
  const EpArgs a = make_args(peers, offs, dims);
  TORCH_CHECK(y.size(0) >= a.cap && dy.size(0) >= a.cap && dw.numel() >= a.cap, "ep_bwd_prep: [cap] rows");
  TORCH_CHECK(y.stride(0) % 8 == 0 && dy.stride(0) % 8 == 0, "ep_bwd_prep: 16-byte rows");
  const at::cuda::CUDAGuard guard(y.device());
  ep_bwd_prep_kernel<<<copy_grid(a.cap), 256, 0, at::cuda::getCurrentCUDAStream()>>>(a, cbf(y), y.stride(0),
      row_off.data_ptr<int>(), local_experts(a), bf(dy), dy.stride(0), dw.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_ep(pybind11::module_& m) {
  m.def("ep_plan", &ep_plan, "all-gather routing counts over peer memory and build the receive layout",
        pybind11::arg("peers"), pybind11::arg("offs"), pybind11::arg("dims"), pybind11::arg("counts"),
        pybind11::arg("expect"), pybind11::arg("sendcnt"), pybind11::arg("cnt_all"), pybind11::arg("send_base"),
        pybind11::arg("row_off"), pybind11::arg("recv_cnt"), pybind11::arg("tile_group"), pybind11::arg("cursor"),
        pybind11::arg("bal_info") = pybind11::none());
  m.def("ep_dispatch", &ep_dispatch, "store routed token rows into their receive slots (P2P)",
        pybind11::arg("peers"), pybind11::arg("offs"), pybind11::arg("dims"), pybind11::arg("x"), pybind11::arg("idx"),
        pybind11::arg("w"), pybind11::arg("send_base"), pybind11::arg("cursor"), pybind11::arg("route"),
        pybind11::arg("row_off"), pybind11::arg("recv_cnt"), pybind11::arg("done"),
        pybind11::arg("bal_info") = pybind11::none());
  m.def("ep_dispatch_bwd", &ep_dispatch_bwd, "send output-gradient rows along the forward routes (P2P)");
  m.def("ep_wait", &ep_wait, "bounded wait for every peer's signal of a phase");
  m.def("ep_send_back", &ep_send_back, "store per-row results into the home ranks' combine inbox (P2P)");
  m.def("ep_bwd_prep", &ep_bwd_prep, "expert-side combine backward: w * dout and <dout, y> per row");
}

}  // namespace dsv3
