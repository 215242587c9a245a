// Host side of the tcgen05 GEMM engine: TMA tensor-map construction and the
// typed entry points used by ops/*.py (dense forward / data-gradient /
// weight-gradient, expert-grouped variants, fused SwiGLU and LM-head
// cross-entropy).  Every entry point runs on the current CUDA stream.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>

#include "gemm_sm100.cuh"
#include "status.h"
#include "tma_host.h"

namespace dsv3 {

namespace {

// A operand, K-major: logical [rows, K] with row stride ld (elements).
CUtensorMap map_a_kmajor(const at::Tensor& t, int64_t rows, int64_t K, int64_t ld) {
  uint64_t dims[2] = {(uint64_t)K, (uint64_t)rows};
  uint64_t st[1] = {(uint64_t)ld * 2};
  uint32_t box[2] = {64, 128};
  return make_map(t.data_ptr(), 2, dims, st, box);
}

// A operand, MN-major: logical [Ktot, rows] with the output-row dim contiguous.
CUtensorMap map_a_mnmajor(const at::Tensor& t, int64_t rows, int64_t Ktot, int64_t ld) {
  uint64_t dims[2] = {(uint64_t)rows, (uint64_t)Ktot};
  uint64_t st[1] = {(uint64_t)ld * 2};
  uint32_t box[2] = {64, 64};
  return make_map(t.data_ptr(), 2, dims, st, box);
}

// B operand, K-major, grouped: [G][N][K], rows of length K (stride ld), group stride gs.
CUtensorMap map_b_kmajor(const at::Tensor& t, int64_t G, int64_t N, int64_t K, int64_t ld, int64_t gs) {
  uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)G};
  uint64_t st[2] = {(uint64_t)ld * 2, (uint64_t)gs * 2};
  uint32_t box[3] = {64, 128, 1};
  return make_map(t.data_ptr(), 3, dims, st, box);
}

// B operand, MN-major, grouped: [G][Kred][N] with N contiguous.
CUtensorMap map_b_mnmajor(const at::Tensor& t, int64_t G, int64_t Kred, int64_t N, int64_t ld, int64_t gs) {
  uint64_t dims[3] = {(uint64_t)N, (uint64_t)Kred, (uint64_t)G};
  uint64_t st[2] = {(uint64_t)ld * 2, (uint64_t)gs * 2};
  uint32_t box[3] = {64, 64, 1};
  return make_map(t.data_ptr(), 3, dims, st, box);
}

// SwiGLU weights [G][2][I][K] (gate rows, then up rows, per group).
CUtensorMap map_b_swiglu(const at::Tensor& t, int64_t G, int64_t I, int64_t K) {
  uint64_t dims[4] = {(uint64_t)K, (uint64_t)I, 2, (uint64_t)G};
  uint64_t st[3] = {(uint64_t)K * 2, (uint64_t)I * K * 2, (uint64_t)2 * I * K * 2};
  uint32_t box[4] = {64, 128, 1, 1};
  return make_map(t.data_ptr(), 4, dims, st, box);
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

int cdiv(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// CTA-pair tiles (cta_group::2, 256 x BN per pair) for the schedules whose
// tiles need not share one expert per 128 rows; DSV3_GEMM_PAIRS=0 disables.
int g_pairs = -1;

bool use_pairs() {
  if (g_pairs < 0) {
    const char* e = getenv("DSV3_GEMM_PAIRS");
    g_pairs = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return g_pairs == 1;
}

// tc: the output's tensor map for the TMA-store epilogues (unused otherwise)
template <int BN, int A_MN, int B_MN, Sched S, Epi E, bool SW, int CG>
void launch_cg(const CUtensorMap& ta, const CUtensorMap& tb, GemmArgs& a, const CUtensorMap* tc = nullptr,
               const CUtensorMap* td = nullptr) {
  using C = GemmCfg<BN, CG, E>;
  auto kern = gemm_sm100_kernel<BN, A_MN, B_MN, S, E, SW, CG>;
  constexpr int kSmem = C::SMEM_BYTES + epi_smem_bytes<E>();
  static_assert(kSmem <= 232448, "GEMM shared memory budget");
  static int max_units = 0;   // resident CTAs (CG = 1) or clusters (CG = 2)
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  if constexpr (CG == 2) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  if (max_units == 0) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    if constexpr (CG == 2) {
      cfg.gridDim = dim3(2 * (num_sms() / 2));
      int clusters = 0;
      C10_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
      max_units = std::max(1, clusters);
    } else {
      max_units = num_sms();
    }
  }
  if (a.num_tiles <= 0) return;
  a.status = status_ptr();
  const int units = std::min(a.num_tiles, max_units);
  cfg.gridDim = dim3(units * CG);
  CUtensorMap none;
  memset(&none, 0, sizeof(none));
  TORCH_CHECK(tc != nullptr || !epi_tma(E), "TMA-store epilogue without an output map");
  TORCH_CHECK(td != nullptr || E != Epi::SwigluFwdTma, "SwiGLU TMA epilogue without the gate / up map");
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc != nullptr ? *tc : none, td != nullptr ? *td : none, a));
}

template <int BN, int A_MN, int B_MN, Sched S, Epi E, bool SW>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, GemmArgs& a, const CUtensorMap* tc = nullptr,
            const CUtensorMap* td = nullptr) {
  if constexpr (BN == 256 || (BN == 128 && B_MN)) {
    // row-grouped tiles may pair only when every expert range is 256-aligned
    const bool grouping_ok = S != Sched::GroupedM || a.tile_rows == 256;
    if (use_pairs() && grouping_ok && a.m_tiles > 0 && a.M >= 256) {
      GemmArgs b = a;                      // re-tile the rows in 256-row pair tiles
      b.m_tiles = cdiv(a.M, 256);
      b.num_tiles = a.num_tiles / a.m_tiles * b.m_tiles;
      launch_cg<BN, A_MN, B_MN, S, E, SW, 2>(ta, tb, b, tc, td);
      return;
    }
  }
  launch_cg<BN, A_MN, B_MN, S, E, SW, 1>(ta, tb, a, tc, td);
}

// LM-head tiles walk 16,384-row panels, rows fastest: the panel's hidden rows
// (25 MB at D 768) stay in L2 while the vocabulary weight (154 MB at V 100K,
// more than the 126 MB L2) streams through once per panel instead of once
// per 256-row tile.  DSV3_CE_PANEL_ROWS overrides (0: columns fastest).
int ce_panel_rows() {
  static int rows = -1;
  if (rows < 0) {
    const char* e = getenv("DSV3_CE_PANEL_ROWS");
    rows = e != nullptr ? std::max(0, atoi(e)) : 16384;
  }
  return rows;
}

// CE-gradient epilogue: bf16 dlogits staged in shared memory and written by
// TMA stores (default) or stored row by row from registers (DSV3_CE_TMA_STORE=0).
bool ce_tma_store() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("DSV3_CE_TMA_STORE");
    on = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// fp32 GEMM outputs staged in shared memory and written (or added, for the
// accumulating and split-K modes) by TMA; DSV3_GEMM_TMA_EPI=0 keeps the row
// stores / vector atomics from registers.
bool gemm_tma_epi() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("DSV3_GEMM_TMA_EPI");
    on = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// 3-D fp32 output map [groups][rows][cols] (row stride ld, group stride
// gstride elements) with 32 x 32 boxes for the TMA epilogues; false when the
// layout does not allow it (TMA writes 16-byte units: cols, ld, gstride
// multiples of 4 and a 16-byte aligned base).
bool map_out_f32(CUtensorMap* m, void* ptr, int64_t rows, int64_t cols, int64_t ld, int64_t groups,
                 int64_t gstride) {
  if (!gemm_tma_epi() || cols % 4 != 0 || ld % 4 != 0 || gstride % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(ptr) & 15) != 0)
    return false;
  uint64_t dims[3] = {(uint64_t)cols, (uint64_t)rows, (uint64_t)groups};
  uint64_t st[2] = {(uint64_t)ld * 4, (uint64_t)std::max<int64_t>(gstride, ld * rows) * 4};
  uint32_t box[3] = {32, 32, 1};
  *m = make_map(ptr, 3, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
  return true;
}

// bf16 output map [rows][cols] (as 3-D with one group) with 32-row x 64-column
// boxes for the bf16 TMA-store epilogue; false when cols or ld is not a
// multiple of 8 or the base is not 16-byte aligned.
bool map_out_bf16(CUtensorMap* m, void* ptr, int64_t rows, int64_t cols, int64_t ld) {
  if (!gemm_tma_epi() || cols % 8 != 0 || ld % 8 != 0 || (reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return false;
  uint64_t dims[3] = {(uint64_t)cols, (uint64_t)rows, 1};
  uint64_t st[2] = {(uint64_t)ld * 2, (uint64_t)ld * rows * 2};
  uint32_t box[3] = {64, 32, 1};
  *m = make_map(ptr, 3, dims, st, box);
  return true;
}

// bf16 [rows][2][I] map of a gate / up pair buffer (row stride ld, the up half
// I columns after the gate half) with 32-row x 64-column boxes.
bool map_pair_bf16(CUtensorMap* m, void* ptr, int64_t rows, int64_t I, int64_t ld) {
  if (!gemm_tma_epi() || I % 64 != 0 || ld % 8 != 0 || (reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return false;
  uint64_t dims[3] = {(uint64_t)I, 2, (uint64_t)rows};
  uint64_t st[2] = {(uint64_t)I * 2, (uint64_t)ld * 2};
  uint32_t box[3] = {64, 1, 32};
  *m = make_map(ptr, 3, dims, st, box);
  return true;
}

GemmArgs blank_args() {
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.k_splits = 1;
  a.groups = 1;
  a.tile_rows = 128;
  return a;
}

void check_bf16_rows(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be a CUDA bf16 tensor");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with unit inner stride");
  TORCH_CHECK(t.stride(0) % 8 == 0, name, " row stride must be a multiple of 8 elements");
}


}  // namespace

// out = a[M,K] @ w[N,K]^T.  bf16 out: store.  fp32 out: accumulate (default),
// plain store (accumulate=false), or out = resid + a @ w^T when resid is given.
void linear_fwd(const at::Tensor& a, const at::Tensor& w, at::Tensor& out, bool accumulate,
                c10::optional<at::Tensor> resid) {
  check_bf16_rows(a, "a");
  check_bf16_rows(w, "w");
  const int64_t M = a.size(0), K = a.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "linear_fwd: K mismatch");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "linear_fwd: out shape");
  const at::cuda::CUDAGuard guard(a.device());
  GemmArgs g = blank_args();
  g.M = M; g.N = N; g.K = K;
  g.out = out.data_ptr(); g.ldo = out.stride(0);
  CUtensorMap ta = map_a_kmajor(a, M, K, a.stride(0));
  CUtensorMap tb = map_b_kmajor(w, 1, N, K, w.stride(0), N * w.stride(0));
  const bool f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || out.scalar_type() == at::kBFloat16, "linear_fwd: out must be bf16 or fp32");
  TORCH_CHECK(out.stride(0) % 8 == 0, "linear_fwd: out row stride must be a multiple of 8");
  int mode = f32 ? (resid ? 2 : (accumulate ? 1 : 3)) : 0;  // 0 bf16, 1 add, 2 resid, 3 store f32
  if (resid) {
    TORCH_CHECK(resid->scalar_type() == at::kFloat && resid->size(0) == M && resid->size(1) == N &&
                resid->stride(1) == 1 && resid->stride(0) % 4 == 0, "linear_fwd: resid must be fp32 [M, N]");
    g.aux = resid->data_ptr(); g.ld_aux = resid->stride(0);
  }
  const int bn = N <= 128 ? 128 : 256;
  g.m_tiles = cdiv(M, 128); g.n_tiles = cdiv(N, bn); g.kb_per_split = cdiv(K, 64);
  g.num_tiles = g.m_tiles * g.n_tiles;
  CUtensorMap tc, tcb;
  const bool tma = f32 && map_out_f32(&tc, out.data_ptr(), M, N, out.stride(0), 1, 0) &&
                   (mode != 2 || (g.ld_aux % 4 == 0 && (reinterpret_cast<uintptr_t>(g.aux) & 15) == 0));
  const bool tmab = !f32 && map_out_bf16(&tcb, out.data_ptr(), M, N, out.stride(0));
#define DSV3_LIN(BN_)                                                                            \
  switch (mode) {                                                                                \
    case 0:                                                                                      \
      if (tmab) launch<BN_, 0, 0, Sched::Dense, Epi::StoreBF16Tma, false>(ta, tb, g, &tcb);      \
      else launch<BN_, 0, 0, Sched::Dense, Epi::StoreBF16, false>(ta, tb, g);                     \
      break;                                                                                     \
    case 1:                                                                                      \
      if (tma) launch<BN_, 0, 0, Sched::Dense, Epi::AddF32Tma, false>(ta, tb, g, &tc);           \
      else launch<BN_, 0, 0, Sched::Dense, Epi::AddF32, false>(ta, tb, g);                        \
      break;                                                                                     \
    case 2:                                                                                      \
      if (tma) launch<BN_, 0, 0, Sched::Dense, Epi::ResidF32Tma, false>(ta, tb, g, &tc);         \
      else launch<BN_, 0, 0, Sched::Dense, Epi::ResidF32, false>(ta, tb, g);                      \
      break;                                                                                     \
    default:                                                                                     \
      if (tma) launch<BN_, 0, 0, Sched::Dense, Epi::StoreF32Tma, false>(ta, tb, g, &tc);         \
      else launch<BN_, 0, 0, Sched::Dense, Epi::StoreF32, false>(ta, tb, g);                      \
      break;                                                                                     \
  }
  if (bn == 128) { DSV3_LIN(128) } else { DSV3_LIN(256) }
#undef DSV3_LIN
}

// out [M,K] = dy[M,N] @ w[N,K]  (bf16 store; fp32 accumulate, or store when accumulate=false)
void linear_dgrad(const at::Tensor& dy, const at::Tensor& w, at::Tensor& out, bool accumulate) {
  check_bf16_rows(dy, "dy");
  check_bf16_rows(w, "w");
  const int64_t M = dy.size(0), N = dy.size(1), K = w.size(1);
  TORCH_CHECK(w.size(0) == N, "linear_dgrad: N mismatch");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == K && out.stride(1) == 1, "linear_dgrad: out shape");
  TORCH_CHECK(out.stride(0) % 8 == 0, "linear_dgrad: out row stride must be a multiple of 8");
  const at::cuda::CUDAGuard guard(dy.device());
  GemmArgs g = blank_args();
  g.M = M; g.N = K; g.K = N;
  g.out = out.data_ptr(); g.ldo = out.stride(0);
  CUtensorMap ta = map_a_kmajor(dy, M, N, dy.stride(0));
  CUtensorMap tb = map_b_mnmajor(w, 1, N, K, w.stride(0), N * w.stride(0));
  const bool f32 = out.scalar_type() == at::kFloat;
  g.m_tiles = cdiv(M, 128); g.n_tiles = cdiv(K, 256); g.kb_per_split = cdiv(N, 64);
  g.num_tiles = g.m_tiles * g.n_tiles;
  CUtensorMap tc;
  const bool tma = f32 && map_out_f32(&tc, out.data_ptr(), M, K, out.stride(0), 1, 0);
  if (f32 && accumulate) {
    if (tma) launch<256, 0, 1, Sched::Dense, Epi::AddF32Tma, false>(ta, tb, g, &tc);
    else launch<256, 0, 1, Sched::Dense, Epi::AddF32, false>(ta, tb, g);
  } else if (f32) {
    if (tma) launch<256, 0, 1, Sched::Dense, Epi::StoreF32Tma, false>(ta, tb, g, &tc);
    else launch<256, 0, 1, Sched::Dense, Epi::StoreF32, false>(ta, tb, g);
  } else {
    CUtensorMap tcb;
    if (map_out_bf16(&tcb, out.data_ptr(), M, K, out.stride(0)))
      launch<256, 0, 1, Sched::Dense, Epi::StoreBF16Tma, false>(ta, tb, g, &tcb);
    else
      launch<256, 0, 1, Sched::Dense, Epi::StoreBF16, false>(ta, tb, g);
  }
}

// dw [N,K] fp32 += dy[M,N]^T @ x[M,K]   (reduction over the M token rows)
void linear_wgrad(const at::Tensor& dy, const at::Tensor& x, at::Tensor& dw) {
  check_bf16_rows(dy, "dy");
  check_bf16_rows(x, "x");
  const int64_t M = dy.size(0), N = dy.size(1), K = x.size(1);
  TORCH_CHECK(x.size(0) == M, "linear_wgrad: M mismatch");
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.is_contiguous() && dw.size(0) == N && dw.size(1) == K,
              "linear_wgrad: dw must be contiguous fp32 [N, K]");
  const at::cuda::CUDAGuard guard(dy.device());
  GemmArgs g = blank_args();
  g.M = N; g.N = K; g.K = M;
  g.out = dw.data_ptr(); g.ldo = K;
  CUtensorMap ta = map_a_mnmajor(dy, N, M, dy.stride(0));
  CUtensorMap tb = map_b_mnmajor(x, 1, M, K, x.stride(0), M * x.stride(0));
  g.m_tiles = cdiv(N, 128); g.n_tiles = cdiv(K, 256);
  const int total_kb = cdiv(M, 64);
  const int base_tiles = g.m_tiles * g.n_tiles;
  int splits = std::max(1, std::min(total_kb / 8, (2 * num_sms() + base_tiles - 1) / base_tiles));
  g.kb_per_split = cdiv(total_kb, splits);
  splits = cdiv(total_kb, g.kb_per_split);
  g.k_splits = splits;
  g.num_tiles = base_tiles * splits;
  CUtensorMap tc;
  if (map_out_f32(&tc, dw.data_ptr(), N, K, K, 1, 0))   // split partials add atomically at L2
    launch<256, 1, 1, Sched::Dense, Epi::AddF32Tma, false>(ta, tb, g, &tc);
  else if (splits > 1) launch<256, 1, 1, Sched::Dense, Epi::AtomicAddF32, false>(ta, tb, g);
  else launch<256, 1, 1, Sched::Dense, Epi::AddF32, false>(ta, tb, g);
}

// SwiGLU up-projection: x[P,D] against w13 [G,2,I,D] (dense when G == 1 and
// tile_group is empty).  Writes h = silu(g) * u [P, I] and gu = [g | u] [P, 2I].
void swiglu_fwd(const at::Tensor& x, const at::Tensor& w13, const at::Tensor& tile_group, at::Tensor& h,
                at::Tensor& gu, int64_t group_rows) {
  check_bf16_rows(x, "x");
  TORCH_CHECK(w13.scalar_type() == at::kBFloat16 && w13.is_contiguous() && w13.dim() == 4 && w13.size(1) == 2,
              "w13 must be contiguous bf16 [G, 2, I, D]");
  const int64_t P = x.size(0), D = x.size(1), G = w13.size(0), I = w13.size(2);
  TORCH_CHECK(w13.size(3) == D, "swiglu_fwd: D mismatch");
  TORCH_CHECK(I % 8 == 0 && D % 8 == 0, "swiglu_fwd: I and D must be multiples of 8");
  check_bf16_rows(h, "h");
  check_bf16_rows(gu, "gu");
  TORCH_CHECK(h.size(0) == P && h.size(1) == I && gu.size(0) == P && gu.size(1) == 2 * I, "swiglu_fwd: outputs");
  const at::cuda::CUDAGuard guard(x.device());
  GemmArgs g = blank_args();
  g.M = P; g.N = I; g.K = D; g.inter = I;
  g.out = h.data_ptr(); g.ldo = h.stride(0);
  g.out2 = gu.data_ptr(); g.ldo2 = gu.stride(0);
  g.m_tiles = cdiv(P, 128); g.n_tiles = cdiv(I, 128); g.kb_per_split = cdiv(D, 64);
  g.num_tiles = g.m_tiles * g.n_tiles;
  CUtensorMap ta = map_a_kmajor(x, P, D, x.stride(0));
  CUtensorMap tb = map_b_swiglu(w13, G, I, D);
  // h and the gate / up pair leave through shared memory and TMA where the maps fit
  CUtensorMap tc, td;
  const bool tma = map_out_bf16(&tc, h.data_ptr(), P, I, h.stride(0)) &&
                   map_pair_bf16(&td, gu.data_ptr(), P, I, gu.stride(0));
  if (tile_group.numel() > 0) {
    TORCH_CHECK(tile_group.scalar_type() == at::kInt && tile_group.numel() >= g.m_tiles, "tile_group: int32 [tiles]");
    g.tile_group = tile_group.data_ptr<int>();
    g.tile_rows = (int)group_rows;
    if (tma) launch<256, 0, 0, Sched::GroupedM, Epi::SwigluFwdTma, true>(ta, tb, g, &tc, &td);
    else launch<256, 0, 0, Sched::GroupedM, Epi::SwigluFwd, true>(ta, tb, g);
  } else {
    TORCH_CHECK(G == 1, "dense SwiGLU expects one weight group");
    if (tma) launch<256, 0, 0, Sched::Dense, Epi::SwigluFwdTma, true>(ta, tb, g, &tc, &td);
    else launch<256, 0, 0, Sched::Dense, Epi::SwigluFwd, true>(ta, tb, g);
  }
}

// SwiGLU backward through the down projection: dh = dy[P,D] @ w2[G](D x I),
// then dgu = [dh * u * silu'(g) | dh * silu(g)] using the saved pre-activations.
void swiglu_dgrad(const at::Tensor& dy, const at::Tensor& w2, const at::Tensor& tile_group, const at::Tensor& gu,
                  at::Tensor& dgu, int64_t group_rows) {
  check_bf16_rows(dy, "dy");
  check_bf16_rows(gu, "gu");
  check_bf16_rows(dgu, "dgu");
  TORCH_CHECK(w2.scalar_type() == at::kBFloat16 && w2.is_contiguous() && w2.dim() == 3, "w2: bf16 [G, D, I]");
  const int64_t P = dy.size(0), D = dy.size(1), G = w2.size(0), I = w2.size(2);
  TORCH_CHECK(w2.size(1) == D && gu.size(1) == 2 * I && dgu.size(1) == 2 * I, "swiglu_dgrad: shapes");
  const at::cuda::CUDAGuard guard(dy.device());
  GemmArgs g = blank_args();
  g.M = P; g.N = I; g.K = D; g.inter = I;
  g.out = dgu.data_ptr(); g.ldo = dgu.stride(0);
  g.aux = gu.data_ptr(); g.ld_aux = gu.stride(0);
  // I a multiple of 128 but not of 256 (the 412M experts' 384): 128-wide
  // column tiles (still CTA pairs) leave no half-empty tile
  const int bn = (I % 256 != 0 && I % 128 == 0) ? 128 : 256;
  g.m_tiles = cdiv(P, 128); g.n_tiles = cdiv(I, bn); g.kb_per_split = cdiv(D, 64);
  g.num_tiles = g.m_tiles * g.n_tiles;
  CUtensorMap ta = map_a_kmajor(dy, P, D, dy.stride(0));
  CUtensorMap tb = map_b_mnmajor(w2, G, D, I, I, D * I);
  CUtensorMap tc;   // dg / du through shared memory and TMA where the map fits
  const bool tma = map_pair_bf16(&tc, dgu.data_ptr(), P, I, dgu.stride(0));
  if (tile_group.numel() > 0) {
    g.tile_group = tile_group.data_ptr<int>();
    g.tile_rows = (int)group_rows;
    if (tma) {
      if (bn == 128) launch<128, 0, 1, Sched::GroupedM, Epi::SwigluBwdTma, false>(ta, tb, g, &tc);
      else launch<256, 0, 1, Sched::GroupedM, Epi::SwigluBwdTma, false>(ta, tb, g, &tc);
    } else {
      if (bn == 128) launch<128, 0, 1, Sched::GroupedM, Epi::SwigluBwd, false>(ta, tb, g);
      else launch<256, 0, 1, Sched::GroupedM, Epi::SwigluBwd, false>(ta, tb, g);
    }
  } else {
    if (tma) {
      if (bn == 128) launch<128, 0, 1, Sched::Dense, Epi::SwigluBwdTma, false>(ta, tb, g, &tc);
      else launch<256, 0, 1, Sched::Dense, Epi::SwigluBwdTma, false>(ta, tb, g, &tc);
    } else {
      if (bn == 128) launch<128, 0, 1, Sched::Dense, Epi::SwigluBwd, false>(ta, tb, g);
      else launch<256, 0, 1, Sched::Dense, Epi::SwigluBwd, false>(ta, tb, g);
    }
  }
}

// Grouped forward: out[P,N] = a[P,K] @ w[g(tile)] ^T, w: [G, N, K].
void grouped_fwd(const at::Tensor& a, const at::Tensor& w, const at::Tensor& tile_group, at::Tensor& out,
                 int64_t group_rows) {
  check_bf16_rows(a, "a");
  check_bf16_rows(out, "out");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.dim() == 3, "w: bf16 [G, N, K]");
  const int64_t P = a.size(0), K = a.size(1), G = w.size(0), N = w.size(1);
  TORCH_CHECK(w.size(2) == K && out.size(0) == P && out.size(1) == N, "grouped_fwd: shapes");
  const at::cuda::CUDAGuard guard(a.device());
  GemmArgs g = blank_args();
  g.M = P; g.N = N; g.K = K;
  g.out = out.data_ptr(); g.ldo = out.stride(0);
  g.tile_group = tile_group.data_ptr<int>();
  g.tile_rows = (int)group_rows;
  g.m_tiles = cdiv(P, 128); g.n_tiles = cdiv(N, 256); g.kb_per_split = cdiv(K, 64);
  g.num_tiles = g.m_tiles * g.n_tiles;
  CUtensorMap ta = map_a_kmajor(a, P, K, a.stride(0));
  CUtensorMap tb = map_b_kmajor(w, G, N, K, K, N * K);
  CUtensorMap tcb;
  if (map_out_bf16(&tcb, out.data_ptr(), P, N, out.stride(0)))
    launch<256, 0, 0, Sched::GroupedM, Epi::StoreBF16Tma, false>(ta, tb, g, &tcb);
  else
    launch<256, 0, 0, Sched::GroupedM, Epi::StoreBF16, false>(ta, tb, g);
}

// Expert-grouped GEMM whose epilogue also stores every output row into its
// home rank's inbox over peer memory (the expert-parallel combine fused with
// the GEMM); the last CTA raises flag [phase][me] on every rank.
//   transpose_w = false: out = a @ w[e]^T  (w [G, N, K]; forward down projection)
//   transpose_w = true:  out = a @ w[e]    (w [G, K, N]; backward through gate/up)
// peers: int64 [R] heap bases (device); origin: int32 [P] (src * tk + slot,
// -1 on padding); extra (optional, fp32 [P]) goes to extra_off[slot].
void grouped_scatter(const at::Tensor& a, const at::Tensor& w, bool transpose_w, const at::Tensor& tile_group,
                     at::Tensor& out, int64_t group_rows, const at::Tensor& peers, int64_t scatter_off,
                     const at::Tensor& origin, const c10::optional<at::Tensor>& extra, int64_t extra_off, int64_t tk,
                     int64_t flags_off, int64_t me, int64_t phase, at::Tensor& done) {
  check_bf16_rows(a, "a");
  check_bf16_rows(out, "out");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.dim() == 3, "w: bf16 3-D");
  const int64_t P = a.size(0), K = a.size(1), G = w.size(0);
  const int64_t N = transpose_w ? w.size(2) : w.size(1);
  TORCH_CHECK((transpose_w ? w.size(1) : w.size(2)) == K && out.size(0) == P && out.size(1) == N,
              "grouped_scatter: shapes");
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong && peers.numel() >= 1 && peers.numel() <= 8,
              "grouped_scatter: peers int64 [R] on the device");
  TORCH_CHECK(origin.scalar_type() == at::kInt && origin.numel() >= P, "grouped_scatter: origin int32 [P]");
  TORCH_CHECK(N % 8 == 0 && scatter_off % 16 == 0, "grouped_scatter: 16-byte rows");
  if (extra.has_value())
    TORCH_CHECK(extra->scalar_type() == at::kFloat && extra->numel() >= P && extra_off % 4 == 0,
                "grouped_scatter: extra fp32 [P]");
  const at::cuda::CUDAGuard guard(a.device());
  GemmArgs g = blank_args();
  g.M = P; g.N = N; g.K = K;
  g.out = out.data_ptr(); g.ldo = out.stride(0);
  g.tile_group = tile_group.data_ptr<int>();
  g.tile_rows = (int)group_rows;
  g.peer_base = reinterpret_cast<const unsigned long long*>(peers.data_ptr<int64_t>());
  g.origin = origin.data_ptr<int>();
  g.scatter_extra = extra.has_value() ? extra->data_ptr<float>() : nullptr;
  g.scatter_extra_off = extra_off;
  g.scatter_off = scatter_off;
  g.flags_off = flags_off;
  g.scatter_tk = (int)tk;
  g.scatter_me = (int)me;
  g.scatter_ranks = (int)peers.numel();
  g.scatter_phase = (int)phase;
  g.done_ctr = reinterpret_cast<unsigned int*>(done.data_ptr());
  g.m_tiles = cdiv(P, 128); g.n_tiles = cdiv(N, 256); g.kb_per_split = cdiv(K, 64);
  g.num_tiles = g.m_tiles * g.n_tiles;
  CUtensorMap ta = map_a_kmajor(a, P, K, a.stride(0));
  if (transpose_w) {
    CUtensorMap tb = map_b_mnmajor(w, G, K, N, N, K * N);
    launch<256, 0, 1, Sched::GroupedM, Epi::ScatterBF16, false>(ta, tb, g);
  } else {
    CUtensorMap tb = map_b_kmajor(w, G, N, K, K, N * K);
    launch<256, 0, 0, Sched::GroupedM, Epi::ScatterBF16, false>(ta, tb, g);
  }
}

// Grouped data gradient: out[P,K] = dy[P,N] @ w[g(tile)], w: [G, N, K].
void grouped_dgrad(const at::Tensor& dy, const at::Tensor& w, const at::Tensor& tile_group, at::Tensor& out,
                   int64_t group_rows) {
  check_bf16_rows(dy, "dy");
  check_bf16_rows(out, "out");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.dim() == 3, "w: bf16 [G, N, K]");
  const int64_t P = dy.size(0), N = dy.size(1), G = w.size(0), K = w.size(2);
  TORCH_CHECK(w.size(1) == N && out.size(0) == P && out.size(1) == K, "grouped_dgrad: shapes");
  const at::cuda::CUDAGuard guard(dy.device());
  GemmArgs g = blank_args();
  g.M = P; g.N = K; g.K = N;
  g.out = out.data_ptr(); g.ldo = out.stride(0);
  g.tile_group = tile_group.data_ptr<int>();
  g.tile_rows = (int)group_rows;
  g.m_tiles = cdiv(P, 128); g.n_tiles = cdiv(K, 256); g.kb_per_split = cdiv(N, 64);
  g.num_tiles = g.m_tiles * g.n_tiles;
  CUtensorMap ta = map_a_kmajor(dy, P, N, dy.stride(0));
  CUtensorMap tb = map_b_mnmajor(w, G, N, K, K, N * K);
  CUtensorMap tcb;
  if (map_out_bf16(&tcb, out.data_ptr(), P, K, out.stride(0)))
    launch<256, 0, 1, Sched::GroupedM, Epi::StoreBF16Tma, false>(ta, tb, g, &tcb);
  else
    launch<256, 0, 1, Sched::GroupedM, Epi::StoreBF16, false>(ta, tb, g);
}

// Grouped weight gradient: out[g] [Ma, Nb] fp32 += a[rows_g, Ma]^T @ b[rows_g, Nb]
// where rows_g = [off[g], off[g+1]) (128-aligned padded expert ranges).
void grouped_wgrad(const at::Tensor& a, const at::Tensor& b, const at::Tensor& row_off, at::Tensor& out) {
  check_bf16_rows(a, "a");
  check_bf16_rows(b, "b");
  const int64_t P = a.size(0), Ma = a.size(1), Nb = b.size(1);
  const int64_t G = row_off.numel() - 1;
  TORCH_CHECK(b.size(0) == P, "grouped_wgrad: row mismatch");
  TORCH_CHECK(row_off.scalar_type() == at::kInt, "row_off must be int32 [G+1]");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == G * Ma * Nb,
              "grouped_wgrad: out must be contiguous fp32 [G, Ma, Nb]");
  const at::cuda::CUDAGuard guard(a.device());
  GemmArgs g = blank_args();
  g.M = Ma; g.N = Nb; g.K = P; g.groups = G;
  g.out = out.data_ptr(); g.ldo = Nb; g.out_group_stride = Ma * Nb;
  g.group_row_off = row_off.data_ptr<int>();
  g.m_tiles = cdiv(Ma, 128); g.n_tiles = cdiv(Nb, 256);
  // Few groups (expert parallelism leaves a rank a handful of experts, each
  // with many rows): split every group's rows so the grid fills the GPU and
  // reduce the partial tiles with vector atomics.
  const int base = g.m_tiles * g.n_tiles * (int)G;
  int splits = 1;
  if (base < num_sms()) splits = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(2 * num_sms(), base), P / (G * 512)));
  g.k_splits = splits;
  g.num_tiles = base * splits;
  CUtensorMap ta = map_a_mnmajor(a, Ma, P, a.stride(0));
  CUtensorMap tb = map_b_mnmajor(b, 1, P, Nb, b.stride(0), P * b.stride(0));
  CUtensorMap tc;
  if (map_out_f32(&tc, out.data_ptr(), Ma, Nb, Nb, G, Ma * Nb))
    launch<256, 1, 1, Sched::GroupedK, Epi::AddF32Tma, false>(ta, tb, g, &tc);
  else if (splits > 1) launch<256, 1, 1, Sched::GroupedK, Epi::AtomicAddF32, false>(ta, tb, g);
  else launch<256, 1, 1, Sched::GroupedK, Epi::AddF32, false>(ta, tb, g);
}

// Fused LM head + cross-entropy, forward half: per (row, 256-column tile)
// online max / sum-exp partials and the target logit.  No logits are stored.
void ce_fwd_partials(const at::Tensor& x, const at::Tensor& w, const at::Tensor& targets, at::Tensor& part_max,
                     at::Tensor& part_sum, at::Tensor& tgt_logit) {
  check_bf16_rows(x, "x");
  check_bf16_rows(w, "w");
  const int64_t T = x.size(0), D = x.size(1), V = w.size(0);
  const int nt = cdiv(V, 256);
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.numel() == T && targets.is_contiguous(),
              "targets: contiguous int64 [T]");
  TORCH_CHECK(part_max.numel() == 2 * T * nt && part_sum.numel() == 2 * T * nt && tgt_logit.numel() == T,
              "ce partial shapes: [T, 2 * ceil(V / 256)]");
  const at::cuda::CUDAGuard guard(x.device());
  GemmArgs g = blank_args();
  g.M = T; g.N = V; g.K = D;
  g.targets = targets.data_ptr<int64_t>();
  g.part_max = part_max.data_ptr<float>();
  g.part_sum = part_sum.data_ptr<float>();
  g.tgt_logit = tgt_logit.data_ptr<float>();
  g.m_tiles = cdiv(T, 128); g.n_tiles = nt; g.kb_per_split = cdiv(D, 64);
  g.panel_rows = ce_panel_rows();
  g.num_tiles = g.m_tiles * g.n_tiles;
  CUtensorMap ta = map_a_kmajor(x, T, D, x.stride(0));
  CUtensorMap tb = map_b_kmajor(w, 1, V, D, w.stride(0), V * w.stride(0));
  launch<256, 0, 0, Sched::Dense, Epi::CeFwd, false>(ta, tb, g);
}

// Backward half: dlogits[T, :V] = (softmax(x w^T) - onehot(target)) * row_scale.
// When dlogits has at least V rounded up to 8 columns, its columns V .. that
// bound are set to zero as well (the TMA-store epilogue writes 16-byte units).
void ce_bwd_logits(const at::Tensor& x, const at::Tensor& w, const at::Tensor& targets, const at::Tensor& lse,
                   const at::Tensor& row_scale, at::Tensor& dlogits) {
  check_bf16_rows(x, "x");
  check_bf16_rows(w, "w");
  check_bf16_rows(dlogits, "dlogits");
  const int64_t T = x.size(0), D = x.size(1), V = w.size(0);
  TORCH_CHECK(dlogits.size(0) == T && dlogits.size(1) >= V, "dlogits shape");
  TORCH_CHECK(targets.is_contiguous() && lse.is_contiguous() && row_scale.is_contiguous(), "ce_bwd: contiguous rows");
  const at::cuda::CUDAGuard guard(x.device());
  GemmArgs g = blank_args();
  g.M = T; g.N = V; g.K = D;
  g.targets = targets.data_ptr<int64_t>();
  g.lse = lse.data_ptr<float>();
  g.row_scale = row_scale.data_ptr<float>();
  g.out = dlogits.data_ptr(); g.ldo = dlogits.stride(0);
  g.m_tiles = cdiv(T, 128); g.n_tiles = cdiv(V, 256); g.kb_per_split = cdiv(D, 64);
  g.panel_rows = ce_panel_rows();
  g.num_tiles = g.m_tiles * g.n_tiles;
  CUtensorMap ta = map_a_kmajor(x, T, D, x.stride(0));
  CUtensorMap tb = map_b_kmajor(w, 1, V, D, w.stride(0), V * w.stride(0));
  if (ce_tma_store() && dlogits.size(1) >= (V + 7) / 8 * 8) {
    // dlogits written in 32-row x 64-column boxes; the store clips rows >= T
    // and columns past V rounded up to 8 (columns V .. that bound get zeros)
    uint64_t dims[2] = {(uint64_t)V, (uint64_t)T};
    uint64_t st[1] = {(uint64_t)dlogits.stride(0) * 2};
    uint32_t box[2] = {64, 32};
    CUtensorMap tc = make_map(dlogits.data_ptr(), 2, dims, st, box);
    launch<256, 0, 0, Sched::Dense, Epi::CeBwdTma, false>(ta, tb, g, &tc);
  } else {
    launch<256, 0, 0, Sched::Dense, Epi::CeBwd, false>(ta, tb, g);
  }
}

}  // namespace dsv3

namespace dsv3 {
// Query (-1) or set (0 / 1) whether eligible GEMMs run on CTA pairs.
int64_t gemm_pairs(int64_t mode) {
  if (mode >= 0) g_pairs = mode ? 1 : 0;
  return use_pairs() ? 1 : 0;
}

void register_gemm(pybind11::module_& m) {
  m.def("gemm_pairs", &gemm_pairs, "query (-1) or set (0/1) the CTA-pair (cta_group::2) GEMM tiles");
  m.def("linear_fwd", &linear_fwd, "out = a @ w^T (bf16 store; fp32: accumulate / store / resid + a @ w^T)",
        pybind11::arg("a"), pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("accumulate") = true,
        pybind11::arg("resid") = pybind11::none());
  m.def("linear_dgrad", &linear_dgrad, "out = dy @ w (bf16 store; fp32 accumulate or store)", pybind11::arg("dy"),
        pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("accumulate") = true);
  m.def("linear_wgrad", &linear_wgrad, "dw (fp32) += dy^T @ x");
  // group_rows: the expert row ranges behind tile_group are multiples of this
  // (256 lets the grouped GEMMs run on CTA pairs)
  m.def("swiglu_fwd", &swiglu_fwd, "h, gu from x @ [w1|w3]^T (dense or expert-grouped)", pybind11::arg("x"),
        pybind11::arg("w13"), pybind11::arg("tile_group"), pybind11::arg("h"), pybind11::arg("gu"),
        pybind11::arg("group_rows") = 128);
  m.def("swiglu_dgrad", &swiglu_dgrad, "dgu from (dy @ w2) and the saved gate/up", pybind11::arg("dy"),
        pybind11::arg("w2"), pybind11::arg("tile_group"), pybind11::arg("gu"), pybind11::arg("dgu"),
        pybind11::arg("group_rows") = 128);
  m.def("grouped_fwd", &grouped_fwd, "expert-grouped out = a @ w[e]^T", pybind11::arg("a"), pybind11::arg("w"),
        pybind11::arg("tile_group"), pybind11::arg("out"), pybind11::arg("group_rows") = 128);
  m.def("grouped_scatter", &grouped_scatter,
        "expert-grouped GEMM whose rows also go to their home ranks' inbox over peer memory (fused combine)");
  m.def("grouped_dgrad", &grouped_dgrad, "expert-grouped out = dy @ w[e]", pybind11::arg("dy"), pybind11::arg("w"),
        pybind11::arg("tile_group"), pybind11::arg("out"), pybind11::arg("group_rows") = 128);
  m.def("grouped_wgrad", &grouped_wgrad, "per-expert dw[e] (fp32) += a_e^T @ b_e");
  m.def("ce_fwd_partials", &ce_fwd_partials, "fused LM head + log-sum-exp partials");
  m.def("ce_bwd_logits", &ce_bwd_logits, "fused LM head + softmax-minus-onehot gradient");
}
}  // namespace dsv3
