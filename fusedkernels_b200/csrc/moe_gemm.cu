// bf16 entry points of the MoE expert GEMMs (kernel template and per-GEMM set-up in
// moe_gemm.cuh), reference moe_layer_sorted.py:70-77 and moe_layer.py:22-31.
#include "moe_gemm.cuh"

namespace fk {
namespace gemm {

EncodeTiledFn encode_fn() {
  // looked up once (thread-safe static initialisation)
  static const EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(f);
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

}  // namespace gemm
}  // namespace fk

namespace G = fk::gemm;

extern "C" int fk_moe_gemm_up(const void* xs, int64_t max_rows, int dim, const void* w13,
                              int hidden, int n_experts, const int* tile_expert, const int* n_mblk,
                              void* h1, void* act, int max_ctas, int* err_flag, void* stream) {
  FK_CHECK_ARG(max_ctas >= 0, "fk_moe_gemm: max_ctas < 0");
  return G::gemm_up<G::KIND_BF16>(xs, nullptr, max_rows, dim, w13, nullptr, hidden, n_experts,
                                  tile_expert, n_mblk, h1, act, err_flag, fk::as_stream(stream),
                                  max_ctas);
}

extern "C" int fk_moe_gemm_down(const void* act, int64_t max_rows, int hidden, const void* w2,
                                int dim, int n_experts, const int* tile_expert, const int* n_mblk,
                                void* y, int max_ctas, int* err_flag, void* stream) {
  FK_CHECK_ARG(max_ctas >= 0, "fk_moe_gemm: max_ctas < 0");
  return G::gemm_down<G::KIND_BF16>(act, nullptr, max_rows, hidden, w2, nullptr, dim, n_experts,
                                    tile_expert, n_mblk, y, err_flag, fk::as_stream(stream),
                                    max_ctas);
}

extern "C" int fk_moe_gemm_down_dgrad(const void* dy, int64_t max_rows, int dim, const void* w2,
                                      int hidden, int n_experts, const int* tile_expert,
                                      const int* n_mblk, const void* h1, void* dh1, int max_ctas,
                                      int* err_flag, void* stream) {
  FK_CHECK_ARG(max_ctas >= 0, "fk_moe_gemm: max_ctas < 0");
  return G::gemm_down_dgrad<G::KIND_BF16>(dy, nullptr, max_rows, dim, w2, nullptr, hidden,
                                          n_experts, tile_expert, n_mblk, h1, dh1, err_flag,
                                          fk::as_stream(stream), max_ctas);
}

extern "C" int fk_moe_gemm_up_dgrad(const void* dh1, int64_t max_rows, int hidden, const void* w13,
                                    int dim, int n_experts, const int* tile_expert,
                                    const int* n_mblk, void* dxs, int max_ctas, int* err_flag,
                                    void* stream) {
  FK_CHECK_ARG(max_ctas >= 0, "fk_moe_gemm: max_ctas < 0");
  return G::gemm_up_dgrad<G::KIND_BF16>(dh1, nullptr, max_rows, hidden, w13, nullptr, dim,
                                        n_experts, tile_expert, n_mblk, dxs, err_flag,
                                        fk::as_stream(stream), max_ctas);
}

extern "C" int fk_moe_gemm_wgrad(const void* a, int m_dim, const void* b, int n_dim,
                                 int64_t max_rows, const int* seg_start, int n_experts, void* dw,
                                 int max_ctas, int* err_flag, void* stream) {
  FK_CHECK_ARG(max_ctas >= 0, "fk_moe_gemm: max_ctas < 0");
  return G::gemm_wgrad<G::KIND_BF16>(a, nullptr, m_dim, b, nullptr, n_dim, max_rows, seg_start,
                                     n_experts, dw, err_flag, fk::as_stream(stream),
                                     max_ctas);
}

// ------------------------------------------------------------------------------------------
// Row-weighted variants (bf16).  The routing weight of every sorted row is applied in the
// SwiGLU epilogues instead of by the combine kernels:
//   forward:  up_weighted(xs) -> h1, act_w = w * silu(g) * u;  down(act_w) -> weighted rows;
//             combine(unweighted) -> out
//   backward: gather(dout) -> dy (unweighted rows);  down_dgrad_weighted(dy) -> dh1 =
//             SwiGLU'(w * dy @ w2) and the routing-weight partials;  dw_from_parts -> dw;
//             wgrad(dy, act_w) -> dW2 (= sum of (w dout)^T act);  up_dgrad, wgrad(dh1, xs)
// so the backward needs a plain row gather of dout instead of the combine backward, which
// also re-read every output row to form the routing-weight gradient (and the output rows
// need not be kept for the backward).
namespace fk {
namespace gemm {
namespace {

constexpr int kPartCols = 64;  // dw_part has one slot per 64 hidden units

inline int check_rows(const int* row_assign, const float* row_w) {
  FK_CHECK_ARG(row_assign && row_w, "fk_moe_gemm_*_weighted: null sorted_assign / sorted_w");
  return FK_OK;
}

// Partial dots -> dw[a] for every sorted row holding assignment a (fixed summation order).
__global__ void dw_from_parts_kernel(const float* __restrict__ part, int n_part,
                                     const int* __restrict__ row_assign,
                                     const int* __restrict__ n_mblk, float* __restrict__ dw) {
  const int64_t rows = (int64_t)(*n_mblk) * BM;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows;
       r += (int64_t)gridDim.x * blockDim.x) {
    const int a = row_assign[r];
    if (a < 0) continue;
    const float* pr = part + r * n_part;
    float s = 0.f;
    for (int i = 0; i < n_part; ++i) s += pr[i];
    dw[a] = s;
  }
}

}  // namespace
}  // namespace gemm
}  // namespace fk

extern "C" int fk_moe_gemm_up_weighted(const void* xs, int64_t max_rows, int dim, const void* w13,
                                       int hidden, int n_experts, const int* tile_expert,
                                       const int* n_mblk, const int* sorted_assign,
                                       const float* sorted_w, void* h1, void* act_w,
                                       int max_ctas, int* err_flag, void* stream) {
  using namespace fk::gemm;
  int st = check_common(xs, w13, tile_expert, n_mblk, max_rows, n_experts);
  if (st) return st;
  FK_CHECK_ARG(max_ctas >= 0, "fk_moe_gemm: max_ctas < 0");
  FK_CHECK_ARG(h1 && act_w && err_flag, "fk_moe_gemm_up_weighted: null pointer");
  FK_CHECK_ARG(dim % 64 == 0 && hidden % 64 == 0,
               "fk_moe_gemm_up_weighted: dim, hidden must be multiples of 64");
  if ((st = check_rows(sorted_assign, sorted_w))) return st;
  if (max_rows == 0) return FK_OK;
  const int bn = hidden % 128 == 0 ? 256 : 128;
  CUtensorMap ma, mb, mc0, mc1;
  uint64_t da[2] = {(uint64_t)dim, (uint64_t)max_rows}, sa[1] = {(uint64_t)dim * 2};
  uint32_t ba[2] = {64, 128};
  if ((st = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xs, 2, da, sa, ba))) return st;
  uint64_t db[3] = {(uint64_t)dim, (uint64_t)2 * hidden, (uint64_t)n_experts};
  uint64_t sb[2] = {(uint64_t)dim * 2, (uint64_t)2 * hidden * dim * 2};
  uint32_t bb[3] = {64, (uint32_t)bn / 2, 1};
  if ((st = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w13, 3, db, sb, bb))) return st;
  if ((st = make_out_map<KIND_BF16>(&mc0, act_w, max_rows, hidden, hidden))) return st;
  if ((st = make_out_map<KIND_BF16>(&mc1, h1, max_rows, 2 * hidden, 2 * hidden))) return st;
  Params p{};
  p.M = (int)max_rows;
  p.N = hidden;
  p.K = dim;
  p.E = n_experts;
  p.H = hidden;
  p.tile_expert = tile_expert;
  p.n_mblk = n_mblk;
  p.out0 = act_w;
  p.ld0 = hidden;
  p.out1 = h1;
  p.ld1 = 2 * (int64_t)hidden;
  p.err = err_flag;
  p.tma_store = 1;
  p.row_assign = sorted_assign;
  p.row_w = sorted_w;
  const int max_tiles = (int)(max_rows / BM) * (hidden / (bn / 2));
  cudaStream_t s = fk::as_stream(stream);
  if (bn == 256)
    return launch<256, false, false, MODE_M, EPI_SWIGLU_FWD, KIND_BF16, true>(
        ma, mb, mc0, mc1, ma, mb, p, max_tiles, s, max_ctas);
  return launch<128, false, false, MODE_M, EPI_SWIGLU_FWD, KIND_BF16, true>(
      ma, mb, mc0, mc1, ma, mb, p, max_tiles, s, max_ctas);
}

extern "C" int fk_moe_gemm_down_dgrad_weighted(const void* dy, int64_t max_rows, int dim,
                                               const void* w2, int hidden, int n_experts,
                                               const int* tile_expert, const int* n_mblk,
                                               const int* sorted_assign, const float* sorted_w,
                                               const void* h1, void* dh1, float* dw_part,
                                               int max_ctas, int* err_flag, void* stream) {
  using namespace fk::gemm;
  int st = check_common(dy, w2, tile_expert, n_mblk, max_rows, n_experts);
  if (st) return st;
  FK_CHECK_ARG(max_ctas >= 0, "fk_moe_gemm: max_ctas < 0");
  FK_CHECK_ARG(h1 && dh1 && dw_part && err_flag, "fk_moe_gemm_down_dgrad_weighted: null pointer");
  FK_CHECK_ARG(hidden % 64 == 0 && dim % 64 == 0,
               "fk_moe_gemm_down_dgrad_weighted: dim, hidden must be multiples of 64");
  if ((st = check_rows(sorted_assign, sorted_w))) return st;
  if (max_rows == 0) return FK_OK;
  const int bn = pick_bn(hidden);
  CUtensorMap ma, mb, mc0;
  uint64_t da[2] = {(uint64_t)dim, (uint64_t)max_rows}, sa[1] = {(uint64_t)dim * 2};
  uint32_t ba[2] = {64, 128};
  if ((st = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dy, 2, da, sa, ba))) return st;
  uint64_t db[3] = {(uint64_t)hidden, (uint64_t)dim, (uint64_t)n_experts};
  uint64_t sb[2] = {(uint64_t)hidden * 2, (uint64_t)dim * hidden * 2};
  uint32_t bb[3] = {64, 64, 1};
  if ((st = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w2, 3, db, sb, bb,
                     mn_swizzle<KIND_BF16>())))
    return st;
  if ((st = make_out_map<KIND_BF16>(&mc0, dh1, max_rows, 2 * hidden, 2 * hidden))) return st;
  Params p{};
  p.M = (int)max_rows;
  p.N = hidden;
  p.K = dim;
  p.E = n_experts;
  p.H = hidden;
  p.tile_expert = tile_expert;
  p.n_mblk = n_mblk;
  p.out0 = dh1;
  p.ld0 = 2 * (int64_t)hidden;
  p.in0 = h1;
  p.ldi0 = 2 * (int64_t)hidden;
  p.err = err_flag;
  p.tma_store = 1;
  p.row_assign = sorted_assign;
  p.row_w = sorted_w;
  p.dw_part = dw_part;
  const int max_tiles = (int)(max_rows / BM) * (hidden / bn);
  cudaStream_t s = fk::as_stream(stream);
  FK_BN_SWITCH(bn, return (launch<BN_, false, true, MODE_M, EPI_SWIGLU_BWD, KIND_BF16, true>(
                       ma, mb, mc0, mc0, ma, mb, p, max_tiles, s, max_ctas)));
  return FK_OK;
}

extern "C" int fk_moe_dw_from_parts(const float* dw_part, int hidden, const int* sorted_assign,
                                    const int* n_mblk, int64_t max_rows, float* dw,
                                    void* stream) {
  using namespace fk::gemm;
  FK_CHECK_ARG(hidden > 0 && hidden % 64 == 0, "fk_moe_dw_from_parts: hidden must be a positive "
               "multiple of 64");
  FK_CHECK_ARG(max_rows >= 0 && max_rows % BM == 0, "fk_moe_dw_from_parts: bad max_rows");
  if (max_rows == 0) return FK_OK;
  FK_CHECK_ARG(dw_part && sorted_assign && n_mblk && dw, "fk_moe_dw_from_parts: null pointer");
  int64_t blocks = (max_rows + 255) / 256;
  const int64_t cap = (int64_t)fk::num_sms() * 4;
  if (blocks > cap) blocks = cap;
  dw_from_parts_kernel<<<(int)blocks, 256, 0, fk::as_stream(stream)>>>(
      dw_part, hidden / kPartCols, sorted_assign, n_mblk, dw);
  return fk::launch_status("fk_moe_dw_from_parts");
}
