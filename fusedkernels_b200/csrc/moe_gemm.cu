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
