// fp16 and fp32 entry points of the MoE expert GEMMs (kernel template in moe_gemm.cuh).
// The reference's layers are plain nn.Modules in whatever dtype the caller gives them
// (fp32 by default: moe_layer_sorted.py:28-37, moe_layer.py:22-31); fp16 layers run on
// kind::f16 MMAs like bf16, fp32 layers on kind::tf32 MMAs with the 3xTF32 split, whose
// operand halves fk_tf32_split produces.
#include "moe_gemm.cuh"

namespace fk {
namespace {

// hi = x with the low 13 mantissa bits cleared (exactly representable in tf32: the tensor
// core reads it without rounding), lo = x - hi (exact in fp32).  16-byte packets.
__global__ void tf32_split_kernel(const float4* __restrict__ src, int64_t n4,
                                  float4* __restrict__ hi, float4* __restrict__ lo) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = src[i];
    float4 h, l;
    h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
    h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
    h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
    h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
    l.x = v.x - h.x;
    l.y = v.y - h.y;
    l.z = v.z - h.z;
    l.w = v.w - h.w;
    hi[i] = h;
    lo[i] = l;
  }
}

__global__ void tf32_split_tail(const float* __restrict__ src, int64_t i0, int64_t n,
                                float* __restrict__ hi, float* __restrict__ lo) {
  const int64_t i = i0 + threadIdx.x;
  if (i < n) {
    const float v = src[i];
    const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    hi[i] = h;
    lo[i] = v - h;
  }
}

}  // namespace
}  // namespace fk

namespace G = fk::gemm;

extern "C" int fk_tf32_split(const float* src, int64_t n, float* hi, float* lo, void* stream) {
  FK_CHECK_ARG(n >= 0, "fk_tf32_split: negative size");
  if (n == 0) return FK_OK;
  FK_CHECK_ARG(src && hi && lo, "fk_tf32_split: null pointer");
  FK_CHECK_ARG(fk::aligned16(src) && fk::aligned16(hi) && fk::aligned16(lo),
               "fk_tf32_split: pointers must be 16-byte aligned");
  cudaStream_t st = fk::as_stream(stream);
  const int64_t n4 = n / 4;
  if (n4 > 0) {
    int64_t blocks = (n4 + 255) / 256;
    const int64_t cap = (int64_t)fk::num_sms() * 8;
    if (blocks > cap) blocks = cap;
    fk::tf32_split_kernel<<<(int)blocks, 256, 0, st>>>(
        reinterpret_cast<const float4*>(src), n4, reinterpret_cast<float4*>(hi),
        reinterpret_cast<float4*>(lo));
    int s = fk::launch_status("fk_tf32_split");
    if (s != FK_OK) return s;
  }
  if (n4 * 4 < n) {
    fk::tf32_split_tail<<<1, 32, 0, st>>>(src, n4 * 4, n, hi, lo);
    return fk::launch_status("fk_tf32_split(tail)");
  }
  return FK_OK;
}

#define FK_KIND_SWITCH(dtype, NAME, ...)                                                    \
  switch (dtype) {                                                                          \
    case FK_BF16: { constexpr int K_ = G::KIND_BF16; __VA_ARGS__; }                         \
    case FK_F16: { constexpr int K_ = G::KIND_F16; __VA_ARGS__; }                           \
    case FK_F32: { constexpr int K_ = G::KIND_TF32X3; __VA_ARGS__; }                        \
    default: return fk::fail(FK_ERR_INVALID_ARG, NAME ": bad dtype code %d", (int)(dtype)); \
  }

extern "C" int fk_moe_gemm_up_typed(const void* xs, const void* xs_lo, int64_t max_rows, int dim,
                                    const void* w13, const void* w13_lo, int hidden, int n_experts,
                                    const int* tile_expert, const int* n_mblk, void* h1, void* act,
                                    int dtype, int* err_flag, void* stream) {
  FK_KIND_SWITCH(dtype, "fk_moe_gemm_up_typed",
                 return G::gemm_up<K_>(xs, xs_lo, max_rows, dim, w13, w13_lo, hidden, n_experts,
                                       tile_expert, n_mblk, h1, act, err_flag,
                                       fk::as_stream(stream)));
}

extern "C" int fk_moe_gemm_down_typed(const void* act, const void* act_lo, int64_t max_rows,
                                      int hidden, const void* w2, const void* w2_lo, int dim,
                                      int n_experts, const int* tile_expert, const int* n_mblk,
                                      void* y, int dtype, int* err_flag, void* stream) {
  FK_KIND_SWITCH(dtype, "fk_moe_gemm_down_typed",
                 return G::gemm_down<K_>(act, act_lo, max_rows, hidden, w2, w2_lo, dim, n_experts,
                                         tile_expert, n_mblk, y, err_flag,
                                         fk::as_stream(stream)));
}

extern "C" int fk_moe_gemm_down_dgrad_typed(const void* dy, const void* dy_lo, int64_t max_rows,
                                            int dim, const void* w2, const void* w2_lo, int hidden,
                                            int n_experts, const int* tile_expert,
                                            const int* n_mblk, const void* h1, void* dh1,
                                            int dtype, int* err_flag, void* stream) {
  FK_KIND_SWITCH(dtype, "fk_moe_gemm_down_dgrad_typed",
                 return G::gemm_down_dgrad<K_>(dy, dy_lo, max_rows, dim, w2, w2_lo, hidden,
                                               n_experts, tile_expert, n_mblk, h1, dh1, err_flag,
                                               fk::as_stream(stream)));
}

extern "C" int fk_moe_gemm_up_dgrad_typed(const void* dh1, const void* dh1_lo, int64_t max_rows,
                                          int hidden, const void* w13, const void* w13_lo, int dim,
                                          int n_experts, const int* tile_expert,
                                          const int* n_mblk, void* dxs, int dtype, int* err_flag,
                                          void* stream) {
  FK_KIND_SWITCH(dtype, "fk_moe_gemm_up_dgrad_typed",
                 return G::gemm_up_dgrad<K_>(dh1, dh1_lo, max_rows, hidden, w13, w13_lo, dim,
                                             n_experts, tile_expert, n_mblk, dxs, err_flag,
                                             fk::as_stream(stream)));
}

extern "C" int fk_moe_gemm_wgrad_typed(const void* a, const void* a_lo, int m_dim, const void* b,
                                       const void* b_lo, int n_dim, int64_t max_rows,
                                       const int* seg_start, int n_experts, void* dw, int dtype,
                                       int* err_flag, void* stream) {
  FK_KIND_SWITCH(dtype, "fk_moe_gemm_wgrad_typed",
                 return G::gemm_wgrad<K_>(a, a_lo, m_dim, b, b_lo, n_dim, max_rows, seg_start,
                                          n_experts, dw, err_flag, fk::as_stream(stream)));
}
