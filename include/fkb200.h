/*
 * fkb200.h -- C ABI of the B200 (sm_100a) kernels behind fusedkernels' training hot path.
 *
 * Every entry point takes raw device pointers, explicit sizes/strides and a CUDA stream
 * (passed as `void*`, i.e. a cudaStream_t / CUstream; NULL = legacy default stream).
 * All buffers are owned by the caller; no entry point allocates device memory.
 * Work is enqueued asynchronously on `stream`; the return value only reports argument
 * and launch errors (FK_OK == 0).  Device-side data errors (e.g. an out-of-range
 * cross-entropy target) are reported through a caller-provided int flag in device memory.
 *
 * Element-type codes (`dtype`): FK_F32, FK_F16, FK_BF16.
 *
 * Each function names the reference interface it replaces (paths are relative to the
 * fusedkernels source tree, Siddhuuuu/fusedKernels v0.2.0).
 */
#ifndef FKB200_H
#define FKB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FK_API __attribute__((visibility("default")))
#else
#define FK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum fk_dtype { FK_F32 = 0, FK_F16 = 1, FK_BF16 = 2 };

enum fk_status {
  FK_OK = 0,
  FK_ERR_INVALID_ARG = 1,  /* null pointer, bad dtype, negative size, k > E ...     */
  FK_ERR_UNSUPPORTED = 2,  /* shape outside what the kernels implement               */
  FK_ERR_LAUNCH = 3,       /* cudaLaunch* failed (message via fk_last_error)         */
  FK_ERR_WORKSPACE = 4,    /* workspace pointer/size too small for this call         */
  FK_ERR_NO_DEVICE = 5     /* no CUDA device / driver entry point unavailable        */
};

/* Library version as an integer (major*10000 + minor*100 + patch). */
FK_API int fk_version(void);
/* Human-readable text for a status code (static storage). */
FK_API const char* fk_status_string(int status);
/* Detail message for the last non-OK status returned on the calling thread. */
FK_API const char* fk_last_error(void);

/* ---------------------------------------------------------------- SwiGLU ---------
 * out = silu(gate) * up, elementwise over n contiguous elements, fp32 arithmetic.
 * Replaces swiglu.py:19-30 (_swiglu_fwd_kernel) launched from swiglu.py:56-67. */
FK_API int fk_swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, int dtype,
                  void* stream);

/* dgate = dout * up * sig(g) * (1 + g * (1 - sig(g))),  dup = dout * silu(g).
 * Replaces swiglu.py:33-51 (_swiglu_bwd_kernel) launched from swiglu.py:70-81. */
FK_API int fk_swiglu_bwd(const void* dout, const void* gate, const void* up, void* dgate,
                  void* dup, int64_t n, int dtype, void* stream);

/* ---------------------------------------------------------------- RMSNorm --------
 * y = x * rsqrt(mean(x^2) + eps) * w per row; rstd[r] saved for the backward.
 * x, y: [rows, cols] with row strides in elements; weight: [cols] of w_dtype.
 * Replaces rmsnorm.py:20-41 (_rmsnorm_fwd_kernel) launched from rmsnorm.py:76-94. */
FK_API int fk_rmsnorm_fwd(const void* x, int64_t x_row_stride, const void* weight, int w_dtype,
                   void* y, int64_t y_row_stride, float* rstd, int64_t rows, int64_t cols,
                   float eps, int dtype, void* stream);

/* Bytes of workspace fk_rmsnorm_bwd needs for this shape on the current device. */
FK_API int fk_rmsnorm_bwd_workspace_size(int64_t rows, int64_t cols, size_t* bytes);

/* dx = rstd*w*dy - x*rstd^3*mean(w*dy*x);  dw = sum_rows(dy*x*rstd) (deterministic:
 * fixed per-CTA fp32 partials in `workspace`, then a fixed-order column reduce).
 * dw is written in w_dtype.  dy/x/dx rows are contiguous (row stride == cols).
 * Replaces rmsnorm.py:44-71 (_rmsnorm_bwd_kernel) plus the torch reduce at
 * rmsnorm.py:104 and rmsnorm.py:112. */
FK_API int fk_rmsnorm_bwd(const void* dy, const void* x, const void* weight, int w_dtype,
                   const float* rstd, void* dx, void* dw, void* workspace,
                   size_t workspace_bytes, int64_t rows, int64_t cols, int dtype,
                   void* stream);

/* ---------------------------------------------------------------- MoE router -----
 * Per row of logits [n_rows, n_experts] (row stride in elements): rank experts by the
 * exact logit value (ties -> lower expert index first; -0.0 == +0.0; NaN ranks above
 * +inf), keep the top k, and write w[r, j] = softmax restricted to the k selected
 * logits (== renormalised full softmax) and idx[r, j] (int64), j in rank order.
 * n_experts <= 256, 1 <= k <= n_experts.
 * Replaces moe_routing_v2.py:44-99 (_moe_route_fwd_kernel_v2) and the launch plus the
 * int32->int64 copy at moe_routing_v2.py:131-160. */
FK_API int fk_router_fwd(const void* logits, int64_t row_stride, int dtype, int64_t n_rows,
                  int n_experts, int k, float* w, int64_t* idx, void* stream);

/* dlogits[r, idx[r,j]] = w[r,j] * (dw[r,j] - sum_m w[r,m]*dw[r,m]); every other entry
 * of the dense fp32 row is written 0 (no separate memset).
 * Replaces moe_routing_v2.py:102-126 (_moe_route_bwd_kernel_v2) and the torch.zeros
 * plus launch at moe_routing_v2.py:162-177. */
FK_API int fk_router_bwd(const float* dw, const float* w, const int64_t* idx, float* dlogits,
                  int64_t n_rows, int n_experts, int k, void* stream);

/* ---------------------------------------------------------------- Cross-entropy --
 * Forward + gradient in one pass over each row of logits [n_rows, n_cols]:
 *   lse = logsumexp(row);  loss_r = (1-ls)(lse - x_t) + ls(lse - mean(row)),
 *   grad_r = (softmax(row) - (1-ls)*onehot(t) - ls/n_cols) / n_valid,
 * rows with target == ignore_index get loss 0 and a zero gradient row.
 * n_valid = max(1, #targets != ignore_index).  `grad` may alias `logits` (in-place
 * gradient write-back).  Outputs: loss_rows[n_rows] (per-row losses, fp32),
 * loss[0] = sum(loss_rows) / n_valid (fixed-order sum), n_valid[0].  An out-of-range
 * target sets *err_flag = 1 and makes that row's loss and gradient NaN.
 * Replaces cross_entropy.py:24-79 (_cross_entropy_fwd_bwd_kernel), the launch at
 * cross_entropy.py:83-110 and the grad_output scale of cross_entropy.py:113-116
 * (folded: the gradient already carries 1/n_valid). */
FK_API int fk_ce_fwd(const void* logits, int64_t row_stride, void* grad, int64_t grad_row_stride,
              const int64_t* targets, int64_t n_rows, int64_t n_cols, int64_t ignore_index,
              float label_smoothing, int dtype, float* loss_rows, float* loss,
              int* n_valid, int* err_flag, void* stream);

/* grad *= grad_output[0] unless grad_output[0] == 1 (decided on the device: the launch
 * exits without touching grad).  grad: [n_rows, n_cols] with row stride.
 * Replaces the `grad * scale` of cross_entropy.py:115-116. */
FK_API int fk_ce_bwd_scale(void* grad, int64_t grad_row_stride, int64_t n_rows, int64_t n_cols,
                    const float* grad_output, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FKB200_H */
