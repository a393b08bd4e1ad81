/*
 * fkb200.h -- C ABI of the B200 (sm_100a) kernels behind fusedkernels' training hot path.
 *
 * Every entry point takes raw device pointers, explicit sizes/strides and a CUDA stream
 * (passed as `void*`, i.e. a cudaStream_t / CUstream; NULL = legacy default stream).
 * All buffers are owned by the caller.  Two exceptions allocate or hold device memory:
 * fk_ipc_alloc (the expert-parallel exchange region) calls cudaMalloc, and
 * fk_rmsnorm_bwd_noalloc keeps its scratch in a module-global device array that the
 * driver creates when the library's device code is first loaded on a device.
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

/* No counterpart in the reference.  Backward of RMSNorm for callers that cannot allocate
 * device memory (for example code that only receives tensors from another framework's
 * memory pool, or that must run inside a fixed, pre-planned memory budget) and therefore
 * cannot pass fk_rmsnorm_bwd its workspace.  Results equal fk_rmsnorm_bwd's (dx exactly;
 * dw up to fp32 summation order when the shape needs more partial rows than fit).
 * The weight-gradient partials go to one fixed 8 MiB device array inside the library, which
 * every GPU that loads the library keeps until the process exits; cols must be at most
 * 2,097,152 (one fp32 partial row), larger cols are rejected with FK_ERR_UNSUPPORTED.
 * Under CUDA's lazy module loading (the default since CUDA 12.2) the array is created on a
 * device when the library's device code is first loaded there, at the latest on the first
 * call, not when the library is opened: a caller with a fixed memory budget makes one call
 * during its set-up, before it plans the rest of its memory.
 * The first call on a device looks the array's device address up (cudaGetSymbolAddress)
 * and keeps it for the life of the process; make that first call before any CUDA stream
 * capture.  The kept address is not valid after cudaDeviceReset on that device: do not
 * call this entry point after a device reset in the same process.  Every call uses the same array:
 * calls that may run at the same time on the GPU (different streams, or different host
 * threads on one device) race on it and must be serialised by the caller.
 * Allocates nothing: no cudaMalloc/cudaFree and no allocating library call. */
FK_API int fk_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* weight, int w_dtype,
                                  const float* rstd, void* dx, void* dw, int64_t rows,
                                  int64_t cols, int dtype, void* stream);

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

/* ---------------------------------------------------------------- MoE sorted dispatch
 * Sorted-row layout: the n_tokens*k (token, slot) assignments are laid out expert-major,
 * each expert's segment padded to a multiple of 128 rows (padding rows hold assignment
 * -1 and zero activations); inside a segment assignments keep (token, slot) order.
 * Every buffer is sized by the shapes alone (max_rows), so no device->host copy is needed.
 * Replaces the argsort / gather / bincount / cumsum / .tolist() / per-expert loop /
 * index_add_ of moe_layer_sorted.py:50-85. */

/* max_rows = round_up(n_tokens*k + n_experts*127, 128) and the metadata workspace size. */
FK_API int fk_moe_capacity(int64_t n_tokens, int k, int n_experts, int64_t* max_rows,
                           size_t* meta_workspace_bytes);

/* From idx/w [n_tokens, k] (int64 / fp32): counts[E], seg_start[E+1] (padded row offsets),
 * tile_expert[max_rows/128] (expert of each 128-row block, -1 past the end), n_mblk[1]
 * (valid 128-row blocks), sorted_assign/sorted_w[max_rows] (assignment index t*k+j and its
 * weight per sorted row), slot_pos[n_tokens*k] (sorted row of each assignment).
 * Deterministic (stable counting sort).  An expert id outside [0, E) sets *err_flag = 1.
 * Replaces moe_layer_sorted.py:50-68. */
FK_API int fk_moe_route_meta(const int64_t* idx, const float* w, int64_t n_tokens, int k,
                             int n_experts, int* counts, int* seg_start, int* tile_expert,
                             int* n_mblk, int* sorted_assign, float* sorted_w, int* slot_pos,
                             int64_t max_rows, void* workspace, size_t workspace_bytes,
                             int* err_flag, void* stream);

/* xs[p, :] = x[sorted_assign[p] / k, :] for the valid rows, zero for padding rows.
 * Replaces gathered_x = x_flat[sorted_token_idx] (moe_layer_sorted.py:63). */
FK_API int fk_moe_gather(const void* x, int dim, const int* sorted_assign, int k,
                         const int* n_mblk, int64_t max_rows, void* xs, int dtype, void* stream);

/* Same result as fk_moe_gather, walked by token: each of the n_tokens rows of x is read once
 * and stored to the sorted rows of its slots (slot_pos[t*k+j], -1 = slot not gathered), then
 * the padding rows (sorted_assign < 0) are zeroed.  The row-order walk reads a token row once
 * per slot; this one reads x once.  Replaces the same line, moe_layer_sorted.py:63. */
FK_API int fk_moe_gather_by_token(const void* x, int dim, const int* slot_pos, int64_t n_tokens,
                                  int k, const int* sorted_assign, const int* n_mblk,
                                  int64_t max_rows, void* xs, int dtype, void* stream);

/* out[t, :] = sum_j w[t,j] * y[slot_pos[t*k+j], :] (w == NULL: plain sum, as after
 * fk_moe_gemm_up_weighted, whose rows already carry the routing weight), fp32
 * accumulation in slot order (deterministic).
 * Replaces the weight multiply and index_add_ of moe_layer_sorted.py:82-85. */
FK_API int fk_moe_combine(const void* y, int dim, const int* slot_pos, const float* w,
                          int64_t n_tokens, int k, void* out, int dtype, void* stream);

/* Backward of the weighted fk_moe_combine: dy[p, :] = sorted_w[p] * dout[token(p), :] (zero
 * on padding rows) and dw[a] = <dout[token(a), :], y[slot_pos[a], :]> for every assignment
 * a.  Replaces the autograd of moe_layer_sorted.py:82-85 (the fp16 and fp32 layers; bf16
 * layers use the row-weighted GEMMs below and fk_moe_dw_from_parts instead). */
FK_API int fk_moe_combine_bwd(const void* dout, const void* y, int dim,
                              const int* sorted_assign, const float* sorted_w, int k,
                              const int* n_mblk, int64_t max_rows, void* dy, float* dw,
                              int dtype, void* stream);

/* Expert GEMMs on tcgen05 tensor cores (bf16 in, fp32 accumulate in TMEM, bf16 out).
 * Weights are stacked per expert: w13 [E, 2H, D] (rows 0..H-1 = w_gate, H..2H-1 = w_up of
 * moe_layer.py:26-27), w2 [E, D, H] (w_down, moe_layer.py:28).  D and H multiples of 64.
 * Kernel-side faults (a wait that timed out) set *err_flag to a non-zero code.
 * fk_moe_gemm_up:   h1 = xs @ w13[e]^T ([max_rows, 2H] = gate | up), act = silu(g) * u
 *                   (moe_layer.py:31, first two Linears and the activation).
 * fk_moe_gemm_down: y = act @ w2[e]^T ([max_rows, D]) (moe_layer.py:31, w_down).
 * fk_moe_gemm_down_dgrad: dh1 = SwiGLU'(dy @ w2[e], h1) ([max_rows, 2H] = dg | du).
 * fk_moe_gemm_up_dgrad:   dxs = dh1 @ w13[e] ([max_rows, D]).
 * fk_moe_gemm_wgrad: dw[e] = a[seg_e]^T @ b[seg_e] for every expert e ([E, m_dim, n_dim]),
 *                   a [max_rows, m_dim], b [max_rows, n_dim] (zero for empty experts).
 * Each kernel is persistent: one CTA per SM walks the tiles.  max_ctas = 0 keeps that; a
 * positive max_ctas caps the grid, leaving the other SMs free for work on another stream
 * (the expert-parallel layer runs a gradient all-reduce beside its backward GEMMs).
 * Together they replace the per-expert cuBLAS calls of moe_layer_sorted.py:70-77 and
 * their autograd backward. */
FK_API int fk_moe_gemm_up(const void* xs, int64_t max_rows, int dim, const void* w13,
                          int hidden, int n_experts, const int* tile_expert, const int* n_mblk,
                          void* h1, void* act, int max_ctas, int* err_flag, void* stream);
FK_API int fk_moe_gemm_down(const void* act, int64_t max_rows, int hidden, const void* w2,
                            int dim, int n_experts, const int* tile_expert, const int* n_mblk,
                            void* y, int max_ctas, int* err_flag, void* stream);
FK_API int fk_moe_gemm_down_dgrad(const void* dy, int64_t max_rows, int dim, const void* w2,
                                  int hidden, int n_experts, const int* tile_expert,
                                  const int* n_mblk, const void* h1, void* dh1, int max_ctas,
                                  int* err_flag, void* stream);
FK_API int fk_moe_gemm_up_dgrad(const void* dh1, int64_t max_rows, int hidden, const void* w13,
                                int dim, int n_experts, const int* tile_expert,
                                const int* n_mblk, void* dxs, int max_ctas, int* err_flag,
                                void* stream);
FK_API int fk_moe_gemm_wgrad(const void* a, int m_dim, const void* b, int n_dim,
                             int64_t max_rows, const int* seg_start, int n_experts, void* dw,
                             int max_ctas, int* err_flag, void* stream);

/* Row-weighted variants (bf16): the routing weight of every sorted row is applied in the
 * SwiGLU epilogues instead of by the combine kernels, and padding rows come out as zeros.
 * fk_moe_gemm_up_weighted: h1 = xs @ w13[e]^T, act_w = sorted_w[r] * silu(g) * u;
 *                         fk_moe_gemm_down on act_w then gives weighted rows, which
 *                         fk_moe_combine sums unweighted (w = NULL).
 * fk_moe_gemm_down_dgrad_weighted: dy holds the UNWEIGHTED output-gradient rows
 *                         (fk_moe_gather of dout); dh1 = SwiGLU'(sorted_w[r] * (dy @ w2[e]),
 *                         h1), and dw_part [max_rows, hidden / 64] fp32 receives, per 64
 *                         hidden units, the partial dots of <dy @ w2[e], act> (act
 *                         recomputed from h1).
 * fk_moe_dw_from_parts:   dw[sorted_assign[r]] = sum of row r's partials (fixed order) =
 *                         <dout[token], y_r> with y_r the row's unweighted expert output:
 *                         the routing-weight gradient fk_moe_combine_bwd computes.
 * With fk_moe_gemm_wgrad(dy, act_w) for dW2 (= sum of (w dout)^T act) they replace
 * fk_moe_combine_bwd in the layer's bf16 backward (moe_layer_sorted.py:70-85): a row gather
 * of dout instead of a pass that also re-reads every output row. */
FK_API int fk_moe_gemm_up_weighted(const void* xs, int64_t max_rows, int dim, const void* w13,
                                   int hidden, int n_experts, const int* tile_expert,
                                   const int* n_mblk, const int* sorted_assign,
                                   const float* sorted_w, void* h1, void* act_w, int max_ctas,
                                   int* err_flag, void* stream);
FK_API int fk_moe_gemm_down_dgrad_weighted(const void* dy, int64_t max_rows, int dim,
                                           const void* w2, int hidden, int n_experts,
                                           const int* tile_expert, const int* n_mblk,
                                           const int* sorted_assign, const float* sorted_w,
                                           const void* h1, void* dh1, float* dw_part,
                                           int max_ctas, int* err_flag, void* stream);
FK_API int fk_moe_dw_from_parts(const float* dw_part, int hidden, const int* sorted_assign,
                                const int* n_mblk, int64_t max_rows, float* dw, void* stream);

/* Typed variants for fp16 and fp32 layers (the reference's layers run in the caller's dtype,
 * fp32 by default: moe_layer_sorted.py:28-37, moe_layer.py:22-31).  dtype: FK_BF16 (same as
 * the entry points above), FK_F16 (fp16 operands and outputs, kind::f16 MMAs) or FK_F32.
 * FK_F32 runs the 3xTF32 split on kind::tf32 MMAs: every operand X is passed as the pair
 * (X, X_lo) produced by fk_tf32_split (X = the hi part), and the kernel accumulates
 * A_hi*B_hi + A_hi*B_lo + A_lo*B_hi in fp32 (about 2^-21 relative error per product,
 * fp32-class results); outputs and the SwiGLU epilogue are fp32.  The *_lo pointers are
 * ignored for the 16-bit dtypes (pass NULL).  Same layouts and shape rules as above; one
 * CTA per SM. */
FK_API int fk_moe_gemm_up_typed(const void* xs, const void* xs_lo, int64_t max_rows, int dim,
                                const void* w13, const void* w13_lo, int hidden, int n_experts,
                                const int* tile_expert, const int* n_mblk, void* h1, void* act,
                                int dtype, int* err_flag, void* stream);
FK_API int fk_moe_gemm_down_typed(const void* act, const void* act_lo, int64_t max_rows,
                                  int hidden, const void* w2, const void* w2_lo, int dim,
                                  int n_experts, const int* tile_expert, const int* n_mblk,
                                  void* y, int dtype, int* err_flag, void* stream);
FK_API int fk_moe_gemm_down_dgrad_typed(const void* dy, const void* dy_lo, int64_t max_rows,
                                        int dim, const void* w2, const void* w2_lo, int hidden,
                                        int n_experts, const int* tile_expert, const int* n_mblk,
                                        const void* h1, void* dh1, int dtype, int* err_flag,
                                        void* stream);
FK_API int fk_moe_gemm_up_dgrad_typed(const void* dh1, const void* dh1_lo, int64_t max_rows,
                                      int hidden, const void* w13, const void* w13_lo, int dim,
                                      int n_experts, const int* tile_expert, const int* n_mblk,
                                      void* dxs, int dtype, int* err_flag, void* stream);
FK_API int fk_moe_gemm_wgrad_typed(const void* a, const void* a_lo, int m_dim, const void* b,
                                   const void* b_lo, int n_dim, int64_t max_rows,
                                   const int* seg_start, int n_experts, void* dw, int dtype,
                                   int* err_flag, void* stream);

/* hi[i] = src[i] with its 13 low mantissa bits cleared (a tf32 value), lo[i] = src[i] - hi[i]
 * (exact), for the fp32 GEMMs above.  src, hi, lo 16-byte aligned, n elements. */
FK_API int fk_tf32_split(const float* src, int64_t n, float* hi, float* lo, void* stream);

/* Same as fk_moe_route_meta with int32 expert ids where a negative id marks an unused
 * slot (expert-parallel receive buffers carry -1 for slots owned by other ranks). */
FK_API int fk_moe_route_meta_skip(const int* idx, const float* w, int64_t n_tokens, int k,
                                  int n_experts, int* counts, int* seg_start,
                                  int* tile_expert, int* n_mblk, int* sorted_assign,
                                  float* sorted_w, int* slot_pos, int64_t max_rows,
                                  void* workspace, size_t workspace_bytes, int* err_flag,
                                  void* stream);

/* ---------------------------------------------------------------- expert parallelism
 * No counterpart in the reference (its experts are all local, moe_layer_sorted.py:37).
 * Each rank holds n_tokens local tokens; every (source, destination) pair has a fixed
 * capacity of n_tokens rows, so the all-to-all buffers are [n_ranks * n_tokens, ...].
 * fk_ep_plan: for every destination rank d, the stable list of local tokens with at least
 *   one slot on d (send_token[d*T + i]), each row's k slot entries (send_e = d's local
 *   expert id or -1, send_w = routing weight), src_pos[t*n_ranks + d] (row of token t in
 *   d's list or -1) and send_count[d].  expert_rank/expert_local: [E] placement tables
 *   (expert_local[e] = e's index among the experts of its owner).  Two passes over chunks
 *   of 256 tokens (per-chunk counts, then positions); workspace from
 *   fk_ep_plan_workspace_size.  n_ranks <= 32.
 * fk_ep_pack: send_x[r, :] = x[send_token[r], :] (rows with no token are left untouched).
 * fk_ep_unpack_sum: out[t, :] = sum_d back[d*T + src_pos[t, d], :] in rank order (fp32).
 * fk_ep_unpack_dw: dw[t, j] = back_dw[(d*T + src_pos[t, d])*k + j], d = rank of idx[t, j]. */
FK_API int fk_ep_plan_workspace_size(int64_t n_tokens, int n_ranks, size_t* bytes);
FK_API int fk_ep_plan(const int64_t* idx, const float* w, int64_t n_tokens, int k,
                      const int* expert_rank, const int* expert_local, int n_experts,
                      int n_ranks, int* send_token, int* send_e, float* send_w, int* src_pos,
                      int* send_count, void* workspace, size_t ws_bytes, int* err_flag,
                      void* stream);
FK_API int fk_ep_pack(const void* x, int dim, const int* send_token, int64_t rows, void* send_x,
                      int dtype, void* stream);
FK_API int fk_ep_unpack_sum(const void* back, int dim, const int* src_pos, int64_t n_tokens,
                            int n_ranks, void* out, int dtype, void* stream);
FK_API int fk_ep_unpack_dw(const float* back_dw, const int64_t* idx, const int* expert_rank,
                           const int* src_pos, int64_t n_tokens, int k, int n_ranks,
                           int n_experts, float* dw, void* stream);

/* ---------------------------------------------------------------- EP over peer memory
 * No counterpart in the reference (it has no distributed code).  The NVLink transport of
 * the expert-parallel layer: each rank owns one exchange region (fk_ipc_alloc, exported by
 * CUDA IPC, opened by the other ranks with fk_ipc_open) with the fixed-capacity layout of
 * fk_ep_plan; put kernels store rows directly into the peers' regions and publish a
 * per-phase sequence number into every rank's flags; fk_ep_peer_wait waits (at most
 * timeout_ms; err_flag = 16 + phase on timeout) until every rank has published the phase.
 * *_bases are DEVICE arrays of n_ranks pointers (this rank's own region included);
 * flag_bases[d] points at rank d's flags [4][n_ranks]; ctl is this rank's 24-word
 * control block (zeroed once).
 * fk_ep_peer_put_rows: row r < n_ranks*T with token send_token[r] >= 0 is copied to
 *   row_bases[r / T] row (my_rank*T + r % T); with send_e, the k slot entries of every
 *   row go to e_bases / w_bases at the same row.  Replaces fk_ep_pack + all-to-all.
 * fk_ep_peer_combine_put: for every received row j with a local slot, the weighted sum
 *   of its slots' y rows (w null: unweighted) goes to row_bases[j / T] row
 *   (my_rank*T + j % T), and with dw_rows its k entries to dw_bases at the same row.
 *   Replaces fk_moe_combine + all-to-all on the expert side. */
FK_API int fk_ipc_alloc(size_t bytes, void** ptr, void* handle64);
FK_API int fk_ipc_open(const void* handle64, void** ptr);
FK_API int fk_ipc_close(void* ptr);
FK_API int fk_ipc_free(void* ptr);
FK_API int fk_ep_peer_put_rows(const void* x, int dim, const int* send_token, int64_t n_tokens,
                               int n_ranks, int my_rank, const int* send_e, const float* send_w,
                               int k, void* const* row_bases, void* const* e_bases,
                               void* const* w_bases, unsigned* const* flag_bases, int phase,
                               unsigned* ctl, int dtype, void* stream);
FK_API int fk_ep_peer_combine_put(const void* y, int dim, const int* slot_pos, const float* w,
                                  int64_t n_tokens, int n_ranks, int my_rank, int k,
                                  const float* dw_rows, void* const* row_bases,
                                  void* const* dw_bases, unsigned* const* flag_bases, int phase,
                                  unsigned* ctl, int dtype, void* stream);
FK_API int fk_ep_peer_wait(const unsigned* flags, int n_ranks, int phase, unsigned* ctl,
                           int timeout_ms, int* err_flag, void* stream);

/* ---------------------------------------------------------------- bitonic utilities
 * int32 row sorts in shared memory, one CTA per row, rows of at most 2048 keys.
 * fk_bitonic_sort_i32: each row ascending (replaces _bitonic_sort_ascending_kernel,
 *   _bitonic_primitive.py:17-76).
 * fk_bitonic_sort_bounded_i32: rows padded to next_pow2(width) with -2^30, every run of
 *   `run` keys sorted ascending, out [n_rows, next_pow2(width)] (replaces
 *   _bitonic_sort_bounded_kernel, _bitonic_primitive.py:79-164).
 * fk_bitonic_merge_topk_i32: top kp of the union of two ascending rows, ascending
 *   (replaces _bitonic_merge_topk_kernel, _bitonic_merge_primitive.py:31-85). */
FK_API int fk_bitonic_sort_i32(const int* x, int64_t n_rows, int width, int64_t row_stride,
                               int* out, int64_t out_stride, void* stream);
FK_API int fk_bitonic_sort_bounded_i32(const int* x, int64_t n_rows, int width,
                                       int64_t row_stride, int run, int* out, void* stream);
FK_API int fk_bitonic_merge_topk_i32(const int* a, const int* b, int64_t n_rows, int kp,
                                     int* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FKB200_H */
