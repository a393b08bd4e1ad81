// Bitonic sorting utilities on int32 rows (reference fusedkernels/_bitonic_primitive.py and
// fusedkernels/_bitonic_merge_primitive.py, used by the reference's v4 router tests).
//
// One CTA per row sorts the row in shared memory: N = next_pow2(width) keys, N/2 threads,
// each performing one compare-exchange per network step with a __syncthreads between
// steps.  The reference runs the same networks through a global-memory scratch row and
// tl.debug_barrier, the combination its DEBUGGING.md traces a race to; here the exchange
// buffer is the CTA's own shared memory.
#include "common.cuh"

namespace fk {
namespace {

constexpr int kMaxSortWidth = 2048;

// Sort runs of `run` keys (run | N, run a power of two) ascending, all runs independent.
__device__ __forceinline__ void block_sort_runs(int* s, int N, int run) {
  for (int k = 2; k <= run; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int t = threadIdx.x; t < N / 2; t += blockDim.x) {
        // t-th pair (i, i ^ j) with i having bit j clear
        const int i = 2 * t - (t & (j - 1));
        const int l = i + j;
        // block of size k: ascending when bit k clear; at k == run every run ascends
        const bool asc = (k == run) ? true : ((i & k) == 0);
        const int a = s[i], b = s[l];
        if ((a > b) == asc) {
          s[i] = b;
          s[l] = a;
        }
      }
      __syncthreads();
    }
  }
}

__global__ void sort_rows_kernel(const int* __restrict__ x, int64_t xs, int n, int N, int run,
                                 int pad, int* __restrict__ out, int64_t os, int out_n) {
  __shared__ int s[kMaxSortWidth];
  const int64_t row = blockIdx.x;
  for (int i = threadIdx.x; i < N; i += blockDim.x) s[i] = i < n ? x[row * xs + i] : pad;
  __syncthreads();
  block_sort_runs(s, N, run);
  for (int i = threadIdx.x; i < out_n; i += blockDim.x) out[row * os + i] = s[i];
}

__global__ void merge_topk_kernel(const int* __restrict__ a, const int* __restrict__ b, int kp,
                                  int* __restrict__ out) {
  __shared__ int s[kMaxSortWidth];
  const int64_t row = blockIdx.x;
  for (int i = threadIdx.x; i < 2 * kp; i += blockDim.x)
    s[i] = i < kp ? a[row * kp + i] : b[row * kp + i - kp];
  __syncthreads();
  block_sort_runs(s, 2 * kp, 2 * kp);
  for (int i = threadIdx.x; i < kp; i += blockDim.x) out[row * kp + i] = s[kp + i];
}

inline int pow2ceil(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

}  // namespace
}  // namespace fk

extern "C" int fk_bitonic_sort_i32(const int* x, int64_t n_rows, int width, int64_t row_stride,
                                   int* out, int64_t out_stride, void* stream) {
  FK_CHECK_ARG(n_rows >= 0 && width >= 0, "fk_bitonic_sort_i32: negative shape");
  if (n_rows == 0 || width == 0) return FK_OK;
  FK_CHECK_ARG(x && out, "fk_bitonic_sort_i32: null pointer");
  const int N = fk::pow2ceil(width);
  if (N > fk::kMaxSortWidth)
    return fk::fail(FK_ERR_UNSUPPORTED, "fk_bitonic_sort_i32: width %d > %d", width, fk::kMaxSortWidth);
  const int threads = N / 2 < 32 ? 32 : (N / 2 > 1024 ? 1024 : N / 2);
  fk::sort_rows_kernel<<<(unsigned)n_rows, threads, 0, fk::as_stream(stream)>>>(
      x, row_stride, width, N, N, 0x7fffffff, out, out_stride, width);
  return fk::launch_status("fk_bitonic_sort_i32");
}

extern "C" int fk_bitonic_sort_bounded_i32(const int* x, int64_t n_rows, int width,
                                           int64_t row_stride, int run, int* out, void* stream) {
  FK_CHECK_ARG(n_rows >= 0 && width >= 0 && run >= 1 && (run & (run - 1)) == 0,
               "fk_bitonic_sort_bounded_i32: run must be a power of two");
  if (n_rows == 0 || width == 0) return FK_OK;
  FK_CHECK_ARG(x && out, "fk_bitonic_sort_bounded_i32: null pointer");
  const int N = fk::pow2ceil(width);
  FK_CHECK_ARG(N % run == 0, "fk_bitonic_sort_bounded_i32: padded width %d not a multiple of %d", N, run);
  if (N > fk::kMaxSortWidth)
    return fk::fail(FK_ERR_UNSUPPORTED, "fk_bitonic_sort_bounded_i32: width %d > %d", width,
                    fk::kMaxSortWidth);
  const int threads = N / 2 < 32 ? 32 : (N / 2 > 1024 ? 1024 : N / 2);
  // Padding value of the reference (bitonic_sort_bounded pads with -2^30).
  fk::sort_rows_kernel<<<(unsigned)n_rows, threads, 0, fk::as_stream(stream)>>>(
      x, row_stride, width, N, run, -1073741824, out, N, N);
  return fk::launch_status("fk_bitonic_sort_bounded_i32");
}

extern "C" int fk_bitonic_merge_topk_i32(const int* a, const int* b, int64_t n_rows, int kp,
                                         int* out, void* stream) {
  FK_CHECK_ARG(n_rows >= 0 && kp >= 1 && (kp & (kp - 1)) == 0,
               "fk_bitonic_merge_topk_i32: kp must be a power of two");
  if (n_rows == 0) return FK_OK;
  FK_CHECK_ARG(a && b && out, "fk_bitonic_merge_topk_i32: null pointer");
  if (2 * kp > fk::kMaxSortWidth)
    return fk::fail(FK_ERR_UNSUPPORTED, "fk_bitonic_merge_topk_i32: kp %d too large", kp);
  const int threads = kp < 32 ? 32 : (kp > 1024 ? 1024 : kp);
  fk::merge_topk_kernel<<<(unsigned)n_rows, threads, 0, fk::as_stream(stream)>>>(a, b, kp, out);
  return fk::launch_status("fk_bitonic_merge_topk_i32");
}
