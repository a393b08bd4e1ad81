// Sorted-dispatch metadata, gather and combine kernels of the MoE layer, reference
// moe_layer_sorted.py:39-87.
//
// Layout in HBM.  The N*k (token, slot) assignments are laid out expert-major in a
// "sorted rows" buffer whose every expert segment starts on a 128-row boundary
// (seg_start[e] = sum over e' < e of round_up(count[e'], 128)).  Inside a segment the
// assignments keep (token, slot) order -- a stable counting sort, unlike the unstable
// argsort of moe_layer_sorted.py:58.  Padding rows carry assignment -1 and are zero in
// every activation buffer, so a 128-row GEMM tile never straddles two experts and the
// weight-gradient GEMM can reduce over whole segments.  The capacity
// N*k + E*127 rows (rounded to 128) is fixed by the shapes alone, so nothing on the path
// needs a device-to-host copy (the reference reads the counts back with .tolist(),
// moe_layer_sorted.py:67-68).
//
// Metadata is two launches: (1) per-CTA expert histograms of a contiguous chunk of
// assignments; the last CTA to finish (atomic ticket, reset by itself) sums them in a
// fixed order and writes seg_start, the per-(CTA, expert) base offsets, the m-block ->
// expert table and the number of m-blocks, and fills the padding rows; (2) each CTA
// re-reads its chunk and places every assignment at base + stable rank, computed with
// warp match/ballot masks and a per-warp prefix over experts in shared memory.
#include "common.cuh"

namespace fk {
namespace {

constexpr int kRowBatch = 4;  // 16-byte packets per lane loaded ahead in row copies

constexpr int kMetaThreads = 256;
constexpr int kMetaWarps = kMetaThreads / 32;
constexpr int kBlockRows = 128;
constexpr int kMaxExperts = 256;

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Workspace: [G][E] int histograms (become base offsets), then one int ticket.
// IDX is int64_t (router output) or int (expert-parallel receive buffers); with SKIP, a
// negative id marks an unused slot instead of an error.
template <typename IDX, bool SKIP>
__global__ void __launch_bounds__(kMetaThreads) moe_hist_kernel(
    const IDX* __restrict__ idx, int64_t n_assign, int E, int64_t chunk,
    int* __restrict__ part, unsigned int* __restrict__ ticket, int* __restrict__ counts,
    int* __restrict__ seg_start, int* __restrict__ tile_expert, int* __restrict__ n_mblk,
    int* __restrict__ sorted_assign, float* __restrict__ sorted_w, int64_t max_rows,
    int* __restrict__ err) {
  __shared__ int h[kMaxExperts];
  __shared__ bool last;
  for (int e = threadIdx.x; e < E; e += kMetaThreads) h[e] = 0;
  __syncthreads();
  const int64_t a0 = (int64_t)blockIdx.x * chunk;
  const int64_t a1 = a0 + chunk < n_assign ? a0 + chunk : n_assign;
  for (int64_t a = a0 + threadIdx.x; a < a1; a += kMetaThreads) {
    int64_t e = idx[a];
    if (e >= 0 && e < E) atomicAdd(&h[e], 1);
    else if (!SKIP || e >= E) atomicExch(err, 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kMetaThreads) part[(int64_t)blockIdx.x * E + e] = h[e];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Last CTA: totals, padded segment starts, per-(CTA, expert) bases.
  const int G = gridDim.x;
  for (int e = threadIdx.x; e < E; e += kMetaThreads) {
    int c = 0;
    for (int g = 0; g < G; ++g) c += ((volatile int*)part)[(int64_t)g * E + e];
    h[e] = c;
    counts[e] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int e = 0; e < E; ++e) {
      seg_start[e] = s;
      s += (h[e] + kBlockRows - 1) / kBlockRows * kBlockRows;
    }
    seg_start[E] = s;
    *n_mblk = s / kBlockRows;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kMetaThreads) {
    int base = seg_start[e];
    for (int g = 0; g < G; ++g) {
      int c = ((volatile int*)part)[(int64_t)g * E + e];
      part[(int64_t)g * E + e] = base;
      base += c;
    }
  }
  // m-block -> expert table and padding rows.
  for (int e = 0; e < E; ++e) {
    const int s0 = seg_start[e], s1 = seg_start[e + 1];
    for (int b = s0 / kBlockRows + threadIdx.x; b < s1 / kBlockRows; b += kMetaThreads)
      tile_expert[b] = e;
    for (int r = s0 + h[e] + threadIdx.x; r < s1; r += kMetaThreads) {
      sorted_assign[r] = -1;
      sorted_w[r] = 0.f;
    }
  }
  const int total = seg_start[E];
  for (int64_t b = total / kBlockRows + threadIdx.x; b < max_rows / kBlockRows; b += kMetaThreads)
    tile_expert[b] = -1;
  if (threadIdx.x == 0) *ticket = 0u;  // ready for the next call
}

template <typename IDX>
__global__ void __launch_bounds__(kMetaThreads) moe_scatter_kernel(
    const IDX* __restrict__ idx, const float* __restrict__ w, int64_t n_assign, int E,
    int64_t chunk, const int* __restrict__ part, int* __restrict__ sorted_assign,
    float* __restrict__ sorted_w, int* __restrict__ slot_pos) {
  __shared__ int run[kMaxExperts];
  __shared__ int wc[kMetaWarps][kMaxExperts];
  const int warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < E; e += kMetaThreads) run[e] = part[(int64_t)blockIdx.x * E + e];
  const int64_t a0 = (int64_t)blockIdx.x * chunk;
  const int64_t a1 = a0 + chunk < n_assign ? a0 + chunk : n_assign;
  for (int64_t r0 = a0; r0 < a1; r0 += kMetaThreads) {
    for (int i = threadIdx.x; i < kMetaWarps * E; i += kMetaThreads) wc[i / E][i % E] = 0;
    __syncthreads();
    const int64_t a = r0 + threadIdx.x;
    int e = -1;
    if (a < a1) {
      int64_t v = idx[a];
      e = (v >= 0 && v < E) ? (int)v : -1;
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lanemask_lt());
    if (e >= 0 && rank == 0) wc[warp][e] = __popc(peers);
    __syncthreads();
    for (int x = threadIdx.x; x < E; x += kMetaThreads) {
      int s = run[x];
      for (int ww = 0; ww < kMetaWarps; ++ww) {
        int c = wc[ww][x];
        wc[ww][x] = s;
        s += c;
      }
      run[x] = s;
    }
    __syncthreads();
    if (e >= 0) {
      const int pos = wc[warp][e] + rank;
      sorted_assign[pos] = (int)a;
      sorted_w[pos] = w[a];
      slot_pos[a] = pos;
    } else if (a < a1) {
      slot_pos[a] = -1;
    }
    __syncthreads();
  }
}

// xs[p, :] = x[token(p), :] for p < n_mblk*128; zero rows for padding.
template <typename T>
__global__ void __launch_bounds__(256) moe_gather_kernel(const T* __restrict__ x, int dim,
                                                         const int* __restrict__ sorted_assign,
                                                         int k, const int* __restrict__ n_mblk,
                                                         T* __restrict__ xs) {
  using V = Vec16<T>;
  const int64_t rows = (int64_t)(*n_mblk) * kBlockRows;
  const int nvec = dim / V::N;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t p = warp; p < rows; p += nwarps) {
    const int a = sorted_assign[p];
    T* dst = xs + p * dim;
    if (a < 0) {
      V z;
      z.u = make_uint4(0, 0, 0, 0);
      for (int v = lane; v < nvec; v += 32) st_plain(dst + v * V::N, z);
    } else {
      // kRowBatch packets per lane are loaded before they are stored (loads in flight)
      const T* src = x + (int64_t)(a / k) * dim;
      for (int v0 = 0; v0 < nvec; v0 += 32 * kRowBatch) {
        V buf[kRowBatch];
#pragma unroll
        for (int b = 0; b < kRowBatch; ++b) {
          const int v = v0 + b * 32 + lane;
          if (v < nvec) buf[b] = ld_keep(src + v * V::N);
        }
#pragma unroll
        for (int b = 0; b < kRowBatch; ++b) {
          const int v = v0 + b * 32 + lane;
          if (v < nvec) st_plain(dst + v * V::N, buf[b]);
        }
      }
    }
  }
}

// The same rows as moe_gather_kernel, walked by token: each token row is read once and
// stored to the sorted rows of its k slots (the row-order walk reads a token row once per
// slot, and x is larger than L2 at the workload's size); padding rows are zeroed after.
template <typename T>
__global__ void __launch_bounds__(256) moe_gather_by_token_kernel(
    const T* __restrict__ x, int dim, const int* __restrict__ slot_pos, int64_t n_tokens, int k,
    const int* __restrict__ sorted_assign, const int* __restrict__ n_mblk, T* __restrict__ xs) {
  using V = Vec16<T>;
  const int nvec = dim / V::N;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t t = warp; t < n_tokens; t += nwarps) {
    const int my_p = lane < k ? slot_pos[t * k + lane] : -1;
    unsigned live = __ballot_sync(0xffffffffu, my_p >= 0);
    if (k > 32) {  // slots past the first 32 (rare): any live one makes the row needed
      bool more = false;
      for (int j = 32 + lane; j < k; j += 32) more |= slot_pos[t * k + j] >= 0;
      if (__any_sync(0xffffffffu, more)) live |= 0x80000000u;  // forces the slow slot loop
    }
    if (live == 0u) continue;
    const T* src = x + t * dim;
    for (int v0 = 0; v0 < nvec; v0 += 32 * kRowBatch) {
      V buf[kRowBatch];
#pragma unroll
      for (int b = 0; b < kRowBatch; ++b) {
        const int v = v0 + b * 32 + lane;
        if (v < nvec) buf[b] = ld_stream(src + v * V::N);
      }
      if (k <= 32) {
        for (unsigned m = live; m != 0u; m &= m - 1u) {
          const int p = __shfl_sync(0xffffffffu, my_p, __ffs(m) - 1);
#pragma unroll
          for (int b = 0; b < kRowBatch; ++b) {
            const int v = v0 + b * 32 + lane;
            if (v < nvec) st_plain(xs + (int64_t)p * dim + v * V::N, buf[b]);
          }
        }
      } else {
        for (int j = 0; j < k; ++j) {
          const int p = slot_pos[t * k + j];
          if (p < 0) continue;
#pragma unroll
          for (int b = 0; b < kRowBatch; ++b) {
            const int v = v0 + b * 32 + lane;
            if (v < nvec) st_plain(xs + (int64_t)p * dim + v * V::N, buf[b]);
          }
        }
      }
    }
  }
  const int64_t rows = (int64_t)(*n_mblk) * kBlockRows;
  V z;
  z.u = make_uint4(0, 0, 0, 0);
  for (int64_t p = warp; p < rows; p += nwarps) {
    if (sorted_assign[p] >= 0) continue;
    T* dst = xs + p * dim;
    for (int v = lane; v < nvec; v += 32) st_plain(dst + v * V::N, z);
  }
}

// out[t, :] = sum_j (w ? w[t,j] : 1) * y[slot_pos[t*k+j], :], fp32 accumulation in slot
// order (deterministic).
template <typename T>
__global__ void __launch_bounds__(256) moe_combine_kernel(const T* __restrict__ y, int dim,
                                                          const int* __restrict__ slot_pos,
                                                          const float* __restrict__ w,
                                                          int64_t n_tokens, int k,
                                                          T* __restrict__ out) {
  using V = Vec16<T>;
  const int nvec = dim / V::N;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t t = warp; t < n_tokens; t += nwarps) {
    if (k <= 32) {
      // Lane j holds slot j's row and weight; the slots are summed in slot order (as
      // below), kRowBatch packets per lane at a time to keep loads in flight.
      const int my_p = lane < k ? slot_pos[t * k + lane] : -1;
      const float my_w = (lane < k && w) ? w[t * k + lane] : 1.0f;
      const unsigned live = __ballot_sync(0xffffffffu, my_p >= 0);
      for (int v0 = 0; v0 < nvec; v0 += 32 * kRowBatch) {
        float acc[kRowBatch][V::N];
#pragma unroll
        for (int b = 0; b < kRowBatch; ++b)
#pragma unroll
          for (int i = 0; i < V::N; ++i) acc[b][i] = 0.f;
        for (unsigned m = live; m != 0u; m &= m - 1u) {
          const int j = __ffs(m) - 1;
          const int p = __shfl_sync(0xffffffffu, my_p, j);
          const float wj = __shfl_sync(0xffffffffu, my_w, j);
          V r[kRowBatch];
#pragma unroll
          for (int b = 0; b < kRowBatch; ++b) {
            const int v = v0 + b * 32 + lane;
            if (v < nvec) r[b] = ld_keep(y + (int64_t)p * dim + v * V::N);
          }
#pragma unroll
          for (int b = 0; b < kRowBatch; ++b)
#pragma unroll
            for (int i = 0; i < V::N; ++i) acc[b][i] = fmaf(wj, Elt<T>::to_f(r[b].e[i]), acc[b][i]);
        }
#pragma unroll
        for (int b = 0; b < kRowBatch; ++b) {
          const int v = v0 + b * 32 + lane;
          if (v >= nvec) continue;
          V o;
#pragma unroll
          for (int i = 0; i < V::N; ++i) o.e[i] = Elt<T>::from_f(acc[b][i]);
          st_plain(out + t * dim + v * V::N, o);
        }
      }
      continue;
    }
    for (int v = lane; v < nvec; v += 32) {
      float acc[V::N];
#pragma unroll
      for (int i = 0; i < V::N; ++i) acc[i] = 0.f;
      for (int j = 0; j < k; ++j) {
        const int p = slot_pos[t * k + j];
        if (p < 0) continue;
        const float wj = w ? w[t * k + j] : 1.0f;
        V r = ld_keep(y + (int64_t)p * dim + v * V::N);
#pragma unroll
        for (int i = 0; i < V::N; ++i) acc[i] = fmaf(wj, Elt<T>::to_f(r.e[i]), acc[i]);
      }
      V o;
#pragma unroll
      for (int i = 0; i < V::N; ++i) o.e[i] = Elt<T>::from_f(acc[i]);
      st_plain(out + t * dim + v * V::N, o);
    }
  }
}

// Backward of the weighted combine.  Per sorted row p holding assignment a (token t):
//   dy[p, :] = w[a] * dout[t, :]            (zero rows for padding)
//   dw[a]    = <dout[t, :], y[p, :]>         (fp32, fixed-order warp reduction)
template <typename T>
__global__ void __launch_bounds__(256) moe_combine_bwd_kernel(
    const T* __restrict__ dout, const T* __restrict__ y, int dim,
    const int* __restrict__ sorted_assign, const float* __restrict__ sorted_w, int k,
    const int* __restrict__ n_mblk, T* __restrict__ dy, float* __restrict__ dw) {
  using V = Vec16<T>;
  const int64_t rows = (int64_t)(*n_mblk) * kBlockRows;
  const int nvec = dim / V::N;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t p = warp; p < rows; p += nwarps) {
    const int a = sorted_assign[p];
    T* dst = dy + p * dim;
    if (a < 0) {
      V z;
      z.u = make_uint4(0, 0, 0, 0);
      for (int v = lane; v < nvec; v += 32) st_plain(dst + v * V::N, z);
      continue;
    }
    const float wa = sorted_w[p];
    const T* g = dout + (int64_t)(a / k) * dim;
    const T* yr = y + p * dim;
    float dot = 0.f;
    // packets in the same order as one-at-a-time processing (the dot product's summation
    // order is unchanged), kRowBatch of each operand loaded ahead
    for (int v0 = 0; v0 < nvec; v0 += 32 * kRowBatch) {
      V gv[kRowBatch], yv[kRowBatch];
#pragma unroll
      for (int b = 0; b < kRowBatch; ++b) {
        const int v = v0 + b * 32 + lane;
        if (v < nvec) {
          gv[b] = ld_keep(g + v * V::N);
          yv[b] = ld_keep(yr + v * V::N);
        }
      }
#pragma unroll
      for (int b = 0; b < kRowBatch; ++b) {
        const int v = v0 + b * 32 + lane;
        if (v >= nvec) continue;
        V o;
#pragma unroll
        for (int i = 0; i < V::N; ++i) {
          const float gf = Elt<T>::to_f(gv[b].e[i]);
          dot = fmaf(gf, Elt<T>::to_f(yv[b].e[i]), dot);
          o.e[i] = Elt<T>::from_f(wa * gf);
        }
        st_plain(dst + v * V::N, o);
      }
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[a] = dot;
  }
}

inline int rows_grid(int64_t rows) {
  int64_t g = (rows + 7) / 8;
  int64_t cap = (int64_t)num_sms() * 8;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

int64_t moe_capacity_rows(int64_t n_tokens, int k, int n_experts) {
  int64_t r = n_tokens * k + (int64_t)n_experts * (kBlockRows - 1);
  return (r + kBlockRows - 1) / kBlockRows * kBlockRows;
}

static int meta_grid(int64_t n_assign) {
  int64_t g = (n_assign + 2047) / 2048;
  int64_t cap = (int64_t)num_sms();
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

size_t moe_meta_ws_bytes(int64_t n_tokens, int k, int n_experts) {
  int G = meta_grid(n_tokens * k);
  return ((size_t)G * n_experts + 4) * sizeof(int);
}

}  // namespace fk

extern "C" int fk_moe_capacity(int64_t n_tokens, int k, int n_experts, int64_t* max_rows,
                               size_t* meta_workspace_bytes) {
  FK_CHECK_ARG(n_tokens >= 0 && k >= 1 && n_experts >= 1 && n_experts <= fk::kMaxExperts,
               "fk_moe_capacity: bad sizes (N=%lld k=%d E=%d)", (long long)n_tokens, k, n_experts);
  FK_CHECK_ARG(max_rows && meta_workspace_bytes, "fk_moe_capacity: null output");
  *max_rows = fk::moe_capacity_rows(n_tokens, k, n_experts);
  *meta_workspace_bytes = fk::moe_meta_ws_bytes(n_tokens, k, n_experts);
  return FK_OK;
}

namespace fk {
template <typename IDX, bool SKIP>
static int route_meta_t(const IDX* idx, const float* w, int64_t n_tokens, int k, int n_experts,
                        int* counts, int* seg_start, int* tile_expert, int* n_mblk,
                        int* sorted_assign, float* sorted_w, int* slot_pos, int64_t max_rows,
                        void* workspace, size_t workspace_bytes, int* err_flag, void* stream) {
  FK_CHECK_ARG(n_tokens >= 0 && k >= 1 && n_experts >= 1 && n_experts <= kMaxExperts,
               "fk_moe_route_meta: bad sizes");
  FK_CHECK_ARG(counts && seg_start && tile_expert && n_mblk && sorted_assign && sorted_w &&
                   err_flag && (n_tokens == 0 || (idx && w && slot_pos)),
               "fk_moe_route_meta: null pointer");
  FK_CHECK_ARG(max_rows >= moe_capacity_rows(n_tokens, k, n_experts),
               "fk_moe_route_meta: max_rows %lld below capacity", (long long)max_rows);
  const size_t need = moe_meta_ws_bytes(n_tokens, k, n_experts);
  if (!workspace || workspace_bytes < need)
    return fail(FK_ERR_WORKSPACE, "fk_moe_route_meta: need %zu workspace bytes", need);
  cudaStream_t st = as_stream(stream);
  const int64_t n_assign = n_tokens * k;
  const int G = meta_grid(n_assign);
  const int64_t chunk = (n_assign + G - 1) / G;
  int* part = static_cast<int*>(workspace);
  unsigned int* ticket = reinterpret_cast<unsigned int*>(part + (size_t)G * n_experts);
  // The ticket must start at zero; the kernel's last CTA resets it after every call.
  cudaMemsetAsync(ticket, 0, sizeof(unsigned int), st);
  cudaMemsetAsync(err_flag, 0, sizeof(int), st);
  moe_hist_kernel<IDX, SKIP><<<G, kMetaThreads, 0, st>>>(idx, n_assign, n_experts,
                                                        chunk < 1 ? 1 : chunk, part, ticket, counts,
                                                        seg_start, tile_expert, n_mblk,
                                                        sorted_assign, sorted_w, max_rows, err_flag);
  int s = launch_status("fk_moe_route_meta(hist)");
  if (s != FK_OK || n_assign == 0) return s;
  moe_scatter_kernel<IDX><<<G, kMetaThreads, 0, st>>>(idx, w, n_assign, n_experts, chunk, part,
                                                      sorted_assign, sorted_w, slot_pos);
  return launch_status("fk_moe_route_meta(scatter)");
}
}  // namespace fk

extern "C" int fk_moe_route_meta(const int64_t* idx, const float* w, int64_t n_tokens, int k,
                                 int n_experts, int* counts, int* seg_start, int* tile_expert,
                                 int* n_mblk, int* sorted_assign, float* sorted_w,
                                 int* slot_pos, int64_t max_rows, void* workspace,
                                 size_t workspace_bytes, int* err_flag, void* stream) {
  return fk::route_meta_t<int64_t, false>(idx, w, n_tokens, k, n_experts, counts, seg_start,
                                          tile_expert, n_mblk, sorted_assign, sorted_w, slot_pos,
                                          max_rows, workspace, workspace_bytes, err_flag, stream);
}

extern "C" int fk_moe_route_meta_skip(const int* idx, const float* w, int64_t n_tokens, int k,
                                      int n_experts, int* counts, int* seg_start,
                                      int* tile_expert, int* n_mblk, int* sorted_assign,
                                      float* sorted_w, int* slot_pos, int64_t max_rows,
                                      void* workspace, size_t workspace_bytes, int* err_flag,
                                      void* stream) {
  return fk::route_meta_t<int, true>(idx, w, n_tokens, k, n_experts, counts, seg_start,
                                     tile_expert, n_mblk, sorted_assign, sorted_w, slot_pos,
                                     max_rows, workspace, workspace_bytes, err_flag, stream);
}

extern "C" int fk_moe_gather(const void* x, int dim, const int* sorted_assign, int k,
                             const int* n_mblk, int64_t max_rows, void* xs, int dtype,
                             void* stream) {
  FK_CHECK_ARG(x && sorted_assign && n_mblk && xs && k >= 1 && max_rows >= 0,
               "fk_moe_gather: bad argument");
  FK_CHECK_ARG(fk::valid_dtype(dtype) && dim > 0 && (dim * fk::dtype_size(dtype)) % 16 == 0,
               "fk_moe_gather: dim*elt must be a multiple of 16 bytes");
  FK_CHECK_ARG(fk::aligned16(x) && fk::aligned16(xs), "fk_moe_gather: unaligned buffers");
  cudaStream_t st = fk::as_stream(stream);
  FK_DISPATCH_DTYPE(dtype, fk::moe_gather_kernel<scalar_t><<<fk::rows_grid(max_rows), 256, 0, st>>>(
                               static_cast<const scalar_t*>(x), dim, sorted_assign, k, n_mblk,
                               static_cast<scalar_t*>(xs)));
  return fk::launch_status("fk_moe_gather");
}

extern "C" int fk_moe_gather_by_token(const void* x, int dim, const int* slot_pos,
                                      int64_t n_tokens, int k, const int* sorted_assign,
                                      const int* n_mblk, int64_t max_rows, void* xs, int dtype,
                                      void* stream) {
  FK_CHECK_ARG(x && slot_pos && sorted_assign && n_mblk && xs && k >= 1 && max_rows >= 0 &&
                   n_tokens >= 0,
               "fk_moe_gather_by_token: bad argument");
  FK_CHECK_ARG(fk::valid_dtype(dtype) && dim > 0 && (dim * fk::dtype_size(dtype)) % 16 == 0,
               "fk_moe_gather_by_token: dim*elt must be a multiple of 16 bytes");
  FK_CHECK_ARG(fk::aligned16(x) && fk::aligned16(xs), "fk_moe_gather_by_token: unaligned buffers");
  if (max_rows == 0) return FK_OK;
  cudaStream_t st = fk::as_stream(stream);
  const int64_t work = n_tokens > max_rows ? n_tokens : max_rows;
  FK_DISPATCH_DTYPE(dtype, fk::moe_gather_by_token_kernel<scalar_t>
                    <<<fk::rows_grid(work), 256, 0, st>>>(
                        static_cast<const scalar_t*>(x), dim, slot_pos, n_tokens, k,
                        sorted_assign, n_mblk, static_cast<scalar_t*>(xs)));
  return fk::launch_status("fk_moe_gather_by_token");
}

extern "C" int fk_moe_combine(const void* y, int dim, const int* slot_pos, const float* w,
                              int64_t n_tokens, int k, void* out, int dtype, void* stream) {
  FK_CHECK_ARG(n_tokens >= 0 && k >= 1, "fk_moe_combine: bad sizes");
  if (n_tokens == 0) return FK_OK;
  FK_CHECK_ARG(y && slot_pos && out, "fk_moe_combine: null pointer");
  FK_CHECK_ARG(fk::valid_dtype(dtype) && dim > 0 && (dim * fk::dtype_size(dtype)) % 16 == 0,
               "fk_moe_combine: dim*elt must be a multiple of 16 bytes");
  FK_CHECK_ARG(fk::aligned16(y) && fk::aligned16(out), "fk_moe_combine: unaligned buffers");
  cudaStream_t st = fk::as_stream(stream);
  FK_DISPATCH_DTYPE(dtype, fk::moe_combine_kernel<scalar_t><<<fk::rows_grid(n_tokens), 256, 0, st>>>(
                               static_cast<const scalar_t*>(y), dim, slot_pos, w, n_tokens, k,
                               static_cast<scalar_t*>(out)));
  return fk::launch_status("fk_moe_combine");
}

extern "C" int fk_moe_combine_bwd(const void* dout, const void* y, int dim,
                                  const int* sorted_assign, const float* sorted_w, int k,
                                  const int* n_mblk, int64_t max_rows, void* dy, float* dw,
                                  int dtype, void* stream) {
  FK_CHECK_ARG(dout && y && sorted_assign && sorted_w && n_mblk && dy && dw && k >= 1,
               "fk_moe_combine_bwd: bad argument");
  FK_CHECK_ARG(fk::valid_dtype(dtype) && dim > 0 && (dim * fk::dtype_size(dtype)) % 16 == 0,
               "fk_moe_combine_bwd: dim*elt must be a multiple of 16 bytes");
  FK_CHECK_ARG(fk::aligned16(dout) && fk::aligned16(y) && fk::aligned16(dy),
               "fk_moe_combine_bwd: unaligned buffers");
  cudaStream_t st = fk::as_stream(stream);
  FK_DISPATCH_DTYPE(dtype, fk::moe_combine_bwd_kernel<scalar_t>
                    <<<fk::rows_grid(max_rows), 256, 0, st>>>(
                        static_cast<const scalar_t*>(dout), static_cast<const scalar_t*>(y), dim,
                        sorted_assign, sorted_w, k, n_mblk, static_cast<scalar_t*>(dy), dw));
  return fk::launch_status("fk_moe_combine_bwd");
}
