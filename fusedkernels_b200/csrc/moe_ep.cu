// Expert-parallel token exchange for the MoE layer: per-destination packing of token
// rows before the dispatch all-to-all and the fixed-order reduction of the returned
// partial rows after the combine all-to-all.  (The reference has no distributed code:
// all experts are local, moe_layer_sorted.py:37.)
//
// Layout.  Each rank holds T local tokens.  A token is sent ONCE to every rank that owns
// at least one of its k experts (deduplication); the row carries k slot entries (the
// destination's LOCAL expert id, or -1 when that slot's expert lives elsewhere, and the
// routing weight).  Every (source, destination) pair has a fixed capacity of T rows, so
// the all-to-all moves [n_ranks, T, D] with equal splits and no host-side sizes; rows at
// or past a destination's count are never read by the receiver (their slots are -1).
// The expert side pre-reduces the outputs of a row's local slots into one partial row,
// and the source adds the partial rows of its token in rank order (deterministic).
#include "common.cuh"

namespace fk {
namespace {

constexpr int kPlanThreads = 256;  // tokens per planning CTA

__device__ __forceinline__ uint32_t lanes_below() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Bit d of the result: token t has at least one slot on rank d.
__device__ __forceinline__ uint32_t dest_mask(const int64_t* __restrict__ idx, int64_t t, int k,
                                              const int* __restrict__ expert_rank, int E,
                                              int* __restrict__ err) {
  uint32_t m = 0;
  for (int j = 0; j < k; ++j) {
    const int64_t e = idx[t * k + j];
    if (e < 0 || e >= E) {
      if (err) atomicExch(err, 1);
      continue;
    }
    m |= 1u << expert_rank[e];
  }
  return m;
}

// Pass 1: per chunk of kPlanThreads tokens, how many have a slot on each rank.
__global__ void __launch_bounds__(kPlanThreads) ep_plan_count_kernel(
    const int64_t* __restrict__ idx, int64_t T, int k, const int* __restrict__ expert_rank, int E,
    int n_ranks, int* __restrict__ chunk_count, int* __restrict__ err) {
  const int64_t t = (int64_t)blockIdx.x * kPlanThreads + threadIdx.x;
  const uint32_t m = t < T ? dest_mask(idx, t, k, expert_rank, E, err) : 0u;
  for (int d = 0; d < n_ranks; ++d) {
    const int c = __syncthreads_count((m >> d) & 1u);
    if (threadIdx.x == 0) chunk_count[(int64_t)blockIdx.x * n_ranks + d] = c;
  }
}

// Pass 2: stable position of every token in every destination's list (counts of the
// earlier chunks + rank inside this chunk), the send lists, and -1 rows past every
// destination's count (rows c*kPlanThreads + tid of each destination).
__global__ void __launch_bounds__(kPlanThreads) ep_plan_fill_kernel(
    const int64_t* __restrict__ idx, const float* __restrict__ w, int64_t T, int k,
    const int* __restrict__ expert_rank, const int* __restrict__ expert_local, int E,
    int n_ranks, const int* __restrict__ chunk_count, int n_chunks, int* __restrict__ send_token,
    int* __restrict__ send_e, float* __restrict__ send_w, int* __restrict__ src_pos,
    int* __restrict__ send_count) {
  constexpr int kWarps = kPlanThreads / 32;
  __shared__ int base[32], total[32];
  __shared__ uint32_t wbal[kWarps][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x;
  if (tid < n_ranks) {
    int b = 0, tot = 0;
    for (int i = 0; i < n_chunks; ++i) {
      const int v = chunk_count[(int64_t)i * n_ranks + tid];
      if (i < c) b += v;
      tot += v;
    }
    base[tid] = b;
    total[tid] = tot;
    if (c == 0) send_count[tid] = tot;
  }
  const int64_t t = (int64_t)c * kPlanThreads + tid;
  const uint32_t m = t < T ? dest_mask(idx, t, k, expert_rank, E, nullptr) : 0u;
  for (int d = 0; d < n_ranks; ++d) {
    const uint32_t bal = __ballot_sync(0xffffffffu, (m >> d) & 1u);
    if (lane == 0) wbal[warp][d] = bal;
  }
  __syncthreads();
  if (t < T) {
    for (int d = 0; d < n_ranks; ++d) {
      if (!((m >> d) & 1u)) {
        src_pos[t * n_ranks + d] = -1;
        continue;
      }
      int pos = base[d] + __popc(wbal[warp][d] & lanes_below());
      for (int i = 0; i < warp; ++i) pos += __popc(wbal[i][d]);
      src_pos[t * n_ranks + d] = pos;
      const int64_t r = (int64_t)d * T + pos;
      send_token[r] = (int)t;
      for (int j = 0; j < k; ++j) {
        const int64_t e = idx[t * k + j];
        const bool mine = e >= 0 && e < E && expert_rank[e] == d;
        send_e[r * k + j] = mine ? expert_local[e] : -1;
        send_w[r * k + j] = w[t * k + j];
      }
    }
  }
  const int64_t p = (int64_t)c * kPlanThreads + tid;
  if (p < T) {
    for (int d = 0; d < n_ranks; ++d) {
      if (p < total[d]) continue;
      const int64_t r = (int64_t)d * T + p;
      send_token[r] = -1;
      for (int j = 0; j < k; ++j) {
        send_e[r * k + j] = -1;
        send_w[r * k + j] = 0.f;
      }
    }
  }
}

// send_x[r, :] = x[send_token[r], :] for every r < n_ranks*T with a token.
template <typename T_>
__global__ void __launch_bounds__(256) ep_pack_kernel(const T_* __restrict__ x, int dim,
                                                      const int* __restrict__ send_token,
                                                      int64_t rows, T_* __restrict__ out) {
  using V = Vec16<T_>;
  const int nvec = dim / V::N;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t r = warp; r < rows; r += nwarps) {
    const int t = send_token[r];
    if (t < 0) continue;
    const T_* src = x + (int64_t)t * dim;
    T_* dst = out + r * dim;
    for (int v = lane; v < nvec; v += 32) st_plain(dst + v * V::N, ld_keep(src + v * V::N));
  }
}

// out[t, :] = sum over ranks d (in order) of back[d*T + src_pos[t, d], :], fp32 accumulation.
template <typename T_>
__global__ void __launch_bounds__(256) ep_unpack_sum_kernel(const T_* __restrict__ back, int dim,
                                                            const int* __restrict__ src_pos,
                                                            int64_t T, int n_ranks,
                                                            T_* __restrict__ out) {
  using V = Vec16<T_>;
  const int nvec = dim / V::N;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t t = warp; t < T; t += nwarps) {
    if (n_ranks <= 32) {
      // Lane d holds rank d's row position; the ranks holding a partial row are summed in
      // rank order (as below), 4 packets per lane at a time to keep loads in flight.
      constexpr int B = 4;
      const int my_p = lane < n_ranks ? src_pos[t * n_ranks + lane] : -1;
      const unsigned live = __ballot_sync(0xffffffffu, my_p >= 0);
      for (int v0 = 0; v0 < nvec; v0 += 32 * B) {
        float acc[B][V::N];
#pragma unroll
        for (int b = 0; b < B; ++b)
#pragma unroll
          for (int i = 0; i < V::N; ++i) acc[b][i] = 0.f;
        for (unsigned m = live; m != 0u; m &= m - 1u) {
          const int d = __ffs(m) - 1;
          const int p = __shfl_sync(0xffffffffu, my_p, d);
          V r[B];
#pragma unroll
          for (int b = 0; b < B; ++b) {
            const int v = v0 + b * 32 + lane;
            if (v < nvec) r[b] = ld_keep(back + ((int64_t)d * T + p) * dim + v * V::N);
          }
#pragma unroll
          for (int b = 0; b < B; ++b)
#pragma unroll
            for (int i = 0; i < V::N; ++i) acc[b][i] += Elt<T_>::to_f(r[b].e[i]);
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const int v = v0 + b * 32 + lane;
          if (v >= nvec) continue;
          V o;
#pragma unroll
          for (int i = 0; i < V::N; ++i) o.e[i] = Elt<T_>::from_f(acc[b][i]);
          st_plain(out + t * dim + v * V::N, o);
        }
      }
      continue;
    }
    for (int v = lane; v < nvec; v += 32) {
      float acc[V::N];
#pragma unroll
      for (int i = 0; i < V::N; ++i) acc[i] = 0.f;
      for (int d = 0; d < n_ranks; ++d) {
        const int p = src_pos[t * n_ranks + d];
        if (p < 0) continue;
        V r = ld_keep(back + ((int64_t)d * T + p) * dim + v * V::N);
#pragma unroll
        for (int i = 0; i < V::N; ++i) acc[i] += Elt<T_>::to_f(r.e[i]);
      }
      V o;
#pragma unroll
      for (int i = 0; i < V::N; ++i) o.e[i] = Elt<T_>::from_f(acc[i]);
      st_plain(out + t * dim + v * V::N, o);
    }
  }
}

// dw[t, j] = back_dw[(d*T + src_pos[t, d]) * k + j] with d = rank of expert idx[t, j].
__global__ void ep_unpack_dw_kernel(const float* __restrict__ back_dw,
                                    const int64_t* __restrict__ idx,
                                    const int* __restrict__ expert_rank,
                                    const int* __restrict__ src_pos, int64_t T, int k,
                                    int n_ranks, int E, float* __restrict__ dw) {
  for (int64_t a = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; a < T * k;
       a += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = a / k;
    const int j = (int)(a % k);
    const int64_t e = idx[a];
    float v = 0.f;
    if (e >= 0 && e < E) {
      const int d = expert_rank[e];
      const int p = src_pos[t * n_ranks + d];
      if (p >= 0) v = back_dw[((int64_t)d * T + p) * k + j];
    }
    dw[a] = v;
  }
}

inline int rows_grid(int64_t rows) {
  int64_t g = (rows + 7) / 8;
  int64_t cap = (int64_t)num_sms() * 8;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace fk

extern "C" int fk_ep_plan_workspace_size(int64_t n_tokens, int n_ranks, size_t* bytes) {
  FK_CHECK_ARG(n_tokens >= 0 && n_ranks >= 1 && n_ranks <= 32 && bytes,
               "fk_ep_plan_workspace_size: bad arguments");
  const int64_t chunks = (n_tokens + fk::kPlanThreads - 1) / fk::kPlanThreads;
  *bytes = (size_t)(chunks < 1 ? 1 : chunks) * n_ranks * sizeof(int);
  return FK_OK;
}

extern "C" int fk_ep_plan(const int64_t* idx, const float* w, int64_t n_tokens, int k,
                          const int* expert_rank, const int* expert_local, int n_experts,
                          int n_ranks, int* send_token, int* send_e, float* send_w,
                          int* src_pos, int* send_count, void* workspace, size_t ws_bytes,
                          int* err_flag, void* stream) {
  FK_CHECK_ARG(n_tokens >= 0 && k >= 1 && n_ranks >= 1 && n_ranks <= 32 && n_experts >= 1,
               "fk_ep_plan: bad sizes (1 <= n_ranks <= 32)");
  FK_CHECK_ARG(expert_rank && expert_local && send_token && send_e && send_w && src_pos &&
                   send_count && err_flag && workspace && (n_tokens == 0 || (idx && w)),
               "fk_ep_plan: null pointer");
  size_t need = 0;
  fk_ep_plan_workspace_size(n_tokens, n_ranks, &need);
  if (ws_bytes < need)
    return fk::fail(FK_ERR_WORKSPACE, "fk_ep_plan: workspace %zu < %zu bytes", ws_bytes, need);
  cudaStream_t st = fk::as_stream(stream);
  cudaMemsetAsync(err_flag, 0, sizeof(int), st);
  const int chunks = (int)((n_tokens + fk::kPlanThreads - 1) / fk::kPlanThreads);
  int* cc = static_cast<int*>(workspace);
  if (chunks == 0) {
    cudaMemsetAsync(send_count, 0, n_ranks * sizeof(int), st);
    return fk::launch_status("fk_ep_plan");
  }
  fk::ep_plan_count_kernel<<<chunks, fk::kPlanThreads, 0, st>>>(idx, n_tokens, k, expert_rank,
                                                               n_experts, n_ranks, cc, err_flag);
  fk::ep_plan_fill_kernel<<<chunks, fk::kPlanThreads, 0, st>>>(
      idx, w, n_tokens, k, expert_rank, expert_local, n_experts, n_ranks, cc, chunks, send_token,
      send_e, send_w, src_pos, send_count);
  return fk::launch_status("fk_ep_plan");
}

extern "C" int fk_ep_pack(const void* x, int dim, const int* send_token, int64_t rows,
                          void* send_x, int dtype, void* stream) {
  FK_CHECK_ARG(rows >= 0 && dim > 0, "fk_ep_pack: bad sizes");
  if (rows == 0) return FK_OK;
  FK_CHECK_ARG(x && send_token && send_x, "fk_ep_pack: null pointer");
  FK_CHECK_ARG(fk::valid_dtype(dtype) && (dim * fk::dtype_size(dtype)) % 16 == 0 &&
                   fk::aligned16(x) && fk::aligned16(send_x),
               "fk_ep_pack: rows must be 16-byte aligned");
  cudaStream_t st = fk::as_stream(stream);
  FK_DISPATCH_DTYPE(dtype, fk::ep_pack_kernel<scalar_t><<<fk::rows_grid(rows), 256, 0, st>>>(
                               static_cast<const scalar_t*>(x), dim, send_token, rows,
                               static_cast<scalar_t*>(send_x)));
  return fk::launch_status("fk_ep_pack");
}

extern "C" int fk_ep_unpack_sum(const void* back, int dim, const int* src_pos, int64_t n_tokens,
                                int n_ranks, void* out, int dtype, void* stream) {
  FK_CHECK_ARG(n_tokens >= 0 && dim > 0 && n_ranks >= 1, "fk_ep_unpack_sum: bad sizes");
  if (n_tokens == 0) return FK_OK;
  FK_CHECK_ARG(back && src_pos && out, "fk_ep_unpack_sum: null pointer");
  FK_CHECK_ARG(fk::valid_dtype(dtype) && (dim * fk::dtype_size(dtype)) % 16 == 0 &&
                   fk::aligned16(back) && fk::aligned16(out),
               "fk_ep_unpack_sum: rows must be 16-byte aligned");
  cudaStream_t st = fk::as_stream(stream);
  FK_DISPATCH_DTYPE(dtype, fk::ep_unpack_sum_kernel<scalar_t>
                    <<<fk::rows_grid(n_tokens), 256, 0, st>>>(
                        static_cast<const scalar_t*>(back), dim, src_pos, n_tokens, n_ranks,
                        static_cast<scalar_t*>(out)));
  return fk::launch_status("fk_ep_unpack_sum");
}

extern "C" int fk_ep_unpack_dw(const float* back_dw, const int64_t* idx, const int* expert_rank,
                               const int* src_pos, int64_t n_tokens, int k, int n_ranks,
                               int n_experts, float* dw, void* stream) {
  FK_CHECK_ARG(n_tokens >= 0 && k >= 1 && n_ranks >= 1, "fk_ep_unpack_dw: bad sizes");
  if (n_tokens == 0) return FK_OK;
  FK_CHECK_ARG(back_dw && idx && expert_rank && src_pos && dw, "fk_ep_unpack_dw: null pointer");
  int64_t n = n_tokens * k;
  int grid = (int)((n + 255) / 256);
  if (grid > fk::num_sms() * 8) grid = fk::num_sms() * 8;
  fk::ep_unpack_dw_kernel<<<grid, 256, 0, fk::as_stream(stream)>>>(
      back_dw, idx, expert_rank, src_pos, n_tokens, k, n_ranks, n_experts, dw);
  return fk::launch_status("fk_ep_unpack_dw");
}
