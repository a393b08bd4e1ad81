// MoE top-k router: softmax + top-k on the logit + renormalisation (forward) and the
// subset-softmax Jacobian (backward), reference moe_routing_v2.py:44-126.
//
// Ranking.  Each expert e gets a 64-bit key  (ordered(logit) << 32) | (E-1-e)  where
// ordered() maps the fp32 bit pattern to an unsigned integer with the same order
// (-0.0 is folded onto +0.0, every NaN becomes the canonical +NaN, which ranks above
// +inf, as torch.sort/topk rank NaN).  Sorting keys in descending order ranks by the
// exact logit and breaks ties toward the LOWER expert index.  Padding slots get key 0,
// which is below every real key (-inf maps to 0x007FFFFF in the high word).
//
// Layout.  A row of E experts is padded to L = S*V (power of two) and held by a
// segment of S lanes (S = min(32, L)), V keys per lane; element i = r*S + lane.
// E <= 32 packs 32/S rows into each warp.
//
// Selection ("group then merge", k <= S): runs of KP = next_pow2(k) keys are
// bitonic-sorted with warp shuffles, then folded pairwise -- the elementwise max of a
// descending and an ascending run holds the top KP of their union as a bitonic run,
// which a log2(KP)-step bitonic merge sorts again -- first across the V registers of a
// lane (no shuffles), then across lanes.  Work is O(L log^2 KP) instead of the
// O(L log^2 L) of a full sort.  For k > S a full bitonic sort of all L keys is used.
// Two rows are processed per warp pass when V <= 2 (independent shuffle chains), and the
// next pass's logits are loaded before the current pass's network runs.
//
// Weights.  The renormalised top-k softmax equals a softmax over the k selected logits:
// w_j = exp(x_j - m) / sum_{i in top-k} exp(x_i - m), with m the largest logit (the
// full-E denominator cancels), so only k exponentials are needed per row.
#include "common.cuh"

namespace fk {
namespace {

__device__ __forceinline__ uint32_t ordered_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if (x != x) u = 0x7FC00000u;   // canonical NaN: ranks above +inf
  if (u == 0x80000000u) u = 0u;  // -0.0 ranks equal to +0.0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float from_ordered(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t shfl_xor64(uint64_t v, int d) {
  uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
  lo = __shfl_xor_sync(0xffffffffu, lo, d);
  hi = __shfl_xor_sync(0xffffffffu, hi, d);
  return ((uint64_t)hi << 32) | lo;
}

__device__ __forceinline__ uint64_t kmax(uint64_t a, uint64_t b) { return a > b ? a : b; }
__device__ __forceinline__ uint64_t kmin(uint64_t a, uint64_t b) { return a < b ? a : b; }

// One bitonic compare-exchange step across lanes at distance d (d < S).
__device__ __forceinline__ uint64_t cx_lanes(uint64_t a, int d, int lane_s, bool desc) {
  uint64_t b = shfl_xor64(a, d);
  bool first = (lane_s & d) == 0;
  return (first == desc) ? kmax(a, b) : kmin(a, b);
}

template <int S>
__device__ __forceinline__ float seg_sum(float v) {
#pragma unroll
  for (int o = S / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Bitonic merge of runs of KP lanes (distances KP/2 .. 1) toward direction `desc`.
template <int KP>
__device__ __forceinline__ uint64_t merge_runs(uint64_t m, int lane_s, bool desc) {
#pragma unroll
  for (int d = KP >> 1; d > 0; d >>= 1) m = cx_lanes(m, d, lane_s, desc);
  return m;
}

// Top-k keys of one row held as key[V] (element i = r*S + lane_s), group-then-merge:
//  A) bitonic-sort runs of KP = next_pow2(k) lanes inside every register;
//  B) fold registers pairwise (elementwise max of a descending and an ascending run is
//     the top KP of both, as a bitonic run) and re-merge, log2(V) levels, no shuffles
//     for the max;
//  C) fold runs across lanes the same way at distances KP, 2KP, .., S/2.
// Run directions are chosen so every fold sees (descending, ascending) partners; the
// result is the top KP, sorted descending, in register 0 of lanes 0..KP-1 of the segment.
template <int S, int V, int KP>
__device__ __forceinline__ uint64_t topk_group_merge(uint64_t (&key)[V], int lane_s) {
  // final direction of the runs of register r after phase A / each phase-B level
  auto lane_alt = [&](int period) { return ((lane_s / period) & 1) == 0; };
  const bool lanes_follow = KP < S;  // phase C exists
  // Phase A
#pragma unroll
  for (int size = 2; size <= KP; size <<= 1) {
#pragma unroll
    for (int d = size >> 1; d > 0; d >>= 1) {
#pragma unroll
      for (int r = 0; r < V; ++r) {
        bool want_desc = (V > 1) ? ((r & 1) == 0) : (lanes_follow ? lane_alt(KP) : true);
        bool natural_desc = ((lane_s & KP) == 0) || KP == S;
        bool desc = (((lane_s & size) == 0) || size == S) != (natural_desc != want_desc);
        if (size == KP) desc = want_desc;
        key[r] = cx_lanes(key[r], d, lane_s, desc);
      }
    }
  }
  // Phase B
#pragma unroll
  for (int h = 1; h < V; h <<= 1) {
#pragma unroll
    for (int r = 0; r < V; r += 2 * h) {
      uint64_t m = kmax(key[r], key[r + h]);
      bool desc;
      if (2 * h < V) desc = ((r / (2 * h)) & 1) == 0;
      else desc = lanes_follow ? lane_alt(KP) : true;
      key[r] = merge_runs<KP>(m, lane_s, desc);
    }
  }
  // Phase C
  uint64_t m = key[0];
#pragma unroll
  for (int d = KP; d < S; d <<= 1) {
    m = kmax(m, shfl_xor64(m, d));
    m = merge_runs<KP>(m, lane_s, lane_alt(2 * d));
  }
  return m;
}

template <typename T, int S, int V, int KP, bool FULL, int RPI>
__global__ void __launch_bounds__(256) router_fwd_kernel(const T* __restrict__ logits,
                                                         int64_t row_stride, int64_t n_rows,
                                                         int E, int k, float* __restrict__ w_out,
                                                         int64_t* __restrict__ idx_out) {
  constexpr int L = S * V;
  constexpr int RPW = 32 / S;  // rows per warp per pass
  const int lane = threadIdx.x & 31;
  const int lane_s = lane % S;
  const int seg = lane / S;
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t n_groups = (n_rows + RPW * RPI - 1) / (RPW * RPI);

  // Logits of group g into x (registers); zeros past the end.
#define FK_ROUTER_LOAD(x, g)                                                            \
  _Pragma("unroll") for (int q = 0; q < RPI; ++q) {                                     \
    const int64_t row_ = ((g) * RPI + q) * RPW + seg;                                   \
    _Pragma("unroll") for (int r = 0; r < V; ++r) {                                     \
      const int e_ = r * S + lane_s;                                                    \
      x[q][r] = ((g) < n_groups && row_ < n_rows && e_ < E)                             \
                    ? Elt<T>::to_f(logits[row_ * row_stride + e_]) : 0.f;               \
    }                                                                                   \
  }
  float cur[RPI][V];
  FK_ROUTER_LOAD(cur, warp_global)
  for (int64_t g = warp_global; g < n_groups; g += n_warps) {
    float nxt[RPI][V];
    FK_ROUTER_LOAD(nxt, g + n_warps)  // next group's logits in flight during this group's sort
    uint64_t top[RPI], keyv[RPI][V];
#pragma unroll
    for (int q = 0; q < RPI; ++q) {
      const int64_t row = (g * RPI + q) * RPW + seg;
#pragma unroll
      for (int r = 0; r < V; ++r) {
        const int e = r * S + lane_s;
        keyv[q][r] = (row < n_rows && e < E)
                         ? (((uint64_t)ordered_bits(cur[q][r]) << 32) | (uint32_t)(E - 1 - e))
                         : 0ull;
      }
    }
    if constexpr (!FULL) {
#pragma unroll
      for (int q = 0; q < RPI; ++q) top[q] = topk_group_merge<S, V, KP>(keyv[q], lane_s);
    } else {
      // Full bitonic sort of L keys, descending (k > 32).
#pragma unroll
      for (int q = 0; q < RPI; ++q) {
#pragma unroll
        for (int size = 2; size <= L; size <<= 1) {
#pragma unroll
          for (int d = size >> 1; d > 0; d >>= 1) {
            if (d >= S) {
              const int rd = d / S;
#pragma unroll
              for (int r = 0; r < V; ++r) {
                if ((r & rd) == 0) {
                  const int i = r * S + lane_s;
                  const bool desc = (i & size) == 0;
                  uint64_t a = keyv[q][r], b = keyv[q][r + rd];
                  keyv[q][r] = desc ? kmax(a, b) : kmin(a, b);
                  keyv[q][r + rd] = desc ? kmin(a, b) : kmax(a, b);
                }
              }
            } else {
#pragma unroll
              for (int r = 0; r < V; ++r) {
                const int i = r * S + lane_s;
                keyv[q][r] = cx_lanes(keyv[q][r], d, lane_s, (i & size) == 0);
              }
            }
          }
        }
        top[q] = keyv[q][0];
      }
    }
#pragma unroll
    for (int q = 0; q < RPI; ++q) {
      const int64_t row = (g * RPI + q) * RPW + seg;
      // Largest logit: rank 0, register 0 of segment lane 0.
      const uint64_t t0 = __shfl_sync(0xffffffffu, top[q], seg * S);
      const float m = from_ordered((uint32_t)(t0 >> 32));
      constexpr int VK = FULL ? V : 1;  // registers that can hold rank < k
      float ex[VK];
      uint64_t kk[VK];
      float ssum = 0.f;
#pragma unroll
      for (int r = 0; r < VK; ++r) {
        const int j = r * S + lane_s;
        kk[r] = FULL ? keyv[q][r] : top[q];
        ex[r] = 0.f;
        if (j < k) {
          ex[r] = expf(from_ordered((uint32_t)(kk[r] >> 32)) - m);
          ssum += ex[r];
        }
      }
      ssum = seg_sum<S>(ssum);
      if (row < n_rows) {
        const float inv = 1.0f / ssum;
#pragma unroll
        for (int r = 0; r < VK; ++r) {
          const int j = r * S + lane_s;
          if (j < k) {
            w_out[row * k + j] = ex[r] * inv;
            idx_out[row * k + j] = (int64_t)(E - 1 - (int)(uint32_t)kk[r]);
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < RPI; ++q)
#pragma unroll
      for (int r = 0; r < V; ++r) cur[q][r] = nxt[q][r];
  }
#undef FK_ROUTER_LOAD
}

// Backward: dense fp32 rows; selected entries get w_j * (dw_j - <w, dw>), others 0.
template <int S, int V>
__global__ void __launch_bounds__(256) router_bwd_kernel(const float* __restrict__ dw,
                                                         const float* __restrict__ w,
                                                         const int64_t* __restrict__ idx,
                                                         float* __restrict__ dlogits,
                                                         int64_t n_rows, int E, int k) {
  constexpr int L = S * V;
  constexpr int RPW = 32 / S;
  __shared__ float buf[8][32 * V];  // per warp: RPW segments of L floats
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int lane_s = lane % S;
  const int seg = lane / S;
  float* sb = &buf[warp][seg * L];
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t n_groups = (n_rows + RPW - 1) / RPW;

  for (int64_t g = warp_global; g < n_groups; g += n_warps) {
    const int64_t row = g * RPW + seg;
    const bool row_ok = row < n_rows;
    float dot = 0.f;
    if (row_ok)
      for (int j = lane_s; j < k; j += S) dot = fmaf(w[row * k + j], dw[row * k + j], dot);
    dot = seg_sum<S>(dot);
#pragma unroll
    for (int r = 0; r < V; ++r) sb[r * S + lane_s] = 0.f;
    __syncwarp();
    if (row_ok)
      for (int j = lane_s; j < k; j += S) {
        int64_t e = idx[row * k + j];
        float wj = w[row * k + j];
        if (e >= 0 && e < E) sb[e] = wj * (dw[row * k + j] - dot);
      }
    __syncwarp();
    if (row_ok) {
#pragma unroll
      for (int r = 0; r < V; ++r) {
        int e = r * S + lane_s;
        if (e < E) dlogits[row * E + e] = sb[e];
      }
    }
    __syncwarp();
  }
}

inline int pow2_at_least(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

inline int warp_grid(int64_t n_groups) {
  int64_t ctas = (n_groups + 7) / 8;  // 8 warps per CTA
  int64_t cap = (int64_t)num_sms() * 8;
  if (ctas > cap) ctas = cap;
  return (int)(ctas < 1 ? 1 : ctas);
}

template <typename T, int S, int V>
int launch_gm(const T* lp, int64_t rs, int64_t n, int E, int k, float* w, int64_t* idx,
              cudaStream_t st) {
  constexpr int RPI = (V <= 2) ? 2 : 1;
  const int64_t groups = (n + (32 / S) * RPI - 1) / ((32 / S) * RPI);
  const int grid = warp_grid(groups);
  const int KP = pow2_at_least(k);
#define FK_KP(KP_)                                                                          \
  case KP_:                                                                                 \
    router_fwd_kernel<T, S, V, (KP_ < S ? KP_ : S), false, RPI><<<grid, 256, 0, st>>>(       \
        lp, rs, n, E, k, w, idx);                                                           \
    break;
  switch (KP) {
    FK_KP(1) FK_KP(2) FK_KP(4) FK_KP(8) FK_KP(16) FK_KP(32)
    default: return fail(FK_ERR_UNSUPPORTED, "fk_router_fwd: k=%d", k);
  }
#undef FK_KP
  return FK_OK;
}

template <typename T, int V>
int launch_full(const T* lp, int64_t rs, int64_t n, int E, int k, float* w, int64_t* idx,
                cudaStream_t st) {
  const int grid = warp_grid(n);
  router_fwd_kernel<T, 32, V, 32, true, 1><<<grid, 256, 0, st>>>(lp, rs, n, E, k, w, idx);
  return FK_OK;
}

template <typename T>
int fwd_t(const void* logits, int64_t rs, int64_t n, int E, int k, float* w, int64_t* idx,
          cudaStream_t st) {
  const T* lp = static_cast<const T*>(logits);
  const int L = pow2_at_least(E);
  const int S = L < 32 ? L : 32;
  const int V = L / S;
  int r = FK_OK;
  if (k > S) {
    switch (V) {
      case 2: r = launch_full<T, 2>(lp, rs, n, E, k, w, idx, st); break;
      case 4: r = launch_full<T, 4>(lp, rs, n, E, k, w, idx, st); break;
      case 8: r = launch_full<T, 8>(lp, rs, n, E, k, w, idx, st); break;
    }
  } else if (S < 32) {
    switch (S) {
      case 1: r = launch_gm<T, 1, 1>(lp, rs, n, E, k, w, idx, st); break;
      case 2: r = launch_gm<T, 2, 1>(lp, rs, n, E, k, w, idx, st); break;
      case 4: r = launch_gm<T, 4, 1>(lp, rs, n, E, k, w, idx, st); break;
      case 8: r = launch_gm<T, 8, 1>(lp, rs, n, E, k, w, idx, st); break;
      case 16: r = launch_gm<T, 16, 1>(lp, rs, n, E, k, w, idx, st); break;
    }
  } else {
    switch (V) {
      case 1: r = launch_gm<T, 32, 1>(lp, rs, n, E, k, w, idx, st); break;
      case 2: r = launch_gm<T, 32, 2>(lp, rs, n, E, k, w, idx, st); break;
      case 4: r = launch_gm<T, 32, 4>(lp, rs, n, E, k, w, idx, st); break;
      case 8: r = launch_gm<T, 32, 8>(lp, rs, n, E, k, w, idx, st); break;
    }
  }
  if (r != FK_OK) return r;
  return launch_status("fk_router_fwd");
}

}  // namespace
}  // namespace fk

extern "C" int fk_router_fwd(const void* logits, int64_t row_stride, int dtype, int64_t n_rows,
                             int n_experts, int k, float* w, int64_t* idx, void* stream) {
  FK_CHECK_ARG(n_rows >= 0, "fk_router_fwd: n_rows < 0");
  FK_CHECK_ARG(n_experts >= 1 && k >= 1 && k <= n_experts,
               "fk_router_fwd: need 1 <= k <= n_experts (k=%d, E=%d)", k, n_experts);
  if (n_experts > 256)
    return fk::fail(FK_ERR_UNSUPPORTED, "fk_router_fwd: n_experts=%d > 256", n_experts);
  if (n_rows == 0) return FK_OK;
  FK_CHECK_ARG(logits && w && idx, "fk_router_fwd: null pointer");
  FK_CHECK_ARG(row_stride >= n_experts, "fk_router_fwd: row_stride < n_experts");
  FK_DISPATCH_DTYPE(dtype, return fk::fwd_t<scalar_t>(logits, row_stride, n_rows, n_experts, k,
                                                      w, idx, fk::as_stream(stream)));
  return FK_OK;
}

extern "C" int fk_router_bwd(const float* dw, const float* w, const int64_t* idx,
                             float* dlogits, int64_t n_rows, int n_experts, int k, void* stream) {
  FK_CHECK_ARG(n_rows >= 0, "fk_router_bwd: n_rows < 0");
  FK_CHECK_ARG(n_experts >= 1 && k >= 1 && k <= n_experts,
               "fk_router_bwd: need 1 <= k <= n_experts (k=%d, E=%d)", k, n_experts);
  if (n_experts > 256)
    return fk::fail(FK_ERR_UNSUPPORTED, "fk_router_bwd: n_experts=%d > 256", n_experts);
  if (n_rows == 0) return FK_OK;
  FK_CHECK_ARG(dw && w && idx && dlogits, "fk_router_bwd: null pointer");
  const int L = fk::pow2_at_least(n_experts);
  const int S = L < 32 ? L : 32;
  const int V = L / S;
  const int64_t groups = (n_rows + (32 / S) - 1) / (32 / S);
  const int grid = fk::warp_grid(groups);
  cudaStream_t st = fk::as_stream(stream);
#define FK_LAUNCH(S_, V_) \
  fk::router_bwd_kernel<S_, V_><<<grid, 256, 0, st>>>(dw, w, idx, dlogits, n_rows, n_experts, k)
  if (S < 32) {
    switch (S) {
      case 1: FK_LAUNCH(1, 1); break;
      case 2: FK_LAUNCH(2, 1); break;
      case 4: FK_LAUNCH(4, 1); break;
      case 8: FK_LAUNCH(8, 1); break;
      case 16: FK_LAUNCH(16, 1); break;
    }
  } else {
    switch (V) {
      case 1: FK_LAUNCH(32, 1); break;
      case 2: FK_LAUNCH(32, 2); break;
      case 4: FK_LAUNCH(32, 4); break;
      case 8: FK_LAUNCH(32, 8); break;
    }
  }
#undef FK_LAUNCH
  return fk::launch_status("fk_router_bwd");
}
