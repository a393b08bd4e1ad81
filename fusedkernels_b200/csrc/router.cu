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
// Two kernel families.  For k <= 8 (every routing configuration of the reference's
// tests and benchmarks) the forward holds a row in a small group of lanes that each
// select over up to 32 logits by sorted insertion and merge their lists by a butterfly
// (the lane-group kernels further down), and for k <= 4 the backward uses lane groups of
// 8 entries per lane.  Otherwise the segment kernels below run a bitonic network.
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
#include <climits>

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

// ---------------------------------------------------------------------------------------
// Lane-group kernels, k <= 8.  A row is held by a group of G lanes (G = next_pow2(E/C),
// 1..32), C logits per lane (C = 32; 8 / 16 for E <= 8 / 16 and 8 for few rows): lane l owns
// the 16-byte packets p*G + l of the row, so one warp load covers 32/G whole rows.
// Each lane keeps the top KP = next_pow2(k) (key, expert) pairs of its C logits in
// registers by sorted insertion -- its logits arrive in increasing expert order, so a
// strict '>' keeps the lower index first on ties -- and the G lists are merged by a
// butterfly over the group: at distance d the partner's list is reversed, the pairwise
// better of the two lists is a bitonic sequence holding the top KP of both, and a
// log2(KP)-step bitonic merge sorts it again.  The comparator (key desc, expert asc) is a
// total order, so every lane of the group ends with the same list.  Per row this costs
// about E*(KP+3) ALU operations and 2*KP*log2(G) shuffles per lane, against the
// shuffle-bound O(E log^2 KP) network of the segment kernel above.
//
// Keys are signed integers: bits ^ ((bits >> 31) & 0x7fffffff) orders like the float and
// is its own inverse; -0.0 is folded onto +0.0 (x + 0.0f) and every NaN becomes INT_MAX,
// above +inf (0x7f800000).  Padding is INT_MIN, below -inf (0x807fffff).
constexpr int kLaneElems = 8;   // dense gradient entries per lane (backward)
// Logits per lane in the forward: 32 (fewer lanes per row, so fewer merge levels: the
// forward is issue-bound), or the padded row when E <= 16.  Measured on B200 at 131072 rows
// against 8 per lane: E=64,k=2 1.33x, E=128,k=8 1.97x, E=256,k=4 1.88x faster.  With too
// few rows to give every SM a CTA of 256 threads at 32 per lane, 8 per lane keeps more
// lanes busy (4096 x 64 rows: 1.9 us against 2.8 us).
inline int fwd_elems(int E, int64_t rows) {
  if (E <= 8) return 8;
  if (E <= 16) return 16;
  const int64_t lanes32 = rows * (int64_t)((E + 31) / 32);
  return lanes32 < (int64_t)num_sms() * 256 ? 8 : 32;
}
constexpr int kLaneMaxKP = 8;   // largest list kept per lane

__device__ __forceinline__ int skey(float x) {
  x = x + 0.0f;
  int s = __float_as_int(x);
  s ^= (s >> 31) & 0x7fffffff;
  return (x != x) ? 0x7fffffff : s;
}

__device__ __forceinline__ float skey_value(int s) {
  return __int_as_float(s ^ ((s >> 31) & 0x7fffffff));
}

__device__ __forceinline__ bool better(int va, int ia, int vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// Insert (v, e) into the descending list kv/ki; e is larger than every index already in it.
template <int KP>
__device__ __forceinline__ void insert_sorted(int (&kv)[KP], int (&ki)[KP], int v, int e) {
  bool c[KP];
#pragma unroll
  for (int i = 0; i < KP; ++i) c[i] = v > kv[i];
#pragma unroll
  for (int i = KP - 1; i > 0; --i) {
    kv[i] = c[i - 1] ? kv[i - 1] : (c[i] ? v : kv[i]);
    ki[i] = c[i - 1] ? ki[i - 1] : (c[i] ? e : ki[i]);
  }
  kv[0] = c[0] ? v : kv[0];
  ki[0] = c[0] ? e : ki[0];
}

// Replace the list by the top KP of it and the list of the lane at xor distance d.
template <int KP>
__device__ __forceinline__ void merge_xor(int (&kv)[KP], int (&ki)[KP], int d) {
  int bv[KP], bi[KP];
#pragma unroll
  for (int i = 0; i < KP; ++i) {
    bv[i] = __shfl_xor_sync(0xffffffffu, kv[i], d);
    bi[i] = __shfl_xor_sync(0xffffffffu, ki[i], d);
  }
#pragma unroll
  for (int i = 0; i < KP; ++i) {
    const int j = KP - 1 - i;
    const bool t = better(kv[i], ki[i], bv[j], bi[j]);
    kv[i] = t ? kv[i] : bv[j];
    ki[i] = t ? ki[i] : bi[j];
  }
#pragma unroll
  for (int s = KP >> 1; s > 0; s >>= 1) {
#pragma unroll
    for (int i = 0; i < KP; ++i) {
      if ((i & s) == 0) {
        const bool t = better(kv[i], ki[i], kv[i + s], ki[i + s]);
        const int av = kv[i], ai = ki[i];
        kv[i] = t ? av : kv[i + s];
        ki[i] = t ? ai : ki[i + s];
        kv[i + s] = t ? kv[i + s] : av;
        ki[i + s] = t ? ki[i + s] : ai;
      }
    }
  }
}

template <typename T, int G, int C, bool VEC>
__device__ __forceinline__ void lanes_load(const T* __restrict__ logits, int64_t row_stride,
                                           int64_t row, bool ok, int E, int l, float (&x)[C]) {
  constexpr int VN = 16 / (int)sizeof(T);
  constexpr int P = C / VN;
  const T* rp = logits + row * row_stride;
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const int e0 = (p * G + l) * VN;
    if constexpr (VEC) {
      if (ok && e0 < E) {
        const Vec16<T> v = ld_keep(rp + e0);
#pragma unroll
        for (int q = 0; q < VN; ++q) x[p * VN + q] = Elt<T>::to_f(v.e[q]);
      } else {
#pragma unroll
        for (int q = 0; q < VN; ++q) x[p * VN + q] = 0.f;
      }
    } else {
#pragma unroll
      for (int q = 0; q < VN; ++q)
        x[p * VN + q] = (ok && e0 + q < E) ? Elt<T>::to_f(rp[e0 + q]) : 0.f;
    }
  }
}

template <typename T, int G, int C, int KP, bool VEC>
__global__ void __launch_bounds__(256) router_fwd_lanes(const T* __restrict__ logits,
                                                        int64_t row_stride, int64_t n_rows,
                                                        int E, int k, float* __restrict__ w_out,
                                                        int64_t* __restrict__ idx_out) {
  constexpr int VN = 16 / (int)sizeof(T);
  constexpr int P = C / VN;
  constexpr int RPW = 32 / G;  // rows per warp per pass
  const int lane = threadIdx.x & 31;
  const int l = lane % G;
  const int grp = lane / G;
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t n_tiles = (n_rows + RPW - 1) / RPW;

  float cur[C];
  {
    const int64_t row = warp_global * RPW + grp;
    lanes_load<T, G, C, VEC>(logits, row_stride, row, warp_global < n_tiles && row < n_rows, E,
                             l, cur);
  }
  // The tile loop is warp-uniform: every lane reaches every shuffle.
  for (int64_t tile = warp_global; tile < n_tiles; tile += n_warps) {
    const int64_t row = tile * RPW + grp;
    const bool row_ok = row < n_rows;
    float nxt[C];
    {
      const int64_t nt = tile + n_warps;
      const int64_t nrow = nt * RPW + grp;
      lanes_load<T, G, C, VEC>(logits, row_stride, nrow, nt < n_tiles && nrow < n_rows, E, l,
                               nxt);
    }
    int kv[KP], ki[KP];
#pragma unroll
    for (int i = 0; i < KP; ++i) {
      kv[i] = INT_MIN;
      ki[i] = INT_MAX;
    }
#pragma unroll
    for (int p = 0; p < P; ++p) {
#pragma unroll
      for (int q = 0; q < VN; ++q) {
        const int e = (p * G + l) * VN + q;
        const int v = (row_ok && e < E) ? skey(cur[p * VN + q]) : INT_MIN;
        insert_sorted<KP>(kv, ki, v, e);
      }
    }
#pragma unroll
    for (int d = 1; d < G; d <<= 1) merge_xor<KP>(kv, ki, d);

    const float m = skey_value(kv[0]);
    float ex[KP];
    float ssum = 0.f;
#pragma unroll
    for (int i = 0; i < KP; ++i) {
      ex[i] = 0.f;
      if (i < k) {
        ex[i] = expf(skey_value(kv[i]) - m);
        ssum += ex[i];
      }
    }
    if (row_ok) {
      const float inv = 1.0f / ssum;
      for (int j = l; j < k; j += G) {
        float exj = ex[0];
        int ij = ki[0];
#pragma unroll
        for (int i = 1; i < KP; ++i)
          if (i == j) {
            exj = ex[i];
            ij = ki[i];
          }
        w_out[row * k + j] = exj * inv;
        idx_out[row * k + j] = (int64_t)ij;
      }
    }
#pragma unroll
    for (int i = 0; i < C; ++i) cur[i] = nxt[i];
  }
}

// Backward with the same row/lane mapping: lane l writes the fp32 packets p*G + l of the
// dense gradient row; an expert listed twice takes the later slot's value.
template <int G, int KP, bool VEC>
__global__ void __launch_bounds__(256) router_bwd_lanes(const float* __restrict__ dw,
                                                        const float* __restrict__ w,
                                                        const int64_t* __restrict__ idx,
                                                        float* __restrict__ dlogits,
                                                        int64_t n_rows, int E, int k) {
  constexpr int P = kLaneElems / 4;
  constexpr int RPW = 32 / G;
  const int lane = threadIdx.x & 31;
  const int l = lane % G;
  const int grp = lane / G;
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t n_tiles = (n_rows + RPW - 1) / RPW;
  for (int64_t tile = warp_global; tile < n_tiles; tile += n_warps) {
    const int64_t row = tile * RPW + grp;
    if (row >= n_rows) continue;
    float wv[KP], dv[KP], g[KP];
    int id[KP];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < KP; ++i) {
      wv[i] = 0.f;
      dv[i] = 0.f;
      id[i] = -1;
      if (i < k) {
        wv[i] = w[row * k + i];
        dv[i] = dw[row * k + i];
        const int64_t e = idx[row * k + i];
        id[i] = (e >= 0 && e < E) ? (int)e : -1;
        dot = fmaf(wv[i], dv[i], dot);
      }
    }
#pragma unroll
    for (int i = 0; i < KP; ++i) g[i] = wv[i] * (dv[i] - dot);
    float* rp = dlogits + row * E;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int e0 = (p * G + l) * 4;
      float o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        o[q] = 0.f;
#pragma unroll
        for (int i = 0; i < KP; ++i)
          if (id[i] == e0 + q) o[q] = g[i];
      }
      if constexpr (VEC) {
        if (e0 < E) *reinterpret_cast<float4*>(rp + e0) = make_float4(o[0], o[1], o[2], o[3]);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (e0 + q < E) rp[e0 + q] = o[q];
      }
    }
  }
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

inline int lanes_per_row(int E, int elems) {
  const int g = pow2_at_least((E + elems - 1) / elems);
  return g > 32 ? 32 : g;
}

// Persistent grid for a lane-group kernel: no more CTAs than are resident at once, so no
// SM runs a second partial wave (the kernels are register-limited below 8 CTAs per SM).
template <typename K>
int resident_grid(K kernel, int64_t n_warp_tiles) {
  // one value per kernel instantiation, computed once (thread-safe static initialisation)
  static const int per_sm = [kernel] {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, 256, 0) != cudaSuccess || b < 1)
      b = 1;
    return b;
  }();
  int64_t ctas = (n_warp_tiles + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * per_sm;
  if (ctas > cap) ctas = cap;
  return (int)(ctas < 1 ? 1 : ctas);
}

template <typename T, int G, int C, int KP>
void launch_lanes_fwd(const T* lp, int64_t rs, int64_t n, int E, int k, float* w, int64_t* idx,
                      bool vec, cudaStream_t st) {
  const int64_t tiles = (n + 32 / G - 1) / (32 / G);
  if (vec) {
    auto* kern = router_fwd_lanes<T, G, C, KP, true>;
    kern<<<resident_grid(kern, tiles), 256, 0, st>>>(lp, rs, n, E, k, w, idx);
  } else {
    auto* kern = router_fwd_lanes<T, G, C, KP, false>;
    kern<<<resident_grid(kern, tiles), 256, 0, st>>>(lp, rs, n, E, k, w, idx);
  }
}

template <typename T, int KP>
void lanes_fwd_g(const T* lp, int64_t rs, int64_t n, int E, int k, float* w, int64_t* idx,
                 bool vec, cudaStream_t st) {
  const int C = fwd_elems(E, n);
  if (C == 8) {
    switch (lanes_per_row(E, 8)) {
      case 1: launch_lanes_fwd<T, 1, 8, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
      case 2: launch_lanes_fwd<T, 2, 8, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
      case 4: launch_lanes_fwd<T, 4, 8, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
      case 8: launch_lanes_fwd<T, 8, 8, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
      case 16: launch_lanes_fwd<T, 16, 8, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
      default: launch_lanes_fwd<T, 32, 8, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
    }
  } else if (C == 16) {
    launch_lanes_fwd<T, 1, 16, KP>(lp, rs, n, E, k, w, idx, vec, st);
  } else {
    switch (lanes_per_row(E, 32)) {  // E <= 256: at most 8 lanes
      case 1: launch_lanes_fwd<T, 1, 32, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
      case 2: launch_lanes_fwd<T, 2, 32, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
      case 4: launch_lanes_fwd<T, 4, 32, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
      default: launch_lanes_fwd<T, 8, 32, KP>(lp, rs, n, E, k, w, idx, vec, st); break;
    }
  }
}

template <typename T>
int fwd_t(const void* logits, int64_t rs, int64_t n, int E, int k, float* w, int64_t* idx,
          cudaStream_t st) {
  const T* lp = static_cast<const T*>(logits);
  const int KPL = pow2_at_least(k);
  // Measured on B200: the lane groups win over the segment network for every k <= 8.
  if (KPL <= kLaneMaxKP) {
    constexpr int VN = 16 / (int)sizeof(T);
    const bool vec = aligned16(logits) && (rs * (int64_t)sizeof(T)) % 16 == 0 && E % VN == 0;
    switch (KPL) {
      case 1: lanes_fwd_g<T, 1>(lp, rs, n, E, k, w, idx, vec, st); break;
      case 2: lanes_fwd_g<T, 2>(lp, rs, n, E, k, w, idx, vec, st); break;
      case 4: lanes_fwd_g<T, 4>(lp, rs, n, E, k, w, idx, vec, st); break;
      default: lanes_fwd_g<T, 8>(lp, rs, n, E, k, w, idx, vec, st); break;
    }
    return launch_status("fk_router_fwd");
  }
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
  cudaStream_t st = fk::as_stream(stream);
  const int KPL = fk::pow2_at_least(k);
  // Every lane reads all k slots of its row, so the lane groups are used for k <= 4 only
  // (measured on B200: faster than the warp-per-row kernel there, slower at k = 8).
  if (KPL <= 4) {
    const int G = fk::lanes_per_row(n_experts, fk::kLaneElems);
    const bool vec = fk::aligned16(dlogits) && n_experts % 4 == 0;
    const int64_t tiles = (n_rows + 32 / G - 1) / (32 / G);
#define FK_LANES(G_, KP_)                                                                  \
  if (vec) {                                                                               \
    auto* kern = fk::router_bwd_lanes<G_, KP_, true>;                                      \
    kern<<<fk::resident_grid(kern, tiles), 256, 0, st>>>(dw, w, idx, dlogits, n_rows,      \
                                                         n_experts, k);                    \
  } else {                                                                                 \
    auto* kern = fk::router_bwd_lanes<G_, KP_, false>;                                     \
    kern<<<fk::resident_grid(kern, tiles), 256, 0, st>>>(dw, w, idx, dlogits, n_rows,      \
                                                         n_experts, k);                    \
  }
#define FK_LANES_G(KP_)                  \
  switch (G) {                           \
    case 1: FK_LANES(1, KP_) break;      \
    case 2: FK_LANES(2, KP_) break;      \
    case 4: FK_LANES(4, KP_) break;      \
    case 8: FK_LANES(8, KP_) break;      \
    case 16: FK_LANES(16, KP_) break;    \
    default: FK_LANES(32, KP_) break;    \
  }
    switch (KPL) {
      case 1: FK_LANES_G(1) break;
      case 2: FK_LANES_G(2) break;
      default: FK_LANES_G(4) break;
    }
#undef FK_LANES_G
#undef FK_LANES
    return fk::launch_status("fk_router_bwd");
  }
  const int L = fk::pow2_at_least(n_experts);
  const int S = L < 32 ? L : 32;
  const int V = L / S;
  const int64_t groups = (n_rows + (32 / S) - 1) / (32 / S);
  const int grid = fk::warp_grid(groups);
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
