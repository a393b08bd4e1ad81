// Fused cross-entropy forward + gradient, reference cross_entropy.py:24-116.
//
// HBM traffic is one read of the logits and one write of the gradient.  A row of V
// logits (250.5 KiB for V=128256 bf16) is larger than one SM's shared memory, so a
// thread-block CLUSTER of C CTAs (C <= 8) owns a row: CTA c bulk-copies (cp.async.bulk,
// mbarrier-completed) its 1/C slice of the row into shared memory, reduces it in ONE pass
// to (max, sum exp, sum x) with an online rescale, and the C partials (plus the target
// logit) are exchanged through distributed shared memory.  Every CTA combines the
// partials in rank order (so all CTAs hold bit-identical statistics), then writes the
// gradient of its slice straight from shared memory.  Nothing is re-read from HBM.
// Clusters are persistent and walk rows r = cluster_id, += n_clusters; each CTA holds two
// slice buffers and copies row r+1 while it works on row r; partial slots are
// double-buffered by row parity so one cluster barrier per row suffices.  Exponentials
// of 16-bit inputs are single ex2 instructions with log2(e) folded into an FMA.
//
// The mean-reduction scale 1/n_valid is folded into the gradient write (n_valid comes
// from a one-CTA prologue that counts non-ignored targets), and the scalar loss is a
// fixed-order reduction of the per-row losses (deterministic).  Rows longer than
// 8 x 108 KiB fall back to a three-sweep kernel that re-reads the row from global memory.
#include "common.cuh"
#include "ptx.cuh"

#include <stdlib.h>

namespace fk {
namespace {

constexpr int kCeThreads = 256;
constexpr int kMaxClusterBytes = 32 * 1024;   // target slice size per CTA
constexpr int kMaxSliceBytes = 108 * 1024;    // hard cap: two slices in shared memory
constexpr uint32_t kBulkPiece = 32 * 1024;    // bytes per cp.async.bulk instruction

template <typename T>
__device__ __forceinline__ float fexp(float x) { return __expf(x); }
template <>
__device__ __forceinline__ float fexp<float>(float x) { return expf(x); }

__global__ void ce_prologue(const int64_t* __restrict__ targets, int64_t n_rows,
                            int64_t ignore_index, int* __restrict__ n_valid,
                            int* __restrict__ err) {
  __shared__ int red[32];
  int c = 0;
  for (int64_t i = threadIdx.x; i < n_rows; i += blockDim.x) c += (targets[i] != ignore_index);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int tot = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    *n_valid = tot < 1 ? 1 : tot;
    *err = 0;
  }
}

__global__ void ce_finalize(const float* __restrict__ loss_rows, int64_t n_rows,
                            const int* __restrict__ n_valid, float* __restrict__ loss) {
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n_rows; i += blockDim.x) s += loss_rows[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    *loss = tot / (float)(*n_valid);
  }
}

// Block-wide reductions of up to 4 floats (max for slot 0 when kMax, else sums).
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
  return m;
}
__device__ __forceinline__ float2 block_sum2(float a, float b, float* red) {
  a = warp_sum(a);
  b = warp_sum(b);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) {
    red[warp] = a;
    red[32 + warp] = b;
  }
  __syncthreads();
  float sa = 0.f, sb = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
    sa += red[i];
    sb += red[32 + i];
  }
  return make_float2(sa, sb);
}

// Online (max, sum of exp) accumulation in the base-2 domain: values are kept as
// x*log2(e), so every exponential is one ex2 (16-bit inputs) or expf (fp32 inputs).
struct Online {
  float m;   // running max of x
  float s;   // sum exp(x - m)
  float sx;  // sum x
};

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

template <typename T>
__device__ __forceinline__ float exp_shift(float x, float m) {  // exp(x - m)
  return ex2f(fmaf(x, kLog2e, -m * kLog2e));
}
template <>
__device__ __forceinline__ float exp_shift<float>(float x, float m) {
  return expf(x - m);
}

template <typename T>
__device__ __forceinline__ Online combine(Online a, Online b) {
  Online r;
  r.m = fmaxf(a.m, b.m);
  r.sx = a.sx + b.sx;
  if (r.m == -INFINITY) {
    r.s = 0.f;
  } else {
    r.s = (a.m == -INFINITY ? 0.f : a.s * exp_shift<T>(a.m, r.m)) +
          (b.m == -INFINITY ? 0.f : b.s * exp_shift<T>(b.m, r.m));
  }
  return r;
}

template <typename T>
__device__ __forceinline__ void online_add_packet(Online& o, const Vec16<T>& p) {
  constexpr int VN = Vec16<T>::N;
  float x[VN];
  float pm = -INFINITY;
#pragma unroll
  for (int e = 0; e < VN; ++e) {
    x[e] = Elt<T>::to_f(p.e[e]);
    pm = fmaxf(pm, x[e]);
    o.sx += x[e];
  }
  const float mn = fmaxf(o.m, pm);
  if (mn == -INFINITY) return;
  if (o.m != mn) {
    o.s = (o.m == -INFINITY) ? 0.f : o.s * exp_shift<T>(o.m, mn);
    o.m = mn;
  }
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < VN; ++e) acc += exp_shift<T>(x[e], mn);
  o.s += acc;
}

template <typename T>
__device__ __forceinline__ void online_add_scalar(Online& o, float x) {
  o.sx += x;
  const float mn = fmaxf(o.m, x);
  if (mn == -INFINITY) return;
  if (o.m != mn) {
    o.s = (o.m == -INFINITY) ? 0.f : o.s * exp_shift<T>(o.m, mn);
    o.m = mn;
  }
  o.s += exp_shift<T>(x, mn);
}

template <typename T>
__device__ __forceinline__ Online warp_combine(Online o) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    Online b;
    b.m = __shfl_xor_sync(0xffffffffu, o.m, d);
    b.s = __shfl_xor_sync(0xffffffffu, o.s, d);
    b.sx = __shfl_xor_sync(0xffffffffu, o.sx, d);
    o = combine<T>(o, b);
  }
  return o;
}

template <typename T>
__global__ void __launch_bounds__(kCeThreads) ce_cluster_kernel(
    const T* __restrict__ logits, int64_t lstride, T* grad, int64_t gstride,
    const int64_t* __restrict__ targets, int64_t n_rows, int n_cols, int64_t ignore_index,
    float lsm, const int* __restrict__ n_valid_p, float* __restrict__ loss_rows,
    int* __restrict__ err, int chunk, int bulk, int gvec) {
  constexpr int VN = 16 / sizeof(T);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  auto buf_of = [&](int b) { return reinterpret_cast<T*>(smem_raw + (size_t)b * chunk * sizeof(T)); };
  __shared__ __align__(8) uint64_t full[2];
  __shared__ float slots[2][4];  // [row parity] {max, sum exp, sum x, target logit}
  __shared__ float wred[3][8];
  __shared__ float stats[4];     // combined {lse, sum x, target logit}
  __shared__ int dead;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t crank = ptx::cluster_ctarank();
  const uint32_t csize = ptx::cluster_nctarank();
  const int64_t c0 = (int64_t)crank * chunk;
  int my_len = (int)((int64_t)n_cols - c0);
  if (my_len > chunk) my_len = chunk;
  if (my_len < 0) my_len = 0;
  const int bulk_len = bulk ? (my_len / VN) * VN : 0;
  const uint32_t bulk_bytes = (uint32_t)bulk_len * sizeof(T);
  const int nvec = my_len / VN;

  const int64_t row0 = ptx::cluster_id_x();
  const int64_t rstep = ptx::nclusters_x();
  auto issue = [&](int64_t row, int b) {
    const unsigned char* src =
        reinterpret_cast<const unsigned char*>(logits + row * lstride + c0);
    unsigned char* dst = reinterpret_cast<unsigned char*>(buf_of(b));
    ptx::fence_proxy_async_smem();
    ptx::mbar_arrive_expect_tx(&full[b], bulk_bytes);
    for (uint32_t off = 0; off < bulk_bytes; off += kBulkPiece) {
      uint32_t n = bulk_bytes - off < kBulkPiece ? bulk_bytes - off : kBulkPiece;
      ptx::bulk_g2s(dst + off, src + off, n, &full[b]);
    }
  };

  if (tid == 0) {
    ptx::mbar_init(&full[0], 1);
    ptx::mbar_init(&full[1], 1);
    ptx::fence_mbar_init();
    dead = 0;
  }
  __syncthreads();
  if (tid == 0 && bulk_len > 0 && row0 < n_rows) issue(row0, 0);

  const float inv_nv = 1.0f / (float)(*n_valid_p);
  const float smooth = lsm / (float)n_cols;
  const float hit = 1.0f - lsm;
  int it = 0;
  for (int64_t row = row0; row < n_rows; row += rstep, ++it) {
    const int b = it & 1;
    const int par = it & 1;
    T* buf = buf_of(b);
    const T* src = logits + row * lstride + c0;
    bool poisoned = false;
    if (bulk_len > 0) {
      if (dead || !ptx::mbar_wait(&full[b], (uint32_t)((it >> 1) & 1))) {
        poisoned = true;
        if (!dead) atomicExch(err, 2);
      }
    }
    for (int i = bulk_len + tid; i < my_len; i += kCeThreads) buf[i] = src[i];
    const int64_t t = targets[row];
    __syncthreads();
    if (poisoned && tid == 0) dead = 1;
    // Prefetch the next row into the other buffer (freed at the end of the last row).
    if (tid == 0 && bulk_len > 0 && !dead && row + rstep < n_rows) issue(row + rstep, b ^ 1);

    // One pass over the slice: online max / sum exp / sum x.
    Online o{-INFINITY, 0.f, 0.f};
    const uint4* bv = reinterpret_cast<const uint4*>(buf);
    for (int v = tid; v < nvec; v += kCeThreads) {
      Vec16<T> p;
      p.u = bv[v];
      online_add_packet<T>(o, p);
    }
    for (int i = nvec * VN + tid; i < my_len; i += kCeThreads)
      online_add_scalar<T>(o, Elt<T>::to_f(buf[i]));
    o = warp_combine<T>(o);
    if (lane == 0) {
      wred[0][warp] = o.m;
      wred[1][warp] = o.s;
      wred[2][warp] = o.sx;
    }
    __syncthreads();
    if (tid == 0) {
      Online c{wred[0][0], wred[1][0], wred[2][0]};
      for (int w = 1; w < kCeThreads / 32; ++w) c = combine<T>(c, Online{wred[0][w], wred[1][w], wred[2][w]});
      float xt = 0.f;
      if (t >= c0 && t < c0 + my_len) xt = Elt<T>::to_f(buf[t - c0]);
      slots[par][0] = c.m;
      slots[par][1] = c.s;
      slots[par][2] = c.sx;
      slots[par][3] = xt;
    }
    ptx::cluster_sync();
    if (tid < 32) {
      // Lane i fetches CTA i's partials; lane 0 combines them in rank order.
      float pm = -INFINITY, ps = 0.f, px = 0.f, pt = 0.f;
      if ((uint32_t)tid < csize) {
        uint32_t a = ptx::mapa(ptx::smem_u32(&slots[par][0]), (uint32_t)tid);
        pm = ptx::ld_dsmem_f32(a);
        ps = ptx::ld_dsmem_f32(a + 4);
        px = ptx::ld_dsmem_f32(a + 8);
        pt = ptx::ld_dsmem_f32(a + 12);
      }
      Online c{-INFINITY, 0.f, 0.f};
      float XT = 0.f;
      for (uint32_t i = 0; i < csize; ++i) {
        Online q{__shfl_sync(0xffffffffu, pm, i), __shfl_sync(0xffffffffu, ps, i),
                 __shfl_sync(0xffffffffu, px, i)};
        c = combine<T>(c, q);
        XT += __shfl_sync(0xffffffffu, pt, i);
      }
      if (tid == 0) {
        stats[0] = c.m + logf(c.s);
        stats[1] = c.sx;
        stats[2] = XT;
      }
    }
    __syncthreads();
    const float lse = stats[0];
    const bool ignored = (t == ignore_index);
    const bool invalid = !ignored && (t < 0 || t >= n_cols);
    if (crank == 0 && tid == 0) {
      float loss = lse - stats[2];
      if (lsm > 0.f) loss = (1.0f - lsm) * loss + lsm * (lse - stats[1] / (float)n_cols);
      if (ignored) loss = 0.f;
      if (invalid || poisoned) loss = __int_as_float(0x7fc00000);
      loss_rows[row] = loss;
      if (invalid) atomicExch(err, 1);
    }

    // Gradient of this slice, straight from shared memory.
    T* dst = grad + row * gstride + c0;
    if (ignored || invalid || poisoned) {
      const T z = Elt<T>::from_f((invalid || poisoned) ? __int_as_float(0x7fc00000) : 0.f);
      if (gvec) {
        Vec16<T> zz;
#pragma unroll
        for (int e = 0; e < VN; ++e) zz.e[e] = z;
        for (int v = tid; v < nvec; v += kCeThreads) st_stream(dst + v * VN, zz);
        for (int i = nvec * VN + tid; i < my_len; i += kCeThreads) dst[i] = z;
      } else {
        for (int i = tid; i < my_len; i += kCeThreads) dst[i] = z;
      }
    } else {
      const int64_t tl = t - c0;  // target position inside this slice (may be outside)
      const float sub = smooth * inv_nv;
      const float hsub = hit * inv_nv;
      // exp(x - lse) * inv_nv == 2^(x*log2e - (lse*log2e - log2(inv_nv)))
      const float cexp = lse * kLog2e - log2f(inv_nv);
      auto gval = [&](float x) -> float {
        if constexpr (sizeof(T) == 4) return expf(x - lse) * inv_nv - sub;
        else return ex2f(fmaf(x, kLog2e, -cexp)) - sub;
      };
      if (gvec) {
        const int tv = (tl >= 0 && tl < nvec * VN) ? (int)(tl / VN) : -1;
        for (int v = tid; v < nvec; v += kCeThreads) {
          Vec16<T> p, o;
          p.u = bv[v];
          float g[VN];
#pragma unroll
          for (int e = 0; e < VN; ++e) g[e] = gval(Elt<T>::to_f(p.e[e]));
          if (v == tv) g[tl - (int64_t)v * VN] -= hsub;
#pragma unroll
          for (int e = 0; e < VN; ++e) o.e[e] = Elt<T>::from_f(g[e]);
          st_stream(dst + v * VN, o);
        }
        for (int i = nvec * VN + tid; i < my_len; i += kCeThreads) {
          float g = gval(Elt<T>::to_f(buf[i]));
          if ((int64_t)i == tl) g -= hsub;
          dst[i] = Elt<T>::from_f(g);
        }
      } else {
        for (int i = tid; i < my_len; i += kCeThreads) {
          float g = gval(Elt<T>::to_f(buf[i]));
          if ((int64_t)i == tl) g -= hsub;
          dst[i] = Elt<T>::from_f(g);
        }
      }
    }
    __syncthreads();  // this buffer is free for the copy issued two rows from now
  }
  ptx::cluster_sync();  // no CTA leaves while a peer may still read its slots
}

// Two-sweep row kernel: one CTA of 1024 threads per row (one CTA per SM, persistent).
// Sweep 1 streams the row from HBM with an L2 evict-last policy and keeps online
// (max, sum exp, sum x) per thread; sweep 2 re-reads the row -- it is still in L2, the
// 148 rows in flight occupy ~37 MB -- with evict-first and writes the gradient with
// evict-first stores, so HBM sees one read and one write per element.
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint4 ld_hint(const void* ptr, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr), "l"(pol));
  return v;
}
__device__ __forceinline__ void st_hint(void* ptr, uint4 v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.v4.u32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(ptr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "l"(pol)
               : "memory");
}

constexpr int kRowThreads = 1024;
constexpr int kRowUnroll = 4;

template <typename T>
__global__ void __launch_bounds__(kRowThreads, 1) ce_row_kernel(
    const T* __restrict__ logits, int64_t lstride, T* grad, int64_t gstride,
    const int64_t* __restrict__ targets, int64_t n_rows, int n_cols, int64_t ignore_index,
    float lsm, const int* __restrict__ n_valid_p, float* __restrict__ loss_rows,
    int* __restrict__ err) {
  constexpr int VN = 16 / sizeof(T);
  __shared__ float wred[3][32];
  __shared__ float stats[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nvec = n_cols / VN;
  const uint64_t keep = policy_evict_last(), drop = policy_evict_first();
  const float inv_nv = 1.0f / (float)(*n_valid_p);
  const float smooth = lsm / (float)n_cols;
  const float sub = smooth * inv_nv, hsub = (1.0f - lsm) * inv_nv;
  for (int64_t row = blockIdx.x; row < n_rows; row += gridDim.x) {
    const T* src = logits + row * lstride;
    const int64_t t = targets[row];
    Online o{-INFINITY, 0.f, 0.f};
    int v = tid;
    for (; v + (kRowUnroll - 1) * kRowThreads < nvec; v += kRowUnroll * kRowThreads) {
      Vec16<T> p[kRowUnroll];
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u) p[u].u = ld_hint(src + (int64_t)(v + u * kRowThreads) * VN, keep);
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u) online_add_packet<T>(o, p[u]);
    }
    for (; v < nvec; v += kRowThreads) {
      Vec16<T> p;
      p.u = ld_hint(src + (int64_t)v * VN, keep);
      online_add_packet<T>(o, p);
    }
    for (int i = nvec * VN + tid; i < n_cols; i += kRowThreads) online_add_scalar<T>(o, Elt<T>::to_f(src[i]));
    o = warp_combine<T>(o);
    if (lane == 0) {
      wred[0][warp] = o.m;
      wred[1][warp] = o.s;
      wred[2][warp] = o.sx;
    }
    __syncthreads();
    if (warp == 0) {
      Online c{wred[0][lane], wred[1][lane], wred[2][lane]};
      c = warp_combine<T>(c);
      if (lane == 0) {
        const float lse = c.m + logf(c.s);
        stats[0] = lse;
        const bool ignored = (t == ignore_index);
        const bool invalid = !ignored && (t < 0 || t >= n_cols);
        float loss = invalid ? 0.f : lse - Elt<T>::to_f(src[ignored ? 0 : t]);
        if (lsm > 0.f) loss = (1.0f - lsm) * loss + lsm * (lse - c.sx / (float)n_cols);
        if (ignored) loss = 0.f;
        if (invalid) {
          loss = __int_as_float(0x7fc00000);
          atomicExch(err, 1);
        }
        loss_rows[row] = loss;
      }
    }
    __syncthreads();
    const float lse = stats[0];
    const bool ignored = (t == ignore_index);
    const bool invalid = !ignored && (t < 0 || t >= n_cols);
    T* dst = grad + row * gstride;
    if (ignored || invalid) {
      const T z = Elt<T>::from_f(invalid ? __int_as_float(0x7fc00000) : 0.f);
      Vec16<T> zz;
#pragma unroll
      for (int e = 0; e < VN; ++e) zz.e[e] = z;
      for (int w = tid; w < nvec; w += kRowThreads) st_hint(dst + (int64_t)w * VN, zz.u, drop);
      for (int i = nvec * VN + tid; i < n_cols; i += kRowThreads) dst[i] = z;
    } else {
      const float cexp = lse * kLog2e - log2f(inv_nv);
      auto gval = [&](float x) -> float {
        if constexpr (sizeof(T) == 4) return expf(x - lse) * inv_nv - sub;
        else return ex2f(fmaf(x, kLog2e, -cexp)) - sub;
      };
      const int tv = (int)(t / VN);
      int w = tid;
      for (; w + (kRowUnroll - 1) * kRowThreads < nvec; w += kRowUnroll * kRowThreads) {
        Vec16<T> p[kRowUnroll];
#pragma unroll
        for (int u = 0; u < kRowUnroll; ++u) p[u].u = ld_hint(src + (int64_t)(w + u * kRowThreads) * VN, drop);
#pragma unroll
        for (int u = 0; u < kRowUnroll; ++u) {
          const int vv = w + u * kRowThreads;
          float g[VN];
#pragma unroll
          for (int e = 0; e < VN; ++e) g[e] = gval(Elt<T>::to_f(p[u].e[e]));
          if (vv == tv && t < (int64_t)nvec * VN) g[t - (int64_t)vv * VN] -= hsub;
          Vec16<T> o2;
#pragma unroll
          for (int e = 0; e < VN; ++e) o2.e[e] = Elt<T>::from_f(g[e]);
          st_hint(dst + (int64_t)vv * VN, o2.u, drop);
        }
      }
      for (; w < nvec; w += kRowThreads) {
        Vec16<T> p;
        p.u = ld_hint(src + (int64_t)w * VN, drop);
        float g[VN];
#pragma unroll
        for (int e = 0; e < VN; ++e) g[e] = gval(Elt<T>::to_f(p.e[e]));
        if (w == tv && t < (int64_t)nvec * VN) g[t - (int64_t)w * VN] -= hsub;
        Vec16<T> o2;
#pragma unroll
        for (int e = 0; e < VN; ++e) o2.e[e] = Elt<T>::from_f(g[e]);
        st_hint(dst + (int64_t)w * VN, o2.u, drop);
      }
      for (int i = nvec * VN + tid; i < n_cols; i += kRowThreads) {
        float g = gval(Elt<T>::to_f(src[i]));
        if ((int64_t)i == t) g -= hsub;
        dst[i] = Elt<T>::from_f(g);
      }
    }
    __syncthreads();  // in-place: every read of this row precedes the next row's stats
  }
}

// Fallback for rows longer than the cluster path holds: one CTA per row, three sweeps.
template <typename T>
__global__ void __launch_bounds__(kCeThreads) ce_generic_kernel(
    const T* __restrict__ logits, int64_t lstride, T* grad, int64_t gstride,
    const int64_t* __restrict__ targets, int64_t n_rows, int64_t n_cols, int64_t ignore_index,
    float lsm, const int* __restrict__ n_valid_p, float* __restrict__ loss_rows,
    int* __restrict__ err) {
  __shared__ float red[64];
  const float inv_nv = 1.0f / (float)(*n_valid_p);
  const float smooth = lsm / (float)n_cols;
  for (int64_t row = blockIdx.x; row < n_rows; row += gridDim.x) {
    const T* src = logits + row * lstride;
    const int64_t t = targets[row];
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < n_cols; i += kCeThreads) m = fmaxf(m, Elt<T>::to_f(src[i]));
    m = block_max(m, red);
    float s = 0.f, sx = 0.f;
    for (int64_t i = threadIdx.x; i < n_cols; i += kCeThreads) {
      float x = Elt<T>::to_f(src[i]);
      if (m != -INFINITY) s += fexp<T>(x - m);
      sx += x;
    }
    float2 ss = block_sum2(s, sx, red);
    const float lse = m + logf(ss.x);
    const bool ignored = t == ignore_index;
    const bool invalid = !ignored && (t < 0 || t >= n_cols);
    if (threadIdx.x == 0) {
      float loss = invalid ? 0.f : lse - Elt<T>::to_f(src[ignored ? 0 : t]);
      if (lsm > 0.f) loss = (1.0f - lsm) * loss + lsm * (lse - ss.y / (float)n_cols);
      if (ignored) loss = 0.f;
      if (invalid) {
        loss = __int_as_float(0x7fc00000);
        atomicExch(err, 1);
      }
      loss_rows[row] = loss;
    }
    T* dst = grad + row * gstride;
    for (int64_t i = threadIdx.x; i < n_cols; i += kCeThreads) {
      float g;
      if (invalid) g = __int_as_float(0x7fc00000);
      else if (ignored) g = 0.f;
      else {
        g = fexp<T>(Elt<T>::to_f(src[i]) - lse) - smooth;
        if (i == t) g -= 1.0f - lsm;
        g *= inv_nv;
      }
      dst[i] = Elt<T>::from_f(g);
    }
    __syncthreads();  // all reads of this row done before a possible in-place overwrite
  }
}

template <typename T>
__global__ void ce_scale_kernel(T* grad, int64_t gstride, int64_t n_rows, int64_t n_cols,
                                const float* __restrict__ go, int vec) {
  const float s = *go;
  if (s == 1.0f) return;
  constexpr int VN = 16 / sizeof(T);
  if (vec) {  // contiguous, aligned: flat 16-byte packets
    const int64_t nv = n_rows * n_cols / VN;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv;
         v += (int64_t)gridDim.x * blockDim.x) {
      Vec16<T> p = ld_stream(grad + v * VN);
#pragma unroll
      for (int e = 0; e < VN; ++e) p.e[e] = Elt<T>::from_f(Elt<T>::to_f(p.e[e]) * s);
      st_stream(grad + v * VN, p);
    }
    for (int64_t i = nv * VN + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_rows * n_cols;
         i += (int64_t)gridDim.x * blockDim.x)
      grad[i] = Elt<T>::from_f(Elt<T>::to_f(grad[i]) * s);
    return;
  }
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x)
    for (int64_t c = threadIdx.x; c < n_cols; c += blockDim.x)
      grad[r * gstride + c] = Elt<T>::from_f(Elt<T>::to_f(grad[r * gstride + c]) * s);
}

template <typename T>
int fwd_t(const void* logits, int64_t ls, void* grad, int64_t gs, const int64_t* targets,
          int64_t n_rows, int64_t n_cols, int64_t ignore, float lsm, float* loss_rows,
          float* loss, int* n_valid, int* err, cudaStream_t st) {
  const T* lp = static_cast<const T*>(logits);
  T* gp = static_cast<T*>(grad);
  ce_prologue<<<1, 1024, 0, st>>>(targets, n_rows, ignore, n_valid, err);
  int s0 = launch_status("fk_ce_fwd(prologue)");
  if (s0 != FK_OK) return s0;
  if (n_rows > 0) {
    constexpr int VN = 16 / sizeof(T);
    int C = 1;
    auto slice = [&](int c) {
      int64_t per = (n_cols + c - 1) / c;
      return ((per + VN - 1) / VN) * VN;
    };
    while (C < 8 && slice(C) * (int64_t)sizeof(T) > kMaxClusterBytes) C <<= 1;
    const int64_t chunk = slice(C);
    const int rowvec = aligned16(lp) && aligned16(gp) && ((ls * (int64_t)sizeof(T)) % 16 == 0) &&
                       ((gs * (int64_t)sizeof(T)) % 16 == 0);
    const char* path = getenv("FKB200_CE_PATH");
    const bool use_row = rowvec && !(path && path[0] == 'c');
    if (use_row) {
      int64_t g = n_rows < (int64_t)num_sms() ? n_rows : (int64_t)num_sms();
      ce_row_kernel<T><<<(int)g, kRowThreads, 0, st>>>(lp, ls, gp, gs, targets, n_rows, (int)n_cols,
                                                       ignore, lsm, n_valid, loss_rows, err);
      int s1 = launch_status("fk_ce_fwd(row)");
      if (s1 != FK_OK) return s1;
    } else if (chunk * (int64_t)sizeof(T) <= kMaxSliceBytes) {
      const int smem = (int)(2 * chunk * sizeof(T));
      auto kern = ce_cluster_kernel<T>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = C;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cfg.blockDim = dim3(kCeThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = st;
      int max_clusters = 0;
      cfg.gridDim = dim3(C * num_sms());
      if (cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg) != cudaSuccess ||
          max_clusters < 1) {
        cudaGetLastError();
        max_clusters = num_sms() / C;
        if (max_clusters < 1) max_clusters = 1;
      }
      int64_t nclu = n_rows < max_clusters ? n_rows : max_clusters;
      cfg.gridDim = dim3((unsigned)(nclu * C));
      const int bulk = aligned16(lp) && ((ls * (int64_t)sizeof(T)) % 16 == 0);
      const int gvec = aligned16(gp) && ((gs * (int64_t)sizeof(T)) % 16 == 0);
      cudaError_t e = cudaLaunchKernelEx(&cfg, kern, lp, ls, gp, gs, targets, n_rows, (int)n_cols,
                                         ignore, lsm, (const int*)n_valid, loss_rows, err,
                                         (int)chunk, bulk, gvec);
      if (e != cudaSuccess) return fail(FK_ERR_LAUNCH, "fk_ce_fwd: %s", cudaGetErrorString(e));
    } else {
      int64_t g = n_rows < (int64_t)num_sms() * 4 ? n_rows : (int64_t)num_sms() * 4;
      ce_generic_kernel<T><<<(int)g, kCeThreads, 0, st>>>(lp, ls, gp, gs, targets, n_rows, n_cols,
                                                         ignore, lsm, n_valid, loss_rows, err);
      int s1 = launch_status("fk_ce_fwd(generic)");
      if (s1 != FK_OK) return s1;
    }
  }
  ce_finalize<<<1, 1024, 0, st>>>(loss_rows, n_rows, n_valid, loss);
  return launch_status("fk_ce_fwd(finalize)");
}

}  // namespace
}  // namespace fk

extern "C" int fk_ce_fwd(const void* logits, int64_t row_stride, void* grad,
                         int64_t grad_row_stride, const int64_t* targets, int64_t n_rows,
                         int64_t n_cols, int64_t ignore_index, float label_smoothing, int dtype,
                         float* loss_rows, float* loss, int* n_valid, int* err_flag,
                         void* stream) {
  FK_CHECK_ARG(n_rows >= 0 && n_cols >= 1, "fk_ce_fwd: bad shape [%lld, %lld]",
               (long long)n_rows, (long long)n_cols);
  FK_CHECK_ARG(n_cols < (int64_t)1 << 31, "fk_ce_fwd: n_cols too large");
  FK_CHECK_ARG(loss && n_valid && err_flag, "fk_ce_fwd: null pointer");
  FK_CHECK_ARG(n_rows == 0 || (logits && grad && targets && loss_rows),
               "fk_ce_fwd: null pointer");
  FK_CHECK_ARG(row_stride >= n_cols && grad_row_stride >= n_cols, "fk_ce_fwd: stride < n_cols");
  FK_CHECK_ARG(label_smoothing >= 0.f && label_smoothing <= 1.f,
               "fk_ce_fwd: label_smoothing outside [0, 1]");
  FK_DISPATCH_DTYPE(dtype, return fk::fwd_t<scalar_t>(logits, row_stride, grad, grad_row_stride,
                                                      targets, n_rows, n_cols, ignore_index,
                                                      label_smoothing, loss_rows, loss, n_valid,
                                                      err_flag, fk::as_stream(stream)));
  return FK_OK;
}

extern "C" int fk_ce_bwd_scale(void* grad, int64_t grad_row_stride, int64_t n_rows,
                               int64_t n_cols, const float* grad_output, int dtype,
                               void* stream) {
  FK_CHECK_ARG(n_rows >= 0 && n_cols >= 0, "fk_ce_bwd_scale: negative shape");
  if (n_rows == 0 || n_cols == 0) return FK_OK;
  FK_CHECK_ARG(grad && grad_output, "fk_ce_bwd_scale: null pointer");
  FK_CHECK_ARG(grad_row_stride >= n_cols, "fk_ce_bwd_scale: stride < n_cols");
  cudaStream_t st = fk::as_stream(stream);
  FK_DISPATCH_DTYPE(dtype, {
    const int vec = fk::aligned16(grad) && grad_row_stride == n_cols;
    int grid = fk::num_sms() * 8;
    fk::ce_scale_kernel<scalar_t><<<grid, 256, 0, st>>>(static_cast<scalar_t*>(grad),
                                                        grad_row_stride, n_rows, n_cols,
                                                        grad_output, vec);
  });
  return fk::launch_status("fk_ce_bwd_scale");
}
