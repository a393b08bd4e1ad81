// Fused cross-entropy forward + gradient, reference cross_entropy.py:24-116.
//
// HBM traffic is one read of the logits and one write of the gradient.  A row of V
// logits (250.5 KiB for V=128256 bf16) is larger than one SM's shared memory; one
// persistent CTA of 1024 threads per SM owns a row and sweeps it twice: the first sweep
// reduces it to (max, sum exp, sum x) with an online rescale, the second re-reads it from
// L2 (one row per SM in flight: ~37 MB) and writes the gradient.  Packets move through a
// per-thread cp.async ring in shared memory, so every thread keeps 8 x 16 bytes in
// flight.  Exponentials of 16-bit inputs are single ex2 instructions with log2(e) folded
// into an FMA.
//
// The mean-reduction scale 1/n_valid is folded into the gradient write (n_valid comes
// from a one-CTA prologue that counts non-ignored targets), and the scalar loss is a
// fixed-order reduction of the per-row losses (deterministic).  Rows that are not
// 16-byte aligned use a scalar three-sweep kernel.
#include "common.cuh"
#include "ptx.cuh"

#include <stdlib.h>

namespace fk {
namespace {

constexpr int kCeThreads = 256;

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

// 16-bit packets in pairs: packed max of the raw pairs, packed fp32 FMA/ADD (f32x2) for
// the exponent arguments and the running sums, so a packet of 8 logits costs 3 packed
// max, 8 conversions, 4 FFMA2, 8 ex2 and 4 FADD2 (plus 4 FADD2 for sum x with label
// smoothing).  The running sum is kept as two partial lanes (s.x, s.y).
template <typename T> struct Pair16;
template <> struct Pair16<__nv_bfloat16> {
  using type = __nv_bfloat162;
  static __device__ __forceinline__ type hmax(type a, type b) { return __hmax2(a, b); }
  static __device__ __forceinline__ float2 to_f2(type v) { return __bfloat1622float2(v); }
  static __device__ __forceinline__ type from_f2(float2 v) { return __float22bfloat162_rn(v); }
};
template <> struct Pair16<__half> {
  using type = __half2;
  static __device__ __forceinline__ type hmax(type a, type b) { return __hmax2(a, b); }
  static __device__ __forceinline__ float2 to_f2(type v) { return __half22float2(v); }
  static __device__ __forceinline__ type from_f2(float2 v) { return __float22half2_rn(v); }
};

template <typename T, bool SX>
__device__ __forceinline__ void online_add_packet2(float& m, float2& s2, float2& sx2,
                                                   const Vec16<T>& p) {
  using P = Pair16<T>;
  using P2 = typename P::type;
  constexpr int NP = Vec16<T>::N / 2;
  const P2* pp = reinterpret_cast<const P2*>(p.e);
  P2 mx = pp[0];
#pragma unroll
  for (int i = 1; i < NP; ++i) mx = P::hmax(mx, pp[i]);
  const float2 mf = P::to_f2(mx);
  const float pm = fmaxf(mf.x, mf.y);
  float2 x[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) x[i] = P::to_f2(pp[i]);
  if constexpr (SX) {
#pragma unroll
    for (int i = 0; i < NP; ++i) sx2 = __fadd2_rn(sx2, x[i]);
  }
  if (pm > m) {  // new running max
    const float sc = (m == -INFINITY) ? 0.f : ex2f((m - pm) * kLog2e);
    s2 = __fmul2_rn(s2, make_float2(sc, sc));
    m = pm;
  }
  if (m == -INFINITY) return;
  const float2 L = make_float2(kLog2e, kLog2e);
  const float2 B = make_float2(-m * kLog2e, -m * kLog2e);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const float2 t = __ffma2_rn(x[i], L, B);
    s2 = __fadd2_rn(s2, make_float2(ex2f(t.x), ex2f(t.y)));
  }
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

// Two-sweep row kernel: one CTA of 1024 threads per SM, persistent over rows.
// Sweep 1 reads the row (HBM) and keeps online (max, sum exp, sum x) per thread; sweep 2
// re-reads it -- it is still in L2: one row per SM is in flight, ~37 MB over the GPU --
// and writes the gradient with evict-first stores, so HBM sees one read and one write per
// element.  Both sweeps move packets with cp.async into a per-thread ring of kDepth
// 16-byte slots in shared memory (each thread reads back only the slots it filled, so no
// barrier is involved): kDepth packets per thread are in flight without holding
// registers, 128 KB per SM.
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
__device__ __forceinline__ void st_hint(void* ptr, uint4 v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.v4.u32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(ptr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kRowThreads = 1024;
constexpr int kDepth = 8;  // packets in flight per thread

// Streams the packets v = tid, tid + 1024, ... < nvec of one row through the cp.async
// ring and calls fn(v, packet) for each, in order.
template <typename T, typename Fn>
__device__ __forceinline__ void stream_row(const T* src, int nvec, uint64_t pol, uint32_t ring,
                                           Fn&& fn) {
  constexpr int VN = 16 / sizeof(T);
  const int tid = threadIdx.x;
  const int n_mine = nvec > tid ? (nvec - 1 - tid) / kRowThreads + 1 : 0;
#pragma unroll
  for (int i = 0; i < kDepth; ++i) {
    if (i < n_mine)
      cp_async16(ring + (uint32_t)(i * kRowThreads) * 16u, src + (int64_t)(tid + i * kRowThreads) * VN, pol);
    cp_async_commit();
  }
  for (int i = 0; i < n_mine; ++i) {
    cp_async_wait<kDepth - 1>();
    const uint32_t slot = ring + (uint32_t)((i % kDepth) * kRowThreads) * 16u;
    Vec16<T> p;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(p.u.x), "=r"(p.u.y), "=r"(p.u.z), "=r"(p.u.w)
                 : "r"(slot));
    fn(tid + i * kRowThreads, p);
    const int nx = i + kDepth;
    if (nx < n_mine) cp_async16(slot, src + (int64_t)(tid + nx * kRowThreads) * VN, pol);
    cp_async_commit();
  }
  cp_async_wait<0>();
}

template <typename T, bool SX>
__global__ void __launch_bounds__(kRowThreads, 1) ce_row_kernel(
    const T* __restrict__ logits, int64_t lstride, T* grad, int64_t gstride,
    const int64_t* __restrict__ targets, int64_t n_rows, int n_cols, int64_t ignore_index,
    float lsm, const int* __restrict__ n_valid_p, float* __restrict__ loss_rows,
    int* __restrict__ err) {
  constexpr int VN = 16 / sizeof(T);
  extern __shared__ __align__(128) unsigned char ring_raw[];
  __shared__ float wred[3][32];
  __shared__ float stats[1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t ring = ptx::smem_u32(ring_raw) + (uint32_t)tid * 16u;
  const int nvec = n_cols / VN;
  const uint64_t keep = policy_evict_last(), drop = policy_evict_first();
  const float inv_nv = 1.0f / (float)(*n_valid_p);
  const float smooth = lsm / (float)n_cols;
  const float sub = smooth * inv_nv, hsub = (1.0f - lsm) * inv_nv;
  for (int64_t row = blockIdx.x; row < n_rows; row += gridDim.x) {
    const T* src = logits + row * lstride;
    const int64_t t = targets[row];
    Online o{-INFINITY, 0.f, 0.f};
    if constexpr (sizeof(T) == 2) {
      float m = -INFINITY;
      float2 s2 = make_float2(0.f, 0.f), sx2 = make_float2(0.f, 0.f);
      stream_row<T>(src, nvec, keep, ring,
                    [&](int, const Vec16<T>& p) { online_add_packet2<T, SX>(m, s2, sx2, p); });
      o.m = m;
      o.s = s2.x + s2.y;
      o.sx = sx2.x + sx2.y;
    } else {
      stream_row<T>(src, nvec, keep, ring, [&](int, const Vec16<T>& p) { online_add_packet<T>(o, p); });
    }
    for (int i = nvec * VN + tid; i < n_cols; i += kRowThreads) online_add_scalar<T>(o, Elt<T>::to_f(src[i]));
    o = warp_combine<T>(o);
    if (lane == 0) {
      wred[0][warp] = o.m;
      wred[1][warp] = o.s;
      wred[2][warp] = o.sx;
    }
    __syncthreads();
    const bool ignored = (t == ignore_index);
    const bool invalid = !ignored && (t < 0 || t >= n_cols);
    if (warp == 0) {
      Online cc{wred[0][lane], wred[1][lane], wred[2][lane]};
      cc = warp_combine<T>(cc);
      if (lane == 0) {
        const float lse = cc.m + logf(cc.s);
        stats[0] = lse;
        float loss = invalid ? 0.f : lse - Elt<T>::to_f(src[ignored ? 0 : t]);
        if (lsm > 0.f) loss = (1.0f - lsm) * loss + lsm * (lse - cc.sx / (float)n_cols);
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
      const int tv = (t < (int64_t)nvec * VN) ? (int)(t / VN) : -1;
      if constexpr (sizeof(T) == 2) {
        using P = Pair16<T>;
        using P2 = typename P::type;
        constexpr int NP = VN / 2;
        const float2 L = make_float2(kLog2e, kLog2e);
        const float2 C = make_float2(-cexp, -cexp);
        const float2 NS = make_float2(-sub, -sub);
        stream_row<T>(src, nvec, drop, ring, [&](int vv, const Vec16<T>& p) {
          const P2* pp = reinterpret_cast<const P2*>(p.e);
          float2 g[NP];
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const float2 a = __ffma2_rn(P::to_f2(pp[i]), L, C);
            g[i] = make_float2(ex2f(a.x), ex2f(a.y));
            if constexpr (SX) g[i] = __fadd2_rn(g[i], NS);
          }
          if (vv == tv) {
            const int te = (int)(t - (int64_t)vv * VN);
#pragma unroll
            for (int i = 0; i < NP; ++i) {
              g[i].x -= (2 * i == te) ? hsub : 0.f;
              g[i].y -= (2 * i + 1 == te) ? hsub : 0.f;
            }
          }
          Vec16<T> o2;
          P2* op = reinterpret_cast<P2*>(o2.e);
#pragma unroll
          for (int i = 0; i < NP; ++i) op[i] = P::from_f2(g[i]);
          st_hint(dst + (int64_t)vv * VN, o2.u, drop);
        });
      } else {
        stream_row<T>(src, nvec, drop, ring, [&](int vv, const Vec16<T>& p) {
          float g[VN];
#pragma unroll
          for (int e = 0; e < VN; ++e) g[e] = gval(Elt<T>::to_f(p.e[e]));
          if (vv == tv) {
            const int te = (int)(t - (int64_t)vv * VN);
#pragma unroll
            for (int e = 0; e < VN; ++e) g[e] -= (e == te) ? hsub : 0.f;
          }
          Vec16<T> o2;
#pragma unroll
          for (int e = 0; e < VN; ++e) o2.e[e] = Elt<T>::from_f(g[e]);
          st_hint(dst + (int64_t)vv * VN, o2.u, drop);
        });
      }
      for (int i = nvec * VN + tid; i < n_cols; i += kRowThreads) {
        float g = gval(Elt<T>::to_f(src[i]));
        if ((int64_t)i == t) g -= hsub;
        dst[i] = Elt<T>::from_f(g);
      }
    }
    __syncthreads();  // in-place: every read of this row precedes later rows' writes
  }
}

// Fallback for rows that are not 16-byte aligned: one CTA per row, three scalar sweeps.
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
    const int rowvec = aligned16(lp) && aligned16(gp) && ((ls * (int64_t)sizeof(T)) % 16 == 0) &&
                       ((gs * (int64_t)sizeof(T)) % 16 == 0);
    if (rowvec) {
      int64_t g = n_rows < (int64_t)num_sms() ? n_rows : (int64_t)num_sms();
      const int smem = kDepth * kRowThreads * 16;
      auto* kern = lsm > 0.f ? ce_row_kernel<T, true> : ce_row_kernel<T, false>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      kern<<<(int)g, kRowThreads, smem, st>>>(lp, ls, gp, gs, targets, n_rows, (int)n_cols,
                                              ignore, lsm, n_valid, loss_rows, err);
      int s1 = launch_status("fk_ce_fwd(row)");
      if (s1 != FK_OK) return s1;
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
