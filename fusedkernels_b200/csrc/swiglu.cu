// SwiGLU forward/backward: out = silu(gate) * up and its gradient.
//
// Pure streaming kernels (HBM-bound): every element is read once and written once.
// Each thread moves 16-byte packets (8 bf16/fp16 or 4 fp32) with evict-first hints,
// UNROLL packets per operand in flight per loop trip, over a grid of
// (SMs x resident CTAs) persistent CTAs.  Arithmetic is fp32, as in the reference
// (swiglu.py:19-51).
#include "common.cuh"

namespace fk {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

template <typename T>
__device__ __forceinline__ float silu_f(float g) { return g * sigmoidf_t<T>(g); }

template <typename T>
__global__ void __launch_bounds__(kThreads) swiglu_fwd_vec(const T* __restrict__ gate,
                                                           const T* __restrict__ up,
                                                           T* __restrict__ out, int64_t n_vec) {
  using V = Vec16<T>;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < n_vec; i += kUnroll * stride) {
    V g[kUnroll], u[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      g[j] = ld_stream(gate + (i + j * stride) * V::N);
      u[j] = ld_stream(up + (i + j * stride) * V::N);
    }
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      V o;
#pragma unroll
      for (int e = 0; e < V::N; ++e) {
        float gf = Elt<T>::to_f(g[j].e[e]);
        o.e[e] = Elt<T>::from_f(silu_f<T>(gf) * Elt<T>::to_f(u[j].e[e]));
      }
      st_stream(out + (i + j * stride) * V::N, o);
    }
  }
  for (; i < n_vec; i += stride) {
    V g = ld_stream(gate + i * V::N), u = ld_stream(up + i * V::N), o;
#pragma unroll
    for (int e = 0; e < V::N; ++e)
      o.e[e] = Elt<T>::from_f(silu_f<T>(Elt<T>::to_f(g.e[e])) * Elt<T>::to_f(u.e[e]));
    st_stream(out + i * V::N, o);
  }
}

template <typename T>
__global__ void swiglu_fwd_scalar(const T* __restrict__ gate, const T* __restrict__ up,
                                  T* __restrict__ out, int64_t begin, int64_t n) {
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float g = Elt<T>::to_f(gate[i]);
    out[i] = Elt<T>::from_f(silu_f<T>(g) * Elt<T>::to_f(up[i]));
  }
}

template <typename T>
__device__ __forceinline__ void swiglu_grad(float d, float g, float u, float& dg, float& du) {
  float s = sigmoidf_t<T>(g);
  float silu = g * s;
  du = d * silu;
  dg = d * u * (s * (1.0f + g * (1.0f - s)));
}

template <typename T>
__global__ void __launch_bounds__(kThreads) swiglu_bwd_vec(const T* __restrict__ dout,
                                                           const T* __restrict__ gate,
                                                           const T* __restrict__ up,
                                                           T* __restrict__ dgate,
                                                           T* __restrict__ dup, int64_t n_vec) {
  using V = Vec16<T>;
  constexpr int U = kUnroll / 2 > 0 ? kUnroll / 2 : 1;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  for (; i + (U - 1) * stride < n_vec; i += U * stride) {
    V d[U], g[U], u[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      d[j] = ld_stream(dout + (i + j * stride) * V::N);
      g[j] = ld_stream(gate + (i + j * stride) * V::N);
      u[j] = ld_stream(up + (i + j * stride) * V::N);
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      V og, ou;
#pragma unroll
      for (int e = 0; e < V::N; ++e) {
        float dg, du;
        swiglu_grad<T>(Elt<T>::to_f(d[j].e[e]), Elt<T>::to_f(g[j].e[e]),
                       Elt<T>::to_f(u[j].e[e]), dg, du);
        og.e[e] = Elt<T>::from_f(dg);
        ou.e[e] = Elt<T>::from_f(du);
      }
      st_stream(dgate + (i + j * stride) * V::N, og);
      st_stream(dup + (i + j * stride) * V::N, ou);
    }
  }
  for (; i < n_vec; i += stride) {
    V d = ld_stream(dout + i * V::N), g = ld_stream(gate + i * V::N), u = ld_stream(up + i * V::N);
    V og, ou;
#pragma unroll
    for (int e = 0; e < V::N; ++e) {
      float dg, du;
      swiglu_grad<T>(Elt<T>::to_f(d.e[e]), Elt<T>::to_f(g.e[e]), Elt<T>::to_f(u.e[e]), dg, du);
      og.e[e] = Elt<T>::from_f(dg);
      ou.e[e] = Elt<T>::from_f(du);
    }
    st_stream(dgate + i * V::N, og);
    st_stream(dup + i * V::N, ou);
  }
}

template <typename T>
__global__ void swiglu_bwd_scalar(const T* __restrict__ dout, const T* __restrict__ gate,
                                  const T* __restrict__ up, T* __restrict__ dgate,
                                  T* __restrict__ dup, int64_t begin, int64_t n) {
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float dg, du;
    swiglu_grad<T>(Elt<T>::to_f(dout[i]), Elt<T>::to_f(gate[i]), Elt<T>::to_f(up[i]), dg, du);
    dgate[i] = Elt<T>::from_f(dg);
    dup[i] = Elt<T>::from_f(du);
  }
}

// Persistent grid: SMs x 8 CTAs of 256 threads (2048 threads/SM), capped by the work.
inline int stream_grid(int64_t n_vec) {
  int64_t want = (n_vec + kThreads - 1) / kThreads;
  int64_t cap = (int64_t)num_sms() * 8;
  if (want > cap) want = cap;
  return (int)(want < 1 ? 1 : want);
}

template <typename T>
int swiglu_fwd_t(const void* gate, const void* up, void* out, int64_t n, cudaStream_t s) {
  const T* g = static_cast<const T*>(gate);
  const T* u = static_cast<const T*>(up);
  T* o = static_cast<T*>(out);
  int64_t begin = 0;
  if (aligned16(g) && aligned16(u) && aligned16(o)) {
    int64_t n_vec = n / Vec16<T>::N;
    if (n_vec > 0) swiglu_fwd_vec<T><<<stream_grid(n_vec), kThreads, 0, s>>>(g, u, o, n_vec);
    begin = n_vec * Vec16<T>::N;
  }
  if (begin < n) {
    int64_t rest = n - begin;
    int grid = (int)((rest + kThreads - 1) / kThreads);
    if (grid > num_sms() * 8) grid = num_sms() * 8;
    swiglu_fwd_scalar<T><<<grid, kThreads, 0, s>>>(g, u, o, begin, n);
  }
  return launch_status("fk_swiglu_fwd");
}

template <typename T>
int swiglu_bwd_t(const void* dout, const void* gate, const void* up, void* dgate, void* dup,
                 int64_t n, cudaStream_t s) {
  const T* d = static_cast<const T*>(dout);
  const T* g = static_cast<const T*>(gate);
  const T* u = static_cast<const T*>(up);
  T* dg = static_cast<T*>(dgate);
  T* du = static_cast<T*>(dup);
  int64_t begin = 0;
  if (aligned16(d) && aligned16(g) && aligned16(u) && aligned16(dg) && aligned16(du)) {
    int64_t n_vec = n / Vec16<T>::N;
    if (n_vec > 0)
      swiglu_bwd_vec<T><<<stream_grid(n_vec), kThreads, 0, s>>>(d, g, u, dg, du, n_vec);
    begin = n_vec * Vec16<T>::N;
  }
  if (begin < n) {
    int64_t rest = n - begin;
    int grid = (int)((rest + kThreads - 1) / kThreads);
    if (grid > num_sms() * 8) grid = num_sms() * 8;
    swiglu_bwd_scalar<T><<<grid, kThreads, 0, s>>>(d, g, u, dg, du, begin, n);
  }
  return launch_status("fk_swiglu_bwd");
}

}  // namespace
}  // namespace fk

extern "C" int fk_swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, int dtype,
                             void* stream) {
  FK_CHECK_ARG(n >= 0, "fk_swiglu_fwd: n=%lld < 0", (long long)n);
  if (n == 0) return FK_OK;
  FK_CHECK_ARG(gate && up && out, "fk_swiglu_fwd: null pointer");
  FK_DISPATCH_DTYPE(dtype, return fk::swiglu_fwd_t<scalar_t>(gate, up, out, n, fk::as_stream(stream)));
  return FK_OK;
}

extern "C" int fk_swiglu_bwd(const void* dout, const void* gate, const void* up, void* dgate,
                             void* dup, int64_t n, int dtype, void* stream) {
  FK_CHECK_ARG(n >= 0, "fk_swiglu_bwd: n=%lld < 0", (long long)n);
  if (n == 0) return FK_OK;
  FK_CHECK_ARG(dout && gate && up && dgate && dup, "fk_swiglu_bwd: null pointer");
  FK_DISPATCH_DTYPE(dtype,
                    return fk::swiglu_bwd_t<scalar_t>(dout, gate, up, dgate, dup, n,
                                                      fk::as_stream(stream)));
  return FK_OK;
}
