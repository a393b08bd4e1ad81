// RMSNorm forward/backward (fp32 accumulation, reference rmsnorm.py:20-71).
//
// Path selection for 16-byte aligned rows (the workloads): rows of at most 4 KB use the
// forward warp rings, rows of at most 16 KB the TMA ring kernels (shared-memory rings
// filled by cp.async.bulk, below), longer rows the register path; unaligned rows the
// generic path.  All share the row walk, the fixed-order reductions and the dw scheme.
//
// Register path: persistent CTAs walk rows r = blockIdx.x, += gridDim.x.
// A CTA of T threads covers one row with VPT 16-byte packets per thread; the packet
// index of (thread t, slot j) is j*T + t, so every slot is one fully coalesced sweep of
// the row.  The weight slice a thread needs is loaded once into registers and reused
// for every row the CTA visits.  The row's sum of squares is a warp-shuffle reduce plus
// one shared-memory exchange (double-buffered by row parity, so one __syncthreads per
// row).  Each CTA keeps PF rows of loads in flight (register ring, refilled as soon as
// a row is consumed), so a CTA always has loads outstanding across its reductions.
//
// Backward: the same walk; dx is written per row and the weight gradient
// sum_r dy*x*rstd accumulates in fp32 registers owned by the thread for its fixed
// columns.  At the end each CTA writes its partial row to the workspace and a second
// kernel reduces the G partial rows in a fixed order (deterministic, no atomics).
//
// Generic path: any cols / alignment, scalar element loops re-reading the row.
#include "common.cuh"
#include "ptx.cuh"
#include <mutex>

namespace fk {
namespace {

template <typename W>
__device__ __forceinline__ float load_w(const void* w, int64_t c) {
  return Elt<W>::to_f(static_cast<const W*>(w)[c]);
}

__device__ __forceinline__ float block_sum(float v, float* red /*[32]*/, int nwarps) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nwarps; ++i) s += red[i];  // fixed order: deterministic
  return s;
}

// ------------------------------------------------------------------ forward (regs) ----
// PF rows are in flight per CTA: the slot consumed for row r is refilled with row
// r + PF*grid right after use, so PF-1 rows of loads overlap every reduction.
template <typename T, typename W, int VPT, int PF>
__global__ void __launch_bounds__(512) rmsnorm_fwd_reg(const T* __restrict__ x, int64_t xs,
                                                        const void* __restrict__ w,
                                                        T* __restrict__ y, int64_t ys,
                                                        float* __restrict__ rstd, int64_t rows,
                                                        int cols, float eps) {
  using V = Vec16<T>;
  constexpr int N = V::N;
  __shared__ float red[2][32];
  const int T_ = blockDim.x, tid = threadIdx.x, nwarps = T_ >> 5;
  const int nvec = cols / N;
  const int64_t G = gridDim.x;
  float wr[VPT][N];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    int v = j * T_ + tid;
#pragma unroll
    for (int e = 0; e < N; ++e) wr[j][e] = (v < nvec) ? load_w<W>(w, (int64_t)v * N + e) : 0.f;
  }
  const float inv_cols = 1.0f / (float)cols;
  V slot[PF][VPT];
  auto load_row = [&](V (&dst)[VPT], int64_t r) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int v = j * T_ + tid;
      if (r < rows && v < nvec) dst[j] = ld_stream(x + r * xs + (int64_t)v * N);
      else dst[j].u = make_uint4(0, 0, 0, 0);
    }
  };
#pragma unroll
  for (int q = 0; q < PF; ++q) load_row(slot[q], blockIdx.x + q * G);
  int parity = 0;
  for (int64_t base = blockIdx.x; base < rows; base += PF * G) {
#pragma unroll
    for (int q = 0; q < PF; ++q) {
      const int64_t r = base + q * G;
      if (r >= rows) break;
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < VPT; ++j)
#pragma unroll
        for (int e = 0; e < N; ++e) {
          float f = Elt<T>::to_f(slot[q][j].e[e]);
          ss = fmaf(f, f, ss);
        }
      const float tot = block_sum(ss, red[parity], nwarps);
      parity ^= 1;
      const float rs = rsqrtf(tot * inv_cols + eps);
      if (tid == 0) rstd[r] = rs;
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        int v = j * T_ + tid;
        if (v < nvec) {
          V o;
#pragma unroll
          for (int e = 0; e < N; ++e)
            o.e[e] = Elt<T>::from_f(Elt<T>::to_f(slot[q][j].e[e]) * rs * wr[j][e]);
          st_stream(y + r * ys + (int64_t)v * N, o);
        }
      }
      load_row(slot[q], r + PF * G);
    }
  }
}

// ------------------------------------------------------------------ backward (regs) ---
template <typename T, typename W, int VPT, int PF>
__global__ void __launch_bounds__(512) rmsnorm_bwd_reg(const T* __restrict__ dy,
                                                        const T* __restrict__ x,
                                                        const void* __restrict__ w,
                                                        const float* __restrict__ rstd,
                                                        T* __restrict__ dx,
                                                        float* __restrict__ part, int64_t rows,
                                                        int cols) {
  using V = Vec16<T>;
  constexpr int N = V::N;
  __shared__ float red[2][32];
  const int T_ = blockDim.x, tid = threadIdx.x, nwarps = T_ >> 5;
  const int nvec = cols / N;
  const int64_t G = gridDim.x;
  float wr[VPT][N], acc[VPT][N];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    int v = j * T_ + tid;
#pragma unroll
    for (int e = 0; e < N; ++e) {
      wr[j][e] = (v < nvec) ? load_w<W>(w, (int64_t)v * N + e) : 0.f;
      acc[j][e] = 0.f;
    }
  }
  const float inv_cols = 1.0f / (float)cols;
  V sdy[PF][VPT], sx[PF][VPT];
  auto load_row = [&](V (&ddy)[VPT], V (&dxx)[VPT], int64_t r) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int v = j * T_ + tid;
      if (r < rows && v < nvec) {
        ddy[j] = ld_stream(dy + r * cols + (int64_t)v * N);
        dxx[j] = ld_stream(x + r * cols + (int64_t)v * N);
      } else {
        ddy[j].u = make_uint4(0, 0, 0, 0);
        dxx[j].u = make_uint4(0, 0, 0, 0);
      }
    }
  };
#pragma unroll
  for (int q = 0; q < PF; ++q) load_row(sdy[q], sx[q], blockIdx.x + q * G);
  int parity = 0;
  for (int64_t base = blockIdx.x; base < rows; base += PF * G) {
#pragma unroll
    for (int q = 0; q < PF; ++q) {
      const int64_t r = base + q * G;
      if (r >= rows) break;
      const float rs = __ldg(rstd + r);
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < VPT; ++j)
#pragma unroll
        for (int e = 0; e < N; ++e) {
          float d = Elt<T>::to_f(sdy[q][j].e[e]), xv = Elt<T>::to_f(sx[q][j].e[e]);
          dot = fmaf(wr[j][e] * d, xv, dot);
          acc[j][e] = fmaf(d * xv, rs, acc[j][e]);
        }
      const float tot = block_sum(dot, red[parity], nwarps);
      parity ^= 1;
      const float c2 = rs * rs * rs * (tot * inv_cols);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        int v = j * T_ + tid;
        if (v < nvec) {
          V o;
#pragma unroll
          for (int e = 0; e < N; ++e) {
            float d = Elt<T>::to_f(sdy[q][j].e[e]), xv = Elt<T>::to_f(sx[q][j].e[e]);
            o.e[e] = Elt<T>::from_f(rs * (wr[j][e] * d) - xv * c2);
          }
          st_stream(dx + r * cols + (int64_t)v * N, o);
        }
      }
      load_row(sdy[q], sx[q], r + PF * G);
    }
  }
  float* prow = part + (int64_t)blockIdx.x * cols;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    int v = j * T_ + tid;
    if (v < nvec) {
#pragma unroll
      for (int e = 0; e < N; e += 4)
        *reinterpret_cast<float4*>(prow + (int64_t)v * N + e) =
            make_float4(acc[j][e], acc[j][e + 1], acc[j][e + 2], acc[j][e + 3]);
    }
  }
}

// ------------------------------------------------------------------ TMA ring path -----
// Rows are staged through a ring of shared-memory buffers filled by cp.async.bulk (one
// mbarrier per stage), so a CTA keeps up to a ring's worth of rows of HBM reads in flight
// without spending registers on them.  Each thread copies its packets out of the stage
// into registers before the block reduction; the reduction's __syncthreads therefore
// also frees the stage, and thread 0 immediately refills it with the row a ring ahead.
// A wait that does not complete within the bound poisons the rest of the CTA's rows
// with NaN instead of spinning.
constexpr int kRingThreads = 256;
// Ring depths measured on B200 at [16384, 4096] and [16384, 8192] bf16: the forward is
// fastest with 2 rows per CTA (5.6 / 5.9 TB/s; 4 rows: 5.1 / 5.5, 6 rows: 5.1 / 5.4,
// register-capping for 6-8 CTAs per SM: slower), the backward with 3-4 row pairs.
constexpr int kRingStages = 3;  // backward: rows of (dy, x) per CTA
constexpr int kFwdStages = 2;   // forward: rows of x per CTA

template <typename T>
__device__ __forceinline__ void ring_issue(unsigned char* stage, uint64_t* bar, const T* src0,
                                           const T* src1, uint32_t row_bytes) {
  ptx::fence_proxy_async_smem();
  ptx::mbar_arrive_expect_tx(bar, src1 ? 2 * row_bytes : row_bytes);
  ptx::bulk_g2s(stage, src0, row_bytes, bar);
  if (src1) ptx::bulk_g2s(stage + row_bytes, src1, row_bytes, bar);
}

template <typename T, typename W, int VPT>
__global__ void __launch_bounds__(kRingThreads) rmsnorm_fwd_ring(
    const T* __restrict__ x, int64_t xs, const void* __restrict__ w, T* __restrict__ y,
    int64_t ys, float* __restrict__ rstd, int64_t rows, int cols, float eps) {
  using V = Vec16<T>;
  constexpr int N = V::N;
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ __align__(8) uint64_t full[kFwdStages];
  __shared__ float red[2][32];
  __shared__ int dead;
  const int tid = threadIdx.x;
  const int nvec = cols / N;
  const uint32_t row_bytes = (uint32_t)cols * sizeof(T);
  const int64_t G = gridDim.x;
  float wr[VPT][N];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    int v = j * kRingThreads + tid;
#pragma unroll
    for (int e = 0; e < N; ++e) wr[j][e] = (v < nvec) ? load_w<W>(w, (int64_t)v * N + e) : 0.f;
  }
  if (tid == 0) {
    for (int q = 0; q < kFwdStages; ++q) ptx::mbar_init(&full[q], 1);
    ptx::fence_mbar_init();
    dead = 0;
  }
  __syncthreads();
  if (tid == 0)
    for (int q = 0; q < kFwdStages; ++q) {
      const int64_t r = blockIdx.x + q * G;
      if (r < rows) ring_issue<T>(ring + (size_t)q * row_bytes, &full[q], x + r * xs, (const T*)nullptr, row_bytes);
    }
  const float inv_cols = 1.0f / (float)cols;
  int i = 0;
  for (int64_t r = blockIdx.x; r < rows; r += G, ++i) {
    const int q = i % kFwdStages;
    const bool ok = !dead && ptx::mbar_wait(&full[q], (uint32_t)((i / kFwdStages) & 1));
    const V* sv = reinterpret_cast<const V*>(ring + (size_t)q * row_bytes);
    V cur[VPT];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int v = j * kRingThreads + tid;
      if (v < nvec) cur[j] = sv[v];
      else cur[j].u = make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int e = 0; e < N; ++e) {
        float f = Elt<T>::to_f(cur[j].e[e]);
        ss = fmaf(f, f, ss);
      }
    }
    const float tot = block_sum(ss, red[i & 1], kRingThreads / 32);  // also frees stage q
    if (tid == 0) {
      if (!ok) dead = 1;
      const int64_t rn = r + kFwdStages * G;
      if (!dead && rn < rows)
        ring_issue<T>(ring + (size_t)q * row_bytes, &full[q], x + rn * xs, (const T*)nullptr, row_bytes);
    }
    const float rs = ok ? rsqrtf(tot * inv_cols + eps) : __int_as_float(0x7fc00000);
    if (tid == 0) rstd[r] = rs;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int v = j * kRingThreads + tid;
      if (v < nvec) {
        V o;
#pragma unroll
        for (int e = 0; e < N; ++e) o.e[e] = Elt<T>::from_f(Elt<T>::to_f(cur[j].e[e]) * rs * wr[j][e]);
        st_stream(y + r * ys + (int64_t)v * N, o);
      }
    }
  }
}

// Forward, warp rings: every warp owns kWarpStages shared-memory row buffers filled by
// cp.async.bulk (one mbarrier each) and walks its own rows, reducing the sum of squares
// with shuffles, so no row waits on a CTA-wide barrier.  x is read twice from shared
// memory (sum of squares, then the scaled output), which keeps the registers independent
// of the row length; the weight row sits in shared memory (fp32) for the whole kernel.
constexpr int kWarpStages = 3;

template <typename T, typename W>
__global__ void __launch_bounds__(256) rmsnorm_fwd_warp(
    const T* __restrict__ x, int64_t xs, const void* __restrict__ w, T* __restrict__ y,
    int64_t ys, float* __restrict__ rstd, int64_t rows, int cols, float eps) {
  using V = Vec16<T>;
  constexpr int N = V::N;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[8][kWarpStages];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int nvec = cols / N;
  const uint32_t row_bytes = (uint32_t)cols * sizeof(T);
  float* wsm = reinterpret_cast<float*>(smem);  // [cols] fp32, then the warps' stages
  unsigned char* stages = smem + (((size_t)cols * 4 + 127) / 128) * 128 +
                          (size_t)warp * kWarpStages * row_bytes;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) wsm[c] = load_w<W>(w, c);
  if (lane == 0) {
    for (int q = 0; q < kWarpStages; ++q) ptx::mbar_init(&full[warp][q], 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  const int64_t G = (int64_t)gridDim.x * nwarps;  // warps in the grid
  const int64_t first = (int64_t)blockIdx.x * nwarps + warp;
  if (lane == 0)
    for (int q = 0; q < kWarpStages; ++q) {
      const int64_t r = first + q * G;
      if (r < rows)
        ring_issue<T>(stages + (size_t)q * row_bytes, &full[warp][q], x + r * xs,
                      (const T*)nullptr, row_bytes);
    }
  const float inv_cols = 1.0f / (float)cols;
  bool dead = false;
  int i = 0;
  for (int64_t r = first; r < rows; r += G, ++i) {
    const int q = i % kWarpStages;
    const bool ok = !dead && ptx::mbar_wait(&full[warp][q], (uint32_t)((i / kWarpStages) & 1));
    const V* sv = reinterpret_cast<const V*>(stages + (size_t)q * row_bytes);
    float ss = 0.f;
#pragma unroll 4
    for (int v = lane; v < nvec; v += 32) {
      const V p = sv[v];
#pragma unroll
      for (int e = 0; e < N; ++e) {
        const float f = Elt<T>::to_f(p.e[e]);
        ss = fmaf(f, f, ss);
      }
    }
    ss = warp_sum(ss);
    const float rs = ok ? rsqrtf(ss * inv_cols + eps) : __int_as_float(0x7fc00000);
    if (lane == 0) rstd[r] = rs;
#pragma unroll 4
    for (int v = lane; v < nvec; v += 32) {
      const V p = sv[v];
      const float4* wp = reinterpret_cast<const float4*>(wsm + (size_t)v * N);
      float wv[N];
#pragma unroll
      for (int e4 = 0; e4 < N / 4; ++e4) {
        const float4 t4 = wp[e4];
        wv[4 * e4] = t4.x;
        wv[4 * e4 + 1] = t4.y;
        wv[4 * e4 + 2] = t4.z;
        wv[4 * e4 + 3] = t4.w;
      }
      V o;
#pragma unroll
      for (int e = 0; e < N; ++e) o.e[e] = Elt<T>::from_f(Elt<T>::to_f(p.e[e]) * rs * wv[e]);
      st_stream(y + r * ys + (int64_t)v * N, o);
    }
    __syncwarp();  // every lane is done with stage q
    if (!ok) dead = true;
    if (lane == 0) {
      const int64_t rn = r + kWarpStages * G;
      if (!dead && rn < rows)
        ring_issue<T>(stages + (size_t)q * row_bytes, &full[warp][q], x + rn * xs,
                      (const T*)nullptr, row_bytes);
    }
  }
}

template <typename T, typename W, int VPT>
__global__ void __launch_bounds__(kRingThreads) rmsnorm_bwd_ring(
    const T* __restrict__ dy, const T* __restrict__ x, const void* __restrict__ w,
    const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ part, int64_t rows,
    int cols) {
  using V = Vec16<T>;
  constexpr int N = V::N;
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ __align__(8) uint64_t full[kRingStages];
  __shared__ float red[2][32];
  __shared__ int dead;
  const int tid = threadIdx.x;
  const int nvec = cols / N;
  const uint32_t row_bytes = (uint32_t)cols * sizeof(T);
  const size_t stage_bytes = 2 * (size_t)row_bytes;
  const int64_t G = gridDim.x;
  float wr[VPT][N], acc[VPT][N];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    int v = j * kRingThreads + tid;
#pragma unroll
    for (int e = 0; e < N; ++e) {
      wr[j][e] = (v < nvec) ? load_w<W>(w, (int64_t)v * N + e) : 0.f;
      acc[j][e] = 0.f;
    }
  }
  if (tid == 0) {
    for (int q = 0; q < kRingStages; ++q) ptx::mbar_init(&full[q], 1);
    ptx::fence_mbar_init();
    dead = 0;
  }
  __syncthreads();
  if (tid == 0)
    for (int q = 0; q < kRingStages; ++q) {
      const int64_t r = blockIdx.x + q * G;
      if (r < rows)
        ring_issue<T>(ring + q * stage_bytes, &full[q], dy + r * cols, x + r * cols, row_bytes);
    }
  const float inv_cols = 1.0f / (float)cols;
  int i = 0;
  for (int64_t r = blockIdx.x; r < rows; r += G, ++i) {
    const int q = i % kRingStages;
    const bool ok = !dead && ptx::mbar_wait(&full[q], (uint32_t)((i / kRingStages) & 1));
    const V* sdy = reinterpret_cast<const V*>(ring + q * stage_bytes);
    const V* sx = reinterpret_cast<const V*>(ring + q * stage_bytes + row_bytes);
    const float rs = __ldg(rstd + r);
    V cdy[VPT], cx[VPT];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int v = j * kRingThreads + tid;
      if (v < nvec) {
        cdy[j] = sdy[v];
        cx[j] = sx[v];
      } else {
        cdy[j].u = make_uint4(0, 0, 0, 0);
        cx[j].u = make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int e = 0; e < N; ++e) {
        float d = Elt<T>::to_f(cdy[j].e[e]), xv = Elt<T>::to_f(cx[j].e[e]);
        dot = fmaf(wr[j][e] * d, xv, dot);
        acc[j][e] = fmaf(d * xv, rs, acc[j][e]);
      }
    }
    const float tot = block_sum(dot, red[i & 1], kRingThreads / 32);  // also frees stage q
    if (tid == 0) {
      if (!ok) dead = 1;
      const int64_t rn = r + kRingStages * G;
      if (!dead && rn < rows)
        ring_issue<T>(ring + q * stage_bytes, &full[q], dy + rn * cols, x + rn * cols, row_bytes);
    }
    const float c2 = ok ? rs * rs * rs * (tot * inv_cols) : __int_as_float(0x7fc00000);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int v = j * kRingThreads + tid;
      if (v < nvec) {
        V o;
#pragma unroll
        for (int e = 0; e < N; ++e) {
          float d = Elt<T>::to_f(cdy[j].e[e]), xv = Elt<T>::to_f(cx[j].e[e]);
          o.e[e] = Elt<T>::from_f(rs * (wr[j][e] * d) - xv * c2);
        }
        st_stream(dx + r * cols + (int64_t)v * N, o);
      }
    }
  }
  float* prow = part + (int64_t)blockIdx.x * cols;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    int v = j * kRingThreads + tid;
    if (v < nvec) {
#pragma unroll
      for (int e = 0; e < N; e += 4)
        *reinterpret_cast<float4*>(prow + (int64_t)v * N + e) =
            make_float4(acc[j][e], acc[j][e + 1], acc[j][e + 2], acc[j][e + 3]);
    }
  }
}

// ------------------------------------------------------------------ generic path ------
template <typename T, typename W>
__global__ void rmsnorm_fwd_generic(const T* __restrict__ x, int64_t xs, const void* __restrict__ w,
                                    T* __restrict__ y, int64_t ys, float* __restrict__ rstd,
                                    int64_t rows, int64_t cols, float eps) {
  __shared__ float red[2][32];
  const int nwarps = blockDim.x >> 5;
  int parity = 0;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x, parity ^= 1) {
    const T* xr = x + r * xs;
    float ss = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      float f = Elt<T>::to_f(xr[c]);
      ss = fmaf(f, f, ss);
    }
    float rs = rsqrtf(block_sum(ss, red[parity], nwarps) / (float)cols + eps);
    if (threadIdx.x == 0) rstd[r] = rs;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
      y[r * ys + c] = Elt<T>::from_f(Elt<T>::to_f(xr[c]) * rs * load_w<W>(w, c));
  }
}

template <typename T, typename W>
__global__ void rmsnorm_bwd_generic(const T* __restrict__ dy, const T* __restrict__ x,
                                    const void* __restrict__ w, const float* __restrict__ rstd,
                                    T* __restrict__ dx, float* __restrict__ part, int64_t rows,
                                    int64_t cols) {
  __shared__ float red[2][32];
  const int nwarps = blockDim.x >> 5;
  float* prow = part + (int64_t)blockIdx.x * cols;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) prow[c] = 0.f;
  int parity = 0;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x, parity ^= 1) {
    const T* dyr = dy + r * cols;
    const T* xr = x + r * cols;
    const float rs = rstd[r];
    float dot = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      float d = Elt<T>::to_f(dyr[c]), xv = Elt<T>::to_f(xr[c]);
      dot = fmaf(load_w<W>(w, c) * d, xv, dot);
      prow[c] = fmaf(d * xv, rs, prow[c]);  // each column owned by one thread
    }
    const float c2 = rs * rs * rs * (block_sum(dot, red[parity], nwarps) / (float)cols);
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      float d = Elt<T>::to_f(dyr[c]), xv = Elt<T>::to_f(xr[c]);
      dx[r * cols + c] = Elt<T>::from_f(rs * (load_w<W>(w, c) * d) - xv * c2);
    }
  }
}

// dw[c] = sum_{g < G} part[g][c] in a fixed order, then cast to W.  One CTA of 32 warps
// per 32 columns: warp w sums partial rows w, w+32, ... (all loads in flight), the 32
// warp sums are added in warp order.
template <typename W>
__global__ void __launch_bounds__(1024) rmsnorm_dw_reduce(const float* __restrict__ part, int G,
                                                          int64_t cols, W* __restrict__ dw) {
  __shared__ float red[32][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  float s = 0.f;
  if (c < cols) {
#pragma unroll 8
    for (int g = warp; g < G; g += 32) s += part[(int64_t)g * cols + c];
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && c < cols) {
    float t = 0.f;
    for (int w = 0; w < 32; ++w) t += red[w][lane];
    dw[c] = Elt<W>::from_f(t);
  }
}

// ------------------------------------------------------------------ launch planning ---
struct Plan {
  bool reg;     // register path usable
  int threads;  // CTA size
  int vpt;      // packets per thread (register path)
};

// Register path: 16-byte aligned rows with cols a multiple of the packet width and at
// most kMaxVpt packets per thread (4 forward, 2 backward, so nothing spills at the
// 128-register budget a 512-thread CTA allows).
inline Plan plan_rows(int64_t cols, int esize, bool aligned, bool bwd) {
  Plan p{false, 256, 0};
  const int per = 16 / esize;
  const int64_t nvec = cols / per;
  const int max_vpt = bwd ? 2 : 4;
  if (aligned && cols % per == 0 && nvec >= 1 && nvec <= 512 * max_vpt) {
    int64_t t = nvec < 512 ? ((nvec + 31) / 32) * 32 : 512;
    int64_t need = (nvec + t - 1) / t;
    int v = 1;
    while (v < need) v <<= 1;
    p.reg = true;
    p.threads = (int)t;
    p.vpt = v;
  }
  return p;
}

// Ring path: 16-byte aligned rows of at most 4 packets per thread (256 threads) and at
// most 16 KiB, so four stages of (dy, x) fit in 128 KiB.  Returns VPT or 0.
inline int ring_vpt(int64_t cols, int esize, bool aligned) {
  const int per = 16 / esize;
  if (!aligned || cols % per != 0 || cols * esize > 16 * 1024) return 0;
  const int64_t nvec = cols / per;
  const int64_t need = (nvec + kRingThreads - 1) / kRingThreads;
  if (need <= 1) return 1;
  if (need <= 2) return 2;
  if (need <= 4) return 4;
  return 0;
}

// Persistent grid: resident CTAs per SM (occupancy of the actual kernel, capped at 8)
// times the SM count, never more than rows.  kMaxGridPerSm bounds the workspace.
constexpr int kMaxGridPerSm = 8;
template <typename K>
inline int persistent_grid(K kernel, int threads, int64_t rows, int smem = 0) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  if (per_sm > kMaxGridPerSm) per_sm = kMaxGridPerSm;
  int64_t g = (int64_t)num_sms() * per_sm;
  if (g > rows) g = rows;
  return (int)(g < 1 ? 1 : g);
}

template <typename T, typename W>
int fwd_t(const void* x, int64_t xs, const void* w, void* y, int64_t ys, float* rstd,
          int64_t rows, int64_t cols, float eps, cudaStream_t s) {
  const bool al = aligned16(x) && aligned16(y) && (xs * (int64_t)sizeof(T)) % 16 == 0 &&
                  (ys * (int64_t)sizeof(T)) % 16 == 0;
  Plan p = plan_rows(cols, sizeof(T), al, false);
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  const int rv = ring_vpt(cols, sizeof(T), al);
  if (rv > 0 && cols * (int64_t)sizeof(T) <= 4096) {
    // Rows of at most 4 KB: warp rings (measured on B200: 1.4x the CTA ring at 2 KB rows,
    // 1.04x at 4 KB; the CTA ring wins from 8 KB rows on, where a warp's row takes too
    // long at 8 warps per SM).  8 warps x kWarpStages rows + the fp32 weight row.
    const int wbytes = (int)(((cols * 4 + 127) / 128) * 128);
    const int nw = 8;
    const int smem = wbytes + nw * kWarpStages * (int)(cols * sizeof(T));
    auto k = rmsnorm_fwd_warp<T, W>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k<<<persistent_grid(k, nw * 32, rows, smem), nw * 32, smem, s>>>(xp, xs, w, yp, ys, rstd,
                                                                     rows, (int)cols, eps);
  } else if (rv > 0) {
    const int smem = kFwdStages * (int)(cols * sizeof(T));
    switch (rv) {
#define FK_CASE(V)                                                                      \
  case V: {                                                                             \
    auto k = rmsnorm_fwd_ring<T, W, V>;                                                 \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);          \
    k<<<persistent_grid(k, kRingThreads, rows, smem), kRingThreads, smem, s>>>(         \
        xp, xs, w, yp, ys, rstd, rows, (int)cols, eps);                                  \
    break;                                                                              \
  }
      FK_CASE(1) FK_CASE(2) FK_CASE(4)
#undef FK_CASE
    }
  } else if (p.reg) {
    switch (p.vpt) {
#define FK_CASE(V)                                                                       \
  case V: {                                                                              \
    auto k = rmsnorm_fwd_reg<T, W, V, (V == 1 ? 4 : 2)>;                                                   \
    k<<<persistent_grid(k, p.threads, rows), p.threads, 0, s>>>(xp, xs, w, yp, ys, rstd, \
                                                                rows, (int)cols, eps);   \
    break;                                                                               \
  }
      FK_CASE(1) FK_CASE(2) FK_CASE(4)
#undef FK_CASE
    }
  } else {
    auto k = rmsnorm_fwd_generic<T, W>;
    k<<<persistent_grid(k, 256, rows), 256, 0, s>>>(xp, xs, w, yp, ys, rstd, rows, cols, eps);
  }
  return launch_status("fk_rmsnorm_fwd");
}

template <typename T, typename W>
int bwd_t(const void* dy, const void* x, const void* w, const float* rstd, void* dx, void* dw,
          float* part, int64_t rows, int64_t cols, cudaStream_t s) {
  const bool al = aligned16(dy) && aligned16(x) && aligned16(dx);
  Plan p = plan_rows(cols, sizeof(T), al, true);
  const T* dyp = static_cast<const T*>(dy);
  const T* xp = static_cast<const T*>(x);
  T* dxp = static_cast<T*>(dx);
  int grid = 1;
  const int rv = ring_vpt(cols, sizeof(T), al);
  if (rv > 0) {
    const int smem = kRingStages * 2 * (int)(cols * sizeof(T));
    switch (rv) {
#define FK_CASE(V)                                                                      \
  case V: {                                                                             \
    auto k = rmsnorm_bwd_ring<T, W, V>;                                                 \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);          \
    grid = persistent_grid(k, kRingThreads, rows, smem);                                \
    k<<<grid, kRingThreads, smem, s>>>(dyp, xp, w, rstd, dxp, part, rows, (int)cols);     \
    break;                                                                              \
  }
      FK_CASE(1) FK_CASE(2) FK_CASE(4)
#undef FK_CASE
    }
  } else if (p.reg) {
    switch (p.vpt) {
#define FK_CASE(V)                                                                      \
  case V: {                                                                             \
    auto k = rmsnorm_bwd_reg<T, W, V, (V == 1 ? 3 : 2)>;                                                  \
    grid = persistent_grid(k, p.threads, rows);                                         \
    k<<<grid, p.threads, 0, s>>>(dyp, xp, w, rstd, dxp, part, rows, (int)cols);         \
    break;                                                                              \
  }
      FK_CASE(1) FK_CASE(2)
#undef FK_CASE
    }
  } else {
    auto k = rmsnorm_bwd_generic<T, W>;
    grid = persistent_grid(k, 256, rows);
    k<<<grid, 256, 0, s>>>(dyp, xp, w, rstd, dxp, part, rows, cols);
  }
  int st = launch_status("fk_rmsnorm_bwd");
  if (st != FK_OK) return st;
  const int rgrid = (int)((cols + 31) / 32);
  rmsnorm_dw_reduce<W><<<rgrid, 1024, 0, s>>>(part, grid, cols, static_cast<W*>(dw));
  return launch_status("fk_rmsnorm_bwd(dw reduce)");
}

}  // namespace

// Upper bound of the backward grid (one fp32 partial row per CTA), valid for every
// dtype and path: min(rows, SMs * kMaxGridPerSm) rows of cols floats.
size_t rmsnorm_bwd_ws_bytes(int64_t rows, int64_t cols) {
  int64_t g = (int64_t)num_sms() * kMaxGridPerSm;
  if (g > rows) g = rows;
  return (size_t)g * (size_t)cols * sizeof(float);
}

}  // namespace fk

#define FK_DISPATCH_W(wd, ...)                                          \
  switch (wd) {                                                         \
    case FK_F32: { using wt = float; __VA_ARGS__; break; }              \
    case FK_F16: { using wt = __half; __VA_ARGS__; break; }             \
    case FK_BF16: { using wt = __nv_bfloat16; __VA_ARGS__; break; }     \
    default: return ::fk::fail(FK_ERR_INVALID_ARG, "bad weight dtype %d", (int)(wd)); \
  }

extern "C" int fk_rmsnorm_fwd(const void* x, int64_t x_row_stride, const void* weight,
                              int w_dtype, void* y, int64_t y_row_stride, float* rstd,
                              int64_t rows, int64_t cols, float eps, int dtype, void* stream) {
  FK_CHECK_ARG(rows >= 0 && cols >= 0, "fk_rmsnorm_fwd: negative shape");
  if (rows == 0) return FK_OK;
  FK_CHECK_ARG(cols > 0, "fk_rmsnorm_fwd: cols == 0");
  FK_CHECK_ARG(x && weight && y && rstd, "fk_rmsnorm_fwd: null pointer");
  FK_CHECK_ARG(x_row_stride >= cols && y_row_stride >= cols, "fk_rmsnorm_fwd: row stride < cols");
  FK_DISPATCH_DTYPE(dtype, FK_DISPATCH_W(w_dtype, return fk::fwd_t<scalar_t, wt>(
                                                      x, x_row_stride, weight, y, y_row_stride,
                                                      rstd, rows, cols, eps,
                                                      fk::as_stream(stream))));
  return FK_OK;
}

extern "C" int fk_rmsnorm_bwd_workspace_size(int64_t rows, int64_t cols, size_t* bytes) {
  FK_CHECK_ARG(bytes != nullptr, "fk_rmsnorm_bwd_workspace_size: null output");
  FK_CHECK_ARG(rows >= 0 && cols >= 0, "fk_rmsnorm_bwd_workspace_size: negative shape");
  *bytes = (rows == 0 || cols == 0) ? 0 : fk::rmsnorm_bwd_ws_bytes(rows, cols);
  return FK_OK;
}

extern "C" int fk_rmsnorm_bwd(const void* dy, const void* x, const void* weight, int w_dtype,
                              const float* rstd, void* dx, void* dw, void* workspace,
                              size_t workspace_bytes, int64_t rows, int64_t cols, int dtype,
                              void* stream) {
  FK_CHECK_ARG(rows >= 0 && cols >= 0, "fk_rmsnorm_bwd: negative shape");
  if (cols == 0) return FK_OK;
  FK_CHECK_ARG(dw && weight, "fk_rmsnorm_bwd: null pointer");
  if (rows == 0) {
    // Empty batch: dw is all zeros.
    cudaMemsetAsync(dw, 0, (size_t)cols * fk::dtype_size(w_dtype), fk::as_stream(stream));
    return fk::launch_status("fk_rmsnorm_bwd(zero dw)");
  }
  FK_CHECK_ARG(dy && x && rstd && dx, "fk_rmsnorm_bwd: null pointer");
  size_t need = fk::rmsnorm_bwd_ws_bytes(rows, cols);
  if (workspace == nullptr || workspace_bytes < need || !fk::aligned16(workspace))
    return fk::fail(FK_ERR_WORKSPACE, "fk_rmsnorm_bwd: need %zu aligned workspace bytes, got %zu",
                    need, workspace_bytes);
  FK_DISPATCH_DTYPE(dtype, FK_DISPATCH_W(w_dtype, return fk::bwd_t<scalar_t, wt>(
                                                      dy, x, weight, rstd, dx, dw,
                                                      static_cast<float*>(workspace), rows, cols,
                                                      fk::as_stream(stream))));
  return FK_OK;
}

// ------------------------------------------------------------------ fixed-scratch variant
// fk_rmsnorm_bwd_noalloc: the same backward for callers that cannot allocate device memory
// -- code that only receives the tensors of another framework's memory pool, runs under a
// pre-planned memory budget, or executes where allocation calls are not allowed -- and so
// cannot hand fk_rmsnorm_bwd its workspace.  The per-CTA weight-gradient partials live in
// a fixed file-scope device array instead (kNoAllocScratchBytes, held by every GPU that
// loads the library until the process exits).
namespace fk {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
constexpr int64_t kNoAllocScratchFloats = (int64_t)(kNoAllocScratchBytes / sizeof(float));
static __device__ __align__(256) float g_rmsnorm_scratch[kNoAllocScratchFloats];

// Device address of g_rmsnorm_scratch for the current device, looked up once per device
// (host code cannot use the symbol itself: on the host it names a stand-in object).
int scratch_address(float** out) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64)
    return fail(FK_ERR_NO_DEVICE, "fk_rmsnorm_bwd_noalloc: no current device (%s)",
                cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rmsnorm_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(FK_ERR_NO_DEVICE, "fk_rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed (%s)",
                  cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return FK_OK;
}

// Same kernels and launch plan as bwd_t, with the grid (= number of partial rows) capped
// so the partials fit the fixed scratch.
template <typename T, typename W>
int bwd_noalloc_t(const void* dy, const void* x, const void* w, const float* rstd, void* dx,
                  void* dw, float* part, int64_t max_grid, int64_t rows, int64_t cols,
                  cudaStream_t s) {
  const bool al = aligned16(dy) && aligned16(x) && aligned16(dx);
  Plan p = plan_rows(cols, sizeof(T), al, true);
  const T* dyp = static_cast<const T*>(dy);
  const T* xp = static_cast<const T*>(x);
  T* dxp = static_cast<T*>(dx);
  auto cap = [&](int g) { return (int)((int64_t)g < max_grid ? g : max_grid); };
  int grid = 1;
  const int rv = ring_vpt(cols, sizeof(T), al);
  if (rv > 0) {
    const int smem = kRingStages * 2 * (int)(cols * sizeof(T));
    switch (rv) {
#define FK_CASE(V)                                                                      \
  case V: {                                                                             \
    auto k = rmsnorm_bwd_ring<T, W, V>;                                                 \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);          \
    grid = cap(persistent_grid(k, kRingThreads, rows, smem));                           \
    k<<<grid, kRingThreads, smem, s>>>(dyp, xp, w, rstd, dxp, part, rows, (int)cols);     \
    break;                                                                              \
  }
      FK_CASE(1) FK_CASE(2) FK_CASE(4)
#undef FK_CASE
    }
  } else if (p.reg) {
    switch (p.vpt) {
#define FK_CASE(V)                                                                      \
  case V: {                                                                             \
    auto k = rmsnorm_bwd_reg<T, W, V, (V == 1 ? 3 : 2)>;                                \
    grid = cap(persistent_grid(k, p.threads, rows));                                    \
    k<<<grid, p.threads, 0, s>>>(dyp, xp, w, rstd, dxp, part, rows, (int)cols);         \
    break;                                                                              \
  }
      FK_CASE(1) FK_CASE(2)
#undef FK_CASE
    }
  } else {
    auto k = rmsnorm_bwd_generic<T, W>;
    grid = cap(persistent_grid(k, 256, rows));
    k<<<grid, 256, 0, s>>>(dyp, xp, w, rstd, dxp, part, rows, cols);
  }
  int st = launch_status("fk_rmsnorm_bwd_noalloc");
  if (st != FK_OK) return st;
  const int rgrid = (int)((cols + 31) / 32);
  rmsnorm_dw_reduce<W><<<rgrid, 1024, 0, s>>>(part, grid, cols, static_cast<W*>(dw));
  return launch_status("fk_rmsnorm_bwd_noalloc(dw reduce)");
}

}  // namespace
}  // namespace fk

extern "C" int fk_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* weight,
                                      int w_dtype, const float* rstd, void* dx, void* dw,
                                      int64_t rows, int64_t cols, int dtype, void* stream) {
  FK_CHECK_ARG(rows >= 0 && cols >= 0, "fk_rmsnorm_bwd_noalloc: negative shape");
  if (cols == 0) return FK_OK;
  FK_CHECK_ARG(dw && weight, "fk_rmsnorm_bwd_noalloc: null pointer");
  if (cols > fk::kNoAllocScratchFloats)
    return fk::fail(FK_ERR_UNSUPPORTED,
                    "fk_rmsnorm_bwd_noalloc: cols=%lld exceeds the fixed scratch (at most %lld "
                    "columns: one fp32 partial row of 8 MiB); use fk_rmsnorm_bwd with a workspace",
                    (long long)cols, (long long)fk::kNoAllocScratchFloats);
  if (rows == 0) {
    cudaMemsetAsync(dw, 0, (size_t)cols * fk::dtype_size(w_dtype), fk::as_stream(stream));
    return fk::launch_status("fk_rmsnorm_bwd_noalloc(zero dw)");
  }
  FK_CHECK_ARG(dy && x && rstd && dx, "fk_rmsnorm_bwd_noalloc: null pointer");
  float* part = nullptr;
  int st = fk::scratch_address(&part);
  if (st != FK_OK) return st;
  const int64_t max_grid = fk::kNoAllocScratchFloats / cols;  // partial rows that fit
  FK_DISPATCH_DTYPE(dtype, FK_DISPATCH_W(w_dtype, return fk::bwd_noalloc_t<scalar_t, wt>(
                                                      dy, x, weight, rstd, dx, dw, part, max_grid,
                                                      rows, cols, fk::as_stream(stream))));
  return FK_OK;
}
