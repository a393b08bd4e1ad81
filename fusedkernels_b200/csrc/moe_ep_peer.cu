// Expert-parallel token exchange over NVLink peer memory (one process per GPU).
//
// Every rank owns one exchange region (cudaMalloc'd, exported with CUDA IPC and mapped
// into every other rank of the node) holding, for T tokens per rank and N ranks:
//   to_expert [N*T, dim]   rows sent to this rank's experts, row s*T + pos from rank s
//   meta_e    [N*T, k]     local expert id per slot (-1: slot not on this rank)
//   meta_w    [N*T, k]     routing weight per slot
//   to_source [N*T, dim]   partial rows returned by the expert ranks, row d*T + pos from d
//   dw        [N*T, k]     routing-weight gradients returned by the expert ranks
//   flags     [4, N]       per phase, how many times each rank has published into it
// The layout is the fixed-capacity all-to-all layout of fk_ep_plan / fk_ep_unpack_*, so
// those kernels are shared with the NCCL transport; only rows that carry a token cross
// NVLink, and the packing of a row and its transfer are one kernel.
//
// A put kernel stores its rows straight into the peers' regions (16-byte stores), then
// every thread fences at system scope, the CTAs count themselves on a local ticket and
// the last one publishes: it bumps its per-phase sequence number and stores it with
// release semantics into flags[phase][me] of every rank.  fk_ep_peer_wait (one small
// CTA) spins with acquire loads until all N flags of a phase reach the next expected
// sequence number, which it keeps in device memory (so a CUDA graph of the step can be
// replayed).  The wait is bounded by wall clock (the caller's limit); on timeout it
// records an error and returns.
//
// Reuse of a region needs no extra barrier because every phase's data is consumed before
// the consumer publishes anything the producer waits for before its next write:
//   to_expert (forward rows, then backward rows): rank s writes into d's copy only after
//     it has received d's partial rows for the previous phase, which d sends after it has
//     gathered the rows it received;
//   to_source: rank d writes into s's copy only after receiving s's next rows, which s
//     sends after it has summed the partial rows of the previous phase.
#include "common.cuh"

#include <string.h>

namespace fk {
namespace {

constexpr int kPutThreads = 256;
constexpr int kPutBatch = 8;  // 16-byte packets per lane in flight in the row copy
constexpr int kCombineBatch = 4;  // packets per lane accumulated at a time in the combine

// ctl layout (uint32, local to each rank): [phase]       ticket of the put kernels
//                                          [8 + phase]   sequence numbers published
//                                          [16 + phase]  sequence numbers consumed
constexpr int kCtlSent = 8, kCtlSeen = 16;

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned ticket_add(unsigned* p) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p) : "memory");
  return old;
}

// End of a put kernel: make this CTA's peer stores visible, and let the last CTA publish.
__device__ __forceinline__ void publish(unsigned* ctl, unsigned* const* flag_bases, int phase,
                                        int n_ranks, int me) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (ticket_add(ctl + phase) == gridDim.x - 1) {
      __threadfence_system();
      const unsigned v = ctl[kCtlSent + phase] + 1u;
      ctl[kCtlSent + phase] = v;
      for (int d = 0; d < n_ranks; ++d) st_release_sys(flag_bases[d] + phase * n_ranks + me, v);
      ctl[phase] = 0u;  // every CTA has taken its ticket
    }
  }
}

// Rows r in [0, N*T): destination d = r / T, row pos = r % T of d's list.  The row of
// token send_token[r] (if any) goes to rows_d[(me*T + pos)], and with metadata the k slot
// entries go to meta_e_d / meta_w_d at the same row (every row: -1 slots past the count).
template <typename T_>
__global__ void __launch_bounds__(kPutThreads) ep_peer_put_rows_kernel(
    const T_* __restrict__ x, int dim, const int* __restrict__ send_token, int64_t T, int n_ranks,
    int me, const int* __restrict__ send_e, const float* __restrict__ send_w, int k,
    void* const* __restrict__ row_bases, void* const* __restrict__ e_bases,
    void* const* __restrict__ w_bases, unsigned* const* __restrict__ flag_bases, int phase,
    unsigned* ctl) {
  using V = Vec16<T_>;
  const int nvec = dim / V::N;
  const int64_t rows = (int64_t)n_ranks * T;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t r = warp; r < rows; r += nwarps) {
    const int d = (int)(r / T);
    const int64_t dst_row = (int64_t)me * T + (r - (int64_t)d * T);
    const int t = send_token[r];
    if (t >= 0) {
      const T_* src = x + (int64_t)t * dim;
      T_* dst = static_cast<T_*>(row_bases[d]) + dst_row * dim;
      // kPutBatch packets per lane are loaded before any is stored, so every lane keeps
      // that many loads in flight ahead of its NVLink stores.
      for (int v0 = 0; v0 < nvec; v0 += 32 * kPutBatch) {
        V buf[kPutBatch];
#pragma unroll
        for (int b = 0; b < kPutBatch; ++b) {
          const int v = v0 + b * 32 + lane;
          if (v < nvec) buf[b] = ld_keep(src + v * V::N);
        }
#pragma unroll
        for (int b = 0; b < kPutBatch; ++b) {
          const int v = v0 + b * 32 + lane;
          if (v < nvec) st_plain(dst + v * V::N, buf[b]);
        }
      }
    }
    if (send_e != nullptr) {
      for (int j = lane; j < k; j += 32) {
        static_cast<int*>(e_bases[d])[dst_row * k + j] = send_e[r * k + j];
        static_cast<float*>(w_bases[d])[dst_row * k + j] = send_w[r * k + j];
      }
    }
  }
  publish(ctl, flag_bases, phase, n_ranks, me);
}

// Expert side of the combine: received row j (source s = j / T, row pos = j % T of s's
// list) with at least one local slot: out = sum over local slots of w * y[slot row]
// (w = 1 when weights are null), stored at rows_s[me*T + pos]; with dw_rows, the row's k
// routing-gradient entries go to dw_s at the same row.
template <typename T_>
__global__ void __launch_bounds__(kPutThreads) ep_peer_combine_put_kernel(
    const T_* __restrict__ y, int dim, const int* __restrict__ slot_pos,
    const float* __restrict__ w, int64_t T, int n_ranks, int me, int k,
    const float* __restrict__ dw_rows, void* const* __restrict__ row_bases,
    void* const* __restrict__ dw_bases, unsigned* const* __restrict__ flag_bases, int phase,
    unsigned* ctl) {
  using V = Vec16<T_>;
  const int nvec = dim / V::N;
  const int64_t rows = (int64_t)n_ranks * T;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t j = warp; j < rows; j += nwarps) {
    bool any = false;
    for (int i = lane; i < k; i += 32) any |= slot_pos[j * k + i] >= 0;
    if (!__any_sync(0xffffffffu, any)) continue;
    const int s = (int)(j / T);
    const int64_t dst_row = (int64_t)me * T + (j - (int64_t)s * T);
    T_* dst = static_cast<T_*>(row_bases[s]) + dst_row * dim;
    if (k <= 32) {
      // Lane i holds slot i's row and weight; the local slots are walked in slot order
      // (the same summation order as below), kCombineBatch packets per lane at a time, so
      // every lane keeps that many loads in flight ahead of its NVLink stores.
      const int my_p = lane < k ? slot_pos[j * k + lane] : -1;
      const float my_w = (lane < k && w) ? w[j * k + lane] : 1.0f;
      const unsigned live = __ballot_sync(0xffffffffu, my_p >= 0);
      for (int v0 = 0; v0 < nvec; v0 += 32 * kCombineBatch) {
        float acc[kCombineBatch][V::N];
#pragma unroll
        for (int b = 0; b < kCombineBatch; ++b)
#pragma unroll
          for (int q = 0; q < V::N; ++q) acc[b][q] = 0.f;
        for (unsigned m = live; m != 0u; m &= m - 1u) {
          const int i = __ffs(m) - 1;
          const int p = __shfl_sync(0xffffffffu, my_p, i);
          const float wi = __shfl_sync(0xffffffffu, my_w, i);
          V r[kCombineBatch];
#pragma unroll
          for (int b = 0; b < kCombineBatch; ++b) {
            const int v = v0 + b * 32 + lane;
            if (v < nvec) r[b] = ld_keep(y + (int64_t)p * dim + v * V::N);
          }
#pragma unroll
          for (int b = 0; b < kCombineBatch; ++b)
#pragma unroll
            for (int q = 0; q < V::N; ++q) acc[b][q] = fmaf(wi, Elt<T_>::to_f(r[b].e[q]), acc[b][q]);
        }
#pragma unroll
        for (int b = 0; b < kCombineBatch; ++b) {
          const int v = v0 + b * 32 + lane;
          if (v >= nvec) continue;
          V o;
#pragma unroll
          for (int q = 0; q < V::N; ++q) o.e[q] = Elt<T_>::from_f(acc[b][q]);
          st_plain(dst + v * V::N, o);
        }
      }
      if (dw_rows != nullptr && lane < k)
        static_cast<float*>(dw_bases[s])[dst_row * k + lane] = dw_rows[j * k + lane];
      continue;
    }
    for (int v = lane; v < nvec; v += 32) {
      float acc[V::N];
#pragma unroll
      for (int i = 0; i < V::N; ++i) acc[i] = 0.f;
      for (int i = 0; i < k; ++i) {
        const int p = slot_pos[j * k + i];
        if (p < 0) continue;
        const float wi = w ? w[j * k + i] : 1.0f;
        V r = ld_keep(y + (int64_t)p * dim + v * V::N);
#pragma unroll
        for (int q = 0; q < V::N; ++q) acc[q] = fmaf(wi, Elt<T_>::to_f(r.e[q]), acc[q]);
      }
      V o;
#pragma unroll
      for (int q = 0; q < V::N; ++q) o.e[q] = Elt<T_>::from_f(acc[q]);
      st_plain(dst + v * V::N, o);
    }
    if (dw_rows != nullptr)
      for (int i = lane; i < k; i += 32)
        static_cast<float*>(dw_bases[s])[dst_row * k + i] = dw_rows[j * k + i];
  }
  publish(ctl, flag_bases, phase, n_ranks, me);
}

__global__ void ep_peer_wait_kernel(const unsigned* flags, int n_ranks, int phase, unsigned* ctl,
                                    uint64_t limit_ns, int* err) {
  const unsigned target = ctl[kCtlSeen + phase] + 1u;
  const int s = threadIdx.x;
  if (s < n_ranks) {
    const unsigned* f = flags + phase * n_ranks + s;
    const uint64_t t0 = gtimer();
    for (unsigned it = 0;; ++it) {
      if ((int)(ld_acquire_sys(f) - target) >= 0) break;
      if ((it & 63u) == 0 && gtimer() - t0 > limit_ns) {
        atomicExch(err, 16 + phase);  // phase whose data did not arrive
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) ctl[kCtlSeen + phase] = target;
}

inline int put_grid(int64_t rows) {
  int64_t g = (rows + 7) / 8;  // 8 warps per CTA
  const int64_t cap = (int64_t)num_sms() * 8;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace fk

extern "C" int fk_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  FK_CHECK_ARG(bytes > 0 && ptr && handle, "fk_ipc_alloc: bad argument");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fk::fail(FK_ERR_LAUNCH, "fk_ipc_alloc: cudaMalloc(%zu): %s", bytes,
                                        cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer can write
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fk::fail(FK_ERR_LAUNCH, "fk_ipc_alloc: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return FK_OK;
}

extern "C" int fk_ipc_open(const void* handle, void** ptr) {
  FK_CHECK_ARG(handle && ptr, "fk_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fk::fail(FK_ERR_LAUNCH, "fk_ipc_open: %s", cudaGetErrorString(e));
  return FK_OK;
}

extern "C" int fk_ipc_close(void* ptr) {
  FK_CHECK_ARG(ptr, "fk_ipc_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fk::fail(FK_ERR_LAUNCH, "fk_ipc_close: %s", cudaGetErrorString(e));
  return FK_OK;
}

extern "C" int fk_ipc_free(void* ptr) {
  FK_CHECK_ARG(ptr, "fk_ipc_free: null pointer");
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fk::fail(FK_ERR_LAUNCH, "fk_ipc_free: %s", cudaGetErrorString(e));
  return FK_OK;
}

extern "C" int fk_ep_peer_put_rows(const void* x, int dim, const int* send_token,
                                   int64_t n_tokens, int n_ranks, int my_rank, const int* send_e,
                                   const float* send_w, int k, void* const* row_bases,
                                   void* const* e_bases, void* const* w_bases,
                                   unsigned* const* flag_bases, int phase, unsigned* ctl,
                                   int dtype, void* stream) {
  FK_CHECK_ARG(n_tokens >= 0 && dim > 0 && k >= 1 && n_ranks >= 1 && n_ranks <= 32 &&
                   my_rank >= 0 && my_rank < n_ranks && phase >= 0 && phase < 4,
               "fk_ep_peer_put_rows: bad sizes");
  FK_CHECK_ARG(send_token && row_bases && flag_bases && ctl && (n_tokens == 0 || x),
               "fk_ep_peer_put_rows: null pointer");
  FK_CHECK_ARG(!send_e || (send_w && e_bases && w_bases), "fk_ep_peer_put_rows: partial metadata");
  FK_CHECK_ARG(fk::valid_dtype(dtype) && (dim * fk::dtype_size(dtype)) % 16 == 0 &&
                   (n_tokens == 0 || fk::aligned16(x)),
               "fk_ep_peer_put_rows: rows must be 16-byte aligned");
  cudaStream_t st = fk::as_stream(stream);
  FK_DISPATCH_DTYPE(dtype, fk::ep_peer_put_rows_kernel<scalar_t>
                    <<<fk::put_grid((int64_t)n_ranks * n_tokens), fk::kPutThreads, 0, st>>>(
                        static_cast<const scalar_t*>(x), dim, send_token, n_tokens, n_ranks,
                        my_rank, send_e, send_w, k, row_bases, e_bases, w_bases, flag_bases,
                        phase, ctl));
  return fk::launch_status("fk_ep_peer_put_rows");
}

extern "C" int fk_ep_peer_combine_put(const void* y, int dim, const int* slot_pos, const float* w,
                                      int64_t n_tokens, int n_ranks, int my_rank, int k,
                                      const float* dw_rows, void* const* row_bases,
                                      void* const* dw_bases, unsigned* const* flag_bases,
                                      int phase, unsigned* ctl, int dtype, void* stream) {
  FK_CHECK_ARG(n_tokens >= 0 && dim > 0 && k >= 1 && n_ranks >= 1 && n_ranks <= 32 &&
                   my_rank >= 0 && my_rank < n_ranks && phase >= 0 && phase < 4,
               "fk_ep_peer_combine_put: bad sizes");
  FK_CHECK_ARG(slot_pos && row_bases && flag_bases && ctl && (!dw_rows || dw_bases),
               "fk_ep_peer_combine_put: null pointer");
  FK_CHECK_ARG(fk::valid_dtype(dtype) && (dim * fk::dtype_size(dtype)) % 16 == 0 &&
                   (!y || fk::aligned16(y)),
               "fk_ep_peer_combine_put: rows must be 16-byte aligned");
  cudaStream_t st = fk::as_stream(stream);
  FK_DISPATCH_DTYPE(dtype, fk::ep_peer_combine_put_kernel<scalar_t>
                    <<<fk::put_grid((int64_t)n_ranks * n_tokens), fk::kPutThreads, 0, st>>>(
                        static_cast<const scalar_t*>(y), dim, slot_pos, w, n_tokens, n_ranks,
                        my_rank, k, dw_rows, row_bases, dw_bases, flag_bases, phase, ctl));
  return fk::launch_status("fk_ep_peer_combine_put");
}

extern "C" int fk_ep_peer_wait(const unsigned* flags, int n_ranks, int phase, unsigned* ctl,
                               int timeout_ms, int* err_flag, void* stream) {
  FK_CHECK_ARG(n_ranks >= 1 && n_ranks <= 32 && phase >= 0 && phase < 4 && timeout_ms > 0,
               "fk_ep_peer_wait: bad arguments");
  FK_CHECK_ARG(flags && ctl && err_flag, "fk_ep_peer_wait: null pointer");
  fk::ep_peer_wait_kernel<<<1, 32, 0, fk::as_stream(stream)>>>(
      flags, n_ranks, phase, ctl, (uint64_t)timeout_ms * 1000000ull, err_flag);
  return fk::launch_status("fk_ep_peer_wait");
}
