// Grouped GEMMs of the MoE expert MLPs on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM, operands staged by TMA), reference
// moe_layer_sorted.py:70-77 (one cuBLAS call per expert per Linear) and moe_layer.py:22-31.
//
// One persistent, warp-specialised kernel template serves every GEMM of the layer:
//   warp 0      TMA producer: fills a ring of STAGES shared-memory stages (A tile
//               128 rows x 128 bytes of K, B tile BN rows x 128 bytes of K, 128-byte
//               swizzle) and arms the stage's "full" mbarrier with the expected byte count;
//   warp 1      TMEM allocator + MMA issuer: one thread issues 4 tcgen05.mma per stage
//               into a 128 x BN fp32 accumulator in TMEM and hands the stage back with
//               tcgen05.commit on its "empty" mbarrier;
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each warp owns a 32-lane quarter
//               of TMEM = 32 rows of the tile), apply the fused epilogue, store.
// Two accumulators (2*BN TMEM columns) let the epilogue of tile i overlap the MMAs of
// tile i+1.  Tiles are handed out round-robin to one CTA per SM.
//
// Operand kinds.  KIND_BF16 / KIND_F16: 16-bit operands (kind::f16, 64 elements of K per
// stage, K = 16 per MMA), 16-bit outputs.  KIND_TF32X3: fp32 layers.  Each fp32 operand
// comes as a pair (hi, lo): hi keeps the sign, exponent and top 10 mantissa bits, lo =
// x - hi (exact in fp32).  The kernel runs the K loop three times into one accumulator --
// (A_hi, B_hi), (A_hi, B_lo), (A_lo, B_hi) -- on kind::tf32 MMAs (32 elements of K per
// stage, K = 8 per MMA).  That is the 3xTF32 decomposition (a*b ~ ah*bh + ah*bl + al*bh,
// dropping al*bl, about 2^-21 relative): fp32-class accuracy on the tensor cores.
// Outputs are fp32.
//
// Grouping.  MODE_M: rows of A are the expert-sorted assignment rows; every 128-row
// block belongs to one expert (segments are padded to 128 rows), whose weight matrix is
// the B operand (3-D tensor map over [E, rows, cols]).  The number of valid row blocks
// is read on the device, so no host synchronisation is needed.  MODE_K (weight
// gradients): for expert e the reduction runs over its token segment; A and B are
// token-major (MN-major operands) and the output is expert e's [M, N] gradient.
//
// 16-bit epilogue stores go through a per-warp ring of shared-memory chunks and TMA
// stores (coalesced 64-byte rows instead of per-thread 16-byte row fragments); fp32
// outputs are stored directly.
// Epilogues: plain store; SwiGLU forward (the B tile holds BN/2 gate rows and the
// matching BN/2 up rows, so the tile yields h1 = (g, u) and act = silu(g) * u); SwiGLU
// backward (reads g, u of the tile's hidden units and writes (dg, du)).
//
// No load uses cluster multicast: every CTA fetches its own tiles.  Every mbarrier wait
// is bounded by a wall-clock budget; a timeout records an error code and the CTA leaves
// its loops (the accumulator memory is still released).
#pragma once

#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"

namespace fk {
namespace gemm {

constexpr int BM = 128;
constexpr int kThreads = 192;
constexpr int kMaxGemmExperts = 256;  // expert ids of the weight-gradient schedule fit a byte
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per wait: far above any legitimate wait

enum Mode { MODE_M = 0, MODE_K = 1 };
enum Epi { EPI_STORE = 0, EPI_SWIGLU_FWD = 1, EPI_SWIGLU_BWD = 2 };
enum Kind { KIND_BF16 = 0, KIND_F16 = 1, KIND_TF32X3 = 2 };

template <int KIND> struct KindT;
template <> struct KindT<KIND_BF16> {
  using T = __nv_bfloat16;
  static constexpr int kBKE = 64;       // elements of K per 128-byte stage row
  static constexpr int kMmaK = 16;      // K per tcgen05.mma
  static constexpr uint32_t kFmt = 1;   // instruction-descriptor operand format (BF16)
  static constexpr int kPasses = 1;
  static constexpr CUtensorMapDataType kMapType = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
};
template <> struct KindT<KIND_F16> {
  using T = __half;
  static constexpr int kBKE = 64;
  static constexpr int kMmaK = 16;
  static constexpr uint32_t kFmt = 0;   // F16
  static constexpr int kPasses = 1;
  static constexpr CUtensorMapDataType kMapType = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
};
template <> struct KindT<KIND_TF32X3> {
  using T = float;
  static constexpr int kBKE = 32;
  static constexpr int kMmaK = 8;
  static constexpr uint32_t kFmt = 2;   // TF32
  static constexpr int kPasses = 3;     // (hi, hi), (hi, lo), (lo, hi)
  static constexpr CUtensorMapDataType kMapType = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
};

struct Params {
  int M, N, K;   // MODE_M: N = output columns (SwiGLU fwd: hidden units H), K = reduction
                 // MODE_K: per-expert output [M, N]
  int E, H;
  const int* seg_start;    // [E+1] padded token offsets
  const int* tile_expert;  // [rows/128] expert of each 128-row block (MODE_M)
  const int* n_mblk;       // valid 128-row blocks (MODE_M)
  void* out0;              // STORE: C; SWIGLU_FWD: act [rows, H]; SWIGLU_BWD: dh1 [rows, 2H]
  int64_t ld0;
  void* out1;              // SWIGLU_FWD: h1 [rows, 2H]
  int64_t ld1;
  const void* in0;         // SWIGLU_BWD: h1 [rows, 2H]
  int64_t ldi0;
  int* err;
  int tma_store;  // epilogue writes through shared memory + TMA stores (tmC0 / tmC1)
  // Row-weighted epilogues (ROWW): row_assign[r] < 0 marks a padding row, row_w[r] is the
  // routing weight of sorted row r; dw_part receives the routing-weight partial dots.
  const int* row_assign;
  const float* row_w;
  float* dw_part;  // EPI_SWIGLU_BWD with ROWW: [rows, H / 64] fp32
};

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded mbarrier wait (wall clock); records `code` in *err on timeout.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer() - t0 > kWaitNs) {
      atomicExch(err, code);
      return false;
    }
  }
}

__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                      uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(ptx::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(ptx::smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                      uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(ptx::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(ptx::smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor, sm_100 version bit.  Layout types: 2 = 128-byte swizzle
// of 16-byte chunks (every K-major tile, and MN-major tiles of 16-bit operands); 1 = 128-byte
// swizzle of 32-byte chunks, the only MN-major layout tf32 operands take (its pattern repeats
// every 4 rows of 128 bytes instead of 8).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout = 2) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)layout << 61;
  return d;
}

template <int KIND>
__device__ __forceinline__ void mma_issue(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  if constexpr (KIND == KIND_TF32X3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                   "r"(ptx::smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets row (lane base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Store 32 fp32 values as T at dst (16-byte aligned).
template <typename T>
__device__ __forceinline__ void store32(T* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      d[q] = make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                        __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      d[q] = make_uint4(pack2<T>(v[8 * q], v[8 * q + 1]), pack2<T>(v[8 * q + 2], v[8 * q + 3]),
                        pack2<T>(v[8 * q + 4], v[8 * q + 5]), pack2<T>(v[8 * q + 6], v[8 * q + 7]));
  }
}

template <typename T>
__device__ __forceinline__ void load32(const T* src, float (&v)[32]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint4 u = s[q];
      v[4 * q] = __uint_as_float(u.x);
      v[4 * q + 1] = __uint_as_float(u.y);
      v[4 * q + 2] = __uint_as_float(u.z);
      v[4 * q + 3] = __uint_as_float(u.w);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u = s[q];
      const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[8 * q + j] = Elt<T>::to_f(h[j]);
    }
  }
}

// Epilogue output path for 16-bit outputs: each epilogue warp owns a ring of kRingBufs
// 2 KB shared-memory buffers; a 32-row x 32-column chunk is written into one (64-byte
// rows, 64-byte swizzle, so the 16-byte writes of a warp hit distinct banks) and stored
// to global memory by one TMA store issued by lane 0.  A buffer is reused only after the
// bulk store that read it four chunks earlier has finished reading.
constexpr int kRingBufs = 4;
constexpr uint32_t kChunkBytes = 32 * 32 * 2;
constexpr uint32_t kRingBytesPerWarp = kRingBufs * kChunkBytes;

template <typename T>
struct StoreRing {
  uint32_t base;
  int next;
  __device__ __forceinline__ void put(const CUtensorMap* map, int col, int row,
                                      const float (&v)[32], int lane) {
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kRingBufs - 1) : "memory");
    __syncwarp();
    const uint32_t buf = base + (uint32_t)next * kChunkBytes;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t addr = buf + (uint32_t)lane * 64u + ((uint32_t)(q ^ ((lane >> 1) & 3)) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                   "r"(pack2<T>(v[8 * q], v[8 * q + 1])), "r"(pack2<T>(v[8 * q + 2], v[8 * q + 3])),
                   "r"(pack2<T>(v[8 * q + 4], v[8 * q + 5])), "r"(pack2<T>(v[8 * q + 6], v[8 * q + 7]))
                   : "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
      asm volatile(
          "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
              reinterpret_cast<uint64_t>(map)),
          "r"(col), "r"(row), "r"(buf)
          : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    next = (next + 1) & (kRingBufs - 1);
  }
  __device__ __forceinline__ void drain(int lane) {
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }
};

struct Tile {
  int e, m0, n0, kb0, kiters;
  bool valid;
};

template <int BN, int MODE, int EPI, int MB>
__device__ __forceinline__ int num_tiles(const Params& p) {
  if (MODE == MODE_M) {
    const int nnb = (EPI == EPI_SWIGLU_FWD) ? p.H / (BN / 2) : p.N / BN;
    return (*p.n_mblk) * nnb;
  }
  const int nmb = (p.M + BM * MB - 1) / (BM * MB), nnb = p.N / BN;
  return p.E * nmb * nnb;
}

// MODE_K visits the experts in descending order of their token count (order[]) and hands
// the tiles out in a serpentine over the CTAs (pass i goes left to right when i is even,
// right to left when odd), so the tiles of the few hot experts of a skewed routing spread
// evenly over the SMs instead of piling up on the CTAs their position happens to hit.
// t runs over whole passes; tiles past the end are invalid.  BKE = elements of K per stage;
// MB = 128-row blocks of M per tile (MODE_K).
template <int BN, int MODE, int EPI, int BKE, int MB>
__device__ __forceinline__ Tile decode(const Params& p, int t, const uint8_t* order, int ntiles) {
  Tile tl;
  tl.valid = true;
  if (MODE == MODE_M) {
    const int nnb = (EPI == EPI_SWIGLU_FWD) ? p.H / (BN / 2) : p.N / BN;
    const int mb = t / nnb, nb = t % nnb;
    tl.e = p.tile_expert[mb];
    tl.valid = tl.e >= 0;
    tl.m0 = mb * BM;
    tl.n0 = nb * ((EPI == EPI_SWIGLU_FWD) ? BN / 2 : BN);
    tl.kb0 = 0;
    tl.kiters = p.K / BKE;
  } else {
    const int nmb = (p.M + BM * MB - 1) / (BM * MB), nnb = p.N / BN;
    const int G = gridDim.x, pass = t / G, j = t % G;
    const int g = pass * G + ((pass & 1) ? G - 1 - j : j);
    if (g >= ntiles) {
      tl.valid = false;
      return tl;
    }
    tl.e = order[g / (nmb * nnb)];
    const int r = g % (nmb * nnb);
    tl.m0 = (r / nnb) * BM * MB;
    tl.n0 = (r % nnb) * BN;
    const int s0 = p.seg_start[tl.e], s1 = p.seg_start[tl.e + 1];
    tl.kb0 = s0 / BKE;
    tl.kiters = (s1 - s0) / BKE;
  }
  return tl;
}

// tmA/tmB: operands (KIND_TF32X3: their hi parts); tmA2/tmB2: the lo parts (TF32X3 only).
// ROWW (MODE_M SwiGLU epilogues): the routing weight of each row is applied in the
// epilogue (forward: out0 = w * silu(g) * u; backward: d(act) = w * accumulator, plus the
// routing-weight gradient partials), and padding rows come out as exact zeros.
// MB = 2 (MODE_K, 16-bit): a tile is 256 x BN, two accumulators side by side in TMEM fed by
// one B stage (a tile of a weight gradient with more tiles per expert than SMs would
// otherwise run in several waves, each re-reading the expert's operands from HBM); the
// accumulators are then single-buffered.
template <int BN, int STAGES, bool A_MN, bool B_MN, int MODE, int EPI, int KIND, bool ROWW = false,
          int MB = 1>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC0,
                    const __grid_constant__ CUtensorMap tmC1,
                    const __grid_constant__ CUtensorMap tmA2,
                    const __grid_constant__ CUtensorMap tmB2, const Params p) {
  using KT = KindT<KIND>;
  using T = typename KT::T;
  constexpr int BKE = KT::kBKE;
  constexpr int PASSES = KT::kPasses;
  static_assert(!ROWW || (MODE == MODE_M && EPI != EPI_STORE), "row weights: SwiGLU epilogues");
  static_assert(MB == 1 || (MB == 2 && MODE == MODE_K && KIND != KIND_TF32X3),
                "256-row tiles: 16-bit weight gradients");
  constexpr int NBUF = MB == 1 ? 2 : 1;  // accumulator sets in TMEM (double-buffered if 2)
  constexpr bool kRing = sizeof(T) == 2;  // TMA-store ring for 16-bit outputs
  constexpr uint32_t A_BYTES = MB * BM * 128;
  constexpr uint32_t B_BYTES = BN * 128;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t BOX_BYTES = BKE * 128;  // one BKE x BKE MN-major box
  constexpr uint32_t TMEM_COLS = NBUF * MB * BN;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t ring_base = ptx::smem_u32(smem + STAGES * STAGE_BYTES);  // 4 warps x ring
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES +
                                               (kRing ? 4 * kRingBytesPerWarp : 0));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ uint8_t order[kMaxGemmExperts];  // MODE_K: experts by descending token count
  if (MODE == MODE_K) {
    for (int e = threadIdx.x; e < p.E; e += blockDim.x) {
      const int len = p.seg_start[e + 1] - p.seg_start[e];
      int rank = 0;
      for (int f = 0; f < p.E; ++f) {
        const int lf = p.seg_start[f + 1] - p.seg_start[f];
        rank += (lf > len) || (lf == len && f < e);
      }
      order[rank] = (uint8_t)e;
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull[a], 1);
      ptx::mbar_init(&tempty[a], 128);
    }
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     ptx::smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ntiles = num_tiles<BN, MODE, EPI, MB>(p);
  const int tiles_loop =
      MODE == MODE_K ? (ntiles + (int)gridDim.x - 1) / (int)gridDim.x * (int)gridDim.x : ntiles;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles_loop && ok; t += gridDim.x) {
        const Tile tl = decode<BN, MODE, EPI, BKE, MB>(p, t, order, ntiles);
        if (!tl.valid) continue;
        const int total = tl.kiters * PASSES;
        for (int it = 0; it < total; ++it) {
          const int pass = PASSES == 1 ? 0 : it / tl.kiters;
          const int kb = it - pass * tl.kiters;
          const CUtensorMap* ma = (PASSES > 1 && pass == 2) ? &tmA2 : &tmA;
          const CUtensorMap* mb = (PASSES > 1 && pass == 1) ? &tmB2 : &tmB;
          if (!wait_bar(&empty[s], ph ^ 1, p.err, 11)) { ok = false; break; }
          unsigned char* sa = smem + s * STAGE_BYTES;
          unsigned char* sb = sa + A_BYTES;
          ptx::mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          const int k0 = (tl.kb0 + kb) * BKE;
          if (!A_MN) {
            tma2d(sa, ma, k0, tl.m0, &full[s]);
          } else {
#pragma unroll
            for (int i = 0; i < MB * BM / BKE; ++i) tma2d(sa + i * BOX_BYTES, ma, tl.m0 + BKE * i, k0, &full[s]);
          }
          if (EPI == EPI_SWIGLU_FWD) {
            tma3d(sb, mb, k0, tl.n0, tl.e, &full[s]);
            tma3d(sb + (BN / 2) * 128, mb, k0, p.H + tl.n0, tl.e, &full[s]);
          } else if (!B_MN) {
            tma3d(sb, mb, k0, tl.n0, tl.e, &full[s]);
          } else if (MODE == MODE_M) {
#pragma unroll
            for (int i = 0; i < BN / BKE; ++i) tma3d(sb + i * BOX_BYTES, mb, tl.n0 + BKE * i, k0, tl.e, &full[s]);
          } else {
#pragma unroll
            for (int i = 0; i < BN / BKE; ++i) tma2d(sb + i * BOX_BYTES, mb, tl.n0 + BKE * i, k0, &full[s]);
          }
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = (1u << 4) | (KT::kFmt << 7) | (KT::kFmt << 10) |
                                 ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16) |
                                 ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
      constexpr uint32_t kMnStep = KT::kMmaK * 128;  // bytes of K per MMA, MN-major tiles
      // MN-major tiles: tf32 uses the 32-byte-chunk swizzle (4-row groups of 512 bytes),
      // 16-bit types the 16-byte-chunk swizzle (8-row groups of 1024 bytes).
      constexpr uint32_t kMnLayout = KIND == KIND_TF32X3 ? 1u : 2u;
      constexpr uint32_t kMnSbo = KIND == KIND_TF32X3 ? 512u : 1024u;
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles_loop && ok; t += gridDim.x) {
        const Tile tl = decode<BN, MODE, EPI, BKE, MB>(p, t, order, ntiles);
        if (!tl.valid) continue;
        const int acc = NBUF == 2 ? (it & 1) : 0;
        const uint32_t aph = (uint32_t)((NBUF == 2 ? (it >> 1) : it) & 1);
        ++it;
        if (!wait_bar(&tempty[acc], aph ^ 1, p.err, 12)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * MB * BN);
        if (tl.kiters == 0) {
          ptx::mbar_arrive(&tfull[acc]);
          continue;
        }
        const int total = tl.kiters * PASSES;
        for (int kb = 0; kb < total; ++kb) {
          if (!wait_bar(&full[s], ph, p.err, 13)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = ptx::smem_u32(smem + s * STAGE_BYTES);
          const uint32_t b_base = a_base + A_BYTES;
#pragma unroll
          for (int ks = 0; ks < BKE / KT::kMmaK; ++ks) {
            const uint64_t bd = B_MN ? smem_desc(b_base + ks * kMnStep, BOX_BYTES, kMnSbo, kMnLayout)
                                     : smem_desc(b_base + ks * 32, 16, 1024);
#pragma unroll
            for (int h = 0; h < MB; ++h) {  // 128-row block h of A into accumulator h
              const uint32_t ah = a_base + (uint32_t)h * (BM * 128);
              const uint64_t ad = A_MN ? smem_desc(ah + ks * kMnStep, BOX_BYTES, kMnSbo, kMnLayout)
                                       : smem_desc(ah + ks * 32, 16, 1024);
              mma_issue<KIND>(d_tmem + (uint32_t)(h * BN), ad, bd, idesc, (kb | ks) != 0);
            }
          }
          mma_commit(&empty[s]);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        mma_commit(&tfull[acc]);
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue (128 thr)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    StoreRing<T> ring{ring_base + (uint32_t)(warp - 2) * kRingBytesPerWarp, 0};
    const bool tma_out = kRing && p.tma_store;
    int it = 0;
    for (int t = blockIdx.x; t < tiles_loop; t += gridDim.x) {
      const Tile tl = decode<BN, MODE, EPI, BKE, MB>(p, t, order, ntiles);
      if (!tl.valid) continue;
      const int acc = NBUF == 2 ? (it & 1) : 0;
      const uint32_t aph = (uint32_t)((NBUF == 2 ? (it >> 1) : it) & 1);
      ++it;
      if (!wait_bar(&tfull[acc], aph, p.err, 14)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (uint32_t)(acc * MB * BN) + ((uint32_t)(q * 32) << 16);
      const bool zero = tl.kiters == 0;
      const int row0 = tl.m0 + q * 32;  // first row of this warp's 32-row slab
      if (MODE == MODE_K) {
        // tcgen05.ld is warp-collective: every lane loads, only rows < M store.
#pragma unroll 1
        for (int h = 0; h < MB; ++h) {  // accumulator h holds rows m0 + 128h ..
          const int m = tl.m0 + h * BM + row_in_tile;
          T* dst = static_cast<T*>(p.out0) + ((int64_t)tl.e * p.M + m) * p.ld0 + tl.n0;
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            float v[32];
            if (zero) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = 0.f;
            } else {
              tmem_ld32(tbase + (uint32_t)(h * BN) + c, v);
            }
            if (tma_out) ring.put(&tmC0, tl.n0 + c, tl.e * p.M + row0 + h * BM, v, lane);
            else if (m < p.M) store32(dst + c, v);
          }
        }
      } else {
        const int64_t row = tl.m0 + row_in_tile;
        if (EPI == EPI_STORE) {
          T* dst = static_cast<T*>(p.out0) + row * p.ld0 + tl.n0;
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            float v[32];
            tmem_ld32(tbase + c, v);
            if (tma_out) ring.put(&tmC0, tl.n0 + c, row0, v, lane);
            else store32(dst + c, v);
          }
        } else if (EPI == EPI_SWIGLU_FWD) {
          // ROWW: out0 is the routing-weighted activation w[row] * silu(g) * u (zero on
          // padding rows), so the down-projection yields weighted rows.
          bool vrow = true;
          float rw = 1.0f;
          if constexpr (ROWW) {
            vrow = p.row_assign[row] >= 0;
            rw = vrow ? p.row_w[row] : 0.0f;
          }
          T* act = static_cast<T*>(p.out0) + row * p.ld0 + tl.n0;
          T* hg = static_cast<T*>(p.out1) + row * p.ld1 + tl.n0;
          T* hu = static_cast<T*>(p.out1) + row * p.ld1 + p.H + tl.n0;
#pragma unroll 1
          for (int c = 0; c < BN / 2; c += 32) {
            float g[32], u[32], a[32];
            tmem_ld32(tbase + c, g);
            tmem_ld32(tbase + BN / 2 + c, u);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              a[i] = g[i] * sigmoidf_t<T>(g[i]) * u[i];
              if constexpr (ROWW) a[i] = vrow ? rw * a[i] : 0.0f;
            }
            if (tma_out) {
              ring.put(&tmC1, tl.n0 + c, row0, g, lane);
              ring.put(&tmC1, p.H + tl.n0 + c, row0, u, lane);
              ring.put(&tmC0, tl.n0 + c, row0, a, lane);
            } else {
              store32(hg + c, g);
              store32(hu + c, u);
              store32(act + c, a);
            }
          }
        } else {  // EPI_SWIGLU_BWD: accumulator = d(act) for hidden units n0 .. n0+BN
          // ROWW: A holds the unweighted output-gradient rows, so the accumulator is
          // dout[token] @ w2.  d(act) is w[row] times it, and the routing-weight gradient of
          // the row, <dout[token], y_row> = <dout[token] @ w2, act_row>, is summed here over
          // this tile's hidden units into dw_part (act recomputed from g, u).  Padding rows
          // give zeros.
          bool vrow = true;
          float rw = 1.0f, dot = 0.0f;
          if constexpr (ROWW) {
            vrow = p.row_assign[row] >= 0;
            rw = vrow ? p.row_w[row] : 0.0f;
          }
          const T* hg = static_cast<const T*>(p.in0) + row * p.ldi0 + tl.n0;
          const T* hu = static_cast<const T*>(p.in0) + row * p.ldi0 + p.H + tl.n0;
          T* dg = static_cast<T*>(p.out0) + row * p.ld0 + tl.n0;
          T* du = static_cast<T*>(p.out0) + row * p.ld0 + p.H + tl.n0;
          // h1's 32 gate and 32 up values of the next chunk are loaded (as raw 16-byte
          // packets) while the current chunk is computed and stored.
          constexpr int QP = 32 * (int)sizeof(T) / 16;  // packets per 32 values
          uint4 ng[QP], nu[QP];
#pragma unroll
          for (int j = 0; j < QP; ++j) {
            ng[j] = reinterpret_cast<const uint4*>(hg)[j];
            nu[j] = reinterpret_cast<const uint4*>(hu)[j];
          }
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            float d[32], g[32], u[32], og[32], ou[32];
            uint4 cg[QP], cu[QP];
#pragma unroll
            for (int j = 0; j < QP; ++j) {
              cg[j] = ng[j];
              cu[j] = nu[j];
            }
            if (c + 32 < BN) {
#pragma unroll
              for (int j = 0; j < QP; ++j) {
                ng[j] = reinterpret_cast<const uint4*>(hg + c + 32)[j];
                nu[j] = reinterpret_cast<const uint4*>(hu + c + 32)[j];
              }
            }
            tmem_ld32(tbase + c, d);
            load32(reinterpret_cast<const T*>(cg), g);
            load32(reinterpret_cast<const T*>(cu), u);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float sg = sigmoidf_t<T>(g[i]);
              float dd = d[i];
              if constexpr (ROWW) {
                dot = fmaf(d[i], g[i] * sg * u[i], dot);
                dd = rw * d[i];
              }
              ou[i] = dd * g[i] * sg;
              og[i] = dd * u[i] * (sg * (1.0f + g[i] * (1.0f - sg)));
              if constexpr (ROWW) {
                ou[i] = vrow ? ou[i] : 0.0f;
                og[i] = vrow ? og[i] : 0.0f;
              }
            }
            if (tma_out) {
              ring.put(&tmC0, tl.n0 + c, row0, og, lane);
              ring.put(&tmC0, p.H + tl.n0 + c, row0, ou, lane);
            } else {
              store32(dg + c, og);
              store32(du + c, ou);
            }
          }
          if constexpr (ROWW) {
            // one slot per 64 hidden units: this tile's dot in its first slot, zeros in the
            // rest, so the layout does not depend on the tile width
            float* dp = p.dw_part + row * (p.H / 64) + tl.n0 / 64;
            dp[0] = vrow ? dot : 0.0f;
#pragma unroll
            for (int j = 1; j < BN / 64; ++j) dp[j] = 0.0f;
          }
        }
      }
      tc_fence_before();
      ptx::mbar_arrive(&tempty[acc]);
    }
    if (kRing) ring.drain(lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------------------ host side -----------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn();  // cuTensorMapEncodeTiled, looked up once (moe_gemm.cu)

// Tensor map, 128-byte swizzle by default; dims/strides innermost first (strides in
// bytes, rank-1 entries), box innermost first.
inline int make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, int rank,
                    const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                    CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(FK_ERR_NO_DEVICE, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t d[3], st[2];
  cuuint32_t b[3], es[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) st[i] = strides[i];
  CUresult r = fn(m, dt, rank, const_cast<void*>(base), d, st, b, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FK_ERR_INVALID_ARG, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FK_OK;
}

// Epilogue output map for 16-bit outputs: [rows, cols] (row stride ld elements), 32 x 32
// boxes, 64-byte swizzle (matching the StoreRing layout).
template <int KIND>
inline int make_out_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld) {
  uint64_t d[2] = {(uint64_t)cols, (uint64_t)rows}, st[1] = {(uint64_t)ld * 2};
  uint32_t box[2] = {32, 32};
  return make_map(m, KindT<KIND>::kMapType, base, 2, d, st, box, CU_TENSOR_MAP_SWIZZLE_64B);
}

// Swizzle of MN-major operand tiles (matches kMnLayout in the kernel).
template <int KIND>
constexpr CUtensorMapSwizzle mn_swizzle() {
  return KIND == KIND_TF32X3 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
}

template <int BN, bool A_MN, bool B_MN, int MODE, int EPI, int KIND, bool ROWW = false, int MB = 1>
int launch(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c0,
           const CUtensorMap& c1, const CUtensorMap& a2, const CUtensorMap& b2, const Params& p,
           int max_tiles, cudaStream_t st, int max_ctas) {
  constexpr bool kRing = sizeof(typename KindT<KIND>::T) == 2;
  constexpr int STAGE_BYTES = (MB * BM + BN) * 128;
  constexpr int STAGES = MB == 2 ? 3 : ((BN == 256) ? 4 : (BN == 128 ? 6 : 8));
  constexpr int SMEM = STAGES * STAGE_BYTES + (kRing ? 4 * (int)kRingBytesPerWarp : 0) + 1024 + 256;
  static_assert(SMEM <= 232448, "shared memory per CTA");
  auto k = moe_gemm_kernel<BN, STAGES, A_MN, B_MN, MODE, EPI, KIND, ROWW, MB>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  int grid = num_sms();
  if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;  // SMs left to concurrent work
  if (max_tiles < grid) grid = max_tiles < 1 ? 1 : max_tiles;
  k<<<grid, kThreads, SMEM, st>>>(a, b, c0, c1, a2, b2, p);
  return launch_status("fk_moe_gemm");
}

inline int pick_bn(int n) {
  if (n % 256 == 0) return 256;
  if (n % 128 == 0) return 128;
  if (n % 64 == 0) return 64;
  return 0;
}

// ---------------------------------------------------------------- GEMM set-up ------------
// One function per GEMM of the layer, shared by the bf16 entry points and the typed ones.
// a2/b2 are the lo parts of the operands (KIND_TF32X3 only; ignored otherwise).
#define FK_BN_SWITCH(bn, ...)                                 \
  switch (bn) {                                               \
    case 256: { constexpr int BN_ = 256; __VA_ARGS__; break; } \
    case 128: { constexpr int BN_ = 128; __VA_ARGS__; break; } \
    case 64: { constexpr int BN_ = 64; __VA_ARGS__; break; }   \
    default: return ::fk::fail(FK_ERR_UNSUPPORTED, "unsupported tile width"); \
  }
// The typed kinds (fp16, fp32) instantiate 128- and 64-wide tiles only.
#define FK_BN_SWITCH_SMALL(bn, ...)                           \
  switch (bn) {                                               \
    case 128: { constexpr int BN_ = 128; __VA_ARGS__; break; } \
    case 64: { constexpr int BN_ = 64; __VA_ARGS__; break; }   \
    default: return ::fk::fail(FK_ERR_UNSUPPORTED, "unsupported tile width"); \
  }

template <int KIND>
inline int bn_for(int n) {
  const int bn = pick_bn(n);
  return (KIND == KIND_BF16 || bn != 256) ? bn : 128;
}

inline int check_common(const void* a, const void* b, const int* tile_expert, const int* n_mblk,
                        int64_t max_rows, int E) {
  FK_CHECK_ARG(a && b && tile_expert && n_mblk, "fk_moe_gemm: null pointer");
  FK_CHECK_ARG(max_rows >= 0 && max_rows % BM == 0, "fk_moe_gemm: max_rows must be a multiple of 128");
  FK_CHECK_ARG(E >= 1, "fk_moe_gemm: E < 1");
  FK_CHECK_ARG(aligned16(a) && aligned16(b), "fk_moe_gemm: operands must be 16-byte aligned");
  return FK_OK;
}

template <int KIND>
inline int check_lo(const void* a2, const void* b2) {
  if (KIND != KIND_TF32X3) return FK_OK;
  FK_CHECK_ARG(a2 && b2 && aligned16(a2) && aligned16(b2),
               "fk_moe_gemm (fp32): the lo parts of both operands are required (16-byte aligned)");
  return FK_OK;
}

template <int KIND>
int gemm_up(const void* xs, const void* xs2, int64_t max_rows, int dim, const void* w13,
            const void* w132, int hidden, int n_experts, const int* tile_expert,
            const int* n_mblk, void* h1, void* act, int* err_flag, cudaStream_t s,
            int max_ctas = 0) {
  using KT = KindT<KIND>;
  constexpr int ES = sizeof(typename KT::T);
  int st = check_common(xs, w13, tile_expert, n_mblk, max_rows, n_experts);
  if (st) return st;
  if ((st = check_lo<KIND>(xs2, w132))) return st;
  FK_CHECK_ARG(h1 && act && err_flag, "fk_moe_gemm_up: null pointer");
  FK_CHECK_ARG(dim % 64 == 0 && hidden % 64 == 0, "fk_moe_gemm_up: dim, hidden must be multiples of 64");
  if (max_rows == 0) return FK_OK;
  const int bn = (KIND == KIND_BF16 && hidden % 128 == 0) ? 256 : 128;
  CUtensorMap ma, mb, ma2, mb2;
  uint64_t da[2] = {(uint64_t)dim, (uint64_t)max_rows}, sa[1] = {(uint64_t)dim * ES};
  uint32_t ba[2] = {(uint32_t)KT::kBKE, 128};
  if ((st = make_map(&ma, KT::kMapType, xs, 2, da, sa, ba))) return st;
  uint64_t db[3] = {(uint64_t)dim, (uint64_t)2 * hidden, (uint64_t)n_experts};
  uint64_t sb[2] = {(uint64_t)dim * ES, (uint64_t)2 * hidden * dim * ES};
  uint32_t bb[3] = {(uint32_t)KT::kBKE, (uint32_t)bn / 2, 1};
  if ((st = make_map(&mb, KT::kMapType, w13, 3, db, sb, bb))) return st;
  ma2 = ma;
  mb2 = mb;
  if (KIND == KIND_TF32X3) {
    if ((st = make_map(&ma2, KT::kMapType, xs2, 2, da, sa, ba))) return st;
    if ((st = make_map(&mb2, KT::kMapType, w132, 3, db, sb, bb))) return st;
  }
  Params p{};
  p.M = (int)max_rows;
  p.N = hidden;
  p.K = dim;
  p.E = n_experts;
  p.H = hidden;
  p.tile_expert = tile_expert;
  p.n_mblk = n_mblk;
  p.out0 = act;
  p.ld0 = hidden;
  p.out1 = h1;
  p.ld1 = 2 * (int64_t)hidden;
  p.err = err_flag;
  const int max_tiles = (int)(max_rows / BM) * (hidden / (bn / 2));
  CUtensorMap mc0 = ma, mc1 = ma;
  p.tma_store = ES == 2 ? 1 : 0;
  if (p.tma_store) {
    if ((st = make_out_map<KIND>(&mc0, act, max_rows, hidden, hidden))) return st;
    if ((st = make_out_map<KIND>(&mc1, h1, max_rows, 2 * hidden, 2 * hidden))) return st;
  }
  if constexpr (KIND == KIND_BF16) {
    if (bn == 256)
      return launch<256, false, false, MODE_M, EPI_SWIGLU_FWD, KIND>(ma, mb, mc0, mc1, ma2, mb2, p, max_tiles, s, max_ctas);
  }
  return launch<128, false, false, MODE_M, EPI_SWIGLU_FWD, KIND>(ma, mb, mc0, mc1, ma2, mb2, p, max_tiles, s, max_ctas);
}

template <int KIND>
int gemm_down(const void* act, const void* act2, int64_t max_rows, int hidden, const void* w2,
              const void* w22, int dim, int n_experts, const int* tile_expert, const int* n_mblk,
              void* y, int* err_flag, cudaStream_t s,
            int max_ctas = 0) {
  using KT = KindT<KIND>;
  constexpr int ES = sizeof(typename KT::T);
  int st = check_common(act, w2, tile_expert, n_mblk, max_rows, n_experts);
  if (st) return st;
  if ((st = check_lo<KIND>(act2, w22))) return st;
  FK_CHECK_ARG(y && err_flag, "fk_moe_gemm_down: null pointer");
  FK_CHECK_ARG(hidden % 64 == 0 && dim % 64 == 0, "fk_moe_gemm_down: dim, hidden must be multiples of 64");
  if (max_rows == 0) return FK_OK;
  const int bn = bn_for<KIND>(dim);
  CUtensorMap ma, mb, ma2, mb2;
  uint64_t da[2] = {(uint64_t)hidden, (uint64_t)max_rows}, sa[1] = {(uint64_t)hidden * ES};
  uint32_t ba[2] = {(uint32_t)KT::kBKE, 128};
  if ((st = make_map(&ma, KT::kMapType, act, 2, da, sa, ba))) return st;
  uint64_t db[3] = {(uint64_t)hidden, (uint64_t)dim, (uint64_t)n_experts};
  uint64_t sb[2] = {(uint64_t)hidden * ES, (uint64_t)dim * hidden * ES};
  uint32_t bb[3] = {(uint32_t)KT::kBKE, (uint32_t)bn, 1};
  if ((st = make_map(&mb, KT::kMapType, w2, 3, db, sb, bb))) return st;
  ma2 = ma;
  mb2 = mb;
  if (KIND == KIND_TF32X3) {
    if ((st = make_map(&ma2, KT::kMapType, act2, 2, da, sa, ba))) return st;
    if ((st = make_map(&mb2, KT::kMapType, w22, 3, db, sb, bb))) return st;
  }
  Params p{};
  p.M = (int)max_rows;
  p.N = dim;
  p.K = hidden;
  p.E = n_experts;
  p.H = hidden;
  p.tile_expert = tile_expert;
  p.n_mblk = n_mblk;
  p.out0 = y;
  p.ld0 = dim;
  p.err = err_flag;
  const int max_tiles = (int)(max_rows / BM) * (dim / bn);
  CUtensorMap mc0 = ma;
  p.tma_store = ES == 2 ? 1 : 0;
  if (p.tma_store && (st = make_out_map<KIND>(&mc0, y, max_rows, dim, dim))) return st;
  if constexpr (KIND == KIND_BF16) {
    FK_BN_SWITCH(bn, return (launch<BN_, false, false, MODE_M, EPI_STORE, KIND>(ma, mb, mc0, mc0, ma2, mb2, p, max_tiles, s, max_ctas)));
  } else {
    FK_BN_SWITCH_SMALL(bn, return (launch<BN_, false, false, MODE_M, EPI_STORE, KIND>(ma, mb, mc0, mc0, ma2, mb2, p, max_tiles, s, max_ctas)));
  }
  return FK_OK;
}

template <int KIND>
int gemm_down_dgrad(const void* dy, const void* dy2, int64_t max_rows, int dim, const void* w2,
                    const void* w22, int hidden, int n_experts, const int* tile_expert,
                    const int* n_mblk, const void* h1, void* dh1, int* err_flag, cudaStream_t s,
            int max_ctas = 0) {
  using KT = KindT<KIND>;
  constexpr int ES = sizeof(typename KT::T);
  int st = check_common(dy, w2, tile_expert, n_mblk, max_rows, n_experts);
  if (st) return st;
  if ((st = check_lo<KIND>(dy2, w22))) return st;
  FK_CHECK_ARG(h1 && dh1 && err_flag, "fk_moe_gemm_down_dgrad: null pointer");
  FK_CHECK_ARG(hidden % 64 == 0 && dim % 64 == 0, "fk_moe_gemm_down_dgrad: dim, hidden must be multiples of 64");
  if (max_rows == 0) return FK_OK;
  const int bn = bn_for<KIND>(hidden);
  CUtensorMap ma, mb, ma2, mb2;
  uint64_t da[2] = {(uint64_t)dim, (uint64_t)max_rows}, sa[1] = {(uint64_t)dim * ES};
  uint32_t ba[2] = {(uint32_t)KT::kBKE, 128};
  if ((st = make_map(&ma, KT::kMapType, dy, 2, da, sa, ba))) return st;
  // B[n = h, k = d] = W2[e][d][h]: hidden-contiguous (MN-major) boxes of BKE x BKE.
  uint64_t db[3] = {(uint64_t)hidden, (uint64_t)dim, (uint64_t)n_experts};
  uint64_t sb[2] = {(uint64_t)hidden * ES, (uint64_t)dim * hidden * ES};
  uint32_t bb[3] = {(uint32_t)KT::kBKE, (uint32_t)KT::kBKE, 1};
  if ((st = make_map(&mb, KT::kMapType, w2, 3, db, sb, bb, mn_swizzle<KIND>()))) return st;
  ma2 = ma;
  mb2 = mb;
  if (KIND == KIND_TF32X3) {
    if ((st = make_map(&ma2, KT::kMapType, dy2, 2, da, sa, ba))) return st;
    if ((st = make_map(&mb2, KT::kMapType, w22, 3, db, sb, bb, mn_swizzle<KIND>()))) return st;
  }
  Params p{};
  p.M = (int)max_rows;
  p.N = hidden;
  p.K = dim;
  p.E = n_experts;
  p.H = hidden;
  p.tile_expert = tile_expert;
  p.n_mblk = n_mblk;
  p.out0 = dh1;
  p.ld0 = 2 * (int64_t)hidden;
  p.in0 = h1;
  p.ldi0 = 2 * (int64_t)hidden;
  p.err = err_flag;
  const int max_tiles = (int)(max_rows / BM) * (hidden / bn);
  CUtensorMap mc0 = ma;
  p.tma_store = ES == 2 ? 1 : 0;
  if (p.tma_store && (st = make_out_map<KIND>(&mc0, dh1, max_rows, 2 * hidden, 2 * hidden))) return st;
  if constexpr (KIND == KIND_BF16) {
    FK_BN_SWITCH(bn, return (launch<BN_, false, true, MODE_M, EPI_SWIGLU_BWD, KIND>(ma, mb, mc0, mc0, ma2, mb2, p, max_tiles, s, max_ctas)));
  } else {
    FK_BN_SWITCH_SMALL(bn, return (launch<BN_, false, true, MODE_M, EPI_SWIGLU_BWD, KIND>(ma, mb, mc0, mc0, ma2, mb2, p, max_tiles, s, max_ctas)));
  }
  return FK_OK;
}

template <int KIND>
int gemm_up_dgrad(const void* dh1, const void* dh12, int64_t max_rows, int hidden, const void* w13,
                  const void* w132, int dim, int n_experts, const int* tile_expert,
                  const int* n_mblk, void* dxs, int* err_flag, cudaStream_t s,
            int max_ctas = 0) {
  using KT = KindT<KIND>;
  constexpr int ES = sizeof(typename KT::T);
  int st = check_common(dh1, w13, tile_expert, n_mblk, max_rows, n_experts);
  if (st) return st;
  if ((st = check_lo<KIND>(dh12, w132))) return st;
  FK_CHECK_ARG(dxs && err_flag, "fk_moe_gemm_up_dgrad: null pointer");
  FK_CHECK_ARG(hidden % 64 == 0 && dim % 64 == 0, "fk_moe_gemm_up_dgrad: dim, hidden must be multiples of 64");
  if (max_rows == 0) return FK_OK;
  const int bn = bn_for<KIND>(dim);
  CUtensorMap ma, mb, ma2, mb2;
  uint64_t da[2] = {(uint64_t)2 * hidden, (uint64_t)max_rows}, sa[1] = {(uint64_t)2 * hidden * ES};
  uint32_t ba[2] = {(uint32_t)KT::kBKE, 128};
  if ((st = make_map(&ma, KT::kMapType, dh1, 2, da, sa, ba))) return st;
  // B[n = d, k = j] = W13[e][j][d]: dim-contiguous (MN-major) boxes of BKE x BKE.
  uint64_t db[3] = {(uint64_t)dim, (uint64_t)2 * hidden, (uint64_t)n_experts};
  uint64_t sb[2] = {(uint64_t)dim * ES, (uint64_t)2 * hidden * dim * ES};
  uint32_t bb[3] = {(uint32_t)KT::kBKE, (uint32_t)KT::kBKE, 1};
  if ((st = make_map(&mb, KT::kMapType, w13, 3, db, sb, bb, mn_swizzle<KIND>()))) return st;
  ma2 = ma;
  mb2 = mb;
  if (KIND == KIND_TF32X3) {
    if ((st = make_map(&ma2, KT::kMapType, dh12, 2, da, sa, ba))) return st;
    if ((st = make_map(&mb2, KT::kMapType, w132, 3, db, sb, bb, mn_swizzle<KIND>()))) return st;
  }
  Params p{};
  p.M = (int)max_rows;
  p.N = dim;
  p.K = 2 * hidden;
  p.E = n_experts;
  p.H = hidden;
  p.tile_expert = tile_expert;
  p.n_mblk = n_mblk;
  p.out0 = dxs;
  p.ld0 = dim;
  p.err = err_flag;
  const int max_tiles = (int)(max_rows / BM) * (dim / bn);
  CUtensorMap mc0 = ma;
  p.tma_store = ES == 2 ? 1 : 0;
  if (p.tma_store && (st = make_out_map<KIND>(&mc0, dxs, max_rows, dim, dim))) return st;
  if constexpr (KIND == KIND_BF16) {
    FK_BN_SWITCH(bn, return (launch<BN_, false, true, MODE_M, EPI_STORE, KIND>(ma, mb, mc0, mc0, ma2, mb2, p, max_tiles, s, max_ctas)));
  } else {
    FK_BN_SWITCH_SMALL(bn, return (launch<BN_, false, true, MODE_M, EPI_STORE, KIND>(ma, mb, mc0, mc0, ma2, mb2, p, max_tiles, s, max_ctas)));
  }
  return FK_OK;
}

template <int KIND>
int gemm_wgrad(const void* a, const void* a2, int m_dim, const void* b, const void* b2, int n_dim,
               int64_t max_rows, const int* seg_start, int n_experts, void* dw, int* err_flag,
               cudaStream_t s, int max_ctas = 0) {
  using KT = KindT<KIND>;
  constexpr int ES = sizeof(typename KT::T);
  FK_CHECK_ARG(a && b && seg_start && dw && err_flag, "fk_moe_gemm_wgrad: null pointer");
  FK_CHECK_ARG(max_rows >= 0 && max_rows % BM == 0, "fk_moe_gemm_wgrad: max_rows must be a multiple of 128");
  FK_CHECK_ARG(n_experts >= 1 && n_experts <= kMaxGemmExperts && m_dim % 64 == 0 &&
                   n_dim % 64 == 0 && m_dim > 0 && n_dim > 0,
               "fk_moe_gemm_wgrad: dims must be positive multiples of 64");
  FK_CHECK_ARG(aligned16(a) && aligned16(b) && aligned16(dw), "fk_moe_gemm_wgrad: unaligned");
  int st;
  if ((st = check_lo<KIND>(a2, b2))) return st;
  const int bn = bn_for<KIND>(n_dim);
  CUtensorMap ma, mb, ma2, mb2;
  const uint64_t rows = max_rows > 0 ? (uint64_t)max_rows : 128;
  uint64_t da[2] = {(uint64_t)m_dim, rows}, sa[1] = {(uint64_t)m_dim * ES};
  uint32_t ba[2] = {(uint32_t)KT::kBKE, (uint32_t)KT::kBKE};
  if ((st = make_map(&ma, KT::kMapType, a, 2, da, sa, ba, mn_swizzle<KIND>()))) return st;
  uint64_t db[2] = {(uint64_t)n_dim, rows}, sb[1] = {(uint64_t)n_dim * ES};
  uint32_t bb[2] = {(uint32_t)KT::kBKE, (uint32_t)KT::kBKE};
  if ((st = make_map(&mb, KT::kMapType, b, 2, db, sb, bb, mn_swizzle<KIND>()))) return st;
  ma2 = ma;
  mb2 = mb;
  if (KIND == KIND_TF32X3) {
    if ((st = make_map(&ma2, KT::kMapType, a2, 2, da, sa, ba, mn_swizzle<KIND>()))) return st;
    if ((st = make_map(&mb2, KT::kMapType, b2, 2, db, sb, bb, mn_swizzle<KIND>()))) return st;
  }
  Params p{};
  p.M = m_dim;
  p.N = n_dim;
  p.E = n_experts;
  p.seg_start = seg_start;
  p.out0 = dw;
  p.ld0 = n_dim;
  p.err = err_flag;
  int max_tiles = n_experts * ((m_dim + BM - 1) / BM) * (n_dim / bn);
  // TMA stores need every 128-row tile inside one expert's [m_dim, n_dim] block.
  CUtensorMap mc0 = ma;
  p.tma_store = (ES == 2 && m_dim % BM == 0) ? 1 : 0;
  if (p.tma_store && (st = make_out_map<KIND>(&mc0, dw, (int64_t)n_experts * m_dim, n_dim, n_dim))) return st;
  // An expert whose 128 x 256 tiles outnumber the SMs would run them in several waves, each
  // streaming the expert's token segment again; 256-row tiles keep it to one wave.
  if constexpr (ES == 2) {
    if (bn == 256 && m_dim % (2 * BM) == 0 && p.tma_store && (m_dim / BM) * (n_dim / bn) > num_sms()) {
      max_tiles = n_experts * (m_dim / (2 * BM)) * (n_dim / bn);
      return launch<256, true, true, MODE_K, EPI_STORE, KIND, false, 2>(ma, mb, mc0, mc0, ma2, mb2,
                                                                       p, max_tiles, s, max_ctas);
    }
  }
  if constexpr (KIND == KIND_BF16) {
    FK_BN_SWITCH(bn, return (launch<BN_, true, true, MODE_K, EPI_STORE, KIND>(ma, mb, mc0, mc0, ma2, mb2, p, max_tiles, s, max_ctas)));
  } else {
    FK_BN_SWITCH_SMALL(bn, return (launch<BN_, true, true, MODE_K, EPI_STORE, KIND>(ma, mb, mc0, mc0, ma2, mb2, p, max_tiles, s, max_ctas)));
  }
  return FK_OK;
}

}  // namespace gemm
}  // namespace fk
