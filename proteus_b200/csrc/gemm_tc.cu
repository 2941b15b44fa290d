// Tensor-core contractions on tcgen05 / TMEM (sm_100a), TMA-fed, warp-specialised:
//   warp 0: TMA producer (one elected lane), warp 1: MMA issuer (one lane; owns the TMEM
//   allocation), warps 2-5: epilogue (TMEM -> registers -> global), one thread per accumulator row.
//
// atlas_gram_upper  C[D, D] += X^T X on the upper 128-block triangle (gram_accumulate,
//                   stats_triton.py:148-169). One CTA per 128x128 output block; bf16/fp16 operands
//                   from the transposed staging XT [D, n] (both operands K-major, 128-byte swizzle);
//                   fp32 accumulation in TMEM in segments of 1024 rows, double-buffered so the
//                   epilogue folds a finished segment into register totals while the next one is
//                   computed (two-level fp32 summation: error of a 1024-row sum, not an n-row one);
//                   diagonal blocks load their single operand once. C is read and written once.
// atlas_count_gemm_i8  out[M, A] += masks[M, n_pad] . annT[A_pad, n_pad]^T, exact (kind::i8,
//                   int32 accumulate, int64 output), one CTA per 128 mask rows.
//
// Every wait is bounded: a wait that gives up records a code in the device status word
// (atlas_device_status) and the kernel finishes without further work.
#include <cuda.h>

#include "tc.cuh"

namespace atlas {

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int esize, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swz) {
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                              const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return fail(ATLAS_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    encode = reinterpret_cast<Encode>(fn);
  }
  (void)esize;
  if ((uintptr_t)base % 16 != 0 || row_stride_bytes % 16 != 0)
    return fail(ATLAS_ERR_ARG, "tensor map: base and row stride must be 16-byte aligned");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ATLAS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return ATLAS_OK;
}

namespace {
using namespace tc;

constexpr int kThreads = 192;
#ifndef ATLAS_GRAM_PAIR
#define ATLAS_GRAM_PAIR 0  // 1: 256 x 256 Gram tiles on CTA pairs (gram_pair_kernel)
#endif
#ifndef ATLAS_GRAM_WIDE
#define ATLAS_GRAM_WIDE 2  // 128 x 256 Gram tiles (gram_wide_kernel): 1 always, 0 never, 2 when they fill a wave
#endif

// ------------------------------------------------------------------------------------------ Gram
constexpr int GB = 128;               // output block (M = N = 128)
constexpr int GK = 64;                // bf16 elements per K chunk (128 bytes)
constexpr int G_STAGES = 6;
constexpr int G_SEG = 16;             // K chunks per TMEM segment (1024 rows)
constexpr uint32_t G_TILE = GB * GK * 2;  // 16 KB

struct GramSmem {
  uint8_t a[G_STAGES][G_TILE];
  uint8_t b[G_STAGES][G_TILE];
  uint64_t full[G_STAGES], empty[G_STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(kThreads, 1)
gram_tc_kernel(const __grid_constant__ CUtensorMap tmap, int64_t n, int64_t D, int nb, float* __restrict__ C,
               uint32_t idesc) {
  extern __shared__ uint8_t gram_raw[];
  GramSmem& s = *reinterpret_cast<GramSmem*>((reinterpret_cast<uintptr_t>(gram_raw) + 1023) & ~uintptr_t(1023));
  int t = blockIdx.x, bi = 0;
  while (t >= nb - bi) {
    t -= nb - bi;
    ++bi;
  }
  const int bj = bi + t;
  const bool diag = bi == bj;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (int)((n + GK - 1) / GK);
  const int nseg = (nk + G_SEG - 1) / G_SEG;
  if (threadIdx.x == 0) {
    for (int i = 0; i < G_STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&s.tmem_base, 256);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmap);
      const uint32_t bytes = diag ? G_TILE : 2 * G_TILE;
      for (int k = 0; k < nk; ++k) {
        const int st = k % G_STAGES;
        const uint32_t ph = (k / G_STAGES) & 1;
        if (k >= G_STAGES && !mbar_wait(&s.empty[st], ph ^ 1, 101)) break;
        mbar_arrive_expect_tx(&s.full[st], bytes);
        tma_load_2d(s.a[st], &tmap, k * GK, bi * GB, &s.full[st]);
        if (!diag) tma_load_2d(s.b[st], &tmap, k * GK, bj * GB, &s.full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int k = 0; k < nk; ++k) {
        const int st = k % G_STAGES;
        const uint32_t ph = (k / G_STAGES) & 1;
        const int seg = k / G_SEG, buf = seg & 1;
        const bool first = (k % G_SEG) == 0;
        if (first && seg >= 2 && !mbar_wait(&s.tempty[buf], ((seg >> 1) - 1) & 1, 102)) break;
        if (!mbar_wait(&s.full[st], ph, 103)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(s.a[st]);
        const uint32_t b_addr = diag ? a_addr : smem_u32(s.b[st]);
#pragma unroll
        for (int kk = 0; kk < GK / 16; ++kk)
          mma_f16(tmem + buf * GB, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                  (first && kk == 0) ? 0u : 1u);
        mma_commit(&s.empty[st]);
        if ((k % G_SEG) == G_SEG - 1 || k == nk - 1) mma_commit(&s.tfull[buf]);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lanes 32q..32q+31 belong to warps with warp % 4 == q
    const int row = q * 32 + lane;
    float tot[GB];
#pragma unroll
    for (int c = 0; c < GB; ++c) tot[c] = 0.f;
    bool ok = true;
    for (int seg = 0; seg < nseg; ++seg) {
      const int buf = seg & 1;
      if (!mbar_wait(&s.tfull[buf], (seg >> 1) & 1, 104)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < GB / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * GB + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) tot[c * 32 + j] += __uint_as_float(r[j]);
      }
      tc_fence_before();
      mbar_arrive(&s.tempty[buf]);
    }
    const int64_t gi = (int64_t)bi * GB + row;
    if (ok && gi < D) {
      float* crow = C + gi * D + (int64_t)bj * GB;
      const int64_t jmax = D - (int64_t)bj * GB;
      const bool vec = (D % 4 == 0) && jmax >= GB;
      if (vec) {
#pragma unroll
        for (int c = 0; c < GB; c += 4) {
          float4 v = *reinterpret_cast<float4*>(crow + c);
          v.x += tot[c]; v.y += tot[c + 1]; v.z += tot[c + 2]; v.w += tot[c + 3];
          *reinterpret_cast<float4*>(crow + c) = v;
        }
      } else {
#pragma unroll
        for (int c = 0; c < GB; ++c)
          if (c < jmax) crow[c] += tot[c];
      }
    }
  }
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 256);
}

// ------------------------------------------------------------------------------------- Gram (wide)
// 128 x 256 output tiles: per 64-row chunk the CTA loads 16 KB of A and 32 KB of B for twice the
// MMA work of a 128 x 128 tile (a third less L2 traffic per FLOP). TMEM holds two 128 x 256 fp32
// accumulators (all 512 columns) for the segment double buffer; eight epilogue warps split the 256
// columns so each thread keeps 128 register totals. A tile whose left 128-block lies below the
// diagonal (block row 2j+1 against column blocks 2j, 2j+1) computes it but never writes it.
constexpr int WN = 256;
constexpr int W_STAGES = 4;
constexpr uint32_t W_TILE_B = WN * GK * 2;  // 32 KB
constexpr int kWideThreads = 320;           // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue

struct GramWideSmem {
  uint8_t a[W_STAGES][G_TILE];
  uint8_t b[W_STAGES][W_TILE_B];
  uint64_t full[W_STAGES], empty[W_STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
};

__device__ __forceinline__ void wide_tile(int t, int nb, int& bi, int& bj2) {
  // tiles in column-superblock order: super-block j holds block rows 0 .. min(nb, 2j+2)-1
  int j = 0;
  while (true) {
    const int rows = min(nb, 2 * j + 2);
    if (t < rows) break;
    t -= rows;
    ++j;
  }
  bi = t;
  bj2 = j;
}

__global__ void __launch_bounds__(kWideThreads, 1)
gram_wide_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb, int64_t n, int64_t D,
                 int nb, float* __restrict__ C, uint32_t idesc) {
  extern __shared__ uint8_t wide_raw[];
  GramWideSmem& s = *reinterpret_cast<GramWideSmem*>((reinterpret_cast<uintptr_t>(wide_raw) + 1023) & ~uintptr_t(1023));
  int bi, bj2;
  wide_tile(blockIdx.x, nb, bi, bj2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (int)((n + GK - 1) / GK);
  const int nseg = (nk + G_SEG - 1) / G_SEG;
  if (threadIdx.x == 0) {
    for (int i = 0; i < W_STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 256);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&s.tmem_base, 512);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tma);
      prefetch_tmap(&tmb);
      for (int k = 0; k < nk; ++k) {
        const int st = k % W_STAGES;
        const uint32_t ph = (k / W_STAGES) & 1;
        if (k >= W_STAGES && !mbar_wait(&s.empty[st], ph ^ 1, 111)) break;
        mbar_arrive_expect_tx(&s.full[st], G_TILE + W_TILE_B);
        tma_load_2d(s.a[st], &tma, k * GK, bi * GB, &s.full[st]);
        tma_load_2d(s.b[st], &tmb, k * GK, bj2 * WN, &s.full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int k = 0; k < nk; ++k) {
        const int st = k % W_STAGES;
        const uint32_t ph = (k / W_STAGES) & 1;
        const int seg = k / G_SEG, buf = seg & 1;
        const bool first = (k % G_SEG) == 0;
        if (first && seg >= 2 && !mbar_wait(&s.tempty[buf], ((seg >> 1) - 1) & 1, 112)) break;
        if (!mbar_wait(&s.full[st], ph, 113)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(s.a[st]);
        const uint32_t b_addr = smem_u32(s.b[st]);
#pragma unroll
        for (int kk = 0; kk < GK / 16; ++kk)
          mma_f16(tmem + buf * WN, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                  (first && kk == 0) ? 0u : 1u);
        mma_commit(&s.empty[st]);
        if ((k % G_SEG) == G_SEG - 1 || k == nk - 1) mma_commit(&s.tfull[buf]);
      }
    }
  } else {
    const int q = warp & 3;             // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;   // 0: columns 0-127, 1: columns 128-255
    const int row = q * 32 + lane;
    float tot[GB];
#pragma unroll
    for (int c = 0; c < GB; ++c) tot[c] = 0.f;
    bool ok = true;
    for (int seg = 0; seg < nseg; ++seg) {
      const int buf = seg & 1;
      if (!mbar_wait(&s.tfull[buf], (seg >> 1) & 1, 114)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < GB / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * WN + half * GB + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) tot[c * 32 + j] += __uint_as_float(r[j]);
      }
      tc_fence_before();
      mbar_arrive(&s.tempty[buf]);
    }
    const int bj = 2 * bj2 + half;  // this thread's 128-column block
    const int64_t gi = (int64_t)bi * GB + row;
    if (ok && bj >= bi && bj < nb && gi < D) {
      float* crow = C + gi * D + (int64_t)bj * GB;
      const int64_t jmax = D - (int64_t)bj * GB;
      if ((D % 4 == 0) && jmax >= GB) {
#pragma unroll
        for (int c = 0; c < GB; c += 4) {
          float4 v = *reinterpret_cast<float4*>(crow + c);
          v.x += tot[c]; v.y += tot[c + 1]; v.z += tot[c + 2]; v.w += tot[c + 3];
          *reinterpret_cast<float4*>(crow + c) = v;
        }
      } else {
#pragma unroll
        for (int c = 0; c < GB; ++c)
          if (c < jmax) crow[c] += tot[c];
      }
    }
  }
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------------------ Gram (CTA pairs)
// 256 x 256 output tiles on a cluster of two CTAs (the two SMs of a TPC) sharing one
// tcgen05.mma.cta_group::2 of M = N = 256: CTA r loads rows 128r..128r+127 of the A block and of
// the B block (32 KB per 64-row chunk, half of what a single-SM 256 x 256 tile would need), the
// even CTA issues the MMAs, and each CTA's TMEM receives its 128 accumulator rows x 256 columns.
// Per SM that is the MMA work of a 128 x 256 tile for the operand bytes of a 128 x 128 one.
//   barriers: full[s] (even CTA; both CTAs' TMA bytes count on it), empty[s] and tfull[b] (one per
//   CTA, signalled by the even CTA's commits), tempty[b] (even CTA; one arrival per epilogue warp
//   of both CTAs). TMEM holds two 256-column accumulators (the segment double buffer).
// Diagonal tiles load their single operand once; the 128-block below the diagonal inside a
// diagonal tile (CTA 1, left half) is computed but never written.
constexpr int P_STAGES = 6;
constexpr int PN = 256;               // tile side (M = N)
constexpr int kPairThreads = 320;     // warp 0 TMA, warp 1 MMA + TMEM owner, warps 2-9 epilogue
constexpr int kPairEpiWarps = 8;

struct GramPairSmem {
  uint8_t a[P_STAGES][G_TILE];
  uint8_t b[P_STAGES][G_TILE];
  uint64_t full[P_STAGES], empty[P_STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
gram_pair_kernel(const __grid_constant__ CUtensorMap tmap, int64_t n, int64_t D, int nb2, int nb, float* __restrict__ C,
                 uint32_t idesc) {
  extern __shared__ uint8_t pair_raw[];
  GramPairSmem& s = *reinterpret_cast<GramPairSmem*>((reinterpret_cast<uintptr_t>(pair_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t rank = cluster_rank();
  int t = blockIdx.x >> 1, bi = 0;
  while (t >= nb2 - bi) {
    t -= nb2 - bi;
    ++bi;
  }
  const int bj = bi + t;
  const bool diag = bi == bj;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (int)((n + GK - 1) / GK);
  const int nseg = (nk + G_SEG - 1) / G_SEG;
  if (threadIdx.x == 0) {
    for (int i = 0; i < P_STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 2 * kPairEpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(&s.tmem_base, 512);
  __syncthreads();
  tc_fence_after();
  cluster_sync();  // the peer's barriers are initialised before anything signals them
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmap);
      const uint32_t bytes = 2u * (diag ? G_TILE : 2 * G_TILE);  // both CTAs' loads of one chunk
      const int32_t arow = bi * PN + (int32_t)rank * GB, brow = bj * PN + (int32_t)rank * GB;
      for (int k = 0; k < nk; ++k) {
        const int st = k % P_STAGES;
        const uint32_t ph = (k / P_STAGES) & 1;
        if (k >= P_STAGES && !mbar_wait(&s.empty[st], ph ^ 1, 121)) break;
        if (rank == 0) mbar_arrive_expect_tx(&s.full[st], bytes);
        const uint32_t fb = cluster_addr(&s.full[st], 0);
        tma_load_2d_pair(s.a[st], &tmap, k * GK, arow, fb);
        if (!diag) tma_load_2d_pair(s.b[st], &tmap, k * GK, brow, fb);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      for (int k = 0; k < nk; ++k) {
        const int st = k % P_STAGES;
        const uint32_t ph = (k / P_STAGES) & 1;
        const int seg = k / G_SEG, buf = seg & 1;
        const bool first = (k % G_SEG) == 0;
        if (first && seg >= 2 && !mbar_wait(&s.tempty[buf], ((seg >> 1) - 1) & 1, 122)) break;
        if (!mbar_wait(&s.full[st], ph, 123)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(s.a[st]);
        const uint32_t b_addr = diag ? a_addr : smem_u32(s.b[st]);
#pragma unroll
        for (int kk = 0; kk < GK / 16; ++kk)
          mma_f16_pair(tmem + buf * PN, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                       (first && kk == 0) ? 0u : 1u);
        mma_commit_pair(cluster_addr(&s.empty[st], 0));
        mma_commit_pair(cluster_addr(&s.empty[st], 1));
        if ((k % G_SEG) == G_SEG - 1 || k == nk - 1) {
          mma_commit_pair(cluster_addr(&s.tfull[buf], 0));
          mma_commit_pair(cluster_addr(&s.tfull[buf], 1));
        }
      }
    }
  } else {
    const int q = warp & 3;            // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;  // 0: columns 0-127 of the tile, 1: columns 128-255
    const int row = q * 32 + lane;
    const uint32_t tempty0 = cluster_addr(&s.tempty[0], 0), tempty1 = cluster_addr(&s.tempty[1], 0);
    float tot[GB];
#pragma unroll
    for (int c = 0; c < GB; ++c) tot[c] = 0.f;
    bool ok = true;
    for (int seg = 0; seg < nseg; ++seg) {
      const int buf = seg & 1;
      if (!mbar_wait(&s.tfull[buf], (seg >> 1) & 1, 124)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < GB / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * PN + half * GB + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) tot[c * 32 + j] += __uint_as_float(r[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(buf ? tempty1 : tempty0);
    }
    const int br = 2 * bi + (int)rank, bc = 2 * bj + half;  // 128-blocks of this thread's rows / columns
    const int64_t gi = (int64_t)br * GB + row;
    if (ok && bc >= br && bc < nb && gi < D) {
      float* crow = C + gi * D + (int64_t)bc * GB;
      const int64_t jmax = D - (int64_t)bc * GB;
      if ((D % 4 == 0) && jmax >= GB) {
#pragma unroll
        for (int c = 0; c < GB; c += 4) {
          float4 v = *reinterpret_cast<float4*>(crow + c);
          v.x += tot[c]; v.y += tot[c + 1]; v.z += tot[c + 2]; v.w += tot[c + 3];
          *reinterpret_cast<float4*>(crow + c) = v;
        }
      } else {
#pragma unroll
        for (int c = 0; c < GB; ++c)
          if (c < jmax) crow[c] += tot[c];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // every MMA, TMEM read and remote arrival of both CTAs is done
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, 512);
}

// ------------------------------------------------------------------------------------------ int8
constexpr int IM = 128;               // mask rows per CTA
constexpr int IK = 128;               // int8 K chunk (128 bytes)
constexpr int I_STAGES = 4;

template <int AP>
struct I8Smem {
  uint8_t a[I_STAGES][IM * IK];
  uint8_t b[I_STAGES][AP * IK];
  uint64_t full[I_STAGES], empty[I_STAGES], tfull;
  uint32_t tmem_base;
};

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

template <int AP>
__global__ void __launch_bounds__(kThreads, 1)
count_i8_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, int64_t M,
                   int64_t n_pad, int64_t* __restrict__ out, int64_t A, uint32_t tcols) {
  extern __shared__ uint8_t i8_raw[];
  I8Smem<AP>& s = *reinterpret_cast<I8Smem<AP>*>((reinterpret_cast<uintptr_t>(i8_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = (int64_t)blockIdx.x * IM;
  const int nk = (int)(n_pad / IK);
  if (threadIdx.x == 0) {
    for (int i = 0; i < I_STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    mbar_init(&s.tfull, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&s.tmem_base, tcols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  constexpr uint32_t idesc = idesc_s8_s32(IM, AP);
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_b);
      for (int k = 0; k < nk; ++k) {
        const int st = k % I_STAGES;
        const uint32_t ph = (k / I_STAGES) & 1;
        if (k >= I_STAGES && !mbar_wait(&s.empty[st], ph ^ 1, 201)) break;
        mbar_arrive_expect_tx(&s.full[st], IM * IK + AP * IK);
        tma_load_2d(s.a[st], &tm_a, k * IK, (int32_t)m0, &s.full[st]);
        tma_load_2d(s.b[st], &tm_b, k * IK, 0, &s.full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int k = 0; k < nk; ++k) {
        const int st = k % I_STAGES;
        const uint32_t ph = (k / I_STAGES) & 1;
        if (!mbar_wait(&s.full[st], ph, 202)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(s.a[st]), b_addr = smem_u32(s.b[st]);
#pragma unroll
        for (int kk = 0; kk < IK / 32; ++kk)
          mma_i8(tmem, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                 (k == 0 && kk == 0) ? 0u : 1u);
        mma_commit(&s.empty[st]);
      }
      mma_commit(&s.tfull);
    }
  } else {
    const int q = warp & 3;
    const int64_t m = m0 + q * 32 + lane;
    if (mbar_wait(&s.tfull, 0, 203)) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < AP; c += 16) {
        uint32_t r[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + c, r);
        tmem_ld_wait();
        if (m < M) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c + j < A) out[m * A + c + j] += (int64_t)(int32_t)r[j];
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, tcols);
}

template <int AP>
int launch_i8(const int8_t* masks, int64_t M, int64_t n_pad, const int8_t* annT, int64_t* out, int64_t A,
              cudaStream_t st) {
  CUtensorMap ta, tb;
  if (int e = make_tmap_2d(&ta, masks, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, n_pad, M, n_pad, IK, IM,
                           CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  if (int e = make_tmap_2d(&tb, annT, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, n_pad, AP, n_pad, IK, AP,
                           CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  const size_t smem = sizeof(I8Smem<AP>) + 1024;
  if (cudaFuncSetAttribute(count_i8_tc_kernel<AP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return fail(ATLAS_ERR_CUDA, "count_gemm_i8: cannot reserve %zu bytes of shared memory", smem);
  uint32_t tcols = 32;
  while (tcols < (uint32_t)AP) tcols <<= 1;
  count_i8_tc_kernel<AP><<<(unsigned)((M + IM - 1) / IM), kThreads, smem, st>>>(ta, tb, M, n_pad, out, A, tcols);
  return check_launch("atlas_count_gemm_i8");
}

// ------------------------------------------------------------------------------------------------
// Fused subsample statistics + enrichment (bf16 staging): one pass over XT gives the moments and
// bin counts of atlas_sub_stats AND the enrichment contingencies of atlas_count_gemm_i8, without
// the int8 masks ever reaching HBM. A CTA owns 128 columns d (the M rows of every mask plane) and a
// range of 128-row slabs of the subsample:
//   16 producer warps: 4 threads per column, 32 rows each per slab, loaded one slab ahead. Each
//     thread compares its rows against the column's edges as packed bf16 pairs (exact for bf16
//     inputs, as atlas_sub_stats), counts by popcount, sums in fp32 per 8 rows and fp64 across, and
//     writes the 0/1 bytes of every (pole, level) plane straight into the UMMA K-major
//     128-byte-swizzled shared-memory tile (row d, byte i: 16-byte chunk (i / 16) ^ (d % 8)); the
//     annotation one-hots of the slab are copied into the same layout. After a proxy fence each
//     warp arrives on the stage's mbarrier (16 arrivals complete it); warps run ahead of each other
//     up to the two stages.
//   the last producer warp also issues the MMAs: once a stage is full, per plane four tcgen05.mma
//     kind::i8 (M=128, N=A_pad, K=32) into its own TMEM accumulator (int32, exact), then a commit
//     that frees the stage (16 warps, 128 registers per thread).
//   epilogue: warps 0-3 read the accumulators (lane = column) and add them into enr (int64).
// Column sums of a CTA range are fp64 partials; with several ranges per column the last CTA to
// finish (ticket counter) adds the partials in range order, so the result does not depend on CTA
// timing. Bin counts and contingencies are integers added atomically.
constexpr int SE_M = 128;
constexpr int SE_K = 128;
constexpr int SE_PW = 16;                // producer warps; the last one also issues the MMAs
constexpr int SE_THREADS = SE_PW * 32;
constexpr int SE_STAGES = 2;
constexpr int SE_PLANES = 6;
constexpr int SE_MAXB = 8;

struct SELevels {
  int v[4];
};

template <int AP>
struct SESmem {
  uint8_t a[SE_STAGES][SE_PLANES][SE_M * SE_K];
  uint8_t b[SE_STAGES][AP * SE_K];
  uint64_t full[SE_STAGES], empty[SE_STAGES], tfull;
  uint32_t tmem_base;
  int last;
  int abort;  // a producer's bounded wait gave up: the others skip the remaining slabs too
};

__device__ __forceinline__ void named_sync_producers() {
  asm volatile("bar.sync 1, %0;" ::"r"(SE_PW * 32) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Packed bf16 compares of two register words: 0xFFFF in each half where the compare holds
// (ordered: false for NaN), the semantics of __hge2_mask / __hle2_mask without a round trip of
// the operands through memory.
__device__ __forceinline__ uint32_t bf2_ge_mask(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("set.ge.u32.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_le_mask(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("set.le.u32.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t bf16x2_bits(float v) {
  const uint32_t h = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
  return h | (h << 16);
}

// 0/1 bytes of 8 rows from the four 32-bit compare masks (0xFFFF per true half) of a vector
__device__ __forceinline__ uint64_t mask_bytes(const uint32_t (&m)[4]) {
  return (uint64_t)(__byte_perm(m[0], m[1], 0x6420) & 0x01010101u) |
         ((uint64_t)(__byte_perm(m[2], m[3], 0x6420) & 0x01010101u) << 32);
}

template <int AP, int NB>
__global__ void __launch_bounds__(SE_THREADS, 1)
stats_enrich_kernel(const __nv_bfloat16* __restrict__ XT, int64_t ldx, int64_t col0, int64_t n, int64_t D,
                    const float* __restrict__ E0, const float* __restrict__ E1, int B, SELevels lev, int NL,
                    const int8_t* __restrict__ annT, int64_t n_pad, int A, double* __restrict__ sum,
                    double* __restrict__ sq, unsigned long long* __restrict__ bins, unsigned long long* __restrict__ enr,
                    double* __restrict__ part, unsigned int* __restrict__ tickets, int spp, int n_slabs,
                    uint32_t tcols) {
  extern __shared__ uint8_t se_raw[];
  SESmem<AP>& s = *reinterpret_cast<SESmem<AP>*>((reinterpret_cast<uintptr_t>(se_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t d0 = (int64_t)blockIdx.x * SE_M;
  const int k_begin = blockIdx.y * spp;
  const int k_end = min(n_slabs, k_begin + spp);
  const int nk = k_end - k_begin;
  const int planes = 2 * NL;
  if (threadIdx.x == 0) {
    for (int i = 0; i < SE_STAGES; ++i) {
      mbar_init(&s.full[i], SE_PW);  // one arrival per producer warp
      mbar_init(&s.empty[i], 1);
    }
    mbar_init(&s.tfull, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  constexpr int kMmaWarp = SE_PW - 1;
  if (warp == kMmaWarp) tmem_alloc(&s.tmem_base, tcols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  {
    // ---------------------------------------------------------------- producers
    const int t = threadIdx.x;
    const int r = t >> 2, prt = t & 3;
    const int64_t d = d0 + r;
    const bool dok = d < D;
    uint32_t pe[NB], ne[NB];  // edges as packed bf16 pairs
    uint32_t levbits = 0;     // bits 3b..3b+2: the levels j sitting on edge b
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const bool ok = dok;
      const uint32_t hp = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_ru(ok ? E0[d * B + b] : __int_as_float(0x7F800000)));
      const uint32_t hn = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rd(ok ? -E1[d * B + b] : __int_as_float(0xFF800000)));
      pe[b] = hp | (hp << 16);
      ne[b] = hn | (hn << 16);
#pragma unroll
      for (int j = 0; j < 3; ++j)
        if (j < NL && lev.v[j] == b) levbits |= 1u << (3 * b + j);
    }
    int c0[NB], c1[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) c0[b] = c1[b] = 0;
    double acc_s = 0.0, acc_q = 0.0;
    const __nv_bfloat16* col = XT + (dok ? d : 0) * ldx + col0;
    // the slab's 4 chunks of this thread (and, for t < AP*8, one 16-byte chunk of the one-hots),
    // loaded one slab ahead of their use so the global-load latency overlaps the compares
#define SE_LOAD_SLAB(KK, RAW0, RAW1, RAW2, RAW3, ANN)                                                        \
  {                                                                                                         \
    const int64_t row0_ = (int64_t)(k_begin + (KK)) * SE_K;                                                 \
    const int64_t i0_ = row0_ + prt * 8;                                                                    \
    RAW0 = (dok && i0_ < n) ? __ldcs(reinterpret_cast<const uint4*>(col + i0_)) : make_uint4(0u, 0u, 0u, 0u);  \
    RAW1 = (dok && i0_ + 32 < n) ? __ldcs(reinterpret_cast<const uint4*>(col + i0_ + 32)) : make_uint4(0u, 0u, 0u, 0u); \
    RAW2 = (dok && i0_ + 64 < n) ? __ldcs(reinterpret_cast<const uint4*>(col + i0_ + 64)) : make_uint4(0u, 0u, 0u, 0u); \
    RAW3 = (dok && i0_ + 96 < n) ? __ldcs(reinterpret_cast<const uint4*>(col + i0_ + 96)) : make_uint4(0u, 0u, 0u, 0u); \
    if (t < AP * 8) ANN = *reinterpret_cast<const uint4*>(annT + (int64_t)(t >> 3) * n_pad + row0_ + (t & 7) * 16); \
  }
    uint4 c0v, c1v, c2v, c3v, n0v, n1v, n2v, n3v;
    uint4 cur_ann = make_uint4(0u, 0u, 0u, 0u), nxt_ann = cur_ann;
    c0v = c1v = c2v = c3v = n0v = n1v = n2v = n3v = cur_ann;
    if (nk > 0) SE_LOAD_SLAB(0, c0v, c1v, c2v, c3v, cur_ann)
    bool ok_run = true;
    for (int k = 0; k < nk && ok_run; ++k) {
      const int st = k % SE_STAGES;
      const uint32_t ph = (k / SE_STAGES) & 1;
      if (*reinterpret_cast<volatile int*>(&s.abort)) {
        ok_run = false;
        break;
      }
      if (k + 1 < nk) SE_LOAD_SLAB(k + 1, n0v, n1v, n2v, n3v, nxt_ann)
      if (k >= SE_STAGES && !mbar_wait(&s.empty[st], ph ^ 1, 212)) {
        s.abort = 1;  // the other warps see it before their next slab
        ok_run = false;
        break;
      }
      const int64_t slab_row0 = (int64_t)(k_begin + k) * SE_K;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int c = q * 4 + prt;  // 8-row chunk of the slab
        const int64_t i = slab_row0 + c * 8;
        const uint4 cq = q == 0 ? c0v : (q == 1 ? c1v : (q == 2 ? c2v : c3v));
        uint32_t w4[4] = {cq.x, cq.y, cq.z, cq.w};
        const bool full = dok && i + 8 <= n;
        uint32_t vm[4] = {0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu};
        if (!full) {  // the ragged end of the subsample (or a column past D): rows >= n neither count nor match
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const int64_t rr = i + 2 * w;
            vm[w] = dok ? ((rr < n ? 0x0000FFFFu : 0u) | (rr + 1 < n ? 0xFFFF0000u : 0u)) : 0u;
            w4[w] &= vm[w];
          }
        }
        {
          float s32 = 0.0f, q32 = 0.0f;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const float lo = __uint_as_float(w4[w] << 16), hi = __uint_as_float(w4[w] & 0xFFFF0000u);
            s32 += lo;
            s32 += hi;
            q32 = fmaf(lo, lo, q32);
            q32 = fmaf(hi, hi, q32);
          }
          acc_s += (double)s32;
          acc_q += (double)q32;
        }
        const uint32_t off = (uint32_t)r * 128u + ((uint32_t)((c >> 1) ^ (r & 7)) << 4) + ((uint32_t)(c & 1) << 3);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          uint32_t mp[4], mn[4];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            mp[w] = bf2_ge_mask(w4[w], pe[b]);
            mn[w] = bf2_le_mask(w4[w], ne[b]);
            if (!full) {
              mp[w] &= vm[w];
              mn[w] &= vm[w];
            }
          }
          c0[b] += __popc(mp[0]) + __popc(mp[1]) + __popc(mp[2]) + __popc(mp[3]);
          c1[b] += __popc(mn[0]) + __popc(mn[1]) + __popc(mn[2]) + __popc(mn[3]);
          const uint32_t lm = (levbits >> (3 * b)) & 7u;
          if (lm) {  // this edge is an enrichment level: its 0/1 bytes go straight to the plane tiles
            const uint64_t bp = mask_bytes(mp), bn = mask_bytes(mn);
#pragma unroll
            for (int j = 0; j < 3; ++j)
              if (lm & (1u << j)) {
                *reinterpret_cast<uint64_t*>(s.a[st][j] + off) = bp;
                *reinterpret_cast<uint64_t*>(s.a[st][NL + j] + off) = bn;
              }
          }
        }
      }
      if (t < AP * 8) {  // the slab's annotation one-hots: row a, 16-byte chunk c16
        const int a_row = t >> 3, c16 = t & 7;
        *reinterpret_cast<uint4*>(s.b[st] + a_row * 128 + ((c16 ^ (a_row & 7)) << 4)) = cur_ann;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.full[st]);  // one arrival per producer warp
      if (warp == kMmaWarp) {  // once every warp has filled the stage: its MMAs, then a commit that frees it
        if (lane == 0) {
          if (mbar_wait(&s.full[st], ph, 211)) {
            tc_fence_after();
            constexpr uint32_t idesc = idesc_s8_s32(SE_M, AP);
            const uint32_t b_addr = smem_u32(s.b[st]);
            for (int pl = 0; pl < planes; ++pl) {
              const uint32_t a_addr = smem_u32(s.a[st][pl]);
#pragma unroll
              for (int kk = 0; kk < SE_K / 32; ++kk)
                mma_i8(tmem + (uint32_t)(pl * AP), sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32),
                       idesc, (k == 0 && kk == 0) ? 0u : 1u);
            }
            mma_commit(&s.empty[st]);
          } else {
            s.abort = 1;
          }
        }
        __syncwarp();
      }
      c0v = n0v;
      c1v = n1v;
      c2v = n2v;
      c3v = n3v;
      cur_ann = nxt_ann;
    }
#undef SE_LOAD_SLAB
    if (warp == kMmaWarp && lane == 0) mma_commit(&s.tfull);  // completes when every MMA above has
    // ---------------------------------------------------------------- column statistics
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      acc_s += __shfl_xor_sync(0xFFFFFFFFu, acc_s, o);
      acc_q += __shfl_xor_sync(0xFFFFFFFFu, acc_q, o);
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        c0[b] += __shfl_xor_sync(0xFFFFFFFFu, c0[b], o);
        c1[b] += __shfl_xor_sync(0xFFFFFFFFu, c1[b], o);
      }
    }
    if (prt == 0 && dok) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const int nx0 = (b + 1 < NB) ? c0[b + 1] : 0;
        const int nx1 = (b + 1 < NB) ? c1[b + 1] : 0;
        const unsigned long long v0 = (unsigned long long)((c0[b] - nx0) >> 4);  // 16 mask bits per row
        const unsigned long long v1 = (unsigned long long)((c1[b] - nx1) >> 4);
        if (v0) atomicAdd(bins + d * B + b, v0);
        if (v1) atomicAdd(bins + (D + d) * B + b, v1);
      }
      if (gridDim.y == 1) {
        sum[d] += acc_s;
        sq[d] += acc_q;
      } else {
        part[((int64_t)blockIdx.y * 2) * D + d] = acc_s;
        part[((int64_t)blockIdx.y * 2 + 1) * D + d] = acc_q;
      }
    }
    // ---------------------------------------------------------------- contingencies
    if (warp < 4 && nk > 0 && mbar_wait(&s.tfull, 0, 213)) {
      tc_fence_after();
      const int64_t dd = d0 + warp * 32 + lane;
      for (int pl = 0; pl < planes; ++pl) {
        const int pole = pl / NL, j = pl - pole * NL;
#pragma unroll
        for (int c = 0; c < AP; c += 16) {
          uint32_t v[16];
          tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(pl * AP + c), v);
          tmem_ld_wait();
          if (dd < D) {
            unsigned long long* row = enr + (((int64_t)pole * NL + j) * D + dd) * A;
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              if (c + jj < A && v[jj]) atomicAdd(row + c + jj, (unsigned long long)v[jj]);
          }
        }
      }
      tc_fence_before();
    }
  }
  // ---------------------------------------------------------------- ordered sum of the range partials
  if (gridDim.y > 1) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned int ticket = atomicAdd(tickets + blockIdx.x, 1u);
      s.last = ticket == gridDim.y - 1;
    }
    __syncthreads();
    if (s.last) {
      __threadfence();
      if (threadIdx.x < SE_M) {
        const int64_t d = d0 + threadIdx.x;
        if (d < D) {
          double S = 0.0, Q = 0.0;
          for (unsigned int y = 0; y < gridDim.y; ++y) {
            S += __ldcg(part + ((int64_t)y * 2) * D + d);
            Q += __ldcg(part + ((int64_t)y * 2 + 1) * D + d);
          }
          sum[d] += S;
          sq[d] += Q;
        }
      }
      if (threadIdx.x == 0) tickets[blockIdx.x] = 0u;
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols);
  }
}

template <int AP, int NB>
int launch_stats_enrich_b(const __nv_bfloat16* XT, int64_t ldx, int64_t col0, int64_t n, int64_t D, const float* E0,
                        const float* E1, int B, const SELevels& lev, int NL, const int8_t* annT, int64_t n_pad, int A,
                        double* sum, double* sq, int64_t* bins, int64_t* enr, void* ws, cudaStream_t st) {
  const int n_slabs = (int)((n + SE_K - 1) / SE_K);
  const int dtiles = (int)((D + SE_M - 1) / SE_M);
  int ks = num_sms() / dtiles;
  ks = ks < 1 ? 1 : (ks > 16 ? 16 : ks);
  if (ks > n_slabs) ks = n_slabs;
  const int spp = (n_slabs + ks - 1) / ks;
  ks = (n_slabs + spp - 1) / spp;  // every range gets at least one slab
  unsigned int* tickets = reinterpret_cast<unsigned int*>(ws);
  double* part = reinterpret_cast<double*>(reinterpret_cast<uint8_t*>(ws) + ((dtiles * 4 + 255) / 256) * 256);
  const size_t smem = sizeof(SESmem<AP>) + 1024;
  static bool attr_set[64] = {};  // once per device and instantiation (one launch per layer and batch)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cudaFuncSetAttribute(stats_enrich_kernel<AP, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return fail(ATLAS_ERR_CUDA, "sub_stats_enrich: cannot reserve %zu bytes of shared memory", smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  uint32_t tcols = 32;
  while (tcols < (uint32_t)(2 * NL * AP)) tcols <<= 1;
  stats_enrich_kernel<AP, NB><<<dim3((unsigned)dtiles, (unsigned)ks), SE_THREADS, smem, st>>>(
      XT, ldx, col0, n, D, E0, E1, B, lev, NL, annT, n_pad, A, sum, sq, reinterpret_cast<unsigned long long*>(bins),
      reinterpret_cast<unsigned long long*>(enr), part, tickets, spp, n_slabs, tcols);
  return check_launch("atlas_sub_stats_enrich");
}

template <int AP>
int launch_stats_enrich(const __nv_bfloat16* XT, int64_t ldx, int64_t col0, int64_t n, int64_t D, const float* E0,
                        const float* E1, int B, const SELevels& lev, int NL, const int8_t* annT, int64_t n_pad, int A,
                        double* sum, double* sq, int64_t* bins, int64_t* enr, void* ws, cudaStream_t st) {
  switch (B) {
#define ATLAS_SE_B(NBV) \
  case NBV:             \
    return launch_stats_enrich_b<AP, NBV>(XT, ldx, col0, n, D, E0, E1, B, lev, NL, annT, n_pad, A, sum, sq, bins, enr, ws, st);
    ATLAS_SE_B(1) ATLAS_SE_B(2) ATLAS_SE_B(3) ATLAS_SE_B(4) ATLAS_SE_B(5) ATLAS_SE_B(6) ATLAS_SE_B(7) ATLAS_SE_B(8)
#undef ATLAS_SE_B
    default: return fail(ATLAS_ERR_ARG, "sub_stats_enrich: B must be 1..%d", SE_MAXB);
  }
}

}  // namespace

// fp32 activations keep an exact-FMA CUDA-core Gram (tcgen05 has no IEEE fp32 operand kind)
int gram_upper_f32(const float* XT, int64_t ldx, int64_t n, int64_t D, float* C, cudaStream_t st);

}  // namespace atlas

using namespace atlas;

namespace atlas {
int filter_device_status(int* v, int reset);  // filter.cu's bounded waits
}

// Status of the bounded waits: the first code recorded by the tensor-core kernels (this file) or,
// when they recorded none, by the bulk-fed filter (filter.cu); each file keeps its own word.
extern "C" int atlas_device_status(int* status_host, int reset) {
  int v = 0, vf = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_device_status, sizeof(int)) != cudaSuccess)
    return fail(ATLAS_ERR_CUDA, "device_status: read failed");
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(tc::g_device_status, &z, sizeof(int)) != cudaSuccess)
      return fail(ATLAS_ERR_CUDA, "device_status: reset failed");
  }
  if (atlas::filter_device_status(&vf, reset) != ATLAS_OK) return fail(ATLAS_ERR_CUDA, "device_status: read failed");
  if (status_host) *status_host = v ? v : vf;
  return ATLAS_OK;
}

// Writes `code` into this file's status word (synchronous). Lets a host exercise its error path
// (check_errors, result, checkpoint refusal) without making a device wait give up.
extern "C" int atlas_device_status_set(int code) {
  if (cudaMemcpyToSymbol(tc::g_device_status, &code, sizeof(int)) != cudaSuccess)
    return fail(ATLAS_ERR_CUDA, "device_status_set: write failed");
  return ATLAS_OK;
}

extern "C" int atlas_gram_upper(const void* XT, int dtype, int64_t ldx, int64_t n, int64_t D, float* C, void* stream) {
  ATLAS_REQUIRE(n >= 0 && D >= 0 && ldx >= n, "gram_upper: bad sizes");
  if (n == 0 || D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(XT && C, "gram_upper: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == ATLAS_F32) return gram_upper_f32((const float*)XT, ldx, n, D, C, st);
  ATLAS_REQUIRE(dtype == ATLAS_BF16 || dtype == ATLAS_F16, "gram_upper: unknown dtype %d", dtype);
  ATLAS_REQUIRE(ldx % 8 == 0 && (uintptr_t)XT % 16 == 0, "gram_upper: XT must be 16-byte aligned with ldx %% 8 == 0");
  ATLAS_REQUIRE(D < (1LL << 31) && n < (1LL << 31), "gram_upper: sizes exceed int32 coordinates");
  CUtensorMap tm;
  if (int e = make_tmap_2d(&tm, XT, dtype == ATLAS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           2, (uint64_t)n, (uint64_t)D, (uint64_t)ldx * 2, GK, GB, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  const int nb = (int)((D + GB - 1) / GB);
#if ATLAS_GRAM_PAIR
  {
    const int nb2 = (int)((D + PN - 1) / PN);
    const int64_t tiles = (int64_t)nb2 * (nb2 + 1) / 2;
    const size_t smem = sizeof(GramPairSmem) + 1024;
    if (cudaFuncSetAttribute(gram_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return fail(ATLAS_ERR_CUDA, "gram_upper: cannot reserve %zu bytes of shared memory", smem);
    const uint32_t idesc = dtype == ATLAS_BF16 ? tc::idesc_bf16_f32(PN, PN) : tc::idesc_f16_f32(PN, PN);
    gram_pair_kernel<<<(unsigned)(2 * tiles), kPairThreads, smem, st>>>(tm, n, D, nb2, nb, C, idesc);
    return check_launch("atlas_gram_upper");
  }
#endif
  // 128 x 256 tiles move a third fewer operand bytes per FLOP than 128 x 128 ones (the narrow
  // tiles are L2-to-SM bound at about half the tensor peak), but they come in half the number: use
  // them once they fill at least one wave of the GPU.
  const int nb2w = (nb + 1) / 2;
  int64_t wide_tiles = 0;
  for (int j = 0; j < nb2w; ++j) wide_tiles += (nb < 2 * j + 2 ? nb : 2 * j + 2);
  if (ATLAS_GRAM_WIDE == 1 || (ATLAS_GRAM_WIDE == 2 && wide_tiles >= num_sms())) {
    CUtensorMap tmb;
    if (int e = make_tmap_2d(&tmb, XT, dtype == ATLAS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             2, (uint64_t)n, (uint64_t)D, (uint64_t)ldx * 2, GK, WN, CU_TENSOR_MAP_SWIZZLE_128B))
      return e;
    const size_t smem = sizeof(GramWideSmem) + 1024;
    if (cudaFuncSetAttribute(gram_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return fail(ATLAS_ERR_CUDA, "gram_upper: cannot reserve %zu bytes of shared memory", smem);
    const uint32_t idesc = dtype == ATLAS_BF16 ? tc::idesc_bf16_f32(GB, WN) : tc::idesc_f16_f32(GB, WN);
    gram_wide_kernel<<<(unsigned)wide_tiles, kWideThreads, smem, st>>>(tm, tmb, n, D, nb, C, idesc);
    return check_launch("atlas_gram_upper");
  }
  const int64_t tiles = (int64_t)nb * (nb + 1) / 2;
  const size_t smem = sizeof(GramSmem) + 1024;
  if (cudaFuncSetAttribute(gram_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return fail(ATLAS_ERR_CUDA, "gram_upper: cannot reserve %zu bytes of shared memory", smem);
  const uint32_t idesc = dtype == ATLAS_BF16 ? tc::idesc_bf16_f32(GB, GB) : tc::idesc_f16_f32(GB, GB);
  gram_tc_kernel<<<(unsigned)tiles, kThreads, smem, st>>>(tm, n, D, nb, C, idesc);
  return check_launch("atlas_gram_upper");
}

extern "C" int atlas_count_gemm_i8(const int8_t* masks, int64_t M, int64_t n_pad, const int8_t* annT, int64_t A_pad,
                                   int64_t* out, int64_t A, void* stream) {
  ATLAS_REQUIRE(M >= 0 && n_pad >= 0 && n_pad % IK == 0, "count_gemm_i8: n_pad must be a multiple of %d", IK);
  ATLAS_REQUIRE(A_pad % 16 == 0 && A_pad >= 16 && A_pad <= 256 && A >= 0 && A <= A_pad, "count_gemm_i8: bad A/A_pad");
  if (M == 0 || n_pad == 0 || A == 0) return ATLAS_OK;
  ATLAS_REQUIRE(masks && annT && out, "count_gemm_i8: null pointer");
  ATLAS_REQUIRE((uintptr_t)masks % 16 == 0 && (uintptr_t)annT % 16 == 0, "count_gemm_i8: operands must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  switch (A_pad) {
    case 16: return launch_i8<16>(masks, M, n_pad, annT, out, A, st);
    case 32: return launch_i8<32>(masks, M, n_pad, annT, out, A, st);
    case 48: return launch_i8<48>(masks, M, n_pad, annT, out, A, st);
    case 64: return launch_i8<64>(masks, M, n_pad, annT, out, A, st);
    case 96: return launch_i8<96>(masks, M, n_pad, annT, out, A, st);
    case 128: return launch_i8<128>(masks, M, n_pad, annT, out, A, st);
    case 256: return launch_i8<256>(masks, M, n_pad, annT, out, A, st);
    default: return fail(ATLAS_ERR_UNSUPPORTED, "count_gemm_i8: A_pad %lld not instantiated", (long long)A_pad);
  }
}

// ------------------------------------------------------------------------------------------------
// Fused subsample statistics + enrichment (see stats_enrich_kernel).
extern "C" int atlas_stats_enrich_supported(int dtype, int64_t B, int64_t NL, int64_t A_pad) {
  return dtype == ATLAS_BF16 && B >= 1 && B <= SE_MAXB && NL >= 1 && NL <= 3 && (A_pad == 16 || A_pad == 32 ||
                                                                               A_pad == 48);
}

extern "C" int64_t atlas_stats_enrich_ws_bytes(int64_t D, int64_t n) {
  if (D <= 0) return 256;
  const int64_t dtiles = (D + SE_M - 1) / SE_M;
  return ((dtiles * 4 + 255) / 256) * 256 + 16 * 2 * D * 8;
}

extern "C" int atlas_sub_stats_enrich(const void* XT, int dtype, int64_t ldx, int64_t col0, int64_t n, int64_t D,
                                      const float* E0, const float* E1, int64_t B, const int32_t* levels_host,
                                      int64_t NL, double* sum, double* sq, int64_t* bins, const int8_t* annT,
                                      int64_t A_pad, int64_t n_pad, int64_t* enr, int64_t A, void* ws,
                                      int64_t ws_bytes, void* stream) {
  ATLAS_REQUIRE(atlas_stats_enrich_supported(dtype, B, NL, A_pad),
                "sub_stats_enrich: unsupported (bf16 staging, 1..%d bins, 1..3 levels, A_pad 16/32/48 only)", SE_MAXB);
  ATLAS_REQUIRE(n >= 0 && D >= 0 && A >= 1 && A <= A_pad, "sub_stats_enrich: bad sizes");
  if (n == 0 || D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(XT && E0 && E1 && sum && sq && bins && annT && enr && ws && levels_host, "sub_stats_enrich: null pointer");
  ATLAS_REQUIRE(col0 % 8 == 0 && ldx % 8 == 0 && (col0 + ((n + 7) / 8) * 8) <= ldx && (uintptr_t)XT % 16 == 0,
                "sub_stats_enrich: XT must be 16-byte aligned, col0 and ldx multiples of 8, columns inside ldx");
  ATLAS_REQUIRE(n_pad % 128 == 0 && n_pad >= n && (uintptr_t)annT % 16 == 0, "sub_stats_enrich: n_pad %% 128 == 0, >= n");
  ATLAS_REQUIRE(ws_bytes >= atlas_stats_enrich_ws_bytes(D, n), "sub_stats_enrich: workspace too small");
  ATLAS_REQUIRE(D < (1LL << 31), "sub_stats_enrich: D too large");
  SELevels lev{};
  for (int j = 0; j < NL; ++j) {
    ATLAS_REQUIRE(levels_host[j] >= 0 && levels_host[j] < B, "sub_stats_enrich: level %d out of range", j);
    lev.v[j] = levels_host[j];
  }
  const auto* x = reinterpret_cast<const __nv_bfloat16*>(XT);
  cudaStream_t st = (cudaStream_t)stream;
  switch (A_pad) {
    case 16: return launch_stats_enrich<16>(x, ldx, col0, n, D, E0, E1, (int)B, lev, (int)NL, annT, n_pad, (int)A, sum,
                                            sq, bins, enr, ws, st);
    case 32: return launch_stats_enrich<32>(x, ldx, col0, n, D, E0, E1, (int)B, lev, (int)NL, annT, n_pad, (int)A, sum,
                                            sq, bins, enr, ws, st);
    default: return launch_stats_enrich<48>(x, ldx, col0, n, D, E0, E1, (int)B, lev, (int)NL, annT, n_pad, (int)A, sum,
                                            sq, bins, enr, ws, st);
  }
}
