// Per-batch helpers: compaction thresholds (begin_batch), subsample row gathers, and the
// subsample-statistics kernel (bin masses, moments, int8 enrichment masks).
#include "common.cuh"

namespace atlas {
namespace {

// ---------------------------------------------------------------------------- thresholds
// One thread per (layer, pole, column) group; reads the K-th slot of the top-K state and the Kr-th
// slot of the B reservoirs (core.py:250-259).
// With top_kth / res_thr it also keeps, for the batch's admission, each group's K-th state key and
// each bin's admission ceiling max(res_s[., Kr-1], res_seed) in compact arrays.
__global__ void thresholds_kernel(const float* __restrict__ top_s, int64_t K, const int64_t* __restrict__ res_s,
                                  int64_t Kr, const float* __restrict__ top_seed, const int64_t* __restrict__ res_seed,
                                  const float* __restrict__ E, int64_t G, int64_t B, int64_t U_res, int reservoir,
                                  float* __restrict__ thr, const int64_t* __restrict__ top_k,
                                  int64_t* __restrict__ top_kth, int64_t* __restrict__ res_thr) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < G; g += (int64_t)gridDim.x * blockDim.x) {
    const float tau = top_s[g * K + (K - 1)];
    const float tau_top = fmaxf(next_down(tau), top_seed[g]);
    if (top_kth) top_kth[g] = top_k[g * K + (K - 1)];
    if (!reservoir) {
      thr[g] = tau_top;
      continue;
    }
    float eps = __int_as_float(0x7F800000);
    for (int64_t b = 0; b < B; ++b) {
      const int64_t gb = g * B + b;
      int64_t kth = res_s[gb * Kr + (Kr - 1)];
      const int64_t sd = res_seed[gb];
      if (sd > kth) kth = sd;
      if (res_thr) res_thr[gb] = kth;
      if (kth < -U_res) eps = fminf(eps, E[gb]);
    }
    thr[g] = fminf(tau_top, next_down(eps));
  }
}

// ---------------------------------------------------------------------------- gathers
// XT[d, col0 + i] = H[rows[i], d]: 32x32 tiles through shared memory (coalesced on both sides).
template <typename T>
__global__ void gather_transpose_kernel(const T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ rows,
                                        int64_t n, int64_t n8, T* __restrict__ XT, int64_t ldx, int64_t col0) {
  __shared__ T tile[32][33];
  const int64_t i0 = (int64_t)blockIdx.x * 32;
  const int64_t d0 = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int k = ty; k < 32; k += 8) {
    const int64_t i = i0 + k, d = d0 + tx;
    T v = T(0.0f);
    if (i < n && d < D) v = H[(int64_t)rows[i] * ld + d];
    tile[k][tx] = v;
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int64_t d = d0 + k, i = i0 + tx;
    if (d < D && i < n8) XT[d * ldx + col0 + i] = tile[tx][k];
  }
}

// 2-byte types with 16-byte-aligned rows: 64 (rows i) x 64 (columns d) tiles; each thread loads
// two 16-byte vectors (8 columns of one row, coalesced along the row) and stores two 16-byte
// vectors of XT (8 consecutive rows of one column). Shared-memory reads walk the tile with the
// column index fastest, so a warp reads one tile row (no bank conflicts). Rows >= n are zeros.
__global__ void __launch_bounds__(256)
gather_transpose16_kernel(const uint16_t* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ rows,
                          int64_t n, int64_t n8, uint16_t* __restrict__ XT, int64_t ldx, int64_t col0) {
  __shared__ __align__(16) uint16_t tile[64][64];
  const int64_t i0 = (int64_t)blockIdx.x * 64, d0 = (int64_t)blockIdx.y * 64;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int c = threadIdx.x + 256 * j;
    const int r = c >> 3, ch = c & 7;
    const int64_t i = i0 + r, d = d0 + ch * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (i < n && d < D) v = __ldg(reinterpret_cast<const uint4*>(H + (int64_t)rows[i] * ld + d));
    *reinterpret_cast<uint4*>(&tile[r][ch * 8]) = v;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int c = threadIdx.x + 256 * j;
    const int dd = c & 63, ch = c >> 6;
    const int64_t d = d0 + dd, i = i0 + ch * 8;
    if (d < D && i < n8) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        w[k] = (uint32_t)tile[ch * 8 + 2 * k][dd] | ((uint32_t)tile[ch * 8 + 2 * k + 1][dd] << 16);
      *reinterpret_cast<uint4*>(XT + d * ldx + col0 + i) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ rows,
                                   int64_t n, T* __restrict__ R) {
  const int64_t total = n * D;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / D, d = e - i * D;
    R[e] = H[(int64_t)rows[i] * ld + d];
  }
}

__global__ void gather_rows_vec_kernel(const uint4* __restrict__ H, int64_t Dv, int64_t ldv, const int32_t* __restrict__ rows,
                                       int64_t n, uint4* __restrict__ R) {
  const int64_t total = n * Dv;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / Dv, d = e - i * Dv;
    R[e] = H[(int64_t)rows[i] * ldv + d];
  }
}

// ---------------------------------------------------------------------------- subsample statistics
// One warp per column d; each lane takes 8 consecutive subsample rows per step (one 16-byte vector
// of XT for 16-bit types). Bin counts use the cumulative form of the reference's v1 path
// (#{s >= E_b} differences, core.py:322-327); masks are (s >= E[lev]) (core.py:329).
constexpr int kMaxB = 8;
constexpr int kMaxNL = 8;

struct Levels {
  int v[kMaxNL];
};

template <int DT>
__device__ __forceinline__ void load8(const typename Elem<DT>::T* p, int64_t i, int64_t n, float (&x)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) x[k] = (i + k < n) ? Elem<DT>::f(p[k]) : 0.0f;
}

template <int DT>
__global__ void __launch_bounds__(256)
sub_stats_kernel(const typename Elem<DT>::T* __restrict__ XT, int64_t ldx, int64_t col0, int64_t n, int64_t D,
                 const float* __restrict__ E0, const float* __restrict__ E1, int B, Levels lev, int NL,
                 double* __restrict__ sum, double* __restrict__ sq, int64_t* __restrict__ bins,
                 int8_t* __restrict__ masks, int64_t n_pad) {
  const int lane = threadIdx.x & 31;
  const int64_t d = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (d >= D) return;
  float e0[kMaxB], e1[kMaxB];
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    e0[b] = b < B ? E0[d * B + b] : __int_as_float(0x7F800000);
    e1[b] = b < B ? E1[d * B + b] : __int_as_float(0x7F800000);
  }
  float m0[kMaxNL], m1[kMaxNL];
#pragma unroll
  for (int j = 0; j < kMaxNL; ++j) {
    m0[j] = j < NL ? E0[d * B + lev.v[j]] : 0.0f;
    m1[j] = j < NL ? E1[d * B + lev.v[j]] : 0.0f;
  }
  int c0[kMaxB], c1[kMaxB];
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) c0[b] = c1[b] = 0;
  double acc_s = 0.0, acc_q = 0.0;
  const typename Elem<DT>::T* col = XT + d * ldx + col0;
  const int64_t n_loop = masks ? n_pad : n;
  for (int64_t i = (int64_t)lane * 8; i < n_loop; i += 256) {
    float x[8];
    load8<DT>(col + i, i, n, x);
    float s32 = 0.0f, q32 = 0.0f;
    uint32_t valid = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const bool v = i + k < n;
      valid |= (v ? 1u : 0u) << k;
      s32 += x[k];
      q32 = fmaf(x[k], x[k], q32);
#pragma unroll
      for (int b = 0; b < kMaxB; ++b) {
        c0[b] += (v && x[k] >= e0[b]) ? 1 : 0;
        c1[b] += (v && -x[k] >= e1[b]) ? 1 : 0;
      }
    }
    acc_s += (double)s32;
    acc_q += (double)q32;
    if (masks) {
#pragma unroll
      for (int j = 0; j < kMaxNL; ++j) {
        if (j >= NL) break;
        uint64_t w0 = 0, w1 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (valid & (1u << k)) {
            w0 |= (uint64_t)(x[k] >= m0[j] ? 1 : 0) << (8 * k);
            w1 |= (uint64_t)(-x[k] >= m1[j] ? 1 : 0) << (8 * k);
          }
        }
        *reinterpret_cast<uint64_t*>(masks + ((int64_t)(0 * NL + j) * D + d) * n_pad + i) = w0;
        *reinterpret_cast<uint64_t*>(masks + ((int64_t)(1 * NL + j) * D + d) * n_pad + i) = w1;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_s += __shfl_xor_sync(0xFFFFFFFFu, acc_s, o);
    acc_q += __shfl_xor_sync(0xFFFFFFFFu, acc_q, o);
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      c0[b] += __shfl_xor_sync(0xFFFFFFFFu, c0[b], o);
      c1[b] += __shfl_xor_sync(0xFFFFFFFFu, c1[b], o);
    }
  }
  if (lane == 0) {
    sum[d] += acc_s;
    sq[d] += acc_q;
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      if (b >= B) break;
      const int nx0 = (b + 1 < B) ? c0[b + 1] : 0;
      const int nx1 = (b + 1 < B) ? c1[b + 1] : 0;
      bins[d * B + b] += (int64_t)(c0[b] - nx0);
      bins[(D + d) * B + b] += (int64_t)(c1[b] - nx1);
    }
  }
}

// One 8-row vector of one column (bf16 path below): fp32 sums of the vector folded into the fp64
// totals, cumulative edge counts from the compare masks (16 bits per counted row), and the int8
// level masks (one byte per row, rows i..i+7 little-endian in one 8-byte store per plane). kFull:
// every row of the vector is < n (no validity mask).
template <bool kFull>
__device__ __forceinline__ void stats_vec8(const uint32_t (&w4)[4], const uint32_t (&vm)[4], const __nv_bfloat162 (&pe)[kMaxB],
                                           const __nv_bfloat162 (&ne)[kMaxB], const uint32_t (&levmask)[kMaxB], int B,
                                           int NL, int (&c0)[kMaxB], int (&c1)[kMaxB], double& acc_s, double& acc_q,
                                           int8_t* __restrict__ mrow, int64_t plane) {
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
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    if (b >= B) break;
    uint32_t mp[4], mn[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[w]);
      mp[w] = __hge2_mask(h2, pe[b]);
      mn[w] = __hle2_mask(h2, ne[b]);
      if (!kFull) {
        mp[w] &= vm[w];
        mn[w] &= vm[w];
      }
    }
    c0[b] += __popc(mp[0]) + __popc(mp[1]) + __popc(mp[2]) + __popc(mp[3]);
    c1[b] += __popc(mn[0]) + __popc(mn[1]) + __popc(mn[2]) + __popc(mn[3]);
    uint32_t lm = mrow ? levmask[b] : 0u;
    if (lm) {
      const uint64_t wp = (uint64_t)(__byte_perm(mp[0], mp[1], 0x6420) & 0x01010101u) |
                          ((uint64_t)(__byte_perm(mp[2], mp[3], 0x6420) & 0x01010101u) << 32);
      const uint64_t wn = (uint64_t)(__byte_perm(mn[0], mn[1], 0x6420) & 0x01010101u) |
                          ((uint64_t)(__byte_perm(mn[2], mn[3], 0x6420) & 0x01010101u) << 32);
      while (lm) {
        const int j = __ffs(lm) - 1;
        lm &= lm - 1;
        *reinterpret_cast<uint64_t*>(mrow + (int64_t)j * plane) = wp;
        *reinterpret_cast<uint64_t*>(mrow + (int64_t)(NL + j) * plane) = wn;
      }
    }
  }
}

// bf16 path of the same statistics, on packed pairs: every edge compare is one bf16x2 compare per
// two rows against the edge rounded to bf16 (up for the positive pole x >= E0; down for the
// negative pole, x <= -E1), which for bf16 values is exactly the fp32 compare: no bf16 lies
// strictly between an fp32 edge and its directed rounding. Counts come from popcounts of the
// compare masks (16 set bits per counted row), and a level's int8 mask reuses the compare words of
// its edge. Sums stay fp32 within the 8-row vector and fp64 across vectors.
__global__ void __launch_bounds__(256)
sub_stats_bf16_kernel(const __nv_bfloat16* __restrict__ XT, int64_t ldx, int64_t col0, int64_t n, int64_t D,
                      const float* __restrict__ E0, const float* __restrict__ E1, int B, Levels lev, int NL,
                      double* __restrict__ sum, double* __restrict__ sq, int64_t* __restrict__ bins,
                      int8_t* __restrict__ masks, int64_t n_pad) {
  const int lane = threadIdx.x & 31;
  const int64_t d = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (d >= D) return;
  __nv_bfloat162 pe[kMaxB], ne[kMaxB];
  uint32_t levmask[kMaxB];  // bit j set when level j sits on edge b
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    const bool ok = b < B;
    pe[b] = __bfloat162bfloat162(__float2bfloat16_ru(ok ? E0[d * B + b] : __int_as_float(0x7F800000)));
    ne[b] = __bfloat162bfloat162(__float2bfloat16_rd(ok ? -E1[d * B + b] : __int_as_float(0xFF800000)));
    uint32_t lm = 0;
#pragma unroll
    for (int j = 0; j < kMaxNL; ++j)
      if (j < NL && lev.v[j] == b) lm |= 1u << j;
    levmask[b] = lm;
  }
  int c0[kMaxB], c1[kMaxB];
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) c0[b] = c1[b] = 0;
  double acc_s = 0.0, acc_q = 0.0;
  const __nv_bfloat16* col = XT + d * ldx + col0;
  const int64_t n_loop = masks ? n_pad : n;
  const int64_t plane = D * n_pad;  // bytes between mask planes (pole, level)
  int64_t i = (int64_t)lane * 8;
  for (; i + 8 <= n; i += 256) {  // whole 8-row vectors: no row is masked
    const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(col + i));
    const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
    stats_vec8<true>(w4, w4, pe, ne, levmask, B, NL, c0, c1, acc_s, acc_q, masks ? masks + d * n_pad + i : nullptr,
                     plane);
  }
  for (; i < n_loop; i += 256) {  // the ragged end of the column (and mask padding past n): rows >= n are zero, uncounted
    const unsigned short* c16 = reinterpret_cast<const unsigned short*>(col);
    uint32_t w4[4], vm[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int64_t r = i + 2 * w;
      const uint32_t lo = r < n ? c16[r] : 0u, hi = r + 1 < n ? c16[r + 1] : 0u;
      w4[w] = lo | (hi << 16);
      vm[w] = (r < n ? 0x0000FFFFu : 0u) | (r + 1 < n ? 0xFFFF0000u : 0u);
    }
    stats_vec8<false>(w4, vm, pe, ne, levmask, B, NL, c0, c1, acc_s, acc_q, masks ? masks + d * n_pad + i : nullptr,
                      plane);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_s += __shfl_xor_sync(0xFFFFFFFFu, acc_s, o);
    acc_q += __shfl_xor_sync(0xFFFFFFFFu, acc_q, o);
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      c0[b] += __shfl_xor_sync(0xFFFFFFFFu, c0[b], o);
      c1[b] += __shfl_xor_sync(0xFFFFFFFFu, c1[b], o);
    }
  }
  if (lane == 0) {
    sum[d] += acc_s;
    sq[d] += acc_q;
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      if (b >= B) break;
      const int nx0 = (b + 1 < B) ? c0[b + 1] : 0;
      const int nx1 = (b + 1 < B) ? c1[b + 1] : 0;
      bins[d * B + b] += (int64_t)((c0[b] - nx0) >> 4);  // 16 mask bits per counted row
      bins[(D + d) * B + b] += (int64_t)((c1[b] - nx1) >> 4);
    }
  }
}

template <int DT>
int launch_stats(const void* XT, int64_t ldx, int64_t col0, int64_t n, int64_t D, const float* E0, const float* E1,
                 int64_t B, const Levels& lev, int64_t NL, double* sum, double* sq, int64_t* bins, int8_t* masks,
                 int64_t n_pad, cudaStream_t st) {
  const int warps = 8;
  dim3 grid((unsigned)((D + warps - 1) / warps));
  if constexpr (DT == ATLAS_BF16) {
    if ((uintptr_t)XT % 16 == 0) {
      sub_stats_bf16_kernel<<<grid, warps * 32, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(XT), ldx, col0, n, D, E0,
                                                         E1, (int)B, lev, (int)NL, sum, sq, bins, masks, n_pad);
      return check_launch("atlas_sub_stats");
    }
  }
  sub_stats_kernel<DT><<<grid, warps * 32, 0, st>>>(reinterpret_cast<const typename Elem<DT>::T*>(XT), ldx, col0, n, D,
                                                     E0, E1, (int)B, lev, (int)NL, sum, sq, bins, masks, n_pad);
  return check_launch("atlas_sub_stats");
}

int esize(int dtype) { return dtype == ATLAS_F32 ? 4 : 2; }

}  // namespace
}  // namespace atlas

using namespace atlas;

namespace atlas {
namespace {
__global__ void batch_counters_kernel(const int32_t* __restrict__ count, int L, uint64_t filt, int64_t cap_main,
                                      int64_t cap_early, int early_layers, const int32_t* __restrict__ n_top,
                                      const int32_t* __restrict__ n_res, int64_t* __restrict__ stats) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int64_t compacted = 0, over = 0;
  for (int l = 0; l < L; ++l) {
    if (!((filt >> l) & 1ull)) continue;
    const int64_t cap = l < early_layers ? cap_early : cap_main;
    const int64_t c = count[l];
    if (c <= cap)
      compacted += c;
    else
      ++over;
  }
  stats[0] += compacted;
  stats[1] += *n_top;
  stats[2] += *n_res;
  stats[3] += over;
}
}  // namespace
}  // namespace atlas

extern "C" int atlas_batch_counters(const int32_t* count, int64_t L, const int8_t* filtered_host, int64_t cap_main,
                                    int64_t cap_early, int64_t early_layers, const int32_t* n_top, const int32_t* n_res,
                                    int64_t* stats, void* stream) {
  ATLAS_REQUIRE(L >= 0 && L <= 64, "batch_counters: L must be 0..64 (got %lld)", (long long)L);
  ATLAS_REQUIRE(count && n_top && n_res && stats, "batch_counters: null pointer");
  uint64_t filt = 0;
  if (filtered_host)
    for (int64_t l = 0; l < L; ++l)
      if (filtered_host[l]) filt |= 1ull << l;
  batch_counters_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(count, (int)L, filt, cap_main, cap_early, (int)early_layers,
                                                           n_top, n_res, stats);
  return check_launch("atlas_batch_counters");
}

extern "C" int atlas_thresholds(const float* top_s, int64_t K, const int64_t* res_s, int64_t Kr, const float* top_seed,
                                const int64_t* res_seed, const float* E, int64_t G, int64_t B, int64_t U_res,
                                int reservoir, float* thr, const int64_t* top_k, int64_t* top_kth, int64_t* res_thr,
                                void* stream) {
  ATLAS_REQUIRE(K >= 1 && Kr >= 1 && G >= 0 && B >= 1, "thresholds: bad sizes K=%lld Kr=%lld G=%lld B=%lld",
                (long long)K, (long long)Kr, (long long)G, (long long)B);
  if (G == 0) return ATLAS_OK;
  ATLAS_REQUIRE(top_s && top_seed && thr && (!reservoir || (res_s && res_seed && E)), "thresholds: null pointer");
  ATLAS_REQUIRE(!top_kth || top_k, "thresholds: top_kth needs top_k");
  thresholds_kernel<<<grid_for(G, 256), 256, 0, (cudaStream_t)stream>>>(top_s, K, res_s, Kr, top_seed, res_seed, E, G,
                                                                        B, U_res, reservoir, thr, top_k, top_kth,
                                                                        reservoir ? res_thr : nullptr);
  return check_launch("atlas_thresholds");
}

extern "C" int atlas_gather_transpose(const void* H, int dtype, int64_t T, int64_t D, int64_t ld, const int32_t* rows,
                                      int64_t n, void* XT, int64_t ldx, int64_t col0, void* stream) {
  ATLAS_REQUIRE(T >= 0 && D >= 0 && ld >= D && n >= 0 && col0 >= 0, "gather_transpose: bad sizes");
  const int64_t n8 = (n + 7) / 8 * 8;
  ATLAS_REQUIRE(col0 + n8 <= ldx, "gather_transpose: columns %lld..%lld exceed ldx %lld", (long long)col0,
                (long long)(col0 + n8), (long long)ldx);
  if (n8 == 0 || D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(H && rows && XT, "gather_transpose: null pointer");
  dim3 grid((unsigned)((n8 + 31) / 32), (unsigned)((D + 31) / 32));
  ATLAS_REQUIRE(grid.y < 65536, "gather_transpose: D too large");
  dim3 block(32, 8);
  cudaStream_t st = (cudaStream_t)stream;
  if ((dtype == ATLAS_BF16 || dtype == ATLAS_F16) && D % 8 == 0 && ld % 8 == 0 && ldx % 8 == 0 && col0 % 8 == 0 &&
      (uintptr_t)H % 16 == 0 && (uintptr_t)XT % 16 == 0) {
    dim3 g16((unsigned)((n8 + 63) / 64), (unsigned)((D + 63) / 64));
    ATLAS_REQUIRE(g16.y < 65536, "gather_transpose: D too large");
    gather_transpose16_kernel<<<g16, 256, 0, st>>>((const uint16_t*)H, D, ld, rows, n, n8, (uint16_t*)XT, ldx, col0);
    return check_launch("atlas_gather_transpose");
  }
  switch (dtype) {
    case ATLAS_BF16:
      gather_transpose_kernel<__nv_bfloat16><<<grid, block, 0, st>>>((const __nv_bfloat16*)H, D, ld, rows, n, n8,
                                                                      (__nv_bfloat16*)XT, ldx, col0);
      break;
    case ATLAS_F16:
      gather_transpose_kernel<__half><<<grid, block, 0, st>>>((const __half*)H, D, ld, rows, n, n8, (__half*)XT, ldx, col0);
      break;
    case ATLAS_F32:
      gather_transpose_kernel<float><<<grid, block, 0, st>>>((const float*)H, D, ld, rows, n, n8, (float*)XT, ldx, col0);
      break;
    default:
      return fail(ATLAS_ERR_ARG, "gather_transpose: unknown dtype %d", dtype);
  }
  return check_launch("atlas_gather_transpose");
}

extern "C" int atlas_gather_rows(const void* H, int dtype, int64_t T, int64_t D, int64_t ld, const int32_t* rows,
                                 int64_t n, void* R, void* stream) {
  ATLAS_REQUIRE(T >= 0 && D >= 0 && ld >= D && n >= 0, "gather_rows: bad sizes");
  if (n == 0 || D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(H && rows && R, "gather_rows: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int es = esize(dtype);
  if ((D * es) % 16 == 0 && (ld * es) % 16 == 0 && (uintptr_t)H % 16 == 0 && (uintptr_t)R % 16 == 0) {
    const int64_t Dv = D * es / 16, ldv = ld * es / 16;
    gather_rows_vec_kernel<<<grid_for(n * Dv, 256), 256, 0, st>>>((const uint4*)H, Dv, ldv, rows, n, (uint4*)R);
    return check_launch("atlas_gather_rows");
  }
  switch (dtype) {
    case ATLAS_BF16:
    case ATLAS_F16:
      gather_rows_kernel<uint16_t><<<grid_for(n * D, 256), 256, 0, st>>>((const uint16_t*)H, D, ld, rows, n, (uint16_t*)R);
      break;
    case ATLAS_F32:
      gather_rows_kernel<float><<<grid_for(n * D, 256), 256, 0, st>>>((const float*)H, D, ld, rows, n, (float*)R);
      break;
    default:
      return fail(ATLAS_ERR_ARG, "gather_rows: unknown dtype %d", dtype);
  }
  return check_launch("atlas_gather_rows");
}

extern "C" int atlas_sub_stats(const void* XT, int dtype, int64_t ldx, int64_t col0, int64_t n, int64_t D,
                               const float* E0, const float* E1, int64_t B, const int32_t* levels_host, int64_t NL,
                               double* sum, double* sq, int64_t* bins, int8_t* masks, int64_t n_pad, void* stream) {
  ATLAS_REQUIRE(n >= 0 && D >= 0 && B >= 1 && B <= kMaxB, "sub_stats: bad sizes (B must be 1..%d)", kMaxB);
  ATLAS_REQUIRE(NL >= 0 && NL <= kMaxNL, "sub_stats: NL must be 0..%d", kMaxNL);
  if (D == 0 || n == 0) return ATLAS_OK;
  ATLAS_REQUIRE(XT && E0 && E1 && sum && sq && bins, "sub_stats: null pointer");
  ATLAS_REQUIRE(col0 % 8 == 0 && ldx % 8 == 0 && col0 + n <= ldx, "sub_stats: col0/ldx must be multiples of 8");
  Levels lev{};
  for (int j = 0; j < NL; ++j) {
    ATLAS_REQUIRE(levels_host && levels_host[j] >= 0 && levels_host[j] < B, "sub_stats: level %d out of range", j);
    lev.v[j] = levels_host[j];
  }
  if (NL > 0) {
    ATLAS_REQUIRE(masks != nullptr, "sub_stats: masks required when NL > 0");
    ATLAS_REQUIRE(n_pad >= n && n_pad % 8 == 0 && (uintptr_t)masks % 8 == 0, "sub_stats: bad n_pad / mask alignment");
  } else {
    masks = nullptr;
  }
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case ATLAS_BF16: return launch_stats<ATLAS_BF16>(XT, ldx, col0, n, D, E0, E1, B, lev, NL, sum, sq, bins, masks, n_pad, st);
    case ATLAS_F16: return launch_stats<ATLAS_F16>(XT, ldx, col0, n, D, E0, E1, B, lev, NL, sum, sq, bins, masks, n_pad, st);
    case ATLAS_F32: return launch_stats<ATLAS_F32>(XT, ldx, col0, n, D, E0, E1, B, lev, NL, sum, sq, bins, masks, n_pad, st);
    default: return fail(ATLAS_ERR_ARG, "sub_stats: unknown dtype %d", dtype);
  }
}
