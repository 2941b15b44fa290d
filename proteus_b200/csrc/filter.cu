// K1: single-pass compare-and-compact over the hook output H (one read of H per layer).
//
// Replaces filter_candidates (atlas/filter_triton.py:19-86). B200 layout: each warp owns a strip of
// 32 * VEC consecutive columns (one 16-byte vector per lane, VEC = 8 for bf16/fp16, 4 for fp32) and
// walks rows with U rows in flight per lane; the per-column thresholds live in registers for the
// whole walk. Padding rows (rowmap < 0) are never read.
// Compaction is two-level: a warp ballot + shuffle prefix sum places a step's survivors in a
// per-CTA staging area in shared memory (one shared-memory atomic per warp step with hits), and
// the CTA reserves its global output range with ONE global atomic at the end, then copies the
// staged survivors out with coalesced stores. At ~0.1-0.5% survivors nearly every warp step has a
// hit, so per-step global atomics on the single counter would serialise the whole pass; a warp
// whose step does not fit the staging area writes directly (global atomic), which keeps the
// count exact for any survivor density.
#include "common.cuh"

namespace atlas {
namespace {

// Raw vector of VEC elements as loaded (16 bytes on the vector paths); elements are widened to
// fp32 on use, so a lane keeps U raw vectors in flight in few registers.
template <int DT, int VEC>
struct Vec;

#ifndef ATLAS_FILTER_PACKED
#define ATLAS_FILTER_PACKED 1  // bf16 vector path: packed compares + software pipeline (filter_bf16_kernel)
#endif
#if !ATLAS_FILTER_PACKED
template <>
struct Vec<ATLAS_BF16, 8> {
  uint4 v;
  __device__ __forceinline__ void load(const void* p) { v = __ldcs(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ float at(int k) const {
    const uint32_t w = k < 2 ? v.x : k < 4 ? v.y : k < 6 ? v.z : v.w;
    return (k & 1) ? __uint_as_float(w & 0xFFFF0000u) : __uint_as_float(w << 16);
  }
};
#endif
template <>
struct Vec<ATLAS_F16, 8> {
  uint4 v;
  __device__ __forceinline__ void load(const void* p) { v = __ldcs(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ float at(int k) const {
    const uint32_t w = k < 2 ? v.x : k < 4 ? v.y : k < 6 ? v.z : v.w;
    return __half2float(__ushort_as_half((unsigned short)((k & 1) ? (w >> 16) : (w & 0xFFFFu))));
  }
};
template <>
struct Vec<ATLAS_F32, 4> {
  float4 v;
  __device__ __forceinline__ void load(const void* p) { v = __ldcs(reinterpret_cast<const float4*>(p)); }
  __device__ __forceinline__ float at(int k) const { return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w; }
};
template <int DT>
struct Vec<DT, 1> {
  float v;
  __device__ __forceinline__ void load(const void* p) { v = Elem<DT>::f(*reinterpret_cast<const typename Elem<DT>::T*>(p)); }
  __device__ __forceinline__ float at(int) const { return v; }
};

#ifndef ATLAS_FILTER_U
#define ATLAS_FILTER_U 4           // rows in flight per lane on the vector paths
#endif
#ifndef ATLAS_FILTER_CTAS_PER_SM
#define ATLAS_FILTER_CTAS_PER_SM 4  // grid = one resident wave of this many 8-warp CTAs per SM
#endif

#ifndef ATLAS_FILTER_WX
#define ATLAS_FILTER_WX 1  // warps of a CTA side by side along a row (contiguous WX*512 bytes per row)
#endif
#ifndef ATLAS_FILTER_WY
#define ATLAS_FILTER_WY 8  // warps of a CTA stacked along rows
#endif

constexpr int kWX = ATLAS_FILTER_WX;
constexpr int kWY = ATLAS_FILTER_WY;
constexpr int kWarps = kWX * kWY;
constexpr int kStage = 2048;  // staged survivors per CTA (24 KB of shared memory)
constexpr int kCtasPerSm = ATLAS_FILTER_CTAS_PER_SM;

template <int DT, int VEC, int U>
__global__ void __launch_bounds__(kWarps * 32, kCtasPerSm)
filter_kernel(const char* __restrict__ H, int64_t T, int64_t D, int64_t ld_bytes, int64_t rows_per_cta,
              const int32_t* __restrict__ rowmap, const float* __restrict__ thr_pos,
              const float* __restrict__ thr_neg, float* __restrict__ out_val, int32_t* __restrict__ out_row,
              int32_t* __restrict__ out_col, int32_t* __restrict__ count, int64_t cap) {
  using E = typename Elem<DT>::T;
  const int lane = threadIdx.x & 31;
  const int warp = (threadIdx.x >> 5) / kWX;  // row position of this warp in the CTA
  const int wx = (threadIdx.x >> 5) % kWX;    // column position
  const int64_t c0 = (((int64_t)blockIdx.x * kWX + wx) * 32 + lane) * VEC;
  const bool col_ok = c0 < D;  // VEC divides D on the vector paths, so a strip is whole or absent
  float tp[VEC], tn[VEC];
#pragma unroll
  for (int k = 0; k < VEC; ++k) {
    const bool ok = col_ok && c0 + k < D;
    tp[k] = ok ? __ldg(thr_pos + c0 + k) : __int_as_float(0x7F800000);    // +inf: never survives
    tn[k] = ok ? -__ldg(thr_neg + c0 + k) : __int_as_float(0xFF800000);   // h < -thr_neg
  }
  __shared__ float s_val[kStage];
  __shared__ int32_t s_row[kStage], s_col[kStage];
  __shared__ int s_n, s_limit, s_base;
  if (threadIdx.x == 0) {
    s_n = 0;
    s_limit = kStage;
  }
  __syncthreads();
  const int64_t r_begin = (int64_t)blockIdx.y * rows_per_cta;
  int64_t r_end = r_begin + rows_per_cta;
  if (r_end > T) r_end = T;

  for (int64_t r = r_begin + warp; r < r_end; r += (int64_t)kWY * U) {
    Vec<DT, VEC> x[U];
    int32_t vr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = r + (int64_t)u * kWY;
      vr[u] = row < r_end ? __ldg(rowmap + row) : -1;
      if (!col_ok) vr[u] = -1;
      if (vr[u] >= 0) x[u].load(H + row * ld_bytes + c0 * (int64_t)sizeof(E));
    }
    uint64_t bits = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (vr[u] < 0) continue;
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        const float h = x[u].at(k);
        const bool hit = (h > tp[k]) || (h < tn[k]);
        bits |= (uint64_t)(hit ? 1u : 0u) << (u * VEC + k);
      }
    }
    if (!__any_sync(0xFFFFFFFFu, bits != 0)) continue;
    int total;
    const int n = __popcll(bits);
    const int pre = warp_excl_scan(n, lane, &total);
    int base = 0;
    if (lane == 31) base = atomicAdd(&s_n, total);
    base = __shfl_sync(0xFFFFFFFFu, base, 31);
    const bool staged = base + total <= kStage;
    if (!staged) {  // staging area full: this step goes straight to global memory
      if (lane == 31) {
        atomicMin(&s_limit, base);  // reservations grow monotonically: the first miss ends the staged prefix
        base = atomicAdd(count, total);
      }
      base = __shfl_sync(0xFFFFFFFFu, base, 31);
    }
    int64_t slot = (int64_t)base + pre;
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        if (bits & (1ull << (u * VEC + k))) {
          if (staged) {
            s_val[slot] = x[u].at(k);
            s_row[slot] = vr[u];
            s_col[slot] = (int32_t)(c0 + k);
          } else if (slot < cap) {
            out_val[slot] = x[u].at(k);
            out_row[slot] = vr[u];
            out_col[slot] = (int32_t)(c0 + k);
          }
          ++slot;
        }
      }
    }
  }
  __syncthreads();
  const int staged_n = s_n < s_limit ? s_n : s_limit;  // [0, staged_n) holds every staged survivor
  if (threadIdx.x == 0) s_base = staged_n > 0 ? atomicAdd(count, staged_n) : 0;
  __syncthreads();
  const int64_t base = s_base;
  for (int i = threadIdx.x; i < staged_n; i += blockDim.x) {
    const int64_t slot = base + i;
    if (slot < cap) {
      out_val[slot] = s_val[i];
      out_row[slot] = s_row[i];
      out_col[slot] = s_col[i];
    }
  }
}

// bf16 fast path. Same contract as filter_kernel, three changes:
//  * compares run on packed bf16 pairs against thresholds rounded to bf16 (toward -inf for the
//    positive pole, toward +inf for the negative pole). For a bf16 value h and an fp32 threshold t,
//    h > t  <=>  h > rd_bf16(t)  and  h < t  <=>  h < ru_bf16(t) (no bf16 lies strictly between
//    t and its directed rounding), so the survivors are exactly those of the fp32 comparison;
//    NaN compares false on both sides as in fp32;
//  * software pipeline: the U rows of the next step are loaded before the current step is
//    compared, so every lane keeps 2*U 16-byte loads in flight;
//  * the row map is read once per 32 rows of a warp (one lane per row, two blocks ahead) and
//    handed out with shuffles, so no H load waits on a dependent row-map load.
template <int U>
__global__ void __launch_bounds__(kWarps * 32, kCtasPerSm)
filter_bf16_kernel(const char* __restrict__ H, int64_t T, int64_t D, int64_t ld_bytes, int64_t rows_per_cta,
                   const int32_t* __restrict__ rowmap, const float* __restrict__ thr_pos,
                   const float* __restrict__ thr_neg, float* __restrict__ out_val, int32_t* __restrict__ out_row,
                   int32_t* __restrict__ out_col, int32_t* __restrict__ count, int64_t cap) {
  static_assert(32 % U == 0 && U * 8 <= 32, "U must divide 32 and give at most 32 hit bits");
  constexpr int kIpb = 32 / U;  // steps per row-map block
  const int lane = threadIdx.x & 31;
  const int warp = (threadIdx.x >> 5) / kWX;
  const int wx = (threadIdx.x >> 5) % kWX;
  const int64_t c0 = (((int64_t)blockIdx.x * kWX + wx) * 32 + lane) * 8;
  const bool col_ok = c0 < D;
  __nv_bfloat162 tp2[4], tn2[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    __nv_bfloat16 p[2], n[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t c = c0 + 2 * w + h;
      const bool ok = col_ok && c < D;
      p[h] = __float2bfloat16_rd(ok ? __ldg(thr_pos + c) : __int_as_float(0x7F800000));
      n[h] = __float2bfloat16_ru(ok ? -__ldg(thr_neg + c) : __int_as_float(0xFF800000));
    }
    tp2[w] = __halves2bfloat162(p[0], p[1]);
    tn2[w] = __halves2bfloat162(n[0], n[1]);
  }
  __shared__ float s_val[kStage];
  __shared__ int32_t s_row[kStage], s_col[kStage];
  __shared__ int s_n, s_limit, s_base;
  if (threadIdx.x == 0) {
    s_n = 0;
    s_limit = kStage;
  }
  __syncthreads();
  const int64_t r_begin = (int64_t)blockIdx.y * rows_per_cta;
  int64_t r_end = r_begin + rows_per_cta;
  if (r_end > T) r_end = T;
  const int64_t rbase = r_begin + warp;  // this warp's rows: rbase + j * kWY, j = 0, 1, ...
  const int64_t n_rows = r_end > rbase ? (r_end - rbase + kWY - 1) / kWY : 0;
  const int64_t n_steps = (n_rows + U - 1) / U;
  auto rm_block = [&](int64_t b) -> int32_t {
    const int64_t row = rbase + (b * 32 + lane) * (int64_t)kWY;
    return row < r_end ? __ldg(rowmap + row) : -1;
  };
  int32_t rm_cur = rm_block(0), rm_nxt = rm_block(1);
  const int64_t rstride = (int64_t)kWY * ld_bytes;  // bytes between a warp's consecutive rows
  const char* p = H + rbase * ld_bytes + c0 * 2;      // row of the step being loaded
  uint4 xa[U];
  int32_t va[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    va[u] = __shfl_sync(0xFFFFFFFFu, rm_cur, u);
    if (!col_ok) va[u] = -1;
    if (va[u] >= 0) xa[u] = __ldcs(reinterpret_cast<const uint4*>(p + u * rstride));
  }
  for (int64_t it = 0; it < n_steps; ++it) {
    const int64_t jt = it + 1;  // the step prefetched now
    if (jt % kIpb == 0) {
      rm_cur = rm_nxt;
      rm_nxt = rm_block(jt / kIpb + 1);
    }
    const int sub = (int)(jt % kIpb) * U;
    p += U * rstride;
    uint4 xb[U];
    int32_t vb[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      vb[u] = __shfl_sync(0xFFFFFFFFu, rm_cur, sub + u);
      if (!col_ok) vb[u] = -1;
      if (vb[u] >= 0) xb[u] = __ldcs(reinterpret_cast<const uint4*>(p + u * rstride));
    }
    uint32_t bits = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (va[u] < 0) continue;
      const uint32_t w4[4] = {xa[u].x, xa[u].y, xa[u].z, xa[u].w};
      uint32_t m[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[w]);
        m[w] = __hgt2_mask(h2, tp2[w]) | __hlt2_mask(h2, tn2[w]);
      }
      const uint32_t lo = __byte_perm(m[0], m[1], 0x6420), hi = __byte_perm(m[2], m[3], 0x6420);
      const uint32_t b = (((lo & 0x80808080u) * 0x00204081u) >> 28) | ((((hi & 0x80808080u) * 0x00204081u) >> 28) << 4);
      bits |= b << (8 * u);
    }
    if (__any_sync(0xFFFFFFFFu, bits != 0)) {
      int total;
      const int n = __popc(bits);
      const int pre = warp_excl_scan(n, lane, &total);
      int base = 0;
      if (lane == 31) base = atomicAdd(&s_n, total);
      base = __shfl_sync(0xFFFFFFFFu, base, 31);
      const bool staged = base + total <= kStage;
      if (!staged) {
        if (lane == 31) {
          atomicMin(&s_limit, base);
          base = atomicAdd(count, total);
        }
        base = __shfl_sync(0xFFFFFFFFu, base, 31);
      }
      int64_t slot = (int64_t)base + pre;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        uint32_t bu = (bits >> (8 * u)) & 0xFFu;
        while (bu) {
          const int k = __ffs(bu) - 1;
          bu &= bu - 1;
          const uint32_t w = k < 2 ? xa[u].x : k < 4 ? xa[u].y : k < 6 ? xa[u].z : xa[u].w;
          const float h = (k & 1) ? __uint_as_float(w & 0xFFFF0000u) : __uint_as_float(w << 16);
          if (staged) {
            s_val[slot] = h;
            s_row[slot] = va[u];
            s_col[slot] = (int32_t)(c0 + k);
          } else if (slot < cap) {
            out_val[slot] = h;
            out_row[slot] = va[u];
            out_col[slot] = (int32_t)(c0 + k);
          }
          ++slot;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      xa[u] = xb[u];
      va[u] = vb[u];
    }
  }
  __syncthreads();
  const int staged_n = s_n < s_limit ? s_n : s_limit;
  if (threadIdx.x == 0) s_base = staged_n > 0 ? atomicAdd(count, staged_n) : 0;
  __syncthreads();
  const int64_t base = s_base;
  for (int i = threadIdx.x; i < staged_n; i += blockDim.x) {
    const int64_t slot = base + i;
    if (slot < cap) {
      out_val[slot] = s_val[i];
      out_row[slot] = s_row[i];
      out_col[slot] = s_col[i];
    }
  }
}

template <int DT, int VEC, int U>
int launch(const void* H, int64_t T, int64_t D, int64_t ld, const int32_t* rowmap, const float* tp,
           const float* tn, float* ov, int32_t* orow, int32_t* ocol, int32_t* count, int64_t cap,
           cudaStream_t st) {
  const int64_t strips = (D + 32 * VEC * kWX - 1) / (32 * VEC * kWX);
  const int64_t target = (int64_t)num_sms() * kCtasPerSm;  // one resident wave of CTAs
  int64_t chunks = (target + strips - 1) / strips;
  const int64_t step = (int64_t)kWY * U;
  int64_t rows = (T + chunks - 1) / chunks;
  rows = ((rows + step - 1) / step) * step;
  if (rows < step) rows = step;
  chunks = (T + rows - 1) / rows;
  if (chunks < 1) chunks = 1;
  ATLAS_REQUIRE(strips < 65536 * 32 && chunks < 65536, "filter: grid too large (T=%lld D=%lld)",
                (long long)T, (long long)D);
  dim3 grid((unsigned)strips, (unsigned)chunks);
  const int64_t ld_bytes = ld * (int64_t)sizeof(typename Elem<DT>::T);
  if constexpr (DT == ATLAS_BF16 && VEC == 8 && ATLAS_FILTER_PACKED)
    filter_bf16_kernel<U><<<grid, kWarps * 32, 0, st>>>(reinterpret_cast<const char*>(H), T, D, ld_bytes, rows,
                                                        rowmap, tp, tn, ov, orow, ocol, count, cap);
  else
    filter_kernel<DT, VEC, U><<<grid, kWarps * 32, 0, st>>>(reinterpret_cast<const char*>(H), T, D, ld_bytes, rows,
                                                            rowmap, tp, tn, ov, orow, ocol, count, cap);
  return check_launch("atlas_filter_compact");
}

}  // namespace
}  // namespace atlas

extern "C" int atlas_filter_compact(const void* H, int dtype, int64_t T, int64_t D, int64_t ld,
                                    const int32_t* rowmap, const float* thr_pos, const float* thr_neg,
                                    float* out_val, int32_t* out_row, int32_t* out_col, int32_t* count,
                                    int64_t cap, void* stream) {
  using namespace atlas;
  ATLAS_REQUIRE(T >= 0 && D >= 0 && ld >= D, "filter: bad shape T=%lld D=%lld ld=%lld", (long long)T,
                (long long)D, (long long)ld);
  ATLAS_REQUIRE(cap >= 0, "filter: cap < 0");
  if (T == 0 || D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(H && rowmap && thr_pos && thr_neg && count, "filter: null pointer");
  ATLAS_REQUIRE(cap == 0 || (out_val && out_row && out_col), "filter: null output");
  ATLAS_REQUIRE(D < (1LL << 31), "filter: D too large");
  cudaStream_t st = (cudaStream_t)stream;
  const uintptr_t a = (uintptr_t)H;
  switch (dtype) {
    case ATLAS_BF16:
      if (D % 8 == 0 && ld % 8 == 0 && a % 16 == 0)
        return launch<ATLAS_BF16, 8, ATLAS_FILTER_U>(H, T, D, ld, rowmap, thr_pos, thr_neg, out_val, out_row, out_col, count, cap, st);
      return launch<ATLAS_BF16, 1, 4>(H, T, D, ld, rowmap, thr_pos, thr_neg, out_val, out_row, out_col, count, cap, st);
    case ATLAS_F16:
      if (D % 8 == 0 && ld % 8 == 0 && a % 16 == 0)
        return launch<ATLAS_F16, 8, ATLAS_FILTER_U>(H, T, D, ld, rowmap, thr_pos, thr_neg, out_val, out_row, out_col, count, cap, st);
      return launch<ATLAS_F16, 1, 4>(H, T, D, ld, rowmap, thr_pos, thr_neg, out_val, out_row, out_col, count, cap, st);
    case ATLAS_F32:
      if (D % 4 == 0 && ld % 4 == 0 && a % 16 == 0)
        return launch<ATLAS_F32, 4, ATLAS_FILTER_U>(H, T, D, ld, rowmap, thr_pos, thr_neg, out_val, out_row, out_col, count, cap, st);
      return launch<ATLAS_F32, 1, 4>(H, T, D, ld, rowmap, thr_pos, thr_neg, out_val, out_row, out_col, count, cap, st);
    default:
      return fail(ATLAS_ERR_ARG, "filter: unknown dtype %d", dtype);
  }
}
