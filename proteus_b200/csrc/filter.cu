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

template <>
struct Vec<ATLAS_BF16, 8> {
  uint4 v;
  __device__ __forceinline__ void load(const void* p) { v = __ldcs(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ float at(int k) const {
    const uint32_t w = k < 2 ? v.x : k < 4 ? v.y : k < 6 ? v.z : v.w;
    return (k & 1) ? __uint_as_float(w & 0xFFFF0000u) : __uint_as_float(w << 16);
  }
};
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

constexpr int kWarps = 8;
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
  const int warp = threadIdx.x >> 5;
  const int64_t c0 = ((int64_t)blockIdx.x * 32 + lane) * VEC;
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

  for (int64_t r = r_begin + warp; r < r_end; r += (int64_t)kWarps * U) {
    Vec<DT, VEC> x[U];
    int32_t vr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = r + (int64_t)u * kWarps;
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

template <int DT, int VEC, int U>
int launch(const void* H, int64_t T, int64_t D, int64_t ld, const int32_t* rowmap, const float* tp,
           const float* tn, float* ov, int32_t* orow, int32_t* ocol, int32_t* count, int64_t cap,
           cudaStream_t st) {
  const int64_t strips = (D + 32 * VEC - 1) / (32 * VEC);
  const int64_t target = (int64_t)num_sms() * kCtasPerSm;  // one resident wave of 8-warp CTAs
  int64_t chunks = (target + strips - 1) / strips;
  const int64_t step = (int64_t)kWarps * U;
  int64_t rows = (T + chunks - 1) / chunks;
  rows = ((rows + step - 1) / step) * step;
  if (rows < step) rows = step;
  chunks = (T + rows - 1) / rows;
  if (chunks < 1) chunks = 1;
  ATLAS_REQUIRE(strips < 65536 * 32 && chunks < 65536, "filter: grid too large (T=%lld D=%lld)",
                (long long)T, (long long)D);
  dim3 grid((unsigned)strips, (unsigned)chunks);
  filter_kernel<DT, VEC, U><<<grid, kWarps * 32, 0, st>>>(
      reinterpret_cast<const char*>(H), T, D, ld * (int64_t)sizeof(typename Elem<DT>::T), rows, rowmap, tp, tn,
      ov, orow, ocol, count, cap);
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
