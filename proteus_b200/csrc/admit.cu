// Candidate admission for the filtered layers of a batch (end of batch): the exact per-group tests
// of _merge_filtered_impl (atlas/core.py:482-527) over the compacted candidates, and the bulk-row
// reservoir path of _bulk_loop / _bulk_stacked (core.py:529-590) stacked over every layer in one
// launch. Admitted records go to SoA lists through warp-aggregated appends (one atomic per warp
// per step), ready for atlas_grouped_merge.
#include "common.cuh"

namespace atlas {
namespace {

struct Lists {
  int32_t* tg; int64_t* tsc; int64_t* ttok; float* tval; int32_t* nt; int64_t tcap;
  int32_t* rg; int64_t* rsc; int64_t* rtok; float* rval; int32_t* nr; int64_t rcap;
  int32_t* err;
};

// Append up to 2 records per lane to one list; the whole warp calls this.
__device__ __forceinline__ void warp_append(int lane, int n, const int32_t (&g)[2], const int64_t (&sc)[2],
                                            const int64_t (&tok)[2], const float (&val)[2], int32_t* gl, int64_t* scl,
                                            int64_t* tokl, float* vall, int32_t* counter, int64_t cap, int32_t* err) {
  if (!__any_sync(0xFFFFFFFFu, n > 0)) return;
  int total;
  const int pre = warp_excl_scan(n, lane, &total);
  int base = 0;
  if (lane == 31) base = atomicAdd(counter, total);
  base = __shfl_sync(0xFFFFFFFFu, base, 31);
  for (int k = 0; k < n; ++k) {
    const int64_t slot = (int64_t)base + pre + k;
    if (slot < cap) {
      gl[slot] = g[k];
      scl[slot] = sc[k];
      tokl[slot] = tok[k];
      vall[slot] = val[k];
    } else {
      atomicExch(err, 1);
    }
  }
}

template <typename T>
__device__ __forceinline__ float ld_elem(const T* p) { return Elem<ATLAS_F32>::f(*p); }
template <>
__device__ __forceinline__ float ld_elem<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float ld_elem<__half>(const __half* p) { return __half2float(*p); }

// Compacted candidates of every admitted layer in one flattened index space (a CTA first builds the
// prefix of the layers' candidate counts in shared memory), so every warp of the grid works on some
// layer's candidates at once instead of the layers taking turns. The state tests read the batch's
// compact thresholds: the group's K-th top key and the bin's ceiling max(res_s[., Kr-1], res_seed).
__global__ void __launch_bounds__(256)
admit_kernel(int64_t L, int64_t D, int64_t B, int64_t U_res, int reservoir, uint64_t mode_mask,
             const int32_t* __restrict__ count, int64_t cap_main, int64_t cap_early, int64_t early_layers,
             const float* __restrict__ cval, const int32_t* __restrict__ crow, const int32_t* __restrict__ ccol,
             int64_t cstride, const int64_t* __restrict__ tok, const int64_t* __restrict__ key,
             const float* __restrict__ top_seed, const int64_t* __restrict__ top_kth,
             const int64_t* __restrict__ res_thr, const float* __restrict__ E, Lists o) {
  __shared__ int64_t s_start[65];
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int64_t l = 0; l < L; ++l) {
      s_start[l] = acc;
      if ((mode_mask >> l) & 1) {
        const int64_t cap = l < early_layers ? cap_early : cap_main;
        const int64_t c = count[l];
        if (c <= cap) acc += c;  // an overflowed layer went through the dense path
      }
    }
    s_start[L] = acc;
  }
  __syncthreads();
  const int64_t total = s_start[L];
  const int64_t warp_id = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t base = warp_id * 32; base < total; base += n_warps * 32) {
    const int64_t f = base + lane;
    int nt = 0, nr = 0;
    int32_t tg[2], rg[2];
    int64_t tsc[2], rsc[2], tt[2], rt[2];
    float tv[2], rv[2];
    if (f < total) {
      int lo = 0, hi = (int)L;  // the layer whose range holds f: last l with s_start[l] <= f
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_start[mid] <= f) lo = mid; else hi = mid;
      }
      const int64_t l = lo, i = f - s_start[lo];
      const float h = cval[l * cstride + i];
      const int32_t row = crow[l * cstride + i];
      const int64_t col = ccol[l * cstride + i];
      const int64_t tk = tok[row], ky = key[row];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float s = p ? -h : h;
        const int64_t g = (l * 2 + p) * D + col;
        if (s > top_seed[g]) {
          const int64_t k64 = top_key(s, tk);
          if (k64 > top_kth[g]) {
            tg[nt] = (int32_t)g; tsc[nt] = k64; tt[nt] = tk; tv[nt] = s; ++nt;
          }
        }
        if (reservoir && ky >= U_res) {
          const int b = bin_of(s, E + g * B, (int)B);
          if (b >= 0) {
            const int64_t gr = g * B + b;
            if (-ky > res_thr[gr]) {
              rg[nr] = (int32_t)gr; rsc[nr] = -ky; rt[nr] = tk; rv[nr] = h; ++nr;
            }
          }
        }
      }
    }
    warp_append(lane, nt, tg, tsc, tt, tv, o.tg, o.tsc, o.ttok, o.tval, o.nt, o.tcap, o.err);
    warp_append(lane, nr, rg, rsc, rt, rv, o.rg, o.rsc, o.rtok, o.rval, o.nr, o.rcap, o.err);
  }
}

// Bulk rows (key < U_res; every element is a reservoir candidate). A CTA takes one layer, 256
// columns and a chunk of up to kAdmRows rows. It first copies its columns' reservoir ceilings
// (both poles, every bin; contiguous in the batch's compact array) into a shared-memory table and
// the chunk's row keys into shared memory; each thread then holds one column's bin edges in
// registers and walks the rows (R read coalesced along the columns).
constexpr int kAdmB = 8;
constexpr int kAdmRows = 64;  // most bulk rows per CTA (grid z); fewer when that leaves the GPU short of CTAs
constexpr int kAdmCols = 256;

template <typename RT, int NB>
__global__ void __launch_bounds__(kAdmCols)
admit_bulk_kernel(int64_t L, int64_t D, int64_t Kr, uint64_t mode_mask, const int32_t* __restrict__ count,
                  int64_t cap_main, int64_t cap_early, int64_t early_layers, const int64_t* __restrict__ tok,
                  const int64_t* __restrict__ key, const RT* __restrict__ R, int64_t n_r, int64_t r_stride,
                  const int32_t* __restrict__ bulk_vidx, const int64_t* __restrict__ res_thr,
                  const float* __restrict__ E, int rows_per_cta, Lists o) {
  const int lane = threadIdx.x & 31;
  const int64_t col = (int64_t)blockIdx.x * kAdmCols + threadIdx.x;
  const int64_t l = blockIdx.y;
  if (!((mode_mask >> l) & 1)) return;  // uniform per CTA
  const int64_t cap = l < early_layers ? cap_early : cap_main;
  if ((int64_t)count[l] > cap) return;  // overflowed: this layer went through the dense path
  __shared__ int64_t s_thr[2][NB][kAdmCols];
  __shared__ int64_t s_key[kAdmRows];
  __shared__ int32_t s_vi[kAdmRows];
  const bool ok = col < D;
  const int64_t i0 = (int64_t)blockIdx.z * rows_per_cta;  // rows_per_cta <= kAdmRows
  const int nrows = (int)(i0 + rows_per_cta < n_r ? rows_per_cta : n_r - i0);
  float e[2][NB];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int64_t g = (l * 2 + p) * D + (ok ? col : 0);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      e[p][b] = ok ? E[g * NB + b] : __int_as_float(0x7F800000);  // +inf: never reached
      s_thr[p][b][threadIdx.x] = ok ? res_thr[g * NB + b] : INT64_MAX;
    }
  }
  if (threadIdx.x < nrows) {
    const int32_t vi = bulk_vidx[i0 + threadIdx.x];
    s_vi[threadIdx.x] = vi;
    s_key[threadIdx.x] = key[vi];
  }
  __syncthreads();
  const RT* Rc = R + (l * r_stride + i0) * D + col;  // this column, first row of the chunk
  for (int r0 = 0; r0 < nrows; r0 += 8) {  // warp-uniform: every lane takes part in the appends
    float hv[8];  // eight rows' values in flight before any compare
#pragma unroll
    for (int u = 0; u < 8; ++u) hv[u] = (ok && r0 + u < nrows) ? ld_elem<RT>(Rc + (int64_t)(r0 + u) * D) : 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
    const int r = r0 + u;
    if (r >= nrows) break;
    int nr = 0;
    int32_t rg[2];
    int64_t rsc[2], rt[2];
    float rv[2];
    const int64_t ky = s_key[r];
    if (ok) {
      const float h = hv[u];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float s = p ? -h : h;
        int b = -1;
#pragma unroll
        for (int q = 0; q < NB; ++q) b += (s >= e[p][q]) ? 1 : 0;
        if (b >= 0 && -ky > s_thr[p][b][threadIdx.x]) {
          rg[nr] = (int32_t)((((l * 2 + p) * D + col) * NB) + b);
          rsc[nr] = -ky;
          rt[nr] = tok[s_vi[r]];
          rv[nr] = h;
          ++nr;
        }
      }
    }
    warp_append(lane, nr, rg, rsc, rt, rv, o.rg, o.rsc, o.rtok, o.rval, o.nr, o.rcap, o.err);
    }
  }
}

template <typename RT, int NB>
void launch_admit_bulk(dim3 gb, cudaStream_t st, int64_t L, int64_t D, int64_t Kr, uint64_t mask, const int32_t* count,
                       int64_t cap_main, int64_t cap_early, int64_t early_layers, const int64_t* tok, const int64_t* key,
                       const void* R, int64_t n_r, int64_t r_stride, const int32_t* bulk_vidx, const int64_t* res_thr,
                       const float* E, int rows_per_cta, Lists o) {
  admit_bulk_kernel<RT, NB><<<gb, kAdmCols, 0, st>>>(L, D, Kr, mask, count, cap_main, cap_early, early_layers, tok, key,
                                                    (const RT*)R, n_r, r_stride, bulk_vidx, res_thr, E, rows_per_cta,
                                                    o);
}

template <typename RT>
int launch_admit_bulk_b(int64_t B, dim3 gb, cudaStream_t st, int64_t L, int64_t D, int64_t Kr, uint64_t mask,
                        const int32_t* count, int64_t cap_main, int64_t cap_early, int64_t early_layers,
                        const int64_t* tok, const int64_t* key, const void* R, int64_t n_r, int64_t r_stride,
                        const int32_t* bulk_vidx, const int64_t* res_thr, const float* E, int rows_per_cta, Lists o) {
#define ATLAS_ADMIT_B(NBV)                                                                                           \
  case NBV:                                                                                                         \
    launch_admit_bulk<RT, NBV>(gb, st, L, D, Kr, mask, count, cap_main, cap_early, early_layers, tok, key, R, n_r,  \
                               r_stride, bulk_vidx, res_thr, E, rows_per_cta, o);                                   \
    return ATLAS_OK;
  switch (B) {
    ATLAS_ADMIT_B(1) ATLAS_ADMIT_B(2) ATLAS_ADMIT_B(3) ATLAS_ADMIT_B(4)
    ATLAS_ADMIT_B(5) ATLAS_ADMIT_B(6) ATLAS_ADMIT_B(7) ATLAS_ADMIT_B(8)
    default: return fail(ATLAS_ERR_ARG, "admit: B must be 1..%d", kAdmB);
  }
#undef ATLAS_ADMIT_B
}

}  // namespace
}  // namespace atlas

using namespace atlas;

extern "C" int atlas_admit(int64_t L, int64_t D, int64_t B, int64_t K, int64_t Kr, int64_t U_res, int reservoir,
                           const int8_t* layer_mode_host, const int32_t* count, int64_t cap_main, int64_t cap_early,
                           int64_t early_layers, const float* cand_val, const int32_t* cand_row, const int32_t* cand_col,
                           int64_t cand_stride, const int64_t* tok, const int64_t* key, const void* R, int dtype,
                           int64_t n_r, int64_t r_stride, const int32_t* bulk_vidx, const float* top_seed,
                           const int64_t* top_kth, const int64_t* res_thr, const float* E, int32_t* top_g,
                           int64_t* top_sc, int64_t* top_tok, float* top_val, int32_t* n_top, int64_t top_cap,
                           int32_t* res_g, int64_t* res_sc, int64_t* res_tok, float* res_val, int32_t* n_res,
                           int64_t res_cap, int32_t* err, void* stream) {
  ATLAS_REQUIRE(L >= 0 && L <= 64, "admit: L must be 0..64");
  ATLAS_REQUIRE(D > 0 && B >= 1 && K >= 1 && Kr >= 1 && n_r >= 0 && r_stride >= n_r, "admit: bad sizes");
  ATLAS_REQUIRE(2 * L * D * B < (1LL << 31), "admit: group ids exceed int32");
  uint64_t mask = 0;
  for (int64_t l = 0; l < L; ++l)
    if (layer_mode_host && layer_mode_host[l]) mask |= 1ull << l;
  if (mask == 0) return ATLAS_OK;
  ATLAS_REQUIRE(count && cand_val && cand_row && cand_col && tok && key && top_seed && top_kth && n_top && top_g &&
                    top_sc && top_tok && top_val && err,
                "admit: null pointer");
  ATLAS_REQUIRE(!reservoir || (res_thr && E && res_g && res_sc && res_tok && res_val && n_res),
                "admit: null reservoir pointer");
  ATLAS_REQUIRE(!reservoir || n_r == 0 || (R && bulk_vidx), "admit: bulk rows missing");
  Lists o{top_g, top_sc, top_tok, top_val, n_top, top_cap, res_g, res_sc, res_tok, res_val, n_res, res_cap, err};
  ATLAS_REQUIRE(B <= kAdmB, "admit: at most %d bins", kAdmB);
  const int64_t per_layer = cap_main > cap_early ? cap_main : cap_early;
  const unsigned grid = grid_for(per_layer * L, 256, 8);
  cudaStream_t st = (cudaStream_t)stream;
  admit_kernel<<<grid, 256, 0, st>>>(L, D, B, U_res, reservoir, mask, count, cap_main, cap_early, early_layers, cand_val,
                                     cand_row, cand_col, cand_stride, tok, key, top_seed, top_kth, res_thr, E, o);
  if (int e = check_launch("atlas_admit")) return e;
  if (!reservoir || n_r == 0) return ATLAS_OK;
  // rows per CTA: up to kAdmRows (the column's thresholds are loaded once per CTA), but at least about
  // one wave of CTAs (8 per SM) when the batch has few layers or bulk rows
  const int64_t col_blocks = (D + kAdmCols - 1) / kAdmCols;
  int64_t rpc = (n_r * col_blocks * L + (int64_t)num_sms() * 8 - 1) / ((int64_t)num_sms() * 8);
  rpc = rpc < 8 ? 8 : (rpc > kAdmRows ? kAdmRows : rpc);
  ATLAS_REQUIRE(L < 65536 && (n_r + rpc - 1) / rpc < 65536, "admit: too many layers or bulk rows");
  const dim3 gb((unsigned)col_blocks, (unsigned)L, (unsigned)((n_r + rpc - 1) / rpc));
  const int rows_per_cta = (int)rpc;
  int e2;
  switch (dtype) {
    case ATLAS_BF16:
      e2 = launch_admit_bulk_b<__nv_bfloat16>(B, gb, st, L, D, Kr, mask, count, cap_main, cap_early, early_layers, tok,
                                              key, R, n_r, r_stride, bulk_vidx, res_thr, E, rows_per_cta, o);
      break;
    case ATLAS_F16:
      e2 = launch_admit_bulk_b<__half>(B, gb, st, L, D, Kr, mask, count, cap_main, cap_early, early_layers, tok, key, R,
                                       n_r, r_stride, bulk_vidx, res_thr, E, rows_per_cta, o);
      break;
    case ATLAS_F32:
      e2 = launch_admit_bulk_b<float>(B, gb, st, L, D, Kr, mask, count, cap_main, cap_early, early_layers, tok, key, R,
                                      n_r, r_stride, bulk_vidx, res_thr, E, rows_per_cta, o);
      break;
    default:
      return fail(ATLAS_ERR_ARG, "admit: unknown dtype %d", dtype);
  }
  if (e2) return e2;
  return check_launch("atlas_admit: bulk rows");
}
