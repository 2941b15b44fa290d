// K1: single-pass compare-and-compact over the hook output H (one read of H per layer).
//
// Replaces filter_candidates (atlas/filter_triton.py:19-86). Two kernels, one contract:
//  * bf16 with 16-byte-aligned rows (the hot case): filter_bulk_kernel, TMA-fed (see its section
//    below): a producer warp streams 32-row x 256-column tiles through shared memory, consumer warps
//    compare packed bf16 pairs and park rare hits in per-warp queues.
//  * fp16 / fp32 and unaligned shapes: filter_kernel, register-fed: each warp owns a strip of
//    32 * VEC consecutive columns (one 16-byte vector per lane, VEC = 8 for 16-bit types, 4 for
//    fp32, 1 when unaligned) and walks rows with U rows in flight per lane; the per-column
//    thresholds live in registers for the whole walk.
// Padding rows (rowmap < 0) are never read by the register path and never copied by the TMA path
// unless they share a 32-row tile with a valid row. Compaction is two-level in both: survivors are
// staged per CTA in shared memory, and the CTA reserves its global output range with ONE global
// atomic at the end and copies them out with coalesced stores (per-step global atomics on the one
// counter would serialise the pass at ~0.1-0.5% survivors); survivors that do not fit the staging
// area go straight to the global list, so the count stays exact for any survivor density.
#include "tc.cuh"

namespace atlas {
namespace {

// Raw vector of VEC elements as loaded (16 bytes on the vector paths); elements are widened to
// fp32 on use, so a lane keeps U raw vectors in flight in few registers.
template <int DT, int VEC>
struct Vec;

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
#ifndef ATLAS_FILTER_STAGE
#define ATLAS_FILTER_STAGE 2048  // staged survivors per CTA (12 bytes each)
#endif
constexpr int kStage = ATLAS_FILTER_STAGE;
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

// ------------------------------------------------------------------ bf16 compare and emit helpers
// Compares run on packed bf16 pairs against thresholds rounded to bf16 (toward -inf for the
// positive pole, toward +inf for the negative pole). For a bf16 value h and an fp32 threshold t,
// h > t  <=>  h > rd_bf16(t)  and  h < t  <=>  h < ru_bf16(t) (no bf16 lies strictly between t and
// its directed rounding), so the survivors are exactly those of the fp32 comparison; NaN compares
// false on both sides as in fp32.
template <int N>
struct StageAreaN {
  static constexpr int kCap = N;
  float val[N];
  int32_t row[N], col[N];
  int n;
};
using StageArea = StageAreaN<kStage>;

// One survivor: a staging slot while the area has room, else straight to the global list (the
// global counter stays exact past `cap`).
template <class SA>
__device__ __forceinline__ void emit_one(SA& sa, float h, int32_t row, int32_t col, float* __restrict__ out_val,
                                         int32_t* __restrict__ out_row, int32_t* __restrict__ out_col,
                                         int32_t* __restrict__ count, int64_t cap) {
  const int slot = atomicAdd(&sa.n, 1);
  if (slot < SA::kCap) {
    sa.val[slot] = h;
    sa.row[slot] = row;
    sa.col[slot] = col;
  } else {
    const int64_t g = atomicAdd(count, 1);
    if (g < cap) {
      out_val[g] = h;
      out_row[g] = row;
      out_col[g] = col;
    }
  }
}

// Hit mask of one 16-byte row vector (8 columns): bit k set when element k survives.
__device__ __forceinline__ uint32_t hit_bits8(const uint4& x, const __nv_bfloat162 (&tp2)[4],
                                              const __nv_bfloat162 (&tn2)[4]) {
  const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
  uint32_t m[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[w]);
    m[w] = __hgt2_mask(h2, tp2[w]) | __hlt2_mask(h2, tn2[w]);
  }
  // one byte per element (0x00 / 0xFF), then the byte signs gathered into 8 bits
  const uint32_t lo = __byte_perm(m[0], m[1], 0x6420), hi = __byte_perm(m[2], m[3], 0x6420);
  return (((lo & 0x80808080u) * 0x00204081u) >> 28) | ((((hi & 0x80808080u) * 0x00204081u) >> 28) << 4);
}

// Per-row "any hit" flags of one step of a lane (U row vectors of 8 columns): 3 instructions per
// 32-bit word, no extraction. Rows with v < 0 (padding) never hit.
template <int U>
__device__ __forceinline__ uint32_t bf16_flags(const uint4 (&x)[U], const int32_t (&v)[U], const __nv_bfloat162 (&tp2)[4],
                                               const __nv_bfloat162 (&tn2)[4]) {
  uint32_t flags = 0;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint32_t w4[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
    uint32_t a = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[w]);
      a |= __hgt2_mask(h2, tp2[w]) | __hlt2_mask(h2, tn2[w]);
    }
    if (a != 0 && v[u] >= 0) flags |= 1u << u;
  }
  return flags;
}

// Survivors of one step of a lane (rows flagged in `flags`): the 8-bit masks of the flagged rows,
// ONE shared-memory reservation for all of them, then plain stores. Slots past the staging area go
// straight to the global list (global atomic per survivor; the count stays exact past `cap`).
template <int U, class SA>
__device__ __forceinline__ void bf16_emit_step(uint32_t flags, const uint4 (&x)[U], const int32_t (&v)[U],
                                               const __nv_bfloat162 (&tp2)[4], const __nv_bfloat162 (&tn2)[4], int c0,
                                               SA& sa, float* __restrict__ out_val, int32_t* __restrict__ out_row,
                                               int32_t* __restrict__ out_col, int32_t* __restrict__ count,
                                               int64_t cap) {
  uint32_t bits[U];
  int n = 0;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    bits[u] = (flags & (1u << u)) ? hit_bits8(x[u], tp2, tn2) : 0u;
    n += __popc(bits[u]);
  }
  int slot = atomicAdd(&sa.n, n);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    uint32_t b = bits[u];
    while (b) {
      const int k = __ffs(b) - 1;
      b &= b - 1;
      const uint32_t w = k < 2 ? x[u].x : k < 4 ? x[u].y : k < 6 ? x[u].z : x[u].w;
      const float h = (k & 1) ? __uint_as_float(w & 0xFFFF0000u) : __uint_as_float(w << 16);
      if (slot < SA::kCap) {
        sa.val[slot] = h;
        sa.row[slot] = v[u];
        sa.col[slot] = c0 + k;
      } else {
        const int64_t g = atomicAdd(count, 1);
        if (g < cap) {
          out_val[g] = h;
          out_row[g] = v[u];
          out_col[g] = c0 + k;
        }
      }
      ++slot;
    }
  }
}

// ------------------------------------------------------------------ bf16, TMA-fed
// The strip of 256 columns (512 bytes per row) a CTA owns is streamed through a ring of shared
// memory stages by TMA: one 2-D tile copy of 32 rows x 256 columns (16 KB) per stage, completion
// counted on an mbarrier. The bytes in flight are bounded by shared memory (kBStages x 16 KB per
// CTA), not by registers, so HBM sees a deep queue however long the compare-and-emit work of a row
// takes; one copy per 16 KB keeps the SM's TMA unit far from its issue limit (per-row 512-byte
// bulk copies saturated it at about half the HBM bandwidth). Warp kBWarps produces (row-map
// entries four stages ahead; a stage of padding rows only is not copied), warps 0..kBWarps-1
// consume 4 rows of each stage (one 16-byte vector per lane per row, read from shared memory),
// release the stage as soon as their vectors are in registers, then compare (per-row "any hit"
// flags) and park flagged row vectors in the warp's hit queue. Padding rows inside a stage are
// copied with it and skipped. Every wait is bounded; a wait that gives up records a code in the
// device status word and the CTA finishes (the producer first waits, again bounded, for the copies
// it issued).
#ifndef ATLAS_FILTER_BSTAGES
#define ATLAS_FILTER_BSTAGES 3
#endif
#ifndef ATLAS_FILTER_BCTAS
#define ATLAS_FILTER_BCTAS 3
#endif
constexpr int kBRows = 32;                       // rows per stage
constexpr int kBStages = ATLAS_FILTER_BSTAGES;   // stages per CTA
constexpr int kBWarps = 8;                       // consumer warps (4 rows of a stage each)
constexpr int kBThreads = (kBWarps + 1) * 32;
constexpr int kBCtasPerSm = ATLAS_FILTER_BCTAS;
constexpr int kBSeg = 512;                       // bytes of one row segment (256 bf16 columns)
#ifndef ATLAS_FILTER_BSTAGE_N
#define ATLAS_FILTER_BSTAGE_N 1024
#endif
constexpr int kBStage = ATLAS_FILTER_BSTAGE_N;   // staged survivors per CTA (12 bytes each)

#ifndef ATLAS_FILTER_QUEUE
#define ATLAS_FILTER_QUEUE 1
#endif
#ifndef ATLAS_FILTER_BQUEUE
#define ATLAS_FILTER_BQUEUE 64
#endif
constexpr int kBQueue = ATLAS_FILTER_BQUEUE;  // flagged row vectors parked per consumer warp

// Flagged row vectors of one consumer warp, waiting for extraction: the 16 bytes, the row-map entry
// and the lane (the lane gives the 8 columns and their thresholds).
struct HitQueue {
  uint4 x[kBQueue];
  int32_t v[kBQueue];
  int32_t lane[kBQueue];
};

struct BulkSmem {
  uint4 data[kBStages][kBRows][kBSeg / 16];
  int32_t rows[kBStages][kBRows];
  uint64_t full[kBStages], empty[kBStages];
  StageAreaN<kBStage> sa;
  uint4 thr[32][2];  // per lane of the strip: bf16x2 thresholds (positive, negative pole)
  HitQueue q[kBWarps];
  int s_base;
};

// Extraction of a warp's parked row vectors: lane i takes entries i, i+32, ..., each with one
// staging reservation (no divergence beyond the per-entry survivor count).
template <class SA>
__device__ __forceinline__ void drain_queue(const HitQueue& q, int qn, const uint4 (&thr)[32][2], int s0, int lane, SA& sa,
                                            float* __restrict__ out_val, int32_t* __restrict__ out_row,
                                            int32_t* __restrict__ out_col, int32_t* __restrict__ count, int64_t cap) {
  __syncwarp();
  for (int e = lane; e < qn; e += 32) {
    const uint4 xe[1] = {q.x[e]};
    const int32_t ve[1] = {q.v[e]};
    const int L = q.lane[e];
    const uint4 tw = thr[L][0], nw = thr[L][1];
    const __nv_bfloat162 tp2[4] = {*reinterpret_cast<const __nv_bfloat162*>(&tw.x), *reinterpret_cast<const __nv_bfloat162*>(&tw.y),
                                   *reinterpret_cast<const __nv_bfloat162*>(&tw.z), *reinterpret_cast<const __nv_bfloat162*>(&tw.w)};
    const __nv_bfloat162 tn2[4] = {*reinterpret_cast<const __nv_bfloat162*>(&nw.x), *reinterpret_cast<const __nv_bfloat162*>(&nw.y),
                                   *reinterpret_cast<const __nv_bfloat162*>(&nw.z), *reinterpret_cast<const __nv_bfloat162*>(&nw.w)};
    bf16_emit_step<1>(1u, xe, ve, tp2, tn2, s0 + L * 8, sa, out_val, out_row, out_col, count, cap);
  }
  __syncwarp();
}

__global__ void __launch_bounds__(kBThreads, kBCtasPerSm)
filter_bulk_kernel(const __grid_constant__ CUtensorMap tmap, int T, int D, int rows_per_cta,
                   const int32_t* __restrict__ rowmap, const float* __restrict__ thr_pos,
                   const float* __restrict__ thr_neg, float* __restrict__ out_val, int32_t* __restrict__ out_row,
                   int32_t* __restrict__ out_col, int32_t* __restrict__ count, int64_t cap) {
  extern __shared__ uint8_t bulk_raw[];
  BulkSmem& sm = *reinterpret_cast<BulkSmem*>((reinterpret_cast<uintptr_t>(bulk_raw) + 127) & ~uintptr_t(127));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int s0 = blockIdx.x * (kBSeg / 2);  // first column of the strip
  const int r_begin = blockIdx.y * rows_per_cta;
  const int r_end = min(r_begin + rows_per_cta, T);
  const int n_stages = r_end > r_begin ? (r_end - r_begin + kBRows - 1) / kBRows : 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kBStages; ++i) {
      tc::mbar_init(&sm.full[i], 1);
      tc::mbar_init(&sm.empty[i], kBWarps);
    }
    sm.sa.n = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  if (warp == kBWarps) {  // producer
    // row-map entries of this lane's row in stages k .. k+3, loaded four stages ahead so no copy
    // waits on a dependent row-map load
    auto rm_at = [&](int k) -> int32_t {
      const int row = r_begin + k * kBRows + lane;
      return row < r_end ? __ldg(rowmap + row) : -1;
    };
    int32_t rm0 = rm_at(0), rm1 = rm_at(1), rm2 = rm_at(2), rm3 = rm_at(3);
    int issued = 0;
    for (int k = 0; k < n_stages; ++k) {
      const int st = k % kBStages;
      const uint32_t ph = (uint32_t)(k / kBStages) & 1;
      // every lane waits (and so acquires the consumers' release); the decision is warp-uniform
      if (k >= kBStages && !__all_sync(0xFFFFFFFFu, tc::mbar_wait(&sm.empty[st], ph ^ 1, 301))) break;
      const int32_t vr = rm0;
      rm0 = rm1;
      rm1 = rm2;
      rm2 = rm3;
      rm3 = rm_at(k + 4);
      sm.rows[st][lane] = vr;
      const bool any_valid = __any_sync(0xFFFFFFFFu, vr >= 0);
      __syncwarp();
      if (lane == 0) {  // one 2-D tile copy per stage: 32 rows x 256 columns (out-of-range parts read as 0)
        if (any_valid) {
          tc::mbar_arrive_expect_tx(&sm.full[st], kBRows * kBSeg);
          tc::tma_load_2d(&sm.data[st][0][0], &tmap, s0, r_begin + k * kBRows, &sm.full[st]);
        } else {
          tc::mbar_arrive(&sm.full[st]);  // a stage of padding rows only: nothing to copy
        }
      }
      issued = k + 1;
    }
    if (issued < n_stages && lane == 0) {  // gave up: let the copies already issued land first
      for (int k = max(0, issued - kBStages); k < issued; ++k)
        tc::mbar_wait(&sm.full[k % kBStages], (uint32_t)(k / kBStages) & 1, 302);
    }
  } else {  // consumers
    const int c0 = s0 + lane * 8;
    const bool col_ok = c0 < D;
    __nv_bfloat162 tp2[4], tn2[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      __nv_bfloat16 p[2], n[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = c0 + 2 * w + h;
        p[h] = __float2bfloat16_rd(col_ok ? __ldg(thr_pos + c) : __int_as_float(0x7F800000));
        n[h] = __float2bfloat16_ru(col_ok ? -__ldg(thr_neg + c) : __int_as_float(0xFF800000));
      }
      tp2[w] = __halves2bfloat162(p[0], p[1]);
      tn2[w] = __halves2bfloat162(n[0], n[1]);
    }
    constexpr int U = kBRows / kBWarps;
#if ATLAS_FILTER_QUEUE
    // Survivors are rare: a lane with hits parks its flagged row vectors in the warp's queue
    // (positions from ballots, no atomics) and the warp extracts them 32 at a time, all lanes
    // busy, instead of the whole warp idling through one lane's extraction.
    if (warp == 0) {
      sm.thr[lane][0] = *reinterpret_cast<const uint4*>(tp2);
      sm.thr[lane][1] = *reinterpret_cast<const uint4*>(tn2);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kBWarps * 32) : "memory");  // consumer warps only
    HitQueue& q = sm.q[warp];
    const uint32_t lt = (1u << lane) - 1u;
    int qn = 0;  // warp-uniform fill of the queue
#endif
    for (int k = 0; k < n_stages; ++k) {
      const int st = k % kBStages;
      if (!__all_sync(0xFFFFFFFFu, tc::mbar_wait(&sm.full[st], (uint32_t)(k / kBStages) & 1, 303))) break;
      uint4 x[U];
      int32_t v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int r = warp + u * kBWarps;
        v[u] = col_ok ? sm.rows[st][r] : -1;
        x[u] = sm.data[st][r][lane];
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&sm.empty[st]);
      const uint32_t flags = bf16_flags<U>(x, v, tp2, tn2);
#if ATLAS_FILTER_QUEUE
      uint32_t bal[U];
      int tot = 0;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        bal[u] = __ballot_sync(0xFFFFFFFFu, (flags >> u) & 1u);
        tot += __popc(bal[u]);
      }
      if (tot) {
        if (tot > kBQueue) {  // denser than the queue: extract in place
          if (flags) bf16_emit_step<U>(flags, x, v, tp2, tn2, c0, sm.sa, out_val, out_row, out_col, count, cap);
        } else {
          if (qn + tot > kBQueue) {
            drain_queue(q, qn, sm.thr, s0, lane, sm.sa, out_val, out_row, out_col, count, cap);
            qn = 0;
          }
          int base = qn;
#pragma unroll
          for (int u = 0; u < U; ++u) {
            if ((flags >> u) & 1u) {
              const int pos = base + __popc(bal[u] & lt);
              q.x[pos] = x[u];
              q.v[pos] = v[u];
              q.lane[pos] = lane;
            }
            base += __popc(bal[u]);
          }
          qn += tot;
          if (qn >= 32) {
            drain_queue(q, qn, sm.thr, s0, lane, sm.sa, out_val, out_row, out_col, count, cap);
            qn = 0;
          }
        }
      }
#else
      if (flags) bf16_emit_step<U>(flags, x, v, tp2, tn2, c0, sm.sa, out_val, out_row, out_col, count, cap);
#endif
    }
#if ATLAS_FILTER_QUEUE
    if (qn) drain_queue(q, qn, sm.thr, s0, lane, sm.sa, out_val, out_row, out_col, count, cap);
#endif
  }
  __syncthreads();
  const int staged_n = sm.sa.n < kBStage ? sm.sa.n : kBStage;  // slots [0, staged_n) are all staged
  if (threadIdx.x == 0) sm.s_base = staged_n > 0 ? atomicAdd(count, staged_n) : 0;
  __syncthreads();
  const int64_t base = sm.s_base;
  for (int i = threadIdx.x; i < staged_n; i += blockDim.x) {
    const int64_t slot = base + i;
    if (slot < cap) {
      out_val[slot] = sm.sa.val[i];
      out_row[slot] = sm.sa.row[i];
      out_col[slot] = sm.sa.col[i];
    }
  }
}

int launch_bulk(const void* H, int64_t T, int64_t D, int64_t ld, const int32_t* rowmap, const float* tp,
                const float* tn, float* ov, int32_t* orow, int32_t* ocol, int32_t* count, int64_t cap,
                cudaStream_t st) {
  const int64_t strips = (D + kBSeg / 2 - 1) / (kBSeg / 2);
  int64_t chunks = (int64_t)num_sms() * kBCtasPerSm / strips;  // at most one resident wave
  if (chunks < 1) chunks = 1;
  int64_t rows = (T + chunks - 1) / chunks;
  rows = (rows + kBRows - 1) / kBRows * kBRows;
  chunks = (T + rows - 1) / rows;
  ATLAS_REQUIRE(strips < 65536 * 32 && chunks < 65536, "filter: grid too large (T=%lld D=%lld)", (long long)T,
                (long long)D);
  const size_t smem = sizeof(BulkSmem) + 128;
  static_assert(kBCtasPerSm * (sizeof(BulkSmem) + 128 + 1024) <= 228 * 1024, "bulk filter: CTAs do not fit an SM");
  static bool attr_set[64] = {};  // per device: a function attribute belongs to one device's context
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cudaFuncSetAttribute(filter_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return fail(ATLAS_ERR_CUDA, "filter: cannot reserve %zu bytes of shared memory", smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  CUtensorMap tm;
  if (int e = make_tmap_2d(&tm, H, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)D, (uint64_t)T, (uint64_t)ld * 2,
                           kBSeg / 2, kBRows, CU_TENSOR_MAP_SWIZZLE_NONE))
    return e;
  dim3 grid((unsigned)strips, (unsigned)chunks);
  filter_bulk_kernel<<<grid, kBThreads, smem, st>>>(tm, (int)T, (int)D, (int)rows, rowmap, tp, tn, ov, orow, ocol, count,
                                                    cap);
  return check_launch("atlas_filter_compact");
}

template <int DT, int VEC, int U>
int launch(const void* H, int64_t T, int64_t D, int64_t ld, const int32_t* rowmap, const float* tp,
           const float* tn, float* ov, int32_t* orow, int32_t* ocol, int32_t* count, int64_t cap,
           cudaStream_t st) {
  const int64_t strips = (D + 32 * VEC * kWX - 1) / (32 * VEC * kWX);
  // At most one resident wave of CTAs: a grid even a few CTAs larger runs those few as a second
  // wave after the first one and nearly doubles the pass.
  const int64_t target = (int64_t)num_sms() * kCtasPerSm;
  int64_t chunks = target / strips;
  if (chunks < 1) chunks = 1;
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
  filter_kernel<DT, VEC, U><<<grid, kWarps * 32, 0, st>>>(reinterpret_cast<const char*>(H), T, D, ld_bytes, rows,
                                                          rowmap, tp, tn, ov, orow, ocol, count, cap);
  return check_launch("atlas_filter_compact");
}

}  // namespace

// The bounded waits of this file record into this translation unit's copy of the status word.
int filter_device_status(int* v, int reset) {
  if (cudaMemcpyFromSymbol(v, tc::g_device_status, sizeof(int)) != cudaSuccess) return ATLAS_ERR_CUDA;
  if (reset && *v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(tc::g_device_status, &z, sizeof(int)) != cudaSuccess) return ATLAS_ERR_CUDA;
  }
  return ATLAS_OK;
}

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
  ATLAS_REQUIRE(D < (1LL << 30) && T < (1LL << 30), "filter: T or D too large (T=%lld D=%lld)", (long long)T, (long long)D);
  cudaStream_t st = (cudaStream_t)stream;
  const uintptr_t a = (uintptr_t)H;
  switch (dtype) {
    case ATLAS_BF16:
      if (D % 8 == 0 && ld % 8 == 0 && a % 16 == 0)
        return launch_bulk(H, T, D, ld, rowmap, thr_pos, thr_neg, out_val, out_row, out_col, count, cap, st);
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
