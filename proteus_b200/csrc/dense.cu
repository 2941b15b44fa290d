// Dense burst path (Atlas._dense, atlas/core.py:407-446) on the live hook output, predicated on the
// device: it runs when the layer is a dense layer (force) or when its compaction buffer overflowed
// (*count > cap, the 0.5%-fill trigger), so the forward is never re-run and the host never syncs.
//
// 1. dense_gather: the valid rows are transposed into a column-major scratch HT [D, n_v] (coalesced
//    reads and writes through shared-memory tiles), so every column below is one contiguous run.
//    The same launch writes the rows' 32-bit hash keys in row order and in ascending key order.
// 2. dense_column: one CTA per column at a time (grid-stride), both poles.
//    top-K: the admissible candidates (s > seed, top_key above the state's K-th key) are counted in
//      a row-order pass; a pole with at most K of them emits exactly those; otherwise an exact radix
//      select (8-bit digits, MSB first, per-warp shared-memory histograms) finds the K-th largest
//      composite key (ordered s bits | 2^32-1-tok), i.e. the reference's top_key; digits that are
//      constant for bf16/fp16 inputs are skipped, and token ids are read only for elements tied on
//      the whole value.
//    reservoir: the same row-order pass counts the rows under each (pole, bin)'s key ceiling; a bin
//      with at most Kr of them admits them all (no ordering needed), and only the bins with more
//      walk the key order, a block-wide chunk at a time, taking their first Kr rows in ascending key
//      order until every such bin is full or the keys pass its ceiling.
//    Records are staged in shared memory and appended with one atomic per list per CTA.
#include <algorithm>

#include "common.cuh"

namespace atlas {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxB = 8;
constexpr int kStage = 1024;  // staged records per CTA (top: <= 2K; reservoir: <= 2*B*Kr)
constexpr int kDenseSmemMax = 227 * 1024;  // opt-in shared memory per CTA

struct Lists {
  int32_t* g; int64_t* sc; int64_t* tok; float* val; int32_t* n; int64_t cap;
};

// High word of the composite key (ordered s bits, unsigned order): top_key's value part.
__device__ __forceinline__ uint32_t key_hi(float s) { return (uint32_t)(int32_t)ordered_f32(s) ^ 0x80000000u; }

template <int DT>
__device__ __forceinline__ bool skip_pass(int pass) {
  if (DT == ATLAS_BF16) return pass == 2 || pass == 3;  // fp32 bits 15..0 of a bf16 value are constant
  if (DT == ATLAS_F16) return pass == 3;                // fp32 bits 7..0 of an fp16 value are constant
  return false;
}

__device__ __forceinline__ bool triggered(const int32_t* count, int64_t cap, int force) {
  return force || (int64_t)*count > cap;
}

// ---------------------------------------------------------------------------------------- gather
// Grid-stride over 32x32 tiles (tile t: rows 32*(t % nti), columns 32*(t / nti)) with a grid bounded
// by the SM count, so the untriggered case costs a few thousand early exits, not one block per tile.
// With key32 given, the same launch first writes the rows' 32-bit hash keys (token keys lie in
// [0, 2^32)): key32[i] in valid-row order for the row-order passes, skey32[j] = key[key_order[j]]
// in ascending key order for the ordered walk.
template <typename T>
__global__ void dense_gather_kernel(const T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ rows,
                                    int64_t n, int64_t n8, T* __restrict__ HT, int64_t ldh,
                                    const int64_t* __restrict__ key, const int32_t* __restrict__ key_order,
                                    uint32_t* __restrict__ key32, uint32_t* __restrict__ skey32,
                                    const int32_t* __restrict__ count, int64_t cap, int force) {
  if (!triggered(count, cap, force)) return;
  __shared__ T tile[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;
  if (key32 != nullptr) {
    const int64_t stride = (int64_t)gridDim.x * 256;
    for (int64_t j = (int64_t)blockIdx.x * 256 + ty * 32 + tx; j < n; j += stride) {
      key32[j] = (uint32_t)key[j];
      skey32[j] = (uint32_t)key[key_order[j]];
    }
  }
  const int64_t nti = (n8 + 31) / 32, ntiles = nti * ((D + 31) / 32);
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t i0 = (t % nti) * 32, d0 = (t / nti) * 32;
    for (int k = ty; k < 32; k += 8) {
      const int64_t i = i0 + k, d = d0 + tx;
      T v = T(0.0f);
      if (i < n && d < D) v = H[(int64_t)rows[i] * ld + d];
      tile[k][tx] = v;
    }
    __syncthreads();
    for (int k = ty; k < 32; k += 8) {
      const int64_t d = d0 + k, i = i0 + tx;
      if (d < D && i < n8) HT[d * ldh + i] = tile[tx][k];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------- column
// Records of one column staged in shared memory: top-K records from slot 0 up (at most 2K),
// reservoir records from slot kStage-1 down (at most kStage - 2K >= 2*B*Kr); each part is appended
// to its list with one global atomic per CTA.
struct Staged {
  int32_t g[kStage];
  int64_t sc[kStage], tok[kStage];
  float val[kStage];
  int n, m;
};

__device__ __forceinline__ void stage_top(Staged& st, int lim, int32_t g, int64_t sc, int64_t tok, float val,
                                          int32_t* err) {
  const int i = atomicAdd(&st.n, 1);
  if (i < lim) {
    st.g[i] = g; st.sc[i] = sc; st.tok[i] = tok; st.val[i] = val;
  } else {
    atomicExch(err, 1);
  }
}

__device__ __forceinline__ void stage_res(Staged& st, int lim, int32_t g, int64_t sc, int64_t tok, float val,
                                          int32_t* err) {
  const int j = atomicAdd(&st.m, 1);
  if (j < lim) {
    const int i = kStage - 1 - j;
    st.g[i] = g; st.sc[i] = sc; st.tok[i] = tok; st.val[i] = val;
  } else {
    atomicExch(err, 1);
  }
}

// Appends staged slots [lo, lo + n) to list o. All threads call it after a barrier.
__device__ void flush_range(const Staged& st, int lo, int n, const Lists& o, int32_t* err, int* s_base) {
  if (threadIdx.x == 0) *s_base = n > 0 ? atomicAdd(o.n, n) : 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t slot = (int64_t)*s_base + i;
    if (slot < o.cap) {
      o.g[slot] = st.g[lo + i]; o.sc[slot] = st.sc[lo + i]; o.tok[slot] = st.tok[lo + i]; o.val[slot] = st.val[lo + i];
    } else {
      atomicExch(err, 1);
    }
  }
  __syncthreads();
}

struct ColShared {
  uint32_t whist[kThreads / 32][2][256];  // per-warp digit histograms (no cross-warp atomics)
  uint32_t hist[2][256];                  // their sum
  unsigned long long P[2];
  int need[2], nbits[2], done[2];
  int cand[2];                            // admissible top-K candidates per pole
  int64_t ceil[2 * kMaxB];                // reservoir key ceiling per (pole, bin) of the column
  int rtot[2 * kMaxB];                    // rows under the ceiling per (pole, bin) in the batch
  int rfound[2 * kMaxB];                  // ordered walk: rows admitted so far per (pole, bin)
  int wcnt[kThreads / 32][2 * kMaxB];     // ordered walk: per-warp counts of one chunk
  int base;
  Staged st;
};

// Reservoir slot (p * kMaxB + bin) of value s for pole p, or -1 below the pole's lowest edge.
// Unused edges are NaN, so bin never exceeds B-1.
template <int P>
__device__ __forceinline__ int res_slot(float s, const float (&e)[2][kMaxB]) {
  if (!(s >= e[P][0])) return -1;
  int bin = 0;
#pragma unroll
  for (int b = 1; b < kMaxB; ++b) bin += (s >= e[P][b]) ? 1 : 0;
  return P * kMaxB + bin;
}

// One column d of the layer (the CTA's threads together).
//  pass A (row order): admissible top-K candidates per pole (s > seed, top_key above the state's
//    K-th key) and rows under the ceiling per reservoir (pole, bin);
//  top-K: when a pole has at most K candidates they are exactly the records to merge; otherwise an
//    exact radix select (8-bit digits, MSB first) of the K-th largest composite key
//    (ordered s bits | 2^32-1-tok), i.e. the reference's top_key, finds the threshold;
//  pass B (row order): the top-K records, and every row of a reservoir bin with at most Kr rows
//    under its ceiling (all of them are admitted, whatever their key order);
//  ordered walk: bins with more than Kr such rows take their first Kr in ascending key order,
//    walking the key order a block-wide chunk at a time until every such bin is full or the keys
//    pass its ceiling (for a dense bin this ends within a few chunks).
template <int DT>
__device__ __forceinline__ void dense_column(ColShared& sh, typename Elem<DT>::T* scol, int64_t d,
                                             const typename Elem<DT>::T* __restrict__ HT,
                                             int64_t ldh, int64_t n_v, const int64_t* __restrict__ tok,
                                             const uint32_t* __restrict__ key32, const uint32_t* __restrict__ skey32,
                                             const int32_t* __restrict__ key_order,
                                             int64_t layer, int64_t D, int B, int64_t K, int64_t Kr, int reservoir,
                                             const float* __restrict__ top_seed, const int64_t* __restrict__ top_k,
                                             const int64_t* __restrict__ res_s, const int64_t* __restrict__ res_seed,
                                             const float* __restrict__ E, Lists top, Lists res, int32_t* __restrict__ err) {
  using T = typename Elem<DT>::T;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const T* col = HT + d * ldh;
  if (scol != nullptr) {  // the whole column in shared memory: every pass below reads it from there
    const int64_t nvec = (ldh * (int64_t)sizeof(T)) / 16;
    const uint4* src = reinterpret_cast<const uint4*>(col);
    uint4* dst = reinterpret_cast<uint4*>(scol);
    for (int64_t i = tid; i < nvec; i += kThreads) dst[i] = __ldcs(src + i);
    col = scol;
  }
  const int top_lim = (int)(2 * K), res_lim = kStage - (int)(2 * K);
  int64_t kth[2];
  float seed[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int64_t g = (layer * 2 + p) * D + d;
    kth[p] = top_k[g * K + (K - 1)];
    seed[p] = top_seed[g];
  }
  // reservoir edges in registers (NaN for unused bins: compares false, even against +inf); the key
  // ceilings in shared memory (admit key < ceiling)
  float e[2][kMaxB];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      e[p][b] = __int_as_float(0x7FC00000);
      if (reservoir && b < B) e[p][b] = E[((layer * 2 + p) * D + d) * B + b];
    }
  }
  if (tid < 2 * kMaxB) {
    const int p = tid / kMaxB, b = tid % kMaxB;
    int64_t c = 0;
    if (reservoir && b < B) {
      const int64_t gr = ((layer * 2 + p) * D + d) * B + b;
      int64_t th = res_s[gr * Kr + (Kr - 1)];
      const int64_t sd = res_seed[gr];
      if (sd > th) th = sd;
      c = (th == kI64Min) ? (1ll << 32) : -th;
    }
    sh.ceil[tid] = c;
    sh.rtot[tid] = 0;
    sh.rfound[tid] = 0;
  }
  if (tid < 2) {
    sh.P[tid] = 0;
    sh.need[tid] = (int)K;
    sh.nbits[tid] = 0;
    sh.cand[tid] = 0;
  }
  if (tid == 0) {
    sh.st.n = 0;
    sh.st.m = 0;
  }
  for (int i = tid; i < (kThreads / 32) * 2 * kMaxB; i += kThreads) (&sh.wcnt[0][0])[i] = 0;
  __syncthreads();
  // ------------------------------------------------------------------ pass A
  {
    int c0 = 0, c1 = 0;
    uint64_t rc[2][2] = {{0ull, 0ull}, {0ull, 0ull}};  // 16-bit counts per (pole, bin): [p][bin / 4]
    const uint64_t ku0 = (uint64_t)kth[0] ^ 0x8000000000000000ull, ku1 = (uint64_t)kth[1] ^ 0x8000000000000000ull;
    for (int64_t i = tid; i < n_v; i += kThreads) {
      const float h = Elem<DT>::f(col[i]);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float s = p ? -h : h;
        if (!(s > seed[p])) continue;
        const uint64_t ku = p ? ku1 : ku0;
        const uint32_t hi = key_hi(s);
        if (hi > (uint32_t)(ku >> 32)) {
          (p ? c1 : c0)++;
        } else if (hi == (uint32_t)(ku >> 32)) {
          const uint64_t c = ((uint64_t)hi << 32) | (uint64_t)(kM32 - (uint32_t)tok[i]);
          if (c > ku) (p ? c1 : c0)++;
        }
      }
      if (reservoir) {
        const int64_t k = (int64_t)key32[i];
        const int sa = res_slot<0>(h, e), sb = res_slot<1>(-h, e);
        if (sa >= 0 && k < sh.ceil[sa]) {
          const uint64_t inc = 1ull << (16 * (sa & 3));
          if (sa < 4) rc[0][0] += inc; else rc[0][1] += inc;
        }
        if (sb >= 0 && k < sh.ceil[sb]) {
          const uint64_t inc = 1ull << (16 * (sb & 3));
          if (sb < kMaxB + 4) rc[1][0] += inc; else rc[1][1] += inc;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      c0 += __shfl_xor_sync(0xFFFFFFFFu, c0, o);
      c1 += __shfl_xor_sync(0xFFFFFFFFu, c1, o);
    }
    if (lane == 0) {
      atomicAdd(&sh.cand[0], c0);
      atomicAdd(&sh.cand[1], c1);
    }
    if (reservoir) {
#pragma unroll
      for (int p = 0; p < 2; ++p) {
#pragma unroll
        for (int b = 0; b < kMaxB; ++b) {
          if (b >= B) break;
          int v = (int)((rc[p][b >> 2] >> (16 * (b & 3))) & 0xFFFFull);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
          if (lane == 0 && v) atomicAdd(&sh.rtot[p * kMaxB + b], v);
        }
      }
    }
  }
  __syncthreads();
  if (tid < 2) sh.done[tid] = (n_v <= K || sh.cand[tid] <= K) ? 1 : 0;
  __syncthreads();
  const bool select_all = sh.done[0] && sh.done[1];
  // ------------------------------------------------------------------ top-K radix select
  if (!select_all) {
    for (int pass = 0; pass < 8; ++pass) {
      if (sh.done[0] && sh.done[1]) break;
      if (skip_pass<DT>(pass)) {
        __syncthreads();
        if (tid < 2 && !sh.done[tid]) {
          const int nb = sh.nbits[tid];
          const unsigned long long P = sh.P[tid];
          const bool nonneg = (P >> (nb - 1)) & 1ull;  // MSB of the key = sign of s (1: s >= 0)
          sh.P[tid] = (P << 8) | (nonneg ? 0x00ull : 0xFFull);
          sh.nbits[tid] = nb + 8;
        }
        __syncthreads();
        continue;
      }
      for (int i = tid; i < (kThreads / 32) * 512; i += kThreads) (&sh.whist[0][0][0])[i] = 0;
      __syncthreads();
      const int shift = 56 - 8 * pass;
      const bool act0 = !sh.done[0], act1 = !sh.done[1];
      const unsigned long long P0 = sh.P[0], P1 = sh.P[1];
      const int nb0 = sh.nbits[0], nb1 = sh.nbits[1];
      // value digits (passes 0-3) need only the high word of the key; token ids are read only
      // for the elements still tied on the whole value (passes 4-7)
      for (int64_t i = tid; i < n_v; i += kThreads) {
        const float h = Elem<DT>::f(col[i]);
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          if (p == 0 ? !act0 : !act1) continue;
          const int nb = p == 0 ? nb0 : nb1;
          const unsigned long long P = p == 0 ? P0 : P1;
          const uint64_t hi = (uint64_t)key_hi(p ? -h : h);
          if (pass < 4) {
            if (nb == 0 || (hi >> (32 - nb)) == P) atomicAdd(&sh.whist[warp][p][(hi >> (24 - 8 * pass)) & 0xFF], 1u);
          } else if (hi == (P >> (nb - 32))) {
            const uint64_t c = (hi << 32) | (uint64_t)(kM32 - (uint32_t)tok[i]);
            if ((c >> (64 - nb)) == P) atomicAdd(&sh.whist[warp][p][(c >> shift) & 0xFF], 1u);
          }
        }
      }
      __syncthreads();
      for (int i = tid; i < 512; i += kThreads) {
        uint32_t t = 0;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) t += (&sh.whist[w][0][0])[i];
        (&sh.hist[0][0])[i] = t;
      }
      __syncthreads();
      if (warp < 2 && !sh.done[warp]) {
        const int p = warp;
        // lane l owns digits 255-8l .. 248-8l (descending); counts from the top digit down
        int c8[8], tot = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          c8[j] = (int)sh.hist[p][255 - 8 * lane - j];
          tot += c8[j];
        }
        int incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += y;
        }
        const int need = sh.need[p];
        const int excl = incl - tot;
        if (excl < need && incl >= need) {
          int cum = excl;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (cum + c8[j] >= need) {
              const int dig = 255 - 8 * lane - j;
              const int rem = need - cum;
              sh.P[p] = (sh.P[p] << 8) | (unsigned long long)dig;
              sh.nbits[p] += 8;
              sh.need[p] = rem;
              if (c8[j] == rem) sh.done[p] = 1;
              break;
            }
            cum += c8[j];
          }
        }
      }
      __syncthreads();
    }
  }
  unsigned long long thr[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int nb = sh.nbits[p];
    thr[p] = (nb >= 64 ? sh.P[p] : (nb == 0 ? 0ull : (sh.P[p] << (64 - nb))));
  }
  // reservoir bins decided by pass A: at most Kr rows under the ceiling -> all admitted here
  uint32_t direct = 0, ordered = 0;
  if (reservoir) {
#pragma unroll
    for (int c = 0; c < 2 * kMaxB; ++c) {
      const int t = sh.rtot[c];
      if (t > 0 && t <= Kr) direct |= 1u << c;
      if (t > Kr) ordered |= 1u << c;
    }
  }
  // ------------------------------------------------------------------ pass B
  for (int64_t i = tid; i < n_v; i += kThreads) {
    const float h = Elem<DT>::f(col[i]);
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float s = p ? -h : h;
      const uint32_t hi = key_hi(s);
      if (hi < (uint32_t)(thr[p] >> 32) || !(s > seed[p])) continue;  // below the K-th value
      const int64_t t = tok[i];
      const uint64_t c = ((uint64_t)hi << 32) | (uint64_t)(kM32 - (uint32_t)t);
      if (c >= thr[p]) {
        const int64_t k64 = (int64_t)(c ^ 0x8000000000000000ull);
        if (k64 > kth[p]) stage_top(sh.st, top_lim, (int32_t)((layer * 2 + p) * D + d), k64, t, s, err);
      }
    }
    if (direct) {
      const int sa = res_slot<0>(h, e), sb = res_slot<1>(-h, e);
      const bool da = sa >= 0 && ((direct >> sa) & 1u), db = sb >= 0 && ((direct >> sb) & 1u);
      if (da || db) {
        const int64_t k = (int64_t)key32[i];
        if (da && k < sh.ceil[sa])
          stage_res(sh.st, res_lim, (int32_t)(((layer * 2) * D + d) * B + sa), -k, tok[i], h, err);
        if (db && k < sh.ceil[sb])
          stage_res(sh.st, res_lim, (int32_t)(((layer * 2 + 1) * D + d) * B + (sb - kMaxB)), -k, tok[i], h, err);
      }
    }
  }
  // ------------------------------------------------------------------ ordered walk
  if (ordered) {
    const uint32_t lt = (1u << lane) - 1u;
    for (int64_t j0 = 0; j0 < n_v; j0 += kThreads) {
      // the open bins and their largest ceiling (every thread reads the same shared values)
      uint32_t open = 0;
      int64_t maxc = 0;
#pragma unroll
      for (int c = 0; c < 2 * kMaxB; ++c) {
        if (((ordered >> c) & 1u) && sh.rfound[c] < Kr) {
          open |= 1u << c;
          maxc = sh.ceil[c] > maxc ? sh.ceil[c] : maxc;
        }
      }
      if (!open || (int64_t)skey32[j0] >= maxc) break;  // keys ascend: nothing further is admissible
      const int64_t j = j0 + tid;
      int sl[2] = {-1, -1};
      int64_t k = 0;
      int32_t vi = 0;
      float h = 0.f;
      if (j < n_v) {
        k = (int64_t)skey32[j];
        if (k < maxc) {
          vi = key_order[j];
          h = Elem<DT>::f(col[vi]);
          const int sa = res_slot<0>(h, e), sb = res_slot<1>(-h, e);
          if (sa >= 0 && ((open >> sa) & 1u) && k < sh.ceil[sa]) sl[0] = sa;
          if (sb >= 0 && ((open >> sb) & 1u) && k < sh.ceil[sb]) sl[1] = sb;
        }
      }
      int rk[2];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const uint32_t peers = __match_any_sync(0xFFFFFFFFu, sl[p]);
        rk[p] = __popc(peers & lt);
        if (sl[p] >= 0 && rk[p] == 0) sh.wcnt[warp][sl[p]] = __popc(peers);
      }
      __syncthreads();
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int c = sl[p];
        if (c < 0) continue;
        int off = sh.rfound[c] + rk[p];
        for (int w = 0; w < warp; ++w) off += sh.wcnt[w][c];
        if (off < Kr) {
          const int bin = p ? c - kMaxB : c;
          stage_res(sh.st, res_lim, (int32_t)(((layer * 2 + p) * D + d) * B + bin), -k, tok[vi], h, err);
        }
      }
      __syncthreads();
      if (tid < 2 * kMaxB) {
        int t = 0;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) {
          t += sh.wcnt[w][tid];
          sh.wcnt[w][tid] = 0;
        }
        sh.rfound[tid] += t;
      }
      __syncthreads();
    }
  }
  __syncthreads();
  const int n_top = sh.st.n < top_lim ? sh.st.n : top_lim;
  const int n_res = sh.st.m < res_lim ? sh.st.m : res_lim;
  flush_range(sh.st, 0, n_top, top, err, &sh.base);
  flush_range(sh.st, kStage - n_res, n_res, res, err, &sh.base);
}

// Columns are taken grid-stride by at most one resident wave of CTAs, so an untriggered launch costs
// about a wave of early exits rather than one CTA per column.
template <int DT>
__global__ void __launch_bounds__(kThreads, 4)
dense_column_kernel(const typename Elem<DT>::T* __restrict__ HT, int64_t ldh, int64_t n_v, const int64_t* __restrict__ tok,
                    const uint32_t* __restrict__ key32, const uint32_t* __restrict__ skey32,
                    const int32_t* __restrict__ key_order, int64_t layer, int64_t D,
                    int B, int64_t K, int64_t Kr, int reservoir, const float* __restrict__ top_seed,
                    const int64_t* __restrict__ top_k, const int64_t* __restrict__ res_s,
                    const int64_t* __restrict__ res_seed, const float* __restrict__ E, const int32_t* __restrict__ count,
                    int64_t cap, int force, Lists top, Lists res, int32_t* __restrict__ err, int col_in_smem) {
  if (!triggered(count, cap, force)) return;
  extern __shared__ __align__(16) unsigned char col_raw[];
  ColShared& sh = *reinterpret_cast<ColShared*>(col_raw);
  // with col_in_smem the column (ldh elements) is staged after the shared state
  auto* scol = col_in_smem ? reinterpret_cast<typename Elem<DT>::T*>(col_raw + ((sizeof(ColShared) + 15) / 16) * 16)
                           : nullptr;
  for (int64_t d = blockIdx.x; d < D; d += gridDim.x) {
    dense_column<DT>(sh, scol, d, HT, ldh, n_v, tok, key32, skey32, key_order, layer, D, B, K, Kr, reservoir, top_seed,
                     top_k, res_s, res_seed, E, top, res, err);
    __syncthreads();  // the next column re-initialises the shared state and the staged column
  }
}

template <int DT>
int launch_dense(const void* H, int64_t D, int64_t ld, int64_t layer, const int32_t* valid_rows, int64_t n_v,
                 const int64_t* tok, const int64_t* key, const int32_t* key_order, int64_t B, int64_t K, int64_t Kr,
                 int reservoir, const float* top_seed, const int64_t* top_k, const int64_t* res_s,
                 const int64_t* res_seed, const float* E, const int32_t* count, int64_t cap, int force, Lists top,
                 Lists res, void* scratch, int32_t* err, cudaStream_t st) {
  using T = typename Elem<DT>::T;
  const int64_t n8 = (n_v + 7) / 8 * 8;
  T* HT = reinterpret_cast<T*>(scratch);
  const int64_t ntiles = (n8 + 31) / 32 * ((D + 31) / 32);
  const unsigned g1 = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ntiles, (int64_t)num_sms() * 8));
  // 32-bit keys in row order, then in key order, after the transposed copy (16-byte aligned:
  // D * n8 * esize is a multiple of 16)
  uint32_t* key32 = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(scratch) + D * n8 * (int64_t)sizeof(T));
  uint32_t* skey32 = key32 + n8;
  dense_gather_kernel<T><<<g1, dim3(32, 8), 0, st>>>(reinterpret_cast<const T*>(H), D, ld, valid_rows, n_v, n8, HT, n8,
                                                     reservoir ? key : nullptr, key_order, reservoir ? key32 : nullptr,
                                                     skey32, count, cap, force);
  if (int e = check_launch("atlas_dense_select: gather")) return e;
  // the column goes to shared memory when it fits next to the shared state (C4: ~62 KB of bf16 per
  // column, two CTAs per SM); otherwise it is read from the transposed copy in global memory
  const size_t base_smem = ((sizeof(ColShared) + 15) / 16) * 16;
  const size_t col_bytes = (size_t)n8 * sizeof(T);
  const int col_in_smem = base_smem + col_bytes <= (size_t)kDenseSmemMax ? 1 : 0;
  const size_t smem = col_in_smem ? base_smem + col_bytes : sizeof(ColShared);
  // the attribute is set once per device and instantiation (this launch runs once per layer and
  // batch, mostly to exit at once on the device, so no per-call host queries)
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cudaFuncSetAttribute(dense_column_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDenseSmemMax) !=
        cudaSuccess)
      return fail(ATLAS_ERR_CUDA, "dense_select: cannot reserve %zu bytes of shared memory", smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  // resident CTAs per SM: registers allow four (at most 64 x 256 per CTA); shared memory as many as
  // fit in the SM's 228 KB (1 KB of it reserved per CTA)
  int per_sm = (int)(((size_t)228 * 1024) / (smem + 1024));
  per_sm = per_sm < 1 ? 1 : (per_sm > 4 ? 4 : per_sm);
  const unsigned g2 = (unsigned)std::max<int64_t>(1, std::min<int64_t>(D, (int64_t)num_sms() * per_sm));
  dense_column_kernel<DT><<<g2, kThreads, smem, st>>>(HT, n8, n_v, tok, key32, skey32, key_order, layer, D, (int)B, K, Kr,
                                                                reservoir, top_seed, top_k, res_s, res_seed, E, count,
                                                                cap, force, top, res, err, col_in_smem);
  return check_launch("atlas_dense_select: column");
}

int esize(int dtype) { return dtype == ATLAS_F32 ? 4 : 2; }

}  // namespace
}  // namespace atlas

using namespace atlas;

extern "C" int64_t atlas_dense_scratch_bytes(int64_t n_v, int64_t D, int64_t B, int dtype) {
  (void)B;
  const int64_t n8 = (n_v + 7) / 8 * 8;
  return D * n8 * esize(dtype) + n8 * 8 + 256;  // transposed valid rows, 32-bit keys in row and key order
}

extern "C" int atlas_dense_select(const void* H, int dtype, int64_t T, int64_t D, int64_t ld, int64_t layer,
                                  const int32_t* valid_rows, int64_t n_v, const int64_t* tok, const int64_t* key,
                                  const int32_t* key_order, int64_t B, int64_t K, int64_t Kr, int reservoir,
                                  const float* top_seed, const int64_t* top_k, const int64_t* res_s,
                                  const int64_t* res_seed, const float* E, const int32_t* count, int64_t cap, int force,
                                  int32_t* top_g, int64_t* top_sc, int64_t* top_tok, float* top_val, int32_t* n_top,
                                  int64_t top_cap, int32_t* res_g, int64_t* res_sc, int64_t* res_tok, float* res_val,
                                  int32_t* n_res, int64_t res_cap, void* scratch, int64_t scratch_bytes, int32_t* flag,
                                  int32_t* err, void* stream) {
  ATLAS_REQUIRE(T >= 0 && D > 0 && ld >= D && n_v >= 0 && n_v <= T && layer >= 0, "dense_select: bad shape");
  ATLAS_REQUIRE(B >= 1 && B <= kMaxB && K >= 1 && Kr >= 1 && K <= 256 && Kr <= 256, "dense_select: B must be 1..%d",
                kMaxB);
  ATLAS_REQUIRE(2 * K + 2 * B * Kr <= kStage, "dense_select: K/Kr too large for the staging area");
  ATLAS_REQUIRE((layer * 2 + 2) * D * B < (1LL << 31) && n_v < (1LL << 31), "dense_select: ids exceed int32");
  ATLAS_REQUIRE(n_v <= (int64_t)kThreads * 65535, "dense_select: more than %d valid rows", kThreads * 65535);
  (void)flag;
  if (n_v == 0) return ATLAS_OK;
  ATLAS_REQUIRE(force || count, "dense_select: count required unless forced");
  ATLAS_REQUIRE(H && valid_rows && tok && top_seed && top_k && top_g && top_sc && top_tok && top_val && n_top && err &&
                    scratch,
                "dense_select: null pointer");
  ATLAS_REQUIRE(scratch_bytes >= atlas_dense_scratch_bytes(n_v, D, B, dtype), "dense_select: scratch too small");
  if (reservoir)
    ATLAS_REQUIRE(key && key_order && res_s && res_seed && E && res_g && res_sc && res_tok && res_val && n_res,
                  "dense_select: null reservoir pointer");
  Lists top{top_g, top_sc, top_tok, top_val, n_top, top_cap};
  Lists res{res_g, res_sc, res_tok, res_val, n_res, res_cap};
  const int32_t* cnt = count ? count : n_top;  // never read when forced
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case ATLAS_BF16:
      return launch_dense<ATLAS_BF16>(H, D, ld, layer, valid_rows, n_v, tok, key, key_order, B, K, Kr, reservoir, top_seed,
                                      top_k, res_s, res_seed, E, cnt, cap, force, top, res, scratch, err, st);
    case ATLAS_F16:
      return launch_dense<ATLAS_F16>(H, D, ld, layer, valid_rows, n_v, tok, key, key_order, B, K, Kr, reservoir, top_seed,
                                     top_k, res_s, res_seed, E, cnt, cap, force, top, res, scratch, err, st);
    case ATLAS_F32:
      return launch_dense<ATLAS_F32>(H, D, ld, layer, valid_rows, n_v, tok, key, key_order, B, K, Kr, reservoir, top_seed,
                                     top_k, res_s, res_seed, E, cnt, cap, force, top, res, scratch, err, st);
    default:
      return fail(ATLAS_ERR_ARG, "dense_select: unknown dtype %d", dtype);
  }
}
