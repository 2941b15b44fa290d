// Dense burst path (Atlas._dense, atlas/core.py:407-446) on the live hook output, predicated on the
// device: it runs when the layer is a dense layer (force) or when its compaction buffer overflowed
// (*count > cap, the 0.5%-fill trigger), so the forward is never re-run and the host never syncs.
//
// 1. dense_gather: the valid rows are transposed into a column-major scratch HT [D, n_v] (coalesced
//    reads and writes through shared-memory tiles), so every column below is one contiguous run.
// 2. dense_column: one CTA per column, both poles.
//    top-K: exact radix select (8-bit digits, MSB first, block-wide shared-memory histograms) of the
//      K-th largest composite key (ordered s bits | 2^32-1-tok), i.e. the reference's top_key;
//      digits that are constant for bf16/fp16 inputs are skipped, and token ids are read only for
//      elements tied on the whole value. Exactly min(K, n_v) batch elements reach the threshold; the
//      state admission tests (s > seed, key > K-th state key) then apply.
//    reservoir: the rows in ascending hash-key order (key_order; their keys gathered once per launch
//      into a sorted array) are split into one run per thread;
//      each thread counts the admissible rows of its run per (pole, bin) (bin match and key under
//      the bin's ceiling), a block scan turns the counts into global ranks, and the first Kr
//      admissible rows of each bin are emitted. Runs that start above every ceiling stop at once.
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
template <typename T>
__global__ void dense_gather_kernel(const T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ rows,
                                    int64_t n, int64_t n8, T* __restrict__ HT, int64_t ldh,
                                    const int32_t* __restrict__ count, int64_t cap, int force) {
  if (!triggered(count, cap, force)) return;
  __shared__ T tile[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;
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

// Keys in key order (skey[j] = key[key_order[j]]), once per triggered launch: the reservoir walk of
// every column then reads them sequentially instead of one random 8-byte load per row and column.
__global__ void dense_sorted_keys_kernel(const int64_t* __restrict__ key, const int32_t* __restrict__ key_order,
                                         int64_t n_v, int64_t* __restrict__ skey, const int32_t* __restrict__ count,
                                         int64_t cap, int force) {
  if (!triggered(count, cap, force)) return;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n_v; j += (int64_t)gridDim.x * blockDim.x)
    skey[j] = key[key_order[j]];
}

// ---------------------------------------------------------------------------------------- column
struct Staged {
  int32_t g[kStage];
  int64_t sc[kStage], tok[kStage];
  float val[kStage];
  int n;
};

__device__ __forceinline__ void stage(Staged& st, int32_t g, int64_t sc, int64_t tok, float val, int32_t* err) {
  const int i = atomicAdd(&st.n, 1);
  if (i < kStage) {
    st.g[i] = g; st.sc[i] = sc; st.tok[i] = tok; st.val[i] = val;
  } else {
    atomicExch(err, 1);
  }
}

__device__ void flush(Staged& st, const Lists& o, int32_t* err, int* s_base) {
  __syncthreads();
  const int n = st.n < kStage ? st.n : kStage;
  if (threadIdx.x == 0) *s_base = n > 0 ? atomicAdd(o.n, n) : 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t slot = (int64_t)*s_base + i;
    if (slot < o.cap) {
      o.g[slot] = st.g[i]; o.sc[slot] = st.sc[i]; o.tok[slot] = st.tok[i]; o.val[slot] = st.val[i];
    } else {
      atomicExch(err, 1);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) st.n = 0;
  __syncthreads();
}

struct ColShared {
  uint32_t whist[kThreads / 32][2][256];  // per-warp digit histograms (no cross-warp atomics)
  uint32_t hist[2][256];                  // their sum
  unsigned long long P[2];
  int need[2], nbits[2], done[2];
  int cand[2];                            // admissible top-K candidates per pole
  int scan[kThreads / 32][2 * kMaxB];
  int64_t ceil[2 * kMaxB];                // reservoir key ceiling per (pole, bin) of the column
  uint16_t rcnt[2 * kMaxB][kThreads];     // per thread and (pole, bin): count, then start rank
  int base;
  Staged st;
};

// One column d of the layer (the CTA's threads together): top-K radix select and reservoir runs.
template <int DT>
__device__ __forceinline__ void dense_column(ColShared& sh, typename Elem<DT>::T* scol, int64_t d,
                                             const typename Elem<DT>::T* __restrict__ HT,
                                             int64_t ldh, int64_t n_v, const int64_t* __restrict__ tok,
                                             const int64_t* __restrict__ skey, const int32_t* __restrict__ key_order,
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
  int64_t kth[2];
  float seed[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int64_t g = (layer * 2 + p) * D + d;
    kth[p] = top_k[g * K + (K - 1)];
    seed[p] = top_seed[g];
  }
  if (tid < 2) {
    sh.P[tid] = 0;
    sh.need[tid] = (int)K;
    sh.nbits[tid] = 0;
    sh.cand[tid] = 0;
  }
  if (tid == 0) sh.st.n = 0;
  __syncthreads();
  // Admissible top-K candidates of the batch: s > seed and top_key(s, tok) above the state's K-th
  // key (only those can enter the state). When a pole has at most K of them they are exactly the
  // records to merge, and its radix select is skipped (the common case once the state is full).
  {
    int c0 = 0, c1 = 0;
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
        if (k64 > kth[p]) stage(sh.st, (int32_t)((layer * 2 + p) * D + d), k64, t, s, err);
      }
    }
  }
  flush(sh.st, top, err, &sh.base);
  if (!reservoir) return;
  // ------------------------------------------------------------------ reservoir bottom-Kr
  // Bin edges in registers; each (pole, bin) slot c = p*kMaxB + b has its key ceiling in shared
  // memory, and each thread its count (then its start rank) per slot in shared memory, so a row
  // costs one shared load / store for its own slot instead of a compare-and-select over all slots.
  // A row belongs to at most the pole whose lowest edge it reaches (both only on a tie with it).
  float e[2][kMaxB];
  int64_t maxceil = 0;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      e[p][b] = __int_as_float(0x7FC00000);  // NaN: an unused edge compares false, even for +inf
      int64_t c = 0;
      if (b < B) {
        const int64_t gr = ((layer * 2 + p) * D + d) * B + b;
        e[p][b] = E[gr];
        int64_t th = res_s[gr * Kr + (Kr - 1)];
        const int64_t sd = res_seed[gr];
        if (sd > th) th = sd;
        c = (th == kI64Min) ? (1ll << 32) : -th;  // admit key < ceil
        if (c > maxceil) maxceil = c;
      }
      if (tid == 0) sh.ceil[p * kMaxB + b] = c;
    }
  }
  for (int c = 0; c < 2 * kMaxB; ++c) sh.rcnt[c][tid] = 0;
  __syncthreads();
  const int64_t run = (n_v + kThreads - 1) / kThreads;
  const int64_t j0 = tid * run;
  const int64_t j1 = j0 + run < n_v ? j0 + run : n_v;
  for (int64_t j = j0; j < j1; ++j) {
    const int64_t k = skey[j];
    if (k >= maxceil) break;
    const float h = Elem<DT>::f(col[key_order[j]]);
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float s = p ? -h : h;
      if (!(s >= e[p][0])) continue;
      int bin = 0;
#pragma unroll
      for (int b = 1; b < kMaxB; ++b) bin += (s >= e[p][b]) ? 1 : 0;
      const int c = p * kMaxB + bin;
      if (k < sh.ceil[c]) {
        const int n = sh.rcnt[c][tid];
        if (n < Kr) sh.rcnt[c][tid] = (uint16_t)(n + 1);
      }
    }
  }
  // block exclusive scan of the per-thread counts, for every (pole, bin); the start ranks replace
  // the counts in place
  bool open = false;
#pragma unroll
  for (int c = 0; c < 2 * kMaxB; ++c) {
    const int v = sh.rcnt[c][tid];
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) sh.scan[warp][c] = incl;
    sh.rcnt[c][tid] = (uint16_t)(incl - v);  // within-warp start, completed below
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < 2 * kMaxB; ++c) {
    int st = sh.rcnt[c][tid];
    for (int w = 0; w < warp; ++w) st += sh.scan[w][c];
    const int b = c % kMaxB;
    open |= (b < B && st < Kr);
    sh.rcnt[c][tid] = (uint16_t)(st < 65535 ? st : 65535);
  }
  if (open) {
    for (int64_t j = j0; j < j1; ++j) {
      const int64_t k = skey[j];
      if (k >= maxceil) break;
      const int32_t vi = key_order[j];
      const float h = Elem<DT>::f(col[vi]);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float s = p ? -h : h;
        if (!(s >= e[p][0])) continue;
        int bin = 0;
#pragma unroll
        for (int b = 1; b < kMaxB; ++b) bin += (s >= e[p][b]) ? 1 : 0;
        const int c = p * kMaxB + bin;
        if (k < sh.ceil[c]) {
          const int st = sh.rcnt[c][tid];
          if (st < Kr) {
            stage(sh.st, (int32_t)(((layer * 2 + p) * D + d) * B + bin), -k, tok[vi], h, err);
            sh.rcnt[c][tid] = (uint16_t)(st + 1);
          }
        }
      }
    }
  }
  flush(sh.st, res, err, &sh.base);
}

// Columns are taken grid-stride by at most one resident wave of CTAs, so an untriggered launch costs
// about a wave of early exits rather than one CTA per column.
template <int DT>
__global__ void __launch_bounds__(kThreads, 4)
dense_column_kernel(const typename Elem<DT>::T* __restrict__ HT, int64_t ldh, int64_t n_v, const int64_t* __restrict__ tok,
                    const int64_t* __restrict__ skey, const int32_t* __restrict__ key_order, int64_t layer, int64_t D,
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
    dense_column<DT>(sh, scol, d, HT, ldh, n_v, tok, skey, key_order, layer, D, B, K, Kr, reservoir, top_seed, top_k,
                     res_s, res_seed, E, top, res, err);
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
  dense_gather_kernel<T><<<g1, dim3(32, 8), 0, st>>>(reinterpret_cast<const T*>(H), D, ld, valid_rows, n_v, n8, HT, n8,
                                                     count, cap, force);
  if (int e = check_launch("atlas_dense_select: gather")) return e;
  // sorted keys after the transposed copy (16-byte aligned: D * n8 * esize is a multiple of 16)
  int64_t* skey = reinterpret_cast<int64_t*>(reinterpret_cast<uint8_t*>(scratch) + D * n8 * (int64_t)sizeof(T));
  if (reservoir) {
    dense_sorted_keys_kernel<<<grid_for(n_v, 256, 2), 256, 0, st>>>(key, key_order, n_v, skey, count, cap, force);
    if (int e = check_launch("atlas_dense_select: sorted keys")) return e;
  }
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
  dense_column_kernel<DT><<<g2, kThreads, smem, st>>>(HT, n8, n_v, tok, skey, key_order, layer, D, (int)B, K, Kr,
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
  return D * n8 * esize(dtype) + n8 * 8 + 256;  // transposed valid rows, then the keys in key order
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
