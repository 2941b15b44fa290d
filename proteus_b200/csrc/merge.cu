// Exact grouped top-K merge (grouped_merge, atlas/core.py:75-104) and row-wise state merge
// (the top-K / reservoir part of Atlas.merge_from, core.py:636-643).
//
// Pipeline for a batch of candidate records (group g, score, tok, val):
//   count   : per-group candidate counts (atomics on a [G] int32 array)
//   scan    : exclusive scan -> segment offsets, a cursor per group, the list of touched groups
//   scatter : records -> group-contiguous segments
//   merge   : one warp per touched group. The group's state row (K scores, sorted descending) sits in
//             shared memory; candidates arrive in chunks of 32 that are bitonic-sorted across the
//             warp, and each chunk is merged by rank (state entry i -> i + #chunk > s_i; chunk entry
//             j -> j + #state >= c_j), so no comparison sort over K is ever needed. Only slots whose
//             content changed are written back.
#include "common.cuh"

namespace atlas {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;  // 2048 groups per scan block
// warps per merge block: the per-warp shared state is 12*KMAX + 256 bytes (static limit 48 KB)
template <int KMAX> struct MergeWarps { static constexpr int value = KMAX > 128 ? 4 : 8; };

int64_t n_scan_blocks(int64_t G) { return (G + kScanTile - 1) / kScanTile; }

// Workspace ints: cnt[G] off[G] cursor[G] touched[G] | bsum[nb] boff[nb] | touched_n (+pad)
struct MergeWs {
  int32_t *cnt, *off, *cursor, *touched, *bsum, *boff, *touched_n;
};

MergeWs carve(int32_t* ws, int64_t G) {
  const int64_t nb = n_scan_blocks(G);
  MergeWs w;
  w.cnt = ws;
  w.off = ws + G;
  w.cursor = ws + 2 * G;
  w.touched = ws + 3 * G;
  w.bsum = ws + 4 * G;
  w.boff = w.bsum + nb;
  w.touched_n = w.boff + nb;
  return w;
}

__global__ void count_kernel(const int32_t* __restrict__ g, const int32_t* __restrict__ n_dev, int64_t n_max,
                             int64_t G, int32_t* __restrict__ cnt) {
  int64_t n = *n_dev;
  if (n > n_max) n = n_max;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t gi = g[i];
    if (gi >= 0 && gi < G) atomicAdd(cnt + gi, 1);
  }
}

__device__ __forceinline__ int block_excl_scan(int v, int* total) {
  __shared__ int wsum[kScanThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int wt;
  const int pre = warp_excl_scan(v, lane, &wt);
  if (lane == 0) wsum[warp] = wt;
  __syncthreads();
  int woff = 0, tot = 0;
  for (int w = 0; w < kScanThreads / 32; ++w) {
    if (w < warp) woff += wsum[w];
    tot += wsum[w];
  }
  __syncthreads();
  *total = tot;
  return woff + pre;
}

__global__ void __launch_bounds__(kScanThreads) scan_sum_kernel(const int32_t* __restrict__ cnt, int64_t G,
                                                                 int32_t* __restrict__ bsum) {
  const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  int s = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k)
    if (base + k < G) s += cnt[base + k];
  int tot;
  block_excl_scan(s, &tot);
  if (threadIdx.x == 0) bsum[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(kScanThreads) scan_blocks_kernel(const int32_t* __restrict__ bsum, int64_t nb,
                                                                    int32_t* __restrict__ boff, int32_t* __restrict__ touched_n) {
  int carry = 0;
  for (int64_t b0 = 0; b0 < nb; b0 += kScanThreads) {
    const int64_t b = b0 + threadIdx.x;
    const int v = b < nb ? bsum[b] : 0;
    int tot;
    const int pre = block_excl_scan(v, &tot);
    if (b < nb) boff[b] = carry + pre;
    carry += tot;
  }
  if (threadIdx.x == 0) *touched_n = 0;
}

__global__ void __launch_bounds__(kScanThreads) scan_final_kernel(const int32_t* __restrict__ cnt, int64_t G,
                                                                   const int32_t* __restrict__ boff,
                                                                   int32_t* __restrict__ off, int32_t* __restrict__ cursor,
                                                                   int32_t* __restrict__ touched,
                                                                   int32_t* __restrict__ touched_n) {
  const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  int v[kScanItems];
  int s = 0, nz = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    v[k] = base + k < G ? cnt[base + k] : 0;
    s += v[k];
    nz += v[k] > 0 ? 1 : 0;
  }
  int tot;
  int pre = block_excl_scan(s, &tot) + boff[blockIdx.x];
  int tpre = block_excl_scan(nz, &tot);
  __shared__ int tbase;
  if (threadIdx.x == 0) tbase = tot > 0 ? atomicAdd(touched_n, tot) : 0;
  __syncthreads();
  tpre += tbase;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    if (base + k < G) {
      off[base + k] = pre;
      cursor[base + k] = pre;
      if (v[k] > 0) touched[tpre++] = (int32_t)(base + k);
      pre += v[k];
    }
  }
}

__global__ void scatter_kernel(const int32_t* __restrict__ g, const int64_t* __restrict__ sc, const int64_t* __restrict__ tok,
                               const float* __restrict__ val, const int32_t* __restrict__ n_dev, int64_t n_max,
                               int64_t G, int32_t* __restrict__ cursor, int64_t* __restrict__ gsc,
                               int64_t* __restrict__ gtok, float* __restrict__ gval) {
  int64_t n = *n_dev;
  if (n > n_max) n = n_max;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t gi = g[i];
    if (gi < 0 || gi >= G) continue;
    const int pos = atomicAdd(cursor + gi, 1);
    gsc[pos] = sc[i];
    gtok[pos] = tok[i];
    gval[pos] = val[i];
  }
}

// ------------------------------------------------------------------ warp merge of one group
template <int KMAX>
struct WarpSmem {
  int64_t sc[2][KMAX];
  int32_t src[2][KMAX];  // >= 0: original state slot; < 0: candidate -(j+1)
  int64_t csc[32];
};

__device__ __forceinline__ void bitonic_desc(int64_t& cs, int& ci, int lane) {
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int64_t o = __shfl_xor_sync(0xFFFFFFFFu, cs, j);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, ci, j);
      const bool desc_block = (lane & k) == 0;
      const bool lower = (lane & j) == 0;
      const bool take_max = (lower == desc_block);
      const bool swap = take_max ? (o > cs) : (o < cs);
      if (swap) {
        cs = o;
        ci = oi;
      }
    }
  }
}

// Merge m candidates (scores via cand_sc(j), payloads via cand_tok / cand_val(j)) into the state row
// (st_sc, st_tok, st_val) of length K. Whole warp participates.
template <int KMAX, class FS, class FT, class FV>
__device__ void warp_merge(int64_t* __restrict__ st_sc, int64_t* __restrict__ st_tok, float* __restrict__ st_val, int K,
                           int m, FS cand_sc, FT cand_tok, FV cand_val, WarpSmem<KMAX>& sm, int lane) {
  for (int i = lane; i < K; i += 32) {
    sm.sc[0][i] = st_sc[i];
    sm.src[0][i] = i;
  }
  __syncwarp();
  int cur = 0;
  bool changed = false;
  for (int c0 = 0; c0 < m; c0 += 32) {
    const int j = c0 + lane;
    const int64_t kth = sm.sc[cur][K - 1];
    int64_t cs = kI64Min;
    int ci = -1;
    if (j < m) {
      const int64_t s = cand_sc(j);
      if (s > kth) {
        cs = s;
        ci = j;
      }
    }
    if (!__any_sync(0xFFFFFFFFu, ci >= 0)) continue;
    changed = true;
    bitonic_desc(cs, ci, lane);
    const int nv = __popc(__ballot_sync(0xFFFFFFFFu, ci >= 0));  // valid entries are lanes [0, nv)
    sm.csc[lane] = cs;
    __syncwarp();
    const int nxt = cur ^ 1;
    for (int i = lane; i < K; i += 32) {
      const int64_t s = sm.sc[cur][i];
      int lo = 0, hi = nv;  // #chunk > s
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (sm.csc[mid] > s) lo = mid + 1; else hi = mid;
      }
      const int r = i + lo;
      if (r < K) {
        sm.sc[nxt][r] = s;
        sm.src[nxt][r] = sm.src[cur][i];
      }
    }
    if (lane < nv) {
      int lo = 0, hi = K;  // #state >= cs
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (sm.sc[cur][mid] >= cs) lo = mid + 1; else hi = mid;
      }
      const int r = lane + lo;
      if (r < K) {
        sm.sc[nxt][r] = cs;
        sm.src[nxt][r] = -(ci + 1);
      }
    }
    __syncwarp();
    cur = nxt;
  }
  if (!changed) return;
  constexpr int PER = KMAX / 32;
  int64_t osc[PER], otok[PER];
  float oval[PER];
  bool w[PER];
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    const int r = lane + 32 * t;
    w[t] = false;
    if (r < K) {
      const int src = sm.src[cur][r];
      if (src != r) {
        w[t] = true;
        osc[t] = sm.sc[cur][r];
        if (src >= 0) {
          otok[t] = st_tok[src];
          oval[t] = st_val[src];
        } else {
          otok[t] = cand_tok(-src - 1);
          oval[t] = cand_val(-src - 1);
        }
      }
    }
  }
  __syncwarp();
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    if (w[t]) {
      const int r = lane + 32 * t;
      st_sc[r] = osc[t];
      st_tok[r] = otok[t];
      st_val[r] = oval[t];
    }
  }
  __syncwarp();
}

template <int KMAX, int kMergeWarps = MergeWarps<KMAX>::value>
__global__ void __launch_bounds__(kMergeWarps * 32)
merge_groups_kernel(int64_t* __restrict__ state_sc, int64_t* __restrict__ state_tok, float* __restrict__ state_val, int K,
                    const int32_t* __restrict__ touched, const int32_t* __restrict__ touched_n,
                    const int32_t* __restrict__ off, const int32_t* __restrict__ cnt, const int64_t* __restrict__ gsc,
                    const int64_t* __restrict__ gtok, const float* __restrict__ gval) {
  __shared__ WarpSmem<KMAX> smem[kMergeWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nt = *touched_n;
  for (int w = blockIdx.x * kMergeWarps + warp; w < nt; w += gridDim.x * kMergeWarps) {
    const int64_t g = touched[w];
    const int o = off[g], m = cnt[g];
    warp_merge<KMAX>(state_sc + g * K, state_tok + g * K, state_val + g * K, K, m,
                     [&](int j) { return gsc[o + j]; }, [&](int j) { return gtok[o + j]; },
                     [&](int j) { return gval[o + j]; }, smem[warp], lane);
  }
}

template <int KMAX, int kMergeWarps = MergeWarps<KMAX>::value>
__global__ void __launch_bounds__(kMergeWarps * 32)
merge_rows_kernel(int64_t* __restrict__ sc, int64_t* __restrict__ tok, float* __restrict__ val,
                  const int64_t* __restrict__ osc, const int64_t* __restrict__ otok, const float* __restrict__ oval,
                  int64_t G, int K) {
  __shared__ WarpSmem<KMAX> smem[kMergeWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t g = (int64_t)blockIdx.x * kMergeWarps + warp; g < G; g += (int64_t)gridDim.x * kMergeWarps) {
    const int64_t* s = osc + g * K;
    const int64_t* t = otok + g * K;
    const float* v = oval + g * K;
    warp_merge<KMAX>(sc + g * K, tok + g * K, val + g * K, K, K, [&](int j) { return s[j]; },
                     [&](int j) { return t[j]; }, [&](int j) { return v[j]; }, smem[warp], lane);
  }
}

template <int KMAX>
int launch_merge(int64_t* ssc, int64_t* stok, float* sval, int64_t K, const MergeWs& w, const int64_t* gsc,
                 const int64_t* gtok, const float* gval, cudaStream_t st) {
  constexpr int kMergeWarps = MergeWarps<KMAX>::value;
  const unsigned blocks = (unsigned)num_sms() * 4;
  merge_groups_kernel<KMAX><<<blocks, kMergeWarps * 32, 0, st>>>(ssc, stok, sval, (int)K, w.touched, w.touched_n, w.off,
                                                                 w.cnt, gsc, gtok, gval);
  return check_launch("atlas_grouped_merge: merge");
}

template <int KMAX>
int launch_rows(int64_t* sc, int64_t* tok, float* val, const int64_t* osc, const int64_t* otok, const float* oval,
                int64_t G, int64_t K, cudaStream_t st) {
  constexpr int kMergeWarps = MergeWarps<KMAX>::value;
  int64_t blocks = (G + kMergeWarps - 1) / kMergeWarps;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  merge_rows_kernel<KMAX><<<(unsigned)blocks, kMergeWarps * 32, 0, st>>>(sc, tok, val, osc, otok, oval, G, (int)K);
  return check_launch("atlas_merge_rows");
}

int64_t bytes_align(int64_t b) { return (b + 255) / 256 * 256; }

}  // namespace
}  // namespace atlas

using namespace atlas;

extern "C" int64_t atlas_merge_ws_i32(int64_t G, int64_t n_max) {
  (void)n_max;
  return 4 * G + 2 * n_scan_blocks(G) + 64;
}

extern "C" int64_t atlas_merge_ws_bytes(int64_t n_max) { return 3 * bytes_align(8 * (n_max > 0 ? n_max : 1)); }

extern "C" int atlas_grouped_merge(int64_t* state_sc, int64_t* state_tok, float* state_val, int64_t G, int64_t K,
                                   const int32_t* g, const int64_t* sc, const int64_t* tok, const float* val,
                                   const int32_t* n_dev, int64_t n_max, int32_t* ws_i32, void* ws_bytes, void* stream) {
  ATLAS_REQUIRE(G >= 0 && K >= 1 && K <= 256, "grouped_merge: K must be 1..256 (got %lld)", (long long)K);
  ATLAS_REQUIRE(G < (1LL << 31) && n_max >= 0 && n_max < (1LL << 31), "grouped_merge: sizes exceed int32");
  if (G == 0 || n_max == 0) return ATLAS_OK;
  ATLAS_REQUIRE(state_sc && state_tok && state_val && g && sc && tok && val && n_dev && ws_i32 && ws_bytes,
                "grouped_merge: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  MergeWs w = carve(ws_i32, G);
  const int64_t nb = n_scan_blocks(G);
  char* wb = (char*)ws_bytes;
  const int64_t seg = bytes_align(8 * n_max);
  int64_t* gsc = (int64_t*)wb;
  int64_t* gtok = (int64_t*)(wb + seg);
  float* gval = (float*)(wb + 2 * seg);
  if (cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * G, st) != cudaSuccess)
    return fail(ATLAS_ERR_CUDA, "grouped_merge: memset failed");
  count_kernel<<<grid_for(n_max, 256), 256, 0, st>>>(g, n_dev, n_max, G, w.cnt);
  if (int e = check_launch("atlas_grouped_merge: count")) return e;
  scan_sum_kernel<<<(unsigned)nb, kScanThreads, 0, st>>>(w.cnt, G, w.bsum);
  scan_blocks_kernel<<<1, kScanThreads, 0, st>>>(w.bsum, nb, w.boff, w.touched_n);
  scan_final_kernel<<<(unsigned)nb, kScanThreads, 0, st>>>(w.cnt, G, w.boff, w.off, w.cursor, w.touched, w.touched_n);
  if (int e = check_launch("atlas_grouped_merge: scan")) return e;
  scatter_kernel<<<grid_for(n_max, 256), 256, 0, st>>>(g, sc, tok, val, n_dev, n_max, G, w.cursor, gsc, gtok, gval);
  if (int e = check_launch("atlas_grouped_merge: scatter")) return e;
  if (K <= 32) return launch_merge<32>(state_sc, state_tok, state_val, K, w, gsc, gtok, gval, st);
  if (K <= 64) return launch_merge<64>(state_sc, state_tok, state_val, K, w, gsc, gtok, gval, st);
  if (K <= 128) return launch_merge<128>(state_sc, state_tok, state_val, K, w, gsc, gtok, gval, st);
  return launch_merge<256>(state_sc, state_tok, state_val, K, w, gsc, gtok, gval, st);
}

extern "C" int atlas_merge_rows(int64_t* sc, int64_t* tok, float* val, const int64_t* other_sc, const int64_t* other_tok,
                                const float* other_val, int64_t G, int64_t K, void* stream) {
  ATLAS_REQUIRE(G >= 0 && K >= 1 && K <= 256, "merge_rows: K must be 1..256");
  if (G == 0) return ATLAS_OK;
  ATLAS_REQUIRE(sc && tok && val && other_sc && other_tok && other_val, "merge_rows: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (K <= 32) return launch_rows<32>(sc, tok, val, other_sc, other_tok, other_val, G, K, st);
  if (K <= 64) return launch_rows<64>(sc, tok, val, other_sc, other_tok, other_val, G, K, st);
  if (K <= 128) return launch_rows<128>(sc, tok, val, other_sc, other_tok, other_val, G, K, st);
  return launch_rows<256>(sc, tok, val, other_sc, other_tok, other_val, G, K, st);
}

// ------------------------------------------------------------------------------------------------
// Allocation-free variant of atlas_grouped_merge. Its workspace is this file-scope device array
// (every GPU that loads the library holds it until the process exits), sized for at most
// kStaticMergeGroups groups and kStaticMergeRecords candidate records per call.
namespace atlas {
namespace {
constexpr int64_t kStaticMergeGroups = 1 << 18;
constexpr int64_t kStaticMergeRecords = 1 << 18;
constexpr int64_t kStaticI32 = 4 * kStaticMergeGroups + 2 * ((kStaticMergeGroups + 2047) / 2048) + 64;
constexpr int64_t kStaticI32Bytes = (kStaticI32 * 4 + 255) / 256 * 256;
constexpr int64_t kStaticRecBytes = 3 * ((8 * kStaticMergeRecords + 255) / 256 * 256);
static __device__ __align__(256) unsigned char g_merge_scratch[kStaticI32Bytes + kStaticRecBytes];

// Device address of g_merge_scratch on the current device, looked up on every call (a cheap lookup).
// It is not cached: after a cudaDeviceReset the module is loaded again and the array can move, so a
// cached address could point at freed memory. Host code only holds a stand-in for the symbol, which
// must never be handed to a kernel. Under lazy module loading (the CUDA default) the first lookup on
// a device is what loads this module there and creates the array.
int static_scratch(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_merge_scratch);
  if (e != cudaSuccess || !p)
    return fail(ATLAS_ERR_CUDA, "grouped_merge_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
  *out = p;
  return ATLAS_OK;
}
}  // namespace
}  // namespace atlas

extern "C" int atlas_grouped_merge_static(int64_t* state_sc, int64_t* state_tok, float* state_val, int64_t G, int64_t K,
                                          const int32_t* g, const int64_t* sc, const int64_t* tok, const float* val,
                                          const int32_t* n_dev, int64_t n_max, void* stream) {
  ATLAS_REQUIRE(G >= 0 && G <= kStaticMergeGroups, "grouped_merge_static: G = %lld exceeds the static workspace limit "
                "of %lld groups (use atlas_grouped_merge with a caller workspace)", (long long)G,
                (long long)kStaticMergeGroups);
  ATLAS_REQUIRE(n_max >= 0 && n_max <= kStaticMergeRecords, "grouped_merge_static: n_max = %lld exceeds the static "
                "workspace limit of %lld records (use atlas_grouped_merge with a caller workspace)", (long long)n_max,
                (long long)kStaticMergeRecords);
  if (G == 0 || n_max == 0) return ATLAS_OK;
  void* base = nullptr;
  if (int e = static_scratch(&base)) return e;
  int32_t* ws_i32 = reinterpret_cast<int32_t*>(base);
  void* ws_bytes = reinterpret_cast<unsigned char*>(base) + kStaticI32Bytes;
  // the pipeline clears its per-group counters itself and rebuilds every other workspace field, so
  // whatever the previous call left in the array does not leak into this one
  return atlas_grouped_merge(state_sc, state_tok, state_val, G, K, g, sc, tok, val, n_dev, n_max, ws_i32, ws_bytes,
                             stream);
}
