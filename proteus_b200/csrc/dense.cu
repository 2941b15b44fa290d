// Dense burst path (Atlas._dense, atlas/core.py:407-446) on the live hook output, predicated on the
// device: it runs when the layer is a dense layer (force) or when the compaction buffer overflowed
// (*count > cap, the 0.5%-fill trigger), so the forward is never re-run and the host never syncs.
//
// top-K: per (column, pole) an exact radix select (8-bit digits, MSB first) of the K-th largest
//   composite key (ordered s bits | 2^32-1-tok), i.e. the reference's top_key; digits that are
//   constant for bf16/fp16 inputs are skipped. Every batch element whose key reaches the K-th is a
//   candidate (exactly min(K, n_v) per column and pole), then the state admission tests apply.
// reservoir: rows are visited in ascending hash-key order (key_order), split in chunks of 512; a
//   count pass records, per chunk, column, pole and bin, how many admissible rows (bin match and
//   key under the bin's ceiling) it holds (saturating at Kr); the emit pass turns the chunk prefix
//   into global ranks and emits the first Kr admissible rows of each bin. Both passes stop as soon
//   as the key passes every ceiling of the warp's columns.
#include "common.cuh"

namespace atlas {
namespace {

constexpr int kTopWarps = 16;
constexpr int kResWarps = 4;
constexpr int kChunk = 512;
constexpr int kMaxB = 8;

struct Lists {
  int32_t* g; int64_t* sc; int64_t* tok; float* val; int32_t* n; int64_t cap;
};

__device__ __forceinline__ void append1(int lane, int n, const int32_t (&g)[2], const int64_t (&sc)[2],
                                        const int64_t (&tok)[2], const float (&val)[2], const Lists& o, int32_t* err) {
  if (!__any_sync(0xFFFFFFFFu, n > 0)) return;
  int total;
  const int pre = warp_excl_scan(n, lane, &total);
  int base = 0;
  if (lane == 31) base = atomicAdd(o.n, total);
  base = __shfl_sync(0xFFFFFFFFu, base, 31);
  for (int k = 0; k < n; ++k) {
    const int64_t slot = (int64_t)base + pre + k;
    if (slot < o.cap) {
      o.g[slot] = g[k]; o.sc[slot] = sc[k]; o.tok[slot] = tok[k]; o.val[slot] = val[k];
    } else {
      atomicExch(err, 1);
    }
  }
}

__device__ __forceinline__ uint64_t comp_key(float s, int64_t tok) {
  const uint32_t hi = (uint32_t)(int32_t)ordered_f32(s) ^ 0x80000000u;
  const uint32_t lo = kM32 - (uint32_t)tok;
  return ((uint64_t)hi << 32) | lo;
}

template <int DT>
__device__ __forceinline__ bool skip_pass(int pass) {
  if (DT == ATLAS_BF16) return pass == 2 || pass == 3;  // fp32 bits 15..0 of a bf16 value are constant
  if (DT == ATLAS_F16) return pass == 3;                // fp32 bits 7..0 of an fp16 value are constant
  return false;
}

struct TopShared {
  uint32_t hist[2][256][32];
  unsigned long long P[2][32];
  int need[2][32];
  int nbits[2][32];
  int done[2][32];
};

template <int DT>
__global__ void __launch_bounds__(kTopWarps * 32)
dense_top_kernel(const typename Elem<DT>::T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ valid_rows,
                 int64_t n_v, const int64_t* __restrict__ tok, int64_t layer, int64_t K,
                 const float* __restrict__ top_seed, const int64_t* __restrict__ top_k, const int32_t* __restrict__ count,
                 int64_t cap, int force, Lists o, int32_t* __restrict__ flag, int32_t* __restrict__ err) {
  if (!force && (int64_t)*count <= cap) return;
  if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(flag, 1);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TopShared& sh = *reinterpret_cast<TopShared*>(smem_raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * 32 + lane;
  const bool cok = col < D;
  const bool select_all = n_v <= K;
  if (threadIdx.x < 64) {
    const int p = threadIdx.x >> 5;
    sh.P[p][lane] = 0;
    sh.need[p][lane] = (int)K;
    sh.nbits[p][lane] = 0;
    sh.done[p][lane] = (select_all || !cok) ? 1 : 0;
  }
  __syncthreads();
  if (!select_all) {
    for (int pass = 0; pass < 8; ++pass) {
      if (skip_pass<DT>(pass)) {
        if (threadIdx.x < 64) {
          const int p = threadIdx.x >> 5;
          if (!sh.done[p][lane]) {
            const int nb = sh.nbits[p][lane];
            const unsigned long long P = sh.P[p][lane];
            const bool nonneg = (P >> (nb - 1)) & 1ull;  // MSB of the key = sign of s (1: s >= 0)
            sh.P[p][lane] = (P << 8) | (nonneg ? 0x00ull : 0xFFull);
            sh.nbits[p][lane] = nb + 8;
          }
        }
        __syncthreads();
        continue;
      }
      for (int i = threadIdx.x; i < 2 * 256 * 32; i += blockDim.x) (&sh.hist[0][0][0])[i] = 0;
      __syncthreads();
      const int shift = 56 - 8 * pass;
      const bool act0 = !sh.done[0][lane], act1 = !sh.done[1][lane];
      const unsigned long long P0 = sh.P[0][lane], P1 = sh.P[1][lane];
      const int nb0 = sh.nbits[0][lane], nb1 = sh.nbits[1][lane];
      if (act0 || act1) {
        for (int64_t i = warp; i < n_v; i += kTopWarps) {
          const float h = Elem<DT>::f(H[(int64_t)valid_rows[i] * ld + col]);
          const int64_t t = tok[i];
          if (act0) {
            const uint64_t c = comp_key(h, t);
            if (nb0 == 0 || (c >> (64 - nb0)) == P0) atomicAdd(&sh.hist[0][(c >> shift) & 0xFF][lane], 1u);
          }
          if (act1) {
            const uint64_t c = comp_key(-h, t);
            if (nb1 == 0 || (c >> (64 - nb1)) == P1) atomicAdd(&sh.hist[1][(c >> shift) & 0xFF][lane], 1u);
          }
        }
      }
      __syncthreads();
      if (warp < 2 && !sh.done[warp][lane]) {
        const int p = warp;
        int need = sh.need[p][lane];
        int cum = 0;
        for (int d = 255; d >= 0; --d) {
          const int c = (int)sh.hist[p][d][lane];
          if (cum + c >= need) {
            need -= cum;
            sh.P[p][lane] = (sh.P[p][lane] << 8) | (unsigned long long)d;
            sh.nbits[p][lane] += 8;
            sh.need[p][lane] = need;
            if (c == need) sh.done[p][lane] = 1;
            break;
          }
          cum += c;
        }
      }
      __syncthreads();
      const int all = __syncthreads_and(threadIdx.x >= 64 || sh.done[threadIdx.x >> 5][lane]);
      if (all) break;
    }
  }
  // threshold per (pole, column): every key >= thr is one of the top min(K, n_v)
  unsigned long long thr[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int nb = sh.nbits[p][lane];
    thr[p] = select_all ? 0ull : (nb >= 64 ? sh.P[p][lane] : (nb == 0 ? 0ull : (sh.P[p][lane] << (64 - nb))));
  }
  int64_t kth[2] = {kI64Max, kI64Max};
  float seed[2] = {0.f, 0.f};
  if (cok) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int64_t g = (layer * 2 + p) * D + col;
      kth[p] = top_k[g * K + (K - 1)];
      seed[p] = top_seed[g];
    }
  }
  for (int64_t i = warp; i < n_v; i += kTopWarps) {
    int n = 0;
    int32_t gg[2];
    int64_t sc[2], tk[2];
    float vv[2];
    if (cok) {
      const float h = Elem<DT>::f(H[(int64_t)valid_rows[i] * ld + col]);
      const int64_t t = tok[i];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float s = p ? -h : h;
        const uint64_t c = comp_key(s, t);
        if (c >= thr[p] && s > seed[p]) {
          const int64_t k64 = (int64_t)(c ^ 0x8000000000000000ull);
          if (k64 > kth[p]) {
            gg[n] = (int32_t)((layer * 2 + p) * D + col); sc[n] = k64; tk[n] = t; vv[n] = s; ++n;
          }
        }
      }
    }
    append1(lane, n, gg, sc, tk, vv, o, err);
  }
}

// ------------------------------------------------------------------ reservoir: count + emit
template <int DT>
struct ResLane {
  float e[2][kMaxB];
  int64_t ceil[2][kMaxB];
};

template <int DT>
__device__ __forceinline__ int64_t res_setup(ResLane<DT>& r, int64_t layer, int64_t D, int64_t col, bool cok, int B,
                                             int64_t Kr, const int64_t* __restrict__ res_s,
                                             const int64_t* __restrict__ res_seed, const float* __restrict__ E) {
  int64_t mx = 0;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      r.e[p][b] = __int_as_float(0x7F800000);
      r.ceil[p][b] = 0;
      if (cok && b < B) {
        const int64_t gr = ((layer * 2 + p) * D + col) * B + b;
        r.e[p][b] = E[gr];
        int64_t thr = res_s[gr * Kr + (Kr - 1)];
        const int64_t sd = res_seed[gr];
        if (sd > thr) thr = sd;
        r.ceil[p][b] = (thr == kI64Min) ? (1ll << 32) : -thr;  // admit key < ceil
        if (r.ceil[p][b] > mx) mx = r.ceil[p][b];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int64_t y = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
    if (y > mx) mx = y;
  }
  return mx;
}

template <int DT>
__device__ __forceinline__ int lane_bin(const ResLane<DT>& r, int p, float s, int B) {
  int c = 0;
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) c += (b < B && s >= r.e[p][b]) ? 1 : 0;
  return c - 1;
}

template <int DT>
__global__ void __launch_bounds__(kResWarps * 32)
dense_res_count_kernel(const typename Elem<DT>::T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ valid_rows,
                       int64_t n_v, const int64_t* __restrict__ key, const int32_t* __restrict__ key_order, int64_t layer,
                       int B, int64_t Kr, const int64_t* __restrict__ res_s, const int64_t* __restrict__ res_seed,
                       const float* __restrict__ E, const int32_t* __restrict__ count, int64_t cap, int force,
                       int32_t* __restrict__ counts, int64_t n_chunks) {
  if (!force && (int64_t)*count <= cap) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t chunk = (int64_t)blockIdx.y * kResWarps + warp;
  if (chunk >= n_chunks) return;
  const int64_t col = (int64_t)blockIdx.x * 32 + lane;
  const bool cok = col < D;
  ResLane<DT> r;
  const int64_t maxceil = res_setup<DT>(r, layer, D, col, cok, B, Kr, res_s, res_seed, E);
  int cnt[2][kMaxB];
#pragma unroll
  for (int p = 0; p < 2; ++p)
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) cnt[p][b] = 0;
  const int64_t j1 = (chunk + 1) * kChunk < n_v ? (chunk + 1) * kChunk : n_v;
  for (int64_t j = chunk * kChunk; j < j1; ++j) {
    const int32_t vi = key_order[j];
    const int64_t k = key[vi];
    if (k >= maxceil) break;  // ascending keys: nothing further is admissible in these columns
    if (!cok) continue;
    const float h = Elem<DT>::f(H[(int64_t)valid_rows[vi] * ld + col]);
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float s = p ? -h : h;
      const int b = lane_bin<DT>(r, p, s, B);
#pragma unroll
      for (int bb = 0; bb < kMaxB; ++bb)
        if (bb == b && k < r.ceil[p][bb] && cnt[p][bb] < Kr) cnt[p][bb]++;
    }
  }
  if (cok) {
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int b = 0; b < kMaxB; ++b)
        if (b < B) counts[((chunk * 2 + p) * B + b) * D + col] = cnt[p][b];
  }
}

template <int DT>
__global__ void __launch_bounds__(kResWarps * 32)
dense_res_emit_kernel(const typename Elem<DT>::T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ valid_rows,
                      int64_t n_v, const int64_t* __restrict__ tok, const int64_t* __restrict__ key,
                      const int32_t* __restrict__ key_order, int64_t layer, int B, int64_t Kr,
                      const int64_t* __restrict__ res_s, const int64_t* __restrict__ res_seed, const float* __restrict__ E,
                      const int32_t* __restrict__ count, int64_t cap, int force, const int32_t* __restrict__ counts,
                      int64_t n_chunks, Lists o, int32_t* __restrict__ err) {
  if (!force && (int64_t)*count <= cap) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t chunk = (int64_t)blockIdx.y * kResWarps + warp;
  if (chunk >= n_chunks) return;
  const int64_t col = (int64_t)blockIdx.x * 32 + lane;
  const bool cok = col < D;
  ResLane<DT> r;
  const int64_t maxceil = res_setup<DT>(r, layer, D, col, cok, B, Kr, res_s, res_seed, E);
  int start[2][kMaxB];
  bool open = false;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      int s = 0;
      if (cok && b < B)
        for (int64_t c = 0; c < chunk && s < Kr; ++c) s += counts[((c * 2 + p) * B + b) * D + col];
      start[p][b] = s;
      if (cok && b < B && s < Kr) open = true;
    }
  }
  if (!__any_sync(0xFFFFFFFFu, open)) return;
  const int64_t j1 = (chunk + 1) * kChunk < n_v ? (chunk + 1) * kChunk : n_v;
  for (int64_t j = chunk * kChunk; j < j1; ++j) {
    const int32_t vi = key_order[j];
    const int64_t k = key[vi];
    if (k >= maxceil) break;
    int n = 0;
    int32_t gg[2];
    int64_t sc[2], tk[2];
    float vv[2];
    if (cok) {
      const float h = Elem<DT>::f(H[(int64_t)valid_rows[vi] * ld + col]);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float s = p ? -h : h;
        const int b = lane_bin<DT>(r, p, s, B);
#pragma unroll
        for (int bb = 0; bb < kMaxB; ++bb) {
          if (bb == b && k < r.ceil[p][bb]) {
            if (start[p][bb] < Kr) {
              gg[n] = (int32_t)(((layer * 2 + p) * D + col) * B + bb); sc[n] = -k; tk[n] = tok[vi]; vv[n] = h; ++n;
            }
            start[p][bb]++;
          }
        }
      }
    }
    append1(lane, n, gg, sc, tk, vv, o, err);
  }
}

template <int DT>
int launch_dense(const void* H, int64_t D, int64_t ld, int64_t layer, const int32_t* valid_rows, int64_t n_v,
                 const int64_t* tok, const int64_t* key, const int32_t* key_order, int64_t B, int64_t K, int64_t Kr,
                 int reservoir, const float* top_seed, const int64_t* top_k, const int64_t* res_s,
                 const int64_t* res_seed, const float* E, const int32_t* count, int64_t cap, int force, Lists top,
                 Lists res, void* scratch, int32_t* flag, int32_t* err, cudaStream_t st) {
  using T = typename Elem<DT>::T;
  const T* h = reinterpret_cast<const T*>(H);
  const unsigned strips = (unsigned)((D + 31) / 32);
  const size_t smem = sizeof(TopShared);
  if (cudaFuncSetAttribute(dense_top_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return fail(ATLAS_ERR_CUDA, "dense_select: cannot reserve %zu bytes of shared memory", smem);
  dense_top_kernel<DT><<<strips, kTopWarps * 32, smem, st>>>(h, D, ld, valid_rows, n_v, tok, layer, K, top_seed, top_k,
                                                              count, cap, force, top, flag, err);
  if (int e = check_launch("atlas_dense_select: top")) return e;
  if (!reservoir) return ATLAS_OK;
  const int64_t n_chunks = (n_v + kChunk - 1) / kChunk;
  if (n_chunks == 0) return ATLAS_OK;
  dim3 grid(strips, (unsigned)((n_chunks + kResWarps - 1) / kResWarps));
  int32_t* counts = reinterpret_cast<int32_t*>(scratch);
  dense_res_count_kernel<DT><<<grid, kResWarps * 32, 0, st>>>(h, D, ld, valid_rows, n_v, key, key_order, layer, (int)B,
                                                               Kr, res_s, res_seed, E, count, cap, force, counts, n_chunks);
  if (int e = check_launch("atlas_dense_select: res count")) return e;
  dense_res_emit_kernel<DT><<<grid, kResWarps * 32, 0, st>>>(h, D, ld, valid_rows, n_v, tok, key, key_order, layer,
                                                              (int)B, Kr, res_s, res_seed, E, count, cap, force, counts,
                                                              n_chunks, res, err);
  return check_launch("atlas_dense_select: res emit");
}

}  // namespace
}  // namespace atlas

using namespace atlas;

extern "C" int64_t atlas_dense_scratch_bytes(int64_t n_v, int64_t D, int64_t B) {
  const int64_t n_chunks = (n_v + kChunk - 1) / kChunk;
  return (n_chunks > 0 ? n_chunks : 1) * 2 * B * D * 4;
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
  ATLAS_REQUIRE(B >= 1 && B <= kMaxB && K >= 1 && Kr >= 1, "dense_select: B must be 1..%d", kMaxB);
  ATLAS_REQUIRE((layer * 2 + 2) * D * B < (1LL << 31), "dense_select: group ids exceed int32");
  if (n_v == 0) return ATLAS_OK;
  ATLAS_REQUIRE(force || count, "dense_select: count required unless forced");
  ATLAS_REQUIRE(H && valid_rows && tok && top_seed && top_k && top_g && top_sc && top_tok && top_val && n_top && flag && err,
                "dense_select: null pointer");
  if (reservoir) {
    ATLAS_REQUIRE(key && key_order && res_s && res_seed && E && res_g && res_sc && res_tok && res_val && n_res && scratch,
                  "dense_select: null reservoir pointer");
    ATLAS_REQUIRE(scratch_bytes >= atlas_dense_scratch_bytes(n_v, D, B), "dense_select: scratch too small");
  }
  Lists top{top_g, top_sc, top_tok, top_val, n_top, top_cap};
  Lists res{res_g, res_sc, res_tok, res_val, n_res, res_cap};
  const int32_t* cnt = count;
  cudaStream_t st = (cudaStream_t)stream;
  if (force && !cnt) cnt = n_top;  // never read when forced
  switch (dtype) {
    case ATLAS_BF16:
      return launch_dense<ATLAS_BF16>(H, D, ld, layer, valid_rows, n_v, tok, key, key_order, B, K, Kr, reservoir, top_seed,
                                      top_k, res_s, res_seed, E, cnt, cap, force, top, res, scratch, flag, err, st);
    case ATLAS_F16:
      return launch_dense<ATLAS_F16>(H, D, ld, layer, valid_rows, n_v, tok, key, key_order, B, K, Kr, reservoir, top_seed,
                                     top_k, res_s, res_seed, E, cnt, cap, force, top, res, scratch, flag, err, st);
    case ATLAS_F32:
      return launch_dense<ATLAS_F32>(H, D, ld, layer, valid_rows, n_v, tok, key, key_order, B, K, Kr, reservoir, top_seed,
                                     top_k, res_s, res_seed, E, cnt, cap, force, top, res, scratch, flag, err, st);
    default:
      return fail(ATLAS_ERR_ARG, "dense_select: unknown dtype %d", dtype);
  }
}
