// Dense burst path (Atlas._dense, atlas/core.py:407-446) on the live hook output, predicated on the
// device: it runs when the layer is a dense layer (force) or when its compaction buffer overflowed
// (*count > cap, the 0.5%-fill trigger), so the forward is never re-run and the host never syncs.
//
// Per column and pole the path selects, from the n_v valid rows, the exact top-K by top_key (the
// only batch elements that can enter the state's top-K) and, per reservoir bin, the Kr smallest keys
// among the rows in the bin under the bin's key ceiling. Two facts make most of that a streaming
// pass over H:
//  * a pole with at most K admissible candidates (s > seed and top_key above the state's K-th key)
//    has exactly those as its records: every larger batch element is a candidate too, so each
//    candidate lies inside the batch's top-K;
//  * a bin with at most Kr rows under its ceiling admits all of them, for the same reason.
// So:
// 1. dense_count (row-major over H, one thread per column of a 256-column strip, one CTA per strip
//    and row range): per column, the admissible top-K candidates per pole and the rows under each
//    (pole, bin) ceiling, as per-range partial counts. The last range of a strip to finish adds the
//    partials up and writes each column's decision: which poles need a select (> K candidates), which
//    bins are direct (1..Kr rows) and which ordered (> Kr rows), and the strip's list of such "hard"
//    columns. The same launch writes the rows' 32-bit keys in ascending key order.
// 2. dense_emit (the same grid): the records of every direct pole and bin, staged per CTA in shared
//    memory and appended with one atomic per list.
// 3. dense_hard (one CTA per hard column at a time, grid-stride): the column staged in shared memory
//    from H; poles that need it take an exact radix select (8-bit digits, MSB first, per-warp
//    shared-memory histograms) of the K-th largest composite key (ordered s bits | 2^32-1-tok), i.e.
//    the reference's top_key, then emit; ordered bins take their first Kr rows in ascending key
//    order, walking the key order a block-wide chunk at a time until every such bin is full or the
//    keys pass its ceiling (a dense bin ends within a few chunks).
// Passes 1 and 2 read H once each (coalesced, 64 bytes per warp and row); pass 3 only touches the
// hard columns, which are all columns only when the state is empty.
#include <algorithm>

#include "common.cuh"

namespace atlas {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxB = 8;
constexpr int kSlots = 2 * kMaxB;         // reservoir (pole, bin) slots: p * kMaxB + bin
constexpr int kStage = 1024;              // staged records per hard-column CTA (top: <= 2K; reservoir: <= 2*B*Kr)
constexpr int kEmitHalf = 256;            // staged records per emit CTA and list (overflow goes straight out)
constexpr int kStrip = 256;               // columns per strip: one per thread of the count and emit kernels
constexpr int kRangesMax = 64;            // row ranges per strip
constexpr int kPartRows = 2 + kSlots;     // partial counts per (range, column): 2 poles + 16 slots
constexpr int kU = 8;                     // rows in flight per thread in the count pass
constexpr int kUE = 4;                    // in the emit pass (its record path needs the registers)
constexpr int kChunk = 128;               // rows whose offsets and keys a row-major CTA stages at a time
constexpr int kDenseSmemMax = 227 * 1024; // opt-in shared memory per CTA

struct Lists {
  int32_t* g; int64_t* sc; int64_t* tok; float* val; int32_t* n; int64_t cap;
};

// Scratch of one call, carved from the caller's buffer (zero-filled before its first use; the
// ticket words are left at zero by every call).
struct DenseWs {
  int32_t* part;     // [R][kPartRows][D] partial counts of the row ranges
  uint32_t* dec;     // [D] reservoir decisions: bits 0-15 direct slots, 16-31 ordered slots
  uint32_t* tdec;    // [D] top-K decisions: bit p set when pole p needs the radix select
  int32_t* hard;     // [strips][kStrip] hard columns of each strip
  int32_t* nhard;    // [strips]
  int32_t* ticket;   // [strips] ranges of the strip done counting
  uint32_t* skey32;  // [n8] keys in ascending key order
};

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }
__host__ __device__ inline int64_t n_strips(int64_t D) { return (D + kStrip - 1) / kStrip; }

int64_t ws_bytes(int64_t n_v, int64_t D) {
  const int64_t S = n_strips(D), n8 = (n_v + 7) / 8 * 8;
  return 256 + align256((int64_t)kRangesMax * kPartRows * D * 4) + 2 * align256(D * 4) + align256(S * kStrip * 4) +
         2 * align256(S * 4) + align256(n8 * 4);
}

DenseWs carve(void* scratch, int64_t n_v, int64_t D) {
  const int64_t S = n_strips(D), n8 = (n_v + 7) / 8 * 8;
  uint8_t* p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(scratch) + 255) & ~uintptr_t(255));
  DenseWs w;
  w.part = reinterpret_cast<int32_t*>(p);
  p += align256((int64_t)kRangesMax * kPartRows * D * 4);
  w.dec = reinterpret_cast<uint32_t*>(p);
  p += align256(D * 4);
  w.tdec = reinterpret_cast<uint32_t*>(p);
  p += align256(D * 4);
  w.hard = reinterpret_cast<int32_t*>(p);
  p += align256(S * kStrip * 4);
  w.nhard = reinterpret_cast<int32_t*>(p);
  p += align256(S * 4);
  w.ticket = reinterpret_cast<int32_t*>(p);
  p += align256(S * 4);
  w.skey32 = reinterpret_cast<uint32_t*>(p);
  (void)n8;
  return w;
}

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

// Per-column parameters of the state: the top-K seed and K-th state key per pole, the reservoir
// edges (NaN for unused bins: compares false, even against +inf) and the key ceilings per slot
// (admit key < ceiling).
struct ColParams {
  float seed[2];
  uint64_t ku[2];  // the state's K-th key in unsigned order (top_key ^ sign bit)
  float e[2][kMaxB];
};

__device__ __forceinline__ void load_params(ColParams& cp, bool ok, int64_t layer, int64_t D, int64_t d, int B,
                                            int64_t K, int reservoir, const float* __restrict__ top_seed,
                                            const int64_t* __restrict__ top_k, const float* __restrict__ E) {
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int64_t g = (layer * 2 + p) * D + d;
    cp.seed[p] = ok ? top_seed[g] : __int_as_float(0x7F800000);  // +inf: no candidate
    cp.ku[p] = (uint64_t)(ok ? top_k[g * K + (K - 1)] : 0) ^ 0x8000000000000000ull;
#pragma unroll
    for (int b = 0; b < kMaxB; ++b)
      cp.e[p][b] = (ok && reservoir && b < B) ? E[g * B + b] : __int_as_float(0x7FC00000);
  }
}

__device__ __forceinline__ int64_t slot_ceiling(int slot, bool ok, int64_t layer, int64_t D, int64_t d, int B,
                                                int64_t Kr, int reservoir, const int64_t* __restrict__ res_s,
                                                const int64_t* __restrict__ res_seed) {
  const int p = slot / kMaxB, b = slot % kMaxB;
  if (!ok || !reservoir || b >= B) return 0;
  const int64_t gr = ((layer * 2 + p) * D + d) * B + b;
  int64_t th = res_s[gr * Kr + (Kr - 1)];
  const int64_t sd = res_seed[gr];
  if (sd > th) th = sd;
  return (th == kI64Min) ? (1ll << 32) : -th;
}

// Admissible top-K candidate once s > seed holds: top_key(s, tok) above the state's K-th key (token
// ids are read only on a tie of the value part).
__device__ __forceinline__ bool top_above(float s, uint64_t ku, const int64_t* __restrict__ tok, int64_t i) {
  const uint32_t hi = key_hi(s), khi = (uint32_t)(ku >> 32);
  if (hi != khi) return hi > khi;
  const uint64_t c = ((uint64_t)hi << 32) | (uint64_t)(kM32 - (uint32_t)tok[i]);
  return c > ku;
}

// Bin of s (at or above the lowest edge) among NB edges; unused edges (NB = kMaxB with B < kMaxB) are
// NaN and never counted.
template <int NB>
__device__ __forceinline__ int bin_in(float s, const float (&ep)[kMaxB]) {
  int bin = 0;
#pragma unroll
  for (int b = 1; b < NB; ++b) bin += (s >= ep[b]) ? 1 : 0;
  return bin;
}

// Reservoir slot (p * kMaxB + bin) of value s for pole P, or -1 below the pole's lowest edge.
template <int P, int NB>
__device__ __forceinline__ int res_slot(float s, const float (&e)[2][kMaxB]) {
  if (!(s >= e[P][0])) return -1;
  return P * kMaxB + bin_in<NB>(s, e[P]);
}

// Row range r of R over n_v rows.
__device__ __forceinline__ void row_range(int64_t n_v, int r, int R, int64_t& i0, int64_t& i1) {
  i0 = n_v * r / R;
  i1 = n_v * (r + 1) / R;
}

// ------------------------------------------------------------------------------------ 1. count
// Necessary condition for a row to enter the bin search of pole p (value s = +-h, key k), kept in
// registers per thread: either s reaches the top bin's edge and k is under the top bin's ceiling, or
// s reaches the lowest edge and k is under the largest ceiling of the other bins. The top bin (the
// rarest values) is the one whose reservoir stays open longest, often with the whole key range as its
// ceiling; apart from it, seeded ceilings are small, so most rows fail both tests without a search.
struct PoleGate {
  float etop[2];                   // edge of the top bin (bin B-1)
  uint32_t lim_top[2], lim_rest[2];  // ceiling - 1 of the top bin / largest ceiling - 1 of the others
  bool on_top[2], on_rest[2];      // a ceiling above 0 exists
};

__device__ __forceinline__ uint32_t ceil_limit(int64_t c) {
  return c > 0 ? (uint32_t)((c > (1ll << 32) ? (1ll << 32) : c) - 1) : 0u;
}

// NB < kMaxB: compiled for exactly NB bins (B == NB), so the top bin's index is a constant and the
// edges stay in registers.
template <int NB>
__device__ __forceinline__ void pole_gate(const int64_t (*s_ceil)[kStrip], int tid, int B, const ColParams& cp,
                                          PoleGate& g) {
  const int tb = NB < kMaxB ? NB - 1 : B - 1;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    int64_t rest = 0, top = 0;
    float et = __int_as_float(0x7FC00000);
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      const int64_t c = s_ceil[p * kMaxB + b][tid];
      if (b == tb) {
        top = c;
        et = cp.e[p][b];
      } else if (b < tb) {
        rest = c > rest ? c : rest;
      }
    }
    g.etop[p] = et;
    g.on_top[p] = top > 0;
    g.lim_top[p] = ceil_limit(top);
    g.on_rest[p] = rest > 0;
    g.lim_rest[p] = ceil_limit(rest);
  }
}

template <int P>
__device__ __forceinline__ bool gate_pass(float s, uint32_t k, const ColParams& cp, const PoleGate& g) {
  return (g.on_top[P] & (s >= g.etop[P]) & (k <= g.lim_top[P])) |
         (g.on_rest[P] & (s >= cp.e[P][0]) & (k <= g.lim_rest[P]));
}

// One row of the count pass for this thread's column: admissible top-K candidates per pole, rows
// under the ceiling of their (pole, bin).
template <int NB>
__device__ __forceinline__ void count_row(float h, uint32_t k, int64_t i, const ColParams& cp, const PoleGate& gt,
                                          const int64_t (*s_ceil)[kStrip], int tid,
                                          const int64_t* __restrict__ tok, int& c0, int& c1, uint64_t (&rc)[2][2]) {
  if ((h > cp.seed[0]) | (-h > cp.seed[1])) {  // rare once seeded: one branch for both poles
    if (h > cp.seed[0] && top_above(h, cp.ku[0], tok, i)) ++c0;
    if (-h > cp.seed[1] && top_above(-h, cp.ku[1], tok, i)) ++c1;
  }
  const bool pa = gate_pass<0>(h, k, cp, gt);
  const bool pb = gate_pass<1>(-h, k, cp, gt);
  if (pa | pb) {
    if (pa) {
      const int b = bin_in<NB>(h, cp.e[0]);
      if ((int64_t)k < s_ceil[b][tid]) {
        const uint64_t inc = 1ull << (16 * (b & 3));
        if (b < 4) rc[0][0] += inc; else rc[0][1] += inc;
      }
    }
    if (pb) {
      const int b = bin_in<NB>(-h, cp.e[1]);
      if ((int64_t)k < s_ceil[kMaxB + b][tid]) {
        const uint64_t inc = 1ull << (16 * (b & 3));
        if (b < 4) rc[1][0] += inc; else rc[1][1] += inc;
      }
    }
  }
}

template <int DT, int NB>
__global__ void __launch_bounds__(kStrip, 4)
dense_count_kernel(const typename Elem<DT>::T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ rows,
                   int64_t n_v, const int64_t* __restrict__ tok, const int64_t* __restrict__ key,
                   const int32_t* __restrict__ key_order, int64_t layer, int B, int64_t K, int64_t Kr, int reservoir,
                   const float* __restrict__ top_seed, const int64_t* __restrict__ top_k,
                   const int64_t* __restrict__ res_s, const int64_t* __restrict__ res_seed, const float* __restrict__ E,
                   const int32_t* __restrict__ count, int64_t cap, int force, DenseWs ws) {
  using T = typename Elem<DT>::T;
  if (!triggered(count, cap, force)) return;
  __shared__ int64_t s_ceil[kSlots][kStrip];
  __shared__ int64_t s_off[kChunk];
  __shared__ uint32_t s_key[kChunk];
  __shared__ int s_wn[kThreads / 32];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int strip = blockIdx.x, r = blockIdx.y, R = gridDim.y;
  const int64_t d = (int64_t)strip * kStrip + tid;
  const bool ok = d < D;
  if (reservoir) {  // the keys in ascending key order, for the hard columns' ordered walks
    const int64_t nth = (int64_t)gridDim.x * gridDim.y * kThreads;
    for (int64_t j = ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * kThreads + tid; j < n_v; j += nth)
      ws.skey32[j] = (uint32_t)key[key_order[j]];
  }
  ColParams cp;
  load_params(cp, ok, layer, D, d, B, K, reservoir, top_seed, top_k, E);
#pragma unroll
  for (int s = 0; s < kSlots; ++s) s_ceil[s][tid] = slot_ceiling(s, ok, layer, D, d, B, Kr, reservoir, res_s, res_seed);
  int64_t i0, i1;
  row_range(n_v, r, R, i0, i1);
  int c0 = 0, c1 = 0;
  uint64_t rc[2][2] = {{0ull, 0ull}, {0ull, 0ull}};  // 16-bit counts per (pole, bin): [p][bin / 4]
  const T* Hc = H + (ok ? d : 0);
  PoleGate gt;
  pole_gate<NB>(s_ceil, tid, B, cp, gt);
  // the rows a chunk at a time: their offsets in H and 32-bit keys staged once per CTA (every
  // thread reads the same rows); whole groups of kU rows without bounds checks, then the tail
  for (int64_t cs = i0; cs < i1; cs += kChunk) {
    const int nrow = (int)(i1 - cs < kChunk ? i1 - cs : kChunk);
    __syncthreads();
    if (tid < nrow) {
      s_off[tid] = (int64_t)rows[cs + tid] * ld;
      s_key[tid] = reservoir ? (uint32_t)key[cs + tid] : 0u;
    }
    __syncthreads();
    const int nfull = nrow & ~(kU - 1);
    for (int j = 0; j < nfull; j += kU) {
      T x[kU];
      uint32_t kk[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        x[u] = Hc[s_off[j + u]];
        kk[u] = s_key[j + u];
      }
#pragma unroll
      for (int u = 0; u < kU; ++u)
        count_row<NB>(Elem<DT>::f(x[u]), kk[u], cs + j + u, cp, gt, s_ceil, tid, tok, c0, c1, rc);
    }
    for (int j = nfull; j < nrow; ++j)
      count_row<NB>(Elem<DT>::f(Hc[s_off[j]]), s_key[j], cs + j, cp, gt, s_ceil, tid, tok, c0, c1, rc);
  }
  if (ok) {
    int32_t* P = ws.part + (int64_t)r * kPartRows * D + d;
    P[0] = c0;
    P[D] = c1;
#pragma unroll
    for (int s = 0; s < kSlots; ++s)
      P[(int64_t)(2 + s) * D] = (int)((rc[s / kMaxB][(s % kMaxB) >> 2] >> (16 * (s & 3))) & 0xFFFFull);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(ws.ticket + strip, 1) == R - 1) ? 1 : 0;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // the strip's last range: totals and decisions per column, then the strip's hard columns
  uint32_t hardf = 0;
  if (ok) {
    int tt[kPartRows];
#pragma unroll
    for (int q = 0; q < kPartRows; ++q) tt[q] = 0;
    for (int q = 0; q < R; ++q) {
      const int32_t* P = ws.part + (int64_t)q * kPartRows * D + d;
#pragma unroll
      for (int k = 0; k < kPartRows; ++k) tt[k] += __ldcg(P + (int64_t)k * D);
    }
    uint32_t direct = 0, ordered = 0, th = 0;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      const int t = tt[2 + s];
      if (t > 0 && t <= Kr) direct |= 1u << s;
      if (t > Kr) ordered |= 1u << s;
    }
    if (tt[0] > K) th |= 1u;
    if (tt[1] > K) th |= 2u;
    ws.dec[d] = direct | (ordered << 16);
    ws.tdec[d] = th;
    hardf = (th | ordered) ? 1u : 0u;
  }
  const uint32_t bal = __ballot_sync(0xFFFFFFFFu, hardf != 0);
  if (lane == 0) s_wn[warp] = __popc(bal);
  __syncthreads();
  int off = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    off += w < warp ? s_wn[w] : 0;
    tot += s_wn[w];
  }
  if (hardf) ws.hard[strip * kStrip + off + __popc(bal & ((1u << lane) - 1u))] = (int32_t)d;
  if (tid == 0) {
    ws.nhard[strip] = tot;
    ws.ticket[strip] = 0;  // ready for the next call
  }
}

// ------------------------------------------------------------------------------------- 2. emit
struct EmitStage {
  int32_t g[2][kEmitHalf];
  int64_t sc[2][kEmitHalf], tok[2][kEmitHalf];
  float val[2][kEmitHalf];
  int n[2];
  int base[2];
};

// One record of list w (0 top, 1 reservoir): a staging slot while the half has room, else straight
// to the list (one global atomic; the list count stays exact past its capacity).
__device__ __forceinline__ void emit_rec(EmitStage& es, int w, const Lists& o, int32_t g, int64_t sc, int64_t tk,
                                         float v, int32_t* err) {
  const int i = atomicAdd(&es.n[w], 1);
  if (i < kEmitHalf) {
    es.g[w][i] = g; es.sc[w][i] = sc; es.tok[w][i] = tk; es.val[w][i] = v;
  } else {
    const int64_t slot = atomicAdd(o.n, 1);
    if (slot < o.cap) {
      o.g[slot] = g; o.sc[slot] = sc; o.tok[slot] = tk; o.val[slot] = v;
    } else {
      atomicExch(err, 1);
    }
  }
}

// One row of the emit pass for this thread's column: the records of its direct poles and bins.
template <int NB>
__device__ __forceinline__ void emit_row(float h, uint32_t k, int64_t i, const ColParams& cp, const PoleGate& gt,
                                         const int64_t (*s_ceil)[kStrip], int tid,
                                         const int64_t* __restrict__ tok, int32_t g0, int32_t g1, int B, EmitStage& es,
                                         const Lists& top, const Lists& res, int32_t* __restrict__ err) {
  if ((h > cp.seed[0]) | (-h > cp.seed[1])) {
    if (h > cp.seed[0] && top_above(h, cp.ku[0], tok, i)) {
      const int64_t t = tok[i];
      emit_rec(es, 0, top, g0,
               (int64_t)((((uint64_t)key_hi(h) << 32) | (uint64_t)(kM32 - (uint32_t)t)) ^ 0x8000000000000000ull), t,
               h, err);
    }
    if (-h > cp.seed[1] && top_above(-h, cp.ku[1], tok, i)) {
      const int64_t t = tok[i];
      emit_rec(es, 0, top, g1,
               (int64_t)((((uint64_t)key_hi(-h) << 32) | (uint64_t)(kM32 - (uint32_t)t)) ^ 0x8000000000000000ull), t,
               -h, err);
    }
  }
  const bool pa = gate_pass<0>(h, k, cp, gt);
  const bool pb = gate_pass<1>(-h, k, cp, gt);
  if (pa | pb) {  // non-direct slots have ceiling 0 here, so they never admit
    if (pa) {
      const int b = bin_in<NB>(h, cp.e[0]);
      if ((int64_t)k < s_ceil[b][tid]) emit_rec(es, 1, res, g0 * B + b, -(int64_t)k, tok[i], h, err);
    }
    if (pb) {
      const int b = bin_in<NB>(-h, cp.e[1]);
      if ((int64_t)k < s_ceil[kMaxB + b][tid]) emit_rec(es, 1, res, g1 * B + b, -(int64_t)k, tok[i], h, err);
    }
  }
}

template <int DT, int NB>
__global__ void __launch_bounds__(kStrip, 4)
dense_emit_kernel(const typename Elem<DT>::T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ rows,
                  int64_t n_v, const int64_t* __restrict__ tok, const int64_t* __restrict__ key, int64_t layer, int B,
                  int64_t K, int64_t Kr, int reservoir, const float* __restrict__ top_seed,
                  const int64_t* __restrict__ top_k, const int64_t* __restrict__ res_s,
                  const int64_t* __restrict__ res_seed, const float* __restrict__ E, const int32_t* __restrict__ count,
                  int64_t cap, int force, DenseWs ws, Lists top, Lists res, int32_t* __restrict__ err) {
  using T = typename Elem<DT>::T;
  if (!triggered(count, cap, force)) return;
  __shared__ int64_t s_ceil[kSlots][kStrip];
  __shared__ int64_t s_off[kChunk];
  __shared__ uint32_t s_key[kChunk];
  __shared__ EmitStage es;
  const int tid = threadIdx.x;
  const int strip = blockIdx.x, r = blockIdx.y, R = gridDim.y;
  const int64_t d = (int64_t)strip * kStrip + tid;
  const bool ok = d < D;
  const uint32_t th = ok ? ws.tdec[d] : 3u;
  const uint32_t direct = ok ? (ws.dec[d] & 0xFFFFu) : 0u;
  ColParams cp;
  load_params(cp, ok, layer, D, d, B, K, reservoir, top_seed, top_k, E);
  if (th & 1u) cp.seed[0] = __int_as_float(0x7F800000);  // pole emitted by the hard-column kernel
  if (th & 2u) cp.seed[1] = __int_as_float(0x7F800000);
#pragma unroll
  for (int s = 0; s < kSlots; ++s)  // ceilings of the direct slots only (0: the slot admits nothing here)
    s_ceil[s][tid] = ((direct >> s) & 1u) ? slot_ceiling(s, ok, layer, D, d, B, Kr, reservoir, res_s, res_seed) : 0;
  PoleGate gt;
  pole_gate<NB>(s_ceil, tid, B, cp, gt);
  if (tid < 2) es.n[tid] = 0;
  __syncthreads();
  const bool any = __syncthreads_or(ok && (((th & 3u) != 3u) || direct != 0)) != 0;
  if (any) {
    int64_t i0, i1;
    row_range(n_v, r, R, i0, i1);
    const T* Hc = H + (ok ? d : 0);
    const int32_t g0 = (int32_t)((layer * 2) * D + d), g1 = (int32_t)((layer * 2 + 1) * D + d);
    for (int64_t cs = i0; cs < i1; cs += kChunk) {
      const int nrow = (int)(i1 - cs < kChunk ? i1 - cs : kChunk);
      __syncthreads();
      if (tid < nrow) {
        s_off[tid] = (int64_t)rows[cs + tid] * ld;
        s_key[tid] = reservoir ? (uint32_t)key[cs + tid] : 0u;
      }
      __syncthreads();
      const int nfull = nrow & ~(kUE - 1);
      for (int j = 0; j < nfull; j += kUE) {
        T x[kUE];
        uint32_t kk[kUE];
#pragma unroll
        for (int u = 0; u < kUE; ++u) {
          x[u] = Hc[s_off[j + u]];
          kk[u] = s_key[j + u];
        }
#pragma unroll
        for (int u = 0; u < kUE; ++u)
          emit_row<NB>(Elem<DT>::f(x[u]), kk[u], cs + j + u, cp, gt, s_ceil, tid, tok, g0, g1, B, es, top, res,
                       err);
      }
      for (int j = nfull; j < nrow; ++j)
        emit_row<NB>(Elem<DT>::f(Hc[s_off[j]]), s_key[j], cs + j, cp, gt, s_ceil, tid, tok, g0, g1, B, es, top,
                     res, err);
    }
  }
  __syncthreads();
  if (tid < 2) {
    const int n = es.n[tid] < kEmitHalf ? es.n[tid] : kEmitHalf;
    es.base[tid] = n > 0 ? atomicAdd(tid ? res.n : top.n, n) : 0;
  }
  __syncthreads();
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const Lists& o = w ? res : top;
    const int n = es.n[w] < kEmitHalf ? es.n[w] : kEmitHalf;
    for (int i = tid; i < n; i += kThreads) {
      const int64_t slot = (int64_t)es.base[w] + i;
      if (slot < o.cap) {
        o.g[slot] = es.g[w][i]; o.sc[slot] = es.sc[w][i]; o.tok[slot] = es.tok[w][i]; o.val[slot] = es.val[w][i];
      } else {
        atomicExch(err, 1);
      }
    }
  }
}

// ---------------------------------------------------------------------------------- 3. hard columns
// Records of one hard column staged in shared memory: top-K records from slot 0 up (at most 2K),
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
  int64_t ceil[kSlots];                   // reservoir key ceiling per (pole, bin) of the column
  int rfound[kSlots];                     // ordered walk: rows admitted so far per (pole, bin)
  int wcnt[kThreads / 32][kSlots];        // ordered walk: per-warp counts of one chunk
  int pre[kRangesMax * 4 + 1];            // hard-list prefix over the strips
  int base;
  Staged st;
};

// One hard column d (the CTA's threads together): the poles flagged in th take the radix select and
// emit their top-K records; the slots flagged in `ordered` take their first Kr rows in key order.
template <int DT, int NB>
__device__ __forceinline__ void hard_column(ColShared& sh, typename Elem<DT>::T* scol, int64_t d,
                                            const typename Elem<DT>::T* __restrict__ H, int64_t ld,
                                            const int32_t* __restrict__ rows, int64_t n_v,
                                            const int64_t* __restrict__ tok, const uint32_t* __restrict__ skey32,
                                            const int32_t* __restrict__ key_order, int64_t layer, int64_t D, int B,
                                            int64_t K, int64_t Kr, const float* __restrict__ top_seed,
                                            const int64_t* __restrict__ top_k, const int64_t* __restrict__ res_s,
                                            const int64_t* __restrict__ res_seed, const float* __restrict__ E,
                                            uint32_t th, uint32_t ordered, Lists top, Lists res,
                                            int32_t* __restrict__ err) {
  using T = typename Elem<DT>::T;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (scol != nullptr)  // the column staged in shared memory: every pass below reads it from there
    for (int64_t i = tid; i < n_v; i += kThreads) scol[i] = H[(int64_t)rows[i] * ld + d];
  auto colv = [&](int64_t i) -> float { return Elem<DT>::f(scol ? scol[i] : H[(int64_t)rows[i] * ld + d]); };
  const int top_lim = (int)(2 * K), res_lim = kStage - (int)(2 * K);
  ColParams cp;
  load_params(cp, true, layer, D, d, B, K, ordered != 0, top_seed, top_k, E);
  if (tid < kSlots) {
    sh.ceil[tid] = ((ordered >> tid) & 1u) ? slot_ceiling(tid, true, layer, D, d, B, Kr, 1, res_s, res_seed) : 0;
    sh.rfound[tid] = 0;
  }
  if (tid < 2) {
    sh.P[tid] = 0;
    sh.need[tid] = (int)K;
    sh.nbits[tid] = 0;
    sh.done[tid] = ((th >> tid) & 1u) ? 0 : 1;
  }
  if (tid == 0) {
    sh.st.n = 0;
    sh.st.m = 0;
  }
  for (int i = tid; i < (kThreads / 32) * kSlots; i += kThreads) (&sh.wcnt[0][0])[i] = 0;
  __syncthreads();
  // ------------------------------------------------------------------ top-K radix select
  if (th) {
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
        const float h = colv(i);
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
    unsigned long long thr[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int nb = sh.nbits[p];
      thr[p] = (nb >= 64 ? sh.P[p] : (nb == 0 ? 0ull : (sh.P[p] << (64 - nb))));
    }
    for (int64_t i = tid; i < n_v; i += kThreads) {
      const float h = colv(i);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        if (!((th >> p) & 1u)) continue;
        const float s = p ? -h : h;
        const uint32_t hi = key_hi(s);
        if (hi < (uint32_t)(thr[p] >> 32) || !(s > cp.seed[p])) continue;  // below the K-th value
        const int64_t t = tok[i];
        const uint64_t c = ((uint64_t)hi << 32) | (uint64_t)(kM32 - (uint32_t)t);
        if (c >= thr[p] && c > cp.ku[p])
          stage_top(sh.st, top_lim, (int32_t)((layer * 2 + p) * D + d), (int64_t)(c ^ 0x8000000000000000ull), t, s,
                    err);
      }
    }
  }
  // ------------------------------------------------------------------ ordered walk
  if (ordered) {
    const uint32_t lt = (1u << lane) - 1u;
    for (int64_t j0 = 0; j0 < n_v; j0 += kThreads) {
      // the open slots and their largest ceiling (every thread reads the same shared values)
      uint32_t open = 0;
      int64_t maxc = 0;
#pragma unroll
      for (int c = 0; c < kSlots; ++c) {
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
          h = colv(vi);
          const int sa = res_slot<0, NB>(h, cp.e), sb = res_slot<1, NB>(-h, cp.e);
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
      if (tid < kSlots) {
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

// Hard columns are taken grid-stride from the strips' lists by at most one resident wave of CTAs,
// so an untriggered launch, or one with no hard column, costs about a wave of early exits.
template <int DT, int NB>
__global__ void __launch_bounds__(kThreads, 4)
dense_hard_kernel(const typename Elem<DT>::T* __restrict__ H, int64_t D, int64_t ld, const int32_t* __restrict__ rows,
                  int64_t n_v, const int64_t* __restrict__ tok, const int32_t* __restrict__ key_order, int64_t layer,
                  int B, int64_t K, int64_t Kr, int reservoir, const float* __restrict__ top_seed,
                  const int64_t* __restrict__ top_k, const int64_t* __restrict__ res_s,
                  const int64_t* __restrict__ res_seed, const float* __restrict__ E, const int32_t* __restrict__ count,
                  int64_t cap, int force, DenseWs ws, Lists top, Lists res, int32_t* __restrict__ err,
                  int col_in_smem) {
  if (!triggered(count, cap, force)) return;
  extern __shared__ __align__(16) unsigned char col_raw[];
  ColShared& sh = *reinterpret_cast<ColShared*>(col_raw);
  // with col_in_smem the column (n_v elements) is staged after the shared state
  auto* scol = col_in_smem ? reinterpret_cast<typename Elem<DT>::T*>(col_raw + ((sizeof(ColShared) + 15) / 16) * 16)
                           : nullptr;
  const int S = (int)n_strips(D);
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int s = 0; s < S; ++s) {
      sh.pre[s] = acc;
      acc += ws.nhard[s];
    }
    sh.pre[S] = acc;
  }
  __syncthreads();
  const int total = sh.pre[S];
  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    int s = 0;
    while (sh.pre[s + 1] <= t) ++s;
    const int64_t d = ws.hard[s * kStrip + (t - sh.pre[s])];
    const uint32_t th = ws.tdec[d];
    const uint32_t ordered = reservoir ? (ws.dec[d] >> 16) : 0u;
    hard_column<DT, NB>(sh, scol, d, H, ld, rows, n_v, tok, ws.skey32, key_order, layer, D, B, K, Kr, top_seed, top_k,
                    res_s, res_seed, E, th, ordered, top, res, err);
    __syncthreads();  // the next column re-initialises the shared state and the staged column
  }
}

template <int DT, int NB>
int launch_dense(const void* Hv, int64_t D, int64_t ld, int64_t layer, const int32_t* valid_rows, int64_t n_v,
                 const int64_t* tok, const int64_t* key, const int32_t* key_order, int64_t B, int64_t K, int64_t Kr,
                 int reservoir, const float* top_seed, const int64_t* top_k, const int64_t* res_s,
                 const int64_t* res_seed, const float* E, const int32_t* count, int64_t cap, int force, Lists top,
                 Lists res, void* scratch, int32_t* err, cudaStream_t st) {
  using T = typename Elem<DT>::T;
  const T* H = reinterpret_cast<const T*>(Hv);
  const DenseWs ws = carve(scratch, n_v, D);
  const int64_t S = n_strips(D);
  // row ranges: about four resident 256-thread CTAs per SM over the strips, at least 64 rows and at
  // most 65535 rows (16-bit per-thread counts) per range
  int64_t R = std::max<int64_t>(1, ((int64_t)num_sms() * 4) / S);  // S x R <= one resident wave
  R = std::min<int64_t>(R, std::max<int64_t>(1, n_v / 64));
  R = std::max<int64_t>(R, (n_v + 65534) / 65535);
  R = std::min<int64_t>(R, kRangesMax);
  const dim3 g1((unsigned)S, (unsigned)R);
  dense_count_kernel<DT, NB><<<g1, kStrip, 0, st>>>(H, D, ld, valid_rows, n_v, tok, key, key_order, layer, (int)B, K, Kr,
                                                reservoir, top_seed, top_k, res_s, res_seed, E, count, cap, force, ws);
  if (int e = check_launch("atlas_dense_select: count")) return e;
  dense_emit_kernel<DT, NB><<<g1, kStrip, 0, st>>>(H, D, ld, valid_rows, n_v, tok, key, layer, (int)B, K, Kr, reservoir,
                                               top_seed, top_k, res_s, res_seed, E, count, cap, force, ws, top, res, err);
  if (int e = check_launch("atlas_dense_select: emit")) return e;
  // the hard column goes to shared memory when it fits next to the shared state (C4: ~61 KB of bf16
  // per column); otherwise every pass reads it from H
  const size_t base_smem = ((sizeof(ColShared) + 15) / 16) * 16;
  const size_t col_bytes = (size_t)((n_v + 7) / 8 * 8) * sizeof(T);
  const int col_in_smem = base_smem + col_bytes <= (size_t)kDenseSmemMax ? 1 : 0;
  const size_t smem = col_in_smem ? base_smem + col_bytes : sizeof(ColShared);
  // the attribute is set once per device and instantiation (this launch runs once per layer and
  // batch, mostly to exit at once on the device, so no per-call host queries)
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cudaFuncSetAttribute(dense_hard_kernel<DT, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDenseSmemMax) !=
        cudaSuccess)
      return fail(ATLAS_ERR_CUDA, "dense_select: cannot reserve %zu bytes of shared memory", smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  // resident CTAs per SM: registers allow four (at most 64 x 256 per CTA); shared memory as many as
  // fit in the SM's 228 KB (1 KB of it reserved per CTA)
  int per_sm = (int)(((size_t)228 * 1024) / (smem + 1024));
  per_sm = per_sm < 1 ? 1 : (per_sm > 4 ? 4 : per_sm);
  const unsigned g3 = (unsigned)std::max<int64_t>(1, std::min<int64_t>(D, (int64_t)num_sms() * per_sm));
  dense_hard_kernel<DT, NB><<<g3, kThreads, smem, st>>>(H, D, ld, valid_rows, n_v, tok, key_order, layer, (int)B, K, Kr,
                                                    reservoir, top_seed, top_k, res_s, res_seed, E, count, cap, force,
                                                    ws, top, res, err, col_in_smem);
  return check_launch("atlas_dense_select: hard columns");
}

int esize(int dtype) { return dtype == ATLAS_F32 ? 4 : 2; }

}  // namespace
}  // namespace atlas

using namespace atlas;

extern "C" int64_t atlas_dense_scratch_bytes(int64_t n_v, int64_t D, int64_t B, int dtype) {
  (void)B;
  (void)dtype;
  return ws_bytes(n_v, D);  // partial counts, decisions, hard-column lists, keys in key order
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
  ATLAS_REQUIRE(n_v <= (int64_t)kRangesMax * 65535, "dense_select: more than %lld valid rows",
                (long long)kRangesMax * 65535);
  ATLAS_REQUIRE(n_strips(D) <= kRangesMax * 4, "dense_select: D above %d", kRangesMax * 4 * kStrip);
  (void)esize;
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
  // bins: B = 5 (the reference's default edges) compiled exactly, other B on kMaxB NaN-padded edges
#define ATLAS_DENSE_CALL(DT, NB)                                                                                   \
  launch_dense<DT, NB>(H, D, ld, layer, valid_rows, n_v, tok, key, key_order, B, K, Kr, reservoir, top_seed, top_k, \
                       res_s, res_seed, E, cnt, cap, force, top, res, scratch, err, st)
  switch (dtype) {
    case ATLAS_BF16:
      return B == 5 ? ATLAS_DENSE_CALL(ATLAS_BF16, 5) : ATLAS_DENSE_CALL(ATLAS_BF16, kMaxB);
    case ATLAS_F16:
      return B == 5 ? ATLAS_DENSE_CALL(ATLAS_F16, 5) : ATLAS_DENSE_CALL(ATLAS_F16, kMaxB);
    case ATLAS_F32:
      return B == 5 ? ATLAS_DENSE_CALL(ATLAS_F32, 5) : ATLAS_DENSE_CALL(ATLAS_F32, kMaxB);
    default:
      return fail(ATLAS_ERR_ARG, "dense_select: unknown dtype %d", dtype);
  }
#undef ATLAS_DENSE_CALL
}
