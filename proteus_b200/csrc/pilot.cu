// Pilot pass on the device: bin edges and exact-preserving seeds from pilot activations
// (atlas/reference.py:55-122: pilot_edges, pilot_seeds), without a sort.
//
// atlas_column_select  exact order statistics of every column: the values at given ascending ranks,
//                      by an MSB-first radix select on order-preserving keys (8-bit digits: 2
//                      passes for bf16 / fp16, 4 for fp32). One CTA per column of the transposed
//                      activations (a contiguous row of XT); per pass, one shared-memory histogram
//                      per distinct prefix among the wanted ranks. Keys order -0.0 below +0.0, as a
//                      radix sort of the float bits does.
// atlas_pilot_edges    E[p, d, b] from the selected values (pole 1 = -h: the value at rank r of
//                      sort(-h) is minus the value at rank n-1-r of sort(h)), then the strictly
//                      increasing fix E_b = max(E_b, nextafter(E_{b-1}, +inf)).
// atlas_pilot_counts   per (pole, column, bin): the number of pilot rows in the bin and, with
//                      protein groups, the sum over groups of the squared per-group count. Rows are
//                      visited in group order (runs); a CTA takes whole runs, so counts are exact
//                      integers whatever the split.
// atlas_pilot_seeds    top seed = nextafter(2K-th largest s, -inf); reservoir key ceiling
//                      floor(min(c*Kr*2^32 / (n_total * m_lo), 2^32)) with m_lo the z-sigma lower
//                      bound of the bin mass, computed with the reference's fp64 operations in its
//                      order, each correctly rounded (no contraction), so the keys are bit-equal.
#include "common.cuh"

namespace atlas {
namespace {

constexpr int kMaxRanks = 32;
constexpr int kSelThreads = 256;

struct Ranks {
  int64_t r[kMaxRanks];
  int n;
};

template <int DT> struct KeyOf;
template <> struct KeyOf<ATLAS_F32> {
  static constexpr int kBits = 32;
  using Raw = uint32_t;
  static __device__ __forceinline__ uint32_t key(uint32_t u) { return (u & 0x80000000u) ? ~u : (u | 0x80000000u); }
  static __device__ __forceinline__ float value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
  }
};
template <> struct KeyOf<ATLAS_BF16> {
  static constexpr int kBits = 16;
  using Raw = uint16_t;
  static __device__ __forceinline__ uint32_t key(uint32_t u) { return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u); }
  static __device__ __forceinline__ float value(uint32_t k) {
    const uint32_t u = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
    return __uint_as_float(u << 16);
  }
};
template <> struct KeyOf<ATLAS_F16> {
  static constexpr int kBits = 16;
  using Raw = uint16_t;
  static __device__ __forceinline__ uint32_t key(uint32_t u) { return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u); }
  static __device__ __forceinline__ float value(uint32_t k) {
    const uint32_t u = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
    return __half2float(__ushort_as_half((unsigned short)u));
  }
};

// One CTA per column d (row d of XT, n elements, contiguous, 16-byte aligned: ldx % 8 == 0).
template <int DT>
__global__ void __launch_bounds__(kSelThreads) column_select_kernel(const void* __restrict__ XT, int64_t ldx,
                                                                    int64_t n, Ranks ranks, float* __restrict__ out) {
  using K = KeyOf<DT>;
  using Raw = typename K::Raw;
  constexpr int kPasses = K::kBits / 8;
  constexpr int kPerVec = 16 / sizeof(Raw);
  __shared__ unsigned int hist[kMaxRanks][256];
  __shared__ uint32_t prefix[kMaxRanks];   // per distinct prefix
  __shared__ uint32_t t_prefix[kMaxRanks];  // per wanted rank: the key bits fixed so far
  __shared__ int64_t t_rem[kMaxRanks];      // rank within the elements sharing t_prefix
  __shared__ int t_slot[kMaxRanks];         // wanted rank -> its distinct-prefix slot
  __shared__ int n_slots;
  const int64_t d = blockIdx.x;
  const Raw* col = reinterpret_cast<const Raw*>(XT) + d * ldx;
  const int R = ranks.n;
  if (threadIdx.x < R) {
    t_prefix[threadIdx.x] = 0;
    t_rem[threadIdx.x] = ranks.r[threadIdx.x];
  }
  const int64_t n_vec = n / kPerVec;
  for (int pass = 0; pass < kPasses; ++pass) {
    const int shift = K::kBits - 8 * (pass + 1);
    __syncthreads();
    if (threadIdx.x == 0) {  // distinct prefixes among the wanted ranks (R <= 32: serial)
      int u = 0;
      for (int t = 0; t < R; ++t) {
        int s = -1;
        for (int j = 0; j < u; ++j)
          if (prefix[j] == t_prefix[t]) s = j;
        if (s < 0) {
          prefix[u] = t_prefix[t];
          s = u++;
        }
        t_slot[t] = s;
      }
      n_slots = u;
    }
    __syncthreads();
    const int U = n_slots;
    for (int i = threadIdx.x; i < U * 256; i += blockDim.x) hist[i >> 8][i & 255] = 0;
    __syncthreads();
    auto visit = [&](uint32_t raw) {
      const uint32_t k = K::key(raw);
      const uint32_t dig = (k >> shift) & 255u;
      if (pass == 0) {
        atomicAdd(&hist[0][dig], 1u);
      } else {
        const uint32_t hi = k >> (shift + 8);
        for (int u = 0; u < U; ++u)
          if (prefix[u] == hi) atomicAdd(&hist[u][dig], 1u);
      }
    };
    const uint4* v4 = reinterpret_cast<const uint4*>(col);
    for (int64_t i = threadIdx.x; i < n_vec; i += blockDim.x) {
      const uint4 w = __ldg(v4 + i);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if constexpr (sizeof(Raw) == 2) {
          visit(ws[q] & 0xFFFFu);
          visit(ws[q] >> 16);
        } else {
          visit(ws[q]);
        }
      }
    }
    for (int64_t i = n_vec * kPerVec + threadIdx.x; i < n; i += blockDim.x) visit((uint32_t)col[i]);
    __syncthreads();
    if (threadIdx.x < R) {  // descend one digit: the bucket holding the wanted rank
      const int t = threadIdx.x;
      const unsigned int* h = hist[t_slot[t]];
      int64_t rem = t_rem[t];
      int dig = 0;
      for (; dig < 255; ++dig) {
        if (rem < (int64_t)h[dig]) break;
        rem -= h[dig];
      }
      t_rem[t] = rem;
      t_prefix[t] = (pass == 0 ? 0u : (t_prefix[t] << 8)) | (uint32_t)dig;
    }
  }
  __syncthreads();
  if (threadIdx.x < R) out[d * R + threadIdx.x] = K::value(t_prefix[threadIdx.x]);
}

__device__ __forceinline__ float next_up(float x) {
  if (x != x) return x;
  const uint32_t u = __float_as_uint(x);
  if (u == 0x7F800000u) return x;                              // +inf stays
  if ((u & 0x7FFFFFFFu) == 0) return __uint_as_float(0x00000001u);  // +-0 -> +min denormal
  return __uint_as_float((u & 0x80000000u) ? u - 1 : u + 1);
}

// sel [D, 2B]: values at ranks r_b (first B) and n-1-r_b (last B) of each column.
__global__ void pilot_edges_kernel(const float* __restrict__ sel, int64_t D, int B, float* __restrict__ E) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * D) return;
  const int p = (int)(i / D);
  const int64_t d = i - (int64_t)p * D;
  float prev = 0.0f;
  for (int b = 0; b < B; ++b) {
    float v = p == 0 ? sel[d * 2 * B + b] : -sel[d * 2 * B + B + b];
    if (b > 0) v = fmaxf(v, next_up(prev));
    E[(p * D + d) * B + b] = v;
    prev = v;
  }
}

__device__ __forceinline__ float as_float(float x) { return x; }
__device__ __forceinline__ float as_float(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float as_float(__half x) { return __half2float(x); }

constexpr int kCntThreads = 128;
constexpr int kMaxBins = 8;

// Thread per column; rows in [chunk_start[y], chunk_start[y+1]) of the visiting order, each chunk
// made of whole group runs (run_last[i] != 0 ends a run). cnt / sumsq: [2, D, B] int64, accumulated.
template <typename T>
__global__ void __launch_bounds__(kCntThreads) pilot_counts_kernel(const T* __restrict__ H, int64_t ld, int64_t D,
                                                                   const int32_t* __restrict__ order,
                                                                   const uint8_t* __restrict__ run_last,
                                                                   const int64_t* __restrict__ chunk_start,
                                                                   const float* __restrict__ E, int B,
                                                                   unsigned long long* __restrict__ cnt,
                                                                   unsigned long long* __restrict__ sumsq) {
  const int64_t d = (int64_t)blockIdx.x * kCntThreads + threadIdx.x;
  if (d >= D) return;
  float e0[kMaxBins], e1[kMaxBins];
#pragma unroll
  for (int b = 0; b < kMaxBins; ++b) {
    e0[b] = b < B ? E[d * B + b] : __int_as_float(0x7F800000);
    e1[b] = b < B ? E[(D + d) * B + b] : __int_as_float(0x7F800000);
  }
  int run[2][kMaxBins] = {};
  unsigned long long c[2][kMaxBins] = {}, q[2][kMaxBins] = {};
  const int64_t i0 = chunk_start[blockIdx.y], i1 = chunk_start[blockIdx.y + 1];
  for (int64_t i = i0; i < i1; ++i) {
    const int64_t row = order ? (int64_t)order[i] : i;
    const float h = as_float(H[row * ld + d]);
    int b0 = -1, b1 = -1;
#pragma unroll
    for (int b = 0; b < kMaxBins; ++b) {
      b0 += (h >= e0[b]) ? 1 : 0;
      b1 += (-h >= e1[b]) ? 1 : 0;
    }
#pragma unroll
    for (int b = 0; b < kMaxBins; ++b) {
      run[0][b] += (b0 == b) ? 1 : 0;
      run[1][b] += (b1 == b) ? 1 : 0;
    }
    if (run_last && run_last[i]) {
#pragma unroll
      for (int p = 0; p < 2; ++p)
#pragma unroll
        for (int b = 0; b < kMaxBins; ++b) {
          const unsigned long long r = (unsigned long long)run[p][b];
          c[p][b] += r;
          q[p][b] += r * r;
          run[p][b] = 0;
        }
    }
  }
#pragma unroll
  for (int p = 0; p < 2; ++p)
#pragma unroll
    for (int b = 0; b < kMaxBins; ++b) {
      if (b >= B) continue;
      const unsigned long long cc = c[p][b] + (unsigned long long)run[p][b];
      if (cc) atomicAdd(cnt + (p * D + d) * B + b, cc);
      if (q[p][b]) atomicAdd(sumsq + (p * D + d) * B + b, q[p][b]);
    }
}

__device__ __forceinline__ float next_down_f(float x) { return next_down(x); }

// One thread per (pole, column): top seed, then the B reservoir key ceilings. sel2 [D, 2]: the
// column's values at ascending ranks n-kk and kk-1 (the kk-th largest of +h and, negated, of -h).
__global__ void pilot_seeds_kernel(const int64_t* __restrict__ cnt, const int64_t* __restrict__ sumsq,
                                   const float* __restrict__ sel2, int64_t D, int B, int64_t n, int64_t Kr,
                                   int64_t n_total, double c, double z, int grouped, float* __restrict__ top_seed,
                                   int64_t* __restrict__ key) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * D) return;
  const int64_t d = i % D;
  top_seed[i] = next_down_f(i < D ? sel2[d * 2] : -sel2[d * 2 + 1]);
  const double two32 = 4294967296.0;
  const double num = __dmul_rn(__dmul_rn(c, (double)Kr), two32);  // c * Kr * 2.0**32, left to right
  const double dn = (double)n, dtot = (double)n_total;
  for (int b = 0; b < B; ++b) {
    const double ct = (double)cnt[i * B + b];
    double m_lo;
    if (!grouped) {  // (cnt - z * sqrt(cnt)).clamp(min=0) / n
      double t = __dsub_rn(ct, __dmul_rn(z, __dsqrt_rn(ct)));
      t = t > 0.0 ? t : 0.0;
      m_lo = __ddiv_rn(t, dn);
    } else {  // n_eff = cnt^2 / max(sum_g c_g^2, 1); m_lo = (cnt / n) * max(1 - z / sqrt(max(n_eff, 1e-9)), 0)
      double s = (double)sumsq[i * B + b];
      s = s > 1.0 ? s : 1.0;
      double ne = __ddiv_rn(__dmul_rn(ct, ct), s);
      ne = ne > 1e-9 ? ne : 1e-9;
      double f = __dsub_rn(1.0, __ddiv_rn(z, __dsqrt_rn(ne)));
      f = f > 0.0 ? f : 0.0;
      m_lo = __dmul_rn(__ddiv_rn(ct, dn), f);
    }
    double theta = m_lo > 0.0 ? __ddiv_rn(num, __dmul_rn(dtot, m_lo)) : two32;
    theta = theta < two32 ? theta : two32;
    key[i * B + b] = (int64_t)floor(theta);
  }
}

template <int DT>
int launch_select(const void* XT, int64_t ldx, int64_t n, int64_t D, const Ranks& r, float* out, cudaStream_t st) {
  column_select_kernel<DT><<<(unsigned)D, kSelThreads, 0, st>>>(XT, ldx, n, r, out);
  return check_launch("column_select");
}

}  // namespace
}  // namespace atlas

using namespace atlas;

extern "C" int atlas_column_select(const void* XT, int dtype, int64_t ldx, int64_t n, int64_t D,
                                   const int64_t* ranks_host, int64_t R, float* out, void* stream) {
  ATLAS_REQUIRE(n >= 1 && D >= 0 && ldx >= n && ldx % 8 == 0, "column_select: need n >= 1, ldx >= n, ldx %% 8 == 0");
  ATLAS_REQUIRE(R >= 1 && R <= kMaxRanks && ranks_host, "column_select: 1..%d ranks", kMaxRanks);
  ATLAS_REQUIRE(D <= 0x7FFFFFFF, "column_select: D too large");
  if (D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(XT && out && ((uintptr_t)XT % 16) == 0, "column_select: XT must be 16-byte aligned");
  Ranks r{};
  r.n = (int)R;
  for (int64_t t = 0; t < R; ++t) {
    ATLAS_REQUIRE(ranks_host[t] >= 0 && ranks_host[t] < n, "column_select: rank %lld outside [0, %lld)",
                  (long long)ranks_host[t], (long long)n);
    r.r[t] = ranks_host[t];
  }
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case ATLAS_F32: return launch_select<ATLAS_F32>(XT, ldx, n, D, r, out, st);
    case ATLAS_BF16: return launch_select<ATLAS_BF16>(XT, ldx, n, D, r, out, st);
    case ATLAS_F16: return launch_select<ATLAS_F16>(XT, ldx, n, D, r, out, st);
    default: return fail(ATLAS_ERR_ARG, "column_select: unknown dtype %d", dtype);
  }
}

extern "C" int atlas_pilot_edges(const float* sel, int64_t D, int64_t B, float* E, void* stream) {
  ATLAS_REQUIRE(D >= 0 && B >= 1 && B <= 16, "pilot_edges: B must be 1..16");
  if (D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(sel && E, "pilot_edges: null pointer");
  const int64_t work = 2 * D;
  pilot_edges_kernel<<<(unsigned)((work + 255) / 256), 256, 0, (cudaStream_t)stream>>>(sel, D, (int)B, E);
  return check_launch("pilot_edges");
}

extern "C" int atlas_pilot_counts(const void* H, int dtype, int64_t ld, int64_t n, int64_t D, const int32_t* order,
                                  const uint8_t* run_last, const int64_t* chunk_start, int64_t n_chunks,
                                  const float* E, int64_t B, int64_t* cnt, int64_t* sumsq, void* stream) {
  ATLAS_REQUIRE(n >= 0 && D >= 0 && ld >= D, "pilot_counts: bad sizes");
  ATLAS_REQUIRE(B >= 1 && B <= kMaxBins, "pilot_counts: B must be 1..%d", kMaxBins);
  ATLAS_REQUIRE(n_chunks >= 1 && n_chunks <= 65535, "pilot_counts: 1..65535 chunks");
  if (n == 0 || D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(H && chunk_start && E && cnt && sumsq, "pilot_counts: null pointer");
  dim3 grid((unsigned)((D + kCntThreads - 1) / kCntThreads), (unsigned)n_chunks);
  cudaStream_t st = (cudaStream_t)stream;
  auto* c = reinterpret_cast<unsigned long long*>(cnt);
  auto* q = reinterpret_cast<unsigned long long*>(sumsq);
  switch (dtype) {
    case ATLAS_F32:
      pilot_counts_kernel<float><<<grid, kCntThreads, 0, st>>>((const float*)H, ld, D, order, run_last, chunk_start, E,
                                                               (int)B, c, q);
      break;
    case ATLAS_BF16:
      pilot_counts_kernel<__nv_bfloat16><<<grid, kCntThreads, 0, st>>>((const __nv_bfloat16*)H, ld, D, order, run_last,
                                                                       chunk_start, E, (int)B, c, q);
      break;
    case ATLAS_F16:
      pilot_counts_kernel<__half><<<grid, kCntThreads, 0, st>>>((const __half*)H, ld, D, order, run_last, chunk_start, E,
                                                                (int)B, c, q);
      break;
    default: return fail(ATLAS_ERR_ARG, "pilot_counts: unknown dtype %d", dtype);
  }
  return check_launch("pilot_counts");
}

extern "C" int atlas_pilot_seeds(const int64_t* cnt, const int64_t* sumsq, const float* sel2, int64_t D, int64_t B,
                                 int64_t n, int64_t Kr, int64_t n_total, double c, double z, int grouped,
                                 float* top_seed, int64_t* res_seed_key, void* stream) {
  ATLAS_REQUIRE(D >= 0 && B >= 1 && B <= kMaxBins && n >= 1 && Kr >= 1 && n_total >= 1, "pilot_seeds: bad sizes");
  if (D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(cnt && sel2 && top_seed && res_seed_key && (sumsq || !grouped), "pilot_seeds: null pointer");
  const int64_t work = 2 * D;
  pilot_seeds_kernel<<<(unsigned)((work + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      cnt, sumsq, sel2, D, (int)B, n, Kr, n_total, c, z, grouped, top_seed, res_seed_key);
  return check_launch("pilot_seeds");
}
