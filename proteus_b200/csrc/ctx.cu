// Batch context on the device: the row-level decisions of Atlas.make_ctx (atlas/core.py:210-237)
// from the batch's valid rows and token ids.
//
// atlas_ctx_rows        key = lowbias32((tok ^ seed) mod 2^32) per valid row; the row map (row of H
//                       -> valid index, -1 for padding); the hashed subsample (key < U_sub) and,
//                       inside it, the bulk reservoir rows (key < U_res), both in increasing valid
//                       index order as torch.nonzero gives them; the valid indices ordered by key
//                       (keys are distinct: the hash is a bijection of distinct token ids) by a
//                       bucket sort on the high key bits and an insertion sort per bucket; counts
//                       n_s, n_r in `counts`.
// atlas_ctx_annotations the subsample's annotation one-hots transposed, annT[a, j] = 1 when class a
//                       is among the ids of subsample row j (padding to n_pad zero), and their
//                       per-class totals (ann_tot increments), as ann_sub / ann_sub_i8 of the
//                       reference's make_ctx.
#include "common.cuh"

namespace atlas {
namespace {

constexpr int kScanThreads = 1024;

__global__ void ctx_keys_kernel(const int64_t* __restrict__ valid_rows, const int64_t* __restrict__ tok, int64_t n_v,
                                uint32_t seed, int64_t T, int64_t* __restrict__ key, int32_t* __restrict__ rowmap,
                                int shift, unsigned int* __restrict__ bucket_count, int32_t* __restrict__ err) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_v; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = tok[i];
    const int64_t r = valid_rows[i];
    if (t < 0 || t > (int64_t)kM32 || r < 0 || r >= T) {
      atomicExch(err, 1);  // token ids must be in [0, 2^32) and rows inside the batch
      continue;
    }
    const uint32_t k = lowbias32((uint32_t)t ^ seed);
    key[i] = (int64_t)k;
    rowmap[r] = (int32_t)i;
    atomicAdd(bucket_count + (k >> shift), 1u);
  }
}

// Block-wide exclusive scan of one int per thread (kScanThreads threads); returns the prefix and
// writes the block total to *total.
__device__ __forceinline__ int block_excl_scan(int v, int* sh, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int tot;
  const int pre = warp_excl_scan(v, lane, &tot);
  if (lane == 31 || lane == (int)blockDim.x - 1) sh[w] = tot;
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    int x = lane < nw ? sh[lane] : 0, t2;
    const int p = warp_excl_scan(x, lane, &t2);
    if (lane < nw) sh[lane] = p;
    if (lane == 0) sh[32] = t2;
  }
  __syncthreads();
  const int out = pre + sh[w];
  *total = sh[32];
  __syncthreads();
  return out;
}

// One CTA: ordered compaction of the subsample and the bulk rows, and the bucket offsets.
__global__ void __launch_bounds__(kScanThreads) ctx_compact_kernel(
    const int64_t* __restrict__ valid_rows, const int64_t* __restrict__ key, int64_t n_v, int64_t U_sub,
    int64_t U_res, int64_t* __restrict__ sub_idx, int64_t* __restrict__ res_in_sub, int32_t* __restrict__ sub_rows32,
    int32_t* __restrict__ res_rows32, int32_t* __restrict__ res_vidx32, const unsigned int* __restrict__ bucket_count,
    unsigned int* __restrict__ bucket_start, int n_buckets, int64_t* __restrict__ counts) {
  __shared__ int sh[33];
  int base_s = 0, base_r = 0;
  for (int64_t t0 = 0; t0 < n_v; t0 += kScanThreads) {
    const int64_t i = t0 + threadIdx.x;
    const int64_t k = i < n_v ? key[i] : INT64_MAX;
    const int fs = k < U_sub ? 1 : 0;
    const int fr = k < U_res ? 1 : 0;  // U_res <= U_sub: bulk rows are subsample rows
    int ts, tr;
    const int ps = block_excl_scan(fs, sh, &ts);
    const int pr = block_excl_scan(fr, sh, &tr);
    if (fs) {
      const int64_t j = base_s + ps;
      const int32_t row = (int32_t)valid_rows[i];
      sub_idx[j] = i;
      sub_rows32[j] = row;
      if (fr) {
        const int64_t q = base_r + pr;
        res_in_sub[q] = j;
        res_rows32[q] = row;
        res_vidx32[q] = (int32_t)i;
      }
    }
    base_s += ts;
    base_r += tr;
  }
  // exclusive offsets of the key buckets
  int carry = 0;
  for (int b0 = 0; b0 < n_buckets; b0 += kScanThreads) {
    const int b = b0 + threadIdx.x;
    const int v = b < n_buckets ? (int)bucket_count[b] : 0;
    int tot;
    const int p = block_excl_scan(v, sh, &tot);
    if (b < n_buckets) bucket_start[b] = (unsigned int)(carry + p);
    carry += tot;
  }
  if (threadIdx.x == 0) {
    bucket_start[n_buckets] = (unsigned int)carry;
    counts[0] = base_s;
    counts[1] = base_r;
  }
}

__global__ void ctx_scatter_kernel(const int64_t* __restrict__ key, int64_t n_v, int shift,
                                   const unsigned int* __restrict__ bucket_start, unsigned int* __restrict__ fill,
                                   uint32_t* __restrict__ skey, int32_t* __restrict__ sidx) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_v; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t k = (uint32_t)key[i];
    const unsigned int b = k >> shift;
    const unsigned int slot = bucket_start[b] + atomicAdd(fill + b, 1u);
    skey[slot] = k;
    sidx[slot] = (int32_t)i;
  }
}

// One thread per bucket: insertion sort of its (key, index) pairs by key, then the indices out.
__global__ void ctx_bucket_sort_kernel(const unsigned int* __restrict__ bucket_start, int n_buckets,
                                       uint32_t* __restrict__ skey, int32_t* __restrict__ sidx,
                                       int32_t* __restrict__ key_order) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n_buckets) return;
  const unsigned int s0 = bucket_start[b], s1 = bucket_start[b + 1];
  for (unsigned int a = s0 + 1; a < s1; ++a) {
    const uint32_t k = skey[a];
    const int32_t v = sidx[a];
    unsigned int c = a;
    while (c > s0 && skey[c - 1] > k) {
      skey[c] = skey[c - 1];
      sidx[c] = sidx[c - 1];
      --c;
    }
    skey[c] = k;
    sidx[c] = v;
  }
  for (unsigned int a = s0; a < s1; ++a) key_order[a] = sidx[a];
}

__global__ void ctx_annot_kernel(const int64_t* __restrict__ sub_idx, const int64_t* __restrict__ counts,
                                 const int64_t* __restrict__ ann, int64_t m_a, int64_t n_a, int8_t* __restrict__ annT,
                                 int64_t n_pad) {
  const int64_t n_s = counts[0];
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_s * m_a; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = e / m_a, m = e - j * m_a;
    const int64_t a = ann[sub_idx[j] * m_a + m];
    if (a >= 0 && a < n_a && j < n_pad) annT[a * n_pad + j] = 1;  // a class listed twice sets the same byte
  }
}

// One CTA per class: its total over the subsample rows (a row counts once per class).
__global__ void ctx_annot_totals_kernel(const int8_t* __restrict__ annT, int64_t n_pad, int64_t* __restrict__ tot) {
  const int64_t a = blockIdx.x;
  int c = 0;
  for (int64_t j = threadIdx.x; j < n_pad; j += blockDim.x) c += annT[a * n_pad + j];
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
  __shared__ int ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += ws[w];
    tot[a] = s;
  }
}

int bucket_bits(int64_t n_v) {
  int bits = 8;
  while (bits < 16 && (int64_t(1) << bits) * 8 < n_v) ++bits;
  return bits;
}

}  // namespace
}  // namespace atlas

using namespace atlas;

extern "C" int64_t atlas_ctx_ws_bytes(int64_t n_v) {
  const int64_t nb = int64_t(1) << bucket_bits(n_v < 1 ? 1 : n_v);
  return (nb * 3 + 1) * 4 + (n_v < 1 ? 1 : n_v) * 8 + 256;
}

extern "C" int atlas_ctx_rows(const int64_t* valid_rows, const int64_t* tok, int64_t n_v, int64_t T, int64_t seed,
                              int64_t U_sub, int64_t U_res, int64_t* key, int32_t* rowmap, int64_t* sub_idx,
                              int64_t* res_in_sub, int32_t* sub_rows32, int32_t* res_rows32, int32_t* res_vidx32,
                              int32_t* key_order, int64_t* counts, int32_t* err, void* ws, int64_t ws_bytes,
                              void* stream) {
  ATLAS_REQUIRE(n_v >= 0 && T >= n_v && n_v < (1LL << 31) && T < (1LL << 31), "ctx_rows: bad sizes");
  ATLAS_REQUIRE(U_res >= 0 && U_res <= U_sub && U_sub <= (1LL << 32), "ctx_rows: need 0 <= U_res <= U_sub <= 2^32");
  ATLAS_REQUIRE(rowmap && counts && err && ws, "ctx_rows: null pointer");
  ATLAS_REQUIRE(ws_bytes >= atlas_ctx_ws_bytes(n_v), "ctx_rows: workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(rowmap, 0xFF, (size_t)T * 4, st) != cudaSuccess) return fail(ATLAS_ERR_CUDA, "ctx_rows: memset");
  if (n_v == 0) {
    if (cudaMemsetAsync(counts, 0, 16, st) != cudaSuccess) return fail(ATLAS_ERR_CUDA, "ctx_rows: memset");
    return ATLAS_OK;
  }
  ATLAS_REQUIRE(valid_rows && tok && key && sub_idx && res_in_sub && sub_rows32 && res_rows32 && res_vidx32 && key_order,
                "ctx_rows: null pointer");
  const int bits = bucket_bits(n_v);
  const int nb = 1 << bits, shift = 32 - bits;
  auto* cnt = reinterpret_cast<unsigned int*>(ws);
  unsigned int* start = cnt + nb;        // nb + 1 entries
  unsigned int* fill = start + nb + 1;   // nb entries
  auto* skey = reinterpret_cast<uint32_t*>(fill + nb);
  int32_t* sidx = reinterpret_cast<int32_t*>(skey + n_v);
  if (cudaMemsetAsync(cnt, 0, (size_t)nb * 4, st) != cudaSuccess ||
      cudaMemsetAsync(fill, 0, (size_t)nb * 4, st) != cudaSuccess)
    return fail(ATLAS_ERR_CUDA, "ctx_rows: memset");
  const unsigned grid = grid_for(n_v, 256, 4);
  ctx_keys_kernel<<<grid, 256, 0, st>>>(valid_rows, tok, n_v, (uint32_t)(seed & kM32), T, key, rowmap, shift, cnt, err);
  ctx_compact_kernel<<<1, kScanThreads, 0, st>>>(valid_rows, key, n_v, U_sub, U_res, sub_idx, res_in_sub, sub_rows32,
                                                 res_rows32, res_vidx32, cnt, start, nb, counts);
  ctx_scatter_kernel<<<grid, 256, 0, st>>>(key, n_v, shift, start, fill, skey, sidx);
  ctx_bucket_sort_kernel<<<(nb + 127) / 128, 128, 0, st>>>(start, nb, skey, sidx, key_order);
  return check_launch("ctx_rows");
}

extern "C" int atlas_ctx_annotations(const int64_t* sub_idx, const int64_t* counts, const int64_t* ann, int64_t n_v,
                                     int64_t m_a, int64_t n_a, int8_t* annT, int64_t A_pad, int64_t n_pad,
                                     int64_t* ann_totals, void* stream) {
  ATLAS_REQUIRE(n_a >= 1 && A_pad >= n_a && n_pad >= 1 && m_a >= 1, "ctx_annotations: bad sizes");
  ATLAS_REQUIRE(sub_idx && counts && ann && annT && ann_totals, "ctx_annotations: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(annT, 0, (size_t)(A_pad * n_pad), st) != cudaSuccess)
    return fail(ATLAS_ERR_CUDA, "ctx_annotations: memset");
  const unsigned grid = grid_for(n_v * m_a, 256, 4);
  ctx_annot_kernel<<<grid, 256, 0, st>>>(sub_idx, counts, ann, m_a, n_a, annT, n_pad);
  ctx_annot_totals_kernel<<<(unsigned)n_a, 256, 0, st>>>(annT, n_pad, ann_totals);
  return check_launch("ctx_annotations");
}
