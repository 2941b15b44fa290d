// Interim CUDA-core versions of the two contractions (upper-block Gram, exact int8 contingency
// counts). They fix the semantics that the tcgen05 kernels must reproduce.
#include "common.cuh"

namespace atlas {
namespace {

constexpr int kGT = 64;   // output tile
constexpr int kGK = 16;   // k step
constexpr int kSegment = 1024;  // rows summed in one fp32 accumulator before folding into the total

template <int DT>
__global__ void __launch_bounds__(256)
gram_simt_kernel(const typename Elem<DT>::T* __restrict__ XT, int64_t ldx, int64_t n, int64_t D, float* __restrict__ C) {
  const int ti = blockIdx.y, tj = blockIdx.x;
  if ((ti * kGT) / 128 > (tj * kGT) / 128) return;  // lower 128-block: untouched
  __shared__ float As[kGK][kGT + 1], Bs[kGK][kGT + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {}, tot[4][4] = {};
  const int64_t i0 = (int64_t)ti * kGT, j0 = (int64_t)tj * kGT;
  for (int64_t k0 = 0; k0 < n; k0 += kGK) {
    if (k0 % kSegment == 0 && k0 > 0) {  // two-level fp32 accumulation: segments of kSegment rows
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) { tot[u][v] += acc[u][v]; acc[u][v] = 0.f; }
    }
    for (int e = threadIdx.x; e < kGK * kGT; e += 256) {
      const int r = e / kGK, k = e % kGK;  // consecutive threads walk k (contiguous in XT)
      const int64_t kk = k0 + k;
      As[k][r] = (i0 + r < D && kk < n) ? Elem<DT>::f(XT[(i0 + r) * ldx + kk]) : 0.f;
      Bs[k][r] = (j0 + r < D && kk < n) ? Elem<DT>::f(XT[(j0 + r) * ldx + kk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kGK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a[u] = As[k][ty * 4 + u];
        b[u] = Bs[k][tx * 4 + u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(a[u], b[v], acc[u][v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int64_t i = i0 + ty * 4 + u, j = j0 + tx * 4 + v;
      if (i < D && j < D) C[i * D + j] += tot[u][v] + acc[u][v];
    }
}

constexpr int kIM = 32;    // rows of masks per block
constexpr int kIK = 128;   // bytes of k per step

__global__ void __launch_bounds__(256)
count_i8_simt_kernel(const int8_t* __restrict__ M, int64_t Mrows, int64_t n_pad, const int8_t* __restrict__ annT,
                     int64_t A_pad, int64_t* __restrict__ out, int64_t A) {
  extern __shared__ int smem_i[];
  int* Ms = smem_i;                        // [kIM][kIK/4 + 1]
  int* As = smem_i + kIM * (kIK / 4 + 1);  // [A_pad][kIK/4 + 1]
  const int W = kIK / 4 + 1;
  const int64_t m0 = (int64_t)blockIdx.x * kIM;
  const int tm = threadIdx.x & 31, ta = threadIdx.x >> 5;  // 8 column groups
  int acc[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i] = 0;
  for (int64_t k0 = 0; k0 < n_pad; k0 += kIK) {
    for (int e = threadIdx.x; e < kIM * (kIK / 4); e += 256) {
      const int r = e / (kIK / 4), w = e % (kIK / 4);
      Ms[r * W + w] = (m0 + r < Mrows) ? *reinterpret_cast<const int*>(M + (m0 + r) * n_pad + k0 + 4 * w) : 0;
    }
    for (int e = threadIdx.x; e < A_pad * (kIK / 4); e += 256) {
      const int r = e / (kIK / 4), w = e % (kIK / 4);
      As[r * W + w] = *reinterpret_cast<const int*>(annT + (int64_t)r * n_pad + k0 + 4 * w);
    }
    __syncthreads();
    for (int w = 0; w < kIK / 4; ++w) {
      const int mv = Ms[tm * W + w];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int a = ta + 8 * i;
        if (a < A_pad) acc[i] = __dp4a(mv, As[a * W + w], acc[i]);
      }
    }
    __syncthreads();
  }
  if (m0 + tm < Mrows) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int a = ta + 8 * i;
      if (a < A) out[(m0 + tm) * A + a] += (int64_t)acc[i];
    }
  }
}

}  // namespace
}  // namespace atlas

using namespace atlas;

extern "C" int atlas_gram_upper(const void* XT, int dtype, int64_t ldx, int64_t n, int64_t D, float* C, void* stream) {
  ATLAS_REQUIRE(n >= 0 && D >= 0 && ldx >= n, "gram_upper: bad sizes");
  if (n == 0 || D == 0) return ATLAS_OK;
  ATLAS_REQUIRE(XT && C, "gram_upper: null pointer");
  const int64_t nt = (D + kGT - 1) / kGT;
  ATLAS_REQUIRE(nt < 65536, "gram_upper: D too large");
  dim3 grid((unsigned)nt, (unsigned)nt);
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case ATLAS_BF16: gram_simt_kernel<ATLAS_BF16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)XT, ldx, n, D, C); break;
    case ATLAS_F16: gram_simt_kernel<ATLAS_F16><<<grid, 256, 0, st>>>((const __half*)XT, ldx, n, D, C); break;
    case ATLAS_F32: gram_simt_kernel<ATLAS_F32><<<grid, 256, 0, st>>>((const float*)XT, ldx, n, D, C); break;
    default: return fail(ATLAS_ERR_ARG, "gram_upper: unknown dtype %d", dtype);
  }
  return check_launch("atlas_gram_upper");
}

extern "C" int atlas_count_gemm_i8(const int8_t* masks, int64_t M, int64_t n_pad, const int8_t* annT, int64_t A_pad,
                                   int64_t* out, int64_t A, void* stream) {
  ATLAS_REQUIRE(M >= 0 && n_pad >= 0 && n_pad % kIK == 0, "count_gemm_i8: n_pad must be a multiple of %d", kIK);
  ATLAS_REQUIRE(A_pad % 16 == 0 && A_pad >= 16 && A_pad <= 256 && A >= 0 && A <= A_pad, "count_gemm_i8: bad A/A_pad");
  if (M == 0 || n_pad == 0 || A == 0) return ATLAS_OK;
  ATLAS_REQUIRE(masks && annT && out, "count_gemm_i8: null pointer");
  const size_t smem = sizeof(int) * (size_t)(kIM + A_pad) * (kIK / 4 + 1);
  if (cudaFuncSetAttribute(count_i8_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return fail(ATLAS_ERR_CUDA, "count_gemm_i8: cannot reserve shared memory");
  count_i8_simt_kernel<<<(unsigned)((M + kIM - 1) / kIM), 256, smem, (cudaStream_t)stream>>>(masks, M, n_pad, annT, A_pad,
                                                                                             out, A);
  return check_launch("atlas_count_gemm_i8");
}
