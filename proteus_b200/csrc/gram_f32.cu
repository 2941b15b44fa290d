// Gram for fp32 activations: exact fp32 FMA on CUDA cores (tcgen05 has no IEEE-fp32 operand kind;
// TF32 would round the products). Same contract as the tensor-core Gram: upper 128-blocks of
// C += X^T X from the transposed staging, two-level fp32 accumulation over 1024-row segments.
#include "common.cuh"

namespace atlas {
namespace {

constexpr int kGT = 64;
constexpr int kGK = 16;
constexpr int kSegment = 1024;

__global__ void __launch_bounds__(256)
gram_f32_kernel(const float* __restrict__ XT, int64_t ldx, int64_t n, int64_t D, float* __restrict__ C) {
  const int ti = blockIdx.y, tj = blockIdx.x;
  if ((ti * kGT) / 128 > (tj * kGT) / 128) return;  // lower 128-block: untouched
  __shared__ float As[kGK][kGT + 1], Bs[kGK][kGT + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {}, tot[4][4] = {};
  const int64_t i0 = (int64_t)ti * kGT, j0 = (int64_t)tj * kGT;
  for (int64_t k0 = 0; k0 < n; k0 += kGK) {
    if (k0 % kSegment == 0 && k0 > 0) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          tot[u][v] += acc[u][v];
          acc[u][v] = 0.f;
        }
    }
    for (int e = threadIdx.x; e < kGK * kGT; e += 256) {
      const int r = e / kGK, k = e % kGK;
      const int64_t kk = k0 + k;
      As[k][r] = (i0 + r < D && kk < n) ? XT[(i0 + r) * ldx + kk] : 0.f;
      Bs[k][r] = (j0 + r < D && kk < n) ? XT[(j0 + r) * ldx + kk] : 0.f;
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

}  // namespace

int gram_upper_f32(const float* XT, int64_t ldx, int64_t n, int64_t D, float* C, cudaStream_t st) {
  const int64_t nt = (D + kGT - 1) / kGT;
  ATLAS_REQUIRE(nt < 65536, "gram_upper: D too large");
  dim3 grid((unsigned)nt, (unsigned)nt);
  gram_f32_kernel<<<grid, 256, 0, st>>>(XT, ldx, n, D, C);
  return check_launch("atlas_gram_upper (fp32)");
}

}  // namespace atlas
