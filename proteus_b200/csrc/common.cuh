// Shared device helpers for the streaming-atlas kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>
#include <stdio.h>

#include "proteus_atlas.h"

namespace atlas {

constexpr int64_t kI64Min = (int64_t)0x8000000000000000ULL;
constexpr int64_t kI64Max = (int64_t)0x7FFFFFFFFFFFFFFFULL;
constexpr uint32_t kM32 = 0xFFFFFFFFu;

// ------------------------------------------------------------------ host-side error reporting
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);

#define ATLAS_REQUIRE(cond, ...)                                                   \
  do {                                                                             \
    if (!(cond)) return ::atlas::fail(ATLAS_ERR_ARG, __VA_ARGS__);                 \
  } while (0)

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

inline unsigned grid_for(int64_t work, int threads, int max_blocks_per_sm = 8) {
  int64_t b = (work + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * max_blocks_per_sm;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (unsigned)b;
}

// ------------------------------------------------------------------ element loads
template <int DT> struct Elem;
template <> struct Elem<ATLAS_F32> {
  using T = float;
  static __device__ __forceinline__ float f(T x) { return x; }
};
template <> struct Elem<ATLAS_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float f(T x) { return __bfloat162float(x); }
};
template <> struct Elem<ATLAS_F16> {
  using T = __half;
  static __device__ __forceinline__ float f(T x) { return __half2float(x); }
};

__device__ __forceinline__ float bf16_bits_to_float(uint32_t b16) { return __uint_as_float(b16 << 16); }

// ------------------------------------------------------------------ keys
// Order-preserving fp32 -> signed int as the reference builds it: bits of (s + 0.0), negatives with
// their 31 low bits flipped (core.py:66-71). Returned widened to int64 (range [-2^31, 2^31)).
__device__ __forceinline__ int64_t ordered_f32(float s) {
  if (s == 0.0f) s = 0.0f;  // -0.0 -> +0.0, as the reference's (s + 0.0)
  int32_t i = __float_as_int(s);
  if (i < 0) i ^= 0x7FFFFFFF;
  return (int64_t)i;
}

// top_key(s, tok) = ordered(s) * 2^32 + (2^32 - 1 - tok)   (core.py:66-71)
__device__ __forceinline__ int64_t top_key(float s, int64_t tok) {
  return ordered_f32(s) * 4294967296LL + ((int64_t)kM32 - tok);
}

// Recover (s, tok) from a top key: exact inverse of top_key for canonical s (never -0.0).
__device__ __forceinline__ float top_key_value(int64_t k) {
  int32_t i = (int32_t)(k >> 32);
  if (i < 0) i ^= 0x7FFFFFFF;
  return __int_as_float(i);
}

// Wellons lowbias32 of (tok ^ seed) & 0xFFFFFFFF (core.py:46-55): exact in uint32 arithmetic.
__device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  x ^= x >> 16;
  return x;
}

// nextafter(x, -inf) for fp32 by bit arithmetic (torch.nextafter semantics; denormals kept).
__device__ __forceinline__ float next_down(float x) {
  if (x != x) return x;                                  // NaN
  uint32_t u = __float_as_uint(x);
  if (u == 0xFF800000u) return x;                        // -inf stays
  if ((u & 0x7FFFFFFFu) == 0) return __uint_as_float(0x80000001u);  // +-0 -> -min denormal
  return __uint_as_float((u & 0x80000000u) ? u + 1 : u - 1);
}

// bin(s) = #{b : s >= E_b} - 1 over the B edges of one (layer, pole, column) (core.py:107-109).
__device__ __forceinline__ int bin_of(float s, const float* __restrict__ E, int B) {
  int c = 0;
  for (int b = 0; b < B; ++b) c += (s >= __ldg(E + b)) ? 1 : 0;
  return c - 1;
}

// ------------------------------------------------------------------ warp helpers
__device__ __forceinline__ int warp_excl_scan(int v, int lane, int* total) {
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  *total = __shfl_sync(0xFFFFFFFFu, x, 31);
  return x - v;
}

}  // namespace atlas
