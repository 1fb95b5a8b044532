// common.cuh — shared device helpers for the Krystal B200 kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define KC_H 128          // hidden size the kernels are built for
#define KC_HEADS 4
#define KC_HEAD_DIM 32
#define KC_RW 8           // record width
#define KC_QUERY_BAND_ID 5u
#define KC_INVALID 0xffffffffu

namespace kc {

// Math.max(a, b) of JavaScript: NaN if either is NaN, +0 beats -0.
__device__ __forceinline__ double js_max(double a, double b) {
  if (a != a || b != b) return __longlong_as_double(0x7ff8000000000000ll);
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}

// reluOracle's Math.max(0, v) on a stored f32 value.
__device__ __forceinline__ float js_relu(float v) {
  if (v != v) return v;
  return v > 0.0f ? v : 0.0f;
}

__device__ __forceinline__ float f32(double v) { return __double2float_rn(v); }
__device__ __forceinline__ float f32(float v) { return v; }

// The record mask's entry for two tokens of one record (compileRecordMask,
// masks.ts:167-198): alpha when both carry the same valid word id, else 0.
__device__ __forceinline__ float word_bias(uint32_t wi, uint32_t wj, float alpha) {
  return (alpha != 0.0f && wi != KC_INVALID && wi == wj) ? alpha : 0.0f;
}

// Exclusive block scan of one value per thread (NT threads, NT % 32 == 0).
// `tmp` holds NT/32 entries. Returns the exclusive prefix; *total gets the sum.
template <int NT, typename T>
__device__ __forceinline__ T block_excl_scan(T v, T* total, T* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    T s = lane < NT / 32 ? tmp[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      T y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < NT / 32) tmp[lane] = s;
  }
  __syncthreads();
  const T prefix = warp ? tmp[warp - 1] : T(0);
  *total = tmp[NT / 32 - 1];
  __syncthreads();
  return prefix + x - v;
}

// One 16-byte asynchronous global -> shared copy (cp.async.wait_all before use).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
               ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src) : "memory");
}

}  // namespace kc
