// Shared device helpers for the stage kernels.
//
// Every kernel in this library computes in fp32 and rounds to the activation
// dtype at exactly the points where the PyTorch stage rounds (each PyTorch op
// on a bf16 tensor returns a bf16 tensor).  `rt<T>(x)` is that rounding step:
// identity for fp32 models, round-to-nearest-even to bf16 for bf16 models.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mg {

enum DType : int { kF32 = 0, kBF16 = 1 };

template <typename T>
struct Num;

template <>
struct Num<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
  static __device__ __forceinline__ float round(float x) { return x; }
};

template <>
struct Num<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};

template <typename T>
__device__ __forceinline__ float rt(float x) { return Num<T>::round(x); }
template <typename T>
__device__ __forceinline__ float ldf(const T* p) { return Num<T>::to_f(*p); }
template <typename T>
__device__ __forceinline__ void stf(T* p, float x) { *p = Num<T>::from_f(x); }

// Number of elements of T in one 16-byte vector.
template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

// Load 16 bytes (8 bf16 or 4 f32) and widen to fp32.
template <typename T>
__device__ __forceinline__ void load16_f(const T* p, float* out);

template <>
__device__ __forceinline__ void load16_f<float>(const float* p, float* out) {
  float4 v = *reinterpret_cast<const float4*>(p);
  out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
}

template <>
__device__ __forceinline__ void load16_f<__nv_bfloat16>(const __nv_bfloat16* p, float* out) {
  uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Round 16 bytes' worth of floats to T (8 bf16 or 4 f32) and store them at once.
template <typename T>
__device__ __forceinline__ void store16_f(T* p, const float* v) {
  if constexpr (sizeof(T) == 2) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i])) |
             ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i + 1])) << 16);
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Device-side error word shared by all kernels of one stage.  Kernels never
// trap: an out-of-range token id or position is clamped, the offending value
// is recorded here, and the host reads the word at its next check.
enum DeviceError : int {
  kErrNone = 0,
  kErrTokenRange = 1,
  kErrPositionRange = 2,
};

__device__ __forceinline__ void flag_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Programmatic dependent launch.  Every kernel of the stage is launched with
// programmatic stream serialisation, so it may start while the kernel before
// it in the stream is still running.  pdl_wait() blocks until that kernel has
// completed and its writes are visible: call it before reading anything the
// previous kernel produced and before writing anything it might still read.
// pdl_trigger() lets the next kernel launch early; its own pdl_wait() keeps it
// correct.  Both are no-ops when there is no programmatic dependency.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Histogram bin of a logit (top-p by value histogram): the order-preserving
// 16-bit key of its bf16 value, -0 counted as +0 so equal values share a bin.
__device__ __forceinline__ uint32_t hist_bin(float v) {
  uint32_t u = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  if ((u & 0x7fffu) == 0u) u = 0u;
  return (u & 0x8000u) ? (~u & 0xffffu) : (u | 0x8000u);
}

// The bf16 value of histogram bin `b` (the inverse of hist_bin).
__device__ __forceinline__ float hist_value(uint32_t b) {
  const uint32_t u = (b & 0x8000u) ? (b & 0x7fffu) : (~b & 0xffffu);
  return __uint_as_float(u << 16);
}

// Streaming multiprocessors a persistent kernel spreads over on the current
// device: the device's count minus the SMs left free for concurrent work
// (NCCL's kernels in a multi-process pipeline; mg_reserve_sms).  Host code.
int usable_sms();

}  // namespace mg
