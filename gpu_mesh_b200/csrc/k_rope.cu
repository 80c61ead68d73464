// QKV post-processing: per-head QK-norm (Qwen3), rotary embedding, and the
// in-place KV-cache append.
//
// The reference grows its cache with torch.cat every step
// (models/llama_dense.py:166-170), copying all past K/V.  Here the slot is
// preallocated and each forward writes only its new positions.  RoPE follows
// _apply_rope (llama_dense.py:112-125) with tables already cast to the
// activation dtype (:431-432): y = round(round(x*cos) + round(rotate_half(x)*sin)).
// QK-norm follows HF Qwen3Attention (q_norm/k_norm over head_dim before RoPE).
#include "common.cuh"
#include "kernels.h"

namespace mg {
namespace {

constexpr int kHeadsPerCta = 4;

template <typename T>
__global__ void __launch_bounds__(kHeadsPerCta * 32) qkv_post_kernel(QkvPostArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ float xs[kHeadsPerCta][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x;
  const int hh = blockIdx.y * kHeadsPerCta + warp;
  const int nh = a.nq + 2 * a.nkv;
  if (hh >= nh) return;
  const int D = a.D, half = D / 2;
  const int b = m / a.S, s = m % a.S;
  const RowDesc rd = a.rows[b];
  const int cache_pos = rd.past + s;
  int64_t pos = a.positions ? a.positions[m] : (int64_t)cache_pos;
  if (pos < 0 || pos >= a.max_pos) {
    flag_error(a.err, kErrPositionRange);
    pos = pos < 0 ? 0 : a.max_pos - 1;
  }

  float* x = xs[warp];
  if (a.use_pieces) {  // the projection's pieces, rounded as its store epilogue would
    for (int d = lane * 4; d < D; d += 128) {
      float acc[4];
      pieces_sum4(a.pieces, m, hh * D + d, acc);
#pragma unroll
      for (int i = 0; i < 4; ++i) x[d + i] = rt<T>(acc[i]);
    }
  } else {
    const T* src = (const T*)a.qkv + (size_t)m * nh * D + (size_t)hh * D;
    for (int d = lane; d < D; d += 32) x[d] = ldf<T>(src + d);
  }
  __syncwarp();

  const bool is_q = hh < a.nq;
  const bool is_k = !is_q && hh < a.nq + a.nkv;
  T* kv = (T*)rd.kv_base;

  if (!is_q && !is_k) {  // value head: plain append
    const int h = hh - a.nq - a.nkv;
    T* dst = kv + kv_offset_elems(a.layer, 1, rd.slot_rows, rd.row, a.nkv, h, rd.cap, D, cache_pos);
    for (int d = lane; d < D; d += 32) stf<T>(dst + d, x[d]);
    return;
  }

  const T* nw = is_q ? (const T*)a.q_norm : (const T*)a.k_norm;
  if (nw) {
    float ss = 0.f;
    for (int d = lane; d < D; d += 32) ss += x[d] * x[d];
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)D + a.eps);
    __syncwarp();
    for (int d = lane; d < D; d += 32) x[d] = rt<T>(rt<T>(x[d] * r) * ldf<T>(nw + d));
    __syncwarp();
  }

  const T* cs = (const T*)a.cos + (size_t)pos * half;
  const T* sn = (const T*)a.sin + (size_t)pos * half;
  T* dst;
  if (is_q) {
    dst = (T*)a.q_out + ((size_t)m * a.nq + hh) * D;
  } else {
    const int h = hh - a.nq;
    dst = kv + kv_offset_elems(a.layer, 0, rd.slot_rows, rd.row, a.nkv, h, rd.cap, D, cache_pos);
  }
  for (int d = lane; d < D; d += 32) {
    const float c = ldf<T>(cs + (d % half)), sv = ldf<T>(sn + (d % half));
    const float rot = d < half ? -x[d + half] : x[d - half];
    stf<T>(dst + d, rt<T>(x[d] * c) + rt<T>(rot * sv));
  }
}

// VEC-wide loads and stores (VEC consecutive elements, 4 to 16 bytes).
template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const T* p, float* out) {
  if constexpr (sizeof(T) == 2 && VEC == 4) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    out[0] = __uint_as_float(v.x << 16); out[1] = __uint_as_float(v.x & 0xffff0000u);
    out[2] = __uint_as_float(v.y << 16); out[3] = __uint_as_float(v.y & 0xffff0000u);
  } else if constexpr (sizeof(T) == 2 && VEC == 2) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
    out[0] = __uint_as_float(v << 16); out[1] = __uint_as_float(v & 0xffff0000u);
  } else if constexpr (VEC == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  } else {
    const float2 v = *reinterpret_cast<const float2*>(p);
    out[0] = v.x; out[1] = v.y;
  }
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T* p, const float* in) {
  if constexpr (sizeof(T) == 2) {
    uint32_t w[VEC / 2];
#pragma unroll
    for (int i = 0; i < VEC / 2; ++i)
      w[i] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(in[2 * i])) |
             ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(in[2 * i + 1])) << 16);
    if constexpr (VEC == 4) *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
    else *reinterpret_cast<uint32_t*>(p) = w[0];
  } else {
    if constexpr (VEC == 4) *reinterpret_cast<float4*>(p) = make_float4(in[0], in[1], in[2], in[3]);
    else *reinterpret_cast<float2*>(p) = make_float2(in[0], in[1]);
  }
}

// The same work with one warp per head and VEC = D / 32 consecutive dims per
// lane (head_dim 64 or 128): vector loads and stores, the rotate-half
// partner (dims d ± D/2) from lane ^ 16 by a shuffle.
template <typename T, int VEC>
__global__ void __launch_bounds__(kHeadsPerCta * 32) qkv_post_vec_kernel(QkvPostArgs a) {
  pdl_trigger();
  pdl_wait();
  constexpr int D = VEC * 32, half = D / 2;
  __shared__ float xs[kHeadsPerCta][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x;
  const int hh = blockIdx.y * kHeadsPerCta + warp;
  const int nh = a.nq + 2 * a.nkv;
  if (hh >= nh) return;
  const int b = m / a.S, s = m % a.S;
  const RowDesc rd = a.rows[b];
  const int cache_pos = rd.past + s;
  int64_t pos = a.positions ? a.positions[m] : (int64_t)cache_pos;
  if (pos < 0 || pos >= a.max_pos) {
    flag_error(a.err, kErrPositionRange);
    pos = pos < 0 ? 0 : a.max_pos - 1;
  }
  const int d0 = lane * VEC;
  float x[VEC];
  if (a.use_pieces) {  // the projection's pieces, rounded as its store epilogue would
    float* xw = xs[warp];
    for (int d = lane * 4; d < D; d += 128) {
      float acc[4];
      pieces_sum4(a.pieces, m, hh * D + d, acc);
#pragma unroll
      for (int i = 0; i < 4; ++i) xw[d + i] = rt<T>(acc[i]);
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < VEC; ++i) x[i] = xw[d0 + i];
  } else {
    load_vec<T, VEC>((const T*)a.qkv + (size_t)m * nh * D + (size_t)hh * D + d0, x);
  }

  const bool is_q = hh < a.nq;
  const bool is_k = !is_q && hh < a.nq + a.nkv;
  T* kv = (T*)rd.kv_base;
  if (!is_q && !is_k) {  // value head: plain append
    const int h = hh - a.nq - a.nkv;
    store_vec<T, VEC>(kv + kv_offset_elems(a.layer, 1, rd.slot_rows, rd.row, a.nkv, h, rd.cap, D, cache_pos) + d0, x);
    return;
  }
  const T* nw = is_q ? (const T*)a.q_norm : (const T*)a.k_norm;
  if (nw) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) ss += x[i] * x[i];
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)D + a.eps);
    float g[VEC];
    load_vec<T, VEC>(nw + d0, g);
#pragma unroll
    for (int i = 0; i < VEC; ++i) x[i] = rt<T>(rt<T>(x[i] * r) * g[i]);
  }
  float c[VEC], sv[VEC], y[VEC];
  const int dh = (lane & 15) * VEC;  // d0 % half
  load_vec<T, VEC>((const T*)a.cos + (size_t)pos * half + dh, c);
  load_vec<T, VEC>((const T*)a.sin + (size_t)pos * half + dh, sv);
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const float partner = __shfl_xor_sync(0xffffffffu, x[i], 16);
    const float rot = lane < 16 ? -partner : partner;
    y[i] = rt<T>(x[i] * c[i]) + rt<T>(rot * sv[i]);
  }
  T* dst;
  if (is_q) {
    dst = (T*)a.q_out + ((size_t)m * a.nq + hh) * D;
  } else {
    const int h = hh - a.nq;
    dst = kv + kv_offset_elems(a.layer, 0, rd.slot_rows, rd.row, a.nkv, h, rd.cap, D, cache_pos);
  }
  store_vec<T, VEC>(dst + d0, y);
}

}  // namespace

cudaError_t launch_qkv_post(const QkvPostArgs& a, cudaStream_t s) {
  const int M = a.B * a.S;
  if (M == 0) return cudaSuccess;
  dim3 grid(M, (a.nq + 2 * a.nkv + kHeadsPerCta - 1) / kHeadsPerCta);
  if (a.D == 128 || a.D == 64) {
    cudaError_t e;
    if (a.dtype == kBF16)
      e = a.D == 128 ? launch_pdl(qkv_post_vec_kernel<__nv_bfloat16, 4>, grid, dim3(kHeadsPerCta * 32), 0, s, a)
                     : launch_pdl(qkv_post_vec_kernel<__nv_bfloat16, 2>, grid, dim3(kHeadsPerCta * 32), 0, s, a);
    else
      e = a.D == 128 ? launch_pdl(qkv_post_vec_kernel<float, 4>, grid, dim3(kHeadsPerCta * 32), 0, s, a)
                     : launch_pdl(qkv_post_vec_kernel<float, 2>, grid, dim3(kHeadsPerCta * 32), 0, s, a);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  if (a.dtype == kBF16)
    { const cudaError_t _le = launch_pdl(qkv_post_kernel<__nv_bfloat16>, dim3(grid), dim3(kHeadsPerCta * 32), 0, s, a); if (_le != cudaSuccess) return _le; }
  else
    { const cudaError_t _le = launch_pdl(qkv_post_kernel<float>, dim3(grid), dim3(kHeadsPerCta * 32), 0, s, a); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

}  // namespace mg
