// Token sampling over logits rows: greedy argmax and top-p (nucleus).
//
// greedy_sample (inference/sampling.py:58-60) is an argmax with the lowest
// index winning ties; bf16 logits tie often, so the tie rule matters.
//
// top_p_sample (sampling.py:63-95) sorts the probabilities, keeps the prefix
// whose exclusive cumulative mass is <= top_p, renormalises and draws.  The
// kernel reaches the same token without sorting the vocabulary: with ties
// ordered by token index, the descending order is fixed by the values, so
//   mass_gt(v) = sum of p_i over p_i > v
// locates every boundary.  Two searches over the fp32 bit patterns find
//   (1) the cut level b*: the smallest v with mass_gt(v) <= top_p, and
//   (2) the drawn level w: the smallest v with mass_gt(v) <= u * Z, Z the
//       kept mass;
// the rank inside a tie group follows from the group's constant probability,
// and a final scan finds the token of that rank.  The uniform draw u is an
// input (one per row), so a seeded caller gets reproducible tokens.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace mg {
namespace {

constexpr int kSampleThreads = 1024;

template <typename T>
__device__ __forceinline__ float logit_at(const T* row, int i) {
  return ldf<T>(row + i);
}

// a beats b: larger value, NaN above everything, lowest index on ties.
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  const bool na = isnan(va), nb = isnan(vb);
  if (na != nb) return na;
  if (!na && va != vb) return va > vb;
  return ia < ib;
}

template <typename T>
__global__ void __launch_bounds__(kSampleThreads) argmax_kernel(const T* __restrict__ logits,
                                                                int vocab, int64_t stride,
                                                                int64_t* __restrict__ ids) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  const T* row = logits + (size_t)blockIdx.x * stride;
  float bv = -INFINITY;
  int bi = INT_MAX;
  constexpr int VEC = Vec16<T>::N;
  if ((vocab % VEC) == 0 && ((uintptr_t)row % 16) == 0) {
    // 16-byte vectors, two in flight per thread; indices within a thread
    // only grow, so keeping the first of equal values keeps the lowest index.
    const int nv = vocab / VEC;
    for (int i = threadIdx.x; i < nv; i += 2 * blockDim.x) {
      float v0[VEC], v1[VEC];
      const int i1 = i + blockDim.x;
      load16_f<T>(row + (size_t)i * VEC, v0);
      if (i1 < nv) load16_f<T>(row + (size_t)i1 * VEC, v1);
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        if (better(v0[j], i * VEC + j, bv, bi)) {
          bv = v0[j];
          bi = i * VEC + j;
        }
      if (i1 < nv) {
#pragma unroll
        for (int j = 0; j < VEC; ++j)
          if (better(v1[j], i1 * VEC + j, bv, bi)) {
            bv = v1[j];
            bi = i1 * VEC + j;
          }
      }
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
      const float v = logit_at<T>(row, i);
      if (better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : INT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) ids[blockIdx.x] = bi == INT_MAX ? 0 : bi;
  }
}

__device__ float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ float block_reduce_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
  return warp_max(t);
}

template <typename T>
__device__ __forceinline__ float scaled(const T* row, int i, float temperature) {
  return logit_at<T>(row, i) / temperature;
}

template <typename T>
__global__ void __launch_bounds__(kSampleThreads) top_p_kernel(const T* __restrict__ logits,
                                                               int vocab, int64_t stride,
                                                               float temperature, float top_p,
                                                               const float* __restrict__ uniforms,
                                                               int64_t* __restrict__ ids) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  __shared__ int cnt_s[32];
  const T* row = logits + (size_t)blockIdx.x * stride;

  // softmax(logits.float() / temperature) in fp32.
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) mx = fmaxf(mx, scaled<T>(row, i, temperature));
  mx = block_reduce_max(mx, red);
  float se = 0.f;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) se += expf(scaled<T>(row, i, temperature) - mx);
  se = block_reduce_sum(se, red);
  auto prob = [&](int i) { return expf(scaled<T>(row, i, temperature) - mx) / se; };

  auto mass_gt = [&](float v) {
    float acc = 0.f;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
      const float p = prob(i);
      if (p > v) acc += p;
    }
    return block_reduce_sum(acc, red);
  };
  auto count_eq = [&](float v) {
    int c = 0;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) c += prob(i) == v;
    c = __reduce_add_sync(0xffffffffu, c);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) cnt_s[warp] = c;
    __syncthreads();
    int t = lane < (int)(blockDim.x >> 5) ? cnt_s[lane] : 0;
    return __reduce_add_sync(0xffffffffu, t);
  };
  // Smallest non-negative float v (by bit pattern) with mass_gt(v) <= target.
  auto search = [&](float target) {
    uint32_t lo = 0u, hi = __float_as_uint(1.0f);
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo) / 2;
      if (mass_gt(__uint_as_float(mid)) <= target) hi = mid;
      else lo = mid + 1;
    }
    return __uint_as_float(lo);
  };

  // (1) The kept prefix.
  const float bstar = search(top_p);
  const float gt_b = mass_gt(bstar);
  const int cnt_b = count_eq(bstar);
  int keep_b = cnt_b;
  if (bstar > 0.f) {
    const float room = floorf((top_p - gt_b) / bstar) + 1.0f;
    keep_b = (int)fminf((float)cnt_b, fmaxf(room, 0.f));
  }
  const float z = gt_b + (float)keep_b * bstar;

  // (2) The drawn level and the rank inside its tie group.
  const float x = uniforms[blockIdx.x] * z;
  const float w = search(x);
  const float gt_w = mass_gt(w);
  const int cnt_w = count_eq(w);
  int limit = (w == bstar) ? keep_b : cnt_w;
  if (limit < 1) limit = 1;
  int rank = w > 0.f ? (int)floorf((x - gt_w) / w) : 0;
  rank = max(0, min(rank, limit - 1));

  // (3) The token holding that rank among the indices with p == w.
  __shared__ int found;
  __shared__ int base_count;
  if (threadIdx.x == 0) {
    found = -1;
    base_count = 0;
  }
  __syncthreads();
  for (int t0 = 0; t0 < vocab; t0 += blockDim.x) {
    const int i = t0 + threadIdx.x;
    const bool hit = i < vocab && prob(i) == w;
    const unsigned bal = __ballot_sync(0xffffffffu, hit);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) cnt_s[warp] = __popc(bal);
    __syncthreads();
    int before = base_count;
    for (int k = 0; k < warp; ++k) before += cnt_s[k];
    before += __popc(bal & ((1u << lane) - 1u));
    if (hit && before == rank) found = i;
    __syncthreads();
    if (threadIdx.x == 0) {
      int tot = 0;
      for (int k = 0; k < (int)(blockDim.x >> 5); ++k) tot += cnt_s[k];
      base_count += tot;
    }
    __syncthreads();
    if (found >= 0) break;
  }
  if (threadIdx.x == 0) ids[blockIdx.x] = found >= 0 ? found : 0;
}

}  // namespace

cudaError_t launch_argmax(int dtype, const void* logits, int rows, int vocab, int64_t stride,
                          int64_t* ids, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (dtype == kBF16)
    { const cudaError_t _le = launch_pdl(argmax_kernel<__nv_bfloat16>, dim3(rows), dim3(kSampleThreads), 0, s, (const __nv_bfloat16*)logits,
                                                                 vocab, stride, ids); if (_le != cudaSuccess) return _le; }
  else
    { const cudaError_t _le = launch_pdl(argmax_kernel<float>, dim3(rows), dim3(kSampleThreads), 0, s, (const float*)logits, vocab, stride, ids); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

cudaError_t launch_top_p(int dtype, const void* logits, int rows, int vocab, int64_t stride,
                         float temperature, float top_p, const float* uniforms, int64_t* ids,
                         cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (!(temperature > 0.f)) return launch_argmax(dtype, logits, rows, vocab, stride, ids, s);
  if (dtype == kBF16)
    { const cudaError_t _le = launch_pdl(top_p_kernel<__nv_bfloat16>, dim3(rows), dim3(kSampleThreads), 0, s, 
        (const __nv_bfloat16*)logits, vocab, stride, temperature, top_p, uniforms, ids); if (_le != cudaSuccess) return _le; }
  else
    { const cudaError_t _le = launch_pdl(top_p_kernel<float>, dim3(rows), dim3(kSampleThreads), 0, s, (const float*)logits, vocab, stride,
                                                        temperature, top_p, uniforms, ids); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

}  // namespace mg
