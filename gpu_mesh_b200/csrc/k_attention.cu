// Grouped-query attention over the stage-owned KV cache.
//
// One CTA handles one query token, one KV head (all G = nq/nkv query heads
// that share it) and one chunk of keys (split-K, "flash decoding").  Keys are
// read once per KV head with 16-byte vector loads, a group of LPK lanes per
// key row.  Partial results (max, sum, unnormalised output) of every chunk are
// merged by a second kernel, which also rounds to the activation dtype.
//
// Visible keys follow LlamaStage's mask policy (models/llama_dense.py:497-532):
// sdpa with a single query token sees every cached key; otherwise key j is
// visible iff j <= position (the additive finfo.min mask and SDPA's is_causal
// both reduce to this prefix).  HF's Qwen3 causal mask uses the cache index
// instead: j <= past + s.  Scale is 1/sqrt(D) as in SDPA (llama_dense.py:175).
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace mg {
namespace {

constexpr int kAttnChunk = 256;
constexpr int kAttnWarps = 4;

__device__ __forceinline__ int visible_keys(const AttnArgs& a, const RowDesc& rd, int m, int s) {
  const int total = rd.past + a.S;
  if (a.mask == kMaskSdpa && a.S == 1) return total;
  if (a.mask == kMaskCacheCausal) return min(rd.past + s + 1, total);
  int64_t pos = a.positions ? a.positions[m] : (int64_t)(rd.past + s);
  if (pos < 0) pos = 0;
  const int64_t lim = pos + 1 < (int64_t)total ? pos + 1 : (int64_t)total;
  return (int)lim;
}

template <typename T, int LPK, int GM>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_split_kernel(AttnArgs a) {
  constexpr int VEC = Vec16<T>::N;
  constexpr int D = LPK * VEC;
  constexpr int KPW = 32 / LPK;  // keys per warp step
  constexpr int NW = kAttnWarps;
  __shared__ float q_s[GM][D];
  __shared__ float sc[GM][kAttnChunk];
  __shared__ float red[NW][GM][D];
  __shared__ float stat[GM][2];

  const int m = blockIdx.x, h = blockIdx.y, sp = blockIdx.z;
  const int G = a.nq / a.nkv;
  const int b = m / a.S, s = m % a.S;
  const RowDesc rd = a.rows[b];
  const int nvis = visible_keys(a, rd, m, s);
  const int k0 = sp * kAttnChunk;
  const int k1 = min(nvis, k0 + kAttnChunk);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  float* part = a.partial + ((size_t)(m * a.nkv + h) * gridDim.z + sp) * (size_t)G * (D + 2);
  if (k0 >= k1) {
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      part[g * (D + 2)] = -INFINITY;
      part[g * (D + 2) + 1] = 0.f;
    }
    return;
  }
  const int n = k1 - k0;

  const T* q = (const T*)a.q + ((size_t)m * a.nq + (size_t)h * G) * D;
  for (int i = threadIdx.x; i < GM * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    q_s[g][d] = g < G ? ldf<T>(q + (size_t)g * D + d) : 0.f;
  }
  __syncthreads();

  const T* kbase = (const T*)rd.kv_base +
                   kv_offset_elems(a.layer, 0, rd.slot_rows, rd.row, a.nkv, h, rd.cap, D, 0);
  const T* vbase = (const T*)rd.kv_base +
                   kv_offset_elems(a.layer, 1, rd.slot_rows, rd.row, a.nkv, h, rd.cap, D, 0);
  const int vs = lane % LPK, kg = lane / LPK;

  // Scores.
  float qv[GM][VEC];
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int e = 0; e < VEC; ++e) qv[g][e] = q_s[g][vs * VEC + e];
#pragma unroll 2
  for (int base = warp * KPW; base < n; base += NW * KPW) {
    const int j = base + kg;
    float kvv[VEC];
    if (j < n) load16_f<T>(kbase + (size_t)(k0 + j) * D + vs * VEC, kvv);
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      float d = 0.f;
      if (j < n) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) d = fmaf(qv[g][e], kvv[e], d);
      }
#pragma unroll
      for (int o = LPK / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      if (vs == 0 && j < n) sc[g][j] = d * a.scale;
    }
  }
  __syncthreads();

  // Softmax statistics of this chunk, one warp per query head.
  for (int g = warp; g < G; g += NW) {
    float mx = -INFINITY;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[g][j]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float p = expf(sc[g][j] - mx);
      sc[g][j] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      stat[g][0] = mx;
      stat[g][1] = sum;
    }
  }
  __syncthreads();

  // Unnormalised output: sum_j p_j * v_j.
  float acc[GM][VEC];
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[g][e] = 0.f;
#pragma unroll 2
  for (int base = warp * KPW; base < n; base += NW * KPW) {
    const int j = base + kg;
    if (j < n) {
      float vv[VEC];
      load16_f<T>(vbase + (size_t)(k0 + j) * D + vs * VEC, vv);
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        const float p = sc[g][j];
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[g][e] = fmaf(p, vv[e], acc[g][e]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      float v = acc[g][e];
#pragma unroll
      for (int o = 16; o >= LPK; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[g][e] = v;
    }
  if (kg == 0) {
#pragma unroll
    for (int g = 0; g < GM; ++g)
#pragma unroll
      for (int e = 0; e < VEC; ++e) red[warp][g][vs * VEC + e] = acc[g][e];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) v += red[w][g][d];
    part[g * (D + 2) + 2 + d] = v;
  }
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    part[g * (D + 2)] = stat[g][0];
    part[g * (D + 2) + 1] = stat[g][1];
  }
}

template <typename T>
__global__ void attn_combine_kernel(AttnArgs a, int splits) {
  const int m = blockIdx.x, hq = blockIdx.y;
  const int G = a.nq / a.nkv, D = a.D;
  const int h = hq / G, g = hq % G;
  const float* base = a.partial + (size_t)(m * a.nkv + h) * splits * G * (D + 2) + (size_t)g * (D + 2);
  const size_t sstride = (size_t)G * (D + 2);
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, base[s * sstride]);
  float l = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ms = base[s * sstride];
    if (ms != -INFINITY) l += base[s * sstride + 1] * expf(ms - mx);
  }
  const float inv = 1.0f / l;
  T* out = (T*)a.out + ((size_t)m * a.nq + hq) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float ms = base[s * sstride];
      if (ms != -INFINITY) o += base[s * sstride + 2 + d] * expf(ms - mx);
    }
    stf<T>(out + d, o * inv);
  }
}

template <typename T, int LPK>
cudaError_t attn_launch_g(const AttnArgs& a, dim3 grid, int G, cudaStream_t s) {
  if constexpr (LPK * Vec16<T>::N > 128) {
    return cudaErrorInvalidValue;  // head_dim above 128 is rejected at stage creation
  } else {
    if (G <= 1) attn_split_kernel<T, LPK, 1><<<grid, kAttnWarps * 32, 0, s>>>(a);
    else if (G <= 2) attn_split_kernel<T, LPK, 2><<<grid, kAttnWarps * 32, 0, s>>>(a);
    else if (G <= 4) attn_split_kernel<T, LPK, 4><<<grid, kAttnWarps * 32, 0, s>>>(a);
    else attn_split_kernel<T, LPK, 8><<<grid, kAttnWarps * 32, 0, s>>>(a);
    note_launch();
    return cudaGetLastError();
  }
}

template <typename T>
cudaError_t attn_launch(const AttnArgs& a, dim3 grid, cudaStream_t s) {
  constexpr int VEC = Vec16<T>::N;
  const int lpk = a.D / VEC;
  const int G = a.nq / a.nkv;
  switch (lpk) {
    case 1: return attn_launch_g<T, 1>(a, grid, G, s);
    case 2: return attn_launch_g<T, 2>(a, grid, G, s);
    case 4: return attn_launch_g<T, 4>(a, grid, G, s);
    case 8: return attn_launch_g<T, 8>(a, grid, G, s);
    case 16: return attn_launch_g<T, 16>(a, grid, G, s);
    case 32: return attn_launch_g<T, 32>(a, grid, G, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

size_t attention_scratch_elems(int M, int nq, int D, int max_keys) {
  const int splits = (max_keys + kAttnChunk - 1) / kAttnChunk;
  return (size_t)M * nq * splits * (D + 2);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s) {
  const int M = a.B * a.S;
  if (M == 0) return cudaSuccess;
  const int splits = (a.max_keys + kAttnChunk - 1) / kAttnChunk;
  if (attention_scratch_elems(M, a.nq, a.D, a.max_keys) > a.partial_elems)
    return cudaErrorInvalidValue;
  dim3 grid(M, a.nkv, splits);
  cudaError_t e = (a.dtype == kBF16) ? attn_launch<__nv_bfloat16>(a, grid, s)
                                     : attn_launch<float>(a, grid, s);
  if (e != cudaSuccess) return e;
  dim3 cgrid(M, a.nq);
  const int threads = a.D < 128 ? a.D : 128;
  if (a.dtype == kBF16)
    { attn_combine_kernel<__nv_bfloat16><<<cgrid, threads, 0, s>>>(a, splits); note_launch(); }
  else
    { attn_combine_kernel<float><<<cgrid, threads, 0, s>>>(a, splits); note_launch(); }
  return cudaGetLastError();
}

}  // namespace mg
