// Token embedding gather, RMSNorm and KV-slot copies.
//
// RMSNorm follows LlamaStage's RMSNorm.forward (models/llama_dense.py:91-93)
// and HF Qwen3RMSNorm: mean of squares in fp32, multiply by 1/sqrt(ms + eps),
// round to the activation dtype, then multiply by the weight in that dtype.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace mg {
namespace {

// One thread waits for the stage's probe flag with the bounded wait every
// kernel of the stage uses; nothing else is in flight, so an expiry leaves
// nothing behind but code 3 in the error word.
__global__ void wait_probe_kernel(const int* flag, uint64_t limit_ns, int* err) {
  if (threadIdx.x == 0) tc::flag_wait(flag, limit_ns, err);
}

template <typename T>
__global__ void embed_kernel(const T* __restrict__ table, const int64_t* __restrict__ ids, int H,
                             int V, T* __restrict__ out, int* err) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x;
  int64_t id = ids[m];
  if (id < 0 || id >= V) {
    flag_error(err, kErrTokenRange);
    id = 0;
  }
  constexpr int VEC = Vec16<T>::N;
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)m * H);
  for (int i = threadIdx.x; i < H / VEC; i += blockDim.x) dst[i] = src[i];
}

// RMSNorm reduction order, shared by every kernel that normalises a row: 512
// threads, thread j adds the squares of the 16-byte vectors j, j + 512, ...
// (each vector's elements in order), then a butterfly over each warp's 32
// lanes, then over the 16 warp sums.
template <typename T>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (lane < nw) ? red[lane] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, int64_t xs, const T* __restrict__ w, int H,
                               float eps, T* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int m = blockIdx.x;
  const T* xr = x + (size_t)m * xs;
  T* yr = y + (size_t)m * H;
  constexpr int VEC = Vec16<T>::N;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H / VEC; i += blockDim.x) {
    float v[VEC];
    load16_f<T>(xr + i * VEC, v);
#pragma unroll
    for (int j = 0; j < VEC; ++j) ss += v[j] * v[j];
  }
  ss = block_sum<T>(ss, red);
  const float r = 1.0f / sqrtf(ss / (float)H + eps);
  for (int i = threadIdx.x; i < H / VEC; i += blockDim.x) {
    float v[VEC], g[VEC];
    load16_f<T>(xr + i * VEC, v);
    load16_f<T>(w + i * VEC, g);
#pragma unroll
    for (int j = 0; j < VEC; ++j) stf<T>(yr + i * VEC + j, rt<T>(rt<T>(v[j] * r) * g[j]));
  }
}

// RMSNorm of many rows (prefill): one warp per row, 8 rows per CTA.  Lane l
// keeps the partial sums of the 16 threads l, 32 + l, ..., 480 + l of the
// 512-thread kernel (same vectors, same order), reduces each over the warp,
// then reduces the 16 warp sums as the block reduction does, so every output
// is bit-identical to rmsnorm_kernel's.
constexpr int kRowsPerCta = 8;

template <typename T>
__global__ void __launch_bounds__(kRowsPerCta * 32) rmsnorm_rows_kernel(const T* __restrict__ x, int64_t xs,
                                                                        const T* __restrict__ w, int H, float eps,
                                                                        T* __restrict__ y, int M) {
  pdl_trigger();
  pdl_wait();
  constexpr int kVirt = kNormThreads / 32;  // warps of the block-per-row kernel
  const int lane = threadIdx.x & 31;
  const int m = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
  if (m >= M) return;
  const T* xr = x + (size_t)m * xs;
  T* yr = y + (size_t)m * H;
  constexpr int VEC = Vec16<T>::N;
  const int nv = H / VEC;
  float part[kVirt];
#pragma unroll
  for (int v = 0; v < kVirt; ++v) part[v] = 0.f;
  for (int base = 0; base < nv; base += kNormThreads) {
#pragma unroll
    for (int v = 0; v < kVirt; ++v) {
      const int i = base + v * 32 + lane;
      if (i < nv) {
        float e[VEC];
        load16_f<T>(xr + i * VEC, e);
#pragma unroll
        for (int j = 0; j < VEC; ++j) part[v] += e[j] * e[j];
      }
    }
  }
  float t = 0.f;
#pragma unroll
  for (int v = 0; v < kVirt; ++v) {
    const float sv = warp_sum(part[v]);
    if (lane == v) t = sv;
  }
  const float ss = warp_sum(t);
  const float r = 1.0f / sqrtf(ss / (float)H + eps);
  for (int i = lane; i < nv; i += 32) {
    float e[VEC], g[VEC], o[VEC];
    load16_f<T>(xr + i * VEC, e);
    load16_f<T>(w + i * VEC, g);
#pragma unroll
    for (int j = 0; j < VEC; ++j) o[j] = rt<T>(rt<T>(e[j] * r) * g[j]);
    store16_f<T>(yr + i * VEC, o);
  }
}

// The residual epilogue of a decode GEMM left as pieces, then (optionally)
// the RMSNorm of the new residual row, in the RMSNorm reduction order (one
// 8-element vector per thread at H <= 4096, so every piece load of the row
// is in flight at once).
__global__ void __launch_bounds__(kNormThreads) resid_norm_pieces_kernel(Pieces pc, __nv_bfloat16* __restrict__ x,
                                                                const __nv_bfloat16* __restrict__ w, int H,
                                                                float eps, __nv_bfloat16* __restrict__ y) {
  pdl_trigger();
  // The norm weights do not depend on the kernels before this one: at
  // H <= 8 * blockDim.x each thread's one vector of them is requested before
  // the wait.
  const bool one = w && H / 8 <= (int)blockDim.x;
  float g0[8];
  if (one && (int)threadIdx.x < H / 8) load16_f<__nv_bfloat16>(w + threadIdx.x * 8, g0);
  pdl_wait();
  __shared__ float red[32];
  const int m = blockIdx.x;
  __nv_bfloat16* xr = x + (size_t)m * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
    float acc[8], v[8];
    pieces_sum8(pc, m, i * 8, acc);
    load16_f<__nv_bfloat16>(xr + i * 8, v);
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j] = __float2bfloat16_rn(v[j] + rt<__nv_bfloat16>(acc[j]));
      const float nv = __bfloat162float(o[j]);
      ss += nv * nv;
    }
    *reinterpret_cast<uint4*>(xr + i * 8) = *reinterpret_cast<const uint4*>(o);
  }
  if (!w) return;
  ss = block_sum<__nv_bfloat16>(ss, red);
  const float r = 1.0f / sqrtf(ss / (float)H + eps);
  __nv_bfloat16* yr = y + (size_t)m * H;
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
    float v[8], g[8], o[8];
    load16_f<__nv_bfloat16>(xr + i * 8, v);  // this thread's own stores
    if (one) {
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = g0[j];
    } else {
      load16_f<__nv_bfloat16>(w + i * 8, g);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = rt<__nv_bfloat16>(rt<__nv_bfloat16>(v[j] * r) * g[j]);
    store16_f<__nv_bfloat16>(yr + i * 8, o);
  }
}

// The same residual + RMSNorm with each row spread over a cluster of
// kNormCluster CTAs of kNormThreads / kNormCluster threads, so a row's piece
// loads come through four SMs instead of one (32 decode rows otherwise keep
// 32 of 148 SMs busy).  CTA c's thread j plays thread 128·c + j of the
// 512-thread kernel (same vectors, same order), each CTA writes its four
// warp sums into all the cluster's CTAs, and after the cluster barrier every
// CTA reduces the 16 warp sums exactly as block_sum does: the outputs are
// bit-identical to resid_norm_pieces_kernel's.  Every CTA of a cluster takes
// the same branches (the only early return depends on a kernel argument), so
// all of them reach the barrier.
constexpr int kNormCluster = 4;
constexpr int kNormCtaThreads = kNormThreads / kNormCluster;

__global__ void __launch_bounds__(kNormCtaThreads) resid_norm_pieces_cluster_kernel(
    Pieces pc, __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w, int H, float eps,
    __nv_bfloat16* __restrict__ y) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  pdl_trigger();
  const int c = (int)cluster.block_rank();
  const int t = c * kNormCtaThreads + (int)threadIdx.x;  // thread of the 512-thread kernel
  const bool one = w && H / 8 <= kNormThreads;
  float g0[8];
  if (one && t < H / 8) load16_f<__nv_bfloat16>(w + t * 8, g0);
  pdl_wait();
  __shared__ float red[32];
  const int m = blockIdx.x / kNormCluster;
  __nv_bfloat16* xr = x + (size_t)m * H;
  float ss = 0.f;
  for (int i = t; i < H / 8; i += kNormThreads) {
    float acc[8], v[8];
    pieces_sum8(pc, m, i * 8, acc);
    load16_f<__nv_bfloat16>(xr + i * 8, v);
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j] = __float2bfloat16_rn(v[j] + rt<__nv_bfloat16>(acc[j]));
      const float nv = __bfloat162float(o[j]);
      ss += nv * nv;
    }
    *reinterpret_cast<uint4*>(xr + i * 8) = *reinterpret_cast<const uint4*>(o);
  }
  if (!w) return;
  // block_sum over the cluster: warp sums first, each written into every CTA.
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0)
    for (int r = 0; r < kNormCluster; ++r) cluster.map_shared_rank(red, r)[c * (kNormCtaThreads / 32) + warp] = ss;
  cluster.sync();
  constexpr int nw = kNormThreads / 32;
  float tsum = lane < nw ? red[lane] : 0.f;
  tsum = warp_sum(tsum);
  const float r = 1.0f / sqrtf(tsum / (float)H + eps);
  __nv_bfloat16* yr = y + (size_t)m * H;
  for (int i = t; i < H / 8; i += kNormThreads) {
    float v[8], g[8], o[8];
    load16_f<__nv_bfloat16>(xr + i * 8, v);  // this thread's own stores
    if (one) {
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = g0[j];
    } else {
      load16_f<__nv_bfloat16>(w + i * 8, g);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = rt<__nv_bfloat16>(rt<__nv_bfloat16>(v[j] * r) * g[j]);
    store16_f<__nv_bfloat16>(yr + i * 8, o);
  }
}

template <typename T>
__global__ void kv_copy_kernel(T* __restrict__ kv, int layer, int kvsel, int slot_rows, int nkv,
                               int cap, int D, int len, T* __restrict__ ext, bool to_slot) {
  pdl_trigger();
  pdl_wait();
  // grid: (len, nkv, slot_rows); block covers D.
  const int pos = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
  T* sp = kv + kv_offset_elems(layer, kvsel, slot_rows, r, nkv, h, cap, D, pos);
  T* ep = ext + (((size_t)r * nkv + h) * len + pos) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    if (to_slot) sp[d] = ep[d];
    else ep[d] = sp[d];
  }
}

}  // namespace

cudaError_t launch_wait_probe(const int* flag, uint64_t limit_ns, int* err, cudaStream_t s) {
  wait_probe_kernel<<<1, 32, 0, s>>>(flag, limit_ns, err);
  return cudaGetLastError();
}

cudaError_t launch_embed(int dtype, const void* table, const int64_t* ids, int M, int H, int V,
                         void* out, int* err, cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  if (dtype == kBF16)
    { const cudaError_t _le = launch_pdl(embed_kernel<__nv_bfloat16>, dim3(M), dim3(128), 0, s, (const __nv_bfloat16*)table, ids, H, V,
                                                  (__nv_bfloat16*)out, err); if (_le != cudaSuccess) return _le; }
  else
    { const cudaError_t _le = launch_pdl(embed_kernel<float>, dim3(M), dim3(128), 0, s, (const float*)table, ids, H, V, (float*)out, err); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

cudaError_t launch_resid_norm_pieces(int dtype, const Pieces& pc, void* x, const void* w, void* xn, int M,
                                     int H, float eps, cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  if (dtype != kBF16 || H % 8 || !pc.slots) return cudaErrorInvalidValue;
  // A cluster of four CTAs per row (bit-identical to the one-CTA kernel,
  // which MESHGPU_NORM_ONE_CTA=1 selects; its tests compare the two).
  const char* one_cta = getenv("MESHGPU_NORM_ONE_CTA");
  if (one_cta && one_cta[0] == '1') {
    const cudaError_t e = launch_pdl(resid_norm_pieces_kernel, dim3(M), dim3(kNormThreads), 0, s, pc,
                                     (__nv_bfloat16*)x, (const __nv_bfloat16*)w, H, eps, (__nv_bfloat16*)xn);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M * kNormCluster);
  cfg.blockDim = dim3(kNormCtaThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kNormCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, resid_norm_pieces_cluster_kernel, pc, (__nv_bfloat16*)x,
                                     (const __nv_bfloat16*)w, H, eps, (__nv_bfloat16*)xn);
  if (e != cudaSuccess) {
    // A device or partition that cannot place a cluster of four: the
    // one-CTA kernel (same rows, bit for bit).
    cudaGetLastError();
    e = launch_pdl(resid_norm_pieces_kernel, dim3(M), dim3(kNormThreads), 0, s, pc, (__nv_bfloat16*)x,
                   (const __nv_bfloat16*)w, H, eps, (__nv_bfloat16*)xn);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(int dtype, const void* x, int64_t xs, const void* w, int M, int H,
                           float eps, void* y, cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  const int threads = kNormThreads;
  if (M > kRowsPerCta * 4) {  // many rows: a warp per row (same results)
    const dim3 grid((M + kRowsPerCta - 1) / kRowsPerCta);
    const cudaError_t e =
        dtype == kBF16
            ? launch_pdl(rmsnorm_rows_kernel<__nv_bfloat16>, grid, dim3(kRowsPerCta * 32), 0, s,
                         (const __nv_bfloat16*)x, xs, (const __nv_bfloat16*)w, H, eps, (__nv_bfloat16*)y, M)
            : launch_pdl(rmsnorm_rows_kernel<float>, grid, dim3(kRowsPerCta * 32), 0, s, (const float*)x, xs,
                         (const float*)w, H, eps, (float*)y, M);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  if (dtype == kBF16)
    { const cudaError_t _le = launch_pdl(rmsnorm_kernel<__nv_bfloat16>, dim3(M), dim3(threads), 0, s, 
        (const __nv_bfloat16*)x, xs, (const __nv_bfloat16*)w, H, eps, (__nv_bfloat16*)y); if (_le != cudaSuccess) return _le; }
  else
    { const cudaError_t _le = launch_pdl(rmsnorm_kernel<float>, dim3(M), dim3(threads), 0, s, (const float*)x, xs, (const float*)w, H, eps,
                                                (float*)y); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

cudaError_t launch_kv_copy(int dtype, void* kv_base, int layer, int kv, int slot_rows, int nkv,
                           int cap, int D, int len, void* ext, bool to_slot, cudaStream_t s) {
  if (len == 0) return cudaSuccess;
  dim3 grid(len, nkv, slot_rows);
  const int threads = D < 128 ? D : 128;
  if (dtype == kBF16)
    { const cudaError_t _le = launch_pdl(kv_copy_kernel<__nv_bfloat16>, dim3(grid), dim3(threads), 0, s, (__nv_bfloat16*)kv_base, layer, kv,
                                                           slot_rows, nkv, cap, D, len,
                                                           (__nv_bfloat16*)ext, to_slot); if (_le != cudaSuccess) return _le; }
  else
    { const cudaError_t _le = launch_pdl(kv_copy_kernel<float>, dim3(grid), dim3(threads), 0, s, (float*)kv_base, layer, kv, slot_rows, nkv, cap,
                                                   D, len, (float*)ext, to_slot); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

}  // namespace mg
