// Grouped-query attention over the stage-owned KV cache.
//
// One CTA handles one query token, one KV head (all G = nq/nkv query heads
// that share it) and one chunk of up to 128 keys (split-K, "flash decoding").
// In the slot layout the chunk's keys, and its values, are each one
// contiguous run of chunk x D elements, so the CTA stages them into shared
// memory with two bulk TMA copies (cp.async.bulk, no multicast) on two
// mbarriers: scoring starts as soon as the keys have landed while the values
// are still in flight.  Scores use a group of LPK lanes per key (16-byte
// vectors, warp-shuffle reduction); the value pass has each thread own one
// (query head, 16-byte slice of D) and walk the chunk's keys.  Chunk partials
// (max, sum, unnormalised output) are merged by a second kernel, which also
// rounds to the activation dtype.
//
// Visible keys follow LlamaStage's mask policy (models/llama_dense.py:497-532):
// sdpa with a single query token sees every cached key; otherwise key j is
// visible iff j <= position (the additive finfo.min mask and SDPA's is_causal
// both reduce to this prefix).  HF's Qwen3 causal mask uses the cache index
// instead: j <= past + s.  Scale is 1/sqrt(D) as in SDPA (llama_dense.py:175).
#include <math.h>

#include "kernels.h"
#include "tc_common.cuh"

namespace mg {
namespace {

using namespace tc;

constexpr int kAttnChunk = 128;
constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;

__device__ __forceinline__ int visible_keys(const AttnArgs& a, const RowDesc& rd, int m, int s) {
  const int total = rd.past + a.S;
  if (a.mask == kMaskSdpa && a.S == 1) return total;
  if (a.mask == kMaskCacheCausal) return min(rd.past + s + 1, total);
  int64_t pos = a.positions ? a.positions[m] : (int64_t)(rd.past + s);
  if (pos < 0) pos = 0;
  const int64_t lim = pos + 1 < (int64_t)total ? pos + 1 : (int64_t)total;
  return (int)lim;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <typename T, int LPK, int GM>
struct AttnLayout {
  static constexpr int VEC = Vec16<T>::N;
  static constexpr int D = LPK * VEC;
  static constexpr int kKV = kAttnChunk * D * sizeof(T);          // bytes of K (or V) per chunk
  static constexpr int kSlots = GM * LPK;                         // (head, slice) pairs
  static constexpr int kGroups = kSlots >= kAttnThreads ? 1 : kAttnThreads / kSlots;
  static constexpr int kQ = GM * D * 4;
  static constexpr int kSc = GM * kAttnChunk * 4;
  static constexpr int kRed = kGroups * GM * D * 4;
  static constexpr int kBytes = 2 * kKV + kQ + kSc + kRed + 128 /*align*/ + 256 /*bars, stats*/;
};

template <typename T, int LPK, int GM>
__global__ void __launch_bounds__(kAttnThreads) attn_chunk_kernel(AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  using L = AttnLayout<T, LPK, GM>;
  constexpr int VEC = L::VEC, D = L::D, KPW = 32 / LPK, NW = kAttnWarps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
  T* Ks = (T*)smem;
  T* Vs = (T*)(smem + L::kKV);
  float* q_s = (float*)(smem + 2 * L::kKV);
  float* sc = (float*)(smem + 2 * L::kKV + L::kQ);
  float* red = (float*)(smem + 2 * L::kKV + L::kQ + L::kSc);
  uint64_t* bar = (uint64_t*)(smem + 2 * L::kKV + L::kQ + L::kSc + L::kRed);
  float* stat = (float*)(bar + 2);  // [GM][2]

  const int m = blockIdx.x, h = blockIdx.y, sp = blockIdx.z;
  const int G = a.nq / a.nkv;
  const int b = m / a.S, s = m % a.S;
  const RowDesc rd = a.rows[b];
  const int nvis = visible_keys(a, rd, m, s);
  const int k0 = sp * kAttnChunk;
  const int k1 = min(nvis, k0 + kAttnChunk);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  float* part = a.partial + ((size_t)(m * a.nkv + h) * gridDim.z + sp) * (size_t)G * (D + 2);
  if (k0 >= k1) {
    for (int g = tid; g < G; g += blockDim.x) {
      part[g * (D + 2)] = -INFINITY;
      part[g * (D + 2) + 1] = 0.f;
    }
    return;
  }
  const int n = k1 - k0;
  const T* kbase = (const T*)rd.kv_base +
                   kv_offset_elems(a.layer, 0, rd.slot_rows, rd.row, a.nkv, h, rd.cap, D, k0);
  const T* vbase = (const T*)rd.kv_base +
                   kv_offset_elems(a.layer, 1, rd.slot_rows, rd.row, a.nkv, h, rd.cap, D, k0);
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t bytes = (uint32_t)(n * D * sizeof(T));
    mbar_expect_tx(&bar[0], bytes);
    bulk_load(Ks, kbase, bytes, &bar[0]);
    mbar_expect_tx(&bar[1], bytes);
    bulk_load(Vs, vbase, bytes, &bar[1]);
  }
  const T* q = (const T*)a.q + ((size_t)m * a.nq + (size_t)h * G) * D;
  for (int i = tid; i < GM * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    q_s[i] = g < G ? ldf<T>(q + (size_t)g * D + d) : 0.f;
  }
  __syncthreads();

  // Scores from the staged keys.
  const bool have_k = mbar_wait(&bar[0], 0, a.err);
  const int vs = lane % LPK, kg = lane / LPK;
  float qv[GM][VEC];
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int e = 0; e < VEC; ++e) qv[g][e] = q_s[g * D + vs * VEC + e];
  for (int base = warp * KPW; base < n; base += NW * KPW) {
    const int j = base + kg;
    float kvv[VEC];
    if (j < n && have_k) load16_f<T>(Ks + (size_t)j * D + vs * VEC, kvv);
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      float d = 0.f;
      if (j < n && have_k) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) d = fmaf(qv[g][e], kvv[e], d);
      }
#pragma unroll
      for (int o = LPK / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      if (vs == 0 && j < n) sc[g * kAttnChunk + j] = d * a.scale;
    }
  }
  __syncthreads();

  // Softmax statistics of this chunk, one warp per query head.
  for (int g = warp; g < G; g += NW) {
    float mx = -INFINITY;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[g * kAttnChunk + j]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float pj = expf(sc[g * kAttnChunk + j] - mx);
      sc[g * kAttnChunk + j] = pj;
      sum += pj;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      stat[2 * g] = mx;
      stat[2 * g + 1] = sum;
    }
  }
  __syncthreads();

  // Unnormalised output: thread (group, head, slice) walks its share of keys.
  const bool have_v = mbar_wait(&bar[1], 0, a.err);
  for (int slot = tid; slot < L::kGroups * L::kSlots; slot += blockDim.x) {
    const int grp = slot / L::kSlots, rem = slot % L::kSlots;
    const int g = rem / LPK, sl = rem % LPK;
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
    if (g < G && have_v) {
      for (int j = grp; j < n; j += L::kGroups) {
        const float pj = sc[g * kAttnChunk + j];
        float vv[VEC];
        load16_f<T>(Vs + (size_t)j * D + sl * VEC, vv);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] = fmaf(pj, vv[e], acc[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) red[(grp * GM + g) * D + sl * VEC + e] = acc[e];
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float v = 0.f;
#pragma unroll
    for (int grp = 0; grp < L::kGroups; ++grp) v += red[(grp * GM + g) * D + d];
    part[g * (D + 2) + 2 + d] = v;
  }
  for (int g = tid; g < G; g += blockDim.x) {
    part[g * (D + 2)] = stat[2 * g];
    part[g * (D + 2) + 1] = stat[2 * g + 1];
  }
}

template <typename T>
__global__ void attn_combine_kernel(AttnArgs a, int splits) {
  pdl_trigger();
  pdl_wait();
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

template <typename T, int LPK, int GM>
cudaError_t attn_launch_one(const AttnArgs& a, dim3 grid, cudaStream_t s) {
  constexpr int smem = AttnLayout<T, LPK, GM>::kBytes;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_chunk_kernel<T, LPK, GM>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  { const cudaError_t _le = launch_pdl(attn_chunk_kernel<T, LPK, GM>, dim3(grid), dim3(kAttnThreads), smem, s, a); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

template <typename T, int LPK>
cudaError_t attn_launch_g(const AttnArgs& a, dim3 grid, int G, cudaStream_t s) {
  if constexpr (LPK * Vec16<T>::N > 128) {
    return cudaErrorInvalidValue;  // head_dim above 128 is rejected at stage creation
  } else {
    if (G <= 1) return attn_launch_one<T, LPK, 1>(a, grid, s);
    if (G <= 2) return attn_launch_one<T, LPK, 2>(a, grid, s);
    if (G <= 4) return attn_launch_one<T, LPK, 4>(a, grid, s);
    return attn_launch_one<T, LPK, 8>(a, grid, s);
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
  const size_t simt = (size_t)M * nq * splits * (D + 2);
  const size_t tc = attention_tc_scratch_elems(nq, D);
  return simt > tc ? simt : tc;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s) {
  const int M = a.B * a.S;
  if (M == 0) return cudaSuccess;
  const int splits = (a.max_keys + kAttnChunk - 1) / kAttnChunk;
  if (attention_scratch_elems(M, a.nq, a.D, a.max_keys) > a.partial_elems)
    return cudaErrorInvalidValue;
  if (a.use_tc && attention_prefill_tc_applicable(a.dtype, a.D, a.nq / a.nkv, a.S))
    return launch_attention_prefill_tc(a, s);  // query tiles on tcgen05, scores and output in TMEM
  if (a.use_tc && attention_tc_applicable(a.dtype, a.D, a.nq / a.nkv))
    return launch_attention_tc(a, splits, s);  // merges its chunks itself
  dim3 grid(M, a.nkv, splits);
  const cudaError_t e =
      (a.dtype == kBF16) ? attn_launch<__nv_bfloat16>(a, grid, s) : attn_launch<float>(a, grid, s);
  if (e != cudaSuccess) return e;
  dim3 cgrid(M, a.nq);
  const int threads = a.D < 128 ? a.D : 128;
  if (a.dtype == kBF16)
    { const cudaError_t _le = launch_pdl(attn_combine_kernel<__nv_bfloat16>, dim3(cgrid), dim3(threads), 0, s, a, splits); if (_le != cudaSuccess) return _le; }
  else
    { const cudaError_t _le = launch_pdl(attn_combine_kernel<float>, dim3(cgrid), dim3(threads), 0, s, a, splits); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

}  // namespace mg
