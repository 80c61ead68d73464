// Linear layers Y = epilogue(X · Wᵀ) with W in nn.Linear layout [N, K].
//
// Two kernels live here:
//  * gemv_mma: the decode path (bf16, M <= 32 token rows).  Decode is a pure
//    weight stream, so the kernel is built around HBM bandwidth: each lane
//    issues 16-byte loads of W, the tensor cores (mma.sync m16n8k16, swap-AB:
//    weight rows are the MMA's M dimension, tokens its N dimension) do the
//    arithmetic, and K is split across warps and, when the output is narrow,
//    across CTAs with an fp32 partial buffer reduced by a second kernel.
//    Because a dot product does not depend on the order of its terms, the
//    kernel uses one fixed permutation of each 32-wide K chunk for both A and
//    B so that every fragment register comes from a single 16-byte load.
//  * linear_simt: fp32 models (the fp32 parity configuration) and shapes the
//    tensor-core kernels do not take.
//
// Epilogues mirror the reference's rounding points: nn.Linear returns a
// rounded tensor; residual adds round again (llama_dense.py:279-280); SwiGLU
// rounds gate, up, silu(gate) and the product (llama_dense.py:243-244).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "linear_tc.h"

namespace mg {
namespace {

using bf16 = __nv_bfloat16;

template <typename T, int EPI>
__device__ __forceinline__ void epi_write(const LinearArgs& a, int tok, int n, float v, float vu) {
  T* Y = (T*)a.Y + (size_t)tok * a.ldy + n;
  if (EPI == kEpiStore) {
    stf<T>(Y, v);
  } else if (EPI == kEpiResid) {
    const float r = ldf<T>((const T*)a.R + (size_t)tok * a.ldr + n);
    stf<T>(Y, r + rt<T>(v));
  } else {
    const float g = rt<T>(v), u = rt<T>(vu);
    const float sg = rt<T>(g / (1.0f + expf(-g)));
    stf<T>(Y, sg * u);
  }
}

// ---------------------------------------------------------------------------
// SIMT tiled GEMM (fp32 models and odd shapes).
// ---------------------------------------------------------------------------
template <typename T, int EPI>
__global__ void __launch_bounds__(256) linear_simt_kernel(LinearArgs a) {
  pdl_trigger();
  pdl_wait();
  constexpr int BM = 64, BN = 64, BK = 16;
  constexpr int NB = (EPI == kEpiSwiGLU) ? 2 : 1;
  __shared__ float Xs[BK][BM + 4];
  __shared__ float Ws[NB][BK][BN + 4];
  const T* X = (const T*)a.X;
  const T* W = (const T*)a.W;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[NB][4][4];
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[b][i][j] = 0.f;

  for (int k0 = 0; k0 < a.K; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      const int r = i / BK, c = i % BK, m = m0 + r, k = k0 + c;
      Xs[c][r] = (m < a.M && k < a.K) ? ldf<T>(X + (size_t)m * a.ldx + k) : 0.f;
    }
#pragma unroll
    for (int b = 0; b < NB; ++b)
      for (int i = threadIdx.x; i < BN * BK; i += 256) {
        const int r = i / BK, c = i % BK, n = n0 + r, k = k0 + c;
        Ws[b][c][r] =
            (n < a.N && k < a.K) ? ldf<T>(W + (size_t)(n + b * a.N) * a.K + k) : 0.f;
      }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float xa[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) xa[i] = Xs[kk][ty * 4 + i];
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        float wb[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) wb[j] = Ws[b][kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[b][i][j] = fmaf(xa[i], wb[j], acc[b][i][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < a.M && n < a.N) epi_write<T, EPI>(a, m, n, acc[0][i][j], acc[NB - 1][i][j]);
    }
}

// ---------------------------------------------------------------------------
// Decode GEMV on tensor cores (bf16, M <= 8*MT).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint4 ld_stream(const bf16* p) {
  // Weights are read once per step: do not keep them in L1.
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t u4_at(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

constexpr int kGemvRG = 4;   // row groups of 16 per CTA
constexpr int kGemvU = 2;    // 32-wide K chunks per warp iteration
constexpr int kGemvNW = 4;   // warps per CTA
constexpr int kGemvChunk = 32 * kGemvU;

// blockIdx.x: output tile; blockIdx.y: K split.  Output rows of a tile:
// store/resid: [64*tile, 64*tile+64); SwiGLU: gate rows [32*tile, +32) and the
// matching up rows N + [32*tile, +32).
template <int MT, int EPI>
__global__ void __launch_bounds__(kGemvNW * 32) gemv_mma_kernel(LinearArgs a, int chunks_per_split) {
  pdl_trigger();
  pdl_wait();
  constexpr int RG = kGemvRG, U = kGemvU, NW = kGemvNW;
  const bf16* __restrict__ X = (const bf16*)a.X;
  const bf16* __restrict__ W = (const bf16*)a.W;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;

  int rbase[RG];
  bool rvalid[RG];
  if (EPI == kEpiSwiGLU) {
    const int f0 = blockIdx.x * 16 * (RG / 2);
#pragma unroll
    for (int i = 0; i < RG / 2; ++i) {
      rbase[i] = f0 + 16 * i;
      rvalid[i] = rbase[i] < a.N;
      rbase[RG / 2 + i] = a.N + rbase[i];
      rvalid[RG / 2 + i] = rvalid[i];
    }
  } else {
    const int f0 = blockIdx.x * 16 * RG;
#pragma unroll
    for (int i = 0; i < RG; ++i) {
      rbase[i] = f0 + 16 * i;
      rvalid[i] = rbase[i] < a.N;
    }
  }

  const int nchunks = a.K / kGemvChunk;
  const int kc_begin = blockIdx.y * chunks_per_split;
  const int kc_end = min(kc_begin + chunks_per_split, nchunks);

  float acc[RG][MT][4];
#pragma unroll
  for (int i = 0; i < RG; ++i)
#pragma unroll
    for (int j = 0; j < MT; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.f;

  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int kc = kc_begin + warp; kc < kc_end; kc += NW) {
    const int kb = kc * kGemvChunk + 8 * t;
    uint4 wv[RG][2][U];
    uint4 xv[MT][U];
#pragma unroll
    for (int i = 0; i < RG; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int u = 0; u < U; ++u)
          wv[i][h][u] = rvalid[i] ? ld_stream(W + (size_t)(rbase[i] + g + 8 * h) * a.K + kb + 32 * u)
                                  : zero;
#pragma unroll
    for (int j = 0; j < MT; ++j) {
      const int n = 8 * j + g;
#pragma unroll
      for (int u = 0; u < U; ++u)
        xv[j][u] = (n < a.M) ? __ldg(reinterpret_cast<const uint4*>(X + (size_t)n * a.ldx + kb + 32 * u))
                             : zero;
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int s = 0; s < 2; ++s)
#pragma unroll
        for (int i = 0; i < RG; ++i) {
          const uint32_t af[4] = {u4_at(wv[i][0][u], 2 * s), u4_at(wv[i][1][u], 2 * s),
                                  u4_at(wv[i][0][u], 2 * s + 1), u4_at(wv[i][1][u], 2 * s + 1)};
#pragma unroll
          for (int j = 0; j < MT; ++j) {
            const uint32_t bfr[2] = {u4_at(xv[j][u], 2 * s), u4_at(xv[j][u], 2 * s + 1)};
            mma_16816(acc[i][j], af, bfr);
          }
        }
  }

  // Reduce the per-warp partial sums of the tile.
  constexpr int E = RG * MT * 4;
  __shared__ float red[NW][E][32];
#pragma unroll
  for (int i = 0; i < RG; ++i)
#pragma unroll
    for (int j = 0; j < MT; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) red[warp][(i * MT + j) * 4 + c][lane] = acc[i][j][c];
  __syncthreads();
  for (int idx = threadIdx.x; idx < E * 32; idx += NW * 32) {
    const int e = idx >> 5, ln = idx & 31;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) v += red[w][e][ln];
    red[0][e][ln] = v;
  }
  __syncthreads();

  const bool split = gridDim.y > 1;
  const int ncols = (EPI == kEpiSwiGLU) ? 2 * a.N : a.N;
  constexpr int IG = (EPI == kEpiSwiGLU) ? RG / 2 : RG;
  for (int idx = threadIdx.x; idx < IG * MT * 4 * 32; idx += NW * 32) {
    const int ln = idx & 31, c = (idx >> 5) & 3, j = (idx >> 7) % MT, i = (idx >> 7) / MT;
    const int gg = ln >> 2, tt = ln & 3;
    const int tok = 8 * j + 2 * tt + (c & 1);
    const int r = gg + 8 * (c >> 1);
    if (!rvalid[i] || tok >= a.M) continue;
    const float v = red[0][(i * MT + j) * 4 + c][ln];
    const float vu = (EPI == kEpiSwiGLU) ? red[0][((i + RG / 2) * MT + j) * 4 + c][ln] : 0.f;
    const int n = rbase[i] + r;
    if (split) {
      float* P = a.partial + ((size_t)blockIdx.y * a.M + tok) * ncols;
      P[n] = v;
      if (EPI == kEpiSwiGLU) P[a.N + n] = vu;
    } else {
      epi_write<bf16, EPI>(a, tok, n, v, vu);
    }
  }
}

template <typename T, int EPI>
__global__ void splitk_reduce_kernel(LinearArgs a, int ksplit) {
  pdl_trigger();
  pdl_wait();
  const int ncols = (EPI == kEpiSwiGLU) ? 2 * a.N : a.N;
  const size_t total = (size_t)a.M * a.N;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int tok = (int)(idx / a.N), n = (int)(idx % a.N);
    float v = 0.f, vu = 0.f;
    for (int s = 0; s < ksplit; ++s) {
      const float* P = a.partial + ((size_t)s * a.M + tok) * ncols;
      v += P[n];
      if (EPI == kEpiSwiGLU) vu += P[a.N + n];
    }
    epi_write<T, EPI>(a, tok, n, v, vu);
  }
}

struct GemvPlan {
  int mt, tiles, ksplit, cps;
};

bool gemv_applicable(int dtype, int M, int N, int K) {
  return dtype == kBF16 && M >= 1 && M <= 32 && K % kGemvChunk == 0 && N % 16 == 0;
}

GemvPlan gemv_plan(int M, int N, int K, int epi) {
  GemvPlan p;
  p.mt = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  p.tiles = (epi == kEpiSwiGLU) ? (N + 31) / 32 : (N + 63) / 64;
  const int nchunks = K / kGemvChunk;
  const int target = 148 * 4;
  int ks = (target + p.tiles - 1) / p.tiles;
  ks = std::min(ks, std::max(1, nchunks / kGemvNW));
  if (ks < 1) ks = 1;
  p.cps = (nchunks + ks - 1) / ks;
  p.ksplit = (nchunks + p.cps - 1) / p.cps;
  return p;
}

template <int MT, int EPI>
cudaError_t gemv_launch(const LinearArgs& a, const GemvPlan& p, cudaStream_t s) {
  dim3 grid(p.tiles, p.ksplit);
  { const cudaError_t _le = launch_pdl(gemv_mma_kernel<MT, EPI>, dim3(grid), dim3(kGemvNW * 32), 0, s, a, p.cps); if (_le != cudaSuccess) return _le; }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || p.ksplit == 1) return e;
  const int blocks = (int)std::min<size_t>(((size_t)a.M * a.N + 255) / 256, 148 * 8);
  { const cudaError_t _le = launch_pdl(splitk_reduce_kernel<bf16, EPI>, dim3(blocks), dim3(256), 0, s, a, p.ksplit); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

template <int EPI>
cudaError_t gemv_dispatch(const LinearArgs& a, const GemvPlan& p, cudaStream_t s) {
  switch (p.mt) {
    case 1: return gemv_launch<1, EPI>(a, p, s);
    case 2: return gemv_launch<2, EPI>(a, p, s);
    default: return gemv_launch<4, EPI>(a, p, s);
  }
}

template <typename T, int EPI>
cudaError_t simt_launch(const LinearArgs& a, cudaStream_t s) {
  dim3 grid((a.N + 63) / 64, (a.M + 63) / 64);
  { const cudaError_t _le = launch_pdl(linear_simt_kernel<T, EPI>, dim3(grid), dim3(256), 0, s, a); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

template <typename T>
cudaError_t simt_dispatch(const LinearArgs& a, cudaStream_t s) {
  switch (a.epilogue) {
    case kEpiStore: return simt_launch<T, kEpiStore>(a, s);
    case kEpiResid: return simt_launch<T, kEpiResid>(a, s);
    default: return simt_launch<T, kEpiSwiGLU>(a, s);
  }
}

}  // namespace

size_t linear_scratch_elems(int dtype, int M, int N, int K, int epilogue) {
  if (gemv_tc_applicable(dtype, M, N, K)) return gemv_tc_scratch_elems(M, N, K, epilogue, true);
  if (gemv_applicable(dtype, M, N, K)) {
    const GemvPlan p = gemv_plan(M, N, K, epilogue);
    if (p.ksplit <= 1) return 0;
    const size_t ncols = (epilogue == kEpiSwiGLU) ? 2 * (size_t)N : (size_t)N;
    return (size_t)p.ksplit * M * ncols;
  }
  if (linear_tc_applicable(dtype, M, N, K)) return linear_tc_scratch_elems(M, N, K, epilogue);
  return 0;
}

cudaError_t launch_linear(const LinearArgs& a, cudaStream_t s) {
  if (a.M == 0) return cudaSuccess;
  if (gemv_tc_applicable(a.dtype, a.M, a.N, a.K)) return launch_gemv_tc(a, s);
  if (a.epilogue == kEpiPieces || a.epilogue == kEpiGreedy || a.epilogue == kEpiHist)
    return cudaErrorInvalidValue;  // decode GEMM only
  if (gemv_applicable(a.dtype, a.M, a.N, a.K)) {
    GemvPlan p = gemv_plan(a.M, a.N, a.K, a.epilogue);
    if (p.ksplit > 1 &&
        (size_t)p.ksplit * a.M * ((a.epilogue == kEpiSwiGLU) ? 2 * (size_t)a.N : (size_t)a.N) >
            a.partial_elems) {
      return cudaErrorInvalidValue;  // caller under-sized the split-K scratch
    }
    switch (a.epilogue) {
      case kEpiStore: return gemv_dispatch<kEpiStore>(a, p, s);
      case kEpiResid: return gemv_dispatch<kEpiResid>(a, p, s);
      default: return gemv_dispatch<kEpiSwiGLU>(a, p, s);
    }
  }
  if (linear_tc_applicable(a.dtype, a.M, a.N, a.K)) return launch_linear_tc(a, s);
  if (a.dtype == kBF16) return simt_dispatch<bf16>(a, s);
  return simt_dispatch<float>(a, s);
}

}  // namespace mg
