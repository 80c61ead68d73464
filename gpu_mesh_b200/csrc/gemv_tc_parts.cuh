// Pieces of the stream-K tcgen05 decode GEMM shared by the single-layer
// kernel (k_gemv_tc.cu) and the layer-chain kernel (k_layer_tc.cu): tile and
// ring geometry, the stream-K split, the epilogue-warp barriers and the
// epilogues with the reference's rounding points.
#pragma once

#include "kernels.h"
#include "tc_common.cuh"

namespace mg {
namespace gemvtc {

using bf16 = __nv_bfloat16;

constexpr int kRows = 128;
constexpr int kKB = 64;
#ifndef MG_GEMV_STAGES
#define MG_GEMV_STAGES 8
#endif
constexpr int kStagesD = MG_GEMV_STAGES;  // 16 KB of weights per stage in flight per SM
constexpr int kThreadsD = 192;
constexpr int kWBytes = kRows * kKB * 2;

template <int NP>
struct DLayout {
  static constexpr int kX = NP * kKB * 2;
  static constexpr int kStage = kWBytes + kX;  // a multiple of 1024
  static constexpr int kTiles = kStagesD * kStage;
  static constexpr int kXchg = 64 * (NP + 1) * 4;  // padded rows: no bank conflicts
  static constexpr int kBarOff = kTiles + kXchg;
  static constexpr int kBytes = kBarOff + 1024 + 512;
};

struct Part {
  long long total;  // units
  int G, nk, tiles;
  __host__ __device__ long long begin(int c) const { return (long long)c * total / G; }
  __host__ __device__ int owner(long long u) const { return (int)(((u + 1) * G - 1) / total); }
  __host__ __device__ int slot(int c, int t) const { return 2 * c + (t == begin(c) / nk ? 0 : 1); }
};

// Persistent grid size on the current device (usable_sms).
inline int sm_count() {
  return usable_sms();
}

// Tiles of 128 W rows (64 gate + 64 up rows for SwiGLU) x K/64 blocks, cut
// into one contiguous range per CTA.
inline Part make_part(int N, int K, int epi) {
  Part p;
  p.tiles = (epi == kEpiSwiGLU) ? (N + 63) / 64 : (N + kRows - 1) / kRows;
  p.nk = K / kKB;
  p.total = (long long)p.tiles * p.nk;
  p.G = (int)(sm_count() < p.total ? sm_count() : p.total);
  return p;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Barrier over the four epilogue warps that also returns the OR of `pred`
// across them, so every warp takes the same branch afterwards.
__device__ __forceinline__ bool epi_bar_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.red.or.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

// Epilogue of W row r of tile t for tokens [m_lo, m_hi) (clipped to M).
template <int NP, int EPI>
__device__ __forceinline__ void apply(const LinearArgs& a, int t, int r, const float* v, float* xchg,
                                      int m_lo = 0, int m_hi = NP) {
  if (m_hi > a.M) m_hi = a.M;
  if (EPI == kEpiSwiGLU) {
    // rows 0-63 gate, 64-127 up of features 64t .. 64t+63
    if (r >= 64) {
#pragma unroll
      for (int i = 0; i < NP; ++i)
        if (i >= m_lo && i < m_hi) xchg[(r - 64) * (NP + 1) + i] = v[i];
    }
    epi_bar();
    if (r < 64) {
      const int f = t * 64 + r;
      if (f < a.N) {
        bf16* Y = (bf16*)a.Y + f;
#pragma unroll
        for (int tok = 0; tok < NP; ++tok) {
          if (tok < m_lo || tok >= m_hi) continue;
          const float g = rt<bf16>(v[tok]), u = rt<bf16>(xchg[r * (NP + 1) + tok]);
          const float sg = rt<bf16>(g / (1.0f + expf(-g)));
          Y[(size_t)tok * a.ldy] = __float2bfloat16_rn(sg * u);
        }
      }
    }
    epi_bar();
    return;
  }
  const int f = t * kRows + r;
  if (f >= a.N) return;
  bf16* Y = (bf16*)a.Y + f;
  if (EPI == kEpiResid) {
    // R may alias Y, so the compiler cannot hoist a load above the previous
    // token's store: read every residual first, then write.
    const bf16* R = (const bf16*)a.R + f;
    float rr[NP];
#pragma unroll
    for (int tok = 0; tok < NP; ++tok)
      rr[tok] = (tok >= m_lo && tok < m_hi) ? __bfloat162float(R[(size_t)tok * a.ldr]) : 0.f;
#pragma unroll
    for (int tok = 0; tok < NP; ++tok)
      if (tok >= m_lo && tok < m_hi) Y[(size_t)tok * a.ldy] = __float2bfloat16_rn(rr[tok] + rt<bf16>(v[tok]));
  } else if (EPI == kEpiStore || a.Y != nullptr) {
#pragma unroll
    for (int tok = 0; tok < NP; ++tok)
      if (tok >= m_lo && tok < m_hi) Y[(size_t)tok * a.ldy] = __float2bfloat16_rn(v[tok]);
  }
}

// Greedy selection key of a logit: the bf16-rounded value in order-preserving
// bits (NaN above everything, -0 as +0) over the complement of the index, so
// the 64-bit maximum is the largest logit with the lowest index.
__device__ __forceinline__ unsigned long long greedy_key(float v, int index) {
  const float y = __bfloat162float(__float2bfloat16_rn(v));
  uint32_t u = __float_as_uint(y);
  if (y == 0.f) u = 0u;
  const uint32_t ord = (y != y) ? 0xffffffffu : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
  return ((unsigned long long)ord << 32) | (uint32_t)(0xffffffffu - (uint32_t)index);
}

// Count the finished logits of W row r of tile t (every token) into the
// per-token value histograms (kEpiHist).
template <int NP>
__device__ __forceinline__ void hist_fold(const LinearArgs& a, int t, int r, const float* v) {
  const int f = t * kRows + r;
  if (f >= a.N) return;
#pragma unroll
  for (int tok = 0; tok < NP; ++tok)
    if (tok < a.M) atomicAdd(a.hist + (size_t)tok * kHistBins + hist_bin(v[tok]), 1);
}

// Fold the finished logits of W row r of tile t (all tokens) into the
// per-token maxima: a transposing butterfly leaves lane l holding the warp's
// best key of token l (l < NP), then one atomic max per token and warp.
template <int NP>
__device__ __forceinline__ void greedy_fold(const LinearArgs& a, int t, int r, int lane, const float* v) {
  const int f = t * kRows + r;
  unsigned long long k[NP];
#pragma unroll
  for (int tok = 0; tok < NP; ++tok) k[tok] = (f < a.N && tok < a.M) ? greedy_key(v[tok], f) : 0ull;
  if (NP == 16) {
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, k[j], 16);
      k[j] = o > k[j] ? o : k[j];
    }
  }
#pragma unroll
  for (int w = NP / 2; w >= 1; w >>= 1) {
    const bool up = (lane & w) != 0;
#pragma unroll
    for (int j = 0; j < w; ++j) {
      const unsigned long long send = up ? k[j] : k[j + w];
      const unsigned long long keep = up ? k[j + w] : k[j];
      const unsigned long long got = __shfl_xor_sync(0xffffffffu, send, w);
      k[j] = got > keep ? got : keep;
    }
  }
  const int tok = lane & (NP - 1);
  if (lane < NP && tok < a.M && k[0] != 0ull) atomicMax(a.greedy.best + tok, k[0]);
}

// After a CTA's last tile: count it in; the last CTA of the grid turns the
// keys into token ids and clears the buffers for the next launch.  `e` is the
// thread's index among the 128 epilogue threads.
__device__ __forceinline__ void greedy_finish(const LinearArgs& a, int e) {
  __threadfence();
  epi_bar();  // every warp's atomics precede the count
  if (e != 0) return;
  if (tc::atomic_add_acq_rel_gpu(a.greedy.done, 1) != (int)gridDim.x - 1) return;
  for (int tok = 0; tok < a.M; ++tok) {
    const unsigned long long key = __ldcg(a.greedy.best + tok);
    a.greedy.ids[tok] = (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
    a.greedy.best[tok] = 0ull;
  }
  *a.greedy.done = 0;
}

// The fix-up of a split tile by the CTA that completed its count: add the
// pieces' fp32 partial sums of W row r (this thread's accumulator row) in
// CTA order (deterministic).  Loads are issued kBatch pieces at a time so
// the L2 round trips overlap.
template <int NP>
__device__ __forceinline__ void fixup_sum(const Part& p, const float* slots, int t, int r, int c_lo, int c_hi,
                                          float* v) {
#pragma unroll
  for (int i = 0; i < NP; ++i) v[i] = 0.f;
  constexpr int kBatch = NP == 16 ? 4 : 2;
  for (int c0 = c_lo; c0 <= c_hi; c0 += kBatch) {
    float4 buf[kBatch][NP / 4];
#pragma unroll
    for (int b2 = 0; b2 < kBatch; ++b2) {
      if (c0 + b2 > c_hi) break;
      const float4* S = reinterpret_cast<const float4*>(slots + ((size_t)p.slot(c0 + b2, t) * kRows + r) * NP);
#pragma unroll
      for (int i = 0; i < NP / 4; ++i) buf[b2][i] = __ldcg(S + i);
    }
#pragma unroll
    for (int b2 = 0; b2 < kBatch; ++b2) {
      if (c0 + b2 > c_hi) break;
#pragma unroll
      for (int i = 0; i < NP / 4; ++i) {
        v[4 * i] += buf[b2][i].x;
        v[4 * i + 1] += buf[b2][i].y;
        v[4 * i + 2] += buf[b2][i].z;
        v[4 * i + 3] += buf[b2][i].w;
      }
    }
  }
}

// A split tile's piece: store this CTA's sums of row r, count the piece in;
// true if this CTA completed the count, in which case `v` now holds the
// whole tile's sums and the counter is reset.  `e` is the thread's index
// among the 128 epilogue threads.
template <int NP>
__device__ __forceinline__ bool piece_done(const Part& p, float* slots, int* counters, int c, int t, int r,
                                           int e, float* v) {
  float4* S = reinterpret_cast<float4*>(slots + ((size_t)p.slot(c, t) * kRows + r) * NP);
#pragma unroll
  for (int i = 0; i < NP / 4; ++i) S[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  // The barrier orders the four warps' slot writes before thread 0's
  // release; its acquire (then the barrier) orders the other pieces' slots
  // before the reads in fixup_sum.
  epi_bar();
  const int c_lo = p.owner((long long)t * p.nk), c_hi = p.owner((long long)(t + 1) * p.nk - 1);
  bool last = false;
  if (e == 0) last = tc::atomic_add_acq_rel_gpu(&counters[t], 1) == c_hi - c_lo;
  if (!epi_bar_any(last)) return false;  // another CTA finishes this tile
  fixup_sum<NP>(p, slots, t, r, c_lo, c_hi, v);
  if (e == 0) counters[t] = 0;
  return true;
}

}  // namespace gemvtc
}  // namespace mg
