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

#include <algorithm>

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

// The row's probabilities are computed once into `pr` (fp32, the row's slice
// of a scratch buffer, 16-byte aligned); every search pass then reads them
// back (L2) instead of recomputing an exponential per token.  Thread t owns
// the 4-element groups t, t + blockDim, ... in every pass, so it only reads
// values it wrote itself, except in the final rank scan (after a barrier).
template <typename T>
__global__ void __launch_bounds__(kSampleThreads) top_p_kernel(const T* __restrict__ logits,
                                                               int vocab, int64_t stride,
                                                               float temperature, float top_p,
                                                               const float* __restrict__ uniforms,
                                                               int64_t* __restrict__ ids,
                                                               float* __restrict__ scratch,
                                                               int64_t scratch_stride) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  __shared__ int cnt_s[32];
  const T* row = logits + (size_t)blockIdx.x * stride;
  float* pr = scratch + (size_t)blockIdx.x * scratch_stride;
  const int groups = (vocab + 3) / 4;

  // softmax(logits.float() / temperature) in fp32.
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) mx = fmaxf(mx, scaled<T>(row, i, temperature));
  mx = block_reduce_max(mx, red);
  float se = 0.f;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) se += expf(scaled<T>(row, i, temperature) - mx);
  se = block_reduce_sum(se, red);
  for (int g = threadIdx.x; g < groups; g += blockDim.x) {
    float4 q;
    float* qq = &q.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * g + e;
      qq[e] = i < vocab ? expf(scaled<T>(row, i, temperature) - mx) / se : -1.f;  // -1: past the row
    }
    reinterpret_cast<float4*>(pr)[g] = q;
  }

  auto mass_gt = [&](float v) {
    float acc = 0.f;
    for (int g = threadIdx.x; g < groups; g += blockDim.x) {
      const float4 q = reinterpret_cast<const float4*>(pr)[g];
      if (q.x > v) acc += q.x;
      if (q.y > v) acc += q.y;
      if (q.z > v) acc += q.z;
      if (q.w > v) acc += q.w;
    }
    return block_reduce_sum(acc, red);
  };
  auto count_eq = [&](float v) {
    int c = 0;
    for (int g = threadIdx.x; g < groups; g += blockDim.x) {
      const float4 q = reinterpret_cast<const float4*>(pr)[g];
      c += (q.x == v) + (q.y == v) + (q.z == v) + (q.w == v);
    }
    c = __reduce_add_sync(0xffffffffu, c);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) cnt_s[warp] = c;
    __syncthreads();
    int t = lane < (int)(blockDim.x >> 5) ? cnt_s[lane] : 0;
    return __reduce_add_sync(0xffffffffu, t);
  };
  // Smallest non-negative float v (by bit pattern) with mass_gt(v) <= target;
  // every v at or above the largest probability qualifies.  (A 32-way search
  // with per-thread buckets in shared memory was measured slower: each pass
  // then costs more than the passes it saves.)
  auto search = [&](float target, uint32_t hi) {
    uint32_t lo = 0u;
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo) / 2;
      if (mass_gt(__uint_as_float(mid)) <= target) hi = mid;
      else lo = mid + 1;
    }
    return __uint_as_float(lo);
  };
  const uint32_t top = __float_as_uint(1.0f / se);  // the largest probability, exp(0) / se

  // (1) The kept prefix.
  const float bstar = search(top_p, top);
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
  const float w = search(x, top);
  const float gt_w = mass_gt(w);
  const int cnt_w = count_eq(w);
  int limit = (w == bstar) ? keep_b : cnt_w;
  if (limit < 1) limit = 1;
  int rank = w > 0.f ? (int)floorf((x - gt_w) / w) : 0;
  rank = max(0, min(rank, limit - 1));

  // (3) The token holding that rank among the indices with p == w: thread t
  // counts its contiguous run of indices, an exclusive scan over threads
  // finds the run holding the rank, and that thread walks its run.
  __syncthreads();  // every probability written above is visible to the block
  const int run = (vocab + blockDim.x - 1) / blockDim.x;
  const int i0 = threadIdx.x * run, i1 = min(vocab, i0 + run);
  int mine = 0;
  for (int i = i0; i < i1; ++i) mine += pr[i] == w;
  // exclusive scan of `mine` over the block
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  __syncthreads();
  if (lane == 31) cnt_s[warp] = incl;
  __syncthreads();
  int before = incl - mine;
  for (int k = 0; k < warp; ++k) before += cnt_s[k];
  __shared__ int found;
  if (threadIdx.x == 0) found = -1;
  __syncthreads();
  if (mine > 0 && rank >= before && rank < before + mine) {
    int k = before;
    for (int i = i0; i < i1; ++i)
      if (pr[i] == w) {
        if (k == rank) {
          found = i;
          break;
        }
        ++k;
      }
  }
  __syncthreads();
  if (threadIdx.x == 0) ids[blockIdx.x] = found >= 0 ? found : 0;
}

// ---------------------------------------------------------------------------
// Top-p over bf16 logits by value histogram.
//
// Every token of one bf16 value has the same probability, so a row's
// histogram of values (65536 bins, hist_bin order = value order) holds the
// whole sorted distribution, tie groups included: the sort of
// top_p_sample becomes a scan over the bins from the largest value down.
// The histogram comes from the lm_head's epilogue (kEpiHist) or from
// logit_hist_kernel.  top_p_select_kernel, one CTA per row, then
//   1. finds the largest value present (m) and the softmax denominator
//      Z0 = sum over bins of count * exp(v / T - m / T),
//   2. gives each bin its probability p = exp(v / T - m / T) / Z0 and the
//      mass of the bins above it (gt), and keeps
//      min(count, floor((top_p - gt) / p) + 1) of its tokens when
//      gt <= top_p (the reference keeps a token while the mass before it is
//      <= top_p: sampling.py:85-88),
//   3. draws x = u * (kept mass) and finds the bin and the rank inside it
//      where the kept mass first exceeds x,
//   4. clears its histogram for the next launch and returns the token of
//      that rank among the row's indices of that value (index order, the
//      stable sort's tie order).
// Sums run in one fixed order (bins in order within a warp's slab, a fixed
// butterfly across its lanes, warps in order), so a seeded draw is
// reproducible.
// ---------------------------------------------------------------------------

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kWarpBins = kHistBins / kSelWarps;  // 2048 bins per warp
constexpr int kSlabs = kWarpBins / 32;            // 64 slabs of 32 bins
constexpr int kMaxCand = 4096;                    // tie-group indices gathered in shared memory

__global__ void logit_hist_kernel(const __nv_bfloat16* __restrict__ logits, int vocab, int64_t stride,
                                  int* __restrict__ hist) {
  pdl_trigger();
  pdl_wait();
  const __nv_bfloat16* row = logits + (size_t)blockIdx.y * stride;
  int* h = hist + (size_t)blockIdx.y * kHistBins;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x)
    atomicAdd(h + hist_bin(__bfloat162float(row[i])), 1);
}

__device__ __forceinline__ float warp_incl_scan(float v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

__global__ void __launch_bounds__(kSelThreads) top_p_select_kernel(
    const __nv_bfloat16* __restrict__ logits, int vocab, int64_t stride, int* __restrict__ hist,
    float temperature, float top_p, const float* __restrict__ uniforms, int64_t* __restrict__ ids) {
  pdl_trigger();
  pdl_wait();
  __shared__ float wsum[kSelWarps];
  __shared__ float wkept[kSelWarps];
  __shared__ int wfirst[kSelWarps];
  __shared__ int cnt_s[kSelWarps];
  __shared__ int sel_bin, sel_rank, found, n_cand, wide;
  __shared__ int cand[kMaxCand];
  // The row's counts, staged once into shared memory as 16-bit values (the
  // passes below then read shared memory, not L2); a row with a count of
  // 65535 or more in one bin reads its counts from the histogram instead.
  extern __shared__ uint16_t c16[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* h = hist + (size_t)blockIdx.x * kHistBins;
  const __nv_bfloat16* row = logits + (size_t)blockIdx.x * stride;
  if (threadIdx.x == 0) wide = 0;
  __syncthreads();
  {
    int big = 0;
    const int4* h4 = reinterpret_cast<const int4*>(h);
#pragma unroll 4
    for (int i = threadIdx.x; i < kHistBins / 4; i += kSelThreads) {
      const int4 q = __ldcg(h4 + i);
      big |= (q.x >= 0xffff) | (q.y >= 0xffff) | (q.z >= 0xffff) | (q.w >= 0xffff);
      c16[4 * i] = (uint16_t)min(q.x, 0xffff);
      c16[4 * i + 1] = (uint16_t)min(q.y, 0xffff);
      c16[4 * i + 2] = (uint16_t)min(q.z, 0xffff);
      c16[4 * i + 3] = (uint16_t)min(q.w, 0xffff);
    }
    if (big) wide = 1;
  }
  __syncthreads();
  const bool from_l2 = wide != 0;
  // warp w, slab k, lane l: the bin at descending position w·2048 + k·32 + l
  auto bin_at = [&](int k) { return (uint32_t)(kHistBins - 1 - (warp * kWarpBins + k * 32 + lane)); };
  auto count_at = [&](uint32_t b) {
    const int c = from_l2 ? __ldcg(h + b) : (int)c16[b];
    const float v = hist_value(b);
    return (v == v) ? c : 0;  // NaN logits take no part
  };

  // 1. The largest value present, and the denominator.
  int first = INT_MAX;
  for (int k = 0; k < kSlabs; ++k) {
    const unsigned m = __ballot_sync(0xffffffffu, count_at(bin_at(k)) > 0);
    if (m) {
      first = warp * kWarpBins + k * 32 + __ffs(m) - 1;
      break;
    }
  }
  if (lane == 0) wfirst[warp] = first;
  if (threadIdx.x == 0) {
    sel_bin = -1;
    sel_rank = 0;
    found = -1;
  }
  __syncthreads();
  int dmax = INT_MAX;
  for (int i = 0; i < kSelWarps; ++i) dmax = min(dmax, wfirst[i]);
  const float ms = dmax == INT_MAX ? 0.f : hist_value((uint32_t)(kHistBins - 1 - dmax)) / temperature;
  // A slab without tokens adds exactly +0 to every sum and scan below, so
  // it is skipped (most of the 65536 values are absent from a row).
  float acc = 0.f;
  for (int k = 0; k < kSlabs; ++k) {
    const uint32_t b = bin_at(k);
    const int c = count_at(b);
    if (!__ballot_sync(0xffffffffu, c > 0)) continue;
    acc += warp_sum(c > 0 ? (float)c * expf(hist_value(b) / temperature - ms) : 0.f);
  }
  if (lane == 0) wsum[warp] = acc;
  __syncthreads();
  float z0 = 0.f;
  for (int i = 0; i < kSelWarps; ++i) z0 += wsum[i];
  __syncthreads();

  // 2. The mass above each warp's bins, then each bin's kept count.
  auto prob = [&](uint32_t b) { return expf(hist_value(b) / temperature - ms) / z0; };
  acc = 0.f;
  for (int k = 0; k < kSlabs; ++k) {
    const uint32_t b = bin_at(k);
    const int c = count_at(b);
    if (!__ballot_sync(0xffffffffu, c > 0)) continue;
    acc += warp_sum(c > 0 ? (float)c * prob(b) : 0.f);
  }
  if (lane == 0) wsum[warp] = acc;
  __syncthreads();
  float above = 0.f;  // mass of the bins before this warp's range
  for (int i = 0; i < warp; ++i) above += wsum[i];
  // Walk this warp's slabs; `visit(k, gt, c, p, kept)` sees each bin of every
  // slab that holds a token.
  auto walk = [&](auto&& visit) {
    float carry = above;
    for (int k = 0; k < kSlabs; ++k) {
      const uint32_t b = bin_at(k);
      const int c = count_at(b);
      if (!__ballot_sync(0xffffffffu, c > 0)) continue;  // nothing kept, no mass: the carry stands
      const float p = c > 0 ? prob(b) : 0.f;
      const float mass = (float)c * p;
      const float incl = warp_incl_scan(mass, lane);
      const float gt = carry + (incl - mass);
      int kept = 0;
      if (c > 0 && gt <= top_p) kept = p > 0.f ? (int)fminf((float)c, floorf((top_p - gt) / p) + 1.0f) : c;
      if (!visit(k, b, c, p, kept)) return;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
  };
  float kacc = 0.f;
  walk([&](int, uint32_t, int, float p, int kept) {
    kacc += warp_sum((float)kept * p);
    return true;
  });
  if (lane == 0) wkept[warp] = kacc;
  __syncthreads();
  float ztot = 0.f, before = 0.f;
  for (int i = 0; i < kSelWarps; ++i) {
    if (i < warp) before += wkept[i];
    ztot += wkept[i];
  }
  const float x = uniforms[blockIdx.x] * ztot;
  // The drawing warp: the first whose kept mass reaches past x (or the last
  // with any kept mass, when rounding puts x at the very end).
  int target = -1, last_nonzero = -1;
  {
    float run = 0.f;
    for (int i = 0; i < kSelWarps; ++i) {
      if (wkept[i] > 0.f) last_nonzero = i;
      if (target < 0 && wkept[i] > 0.f && run + wkept[i] > x) target = i;
      run += wkept[i];
    }
    if (target < 0) target = last_nonzero;
  }

  // 3. The drawn bin and the rank inside it.
  if (warp == target) {
    float kcarry = before;
    int last_b = -1, last_k = 0;
    walk([&](int, uint32_t b, int, float p, int kept) {
      const float km = (float)kept * p;
      const float kincl = warp_incl_scan(km, lane);
      const unsigned hit = __ballot_sync(0xffffffffu, kept > 0 && kcarry + kincl > x);
      const unsigned any = __ballot_sync(0xffffffffu, kept > 0);
      if (any) {
        const int hl = 31 - __clz(any);
        last_b = __shfl_sync(0xffffffffu, (int)b, hl);
        last_k = __shfl_sync(0xffffffffu, kept, hl);
      }
      if (hit) {
        const int l = __ffs(hit) - 1;
        if (lane == l) {
          const float lo = kcarry + (kincl - km);
          int rank = p > 0.f ? (int)floorf((x - lo) / p) : 0;
          rank = max(0, min(rank, kept - 1));
          sel_bin = (int)b;
          sel_rank = rank;
        }
        return false;
      }
      kcarry += __shfl_sync(0xffffffffu, kincl, 31);
      return true;
    });
    if (lane == 0 && sel_bin < 0 && last_b >= 0) {  // x at the very end of the kept mass
      sel_bin = last_b;
      sel_rank = last_k - 1;
    }
  }
  __syncthreads();

  // 4. Clear the histogram; find the token of that rank.
  {
    int4* h4 = reinterpret_cast<int4*>(h);
    for (int i = threadIdx.x; i < kHistBins / 4; i += kSelThreads) h4[i] = make_int4(0, 0, 0, 0);
  }
  if (sel_bin < 0) {  // no finite logits
    if (threadIdx.x == 0) ids[blockIdx.x] = 0;
    return;
  }
  const float wv = hist_value((uint32_t)sel_bin);
  const int rank = sel_rank;
  if (threadIdx.x == 0) n_cand = 0;
  __syncthreads();
  // The tie group's indices, gathered with coalesced loads (unordered); the
  // token is the one with exactly `rank` smaller indices in the group.
  auto take = [&](int i) {
    const int slot = atomicAdd(&n_cand, 1);
    if (slot < kMaxCand) cand[slot] = i;
  };
  if ((stride % 8) == 0 && ((uintptr_t)row % 16) == 0) {  // 16-byte loads of 8 logits
    const uint4* r4 = reinterpret_cast<const uint4*>(row);
    for (int g8 = threadIdx.x; g8 < vocab / 8; g8 += kSelThreads) {
      const uint4 q = r4[g8];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (__bfloat162float(e[j]) == wv) take(8 * g8 + j);
    }
    for (int i = vocab / 8 * 8 + threadIdx.x; i < vocab; i += kSelThreads)
      if (__bfloat162float(row[i]) == wv) take(i);
  } else {
    for (int i = threadIdx.x; i < vocab; i += kSelThreads)
      if (__bfloat162float(row[i]) == wv) take(i);
  }
  __syncthreads();
  const int nc = n_cand;
  if (nc <= kMaxCand) {
    for (int j = threadIdx.x; j < nc; j += kSelThreads) {
      const int me = cand[j];
      int smaller = 0;
      for (int k = 0; k < nc; ++k) smaller += cand[k] < me;
      if (smaller == rank) found = me;
    }
  } else {
    // ordered runs: thread t counts its contiguous run, an exclusive scan
    // over threads finds the run holding the rank, that thread walks it
    const int run = (vocab + kSelThreads - 1) / kSelThreads;
    const int i0 = threadIdx.x * run, i1 = min(vocab, i0 + run);
    int mine = 0;
    for (int i = i0; i < i1; ++i) mine += __bfloat162float(row[i]) == wv;
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) cnt_s[warp] = incl;
    __syncthreads();
    int prior = incl - mine;
    for (int k = 0; k < warp; ++k) prior += cnt_s[k];
    if (mine > 0 && rank >= prior && rank < prior + mine) {
      int k = prior;
      for (int i = i0; i < i1; ++i)
        if (__bfloat162float(row[i]) == wv) {
          if (k == rank) {
            found = i;
            break;
          }
          ++k;
        }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) ids[blockIdx.x] = found >= 0 ? found : 0;
}

}  // namespace

int* top_p_hist_buffer(int rows) {
  static int* buf[64] = {};
  static size_t cap[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || rows < 0) return nullptr;
  const size_t need = (size_t)(rows > 0 ? rows : 1) * kHistBins;
  if (need > cap[dev]) {
    if (buf[dev]) {
      cudaDeviceSynchronize();
      cudaFree(buf[dev]);
      buf[dev] = nullptr;
      cap[dev] = 0;
    }
    if (cudaMalloc(&buf[dev], need * sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(buf[dev], 0, need * sizeof(int)) != cudaSuccess) return nullptr;
    cap[dev] = need;
  }
  return buf[dev];
}

cudaError_t launch_logit_hist(const void* logits, int rows, int vocab, int64_t stride, int* hist,
                              cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const int blocks = std::min(64, (vocab + 255) / 256);
  const cudaError_t e = launch_pdl(logit_hist_kernel, dim3(blocks, rows), dim3(256), 0, s,
                                   (const __nv_bfloat16*)logits, vocab, stride, hist);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_top_p_select(const void* logits, int rows, int vocab, int64_t stride, int* hist,
                                float temperature, float top_p, const float* uniforms, int64_t* ids,
                                cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  constexpr int smem = kHistBins * (int)sizeof(uint16_t);  // 128 KB of staged counts
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(top_p_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const cudaError_t e = launch_pdl(top_p_select_kernel, dim3(rows), dim3(kSelThreads), smem, s,
                                   (const __nv_bfloat16*)logits, vocab, stride, hist, temperature, top_p,
                                   uniforms, ids);
  return e != cudaSuccess ? e : cudaGetLastError();
}

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
  if (dtype == kBF16) {  // by value histogram (see top_p_select_kernel)
    int* hist = top_p_hist_buffer(rows);
    if (!hist) return cudaErrorMemoryAllocation;
    cudaError_t e = launch_logit_hist(logits, rows, vocab, stride, hist, s);
    if (e != cudaSuccess) return e;
    return launch_top_p_select(logits, rows, vocab, stride, hist, temperature, top_p, uniforms, ids, s);
  }
  // fp32 logits: the rows' probabilities: a per-device scratch buffer, grown on demand
  // (the growth synchronises the device once).
  static float* scratch[64] = {};
  static size_t scratch_elems[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const int64_t pstride = ((int64_t)vocab + 3) / 4 * 4;
  const size_t need = (size_t)rows * (size_t)pstride;
  if (need > scratch_elems[dev]) {
    if (scratch[dev]) {
      cudaDeviceSynchronize();
      cudaFree(scratch[dev]);
      scratch[dev] = nullptr;
      scratch_elems[dev] = 0;
    }
    const cudaError_t e = cudaMalloc(&scratch[dev], need * sizeof(float));
    if (e != cudaSuccess) return e;
    scratch_elems[dev] = need;
  }
  if (dtype == kBF16)
    { const cudaError_t _le = launch_pdl(top_p_kernel<__nv_bfloat16>, dim3(rows), dim3(kSampleThreads), 0, s,
        (const __nv_bfloat16*)logits, vocab, stride, temperature, top_p, uniforms, ids, scratch[dev], pstride); if (_le != cudaSuccess) return _le; }
  else
    { const cudaError_t _le = launch_pdl(top_p_kernel<float>, dim3(rows), dim3(kSampleThreads), 0, s, (const float*)logits, vocab, stride,
                                                        temperature, top_p, uniforms, ids, scratch[dev], pstride); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

}  // namespace mg
