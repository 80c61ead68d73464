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

// Decode rows (bf16, head_dim 64 or 128) from the qkv projection's pieces,
// 16 bytes per lane: VEC = 8 consecutive dims, LPH = D / VEC lanes per head,
// so a warp takes HPW = 32 / LPH heads of one token (a group) at once and
// the rotate-half partner (dims d ± D/2) sits LPH / 2 lanes away.  Warps
// stride over the (token, group) units; each lane sums its dims' pieces
// straight into registers.
constexpr int kVecWarps = 8;

// Streaming multiprocessors of the current device (cached per device).
inline int sm_count_cached() {
  static int n[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

template <typename T, int D>
__global__ void __launch_bounds__(kVecWarps * 32) qkv_post_pieces_kernel(QkvPostArgs a) {
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T), LPH = D / VEC, HPW = 32 / LPH, half = D / 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPH, hl = lane % LPH;
  const int d0 = hl * VEC, dh = d0 % half;
  const bool lower = d0 < half;
  const int nh = a.nq + 2 * a.nkv;
  const int groups = (nh + HPW - 1) / HPW;
  const long long units = (long long)a.B * a.S * groups;
  const long long u_first = (long long)blockIdx.x * kVecWarps + warp;
  // The first unit's row descriptor and rotary table entries do not depend on
  // the kernel before this one (the row table is uploaded before the
  // forward's first kernel, the tables at stage creation; without explicit
  // positions the position follows from the row), so they are read before
  // the programmatic-launch wait, leaving only the piece loads after it.
  const bool early = a.positions == nullptr && u_first < units;
  RowDesc rd0{};
  float c0[VEC], s0[VEC];
  if (early) {
    const int m = (int)(u_first / groups);
    rd0 = a.rows[m / a.S];
    int64_t pos = (int64_t)rd0.past + m % a.S;
    pos = pos < 0 ? 0 : (pos >= a.max_pos ? a.max_pos - 1 : pos);
    load16_f<T>((const T*)a.cos + (size_t)pos * half + dh, c0);
    load16_f<T>((const T*)a.sin + (size_t)pos * half + dh, s0);
  }
  pdl_wait();
  for (long long u = u_first; u < units; u += (long long)gridDim.x * kVecWarps) {
    const bool first = early && u == u_first;
    const int m = (int)(u / groups);
    const int hh = (int)(u % groups) * HPW + sub;
    const bool valid = hh < nh;  // lanes past the last head still join the shuffles
    const int b = m / a.S, s = m % a.S;
    const RowDesc rd = first ? rd0 : a.rows[b];
    const int cache_pos = rd.past + s;
    int64_t pos = a.positions ? a.positions[m] : (int64_t)cache_pos;
    if (pos < 0 || pos >= a.max_pos) {
      if (valid && hl == 0) flag_error(a.err, kErrPositionRange);
      pos = pos < 0 ? 0 : a.max_pos - 1;
    }
    float x[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) x[i] = 0.f;
    if (valid) {
      // the projection's pieces, rounded as its store epilogue would
      if constexpr (VEC == 8) {
        pieces_sum8(a.pieces, m, hh * D + d0, x);
      } else {
        pieces_sum4(a.pieces, m, hh * D + d0, x);
      }
#pragma unroll
      for (int i = 0; i < VEC; ++i) x[i] = rt<T>(x[i]);
    }
    const bool is_q = hh < a.nq;
    const bool is_k = !is_q && hh < a.nq + a.nkv;
    const bool is_v = valid && !is_q && !is_k;
    T* kv = (T*)rd.kv_base;
    const T* nw = is_q ? (const T*)a.q_norm : (const T*)a.k_norm;
    // QK-norm: a head's LPH lanes reduce among themselves (every lane runs
    // the shuffles; only Q / K lanes of a model with the norm use the sum).
    if (a.q_norm || a.k_norm) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) ss += x[i] * x[i];
#pragma unroll
      for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (valid && !is_v && nw) {
        const float r = 1.0f / sqrtf(ss / (float)D + a.eps);
        float g[VEC];
        load16_f<T>(nw + d0, g);
#pragma unroll
        for (int i = 0; i < VEC; ++i) x[i] = rt<T>(rt<T>(x[i] * r) * g[i]);
      }
    }
    float c[VEC], sv[VEC], y[VEC];
    if (first) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) c[i] = c0[i], sv[i] = s0[i];
    } else {
      load16_f<T>((const T*)a.cos + (size_t)pos * half + dh, c);
      load16_f<T>((const T*)a.sin + (size_t)pos * half + dh, sv);
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[i], LPH / 2);
      const float rot = lower ? -partner : partner;
      y[i] = rt<T>(x[i] * c[i]) + rt<T>(rot * sv[i]);
    }
    if (!valid) continue;
    if (is_v) {  // value head: plain append
      store16_f<T>(kv + kv_offset_elems(a.layer, 1, rd.slot_rows, rd.row, a.nkv, hh - a.nq - a.nkv, rd.cap, D,
                                        cache_pos) + d0,
                   x);
    } else if (is_q) {
      store16_f<T>((T*)a.q_out + ((size_t)m * a.nq + hh) * D + d0, y);
    } else {
      store16_f<T>(kv + kv_offset_elems(a.layer, 0, rd.slot_rows, rd.row, a.nkv, hh - a.nq, rd.cap, D, cache_pos) +
                       d0,
                   y);
    }
  }
}

// Many tokens (prefill): one CTA per token at a time.  The 256 threads take
// the token's qkv row as 16-byte vectors (thread i holds vectors i, i + 256,
// ..., up to kRowVecs of them, all loaded before any arithmetic), so the
// row, the row descriptor and the token's cos / sin are read once and in
// parallel; a head's LPH lanes stay inside one warp, so the QK-norm sum and
// the rotate-half partner are shuffles as above.
constexpr int kRowThreads = 256;
constexpr int kRowVecs = 4;

template <typename T, int D>
__global__ void __launch_bounds__(kRowThreads) qkv_post_rows_kernel(QkvPostArgs a) {
  pdl_trigger();
  pdl_wait();
  constexpr int VEC = 16 / sizeof(T), LPH = D / VEC, half = D / 2;
  static_assert(kRowThreads % LPH == 0, "a head's lanes must not straddle threads of different rounds");
  const int t = threadIdx.x;
  const int hl = t % LPH;
  const int d0 = hl * VEC, dh = d0 % half;
  const bool lower = d0 < half;
  const int nh = a.nq + 2 * a.nkv;
  const int vecs = nh * LPH;  // 16-byte vectors in a token's qkv row
  const int M = a.B * a.S;
  for (int m = blockIdx.x; m < M; m += gridDim.x) {
    const T* row = (const T*)a.qkv + (size_t)m * nh * D;
    const int b = m / a.S, s = m % a.S;
    for (int v0 = 0; v0 < vecs; v0 += kRowVecs * kRowThreads) {
      float x[kRowVecs][VEC];
#pragma unroll
      for (int j = 0; j < kRowVecs; ++j) {
        const int v = v0 + j * kRowThreads + t;
        if (v < vecs) {
          load16_f<T>(row + (size_t)v * VEC, x[j]);
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) x[j][i] = 0.f;
        }
      }
      const RowDesc rd = a.rows[b];
      const int cache_pos = rd.past + s;
      int64_t pos = a.positions ? a.positions[m] : (int64_t)cache_pos;
      if (pos < 0 || pos >= a.max_pos) {
        if (t == 0 && v0 == 0) flag_error(a.err, kErrPositionRange);
        pos = pos < 0 ? 0 : a.max_pos - 1;
      }
      float c[VEC], sv[VEC];
      load16_f<T>((const T*)a.cos + (size_t)pos * half + dh, c);
      load16_f<T>((const T*)a.sin + (size_t)pos * half + dh, sv);
      T* kv = (T*)rd.kv_base;
#pragma unroll
      for (int j = 0; j < kRowVecs; ++j) {
        const int v = v0 + j * kRowThreads + t;
        if (v0 + j * kRowThreads >= vecs) break;  // uniform over the CTA
        const bool valid = v < vecs;
        const int hh = v / LPH;
        const bool is_q = hh < a.nq;
        const bool is_k = !is_q && hh < a.nq + a.nkv;
        const bool is_v = valid && !is_q && !is_k;
        const T* nw = is_q ? (const T*)a.q_norm : (const T*)a.k_norm;
        if (a.q_norm || a.k_norm) {
          float ss = 0.f;
#pragma unroll
          for (int i = 0; i < VEC; ++i) ss += x[j][i] * x[j][i];
#pragma unroll
          for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          if (valid && !is_v && nw) {
            const float r = 1.0f / sqrtf(ss / (float)D + a.eps);
            float g[VEC];
            load16_f<T>(nw + d0, g);
#pragma unroll
            for (int i = 0; i < VEC; ++i) x[j][i] = rt<T>(rt<T>(x[j][i] * r) * g[i]);
          }
        }
        float y[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const float partner = __shfl_xor_sync(0xffffffffu, x[j][i], LPH / 2);
          const float rot = lower ? -partner : partner;
          y[i] = rt<T>(x[j][i] * c[i]) + rt<T>(rot * sv[i]);
        }
        if (!valid) continue;
        if (is_v) {  // value head: plain append
          store16_f<T>(kv + kv_offset_elems(a.layer, 1, rd.slot_rows, rd.row, a.nkv, hh - a.nq - a.nkv, rd.cap, D,
                                            cache_pos) + d0,
                       x[j]);
        } else if (is_q) {
          store16_f<T>((T*)a.q_out + ((size_t)m * a.nq + hh) * D + d0, y);
        } else {
          store16_f<T>(kv + kv_offset_elems(a.layer, 0, rd.slot_rows, rd.row, a.nkv, hh - a.nq, rd.cap, D,
                                            cache_pos) + d0,
                       y);
        }
      }
    }
  }
}

// Resident CTAs per SM of a kernel at `threads` threads.
inline int resident_ctas(void (*kernel)(QkvPostArgs), int threads) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, 0) != cudaSuccess || n < 1) n = 1;
  return n;
}

}  // namespace

cudaError_t launch_qkv_post(const QkvPostArgs& a, cudaStream_t s) {
  const int M = a.B * a.S;
  if (M == 0) return cudaSuccess;
  cudaError_t e;
  const bool vec = a.D == 128 || a.D == 64;
  if (vec && a.use_pieces && a.dtype == kBF16) {  // decode rows: a warp per (token, head group)
    const int hpw = 32 / (a.D * 2 / 16);
    const long long units = (long long)M * ((a.nq + 2 * a.nkv + hpw - 1) / hpw);
    long long blocks = (units + kVecWarps - 1) / kVecWarps;
    const long long cap = 8LL * sm_count_cached();
    if (blocks > cap) blocks = cap;
    e = launch_pdl(a.D == 128 ? qkv_post_pieces_kernel<__nv_bfloat16, 128>
                              : qkv_post_pieces_kernel<__nv_bfloat16, 64>,
                   dim3((unsigned)blocks), dim3(kVecWarps * 32), 0, s, a);
  } else if (vec && !a.use_pieces) {  // a CTA per token
    void (*k)(QkvPostArgs);
    if (a.dtype == kBF16)
      k = a.D == 128 ? qkv_post_rows_kernel<__nv_bfloat16, 128> : qkv_post_rows_kernel<__nv_bfloat16, 64>;
    else
      k = a.D == 128 ? qkv_post_rows_kernel<float, 128> : qkv_post_rows_kernel<float, 64>;
    const long long cap = (long long)resident_ctas(k, kRowThreads) * sm_count_cached();
    const unsigned blocks = (unsigned)(M < cap ? M : cap);
    e = launch_pdl(k, dim3(blocks), dim3(kRowThreads), 0, s, a);
  } else {
    const dim3 grid(M, (a.nq + 2 * a.nkv + kHeadsPerCta - 1) / kHeadsPerCta), block(kHeadsPerCta * 32);
    e = a.dtype == kBF16 ? launch_pdl(qkv_post_kernel<__nv_bfloat16>, grid, block, 0, s, a)
                         : launch_pdl(qkv_post_kernel<float>, grid, block, 0, s, a);
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace mg
