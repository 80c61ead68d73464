// Decode / prefill GQA attention on the tensor cores (bf16, head_dim 64 or 128).
//
// With G query heads sharing one KV head, every key and value element feeds
// 2·G FLOPs; at G = 4 and 6.5 TB/s that is more fp32 FMA work than the CUDA
// cores sustain next to the loads, so the dot products run on mma.sync
// (m16n8k16, bf16 in, fp32 out) with the G heads padded to the MMA's 16 rows.
//
// Work split (stream-K over keys): the units are (token, KV head, 128-key
// chunk), and each persistent CTA takes one contiguous run of them, so every
// SM streams the same number of chunks.  Warp 8 (one lane) loads each chunk's
// keys and values with 2-D TMA (box 128 keys x 64 dims, 128-byte swizzle, no
// multicast) through the slot's tensor map, plus the pair's G query rows with
// a bulk copy, into a 2- or 3-stage ring.  Keys of positions before this
// forward are not written by the kernels ahead of this one, so for a decode
// batch (positions implied by the cache length) the producer requests those
// chunks before its programmatic-launch wait.
//
// Warps 0-7 each own 16 keys of every chunk (two warps per scheduler hide the
// MMA, ldmatrix and exp latencies of each other):
//   S = Q·Kᵀ   A = Q (heads x dims), B = K rows via ldmatrix
//   P = exp(S·scale - max)   online over the pair's chunks, quad shuffles
//   O = O·keep + P·V   A = P (bf16 hi + lo), B = V via ldmatrix.trans
// At the end of a pair the eight warps' (max, sum, O) are merged in shared
// memory.  A pair wholly inside the CTA's run is normalised and written to the
// output; a pair cut by the run's ends leaves an fp32 partial, and the CTA
// that completes the pair's counter merges the partials in CTA order
// (deterministic) and writes the output.  Every wait is bounded (code 3 in
// the error word on expiry); on a timeout the CTA stops, lets the copies it
// issued land and returns.
#include <math.h>

#include <algorithm>

#include "attn_tc_common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

#ifndef MG_ATTN_CUT_COST
#define MG_ATTN_CUT_COST 4  // chunks a CTA pays for merging its cut pairs
#endif

namespace mg {
namespace {

using namespace tc;
using namespace attn;

constexpr int kWarps = 8;                      // consumer warps (two per scheduler)
constexpr int kThreadsA = (kWarps + 1) * 32;   // + the producer warp
constexpr int kKeysW = 16;                     // keys per consumer warp
constexpr int kChunk = kWarps * kKeysW;        // keys per work item (128)
constexpr int kConsumers = kWarps * 32;
constexpr int kMaxStages = 3;
constexpr int kBoxBytes = kKvBoxKeys * 128;    // one 128-key x 64-dim box
constexpr int kMaxSmem = 227 * 1024;           // dynamic shared memory a CTA may use
static_assert(kKvBoxKeys == kChunk, "a chunk is one box high");

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Barrier over the consumer warps that returns the OR of `pred`, so all of
// them take the same branch afterwards.
__device__ __forceinline__ bool consumer_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.red.or.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

// Shared memory: `stages` ring stages (K, V, Q), the warps' merge area for G
// heads (m, l, O per warp, then one factor per warp and head, then M and L
// per head), the barriers.
template <int D>
struct TcAttnLayout {
  static constexpr int kDB = D / 64;                       // 64-dim boxes per key row
  static constexpr int kKV = kDB * kBoxBytes;              // K (or V) bytes of a chunk
  static constexpr int kQ = 8 * D * 2;                     // <= 8 query heads
  static constexpr int kStage = (2 * kKV + kQ + 1023) / 1024 * 1024;
  static constexpr int kBars = 2 * kMaxStages * 8 + 16;
  __host__ __device__ static constexpr int merge_floats(int G) {
    return kWarps * G * (D + 2) + kWarps * G + 2 * G;
  }
  __host__ __device__ static constexpr int bytes(int stages, int G) {
    return stages * kStage + (merge_floats(G) * 4 + 15) / 16 * 16 + kBars + 1024;
  }
};

// Split of the (token, KV head, chunk) units: pair p = m·nkv + h owns units
// p·C .. p·C + C - 1 (C = 128-key chunks of the longest row); CTA c takes
// units [begin(c), begin(c + 1)).  Stream-K ranges are equal; whole-pair
// ranges end on pair boundaries (chosen when that loses less to imbalance
// than the cut pairs cost).  A pair inside one CTA's range is finished by
// that CTA; a pair cut by range ends leaves one partial per CTA in that CTA's
// slot 0 (its first pair) or 1 (its last), and the CTA that completes the
// pair's counter merges them in CTA order.
struct Plan {
  long long total;  // P·C units
  long long pairs;  // P
  int C, grid, whole;
  __host__ __device__ long long begin(int c) const {
    return whole ? (long long)c * pairs / grid * C : (long long)c * total / grid;
  }
  __host__ __device__ int owner(long long u) const {
    return whole ? (int)(((u / C + 1) * grid - 1) / pairs) : (int)(((u + 1) * grid - 1) / total);
  }
  __host__ __device__ int slot(int c, long long p) const { return 2 * c + (p == begin(c) / C ? 0 : 1); }
};

template <int D>
__global__ void __launch_bounds__(kThreadsA, 1) attn_tc_kernel(AttnArgs a, Plan pl, int stages) {
  using L = TcAttnLayout<D>;
  constexpr int DB = L::kDB;
  constexpr int KS = D / 16;  // k-steps of the score MMA
  constexpr int DM = D / 16;  // dim tiles of Oᵀ
  const int G = a.nq / a.nkv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* merge = (float*)(smem + stages * L::kStage);  // [warp][head][m, l, O(D)]
  float* fac = merge + kWarps * G * (D + 2);           // [warp][head]
  float* mh = fac + kWarps * G;                        // [head] max
  float* lh = mh + G;                                  // [head] sum
  uint64_t* full = (uint64_t*)(smem + stages * L::kStage + (L::merge_floats(G) * 4 + 15) / 16 * 16);
  uint64_t* empty = full + kMaxStages;
  volatile int* abort_flag = (volatile int*)(empty + kMaxStages);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x;
  const long long u0 = pl.begin(c), u1 = pl.begin(c + 1);
  const int C = pl.C;
  const uint32_t qbytes = (uint32_t)(G * D * 2);

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 2);  // K/V arrival + Q arrival (or a plain arrival)
      mbar_init(&empty[s], kWarps);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kWarps) {
    if (lane == 0) {
      // Producer.  Before its wait it fills at most `stages` stages, and only
      // with keys of positions that existed before this forward; query rows
      // (written by the kernel before this one) always come after the wait.
      bool waited = false;
      if (a.positions != nullptr) {  // visibility depends on device positions
        pdl_wait();
        waited = true;
      }
      int qpend[kMaxStages];
      const __nv_bfloat16* qsrc[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) qpend[s] = 0, qsrc[s] = nullptr;
      auto issue_q = [&](int s, const __nv_bfloat16* src) {
        mbar_expect_tx(&full[s], qbytes);
        bulk_load(smem + s * L::kStage + 2 * L::kKV, src, qbytes, &full[s]);
      };
      long long n = 0, cur_p = -1;
      int m = 0, h = 0, nvis = 0;
      bool q_done = false;
      RowDesc rd{};
      for (long long u = u0; u < u1 && !*abort_flag; ++u) {
        const long long p = u / C;
        const int k0 = (int)(u - p * C) * kChunk;
        if (p != cur_p) {
          cur_p = p;
          m = (int)(p / a.nkv);
          h = (int)(p % a.nkv);
          rd = a.rows[m / a.S];
          nvis = visible(a, rd, m, m % a.S);
          q_done = false;
        }
        if (k0 >= nvis) continue;  // consumers skip it too
        if (!waited && (k0 + kChunk > rd.past || n >= stages)) {
          pdl_wait();
          waited = true;
          for (int s = 0; s < stages; ++s)
            if (qpend[s]) {
              issue_q(s, qsrc[s]);
              qpend[s] = 0;
            }
        }
        const int s = (int)(n % stages);
        if (n >= stages && !mbar_wait(&empty[s], (int)((n / stages) - 1) & 1, a.err)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * L::kStage;
        const int yk = (int)kv_row(a.layer, 0, rd.slot_rows, rd.row, a.nkv, h, rd.cap, k0);
        const int yv = (int)kv_row(a.layer, 1, rd.slot_rows, rd.row, a.nkv, h, rd.cap, k0);
        // A chunk that is only partly visible (the sequence's last) is loaded
        // in slices of kKvTailKeys keys up to its last visible key, in the
        // same layout; the consumers mask the keys past it.
        const int nsl = (min(kChunk, nvis - k0) + kKvTailKeys - 1) / kKvTailKeys;
        if (nsl * kKvTailKeys < kChunk) {
          const uint64_t tail = rd.kv_tmap + sizeof(CUtensorMap);
          constexpr int kSlice = kKvTailKeys * 128;
          mbar_expect_tx(&full[s], 2 * DB * nsl * kSlice);
          for (int j = 0; j < nsl; ++j)
            for (int db = 0; db < DB; ++db) {
              tma_load_2d_gmap(st + db * kBoxBytes + j * kSlice, tail, &full[s], db * 64, yk + j * kKvTailKeys);
              tma_load_2d_gmap(st + L::kKV + db * kBoxBytes + j * kSlice, tail, &full[s], db * 64,
                               yv + j * kKvTailKeys);
            }
        } else {
          mbar_expect_tx(&full[s], 2 * L::kKV);
          for (int db = 0; db < DB; ++db)
            tma_load_2d_gmap(st + db * kBoxBytes, rd.kv_tmap, &full[s], db * 64, yk);
          for (int db = 0; db < DB; ++db)
            tma_load_2d_gmap(st + L::kKV + db * kBoxBytes, rd.kv_tmap, &full[s], db * 64, yv);
        }
        if (!q_done) {  // the piece's first loaded chunk carries its query rows
          const __nv_bfloat16* src = (const __nv_bfloat16*)a.q + ((size_t)m * a.nq + (size_t)h * G) * D;
          if (waited) {
            issue_q(s, src);
          } else {
            qpend[s] = 1;
            qsrc[s] = src;
          }
          q_done = true;
        } else {
          mbar_arrive(&full[s]);
        }
        ++n;
      }
      if (!waited) {
        pdl_wait();
        for (int s = 0; s < stages; ++s)
          if (qpend[s] && !*abort_flag) {
            issue_q(s, qsrc[s]);
            qpend[s] = 0;
          }
      }
      if (*abort_flag) {
        // Complete the arrivals still owed, then let every issued copy land
        // before shared memory is released.
        for (int s = 0; s < stages; ++s)
          if (qpend[s]) mbar_arrive(&full[s]);
        for (long long i = n > stages ? n - stages : 0; i < n; ++i)
          mbar_wait(&full[i % stages], (int)(i / stages) & 1, a.err);
      }
    }
  } else {
    // Consumers: warp w owns keys 16w .. 16w + 15 of each chunk and keeps an
    // online softmax (max, sum, O) over the chunks of the current pair.
    // The first piece's visible length (from its row descriptor) does not depend on
    // the kernel before this one (the row table is uploaded before the
    // forward's first kernel, as the producer's early loads assume; without
    // explicit positions the visible length follows from it), so they are
    // read before the programmatic-launch wait instead of after it (about a
    // microsecond of each launch's start).
    const bool early = a.positions == nullptr && u0 < u1;
    int nvis0 = 0;
    if (early) {
      const int m0 = (int)(u0 / C / a.nkv);
      nvis0 = visible(a, a.rows[m0 / a.S], m0, m0 % a.S);
    }
    pdl_wait();
    const int g = lane >> 2, t = lane & 3;
    // Scores are kept in base 2 (scale·log2 e folded in), so every
    // exponential below is exp2; maxima in the partials are base 2 too.
    const float scale2 = a.scale * 1.4426950408889634f;
    long long n = 0;
    for (long long u = u0; u < u1;) {
      const long long p = u / C;
      const long long pe = min(u1, (p + 1) * (long long)C);
      const int m = (int)(p / a.nkv), h = (int)(p % a.nkv);
      const int nvis = early && u == u0 ? nvis0 : visible(a, a.rows[m / a.S], m, m % a.S);
      const int kb = (int)(u - p * C), ke = (int)(pe - p * C);
      const int kl = min(ke, (nvis + kChunk - 1) / kChunk);  // chunks [kb, kl) hold visible keys

      // Transposed products, so the G <= 8 query heads sit on the MMA's N = 8
      // side instead of padding its M = 16: Sᵀ = K·Qᵀ (M = this warp's 16
      // keys, N = heads, K = dims) and Oᵀ = Vᵀ·Pᵀ (M = 16 dims per tile,
      // N = heads, K = the 16 keys).  A thread holds keys g, g + 8 (dims g,
      // g + 8 of Oᵀ) for heads 2t and 2t + 1.
      float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
      float o[DM][4];
#pragma unroll
      for (int i = 0; i < DM; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      uint32_t qb[KS][2];  // B fragments of Qᵀ
      for (int kc = kb; kc < kl; ++kc) {
        const int s = (int)(n % stages);
        if (!mbar_wait(&full[s], (int)(n / stages) & 1, a.err)) *abort_flag = 1;
        ++n;
        if (*abort_flag) break;  // the vote at the end of the piece stops every warp
        uint8_t* st = smem + s * L::kStage;
        if (kc == kb) {
          const __nv_bfloat16* Qs = (const __nv_bfloat16*)(st + 2 * L::kKV);
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            if (g < G) {
              qb[ks][0] = *reinterpret_cast<const uint32_t*>(Qs + g * D + 16 * ks + 2 * t);
              qb[ks][1] = *reinterpret_cast<const uint32_t*>(Qs + g * D + 16 * ks + 8 + 2 * t);
            } else {
              qb[ks][0] = qb[ks][1] = 0u;
            }
          }
        }
        const int nk = max(0, min(kKeysW, nvis - (kc * kChunk + warp * kKeysW)));
        if (nk > 0) {
          float sc[4] = {0.f, 0.f, 0.f, 0.f};  // Sᵀ: keys g, g + 8 x heads 2t, 2t + 1
          const uint32_t kbase = smem_u32(st);
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            // A = keys x 16 dims: four 8x8 matrices (keys 0-7 / 8-15, dim chunks 2ks / 2ks + 1)
            const int r = warp * kKeysW + (lane & 7) + 8 * ((lane >> 3) & 1);
            const int cc = 2 * ks + (lane >> 4);
            uint32_t afr[4];
            ldsm_x4(kbase + (cc >> 3) * kBoxBytes + swz(r, cc & 7), afr);
            mma16816_full(sc, afr[0], afr[1], afr[2], afr[3], qb[ks][0], qb[ks][1]);
          }
          // Online softmax per head (column): keys g (c0, c1) and g + 8 (c2, c3).
          const bool vA = g < nk, vB = g + 8 < nk;
          float s0 = vA ? sc[0] * scale2 : -INFINITY, s1 = vA ? sc[1] * scale2 : -INFINITY;
          float s2 = vB ? sc[2] * scale2 : -INFINITY, s3 = vB ? sc[3] * scale2 : -INFINITY;
          float mx0 = fmaxf(mrow[0], fmaxf(s0, s2)), mx1 = fmaxf(mrow[1], fmaxf(s1, s3));
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
          }
          const float keep0 = mrow[0] == -INFINITY ? 0.f : exp2f(mrow[0] - mx0);
          const float keep1 = mrow[1] == -INFINITY ? 0.f : exp2f(mrow[1] - mx1);
          s0 = s0 == -INFINITY ? 0.f : exp2f(s0 - mx0);
          s1 = s1 == -INFINITY ? 0.f : exp2f(s1 - mx1);
          s2 = s2 == -INFINITY ? 0.f : exp2f(s2 - mx0);
          s3 = s3 == -INFINITY ? 0.f : exp2f(s3 - mx1);
          float sum0 = s0 + s2, sum1 = s1 + s3;
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) {
            sum0 += __shfl_xor_sync(0xffffffffu, sum0, off);
            sum1 += __shfl_xor_sync(0xffffffffu, sum1, off);
          }
          mrow[0] = mx0;
          mrow[1] = mx1;
          lrow[0] = lrow[0] * keep0 + sum0;
          lrow[1] = lrow[1] * keep1 + sum1;
#pragma unroll
          for (int i = 0; i < DM; ++i) {
            o[i][0] *= keep0;
            o[i][1] *= keep1;
            o[i][2] *= keep0;
            o[i][3] *= keep1;
          }
          // Pᵀ as the B operand of Oᵀ += Vᵀ·Pᵀ: the accumulator pairs are an 8x8
          // (keys x heads) matrix each, transposed in registers.  P = hi + lo,
          // both bf16: two MMAs keep P to ~2^-17 relative (an fp32 P·V).
          const uint32_t h01 = pack2(s0, s1), h23 = pack2(s2, s3);
          const uint32_t l01 = pack2(s0 - lo_bf16(h01), s1 - hi_bf16(h01));
          const uint32_t l23 = pack2(s2 - lo_bf16(h23), s3 - hi_bf16(h23));
          const uint32_t pb0 = movm_trans(h01), pb1 = movm_trans(h23);
          const uint32_t pc0 = movm_trans(l01), pc1 = movm_trans(l23);
          // Value rows past the visible keys can hold anything (P is 0 there,
          // but 0 * NaN is not): their halves of the A fragments are cleared.
          const int kr = 2 * t;  // A fragment keys: kr, kr + 1 (a0, a1) and kr + 8, kr + 9 (a2, a3)
          const uint32_t m01 = (kr < nk ? 0x0000ffffu : 0u) | (kr + 1 < nk ? 0xffff0000u : 0u);
          const uint32_t m89 = (kr + 8 < nk ? 0x0000ffffu : 0u) | (kr + 9 < nk ? 0xffff0000u : 0u);
          const uint32_t vbase = smem_u32(st + L::kKV);
#pragma unroll
          for (int dm = 0; dm < DM; ++dm) {
            // A = Vᵀ (16 dims x 16 keys): matrices (keys 0-7 / 8-15) x (dim chunks 2dm / 2dm + 1)
            const int mi = lane >> 3;
            const int r = warp * kKeysW + (lane & 7) + 8 * (mi >> 1);
            const int cc = 2 * dm + (mi & 1);
            uint32_t afr[4];
            ldsm_x4_t(vbase + (cc >> 3) * kBoxBytes + swz(r, cc & 7), afr);
            afr[0] &= m01;
            afr[1] &= m01;
            afr[2] &= m89;
            afr[3] &= m89;
            mma16816_full(o[dm], afr[0], afr[1], afr[2], afr[3], pb0, pb1);
            mma16816_full(o[dm], afr[0], afr[1], afr[2], afr[3], pc0, pc1);
          }
        }
        // The stage's data is in registers now: hand it back to the producer.
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }

      // End of the piece: merge the warps.
      float* mw = merge + warp * G * (D + 2);
#pragma unroll
      for (int e = 0; e < 2; ++e) {  // heads 2t and 2t + 1
        const int hh = 2 * t + e;
        if (hh < G) {
          if (g == 0) {
            mw[hh * (D + 2)] = mrow[e];
            mw[hh * (D + 2) + 1] = lrow[e];
          }
#pragma unroll
          for (int dm = 0; dm < DM; ++dm) {
            mw[hh * (D + 2) + 2 + 16 * dm + g] = o[dm][e];
            mw[hh * (D + 2) + 2 + 16 * dm + g + 8] = o[dm][2 + e];
          }
        }
      }
      if (consumer_any(*abort_flag)) {  // also orders the writes above
        *abort_flag = 1;
        break;
      }
      if (tid < G) {
        float Mx = -INFINITY;
        for (int w = 0; w < kWarps; ++w) Mx = fmaxf(Mx, merge[(w * G + tid) * (D + 2)]);
        float Ls = 0.f;
        for (int w = 0; w < kWarps; ++w) {
          const float mwv = merge[(w * G + tid) * (D + 2)];
          const float f = mwv == -INFINITY ? 0.f : exp2f(mwv - Mx);
          fac[w * G + tid] = f;
          Ls += f * merge[(w * G + tid) * (D + 2) + 1];
        }
        mh[tid] = Mx;
        lh[tid] = Ls;
      }
      consumer_bar();
      const int c_lo = pl.owner(p * C), c_hi = pl.owner((p + 1) * (long long)C - 1);
      __nv_bfloat16* out = (__nv_bfloat16*)a.out + ((size_t)m * a.nq + (size_t)h * G) * D;
      if (c_lo == c_hi) {
        for (int i = tid; i < G * D; i += kConsumers) {
          const int hh = i / D, d = i % D;
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) acc += fac[w * G + hh] * merge[(w * G + hh) * (D + 2) + 2 + d];
          out[i] = __float2bfloat16_rn(acc * (1.0f / lh[hh]));
        }
      } else {
        float* part = a.partial + (size_t)pl.slot(c, p) * G * (D + 2);
        for (int i = tid; i < G * D; i += kConsumers) {
          const int hh = i / D, d = i % D;
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) acc += fac[w * G + hh] * merge[(w * G + hh) * (D + 2) + 2 + d];
          part[hh * (D + 2) + 2 + d] = acc;
        }
        if (tid < G) {
          part[tid * (D + 2)] = mh[tid];
          part[tid * (D + 2) + 1] = lh[tid];
        }
        // The barrier orders the slot writes before thread 0's release; its
        // acquire (then the barrier) orders the other pieces before the reads.
        consumer_bar();
        bool last = false;
        if (tid == 0) last = atomic_add_acq_rel_gpu(&a.counters[p], 1) == c_hi - c_lo;
        if (consumer_any(last)) {
          // Per head: the pieces' maxima give one factor per piece (kept in
          // the factor area), then every output adds its pieces in CTA order.
          const int npc = c_hi - c_lo + 1;  // <= grid, so 2·G·npc fits the merge area
          float* pf = merge;                 // [head][piece] max, then factor
          float* pls = merge + G * npc;      // [head][piece] sum
          for (int i = tid; i < G * npc; i += kConsumers) {
            const int hh = i / npc, k = i % npc;
            const float* q = a.partial + ((size_t)pl.slot(c_lo + k, p) * G + hh) * (D + 2);
            pf[i] = __ldcg(q);
            pls[i] = __ldcg(q + 1);
          }
          consumer_bar();
          if (tid < G) {
            float Mx = -INFINITY;
            for (int k = 0; k < npc; ++k) Mx = fmaxf(Mx, pf[tid * npc + k]);
            float Ls = 0.f;
            for (int k = 0; k < npc; ++k) {
              const float mk = pf[tid * npc + k];
              const float f = mk == -INFINITY ? 0.f : exp2f(mk - Mx);
              Ls += f * pls[tid * npc + k];
              pf[tid * npc + k] = f;
            }
            lh[tid] = Ls;
          }
          consumer_bar();
          for (int i = tid; i < G * D; i += kConsumers) {
            const int hh = i / D, d = i % D;
            float acc = 0.f;
            for (int k0 = 0; k0 < npc; k0 += 8) {
              float v[8];
#pragma unroll
              for (int k = 0; k < 8; ++k)  // eight independent loads in flight
                v[k] = k0 + k < npc
                           ? __ldcg(a.partial + ((size_t)pl.slot(c_lo + k0 + k, p) * G + hh) * (D + 2) + 2 + d)
                           : 0.f;
#pragma unroll
              for (int k = 0; k < 8; ++k)
                if (k0 + k < npc) acc += pf[hh * npc + k0 + k] * v[k];
            }
            out[i] = __float2bfloat16_rn(acc * (1.0f / lh[hh]));
          }
          if (tid == 0) a.counters[p] = 0;
        }
      }
      consumer_bar();  // the merge area is rewritten by the next piece
      u = pe;
    }
  }
  __syncthreads();
}

int sm_count_attn() {
  return usable_sms();
}

}  // namespace

bool attention_tc_applicable(int dtype, int D, int G) {
  return dtype == kBF16 && (D == 64 || D == 128) && G <= 8;
}

size_t attention_tc_scratch_elems(int nq, int D) {
  // Two partial slots per CTA, at most two CTAs per SM, G <= 8 heads each.
  return (size_t)2 * 2 * sm_count_attn() * (size_t)(nq < 8 ? nq : 8) * (D + 2);
}

cudaError_t launch_attention_tc(const AttnArgs& a, int splits, cudaStream_t s) {
  if ((uintptr_t)a.q % 16) return cudaErrorInvalidValue;
  const long long pairs = (long long)a.B * a.S * a.nkv;
  if (pairs <= 0) return cudaSuccess;
  if (!a.counters || a.counters_elems < (size_t)pairs) return cudaErrorInvalidValue;
  const int G = a.nq / a.nkv;
  auto go = [&](auto kernel, int smem, int stages) -> cudaError_t {
    static bool configured[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    bool& done = configured[a.D == 128][dev];
    if (!done) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
      if (e != cudaSuccess) return e;
      done = true;
    }
    static int per_sm_cache[2][9][64] = {};  // [D == 128][G][device]
    int& per_sm = per_sm_cache[a.D == 128][G][dev];
    if (!per_sm) {
      int n = 0;
      cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreadsA, smem);
      if (e != cudaSuccess) return e;
      per_sm = n > 0 ? (n < 2 ? n : 2) : 1;
    }
    Plan pl;
    pl.C = splits;
    pl.pairs = pairs;
    pl.total = pairs * splits;
    // A cut pair's pieces (at most one per CTA) are merged through the merge
    // area, which holds 4·(D + 2) pieces per head.
    const long long cap = std::min<long long>((long long)sm_count_attn() * per_sm, 4 * (a.D + 2));
    // Whole pairs when the busiest CTA then streams no more chunks than an
    // equal stream-K range plus what its cut pairs cost (about 4 chunks).
    const long long whole_span = (pairs + cap - 1) / cap * splits;
    const long long sk_span = (pl.total + cap - 1) / cap + MG_ATTN_CUT_COST;
    pl.whole = whole_span <= sk_span;
    const long long units = pl.whole ? pairs : pl.total;
    pl.grid = (int)(units < cap ? units : cap);
    if ((size_t)2 * pl.grid * G * (a.D + 2) > a.partial_elems) return cudaErrorInvalidValue;
    return launch_pdl(kernel, dim3(pl.grid), dim3(kThreadsA), smem, s, a, pl, stages);
  };
  // Three stages where they fit next to the merge area, else two.
  if (a.D == 128) {
    using L = TcAttnLayout<128>;
    const int stages = L::bytes(3, G) <= kMaxSmem ? 3 : 2;
    return go(attn_tc_kernel<128>, L::bytes(stages, G), stages);
  }
  using L = TcAttnLayout<64>;
  return go(attn_tc_kernel<64>, L::bytes(3, G), 3);
}

}  // namespace mg
