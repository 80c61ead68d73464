// Prefill / multi-token GQA attention on tcgen05 (bf16, head_dim 64 or 128).
//
// A work item is one cache row b, one KV head h and a tile of 128 query rows:
// 128 / G tokens x the G query heads that share h (row r = token r / G, head
// r % G), so every key and value chunk feeds 128 rows.  The kernel is
// persistent (one CTA per SM, items heaviest first) and splits the flash
// recurrence over its warps:
//   * warp 0, one lane: loads each 128-key chunk of keys and values with 2-D
//     TMA through the slot's tensor map (box 128 keys x 64 dims, 128-byte
//     swizzle, no multicast) into a 2-stage ring;
//   * warp 1, one lane: issues tcgen05.mma.  S = Q·Kᵀ (M = 128 query rows,
//     N = 128 keys, K = D; Q and K K-major in shared memory) into one of two
//     TMEM score buffers; O += P·V (M = 128 rows, N = D, K = 128 keys) into
//     the TMEM output, with P read from TMEM (where the softmax left it, in
//     the chunk's score buffer) and V read MN-major straight from its TMA
//     box.  The score product of chunk j + 1 is issued before the value
//     product of chunk j, so it overlaps that chunk's softmax;
//   * warps 2-9: two threads per query row (its TMEM lane), each owning 64
//     of a chunk's 128 keys and half of the head dims; the pair exchanges
//     its partial row maxima through shared memory.  They write the tile's
//     query rows into shared memory, and per chunk read their part of S's
//     row, mask it by the reference's visible-key rule and keep the online
//     softmax in base 2 (P = 2^(S·scale2 - m·scale2), l = l·α + ΣP).  The
//     running maximum m is moved only when a row's scores exceed it by more
//     than 2^8, and only then is the row of O in TMEM rescaled by α (the
//     result O / l does not depend on which m is used).  The exponentials
//     of chunk j are computed while the value product of chunk j - 1 runs;
//     P goes back into TMEM as bf16 (the precision the reference's own
//     attention multiplies the values in), l sums it in fp32.  At the end
//     they write O / l.
// Value rows at or past the cache end were never written: they are cleared
// in shared memory before the value product (P is 0 there, but 0 * NaN is
// not).  Every wait is bounded (code 3 in the error word on expiry); on
// expiry the roles stop, issued loads and MMAs drain, and TMEM is freed.
#include <math.h>

#include "attn_tc_common.cuh"
#include "kernels.h"
#include "tc_common.cuh"


namespace mg {
namespace {

using namespace tc;
using namespace attn;
using bf16 = __nv_bfloat16;

constexpr int kRowsT = 128;              // query rows of a tile = TMEM lanes
constexpr int kChunkT = kKvBoxKeys;      // keys per chunk (128)
constexpr int kBoxT = kKvBoxKeys * 128;  // a 128-row x 128-byte swizzled block (16 KB)
constexpr int kSoftWarps = 8;            // two per TMEM lane quadrant, 64 keys each
constexpr int kThreadsT = 64 + 32 * kSoftWarps;
constexpr int kColS = 0;                 // TMEM columns: scores [0, 256) in two buffers,
constexpr int kColO = 256;               // the output [256, 256 + D)

template <int D>
struct TcPrefillLayout {
  static constexpr int kDB = D / 64;       // 64-wide blocks of D
  static constexpr int kQ = kDB * kBoxT;   // query tile (A of S)
  static constexpr int kKV = kDB * kBoxT;  // keys (or values) of a chunk
  static constexpr int kStages = 2;
  static constexpr int kOffQ = 0;
  static constexpr int kOffKV = kOffQ + kQ;
  static constexpr int kOffBar = kOffKV + kStages * 2 * kKV;
  static constexpr int kOffX = kOffBar + 128;          // [2 chunk parities][2 halves][128 rows] floats
  static constexpr int kBytes = kOffX + 2048 + 1024;
};

// Shared-memory descriptor of an MN-major operand with 128-byte swizzle: 64
// MN elements per 128-byte row, K rows 128 bytes apart in 1024-byte groups of
// 8 (SBO), the next 64 MN elements `lbo` bytes on (LBO).
__device__ __forceinline__ uint64_t smem_desc_mn(const void* p, uint32_t lbo) {
  const uint64_t addr = smem_u32(p);
  return ((addr & 0x3FFFFull) >> 4) | ((uint64_t)(lbo >> 4) << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

// Byte offset of the 16-byte chunk c (of a 128-element row) of row r in a
// K-major tile stored as 64-element blocks with the 128-byte swizzle.
__device__ __forceinline__ int swz_off(int r, int c) {
  return (c >> 3) * kBoxT + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

// D (TMEM) += A (TMEM, M lanes x K bf16 packed two per column) · B (shared).
__device__ __forceinline__ void mma_bf16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Two floats to a bf16 pair (round to nearest even), `lo` in the low half.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// 2^x on the special-function unit (ex2.approx.ftz.f32: -inf -> +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, err));
}

template <int D>
__global__ void __launch_bounds__(kThreadsT, 1) attn_prefill_tc_kernel(AttnArgs a, PrefillPlan pl) {
  using L = TcPrefillLayout<D>;
  constexpr int DB = L::kDB;
  const int G = a.nq / a.nkv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sq = smem + L::kOffQ;
  uint8_t* skv = smem + L::kOffKV;  // stage s: keys at skv + 2·s·kKV, values kKV after them
  uint64_t* bars = (uint64_t*)(smem + L::kOffBar);
  uint64_t* kvfull = bars;       // [2] chunk landed
  uint64_t* kvempty = bars + 2;  // [2] chunk's value product done
  uint64_t* sfull = bars + 4;    // [2] scores ready in TMEM buffer
  uint64_t* pready = bars + 6;   // P written, O rescaled (softmax warps)
  uint64_t* odone = bars + 7;    // value product done
  uint64_t* qready = bars + 8;   // query tile written (softmax warps)
  uint64_t* drain = bars + 9;    // every MMA finished
  uint32_t* tmem_holder = (uint32_t*)(bars + 10);
  volatile int* abort_flag = (volatile int*)(tmem_holder + 1);
  float* xch = (float*)(smem + L::kOffX);  // a row's partial maxima (then sums) of the two halves

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kvfull[s], 1);
      mbar_init(&kvempty[s], 1);
      mbar_init(&sfull[s], 1);
    }
    mbar_init(pready, kSoftWarps);
    mbar_init(odone, 1);
    mbar_init(qready, kSoftWarps);
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  pdl_trigger();
  pdl_wait();  // the query rows and this forward's keys come from the kernel before

  long long issued = 0;
  if (warp == 0) {
    if (lane == 0) {
      long long n = 0;
      for (long long i = blockIdx.x; i < pl.items && !*abort_flag; i += gridDim.x) {
        int qt, b, h;
        item_of(a, pl, i, qt, b, h);
        const RowDesc rd = a.rows[b];
        const int nch = (tile_keys(a, rd, pl, b, qt) + kChunkT - 1) / kChunkT;
        for (int ch = 0; ch < nch; ++ch, ++n) {
          const int s = (int)(n & 1);
          if (n >= 2 && !mbar_wait(&kvempty[s], (int)((n >> 1) - 1) & 1, a.err)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          uint8_t* st = skv + s * 2 * L::kKV;
          const int k0 = ch * kChunkT;
          const int yk = (int)kv_row(a.layer, 0, rd.slot_rows, rd.row, a.nkv, h, rd.cap, k0);
          const int yv = (int)kv_row(a.layer, 1, rd.slot_rows, rd.row, a.nkv, h, rd.cap, k0);
          mbar_expect_tx(&kvfull[s], 2 * L::kKV);
          for (int db = 0; db < DB; ++db) {
            tma_load_2d_gmap(st + db * kBoxT, rd.kv_tmap, &kvfull[s], db * 64, yk);
            tma_load_2d_gmap(st + L::kKV + db * kBoxT, rd.kv_tmap, &kvfull[s], db * 64, yv);
          }
          issued = n + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer.  Per item: wait for the query tile; per chunk n: the
      // score product into TMEM buffer n & 1 (once the value product of chunk
      // n - 2, which read its P from that buffer, has finished), then the
      // value product of chunk n - 1 once its P is written (and of the item's
      // last chunk at the end).
      constexpr uint32_t idS = instr_desc(kChunkT);
      constexpr uint32_t idPV = instr_desc(D) | (1u << 16);  // B (the values) MN-major
      long long n = 0;
      int it = 0;
      // odone phases this thread has seen complete, waited strictly in order
      // and never after the next value product was issued (a parity wait
      // two phases behind would match the wrong phase).
      long long o_seen = -1;
      auto wait_odone = [&](long long upto) -> bool {
        for (; o_seen < upto; ++o_seen)
          if (!mbar_wait(odone, (int)((o_seen + 1) & 1), a.err)) return false;
        return true;
      };
      auto value_product = [&](long long m, bool first) -> bool {
        if (!mbar_wait(pready, (int)(m & 1), a.err)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint8_t* v = skv + (int)(m & 1) * 2 * L::kKV + L::kKV;
        const uint32_t pt = tmem + kColS + (uint32_t)(m & 1) * kChunkT;  // P: 128 keys in 64 columns
#pragma unroll
        for (int kk = 0; kk < kChunkT / 16; ++kk)
          mma_bf16_ta(tmem + kColO, pt + kk * 8, smem_desc_mn(v + kk * 16 * 128, kBoxT), idPV,
                      (first && kk == 0) ? 0u : 1u);
        mma_commit(odone);
        mma_commit(&kvempty[m & 1]);
        return true;
      };
      bool ok = true;
      for (long long i = blockIdx.x; i < pl.items && ok && !*abort_flag; i += gridDim.x) {
        int qt, b, h;
        item_of(a, pl, i, qt, b, h);
        const RowDesc rd = a.rows[b];
        const int nch = (tile_keys(a, rd, pl, b, qt) + kChunkT - 1) / kChunkT;
        if (!mbar_wait(qready, it & 1, a.err)) {
          ok = false;
          break;
        }
        ++it;
        for (int ch = 0; ch < nch; ++ch, ++n) {
          if (!mbar_wait(&kvfull[n & 1], (int)(n >> 1) & 1, a.err) || !wait_odone(n - 2) || *abort_flag) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint8_t* k = skv + (int)(n & 1) * 2 * L::kKV;
#pragma unroll
          for (int kd = 0; kd < D / 16; ++kd) {
            const uint64_t da = smem_desc(sq + (kd >> 2) * kBoxT) + (uint64_t)((kd & 3) * 2);
            const uint64_t db = smem_desc(k + (kd >> 2) * kBoxT) + (uint64_t)((kd & 3) * 2);
            mma_bf16(tmem + kColS + (uint32_t)(n & 1) * kChunkT, da, db, idS, kd > 0 ? 1u : 0u);
          }
          mma_commit(&sfull[n & 1]);
          if (ch > 0 && !value_product(n - 1, ch == 1)) {
            ok = false;
            break;
          }
        }
        if (ok && nch > 0 && (!wait_odone(n - 2) || !value_product(n - 1, nch == 1))) ok = false;
      }
      if (!ok) *abort_flag = 1;
      mma_commit(drain);  // arrives once every MMA issued above has finished
    }
  } else {
    // Softmax warps 2-9: warp w owns TMEM lanes 32·(w % 4) .. + 31 (one query
    // row per thread) and half (w - 2) / 4 of every chunk's keys (and of the
    // head dims for the query, output and rescale).
    const int q4 = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = q4 * 32 + lane;
    const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
    const float scale2 = a.scale * 1.4426950408889634f;
    constexpr int kHK = kChunkT / 2;  // keys of this half
    constexpr int kHD = D / 2;        // dims of this half
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + q4) : "memory"); };
    // The two warps of a row pair decide together whether a wait failed, so
    // neither is left at a pair barrier the other has abandoned.
    auto pair_any = [&](bool pred) -> bool {
      uint32_t res;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\t"
          "setp.ne.u32 p, %1, 0;\n\t"
          "barrier.red.or.pred q, %2, 64, p;\n\t"
          "selp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(res)
          : "r"((uint32_t)pred), "r"(1 + q4)
          : "memory");
      return res != 0;
    };
    // Value products this warp has seen finish: odone phases are waited in
    // order, never skipping one (a parity wait could otherwise match an older
    // phase).
    long long o_seen = -1;
    auto wait_odone = [&](long long upto) -> bool {
      for (; o_seen < upto; ++o_seen)
        if (!warp_wait(odone, (int)((o_seen + 1) & 1), a.err)) return false;
      return true;
    };
    long long n = 0;
    bool ok = true;
    for (long long i = blockIdx.x; i < pl.items && ok; i += gridDim.x) {
      int qt, b, h;
      item_of(a, pl, i, qt, b, h);
      const RowDesc rd = a.rows[b];
      const int nch = (tile_keys(a, rd, pl, b, qt) + kChunkT - 1) / kChunkT;
      const int s_tok = qt * pl.tq + r / G;  // this row's query token
      const int g = r % G;
      const bool valid = r / G < pl.tq && s_tok < a.S;
      const int vis = valid ? visible(a, rd, b * a.S + s_tok, s_tok) : 0;
      const int tot = rd.past + a.S;  // keys written so far
      // This half of the query row into the tile (zeros for rows past the sequence).
      {
        const uint4* src = reinterpret_cast<const uint4*>(
            (const bf16*)a.q + (((size_t)b * a.S + (valid ? s_tok : 0)) * a.nq + (size_t)h * G + g) * D);
#pragma unroll
        for (int c = half * (kHD / 8); c < (half + 1) * (kHD / 8); ++c) {
          const uint4 val = valid ? src[c] : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(sq + swz_off(r, c)) = val;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(qready);

      float m = -INFINITY, l = 0.f;  // m: the running maximum P is taken against (raw scores); l: this half's sum
      for (int ch = 0; ch < nch; ++ch, ++n) {
        const int sb = (int)(n & 1);
        // scores ready; the chunk's load is complete too (it orders the TMA
        // writes before the value clearing below)
        const bool late = !warp_wait(&sfull[sb], (int)(n >> 1) & 1, a.err) ||
                          !warp_wait(&kvfull[sb], (int)(n >> 1) & 1, a.err);
        if (pair_any(late)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float sc[kHK];
        if constexpr (D == 128) {  // one 64-column load and one wait (head_dim 64 would spill)
          tmem_ld64(tmem + lanes + kColS + (uint32_t)sb * kChunkT + half * kHK, sc);
        } else {
#pragma unroll
          for (int c4 = 0; c4 < kHK / 32; ++c4)
            tmem_ld32(tmem + lanes + kColS + (uint32_t)sb * kChunkT + half * kHK + c4 * 32, sc + c4 * 32);
        }
        const int nv = vis - ch * kChunkT - half * kHK;  // visible keys of this half for this row
        // Row maximum of the raw scores (the scale is positive, so it commutes
        // with the maximum), as a tree; invisible keys become -inf.
        if (!__all_sync(0xffffffffu, nv >= kHK)) {
#pragma unroll
          for (int c = 0; c < kHK; ++c) sc[c] = c < nv ? sc[c] : -INFINITY;
        }
        float t8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t8[j] = sc[j];
#pragma unroll
        for (int c = 8; c < kHK; ++c) t8[c & 7] = fmaxf(t8[c & 7], sc[c]);
        const float pm = fmaxf(fmaxf(fmaxf(t8[0], t8[1]), fmaxf(t8[2], t8[3])),
                               fmaxf(fmaxf(t8[4], t8[5]), fmaxf(t8[6], t8[7])));
        float* xs = xch + (size_t)(sb * 2) * kRowsT;
        xs[half * kRowsT + r] = pm;
        pair_sync();  // (double-buffered by chunk parity: one barrier per chunk)
        const float mt = fmaxf(pm, xs[(1 - half) * kRowsT + r]);
        // Move the maximum only when the scores outgrow it by 2^8.
        float m_new = m;
        bool moved = false;
        if (m == -INFINITY) {
          m_new = mt;
        } else if ((mt - m) * scale2 > 8.f) {
          m_new = mt;
          moved = true;
        }
        const float alpha = moved ? ex2_approx((m - m_new) * scale2) : 1.f;
        // P = 2^(S·scale2 - m·scale2): one fused multiply-add and one ex2 per
        // key (invisible keys are -inf and give 0).  This runs while the
        // previous chunk's value product is still on the tensor cores.
        const float mb = m_new == -INFINITY ? 0.f : m_new * scale2;
#pragma unroll
        for (int j = 0; j < 8; ++j) t8[j] = 0.f;
#pragma unroll
        for (int c = 0; c < kHK; ++c) {
          sc[c] = ex2_approx(fmaf(sc[c], scale2, -mb));
          t8[c & 7] += sc[c];
        }
        l = l * alpha + (((t8[0] + t8[1]) + (t8[2] + t8[3])) + ((t8[4] + t8[5]) + (t8[6] + t8[7])));
        m = m_new;
        // The previous value product is done before O is rescaled and this
        // chunk's P is handed over.  Waiting for it on every chunk (not for
        // the one before) also keeps this thread's odone waits within one
        // phase of the barrier: value product n can only start after this
        // chunk's P is handed over.
        const bool rescale = __any_sync(0xffffffffu, moved);
        if (pair_any(!wait_odone(n - 1))) {
          ok = false;
          break;
        }
        if (rescale) {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll 1
          for (int c4 = 0; c4 < kHD / 32; ++c4) {
            float o[32];
            tmem_ld32(tmem + lanes + kColO + half * kHD + c4 * 32, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(tmem + lanes + kColO + half * kHD + c4 * 32, o);
          }
        }
        // Value rows past the written keys: clear this half of them before the product.
        if (ch * kChunkT + kChunkT > tot && ch * kChunkT + r >= tot) {
          uint8_t* v = skv + sb * 2 * L::kKV + L::kKV;
#pragma unroll
          for (int c = half * (kHD / 8); c < (half + 1) * (kHD / 8); ++c)
            *reinterpret_cast<uint4*>(v + (c >> 3) * kBoxT + r * 128 + (c & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        // P as bf16 into the chunk's score buffer (its scores are in
        // registers on both halves: the pair barrier above), two keys per
        // column, this half's keys at columns [32·half, +32).
        {
          float pw[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) pw[j] = __uint_as_float(cvt_bf16x2(sc[2 * j], sc[2 * j + 1]));
          tmem_st32(tmem + lanes + kColS + (uint32_t)sb * kChunkT + half * 32, pw);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(pready);
      }
      if (!ok) break;
      // The row sum from both halves, then O / l for this half of the dims.
      {
        float* xs = xch + (size_t)((n & 1) * 2) * kRowsT;
        xs[half * kRowsT + r] = l;
        pair_sync();
        const float lo = xs[(1 - half) * kRowsT + r];
        pair_sync();  // read before the next item's chunk of the same parity writes
        l += lo;
      }
      if (nch > 0) {
        if (pair_any(!wait_odone(n - 1))) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      }
      const float lrow = l;
      const float inv = lrow > 0.f ? 1.0f / lrow : 0.f;
      bf16* out = (bf16*)a.out + (((size_t)b * a.S + (valid ? s_tok : 0)) * a.nq + (size_t)h * G + g) * D;
#pragma unroll 1
      for (int c4 = 0; c4 < kHD / 32; ++c4) {
        float o[32];
        if (nch > 0) {
          tmem_ld32(tmem + lanes + kColO + half * kHD + c4 * 32, o);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0.f;
        }
        if (valid) {
#pragma unroll
          for (int e8 = 0; e8 < 4; ++e8) {
            uint4 w;
            w.x = pack2(o[8 * e8 + 0] * inv, o[8 * e8 + 1] * inv);
            w.y = pack2(o[8 * e8 + 2] * inv, o[8 * e8 + 3] * inv);
            w.z = pack2(o[8 * e8 + 4] * inv, o[8 * e8 + 5] * inv);
            w.w = pack2(o[8 * e8 + 6] * inv, o[8 * e8 + 7] * inv);
            *reinterpret_cast<uint4*>(out + half * kHD + c4 * 32 + 8 * e8) = w;
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    if (!ok) *abort_flag = 1;
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // Let the loads this CTA issued land before its shared memory goes away.
    for (long long i = issued > 2 ? issued - 2 : 0; i < issued; ++i)
      mbar_wait(&kvfull[i & 1], (int)(i >> 1) & 1, a.err);
  }
  if (warp == 1 && lane == 0) mbar_wait(drain, 0, a.err);  // every MMA has finished
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

int sm_count_prefill_tc() {
  return usable_sms();
}

}  // namespace

bool attention_prefill_tc_applicable(int dtype, int D, int G, int S) {
  return dtype == kBF16 && (D == 64 || D == 128) && G >= 1 && G <= 16 && 16 % G == 0 && S >= 8 &&
         tc_host::encoder() != nullptr;
}

cudaError_t launch_attention_prefill_tc(const AttnArgs& a, cudaStream_t s) {
  if ((uintptr_t)a.q % 16 || (uintptr_t)a.out % 16) return cudaErrorInvalidValue;
  const int G = a.nq / a.nkv;
  PrefillPlan pl;
  pl.tq = kRowsT / G;
  pl.ntiles = (a.S + pl.tq - 1) / pl.tq;
  pl.items = (long long)pl.ntiles * a.B * a.nkv;
  if (pl.items <= 0) return cudaSuccess;
  auto go = [&](auto kernel, int smem) -> cudaError_t {
    static bool configured[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    bool& done = configured[a.D == 128][dev];
    if (!done) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      done = true;
    }
    const long long cap = sm_count_prefill_tc();
    const int grid = (int)(pl.items < cap ? pl.items : cap);
    return launch_pdl(kernel, dim3(grid), dim3(kThreadsT), smem, s, a, pl);
  };
  if (a.D == 128) return go(attn_prefill_tc_kernel<128>, TcPrefillLayout<128>::kBytes);
  return go(attn_prefill_tc_kernel<64>, TcPrefillLayout<64>::kBytes);
}

}  // namespace mg
