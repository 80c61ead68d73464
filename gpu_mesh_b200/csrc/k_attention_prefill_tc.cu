// Prefill / multi-token GQA attention on tcgen05 (bf16, head_dim 64 or 128).
//
// A query tile is 128 rows of one cache row b and one KV head h: 128 / G
// tokens x the G query heads that share h (row r = token r / G, head r % G),
// so every key and value chunk feeds 128 rows.  A work item is two adjacent
// tiles of the same (b, h), A (earlier tokens) and B, which share every key
// and value chunk they both see.  The kernel is persistent (one CTA per SM,
// items heaviest first) and splits the flash recurrence over its warps:
//   * warp 0, one lane: loads both tiles' query rows with 4-D TMA over the
//     query buffer {D, heads, tokens, rows} (box 64 dims x G heads x 128 / G
//     tokens, tokens past the sequence read as zeros), the next item's as soon
//     as the current item's last score product of the tile is done; and each
//     128-key chunk of keys and values with 2-D TMA through the slot's tensor
//     map (box 128 keys x 64 dims, 128-byte swizzle, no multicast) into a
//     2-stage ring;
//   * warp 1, one lane: issues tcgen05.mma.  For tile X: S_X = Q_X·Kᵀ (M =
//     128 query rows, N = 128 keys, K = D) into X's TMEM score columns, and
//     O_X += P_X·V (M = 128 rows, N = D, K = 128 keys) into X's TMEM output,
//     with P_X read from TMEM (where the softmax left it, over S_X) and V
//     read MN-major straight from its TMA box.  The two tiles ping-pong: when
//     A's P of chunk j is ready, its value product and (once that is done)
//     its score product of chunk j + 1 run while B's softmax works on chunk
//     j, and the other way round;
//   * warps 2-5 (tile A) and 6-9 (tile B): one thread per query row (its
//     TMEM lane).  Per chunk they read S's row, mask it by the reference's
//     visible-key rule and keep the online softmax in base 2
//     (P = 2^(S·scale2 - m·scale2), l = l·α + ΣP).  The running maximum m is moved only when a row's scores
//     exceed it by more than 2^8, and only then is the row of O in TMEM
//     rescaled by α (the result O / l does not depend on which m is used).
//     P goes back into TMEM as bf16 (the precision the reference's own
//     attention multiplies the values in), l sums it in fp32.  At the end
//     they write O / l.
// Value rows at or past the cache end were never written: they are cleared
// in shared memory before the value products (P is 0 there, but 0 * NaN is
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
constexpr int kSoftWarps = 8;            // four per tile, one query row per thread
constexpr int kThreadsT = 64 + 32 * kSoftWarps;
// TMEM columns: tile X's scores (then P) at [128·X, +128), its output at
// 256 + D·X.
constexpr int kColS = 0;
constexpr int kColO = 256;

template <int D>
struct TcPrefillLayout {
  static constexpr int kDB = D / 64;       // 64-wide blocks of D
  static constexpr int kQ = kDB * kBoxT;   // one tile's query rows (A of S)
  static constexpr int kKV = kDB * kBoxT;  // keys (or values) of a chunk
  static constexpr int kStages = 2;
  static constexpr int kOffQ = 0;          // tile X at kOffQ + X·kQ
  static constexpr int kOffKV = kOffQ + 2 * kQ;
  static constexpr int kOffBar = kOffKV + kStages * 2 * kKV;
  static constexpr int kBytes = kOffBar + 256 + 1024;
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

// Item i (heaviest first): its tile pair (tiles 2j and 2j + 1), cache row,
// KV head.
__device__ __forceinline__ void pair_of(const AttnArgs& a, const PrefillPlan& pl, long long i, int& qa, int& b,
                                        int& h) {
  const long long bh = (long long)a.B * a.nkv;
  const int npairs = (pl.ntiles + 1) / 2;
  qa = 2 * (npairs - 1 - (int)(i / bh));
  const int rem = (int)(i % bh);
  b = rem / a.nkv;
  h = rem % a.nkv;
}

// Chunks tile qt of row b needs (0 for a tile past the sequence).
__device__ __forceinline__ int tile_chunks(const AttnArgs& a, const RowDesc& rd, const PrefillPlan& pl, int b,
                                           int qt) {
  if (qt >= pl.ntiles) return 0;
  return (tile_keys(a, rd, pl, b, qt) + kChunkT - 1) / kChunkT;
}

template <int D>
__global__ void __launch_bounds__(kThreadsT, 1) attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                                    AttnArgs a, PrefillPlan pl) {
  using L = TcPrefillLayout<D>;
  const int G = a.nq / a.nkv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sq = smem + L::kOffQ;    // tile X's query rows at sq + X·kQ
  uint8_t* skv = smem + L::kOffKV;  // stage s: keys at skv + 2·s·kKV, values kKV after them
  uint64_t* bars = (uint64_t*)(smem + L::kOffBar);
  uint64_t* kvfull = bars;        // [2] chunk landed
  uint64_t* kvempty = bars + 2;   // [2] chunk's products done
  uint64_t* sfull = bars + 4;     // [tile] scores ready in TMEM
  uint64_t* pready = bars + 6;    // [tile] P written, O rescaled (the tile's four softmax warps)
  uint64_t* odone = bars + 8;     // [tile] value product done
  uint64_t* qfull = bars + 10;    // [tile] query rows landed
  uint64_t* qempty = bars + 12;   // [tile] the item's score products read them
  uint64_t* drain = bars + 14;    // every MMA finished
  uint32_t* tmem_holder = (uint32_t*)(bars + 15);
  volatile int* abort_flag = (volatile int*)(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kvfull[s], 1);
      mbar_init(&kvempty[s], 1);
      mbar_init(&sfull[s], 1);
      mbar_init(&pready[s], kSoftWarps / 2);
      mbar_init(&odone[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&qfull[x], 1);
      mbar_init(&qempty[x], 1);
    }
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
  int qn[2] = {0, 0};  // query tile loads issued per tile (producer)
  if (warp == 0) {
    if (lane == 0) {
      long long n = 0;  // ring position of the next chunk
      for (long long i = blockIdx.x; i < pl.items && !*abort_flag; i += gridDim.x) {
        int qa, b, h;
        pair_of(a, pl, i, qa, b, h);
        const RowDesc rd = a.rows[b];
        const int nx[2] = {tile_chunks(a, rd, pl, b, qa), tile_chunks(a, rd, pl, b, qa + 1)};
        const int nch = max(nx[0], nx[1]);
        // The tiles' query rows (tokens past the sequence read as zeros), once
        // the previous item's score products of the tile have read theirs.
        for (int x = 0; x < 2; ++x) {
          if (nx[x] == 0) continue;
          if (qn[x] > 0 && !mbar_wait(&qempty[x], (qn[x] - 1) & 1, a.err)) {
            *abort_flag = 1;
            break;
          }
          mbar_expect_tx(&qfull[x], L::kQ);
          for (int db = 0; db < L::kDB; ++db)
            tma_load_4d(sq + x * L::kQ + db * kBoxT, &tm_q, &qfull[x], db * 64, h * G, (qa + x) * pl.tq, b);
          ++qn[x];
        }
        if (*abort_flag) break;
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
          for (int db = 0; db < L::kDB; ++db) {
            tma_load_2d_gmap(st + db * kBoxT, rd.kv_tmap, &kvfull[s], db * 64, yk);
            tma_load_2d_gmap(st + L::kKV + db * kBoxT, rd.kv_tmap, &kvfull[s], db * 64, yv);
          }
          issued = n + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer.  Per item: wait for both query tiles, issue both score
      // products of chunk 0; then per chunk, for each tile that sees it: wait
      // for its P, issue its value product, wait for that to finish (the next
      // score product overwrites the columns P is read from) and issue its
      // score product of the next chunk.
      constexpr uint32_t idS = instr_desc(kChunkT);
      constexpr uint32_t idPV = instr_desc(D) | (1u << 16);  // B (the values) MN-major
      long long n = 0;        // ring position of the item's first chunk
      long long kv_seen = 0;  // ring positions whose load this thread has waited for
      long long cnt[2] = {0, 0};  // chunks of each tile so far (its sfull / pready / odone phases)
      int qm[2] = {0, 0};         // query tiles of each tile so far (qfull / qempty phases)
      bool ok = true;
      auto wait_kv = [&](long long upto) -> bool {  // loads of ring positions < upto have landed
        for (; kv_seen < upto; ++kv_seen)
          if (!mbar_wait(&kvfull[kv_seen & 1], (int)(kv_seen >> 1) & 1, a.err)) return false;
        return true;
      };
      auto score = [&](int x, long long pos) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint8_t* k = skv + (int)(pos & 1) * 2 * L::kKV;
        const uint8_t* q = sq + x * L::kQ;
#pragma unroll
        for (int kd = 0; kd < D / 16; ++kd) {
          const uint64_t da = smem_desc(q + (kd >> 2) * kBoxT) + (uint64_t)((kd & 3) * 2);
          const uint64_t db = smem_desc(k + (kd >> 2) * kBoxT) + (uint64_t)((kd & 3) * 2);
          mma_bf16(tmem + kColS + 128 * x, da, db, idS, kd > 0 ? 1u : 0u);
        }
        mma_commit(&sfull[x]);
      };
      auto value = [&](int x, long long pos, bool first) -> bool {
        if (!mbar_wait(&pready[x], (int)(cnt[x] & 1), a.err)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint8_t* v = skv + (int)(pos & 1) * 2 * L::kKV + L::kKV;
#pragma unroll
        for (int kk = 0; kk < kChunkT / 16; ++kk)
          mma_bf16_ta(tmem + kColO + D * x, tmem + kColS + 128 * x + kk * 8, smem_desc_mn(v + kk * 16 * 128, kBoxT),
                      idPV, (first && kk == 0) ? 0u : 1u);
        mma_commit(&odone[x]);
        const bool done = mbar_wait(&odone[x], (int)(cnt[x] & 1), a.err);
        ++cnt[x];
        return done;
      };
      for (long long i = blockIdx.x; i < pl.items && ok && !*abort_flag; i += gridDim.x) {
        int qa, b, h;
        pair_of(a, pl, i, qa, b, h);
        const RowDesc rd = a.rows[b];
        const int nx[2] = {tile_chunks(a, rd, pl, b, qa), tile_chunks(a, rd, pl, b, qa + 1)};
        const int nch = max(nx[0], nx[1]);
        if (nch > 0) {
          if (!wait_kv(n + 1)) {
            ok = false;
            break;
          }
          for (int x = 0; x < 2 && ok; ++x) {
            if (nx[x] == 0) continue;
            if (!mbar_wait(&qfull[x], qm[x] & 1, a.err)) {
              ok = false;
              break;
            }
            score(x, n);
            if (nx[x] == 1) mma_commit(&qempty[x]);  // the tile's last score product
            ++qm[x];
          }
          if (!ok) break;
        }
        for (int ch = 0; ch < nch && ok; ++ch) {
          for (int x = 0; x < 2 && ok; ++x) {
            if (ch >= nx[x]) continue;
            if (!value(x, n + ch, ch == 0) || *abort_flag) {
              ok = false;
              break;
            }
            if (ch + 1 < nx[x]) {
              if (!wait_kv(n + ch + 2)) {
                ok = false;
                break;
              }
              score(x, n + ch + 1);
              if (ch + 2 == nx[x]) mma_commit(&qempty[x]);  // the tile's last score product
            }
          }
          mma_commit(&kvempty[(n + ch) & 1]);  // every product reading this chunk is issued
        }
        n += nch;
      }
      if (!ok) *abort_flag = 1;
      mma_commit(drain);  // arrives once every MMA issued above has finished
    }
  } else {
    // Softmax warps: warps 2-5 tile A, 6-9 tile B; warp w owns TMEM lanes
    // 32·(w % 4) .. + 31, one query row per thread.
    const int x = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
    const float scale2 = a.scale * 1.4426950408889634f;
    int n = 0;    // ring position of the item's first chunk
    int cnt = 0;  // this tile's chunks so far (its sfull / pready / odone phases)
    bool ok = true;
    for (int i = blockIdx.x; i < (int)pl.items && ok; i += gridDim.x) {
      int qa, b, h;
      pair_of(a, pl, i, qa, b, h);
      const RowDesc rd = a.rows[b];
      const int qt = qa + x;
      const int nchx = tile_chunks(a, rd, pl, b, qt);
      const int nch = max(tile_chunks(a, rd, pl, b, qa), tile_chunks(a, rd, pl, b, qa + 1));
      const int s_tok = qt * pl.tq + r / G;  // this row's query token
      const int g = r % G;
      const bool valid = qt < pl.ntiles && r / G < pl.tq && s_tok < a.S;
      const int vis = valid ? visible(a, rd, b * a.S + s_tok, s_tok) : 0;
      const int tot = rd.past + a.S;  // keys written so far

      float m = -INFINITY, l = 0.f;  // m: the running maximum P is taken against (raw scores)
      for (int ch = 0; ch < nchx; ++ch, ++cnt) {
        const int pos = n + ch;
        if (!warp_wait(&sfull[x], (int)(cnt & 1), a.err)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float sc[kChunkT];
        tmem_ld128(tmem + lanes + kColS + 128 * x, sc);
        const int nv = vis - ch * kChunkT;  // visible keys of this chunk for this row
        if (!__all_sync(0xffffffffu, nv >= kChunkT)) {
#pragma unroll
          for (int c = 0; c < kChunkT; ++c) sc[c] = c < nv ? sc[c] : -INFINITY;
        }
        // Row maximum of the raw scores (the scale is positive, so it
        // commutes with the maximum), as a tree; invisible keys are -inf.
        float t8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t8[j] = sc[j];
#pragma unroll
        for (int c = 8; c < kChunkT; ++c) t8[c & 7] = fmaxf(t8[c & 7], sc[c]);
        const float mt = fmaxf(fmaxf(fmaxf(t8[0], t8[1]), fmaxf(t8[2], t8[3])),
                               fmaxf(fmaxf(t8[4], t8[5]), fmaxf(t8[6], t8[7])));
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
        // key (invisible keys are -inf and give 0).
        const float mb = m_new == -INFINITY ? 0.f : m_new * scale2;
#pragma unroll
        for (int j = 0; j < 8; ++j) t8[j] = 0.f;
#pragma unroll
        for (int c = 0; c < kChunkT; ++c) {
          sc[c] = ex2_approx(fmaf(sc[c], scale2, -mb));
          t8[c & 7] += sc[c];
        }
        l = l * alpha + (((t8[0] + t8[1]) + (t8[2] + t8[3])) + ((t8[4] + t8[5]) + (t8[6] + t8[7])));
        m = m_new;
        // P as bf16 over the chunk's scores, two keys per column.
        {
          float pw[kChunkT / 2];
#pragma unroll
          for (int j = 0; j < kChunkT / 2; ++j) pw[j] = __uint_as_float(cvt_bf16x2(sc[2 * j], sc[2 * j + 1]));
          tmem_st64(tmem + lanes + kColS + 128 * x, pw);
        }
        // The previous value product of this tile has finished (the score
        // product just read was issued after it): rescale O's row in TMEM
        // before this chunk's value product adds to it.
        if (__any_sync(0xffffffffu, moved)) {
#pragma unroll 1
          for (int c4 = 0; c4 < D / 32; ++c4) {
            float o[32];
            tmem_ld32(tmem + lanes + kColO + D * x + c4 * 32, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(tmem + lanes + kColO + D * x + c4 * 32, o);
          }
        }
        // Value rows past the written keys: clear them before the value
        // products (both tiles' rows clear the same zeros; each tile's value
        // product waits only for its own rows' clearing).
        if (ch * kChunkT + kChunkT > tot && ch * kChunkT + r >= tot) {
          if (!mbar_wait(&kvfull[pos & 1], (int)(pos >> 1) & 1, a.err)) ok = false;
          uint8_t* v = skv + (int)(pos & 1) * 2 * L::kKV + L::kKV;
#pragma unroll
          for (int c = 0; c < D / 8; ++c)
            *reinterpret_cast<uint4*>(v + (c >> 3) * kBoxT + r * 128 + (c & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&pready[x]);
      }
      if (!ok) break;
      if (nchx > 0) {
        if (!warp_wait(&odone[x], (int)((cnt - 1) & 1), a.err)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      }
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      bf16* out = (bf16*)a.out + (((size_t)b * a.S + (valid ? s_tok : 0)) * a.nq + (size_t)h * G + g) * D;
      {
        // The row of O in one TMEM load (one wait), then 16-byte stores.
        float o[D];
        if (nchx > 0) {
          if constexpr (D == 128) {
            tmem_ld128(tmem + lanes + kColO + D * x, o);
          } else {
            tmem_ld64(tmem + lanes + kColO + D * x, o);
          }
        } else {
#pragma unroll
          for (int e = 0; e < D; ++e) o[e] = 0.f;
        }
        if (valid) {
#pragma unroll
          for (int e8 = 0; e8 < D / 8; ++e8) {
            uint4 w;
            w.x = pack2(o[8 * e8 + 0] * inv, o[8 * e8 + 1] * inv);
            w.y = pack2(o[8 * e8 + 2] * inv, o[8 * e8 + 3] * inv);
            w.z = pack2(o[8 * e8 + 4] * inv, o[8 * e8 + 5] * inv);
            w.w = pack2(o[8 * e8 + 6] * inv, o[8 * e8 + 7] * inv);
            *reinterpret_cast<uint4*>(out + 8 * e8) = w;
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      n += nch;
    }
    if (!ok) *abort_flag = 1;
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // Let the loads this CTA issued land before its shared memory goes away.
    for (long long i = issued > 2 ? issued - 2 : 0; i < issued; ++i)
      mbar_wait(&kvfull[i & 1], (int)(i >> 1) & 1, a.err);
    for (int x = 0; x < 2; ++x)
      if (qn[x] > 0) mbar_wait(&qfull[x], (qn[x] - 1) & 1, a.err);
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
  pl.items = (long long)((pl.ntiles + 1) / 2) * a.B * a.nkv;  // tile pairs
  if (pl.items <= 0) return cudaSuccess;
  // The query rows as a 4-D bf16 array {D, nq, S, B}: a box of 64 dims x G
  // heads x tq tokens x 1 row is one 64-wide block of a tile, rows in tile
  // order (token r / G, head r % G); tokens past S read as zeros.
  CUtensorMap tq;
  {
    tc_host::EncodeTiled enc = tc_host::encoder();
    if (!enc) return cudaErrorNotSupported;
    const cuuint64_t dims[4] = {(cuuint64_t)a.D, (cuuint64_t)a.nq, (cuuint64_t)a.S, (cuuint64_t)a.B};
    const cuuint64_t strides[3] = {(cuuint64_t)a.D * 2, (cuuint64_t)a.nq * a.D * 2,
                                   (cuuint64_t)a.S * a.nq * a.D * 2};
    const cuuint32_t box[4] = {64, (cuuint32_t)G, (cuuint32_t)pl.tq, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (enc(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(a.q), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
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
    return launch_pdl(kernel, dim3(grid), dim3(kThreadsT), smem, s, tq, a, pl);
  };
  if (a.D == 128) return go(attn_prefill_tc_kernel<128>, TcPrefillLayout<128>::kBytes);
  return go(attn_prefill_tc_kernel<64>, TcPrefillLayout<64>::kBytes);
}

}  // namespace mg
