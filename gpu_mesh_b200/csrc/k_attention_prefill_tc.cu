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
//     N = 128 keys, K = D; Q and K both K-major) into one of two TMEM score
//     buffers, then O += P·V (M = 128 rows, N = D, K = 128 keys; P K-major,
//     V read MN-major straight from its TMA box) into the TMEM output.  The
//     score product of chunk j + 1 is issued before the value product of
//     chunk j, so it overlaps that chunk's softmax;
//   * warps 2-5: one thread per query row (its TMEM lane).  They write the
//     tile's query rows into shared memory, and per chunk read their row of
//     S, mask it by the reference's visible-key rule, keep the online softmax
//     in base 2 (m' = max(m, max S), P = exp2(S - m'), l = l·exp2(m - m') +
//     ΣP), rescale their row of O in TMEM when the maximum moved, and write
//     P as bf16 high + low parts (two MMAs, so the weights keep fp32
//     accuracy) for the value product.  At the end they write O / l.
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
constexpr int kThreadsT = 192;
constexpr int kColS = 0;                 // TMEM columns: scores [0, 256) in two buffers,
constexpr int kColO = 256;               // the output [256, 256 + D)

template <int D>
struct TcPrefillLayout {
  static constexpr int kDB = D / 64;       // 64-wide blocks of D
  static constexpr int kQ = kDB * kBoxT;   // query tile (A of S)
  static constexpr int kP = 2 * kBoxT;     // P tile (128 rows x 128 keys), each of high / low
  static constexpr int kKV = kDB * kBoxT;  // keys (or values) of a chunk
  static constexpr int kStages = 2;
  static constexpr int kOffQ = 0;
  static constexpr int kOffPh = kOffQ + kQ;
  static constexpr int kOffPl = kOffPh + kP;
  static constexpr int kOffKV = kOffPl + kP;
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
  uint8_t* sph = smem + L::kOffPh;
  uint8_t* spl = smem + L::kOffPl;
  uint8_t* skv = smem + L::kOffKV;  // stage s: keys at skv + 2·s·kKV, values kKV after them
  uint64_t* bars = (uint64_t*)(smem + L::kOffBar);
  uint64_t* kvfull = bars;       // [2] chunk landed
  uint64_t* kvempty = bars + 2;  // [2] chunk's value product done
  uint64_t* sfull = bars + 4;    // [2] scores ready in TMEM buffer
  uint64_t* pready = bars + 6;   // P written, O rescaled (4 warps)
  uint64_t* odone = bars + 7;    // value product done
  uint64_t* qready = bars + 8;   // query tile written (4 warps)
  uint64_t* drain = bars + 9;    // every MMA finished
  uint32_t* tmem_holder = (uint32_t*)(bars + 10);
  volatile int* abort_flag = (volatile int*)(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kvfull[s], 1);
      mbar_init(&kvempty[s], 1);
      mbar_init(&sfull[s], 1);
    }
    mbar_init(pready, 4);
    mbar_init(odone, 1);
    mbar_init(qready, 4);
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
      // score product into TMEM buffer n & 1, then the value product of chunk
      // n - 1 once its P is written (and of the item's last chunk at the end).
      constexpr uint32_t idS = instr_desc(kChunkT);
      constexpr uint32_t idPV = instr_desc(D) | (1u << 16);  // B (the values) MN-major
      long long n = 0;
      int it = 0;
      auto value_product = [&](long long m, bool first) -> bool {
        if (!mbar_wait(pready, (int)(m & 1), a.err)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint8_t* v = skv + (int)(m & 1) * 2 * L::kKV + L::kKV;
#pragma unroll
        for (int part = 0; part < 2; ++part) {  // P high, then P low
          const uint8_t* pp = part ? spl : sph;
#pragma unroll
          for (int kk = 0; kk < kChunkT / 16; ++kk) {
            const uint64_t da = smem_desc(pp + (kk >> 2) * kBoxT) + (uint64_t)((kk & 3) * 2);
            const uint64_t db = smem_desc_mn(v + kk * 16 * 128, kBoxT);
            mma_bf16(tmem + kColO, da, db, idPV, (first && part == 0 && kk == 0) ? 0u : 1u);
          }
        }
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
          if (!mbar_wait(&kvfull[n & 1], (int)(n >> 1) & 1, a.err) || *abort_flag) {
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
        if (ok && nch > 0 && !value_product(n - 1, nch == 1)) ok = false;
      }
      if (!ok) *abort_flag = 1;
      mma_commit(drain);  // arrives once every MMA issued above has finished
    }
  } else {
    // Softmax warps 2-5: warp w owns TMEM lanes 32·(w % 4) .. + 31, one
    // query row per thread.
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
    const float scale2 = a.scale * 1.4426950408889634f;
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
      // The query row into the tile (zeros for rows past the sequence).
      {
        const uint4* src = reinterpret_cast<const uint4*>(
            (const bf16*)a.q + (((size_t)b * a.S + (valid ? s_tok : 0)) * a.nq + (size_t)h * G + g) * D);
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          const uint4 val = valid ? src[c] : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(sq + swz_off(r, c)) = val;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(qready);

      float m = -INFINITY, l = 0.f;
      for (int ch = 0; ch < nch; ++ch, ++n) {
        const int sb = (int)(n & 1);
        // scores ready; the chunk's load is complete too (it orders the TMA
        // writes before the value clearing below)
        if (!warp_wait(&sfull[sb], (int)(n >> 1) & 1, a.err) ||
            !warp_wait(&kvfull[sb], (int)(n >> 1) & 1, a.err)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float sc[kChunkT];
#pragma unroll
        for (int c4 = 0; c4 < kChunkT / 32; ++c4)
          tmem_ld32(tmem + lanes + kColS + (uint32_t)sb * kChunkT + c4 * 32, sc + c4 * 32);
        const int nv = vis - ch * kChunkT;  // visible keys of this chunk for this row
        float mx = m;
#pragma unroll
        for (int c = 0; c < kChunkT; ++c) {
          sc[c] = c < nv ? sc[c] * scale2 : -INFINITY;
          mx = fmaxf(mx, sc[c]);
        }
        const float alpha = (m == -INFINITY) ? 1.f : exp2f(m - mx);
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < kChunkT; ++c) {
          sc[c] = sc[c] == -INFINITY ? 0.f : exp2f(sc[c] - mx);
          sum += sc[c];
        }
        l = l * alpha + sum;
        m = mx;
        if (ch > 0) {
          // The previous value product is done: O is stable and P is free.
          if (!warp_wait(odone, (int)((n - 1) & 1), a.err)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
            for (int c4 = 0; c4 < D / 32; ++c4) {
              float o[32];
              tmem_ld32(tmem + lanes + kColO + c4 * 32, o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] *= alpha;
              tmem_st32(tmem + lanes + kColO + c4 * 32, o);
            }
          }
        }
        // Value rows past the written keys: clear them before the product.
        if (ch * kChunkT + kChunkT > tot && ch * kChunkT + r >= tot) {
          uint8_t* v = skv + sb * 2 * L::kKV + L::kKV;
#pragma unroll
          for (int db = 0; db < DB; ++db)
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(v + db * kBoxT + r * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        // P = high + low bf16 parts, this row of the K-major P tiles.
#pragma unroll
        for (int c8 = 0; c8 < kChunkT / 8; ++c8) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x0 = sc[8 * c8 + 2 * e], x1 = sc[8 * c8 + 2 * e + 1];
            hw[e] = pack2(x0, x1);
            lw[e] = pack2(x0 - lo_bf16(hw[e]), x1 - hi_bf16(hw[e]));
          }
          const int off = swz_off(r, c8);
          *reinterpret_cast<uint4*>(sph + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(spl + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(pready);
      }
      if (!ok) break;
      // O / l for this row.
      if (nch > 0) {
        if (!warp_wait(odone, (int)((n - 1) & 1), a.err)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      }
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      bf16* out = (bf16*)a.out + (((size_t)b * a.S + (valid ? s_tok : 0)) * a.nq + (size_t)h * G + g) * D;
#pragma unroll 1
      for (int c4 = 0; c4 < D / 32; ++c4) {
        float o[32];
        if (nch > 0) {
          tmem_ld32(tmem + lanes + kColO + c4 * 32, o);
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
            *reinterpret_cast<uint4*>(out + c4 * 32 + 8 * e8) = w;
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
