// Prefill / multi-token GQA attention on the tensor cores (bf16, head_dim 64
// or 128): query tiles against 128-key chunks of the stage-owned KV.
//
// A work item is one cache row b, one KV head h and a tile of 128 query rows:
// 128 / G tokens x the G query heads that share h (so every key and value
// chunk loaded feeds 128 query rows).  The kernel is persistent, one CTA per
// SM, items in order of decreasing key count, CTA c taking items c, c + grid,
// ...  Warp 8 (one lane) loads the item's query rows with bulk copies and
// each 128-key chunk of keys and values with 2-D TMA through the slot's
// tensor map (box 128 keys x 64 dims, 128-byte swizzle, no multicast) into a
// 2- or 3-stage ring.  Warps 0-7 own 16 query rows each and stream through
// the chunks with the flash-attention recurrence on mma.sync m16n8k16:
//   S = Q·Kᵀ (A = Q rows, B = keys via ldmatrix), masked by the visible-key
//   rule of the reference's mask policy, scores in base 2;
//   m' = max(m, rowmax S), P = exp2(S - m'), l = l·exp2(m - m') + rowsum P;
//   O = O·exp2(m - m') + P·V (P from S's accumulators as bf16 high + low
//   parts, two MMAs, so the weights keep fp32 accuracy; B = V via
//   ldmatrix.trans);
// and write O / l for their rows.  No state crosses warps or CTAs.  Every
// wait is bounded (code 3 in the error word on expiry).
#include <math.h>

#include "attn_tc_common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace mg {
namespace {

using namespace tc;
using namespace attn;

constexpr int kWarpsP = 8;
constexpr int kThreadsP = (kWarpsP + 1) * 32;
constexpr int kRowsP = kWarpsP * 16;        // query rows of a tile
constexpr int kChunkP = kKvBoxKeys;         // keys per chunk (128)
constexpr int kBoxP = kKvBoxKeys * 128;     // one 128-key x 64-dim box
constexpr int kMaxStagesP = 3;
constexpr int kMaxSmemP = 227 * 1024;

template <int D>
struct PrefillLayout {
  static constexpr int kDB = D / 64;
  static constexpr int kKV = kDB * kBoxP;   // K (or V) of a chunk
  static constexpr int kQ = kRowsP * D * 2;  // the tile's query rows
  static constexpr int kStage = 2 * kKV + kQ;
  static constexpr int bytes(int stages) { return stages * kStage + 2 * kMaxStagesP * 8 + 16 + 1024; }
};

template <int D>
__global__ void __launch_bounds__(kThreadsP, 1) attn_prefill_kernel(AttnArgs a, PrefillPlan pl, int stages) {
  using L = PrefillLayout<D>;
  constexpr int DB = L::kDB;
  constexpr int KS = D / 16;  // k-steps of the score MMA
  constexpr int DN = D / 8;   // dim n-tiles of the output
  const int G = a.nq / a.nkv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + stages * L::kStage);
  uint64_t* empty = full + kMaxStagesP;
  volatile int* abort_flag = (volatile int*)(empty + kMaxStagesP);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarpsP);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // the query rows and this forward's keys come from the kernel before

  if (warp == kWarpsP) {
    if (lane == 0) {
      long long n = 0;
      for (long long i = blockIdx.x; i < pl.items && !*abort_flag; i += gridDim.x) {
        int qt, b, h;
        item_of(a, pl, i, qt, b, h);
        const RowDesc rd = a.rows[b];
        const int nch = (tile_keys(a, rd, pl, b, qt) + kChunkP - 1) / kChunkP;
        int s_hi = (qt + 1) * pl.tq;
        if (s_hi > a.S) s_hi = a.S;
        for (int ch = 0; ch < nch; ++ch, ++n) {
          const int s = (int)(n % stages);
          if (n >= stages && !mbar_wait(&empty[s], (int)((n / stages) - 1) & 1, a.err)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* st = smem + s * L::kStage;
          const int k0 = ch * kChunkP;
          const int yk = (int)kv_row(a.layer, 0, rd.slot_rows, rd.row, a.nkv, h, rd.cap, k0);
          const int yv = (int)kv_row(a.layer, 1, rd.slot_rows, rd.row, a.nkv, h, rd.cap, k0);
          uint32_t bytes = 2 * L::kKV;
          if (ch == 0) bytes += (uint32_t)((s_hi - qt * pl.tq) * G * D * 2);
          mbar_expect_tx(&full[s], bytes);
          for (int db = 0; db < DB; ++db) tma_load_2d_gmap(st + db * kBoxP, rd.kv_tmap, &full[s], db * 64, yk);
          for (int db = 0; db < DB; ++db)
            tma_load_2d_gmap(st + L::kKV + db * kBoxP, rd.kv_tmap, &full[s], db * 64, yv);
          if (ch == 0) {
            // Query rows of the tile: token s, heads h·G .. h·G + G - 1, one run each.
            for (int t = qt * pl.tq; t < s_hi; ++t)
              bulk_load(st + 2 * L::kKV + (size_t)(t - qt * pl.tq) * G * D * 2,
                        (const __nv_bfloat16*)a.q + (((size_t)b * a.S + t) * a.nq + (size_t)h * G) * D,
                        (uint32_t)(G * D * 2), &full[s]);
          }
        }
      }
      if (*abort_flag) {
        for (long long i = n > stages ? n - stages : 0; i < n; ++i)
          mbar_wait(&full[i % stages], (int)(i / stages) & 1, a.err);
      }
    }
  } else {
    const int g = lane >> 2, t = lane & 3;
    const float scale2 = a.scale * 1.4426950408889634f;
    long long n = 0;
    for (long long i = blockIdx.x; i < pl.items; i += gridDim.x) {
      int qt, b, h;
      item_of(a, pl, i, qt, b, h);
      const RowDesc rd = a.rows[b];
      const int nch = (tile_keys(a, rd, pl, b, qt) + kChunkP - 1) / kChunkP;
      // This thread's two rows of the warp's 16: tile rows 16w + g and + 8.
      const int rA = warp * 16 + g, rB = rA + 8;
      const int sA = qt * pl.tq + rA / G, sB = qt * pl.tq + rB / G;
      const int visA = sA < a.S ? visible(a, rd, b * a.S + sA, sA) : 0;
      const int visB = sB < a.S ? visible(a, rd, b * a.S + sB, sB) : 0;
      int wvis = max(visA, visB);  // the warp's furthest visible key
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) wvis = max(wvis, __shfl_xor_sync(0xffffffffu, wvis, o));
      float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
      float o[DN][4];
#pragma unroll
      for (int i2 = 0; i2 < DN; ++i2) o[i2][0] = o[i2][1] = o[i2][2] = o[i2][3] = 0.f;
      uint32_t qa[KS][4];
      bool stop = false;
      for (int ch = 0; ch < nch; ++ch) {
        const int s = (int)(n % stages);
        const bool ok = mbar_wait(&full[s], (int)(n / stages) & 1, a.err);
        ++n;
        if (!ok || *abort_flag) {
          *abort_flag = 1;
          stop = true;
          break;
        }
        uint8_t* st = smem + s * L::kStage;
        if (ch == 0) {
          const __nv_bfloat16* Q = (const __nv_bfloat16*)(st + 2 * L::kKV);
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            qa[ks][0] = *reinterpret_cast<const uint32_t*>(Q + rA * D + 16 * ks + 2 * t);
            qa[ks][1] = *reinterpret_cast<const uint32_t*>(Q + rB * D + 16 * ks + 2 * t);
            qa[ks][2] = *reinterpret_cast<const uint32_t*>(Q + rA * D + 16 * ks + 8 + 2 * t);
            qa[ks][3] = *reinterpret_cast<const uint32_t*>(Q + rB * D + 16 * ks + 8 + 2 * t);
          }
        }
        const uint32_t kbase = smem_u32(st), vbase = smem_u32(st + L::kKV);
        // The chunk in two halves of 64 keys (register budget).
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
          const int k0 = ch * kChunkP + 64 * hf;  // first key of the half
          if (k0 >= wvis) break;
          const int nt_end = min(8, (wvis - k0 + 7) / 8);  // n-tiles of 8 keys with a visible key
          float sc[8][4];
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) {
            if (nt >= nt_end) break;
#pragma unroll
            for (int ks = 0; ks < KS; ks += 2) {
              const int r = 64 * hf + 8 * nt + (lane & 7);
              const int cc = 2 * ks + (lane >> 3);
              uint32_t bfr[4];
              ldsm_x4(kbase + (cc >> 3) * kBoxP + swz(r, cc & 7), bfr);
              mma16816_full(sc[nt], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], bfr[0], bfr[1]);
              mma16816_full(sc[nt], qa[ks + 1][0], qa[ks + 1][1], qa[ks + 1][2], qa[ks + 1][3], bfr[2], bfr[3]);
            }
          }
          // Mask, scale to base 2, row maxima (rows rA: c0/c1, rB: c2/c3).
          float mxA = mA, mxB = mB;
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) {
            const int key = k0 + 8 * nt + 2 * t;
            sc[nt][0] = key < visA ? sc[nt][0] * scale2 : -INFINITY;
            sc[nt][1] = key + 1 < visA ? sc[nt][1] * scale2 : -INFINITY;
            sc[nt][2] = key < visB ? sc[nt][2] * scale2 : -INFINITY;
            sc[nt][3] = key + 1 < visB ? sc[nt][3] * scale2 : -INFINITY;
            mxA = fmaxf(mxA, fmaxf(sc[nt][0], sc[nt][1]));
            mxB = fmaxf(mxB, fmaxf(sc[nt][2], sc[nt][3]));
          }
          mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
          mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
          mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
          mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
          const float keepA = (mA == -INFINITY || mxA == -INFINITY) ? 0.f : exp2f(mA - mxA);
          const float keepB = (mB == -INFINITY || mxB == -INFINITY) ? 0.f : exp2f(mB - mxB);
          float sumA = 0.f, sumB = 0.f;
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) {
            sc[nt][0] = sc[nt][0] == -INFINITY ? 0.f : exp2f(sc[nt][0] - mxA);
            sc[nt][1] = sc[nt][1] == -INFINITY ? 0.f : exp2f(sc[nt][1] - mxA);
            sc[nt][2] = sc[nt][2] == -INFINITY ? 0.f : exp2f(sc[nt][2] - mxB);
            sc[nt][3] = sc[nt][3] == -INFINITY ? 0.f : exp2f(sc[nt][3] - mxB);
            sumA += sc[nt][0] + sc[nt][1];
            sumB += sc[nt][2] + sc[nt][3];
          }
          sumA += __shfl_xor_sync(0xffffffffu, sumA, 1);
          sumA += __shfl_xor_sync(0xffffffffu, sumA, 2);
          sumB += __shfl_xor_sync(0xffffffffu, sumB, 1);
          sumB += __shfl_xor_sync(0xffffffffu, sumB, 2);
          lA = lA * keepA + sumA;
          lB = lB * keepB + sumB;
          if (mxA != -INFINITY) mA = mxA;
          if (mxB != -INFINITY) mB = mxB;
#pragma unroll
          for (int dn = 0; dn < DN; ++dn) {
            o[dn][0] *= keepA;
            o[dn][1] *= keepA;
            o[dn][2] *= keepB;
            o[dn][3] *= keepB;
          }
          // O += P·V, 16 keys per k-step, taken while a key of the step is
          // visible.  Value rows at or past the cache's end were never
          // written (P is 0 there, but 0 * NaN is not): their halves of the
          // value fragments are cleared.
          const int tot = rd.past + a.S - k0;  // written keys from k0 on
#pragma unroll
          for (int kt = 0; kt < 4; ++kt) {
            if (2 * kt >= nt_end) break;
            const int kr = 16 * kt + 2 * t;  // this thread's fragment keys: kr, kr+1, kr+8, kr+9
            const uint32_t m0 = (kr < tot ? 0x0000ffffu : 0u) | (kr + 1 < tot ? 0xffff0000u : 0u);
            const uint32_t m1 = (kr + 8 < tot ? 0x0000ffffu : 0u) | (kr + 9 < tot ? 0xffff0000u : 0u);
            const uint32_t pa0 = pack2(sc[2 * kt][0], sc[2 * kt][1]);
            const uint32_t pa1 = pack2(sc[2 * kt][2], sc[2 * kt][3]);
            const uint32_t pa2 = pack2(sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
            const uint32_t pa3 = pack2(sc[2 * kt + 1][2], sc[2 * kt + 1][3]);
            const uint32_t pl0 = pack2(sc[2 * kt][0] - lo_bf16(pa0), sc[2 * kt][1] - hi_bf16(pa0));
            const uint32_t pl1 = pack2(sc[2 * kt][2] - lo_bf16(pa1), sc[2 * kt][3] - hi_bf16(pa1));
            const uint32_t pl2 = pack2(sc[2 * kt + 1][0] - lo_bf16(pa2), sc[2 * kt + 1][1] - hi_bf16(pa2));
            const uint32_t pl3 = pack2(sc[2 * kt + 1][2] - lo_bf16(pa3), sc[2 * kt + 1][3] - hi_bf16(pa3));
#pragma unroll
            for (int dn = 0; dn < DN; dn += 2) {
              const int mi = lane >> 3;
              const int r = 64 * hf + 16 * kt + (lane & 7) + 8 * (mi & 1);
              const int cc = dn + (mi >> 1);
              uint32_t bfr[4];
              ldsm_x4_t(vbase + (cc >> 3) * kBoxP + swz(r, cc & 7), bfr);
              bfr[0] &= m0;
              bfr[1] &= m1;
              bfr[2] &= m0;
              bfr[3] &= m1;
              mma16816_full(o[dn], pa0, pa1, pa2, pa3, bfr[0], bfr[1]);
              mma16816_full(o[dn], pl0, pl1, pl2, pl3, bfr[0], bfr[1]);
              mma16816_full(o[dn + 1], pa0, pa1, pa2, pa3, bfr[2], bfr[3]);
              mma16816_full(o[dn + 1], pl0, pl1, pl2, pl3, bfr[2], bfr[3]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      if (stop) break;
      // Normalise and store this thread's two rows.
      const float invA = lA > 0.f ? 1.0f / lA : 0.f, invB = lB > 0.f ? 1.0f / lB : 0.f;
      __nv_bfloat16* out = (__nv_bfloat16*)a.out;
      if (sA < a.S) {
        __nv_bfloat16* oa = out + (((size_t)b * a.S + sA) * a.nq + (size_t)h * G + rA % G) * D;
#pragma unroll
        for (int dn = 0; dn < DN; ++dn)
          *reinterpret_cast<uint32_t*>(oa + 8 * dn + 2 * t) = pack2(o[dn][0] * invA, o[dn][1] * invA);
      }
      if (sB < a.S) {
        __nv_bfloat16* ob = out + (((size_t)b * a.S + sB) * a.nq + (size_t)h * G + rB % G) * D;
#pragma unroll
        for (int dn = 0; dn < DN; ++dn)
          *reinterpret_cast<uint32_t*>(ob + 8 * dn + 2 * t) = pack2(o[dn][2] * invB, o[dn][3] * invB);
      }
    }
  }
  __syncthreads();
}

int sm_count_prefill() {
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

bool attention_prefill_applicable(int dtype, int D, int G, int S) {
  return dtype == kBF16 && (D == 64 || D == 128) && G >= 1 && G <= 16 && 16 % G == 0 && S >= 8;
}

cudaError_t launch_attention_prefill(const AttnArgs& a, cudaStream_t s) {
  if ((uintptr_t)a.q % 16 || (uintptr_t)a.out % 16) return cudaErrorInvalidValue;
  const int G = a.nq / a.nkv;
  PrefillPlan pl;
  pl.tq = kRowsP / G;
  pl.ntiles = (a.S + pl.tq - 1) / pl.tq;
  pl.items = (long long)pl.ntiles * a.B * a.nkv;
  if (pl.items <= 0) return cudaSuccess;
  auto go = [&](auto kernel, int stages) -> cudaError_t {
    const int smem = (a.D == 128 ? PrefillLayout<128>::bytes(stages) : PrefillLayout<64>::bytes(stages));
    static bool configured[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    bool& done = configured[a.D == 128][dev];
    if (!done) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmemP);
      if (e != cudaSuccess) return e;
      done = true;
    }
    const long long cap = sm_count_prefill();
    const int grid = (int)(pl.items < cap ? pl.items : cap);
    return launch_pdl(kernel, dim3(grid), dim3(kThreadsP), smem, s, a, pl, stages);
  };
  if (a.D == 128) return go(attn_prefill_kernel<128>, 2);
  return go(attn_prefill_kernel<64>, 3);
}

}  // namespace mg
