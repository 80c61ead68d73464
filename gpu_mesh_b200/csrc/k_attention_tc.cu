// Decode / prefill GQA attention on the tensor cores (bf16, head_dim 64 or 128).
//
// With G query heads sharing one KV head, every key and value element feeds
// 2·G FLOPs; at G = 4 and 6.5 TB/s that is more fp32 FMA work than the CUDA
// cores sustain next to the loads, so the dot products run on mma.sync
// (m16n8k16, bf16 in, fp32 out) with the G heads padded to the MMA's 16 rows.
//
// One CTA = one query token x one KV head x a 128-key chunk; each of its 4
// warps owns 32 keys.  A warp's lane 0 loads its keys and values with 2-D TMA
// (box 32 keys x 64 dims, 128-byte swizzle, no multicast) through the slot's
// tensor map, so ldmatrix reads are bank-conflict free; keys arrive on one
// mbarrier and values on another, so scoring overlaps the value load.
//   S = Q·Kᵀ   A = Q (heads x dims, registers), B = K rows via ldmatrix
//   P = exp(S·scale - max)   per head row, quad shuffles
//   O = P·V    A = P (bf16 hi + lo, from S's accumulators), B = V via ldmatrix.trans
// The four warps' (max, sum, O) are merged in shared memory into the chunk's
// partial, which the combine kernel (k_attention.cu) merges across chunks.
// Every wait is bounded (code 3 in the error word on expiry).
#include <math.h>

#include "kernels.h"
#include "tc_common.cuh"

namespace mg {
namespace {

using namespace tc;

constexpr int kWarps = 4;
constexpr int kKeysW = kKvBoxKeys;            // keys per warp (32)
constexpr int kChunk = kWarps * kKeysW;        // keys per CTA (128)
constexpr int kBox = kKeysW * 128;             // bytes of one 32 x 64 box

__device__ __forceinline__ int visible(const AttnArgs& a, const RowDesc& rd, int m, int s) {
  const int total = rd.past + a.S;
  if (a.mask == kMaskSdpa && a.S == 1) return total;
  if (a.mask == kMaskCacheCausal) return min(rd.past + s + 1, total);
  int64_t pos = a.positions ? a.positions[m] : (int64_t)(rd.past + s);
  if (pos < 0) pos = 0;
  return (int)(pos + 1 < (int64_t)total ? pos + 1 : (int64_t)total);
}

__device__ __forceinline__ void tma_load_2d_gmap(void* dst, uint64_t tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  // rows 8-15 of A (heads >= 8) are zero: a1 = a3 = 0
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const uint32_t a = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return a | (b << 16);
}

// The two bf16 halves of a packed pair, widened.
__device__ __forceinline__ float lo_bf16(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Byte offset of (key row r, 16-byte chunk c of 64 dims) inside a swizzled box.
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

template <int D>
struct TcAttnLayout {
  static constexpr int kDB = D / 64;                      // 64-dim boxes per key row
  static constexpr int kWarpKV = 2 * kDB * kBox;           // K and V bytes of one warp
  static constexpr int kTiles = kWarps * kWarpKV;
  static constexpr int kMerge = kWarps * 8 * (D + 2) * 4;  // per-warp m, l, O of <= 8 heads
  static constexpr int kBytes = kTiles + kMerge + 1024 + 256;
};

template <int D>
__global__ void __launch_bounds__(kWarps * 32) attn_tc_kernel(AttnArgs a) {
  using L = TcAttnLayout<D>;
  constexpr int DB = L::kDB;
  constexpr int KS = D / 16;  // k-steps of the score MMA
  constexpr int DN = D / 8;   // dim n-tiles of the output
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* merge = (float*)(smem + L::kTiles);
  uint64_t* bars = (uint64_t*)(smem + L::kTiles + L::kMerge);  // [warp][K, V]

  pdl_trigger();
  pdl_wait();

  const int m = blockIdx.x, h = blockIdx.y, sp = blockIdx.z;
  const int G = a.nq / a.nkv;
  const int bidx = m / a.S, s = m % a.S;
  const RowDesc rd = a.rows[bidx];
  const int nvis = visible(a, rd, m, s);
  const int k0 = sp * kChunk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  float* part = a.partial + ((size_t)(m * a.nkv + h) * gridDim.z + sp) * (size_t)G * (D + 2);
  if (k0 >= nvis) {
    for (int i = tid; i < G; i += blockDim.x) {
      part[i * (D + 2)] = -INFINITY;
      part[i * (D + 2) + 1] = 0.f;
    }
    return;
  }

  const int kw0 = k0 + warp * kKeysW;                   // this warp's first key
  const int nk = max(0, min(kKeysW, nvis - kw0));        // its visible keys
  uint8_t* Kw = smem + warp * L::kWarpKV;
  uint8_t* Vw = Kw + DB * kBox;
  uint64_t* kbar = bars + 2 * warp;
  uint64_t* vbar = kbar + 1;
  if (lane == 0 && nk > 0) {
    mbar_init(kbar, 1);
    mbar_init(vbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const int yk = (int)kv_row(a.layer, 0, rd.slot_rows, rd.row, a.nkv, h, rd.cap, kw0);
    const int yv = (int)kv_row(a.layer, 1, rd.slot_rows, rd.row, a.nkv, h, rd.cap, kw0);
    mbar_expect_tx(kbar, DB * kBox);
    for (int db = 0; db < DB; ++db) tma_load_2d_gmap(Kw + db * kBox, rd.kv_tmap, kbar, db * 64, yk);
    mbar_expect_tx(vbar, DB * kBox);
    for (int db = 0; db < DB; ++db) tma_load_2d_gmap(Vw + db * kBox, rd.kv_tmap, vbar, db * 64, yv);
  }
  __syncwarp();

  // Q fragments (rows = heads g < G, the rest zero), straight from global.
  uint32_t qa[KS][2];
  {
    const __nv_bfloat16* q = (const __nv_bfloat16*)a.q + ((size_t)m * a.nq + (size_t)h * G + g) * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      if (g < G) {
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(q + 16 * ks + 2 * t);
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(q + 16 * ks + 8 + 2 * t);
      } else {
        qa[ks][0] = qa[ks][1] = 0u;
      }
    }
  }

  float mrow = -INFINITY, lrow = 0.f;
  float o[DN][4];
#pragma unroll
  for (int i = 0; i < DN; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  if (nk > 0) {
    const bool ok_k = mbar_wait(kbar, 0, a.err);
    // Scores for 32 keys = 4 n-tiles of 8.
    float sc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
    const uint32_t kbase = smem_u32(Kw);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int ks = 0; ks < KS; ks += 2) {
        // four 8x8 matrices: keys 8nt..8nt+7, dim chunks 2ks .. 2ks+3
        const int r = 8 * nt + (lane & 7);
        const int c = 2 * ks + (lane >> 3);
        uint32_t bfr[4];
        ldsm_x4(kbase + (c >> 3) * kBox + swz(r, c & 7), bfr);
        mma16816(sc[nt], qa[ks][0], qa[ks][1], bfr[0], bfr[1]);
        mma16816(sc[nt], qa[ks + 1][0], qa[ks + 1][1], bfr[2], bfr[3]);
      }
    }
    // Softmax of head g over this warp's keys (columns 2t, 2t+1 of each n-tile).
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = 8 * nt + 2 * t + e;
        const float v = (key < nk && ok_k) ? sc[nt][e] * a.scale : -INFINITY;
        sc[nt][e] = v;
        mx = fmaxf(mx, v);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    float sum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float p = sc[nt][e] == -INFINITY ? 0.f : expf(sc[nt][e] - mx);
        sc[nt][e] = p;
        sum += p;
      }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    mrow = mx;
    lrow = sum;

    // O = P·V over 2 k-tiles of 16 keys.
    const bool ok_v = mbar_wait(vbar, 0, a.err);
    if (nk < kKeysW) {
      // Rows past the visible keys hold whatever the cache held (or the next
      // head's values): P is 0 there, but 0 * NaN is not, so clear them.
      const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
      for (int i = lane; i < (kKeysW - nk) * DB * 8; i += 32) {
        const int rr = nk + i / (DB * 8), rem = i % (DB * 8);
        *reinterpret_cast<uint4*>(Vw + (rem >> 3) * kBox + rr * 128 + (rem & 7) * 16) = zero;
      }
      __syncwarp();
    }
    const uint32_t vbase = smem_u32(Vw);
#pragma unroll
    for (int kt = 0; kt < 2; ++kt) {
      // P = hi + lo, both bf16: two MMAs keep P to ~2^-17 relative, so the
      // product matches an fp32 P·V instead of a bf16-rounded one.
      const uint32_t pa0 = pack2(sc[2 * kt][0], sc[2 * kt][1]);
      const uint32_t pa2 = pack2(sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
      const uint32_t pl0 = pack2(sc[2 * kt][0] - lo_bf16(pa0), sc[2 * kt][1] - hi_bf16(pa0));
      const uint32_t pl2 = pack2(sc[2 * kt + 1][0] - lo_bf16(pa2), sc[2 * kt + 1][1] - hi_bf16(pa2));
#pragma unroll
      for (int dn = 0; dn < DN; dn += 2) {
        // matrices: keys 16kt+0..7 / +8..15, dim chunks dn / dn+1
        const int mi = lane >> 3;
        const int r = 16 * kt + (lane & 7) + 8 * (mi & 1);
        const int c = dn + (mi >> 1);
        uint32_t bfr[4];
        ldsm_x4_t(vbase + (c >> 3) * kBox + swz(r, c & 7), bfr);
        if (ok_v) {
          mma16816(o[dn], pa0, pa2, bfr[0], bfr[1]);
          mma16816(o[dn], pl0, pl2, bfr[0], bfr[1]);
          mma16816(o[dn + 1], pa0, pa2, bfr[2], bfr[3]);
          mma16816(o[dn + 1], pl0, pl2, bfr[2], bfr[3]);
        }
      }
    }
  }

  // Merge the four warps: per head, max, rescaled sum and output.
  float* mw = merge + warp * 8 * (D + 2);
  if (g < G && t == 0) {
    mw[g * (D + 2)] = mrow;
    mw[g * (D + 2) + 1] = lrow;
  }
  if (g < G) {
#pragma unroll
    for (int dn = 0; dn < DN; ++dn) {
      mw[g * (D + 2) + 2 + 8 * dn + 2 * t] = o[dn][0];
      mw[g * (D + 2) + 2 + 8 * dn + 2 * t + 1] = o[dn][1];
    }
  }
  __syncthreads();
  for (int i = tid; i < G * (D + 1); i += blockDim.x) {
    const int hh = i / (D + 1), d = i % (D + 1);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, merge[w * 8 * (D + 2) + hh * (D + 2)]);
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mwv = merge[w * 8 * (D + 2) + hh * (D + 2)];
      if (mwv == -INFINITY) continue;
      const float f = expf(mwv - M);
      acc += f * merge[w * 8 * (D + 2) + hh * (D + 2) + (d == D ? 1 : 2 + d)];
    }
    if (d == D) {
      part[hh * (D + 2)] = M;
      part[hh * (D + 2) + 1] = acc;
    } else {
      part[hh * (D + 2) + 2 + d] = acc;
    }
  }
}

}  // namespace

bool attention_tc_applicable(int dtype, int D, int G) {
  return dtype == kBF16 && (D == 64 || D == 128) && G <= 8;
}

size_t attention_tc_chunk() { return kChunk; }

cudaError_t launch_attention_tc(const AttnArgs& a, dim3 grid, cudaStream_t s) {
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
    return launch_pdl(kernel, grid, dim3(kWarps * 32), smem, s, a);
  };
  if (a.D == 128) return go(attn_tc_kernel<128>, TcAttnLayout<128>::kBytes);
  return go(attn_tc_kernel<64>, TcAttnLayout<64>::kBytes);
}

}  // namespace mg
