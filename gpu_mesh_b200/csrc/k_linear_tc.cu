// Prefill GEMM on the 5th-generation tensor cores: Y = epilogue(X · Wᵀ).
//
// X [M, K] and W [N, K] are both K-major (nn.Linear layout).  Two persistent
// kernels share the roles and the epilogues:
//   * gemm_pair_kernel (the default): clusters of two CTAs on neighbouring
//     SMs run the 2-SM MMA (tcgen05.mma.cta_group::2, M = 256) over 256 x 256
//     tiles; each CTA loads its half of X's rows and of W's rows, so an SM
//     moves 32 KB per 64-deep K block instead of 48 KB (description below);
//   * gemm_tc_kernel: the same on one SM (M = 128 x N = BN tiles), for a
//     device that cannot co-schedule a CTA pair.
// One CTA per SM (pair) walks the output tiles t = c, c + G, ... in the
// L2-aware order of TileGrid, and the roles overlap one tile's epilogue with
// the next tile's main loop:
//   * warp 0, one lane: TMA producer — cp.async.bulk.tensor 2-D loads of the
//     X and W tiles of each K block (128 x 64 boxes, 128-byte swizzle) into
//     an mbarrier-guarded ring (no multicast);
//   * warp 1, one lane: MMA issuer — four tcgen05.mma (K = 16) per K block
//     into one of two TMEM accumulators (2 x 256 = 512 columns), alternating
//     per tile; tcgen05.commit releases each smem stage and hands a finished
//     accumulator to the epilogue;
//   * warps 2-9: epilogue — warp w drains TMEM lanes 32·(w % 4) .. +31 (tile
//     rows) for one half of the output columns: tcgen05.ld, rounding with
//     the reference's rounding points, residual add or SwiGLU, 16-byte
//     global stores; then it returns the accumulator to the MMA issuer.
// For SwiGLU the 256 W rows of a tile are 128 gate rows followed by the
// matching 128 up rows, so each thread holds gate and up of the same output
// column.  Every mbarrier wait is bounded (about two seconds of
// %globaltimer); on expiry the kernel records kErrTimeout in the stage's
// error word, stops issuing, lets its issued loads and MMAs finish, frees
// its TMEM and returns.
#include <algorithm>
#include <cstdlib>

#include "linear_tc.h"
#include "tc_common.cuh"

namespace mg {
namespace {

using namespace tc;
using tc_host::make_map;
using tc_host::encoder;

using bf16 = __nv_bfloat16;

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = 128 bytes: one swizzle atom row
constexpr int kStages = 4;
#ifndef MG_GEMM_EPI_WARPS
#define MG_GEMM_EPI_WARPS 8
#endif
#ifndef MG_GEMM_ORDER
#define MG_GEMM_ORDER 0  // 0: by operand size, 1: M tiles fastest, 2: N tiles fastest
#endif
#ifndef MG_GEMM_BAND_MB
#define MG_GEMM_BAND_MB 32  // bytes of the reused operand per band of tiles (0: one band)
#endif
constexpr int kEpiWarps = MG_GEMM_EPI_WARPS;
// The qkv projection with RoPE, QK-norm and the KV append in its epilogue
// (prefill, head_dim 128; CTA-pair kernel only).  Local to this file.
constexpr int kEpiRopeKv = 5;
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN>
struct TcSmem {
  static constexpr int kA = kBM * kBK * 2;     // bytes per A stage
  static constexpr int kB = BN * kBK * 2;      // bytes per B stage
  static constexpr int kTiles = kStages * (kA + kB);
  static constexpr int kBytes = kTiles + 1024 /*align*/ + 256 /*barriers*/;
};

// Tile order: the operand that stays in L2 while the other streams is the
// smaller one, so M tiles run fastest (consecutive CTAs share a W tile) when
// X is the smaller, N tiles fastest otherwise.  The fast dimension is walked
// in bands of `band` tiles (every N column of a band of M tiles, then the
// next band), so the band of the smaller operand that the running tiles
// reuse stays within L2 while the larger operand streams past it.
struct TileGrid {
  int mt, nt;  // tiles along M and N
  int m_fast;
  int band;    // tiles of the fast dimension per band (>= 1)
  __device__ int count() const { return mt * nt; }
  __device__ void mn(int t, int& m, int& n) const {
    const int fast = m_fast ? mt : nt, slow = m_fast ? nt : mt;
    const int per = band * slow;
    const int b = t / per, local = t - b * per;
    const int width = min(band, fast - b * band);
    const int f = b * band + local % width, w = local / width;
    m = m_fast ? f : w;
    n = m_fast ? w : f;
  }
  __device__ int m(int t) const { int mm, nn; mn(t, mm, nn); return mm; }
  __device__ int n(int t) const { int mm, nn; mn(t, mm, nn); return nn; }
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   LinearArgs a, TileGrid tg, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  using L = TcSmem<BN>;
  uint8_t* sa = smem;
  uint8_t* sb = smem + kStages * L::kA;
  uint64_t* full = (uint64_t*)(smem + L::kTiles);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;  // [2] accumulator ready for the epilogue
  uint64_t* tempty = tfull + 2;       // [2] accumulator drained
  uint64_t* drain = tempty + 2;       // every MMA finished
  uint32_t* tmem_holder = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (a.K + kBK - 1) / kBK;
  const int ntile = tg.count();
  constexpr int NOUT = (EPI == kEpiSwiGLU) ? BN / 2 : BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;

  // Barrier and TMEM set-up above overlap the previous kernel's tail.
  pdl_trigger();
  long long issued = 0;
  if (warp == 0) {
    if (lane == 0) {
      // TMA producer over this CTA's tiles and their K blocks.  W does not
      // depend on the kernel before this one: the first ring's W tiles are
      // requested before waiting for it, X only after.
      auto load_w = [&](int t, int kb, int s) {
        const int n0 = tg.n(t) * NOUT;
        mbar_expect_tx(&full[s], L::kA + L::kB);
#pragma unroll
        for (int j = 0; j < BN / 128; ++j) {
          const int row = (EPI == kEpiSwiGLU) ? (j == 0 ? n0 : a.N + n0) : n0 + 128 * j;
          tma_load_2d(sb + s * L::kB + j * 128 * kBK * 2, &tm_w, &full[s], kb * kBK, row);
        }
      };
      auto load_x = [&](int t, int kb, int s) {
        tma_load_2d(sa + s * L::kA, &tm_x, &full[s], kb * kBK, tg.m(t) * kBM);
      };
      long long i = 0;
      const int first = blockIdx.x;
      const int pre = first < ntile ? min(kStages, nk) : 0;
      for (int kb = 0; kb < pre; ++kb) load_w(first, kb, kb);
      pdl_wait();
      for (int kb = 0; kb < pre; ++kb) load_x(first, kb, kb);
      i = pre;
      issued = pre;
      for (int t = first; t < ntile && !*abort_flag; t += gridDim.x) {
        for (int kb = (t == first ? pre : 0); kb < nk; ++kb, ++i) {
          const int s = (int)(i % kStages);
          const int round = (int)(i / kStages);
          if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, err)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          load_w(t, kb, s);
          load_x(t, kb, s);
          issued = i + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer: tile j of this CTA accumulates into TMEM half j & 1.
      constexpr uint32_t idesc = instr_desc(BN);
      long long i = 0;
      int j = 0;
      for (int t = blockIdx.x; t < ntile && !*abort_flag; t += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&tempty[b], ((j >> 1) - 1) & 1, err)) {
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + b * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++i) {
          const int s = (int)(i % kStages);
          if (!mbar_wait(&full[s], (int)(i / kStages) & 1, err)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t da = smem_desc(sa + s * L::kA);
          const uint64_t db = smem_desc(sb + s * L::kB);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_bf16(d, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&tfull[b]);
      }
      mma_commit(drain);
    }
  } else {
    // Epilogue warps 2-9: warp w reads TMEM lanes 32·(w % 4) .. +31 (tile
    // rows) and the output columns of half (w - 2) / 4 of the tile.
    pdl_wait();  // R and Y belong to the kernels around this one
    const int q = warp & 3;
    constexpr int kParts = kEpiWarps / 4;  // column parts per TMEM lane quadrant
    const int half = (warp - 2) >> 2;
    const uint32_t lanes = (uint32_t)(q * 32) << 16;
    int j = 0;
    for (int t = blockIdx.x; t < ntile; t += gridDim.x, ++j) {
      const int b = j & 1;
      if (!mbar_wait(&tfull[b], (j >> 1) & 1, err)) {
        *abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int row = tg.m(t) * kBM + q * 32 + lane;
      const int n0 = tg.n(t) * NOUT;
      const uint32_t trow = tmem + lanes + b * BN;
#pragma unroll 1
      for (int c = half * (NOUT / kParts); c < (half + 1) * (NOUT / kParts); c += 32) {
        float v[32], u[32];
        __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the stores
        tmem_ld32(trow + c, v);
        if (EPI == kEpiSwiGLU) tmem_ld32(trow + BN / 2 + c, u);
        const int n = n0 + c;
        if (row >= a.M || n >= a.N) continue;
        bf16* y = (bf16*)a.Y + (size_t)row * a.ldy + n;
        const int cols = min(32, a.N - n);  // multiple of 16 by the applicability check
        if (EPI == kEpiResid) {
          const bf16* r = (const bf16*)a.R + (size_t)row * a.ldr + n;
          for (int i = 0; i < cols; i += 8) {
            float rv[8];
            load16_f<bf16>(r + i, rv);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[i + e] = rv[e] + rt<bf16>(v[i + e]);
          }
        } else if (EPI == kEpiSwiGLU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float g = rt<bf16>(v[i]), up = rt<bf16>(u[i]);
            v[i] = rt<bf16>(g / (1.0f + expf(-g))) * up;
          }
        }
        for (int i = 0; i < cols; i += 8) {
          uint4 o;
          o.x = pack_bf16(v[i + 0], v[i + 1]);
          o.y = pack_bf16(v[i + 2], v[i + 3]);
          o.z = pack_bf16(v[i + 4], v[i + 5]);
          o.w = pack_bf16(v[i + 6], v[i + 7]);
          *reinterpret_cast<uint4*>(y + i) = o;
        }
      }
      // The accumulator is in registers and stored: hand it back.
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&tempty[b])) : "memory");
      if (*abort_flag) break;
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // Let the loads this CTA issued land before its shared memory goes away.
    for (long long i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
      mbar_wait(&full[i % kStages], (int)(i / kStages) & 1, err);
  }
  if (warp == 1 && lane == 0) mbar_wait(drain, 0, err);  // every MMA has finished
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
  }
}

// Epilogue of the qkv projection for one token row and one head of 128
// columns (this warp's half of a 256-column tile): the accumulator rounded to
// bf16 as the store epilogue would, then, as the RoPE / KV-append kernel does,
// QK-norm (q / k heads, if the model has it), rotary embedding with the
// rotate-half partner 64 columns away, and the store to the query buffer or
// the slot's KV cache.  `trow` addresses this lane's TMEM row at the head's
// first column; every lane runs the warp-collective TMEM loads.
__device__ __forceinline__ void rope_kv_epilogue(const LinearArgs& a, const QkvPostArgs& qp, int row, int n,
                                                 uint32_t trow) {
  const int nh = qp.nq + 2 * qp.nkv;
  const int hh = n / 128;
  if (n >= a.N || hh >= nh) return;  // uniform over the warp
  const bool live = row < a.M;
  int cache_pos = 0;
  int64_t pos = 0;
  RowDesc rd{};
  if (live) {
    const int b = row / qp.S, s = row % qp.S;
    rd = qp.rows[b];
    cache_pos = rd.past + s;
    pos = qp.positions ? qp.positions[row] : (int64_t)cache_pos;
    if (pos < 0 || pos >= qp.max_pos) {
      flag_error(qp.err, kErrPositionRange);
      pos = pos < 0 ? 0 : qp.max_pos - 1;
    }
  }
  const bool is_q = hh < qp.nq;
  const bool is_k = !is_q && hh < qp.nq + qp.nkv;
  bf16* kv = (bf16*)rd.kv_base;
  bf16* dst = nullptr;
  if (live) {
    if (is_q)
      dst = (bf16*)qp.q_out + ((size_t)row * qp.nq + hh) * 128;
    else if (is_k)
      dst = kv + kv_offset_elems(qp.layer, 0, rd.slot_rows, rd.row, qp.nkv, hh - qp.nq, rd.cap, 128, cache_pos);
    else
      dst = kv + kv_offset_elems(qp.layer, 1, rd.slot_rows, rd.row, qp.nkv, hh - qp.nq - qp.nkv, rd.cap, 128,
                                 cache_pos);
  }
  float v[32], u[32];
  if (!is_q && !is_k) {  // value head: the rounded accumulator, appended as is
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      __syncwarp();
      tmem_ld32(trow + c, v);
      if (!live) continue;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 o;
        o.x = pack_bf16(v[i + 0], v[i + 1]);
        o.y = pack_bf16(v[i + 2], v[i + 3]);
        o.z = pack_bf16(v[i + 4], v[i + 5]);
        o.w = pack_bf16(v[i + 6], v[i + 7]);
        *reinterpret_cast<uint4*>(dst + c + i) = o;
      }
    }
    return;
  }
  const bf16* nw = (const bf16*)(is_q ? qp.q_norm : qp.k_norm);
  float r = 1.f;
  if (nw) {
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      __syncwarp();
      tmem_ld32(trow + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float x = rt<bf16>(v[i]);
        ss += x * x;
      }
    }
    r = 1.0f / sqrtf(ss / 128.0f + qp.eps);
  }
  const bf16* cs = (const bf16*)qp.cos + (size_t)pos * 64;
  const bf16* sn = (const bf16*)qp.sin + (size_t)pos * 64;
#pragma unroll 1
  for (int c = 0; c < 64; c += 32) {
    __syncwarp();
    tmem_ld32(trow + c, v);       // dims c .. c + 31
    tmem_ld32(trow + c + 64, u);  // their rotate-half partners
    if (!live) continue;
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      float cv[8], sv[8], gl[8], gh[8];
      load16_f<bf16>(cs + c + i, cv);
      load16_f<bf16>(sn + c + i, sv);
      if (nw) {
        load16_f<bf16>(nw + c + i, gl);
        load16_f<bf16>(nw + c + 64 + i, gh);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float xl = rt<bf16>(v[i + e]), xh = rt<bf16>(u[i + e]);
        if (nw) {
          xl = rt<bf16>(rt<bf16>(xl * r) * gl[e]);
          xh = rt<bf16>(rt<bf16>(xh * r) * gh[e]);
        }
        v[i + e] = rt<bf16>(xl * cv[e]) + rt<bf16>(-xh * sv[e]);
        u[i + e] = rt<bf16>(xh * cv[e]) + rt<bf16>(xl * sv[e]);
      }
    }
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      uint4 o, p;
      o.x = pack_bf16(v[i + 0], v[i + 1]);
      o.y = pack_bf16(v[i + 2], v[i + 3]);
      o.z = pack_bf16(v[i + 4], v[i + 5]);
      o.w = pack_bf16(v[i + 6], v[i + 7]);
      p.x = pack_bf16(u[i + 0], u[i + 1]);
      p.y = pack_bf16(u[i + 2], u[i + 3]);
      p.z = pack_bf16(u[i + 4], u[i + 5]);
      p.w = pack_bf16(u[i + 6], u[i + 7]);
      *reinterpret_cast<uint4*>(dst + c + i) = o;
      *reinterpret_cast<uint4*>(dst + c + 64 + i) = p;
    }
  }
}

// CTA pairs (clusters of two SMs) on the 2-SM MMA: a tile is 256 rows of X
// x 256 rows of W (SwiGLU: 128 gate + 128 up rows -> 128 outputs).  CTA r of
// the pair loads X rows 128r .. 128r + 127 of the tile and W rows
// 128r .. 128r + 127 (SwiGLU: the gate rows in CTA 0, the up rows in CTA 1)
// of each 128-deep K block (two 64-column boxes per operand) into a 3-stage
// ring, 64 KB per stage; both CTAs' loads complete on the even CTA's
// barrier, whose MMA warp issues eight M = 256 MMAs per stage that read both
// CTAs' shared memory and leave each CTA's 128 rows x 256 columns in its own
// TMEM (two accumulators, 512 columns).  Per SM that is 32 KB of operands
// per 64 of K instead of the single-CTA tile's 48 KB for the same MMA work;
// 128-deep stages halve the barrier waits and commits per MMA (measured:
// 0.93-0.97 x cuBLAS against 0.81 with 64-deep stages in a 6-stage ring).  Completions (stage free, accumulator ready, all done) are multicast
// to both CTAs; each CTA's epilogue drains its own TMEM and arrives on the
// even CTA's accumulator-free barrier.  No load is multicast.  Every wait is
// bounded; both CTAs reach the final cluster barrier on every path.
#ifndef MG_GEMM_PAIR_STAGES
#define MG_GEMM_PAIR_STAGES 3
#endif
constexpr int kStagesP = MG_GEMM_PAIR_STAGES;
#ifndef MG_GEMM_PAIR_SUB
#define MG_GEMM_PAIR_SUB 2
#endif
constexpr int kSubP = MG_GEMM_PAIR_SUB;  // 64-wide K boxes per stage and operand
constexpr int kBKP = kSubP * kBK;         // K depth of a stage
struct PairSmem {
  static constexpr int kSub = 128 * kBK * 2;  // one 128 x 64 box
  static constexpr int kA = kSubP * kSub;
  static constexpr int kB = kSubP * kSub;
  static constexpr int kTiles = kStagesP * (kA + kB);
  static constexpr int kBytes = kTiles + 1024 /*align*/ + 256 /*barriers*/;
};

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     LinearArgs a, TileGrid tg, int* err, const __grid_constant__ QkvPostArgs qp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  using L = PairSmem;
  uint8_t* sa = smem;
  uint8_t* sb = smem + kStagesP * L::kA;
  uint64_t* full = (uint64_t*)(smem + L::kTiles);  // used in the even CTA
  uint64_t* empty = full + kStagesP;
  uint64_t* tfull = empty + kStagesP;  // [2]
  uint64_t* tempty = tfull + 2;        // [2] (even CTA: both CTAs' epilogue warps arrive)
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_holder + 1);

  constexpr int BN = 256;
  constexpr int NOUT = (EPI == kEpiSwiGLU) ? BN / 2 : BN;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nk = (a.K + kBKP - 1) / kBKP;
  const int ntile = tg.count();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesP; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any load, commit or arrival reaches them
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  const uint32_t full_lead = mapa_shared(smem_u32(full), 0);
  const uint32_t tempty_lead = mapa_shared(smem_u32(tempty), 0);

  pdl_trigger();
  long long issued = 0;
  if (warp == 0) {
    if (lane == 0) {
      // TMA producer (both CTAs): this CTA's halves of each tile's K blocks.
      auto load_w = [&](int t, int kb, int s) {
        const int n0 = tg.n(t) * NOUT;
        if (rank == 0) mbar_expect_tx(&full[s], 2 * (L::kA + L::kB));
        const int row = (EPI == kEpiSwiGLU) ? (rank == 0 ? n0 : a.N + n0) : n0 + 128 * (int)rank;
#pragma unroll
        for (int q = 0; q < kSubP; ++q)
          tma_load_2d_pair(sb + s * L::kB + q * L::kSub, &tm_w, full_lead + 8 * s, kb * kBKP + q * kBK, row);
      };
      auto load_x = [&](int t, int kb, int s) {
#pragma unroll
        for (int q = 0; q < kSubP; ++q)
          tma_load_2d_pair(sa + s * L::kA + q * L::kSub, &tm_x, full_lead + 8 * s, kb * kBKP + q * kBK,
                           tg.m(t) * 256 + 128 * (int)rank);
      };
      long long i = 0;
      const int first = pair;
      const int pre = first < ntile ? min(kStagesP, nk) : 0;
      for (int kb = 0; kb < pre; ++kb) load_w(first, kb, kb);
      pdl_wait();
      for (int kb = 0; kb < pre; ++kb) load_x(first, kb, kb);
      i = pre;
      issued = pre;
      for (int t = first; t < ntile && !*abort_flag; t += npairs) {
        for (int kb = (t == first ? pre : 0); kb < nk; ++kb, ++i) {
          const int s = (int)(i % kStagesP);
          const int round = (int)(i / kStagesP);
          if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, err)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          load_w(t, kb, s);
          load_x(t, kb, s);
          issued = i + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // MMA issuer (even CTA): tile j of the pair accumulates into TMEM half j & 1.
      constexpr uint32_t idesc = instr_desc_mn(256, BN);
      long long i = 0;
      int j = 0;
      for (int t = pair; t < ntile && !*abort_flag; t += npairs, ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait_cluster(&tempty[b], ((j >> 1) - 1) & 1, err)) {
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + b * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++i) {
          const int s = (int)(i % kStagesP);
          if (!mbar_wait(&full[s], (int)(i / kStagesP) & 1, err)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
          for (int q = 0; q < kSubP; ++q) {
            const uint64_t da = smem_desc(sa + s * L::kA + q * L::kSub);
            const uint64_t db = smem_desc(sb + s * L::kB + q * L::kSub);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              mma_bf16_pair(d, da + 2 * k, db + 2 * k, idesc, (kb > 0 || q > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit_pair(&empty[s]);
        }
        if (!ok) break;
        mma_commit_pair(&tfull[b]);
      }
      mma_commit_pair(drain);
    }
  } else {
    // Epilogue warps 2-9 (both CTAs): warp w reads TMEM lanes 32·(w % 4) ..
    // +31 (this CTA's tile rows) and the output columns of half (w - 2) / 4.
    pdl_wait();  // R and Y belong to the kernels around this one
    const int q = warp & 3;
    constexpr int kParts = kEpiWarps / 4;
    const int half = (warp - 2) >> 2;
    const uint32_t lanes = (uint32_t)(q * 32) << 16;
    int j = 0;
    for (int t = pair; t < ntile; t += npairs, ++j) {
      const int b = j & 1;
      if (!mbar_wait(&tfull[b], (j >> 1) & 1, err)) {
        *abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int row = tg.m(t) * 256 + 128 * (int)rank + q * 32 + lane;
      const int n0 = tg.n(t) * NOUT;
      const uint32_t trow = tmem + lanes + b * BN;
      if constexpr (EPI == kEpiRopeKv) {
        rope_kv_epilogue(a, qp, row, n0 + half * 128, trow + half * 128);
      } else {
#pragma unroll 1
      for (int c = half * (NOUT / kParts); c < (half + 1) * (NOUT / kParts); c += 32) {
        float v[32], u[32];
        __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the stores
        tmem_ld32(trow + c, v);
        if (EPI == kEpiSwiGLU) tmem_ld32(trow + BN / 2 + c, u);
        const int n = n0 + c;
        if (row >= a.M || n >= a.N) continue;
        bf16* y = (bf16*)a.Y + (size_t)row * a.ldy + n;
        const int cols = min(32, a.N - n);  // multiple of 16 by the applicability check
        if (EPI == kEpiResid) {
          const bf16* r = (const bf16*)a.R + (size_t)row * a.ldr + n;
          for (int i = 0; i < cols; i += 8) {
            float rv[8];
            load16_f<bf16>(r + i, rv);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[i + e] = rv[e] + rt<bf16>(v[i + e]);
          }
        } else if (EPI == kEpiSwiGLU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float g = rt<bf16>(v[i]), up = rt<bf16>(u[i]);
            v[i] = rt<bf16>(g / (1.0f + expf(-g))) * up;
          }
        }
        for (int i = 0; i < cols; i += 8) {
          uint4 o;
          o.x = pack_bf16(v[i + 0], v[i + 1]);
          o.y = pack_bf16(v[i + 2], v[i + 3]);
          o.z = pack_bf16(v[i + 4], v[i + 5]);
          o.w = pack_bf16(v[i + 6], v[i + 7]);
          *reinterpret_cast<uint4*>(y + i) = o;
        }
      }
      }
      // This CTA's rows of the accumulator are stored: hand it back to the MMA warp.
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_lead + 8 * b);
      if (*abort_flag) break;
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && rank == 0 && *abort_flag) {
    // Let the loads of both CTAs that completed on this CTA's barriers land.
    for (long long i = issued > kStagesP ? issued - kStagesP : 0; i < issued; ++i)
      mbar_wait(&full[i % kStagesP], (int)(i / kStagesP) & 1, err);
  }
  if (warp == 1 && lane == 0) mbar_wait(drain, 0, err);  // every MMA of the pair has finished
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair's MMAs or arrivals may still reach it
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
  }
}

template <int BN, int EPI>
cudaError_t launch_tc(const LinearArgs& a, cudaStream_t s) {
  CUtensorMap tx, tw;
  const uint64_t wrows = (EPI == kEpiSwiGLU) ? 2ull * a.N : (uint64_t)a.N;
  if (!make_map(&tx, a.X, a.M, a.K, a.ldx) || !make_map(&tw, a.W, wrows, a.K, a.K))
    return cudaErrorInvalidValue;
  constexpr int smem = TcSmem<BN>::kBytes;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int nout = (EPI == kEpiSwiGLU) ? BN / 2 : BN;
  TileGrid tg;
  tg.mt = (a.M + kBM - 1) / kBM;
  tg.nt = (a.N + nout - 1) / nout;
  tg.m_fast = MG_GEMM_ORDER == 1 || (MG_GEMM_ORDER == 0 && (uint64_t)a.M <= wrows);  // X no larger than W
  {
    const int fast = tg.m_fast ? tg.mt : tg.nt;
    const uint64_t tile_bytes = (uint64_t)(tg.m_fast ? kBM : BN) * a.K * 2;  // one tile row of the reused operand
    const uint64_t band = MG_GEMM_BAND_MB ? ((uint64_t)MG_GEMM_BAND_MB << 20) / tile_bytes : (uint64_t)fast;
    tg.band = (int)std::max<uint64_t>(1, std::min<uint64_t>(band, (uint64_t)fast));
  }
  static int sms[64] = {};
  if (!sms[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = v > 0 ? v : 148;
  }
  const long long tiles = (long long)tg.mt * tg.nt;
  if (tiles > (1ll << 30)) return cudaErrorInvalidValue;
  const int grid = (int)std::min<long long>(tiles, sms[dev]);
  { const cudaError_t _le = launch_pdl(gemm_tc_kernel<BN, EPI>, dim3(grid), dim3(kThreads), smem, s, tx, tw, a, tg, a.err); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

template <int EPI>
cudaError_t launch_pair(const LinearArgs& a, cudaStream_t s, const QkvPostArgs* qp = nullptr) {
  CUtensorMap tx, tw;
  const uint64_t wrows = (EPI == kEpiSwiGLU) ? 2ull * a.N : (uint64_t)a.N;
  if (!make_map(&tx, a.X, a.M, a.K, a.ldx) || !make_map(&tw, a.W, wrows, a.K, a.K)) return cudaErrorInvalidValue;
  constexpr int smem = PairSmem::kBytes;
  static bool configured[64] = {};
  static int max_pairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cfg.gridDim = dim3(sms > 1 ? sms & ~1 : 2);
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<EPI>, &cfg);
    if (e != cudaSuccess) return e;
    max_pairs[dev] = n;
    configured[dev] = true;
  }
  if (max_pairs[dev] < 1) return cudaErrorNotSupported;  // no CTA pair fits: the caller takes one SM per tile
  const int nout = (EPI == kEpiSwiGLU) ? 128 : 256;
  TileGrid tg;
  tg.mt = (a.M + 255) / 256;
  tg.nt = (a.N + nout - 1) / nout;
  tg.m_fast = MG_GEMM_ORDER == 1 || (MG_GEMM_ORDER == 0 && (uint64_t)a.M <= wrows);
  {
    const int fast = tg.m_fast ? tg.mt : tg.nt;
    const uint64_t tile_bytes = (uint64_t)256 * a.K * 2;  // one tile row of the reused operand
    const uint64_t band = MG_GEMM_BAND_MB ? ((uint64_t)MG_GEMM_BAND_MB << 20) / tile_bytes : (uint64_t)fast;
    tg.band = (int)std::max<uint64_t>(1, std::min<uint64_t>(band, (uint64_t)fast));
  }
  const long long tiles = (long long)tg.mt * tg.nt;
  if (tiles > (1ll << 30)) return cudaErrorInvalidValue;
  const int pairs = (int)std::min<long long>(tiles, max_pairs[dev]);
  cfg.gridDim = dim3(2 * pairs);
  cfg.numAttrs = 2;
  const QkvPostArgs none{};
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_pair_kernel<EPI>, tx, tw, a, tg, a.err, qp ? *qp : none);
  note_launch();
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

bool linear_tc_applicable(int dtype, int M, int N, int K) {
  return dtype == kBF16 && M > 32 && N % 16 == 0 && K % kBK == 0 && encoder() != nullptr;
}

size_t linear_tc_scratch_elems(int, int, int, int) { return 0; }

cudaError_t launch_linear_tc(const LinearArgs& a, cudaStream_t s) {
  if (((uintptr_t)a.X % 16) || ((uintptr_t)a.W % 16) || (a.ldx % 8)) return cudaErrorInvalidValue;
  // CTA pairs on the 2-SM MMA; the single-SM persistent kernel where the
  // device cannot co-schedule a pair (or MESHGPU_GEMM_SINGLE_SM=1 asks for it).
  const char* single = getenv("MESHGPU_GEMM_SINGLE_SM");
  if (!(single && single[0] == '1')) {
    cudaError_t e;
    switch (a.epilogue) {
      case kEpiStore: e = launch_pair<kEpiStore>(a, s); break;
      case kEpiResid: e = launch_pair<kEpiResid>(a, s); break;
      default: e = launch_pair<kEpiSwiGLU>(a, s); break;
    }
    if (e != cudaErrorNotSupported) return e;
  }
  switch (a.epilogue) {
    case kEpiStore: return launch_tc<256, kEpiStore>(a, s);
    case kEpiResid: return launch_tc<256, kEpiResid>(a, s);
    default: return launch_tc<256, kEpiSwiGLU>(a, s);
  }
}

bool qkv_rope_fusable(const LinearArgs& a, const QkvPostArgs& q) {
  return a.dtype == kBF16 && q.dtype == kBF16 && q.D == 128 && !q.use_pieces && a.epilogue == kEpiStore &&
         a.Y == q.qkv && a.N == (q.nq + 2 * q.nkv) * 128 && a.M == q.B * q.S &&
         linear_tc_applicable(a.dtype, a.M, a.N, a.K);
}

cudaError_t launch_qkv_rope_kv(const LinearArgs& a, const QkvPostArgs& q, cudaStream_t s) {
  if (!qkv_rope_fusable(a, q)) return cudaErrorInvalidValue;
  if (((uintptr_t)a.X % 16) || ((uintptr_t)a.W % 16) || (a.ldx % 8)) return cudaErrorInvalidValue;
  const char* single = getenv("MESHGPU_GEMM_SINGLE_SM");
  if (!(single && single[0] == '1')) {
    const cudaError_t e = launch_pair<kEpiRopeKv>(a, s, &q);
    if (e != cudaErrorNotSupported) return e;
  }
  // No CTA pair: the projection into the qkv buffer, then the RoPE / append kernel.
  const cudaError_t e = launch_linear_tc(a, s);
  if (e != cudaSuccess) return e;
  return launch_qkv_post(q, s);
}

}  // namespace mg
