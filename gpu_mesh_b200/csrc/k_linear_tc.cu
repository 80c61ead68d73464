// Prefill GEMM on the 5th-generation tensor cores: Y = epilogue(X · Wᵀ).
//
// X [M, K] and W [N, K] are both K-major (nn.Linear layout).  Two kernels
// share the tile geometry: gemm_tile_kernel (one output tile per CTA, below)
// for the light store / residual epilogues, and gemm_tc_kernel for SwiGLU,
// whose exp / divide epilogue would otherwise idle the tensor pipe.  The
// latter is persistent: one CTA per SM walks the 128 x BN output tiles t = c, c + G,
// ... (M tiles fastest, so CTAs running together share W tiles in L2), and
// its roles overlap one tile's epilogue with the next tile's main loop:
//   * warp 0, one lane: TMA producer — cp.async.bulk.tensor 2-D loads of a
//     128 x 64 X tile and BN/128 W tiles of 128 x 64 per K block, 128-byte
//     swizzle, into a kStages-deep ring guarded by mbarriers (no multicast);
//   * warp 1, one lane: MMA issuer — four tcgen05.mma (M=128, N=BN, K=16)
//     per K block into one of two TMEM accumulators (2 x BN = 512 columns),
//     alternating per tile; tcgen05.commit releases each smem stage and
//     hands a finished accumulator to the epilogue;
//   * warps 2-9: epilogue — warp w drains TMEM lanes 32·(w % 4) .. +31 (tile
//     rows) for one half of the output columns: tcgen05.ld, rounding with
//     the reference's rounding points, residual add or SwiGLU, 16-byte
//     global stores; then it returns the accumulator to the MMA issuer.
// For SwiGLU the BN = 256 tile is 128 gate rows followed by the matching 128
// up rows, so each thread holds gate and up of the same output column.
// Every mbarrier wait is bounded (about two seconds of %globaltimer); on
// expiry the kernel records kErrTimeout in the stage's error word, stops
// issuing, lets its issued loads and MMAs finish, frees its TMEM and returns.
#include <algorithm>

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
constexpr int kEpiWarps = MG_GEMM_EPI_WARPS;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kTileThreads = 128;

template <int BN>
struct TcSmem {
  static constexpr int kA = kBM * kBK * 2;     // bytes per A stage
  static constexpr int kB = BN * kBK * 2;      // bytes per B stage
  static constexpr int kTiles = kStages * (kA + kB);
  static constexpr int kBytes = kTiles + 1024 /*align*/ + 256 /*barriers*/;
};

// Tile order: the operand that stays in L2 while the other streams is the
// smaller one, so M tiles run fastest (consecutive CTAs share a W tile) when
// X is the smaller, N tiles fastest otherwise.
struct TileGrid {
  int mt, nt;  // tiles along M and N
  int m_fast;
  __device__ int count() const { return mt * nt; }
  __device__ int m(int t) const { return m_fast ? t % mt : t / nt; }
  __device__ int n(int t) const { return m_fast ? t / mt : t % nt; }
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

// One output tile per CTA (grid = N tiles x M tiles), 4 warps: warp 0 lane 0
// loads, warp 1 lane 0 issues the MMAs into one BN-column accumulator, then
// all four warps run the epilogue.  Used where the epilogue is light (store,
// residual): in measurements it keeps the tensor pipe fuller than the
// persistent kernel for those.
template <int BN, int EPI>
__global__ void __launch_bounds__(kTileThreads, 1)
    gemm_tile_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   LinearArgs a, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  using L = TcSmem<BN>;
  uint8_t* sa = smem;
  uint8_t* sb = smem + kStages * L::kA;
  uint64_t* full = (uint64_t*)(smem + L::kTiles);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint32_t* tmem_holder = (uint32_t*)(acc_full + 1);
  int* abort_flag = (int*)(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM;
  const int n0 = (EPI == kEpiSwiGLU) ? blockIdx.x * (BN / 2) : blockIdx.x * BN;
  const int nk = (a.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;

  // Barrier and TMEM set-up above overlap the previous kernel's tail.
  pdl_trigger();
  pdl_wait();
  int issued = 0;
  if (warp == 0 && lane == 0) {
    // TMA producer.
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kStages, round = kb / kStages;
      if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, err)) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      if (*(volatile int*)abort_flag) break;
      mbar_expect_tx(&full[s], L::kA + L::kB);
      tma_load_2d(sa + s * L::kA, &tm_x, &full[s], kb * kBK, m0);
#pragma unroll
      for (int j = 0; j < BN / 128; ++j) {
        const int row = (EPI == kEpiSwiGLU) ? (j == 0 ? n0 : a.N + n0) : n0 + 128 * j;
        tma_load_2d(sb + s * L::kB + j * 128 * kBK * 2, &tm_w, &full[s], kb * kBK, row);
      }
      issued = kb + 1;
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer.
    constexpr uint32_t idesc = instr_desc(BN);
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kStages, round = kb / kStages;
      if (!mbar_wait(&full[s], round & 1, err)) {
        *(volatile int*)abort_flag = 1;
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint64_t da = smem_desc(sa + s * L::kA);
      const uint64_t db = smem_desc(sb + s * L::kB);
#pragma unroll
      for (int j = 0; j < kBK / 16; ++j)
        mma_bf16(tmem, da + 2 * j, db + 2 * j, idesc, (kb > 0 || j > 0) ? 1u : 0u);
      mma_commit(&empty[s]);
    }
    (void)ok;
    // Arrives once every MMA issued above has finished (immediately if none).
    mma_commit(acc_full);
  }
  __syncwarp();

  // Epilogue: warp w owns TMEM lanes (tile rows) 32w .. 32w+31.
  const bool have = mbar_wait(acc_full, 0, err) && !*(volatile int*)abort_flag;
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const int row = m0 + warp * 32 + lane;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  constexpr int NOUT = (EPI == kEpiSwiGLU) ? BN / 2 : BN;
  if (have) {
#pragma unroll 1
    for (int c = 0; c < NOUT; c += 32) {
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
  if (warp == 0 && lane == 0 && *(volatile int*)abort_flag) {
    // After a timeout, let the loads this CTA issued land before it exits.
    for (int kb = issued > kStages ? issued - kStages : 0; kb < issued; ++kb)
      mbar_wait(&full[kb % kStages], (kb / kStages) & 1, err);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
  }
}


template <int BN, int EPI>
cudaError_t launch_tile(const LinearArgs& a, cudaStream_t s) {
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
    cudaError_t e = cudaFuncSetAttribute(gemm_tile_kernel<BN, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int ntile = (EPI == kEpiSwiGLU) ? BN / 2 : BN;
  dim3 grid((a.N + ntile - 1) / ntile, (a.M + kBM - 1) / kBM);
  { const cudaError_t _le = launch_pdl(gemm_tile_kernel<BN, EPI>, dim3(grid), dim3(kTileThreads), smem, s, tx, tw, a, a.err); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
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

}  // namespace

bool linear_tc_applicable(int dtype, int M, int N, int K) {
  return dtype == kBF16 && M > 32 && N % 16 == 0 && K % kBK == 0 && encoder() != nullptr;
}

size_t linear_tc_scratch_elems(int, int, int, int) { return 0; }

cudaError_t launch_linear_tc(const LinearArgs& a, cudaStream_t s) {
  if (((uintptr_t)a.X % 16) || ((uintptr_t)a.W % 16) || (a.ldx % 8)) return cudaErrorInvalidValue;
  switch (a.epilogue) {
    // light epilogues: one tile per CTA; SwiGLU: persistent, its epilogue
    // overlapped with the next tile's main loop
    case kEpiStore: return launch_tile<256, kEpiStore>(a, s);
    case kEpiResid: return launch_tile<256, kEpiResid>(a, s);
    default: return launch_tc<256, kEpiSwiGLU>(a, s);
  }
}

}  // namespace mg
