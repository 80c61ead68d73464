// Decode linear layers (<= 32 token rows) on tcgen05: a persistent, stream-K
// weight stream.
//
// At decode the layer is Y[M, N] = X[M, K] · W[N, K]ᵀ with M <= 32, so every
// byte of W is used once per step: the kernel is an HBM stream and its job
// is to keep enough W bytes in flight on every SM.  Swap-AB puts W on the
// MMA's M side (128 W rows per tile) and the M token rows (padded to NP = 16
// or 32 by the TMA's zero fill) on its N side.
//
// Work split: a tile is 128 W rows (64 gate + 64 up rows for SwiGLU), a unit
// is one tile x 64-wide K block (16 KB of W).  The tiles x K/64 units are cut
// into one contiguous range per CTA (grid = SM count), so every SM streams
// the same number of bytes whatever N and K are.  A CTA's range covers whole
// tiles and at most a partial tile at each end; a partial tile's fp32 sums
// go to a scratch slot, and the CTA that completes the tile's piece count
// (an atomic counter, reset to zero by that CTA) adds the pieces in CTA
// order, so results are deterministic.
//
// Roles (6 warps): warp 0 lane 0 issues TMA loads (W: two 64 x 64 boxes,
// X: NP x 64, 128-byte swizzle) into an 8-stage mbarrier ring; warp 1 lane 0
// issues tcgen05.mma (M=128, N=NP, K=16) into one of two TMEM accumulators;
// warps 2-5 drain the other accumulator with tcgen05.ld (warp w reads TMEM
// lanes 32*(w%4)..+31) and run the epilogue (store / residual / SwiGLU with
// the reference's rounding points; for lm_head optionally the greedy
// selection, see Greedy).  Launched with programmatic dependent
// launch, the producer requests its first weights before waiting for the
// previous kernel.  Every wait is bounded; on a timeout the
// kernel records code 3 in the error word, drains what it issued, frees its
// TMEM and returns.
#include "gemv_tc_parts.cuh"
#include "linear_tc.h"

namespace mg {
namespace {

using namespace tc;
using namespace gemvtc;

template <int NP, int EPI>
__global__ void __launch_bounds__(kThreadsD, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   LinearArgs a, Part p, int* counters, float* slots, int* err) {
  using L = DLayout<NP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* xchg = (float*)(smem + L::kTiles);
  uint64_t* full = (uint64_t*)(smem + L::kBarOff);
  uint64_t* empty = full + kStagesD;
  uint64_t* tfull = empty + kStagesD;    // [2]
  uint64_t* tempty = tfull + 2;          // [2]
  uint64_t* drain = tempty + 2;          // final MMA completion
  uint32_t* tmem_holder = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const long long u0 = p.begin(c), u1 = p.begin(c + 1);
  const int t_first = (int)(u0 / p.nk);
  const int t_last = u1 > u0 ? (int)((u1 - 1) / p.nk) : t_first - 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesD; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(2 * NP < 32 ? 32 : 2 * NP));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  long long issued = 0;

  pdl_trigger();
  if (warp == 0) {
    if (lane == 0) {
      // TMA producer over this CTA's units.  The weights do not depend on the
      // kernel before this one, so the first ring's worth of W is requested
      // before waiting for it; the activations X only after.
      auto load_w = [&](long long u, int s) {
        const int t = (int)(u / p.nk), kb = (int)(u % p.nk);
        const int r0 = (EPI == kEpiSwiGLU) ? t * 64 : t * kRows;
        const int r1 = (EPI == kEpiSwiGLU) ? a.N + t * 64 : t * kRows + 64;
        uint8_t* st = smem + s * L::kStage;
        mbar_expect_tx(&full[s], L::kStage);
        tma_load_2d(st, &tm_w, &full[s], kb * kKB, r0);
        tma_load_2d(st + kWBytes / 2, &tm_w, &full[s], kb * kKB, r1);
      };
      auto load_x = [&](long long u, int s) {
        tma_load_2d(smem + s * L::kStage + kWBytes, &tm_x, &full[s], (int)(u % p.nk) * kKB, 0);
      };
      const long long pre = min((long long)kStagesD, u1 - u0);
      for (long long i = 0; i < pre; ++i) load_w(u0 + i, (int)i);
      pdl_wait();
      for (long long i = 0; i < pre; ++i) load_x(u0 + i, (int)i);
      issued = pre;
      for (long long u = u0 + pre; u < u1; ++u) {
        const long long i = u - u0;
        const int s = (int)(i % kStagesD);
        const int round = (int)(i / kStagesD);
        if (!mbar_wait(&empty[s], (round - 1) & 1, err)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        load_w(u, s);
        load_x(u, s);
        issued = i + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer: one accumulator per tile piece, alternating TMEM halves.
      constexpr uint32_t idesc = instr_desc(NP);
      long long i = 0;
      int pi = 0;
      for (int t = t_first; t <= t_last && !*abort_flag; ++t, ++pi) {
        const long long lo = max(u0, (long long)t * p.nk), hi = min(u1, (long long)(t + 1) * p.nk);
        const int b = pi & 1;
        if (pi >= 2 && !mbar_wait(&tempty[b], ((pi >> 1) - 1) & 1, err)) {
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + b * NP;
        for (long long u = lo; u < hi; ++u, ++i) {
          const int s = (int)(i % kStagesD);
          if (!mbar_wait(&full[s], (int)(i / kStagesD) & 1, err)) {
            *abort_flag = 1;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint8_t* st = smem + s * L::kStage;
          const uint64_t da = smem_desc(st), db = smem_desc(st + kWBytes);
#pragma unroll
          for (int j = 0; j < kKB / 16; ++j)
            mma_bf16(d, da + 2 * j, db + 2 * j, idesc, (u > lo || j > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        mma_commit(&tfull[b]);
      }
      mma_commit(drain);
    }
  } else {
    // Epilogue warps 2-5: they read R and write Y, slots and counters.
    pdl_wait();
    const int q = warp & 3;
    const int r = q * 32 + lane;  // W row within the tile
    const int e = threadIdx.x - 64;
    int pi = 0;
    bool ok = true;
    for (int t = t_first; t <= t_last; ++t, ++pi) {
      const int b = pi & 1;
      ok = mbar_wait(&tfull[b], (pi >> 1) & 1, err);
      if (epi_bar_any(!ok)) {  // a timeout anywhere stops all four warps together
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float v[NP];
      __syncwarp();
      tmem_ld<NP>(tmem + ((uint32_t)(q * 32) << 16) + b * NP, v);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&tempty[b])) : "memory");

      if (EPI == kEpiPieces) {  // leave the sums for the consuming kernel
        float* S = slots + (size_t)(c + t) * NP * kRows + r;
#pragma unroll
        for (int tok = 0; tok < NP; ++tok)
          if (tok < a.M) S[tok * kRows] = v[tok];
        continue;
      }
      const long long lo = max(u0, (long long)t * p.nk), hi = min(u1, (long long)(t + 1) * p.nk);
      const bool whole = lo == (long long)t * p.nk && hi == (long long)(t + 1) * p.nk;
      if (!whole && !piece_done<NP>(p, slots, counters, c, t, r, e, v)) continue;  // another CTA finishes it
      apply<NP, EPI>(a, t, r, v, xchg);
      if (EPI == kEpiGreedy) greedy_fold<NP>(a, t, r, lane, v);
      if (EPI == kEpiHist) hist_fold<NP>(a, t, r, v);
    }
    if (EPI == kEpiGreedy && ok) greedy_finish(a, e);
    if (!ok) *abort_flag = 1;
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // Let the loads this CTA issued land before its shared memory goes away.
    for (long long i = issued > kStagesD ? issued - kStagesD : 0; i < issued; ++i)
      mbar_wait(&full[i % kStagesD], (int)(i / kStagesD) & 1, err);
  }
  if (warp == 1 && lane == 0) mbar_wait(drain, 0, err);  // every MMA has finished
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(2 * NP < 32 ? 32 : 2 * NP));
  }
}

size_t counters_elems(const Part& p) { return ((size_t)p.tiles + 63) / 64 * 64; }

template <int NP, int EPI>
cudaError_t launch(const LinearArgs& a, cudaStream_t s) {
  const Part p = make_part(a.N, a.K, a.epilogue);
  int* counters = a.counters;
  float* slots = a.partial;
  size_t slot_elems = a.partial_elems;
  if (!counters) {  // carve the counters from the scratch and clear them
    if (!a.partial || a.partial_elems < counters_elems(p)) return cudaErrorInvalidValue;
    counters = reinterpret_cast<int*>(a.partial);
    slots = a.partial + counters_elems(p);
    slot_elems = a.partial_elems - counters_elems(p);
    cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)p.tiles * sizeof(int), s);
    if (e != cudaSuccess) return e;
  } else if (a.counters_elems < (size_t)p.tiles) {
    return cudaErrorInvalidValue;
  }
  const size_t nslots = EPI == kEpiPieces ? (size_t)p.G + p.tiles : (size_t)2 * p.G;
  if (!slots || slot_elems < nslots * kRows * NP) return cudaErrorInvalidValue;
  CUtensorMap tw, tx;
  const uint64_t wrows = (EPI == kEpiSwiGLU) ? 2ull * a.N : (uint64_t)a.N;
  if (!tc_host::make_map(&tw, a.W, wrows, a.K, a.K, 64) ||
      !tc_host::make_map(&tx, a.X, a.M, a.K, a.ldx, NP))
    return cudaErrorInvalidValue;
  constexpr int smem = DLayout<NP>::kBytes;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_tc_kernel<NP, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  { const cudaError_t _le = launch_pdl(gemv_tc_kernel<NP, EPI>, dim3(p.G), dim3(kThreadsD), smem, s, tw, tx, a, p, counters, slots, a.err); if (_le != cudaSuccess) return _le; }
  return cudaGetLastError();
}

template <int EPI>
cudaError_t launch_np(const LinearArgs& a, cudaStream_t s) {
  return a.M <= 16 ? launch<16, EPI>(a, s) : launch<32, EPI>(a, s);
}

}  // namespace

bool gemv_tc_applicable(int dtype, int M, int N, int K) {
  return dtype == kBF16 && M >= 1 && M <= 32 && N % 16 == 0 && K % kKB == 0 &&
         tc_host::encoder() != nullptr;
}

size_t gemv_tc_scratch_elems(int M, int N, int K, int epilogue, bool with_counters) {
  const Part p = make_part(N, K, epilogue);
  const int np = M <= 16 ? 16 : 32;
  const size_t nslots = epilogue == kEpiPieces ? (size_t)p.G + p.tiles : (size_t)2 * p.G;
  return (with_counters ? counters_elems(p) : 0) + nslots * kRows * np;
}

bool gemv_pieces_plan(int dtype, int M, int N, int K, Pieces* out) {
  if (!gemv_tc_applicable(dtype, M, N, K)) return false;
  const Part p = make_part(N, K, kEpiPieces);
  out->slots = nullptr;
  out->total = p.total;
  out->G = p.G;
  out->nk = p.nk;
  out->np = M <= 16 ? 16 : 32;
  return true;
}

size_t gemv_tc_tiles(int N, int epilogue) {
  return (epilogue == kEpiSwiGLU) ? (N + 63) / 64 : (N + kRows - 1) / kRows;
}

cudaError_t launch_gemv_tc(const LinearArgs& a, cudaStream_t s) {
  if (((uintptr_t)a.X % 16) || ((uintptr_t)a.W % 16) || (a.ldx % 8)) return cudaErrorInvalidValue;
  switch (a.epilogue) {
    case kEpiStore: return launch_np<kEpiStore>(a, s);
    case kEpiResid: return launch_np<kEpiResid>(a, s);
    case kEpiPieces: return launch_np<kEpiPieces>(a, s);
    case kEpiGreedy:
      if (!a.greedy.best || !a.greedy.done || !a.greedy.ids) return cudaErrorInvalidValue;
      return launch_np<kEpiGreedy>(a, s);
    case kEpiHist:
      if (!a.hist || !a.Y) return cudaErrorInvalidValue;
      return launch_np<kEpiHist>(a, s);
    default: return launch_np<kEpiSwiGLU>(a, s);
  }
}

}  // namespace mg
