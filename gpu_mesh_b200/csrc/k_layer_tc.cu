// Decode layer chain: the decoder work between two attention launches in one
// persistent kernel.
//
// A decode layer (<= 32 token rows) is four weight streams (o_proj, gate/up,
// down, the next layer's qkv) and two RMSNorms.  As separate launches every
// weight stream pays a ramp-up and a drain (its last CTAs finish split tiles
// while the other SMs idle) and every norm pays a launch: at 32 rows that is
// about half of the step.  Here one CTA per SM runs the steps in order,
// separated by grid barriers, and the TMA producer keeps streaming: it
// requests the next step's weights (which depend on nothing) into its ring
// while the epilogue warps finish the current step and wait at the barrier;
// only the activation tiles wait for the barrier.
//
// Steps (ChainArgs, at most kMaxChainSteps):
//   linear   Y = f(X · Wᵀ), the stream-K tcgen05 GEMM of k_gemv_tc.cu with the
//            same split, fix-up order and epilogues (bit-identical results);
//   rmsnorm  rows of x into y, one row per CTA on the four epilogue warps,
//            with the reduction order of rmsnorm_kernel at 128 threads.
// The grid barrier is a counter and a generation word in global memory; a
// CTA arrives with a release, waits with acquire loads, and gives up after
// the bounded wait (code 3 in the error word), skipping its remaining steps.
// The grid is one CTA per SM and a CTA fills an SM's shared memory, so once
// the kernels ahead of it drain every CTA is resident; the grid barrier's
// bounded wait covers the case where another stream keeps an SM busy.
#include "gemv_tc_parts.cuh"
#include "linear_tc.h"

namespace mg {
namespace {

using namespace tc;
using namespace gemvtc;

constexpr int kMaxChainGemm = 4;

struct StepDesc {
  int kind;  // kChainLinear / kChainNorm
  int map;   // linear: index of its tensor maps
  int N, K, epi;
  void* Y;
  int64_t ldy;
  const void* R;
  int64_t ldr;
  Part part;
  const void* nx;  // rmsnorm
  int64_t nxs;
  const void* nw;
  void* ny;
  int H;
  float eps;
};

struct ChainParams {
  CUtensorMap tw[kMaxChainGemm];
  CUtensorMap tx[kMaxChainGemm];
  StepDesc st[kMaxChainSteps];
  int nst;
  int M;
  int* counters;
  float* slots;
  int* err;
  int* bar;      // arrivals since the work memory was set up (wrapping)
  int bar_base;  // generation before this launch
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The barrier word counts arrivals since the stage's work memory was set up
// (it wraps; comparisons are differences).  The barrier before step j of a
// launch is complete once it holds base + j·grid.
__device__ __forceinline__ bool gen_reached(const int* bar, int target) {
  return (int)((unsigned)ld_acquire_gpu(bar) - (unsigned)target) >= 0;
}

__device__ bool gen_wait(const int* bar, int target, int* err) {
  if (gen_reached(bar, target)) return true;
  const uint64_t t0 = globaltimer();
  while (!gen_reached(bar, target)) {
    if (globaltimer() - t0 > kWaitNs) {
      atomicCAS(err, 0, kErrTimeout);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

// Arrive: a fire-and-forget add with release semantics (this thread's
// writes, and after the preceding CTA barrier the whole CTA's, are visible to
// whoever observes the count).
__device__ __forceinline__ void grid_arrive(int* bar) {
  asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(bar) : "memory");
}

__device__ __forceinline__ int ld_acquire_cta_shared(const volatile int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared.s32 %0, [%1];" : "=r"(v) : "r"(smem_u32((const void*)p)) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_cta_shared(volatile int* p, int v) {
  asm volatile("st.release.cta.shared.s32 [%0], %1;" ::"r"(smem_u32((const void*)p)), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// CTA c's units of a step: the standalone GEMM's split over part.G CTAs;
// CTAs beyond part.G (small matrices) have none.
__device__ __forceinline__ void unit_range(const Part& p, int c, long long& u0, long long& u1) {
  if (c < p.G) {
    u0 = p.begin(c);
    u1 = p.begin(c + 1);
  } else {
    u0 = u1 = p.total;
  }
}

template <int NP>
__device__ __forceinline__ void apply_rt(const LinearArgs& a, int epi, int t, int r, const float* v,
                                         float* xchg) {
  if (epi == kEpiSwiGLU) apply<NP, kEpiSwiGLU>(a, t, r, v, xchg);
  else if (epi == kEpiResid) apply<NP, kEpiResid>(a, t, r, v, xchg);
  else apply<NP, kEpiStore>(a, t, r, v, xchg);
}

template <int NP>
__global__ void __launch_bounds__(kThreadsD, 1) layer_chain_kernel(const __grid_constant__ ChainParams P) {
  using L = DLayout<NP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* xchg = (float*)(smem + L::kTiles);
  uint64_t* full = (uint64_t*)(smem + L::kBarOff);
  uint64_t* empty = full + kStagesD;
  uint64_t* tfull = empty + kStagesD;  // [2]
  uint64_t* tempty = tfull + 2;        // [2]
  uint64_t* drain = tempty + 2;        // final MMA completion
  uint32_t* tmem_holder = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_holder + 1);
  float* red = (float*)(tmem_holder + 4);  // [16] norm partial sums
  volatile int* gate = (volatile int*)(tmem_holder + 20);  // highest step whose barrier this CTA passed

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesD; ++s) {
      mbar_init(&full[s], 2);  // weight tile + activation tile (the latter after its barrier)
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *gate = 0;
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
  pdl_trigger();

  // Stage-ring bookkeeping shared by the producer's abort path.
  long long issued = 0;
  int xpend_mask = 0;  // stages whose activation tile is still owed

  if (warp == 0) {
    if (lane == 0) {
      // Producer.  Activation tiles of step j may be loaded once generation
      // bar_base + j is reached (step 0: once the previous kernel is done).
      int open_upto = -1;  // highest step whose activations may be loaded
      bool waited = false;
      int pend_step[kStagesD], pend_kx[kStagesD];
      const CUtensorMap* pend_map[kStagesD];
      long long pend_i[kStagesD];
      // Step j > 0 opens when this CTA's epilogue warps have passed the grid
      // barrier before it (they publish it in `gate`, release/acquire).
      auto try_open = [&](int j, bool block) -> bool {
        if (j <= open_upto) return true;
        if (!waited) {
          if (!block) return false;
          pdl_wait();
          waited = true;
        }
        if (j > 0 && ld_acquire_cta_shared(gate) < j) {
          if (!block) return false;
          const uint64_t t0 = globaltimer();
          while (ld_acquire_cta_shared(gate) < j) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > kWaitNs) {
              atomicCAS(P.err, 0, kErrTimeout);
              return false;
            }
          }
        }
        fence_proxy_global();
        open_upto = j;
        return true;
      };
      auto load_x = [&](const CUtensorMap* tx, int kx, int s) {
        mbar_expect_tx(&full[s], L::kX);
        tma_load_2d(smem + s * L::kStage + kWBytes, tx, &full[s], kx, 0);
      };
      // Issue owed activation tiles oldest first (their steps never decrease).
      // With need >= 0, every tile up to ring position `need` must go out,
      // waiting for its step's barrier if necessary; the barrier of step j
      // only needs this CTA's tiles of steps before j, which go out first.
      auto flush = [&](long long need) -> bool {
        while (xpend_mask) {
          int s = -1;
          for (int k = 0; k < kStagesD; ++k)
            if ((xpend_mask >> k & 1) && (s < 0 || pend_i[k] < pend_i[s])) s = k;
          const bool must = need >= 0 && pend_i[s] <= need;
          if (!try_open(pend_step[s], must)) return !must;
          load_x(pend_map[s], pend_kx[s], s);
          xpend_mask &= ~(1 << s);
        }
        return true;
      };
      long long i = 0;
      for (int j = 0; j < P.nst && !*abort_flag; ++j) {
        if (P.st[j].kind != kChainLinear) continue;
        // Copies in registers: the descriptors live in parameter memory.
        const Part part = P.st[j].part;
        const int N = P.st[j].N, epi = P.st[j].epi;
        const CUtensorMap* tw = &P.tw[P.st[j].map];
        const CUtensorMap* tx = &P.tx[P.st[j].map];
        long long u0, u1;
        unit_range(part, c, u0, u1);
        for (long long u = u0; u < u1; ++u, ++i) {
          const int s = (int)(i % kStagesD);
          if (i >= kStagesD) {
            if (!flush(i - kStagesD)) {  // the stage's last occupant needs its activations
              *abort_flag = 1;
              break;
            }
            if (!mbar_wait(&empty[s], (int)((i / kStagesD) - 1) & 1, P.err)) {
              *abort_flag = 1;
              break;
            }
          }
          const int t = (int)(u / part.nk), kb = (int)(u % part.nk);
          const int r0 = (epi == kEpiSwiGLU) ? t * 64 : t * kRows;
          const int r1 = (epi == kEpiSwiGLU) ? N + t * 64 : t * kRows + 64;
          uint8_t* stg = smem + s * L::kStage;
          mbar_expect_tx(&full[s], kWBytes);
          tma_load_2d(stg, tw, &full[s], kb * kKB, r0);
          tma_load_2d(stg + kWBytes / 2, tw, &full[s], kb * kKB, r1);
          issued = i + 1;
          if (!xpend_mask && try_open(j, false)) {
            load_x(tx, kb * kKB, s);
          } else {
            pend_step[s] = j;
            pend_map[s] = tx;
            pend_kx[s] = kb * kKB;
            pend_i[s] = i;
            xpend_mask |= 1 << s;
            flush(-1);
          }
        }
        if (*abort_flag) break;
      }
      if (xpend_mask && !*abort_flag && !flush(issued - 1)) *abort_flag = 1;  // the last owed tiles
      if (!waited) pdl_wait();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer: one accumulator per tile piece, alternating TMEM halves.
      constexpr uint32_t idesc = instr_desc(NP);
      long long i = 0;
      int pi = 0;
      for (int j = 0; j < P.nst && !*abort_flag; ++j) {
        if (P.st[j].kind != kChainLinear) continue;
        const Part p = P.st[j].part;
        long long u0, u1;
        unit_range(p, c, u0, u1);
        const int t_first = (int)(u0 / p.nk);
        const int t_last = u1 > u0 ? (int)((u1 - 1) / p.nk) : t_first - 1;
        for (int t = t_first; t <= t_last && !*abort_flag; ++t, ++pi) {
          const long long lo = max(u0, (long long)t * p.nk), hi = min(u1, (long long)(t + 1) * p.nk);
          const int b = pi & 1;
          if (pi >= 2 && !mbar_wait(&tempty[b], ((pi >> 1) - 1) & 1, P.err)) {
            *abort_flag = 1;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t dt = tmem + b * NP;
          for (long long u = lo; u < hi; ++u, ++i) {
            const int s = (int)(i % kStagesD);
            if (!mbar_wait(&full[s], (int)(i / kStagesD) & 1, P.err)) {
              *abort_flag = 1;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint8_t* stg = smem + s * L::kStage;
            const uint64_t da = smem_desc(stg), db = smem_desc(stg + kWBytes);
#pragma unroll
            for (int k = 0; k < kKB / 16; ++k)
              mma_bf16(dt, da + 2 * k, db + 2 * k, idesc, (u > lo || k > 0) ? 1u : 0u);
            mma_commit(&empty[s]);
          }
          mma_commit(&tfull[b]);
        }
      }
      mma_commit(drain);
    }
  } else {
    // Epilogue warps 2-5: steps in order, a grid barrier between steps.
    pdl_wait();
    const int q = warp & 3;
    const int e = threadIdx.x - 64;  // 0..127
    const int r = q * 32 + lane;     // W row within the tile
    int pi = 0;
    bool ok = true;
    for (int j = 0; j < P.nst && ok; ++j) {
      if (j > 0) {
        // This CTA's writes of step j - 1 are done: make them visible to
        // every CTA (and to their TMA loads), then wait for all CTAs.
        fence_proxy_global();
        epi_bar();
        bool good = true;
        if (e == 0) {
          grid_arrive(P.bar);
          good = gen_wait(P.bar, (int)((unsigned)P.bar_base + (unsigned)j * gridDim.x), P.err) && !*abort_flag;
          if (good) st_release_cta_shared(gate, j);
        }
        if (epi_bar_any(!good)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
      }
      const StepDesc d = P.st[j];  // a copy in registers
      if (d.kind == kChainNorm) {
        if (c < P.M) {
          // RMSNorm of row c in the RMSNorm reduction order (512 threads): the
          // 128 threads play virtual threads e + 128·k, k = 0..3, and thread
          // j's warp butterfly becomes this warp's for round k.
          const bf16* xr = (const bf16*)d.nx + (size_t)c * d.nxs;
          const bf16* w = (const bf16*)d.nw;
          bf16* yr = (bf16*)d.ny + (size_t)c * d.H;
          const int ew = e >> 5;  // 0..3
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float ss = 0.f;
            for (int i = e + 128 * k; i < d.H / 8; i += kNormThreads) {
              float v[8];
              load16_f<bf16>(xr + i * 8, v);
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) ss += v[jj] * v[jj];
            }
            ss = warp_sum(ss);
            if (lane == 0) red[ew + 4 * k] = ss;
          }
          epi_bar();
          float tot = lane < 16 ? red[lane] : 0.f;
          tot = warp_sum(tot);
          epi_bar();
          const float4* w4 = reinterpret_cast<const float4*>(w);
          float4 wv[4];  // the weights of this thread's (first four) vectors
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (e + k * 128 < d.H / 8) wv[k] = __ldg(w4 + e + k * 128);
          const float rs = 1.0f / sqrtf(tot / (float)d.H + d.eps);
          for (int i = e, k4 = 0; i < d.H / 8; i += 128, ++k4) {
            float v[8], g[8];
            load16_f<bf16>(xr + i * 8, v);
            if (k4 < 4) {
              const float4 wk = k4 == 0 ? wv[0] : k4 == 1 ? wv[1] : k4 == 2 ? wv[2] : wv[3];
              const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wk);
#pragma unroll
              for (int k = 0; k < 8; ++k) g[k] = __bfloat162float(wb[k]);
            } else {
              load16_f<bf16>(w + i * 8, g);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) stf<bf16>(yr + i * 8 + k, rt<bf16>(rt<bf16>(v[k] * rs) * g[k]));
          }
        }
        continue;
      }
      LinearArgs a{};
      a.M = P.M;
      a.N = d.N;
      a.K = d.K;
      a.Y = d.Y;
      a.ldy = d.ldy;
      a.R = d.R;
      a.ldr = d.ldr;
      a.epilogue = d.epi;
      const Part p = d.part;
      long long u0, u1;
      unit_range(p, c, u0, u1);
      const int t_first = (int)(u0 / p.nk);
      const int t_last = u1 > u0 ? (int)((u1 - 1) / p.nk) : t_first - 1;
      for (int t = t_first; t <= t_last; ++t, ++pi) {
        const int b = pi & 1;
        const bool okw = mbar_wait(&tfull[b], (pi >> 1) & 1, P.err);
        if (epi_bar_any(!okw)) {  // a timeout anywhere stops all four warps together
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

        const long long lo = max(u0, (long long)t * p.nk), hi = min(u1, (long long)(t + 1) * p.nk);
        const bool whole = lo == (long long)t * p.nk && hi == (long long)(t + 1) * p.nk;
        if (!whole && !piece_done<NP>(p, P.slots, P.counters, c, t, r, e, v)) continue;  // another CTA finishes it
        apply_rt<NP>(a, d.epi, t, r, v, xchg);
      }
      if (!ok) {
        *abort_flag = 1;
        break;
      }
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // Complete the arrivals still owed, then let the loads this CTA issued
    // land before its shared memory goes away.
    for (int s = 0; s < kStagesD; ++s)
      if (xpend_mask >> s & 1) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&full[s])) : "memory");
    for (long long i = issued > kStagesD ? issued - kStagesD : 0; i < issued; ++i)
      mbar_wait(&full[i % kStagesD], (int)(i / kStagesD) & 1, P.err);
  }
  if (warp == 1 && lane == 0) mbar_wait(drain, 0, P.err);  // every MMA has finished
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(2 * NP < 32 ? 32 : 2 * NP));
  }
}

template <int NP>
cudaError_t launch_np(const ChainParams& P, cudaStream_t s) {
  constexpr int smem = DLayout<NP>::kBytes;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(layer_chain_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(kThreadsD);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, layer_chain_kernel<NP>, P);
  note_launch();
  return e;
}

}  // namespace

bool layer_chain_applicable(const ChainArgs& a) {
  if (a.dtype != kBF16 || a.M < 1 || a.M > 32 || a.nsteps < 1 || a.nsteps > kMaxChainSteps) return false;
  int gemms = 0;
  for (int j = 0; j < a.nsteps; ++j) {
    const ChainStep& st = a.step[j];
    if (st.kind == kChainLinear) {
      if (!gemv_tc_applicable(a.dtype, a.M, st.N, st.K) || ++gemms > kMaxChainGemm) return false;
    } else if (st.kind == kChainNorm) {
      if (st.H % 8) return false;
    } else {
      return false;
    }
  }
  return true;
}

size_t layer_chain_scratch_elems() { return (size_t)2 * sm_count() * kRows * 32; }

int layer_chain_grid() { return sm_count(); }

cudaError_t launch_layer_chain(const ChainArgs& a, cudaStream_t s) {
  if (!layer_chain_applicable(a) || !a.bar || !a.counters) return cudaErrorInvalidValue;
  const int NP = a.M <= 16 ? 16 : 32;
  ChainParams P;
  memset(&P, 0, sizeof(P));
  P.nst = a.nsteps;
  P.M = a.M;
  P.counters = a.counters;
  P.slots = a.partial;
  P.err = a.err;
  P.bar = a.bar;
  P.bar_base = a.bar_base;
  if ((size_t)2 * sm_count() * kRows * NP > a.partial_elems) return cudaErrorInvalidValue;
  int gm = 0;
  for (int j = 0; j < a.nsteps; ++j) {
    const ChainStep& st = a.step[j];
    StepDesc& d = P.st[j];
    d.kind = st.kind;
    if (st.kind == kChainNorm) {
      d.nx = st.x;
      d.nxs = st.xs;
      d.nw = st.w;
      d.ny = st.y;
      d.H = st.H;
      d.eps = st.eps;
      continue;
    }
    if (((uintptr_t)st.X % 16) || ((uintptr_t)st.W % 16) || (st.ldx % 8)) return cudaErrorInvalidValue;
    d.map = gm;
    d.N = st.N;
    d.K = st.K;
    d.epi = st.epilogue;
    d.Y = st.Y;
    d.ldy = st.ldy;
    d.R = st.R;
    d.ldr = st.ldr;
    d.part = make_part(st.N, st.K, st.epilogue);  // CTAs >= part.G sit the step out
    if (a.counters_elems < (size_t)d.part.tiles) return cudaErrorInvalidValue;
    const uint64_t wrows = (st.epilogue == kEpiSwiGLU) ? 2ull * st.N : (uint64_t)st.N;
    if (!tc_host::make_map(&P.tw[gm], st.W, wrows, st.K, st.K, 64) ||
        !tc_host::make_map(&P.tx[gm], st.X, a.M, st.K, st.ldx, NP))
      return cudaErrorInvalidValue;
    ++gm;
  }
  return NP == 16 ? launch_np<16>(P, s) : launch_np<32>(P, s);
}

}  // namespace mg
