// Prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
#pragma once

#include "kernels.h"

namespace mg {

bool linear_tc_applicable(int dtype, int M, int N, int K);
size_t linear_tc_scratch_elems(int M, int N, int K, int epilogue);
cudaError_t launch_linear_tc(const LinearArgs& a, cudaStream_t s);
// The prefill qkv projection (store epilogue into q.qkv, bf16, head_dim 128,
// more than 32 rows) with RoPE, QK-norm and the KV append done in the GEMM's
// epilogue: q.q_out and the slots' caches receive what the projection
// followed by launch_qkv_post would write.
bool qkv_rope_fusable(const LinearArgs& a, const QkvPostArgs& q);
cudaError_t launch_qkv_rope_kv(const LinearArgs& a, const QkvPostArgs& q, cudaStream_t s);

// Decode linear layers (<= 32 token rows): stream-K tcgen05 weight stream.
bool gemv_tc_applicable(int dtype, int M, int N, int K);
// fp32 scratch: partial-sum slots, plus the tile counters when the caller
// does not provide a separate counter array.
size_t gemv_tc_scratch_elems(int M, int N, int K, int epilogue, bool with_counters);
// Tile counters a launch needs.
size_t gemv_tc_tiles(int N, int epilogue);
cudaError_t launch_gemv_tc(const LinearArgs& a, cudaStream_t s);

// Decode layer chain (k_layer_tc.cu): linear and RMSNorm steps of <= 32 token
// rows in one persistent, cooperative launch with grid barriers between
// steps.  Linear steps are the decode GEMM above (same results); norm steps
// normalise rows of x (row stride xs) into y (row stride H).
constexpr int kChainLinear = 0;
constexpr int kChainNorm = 1;
constexpr int kMaxChainSteps = 6;
struct ChainStep {
  int kind;
  const void* X; int64_t ldx;   // linear
  const void* W;
  void* Y; int64_t ldy;
  const void* R; int64_t ldr;
  int N, K, epilogue;
  const void* x; int64_t xs;    // rmsnorm
  const void* w;
  void* y;
  int H;
  float eps;
};
struct ChainArgs {
  int dtype;
  int M;
  int nsteps;
  ChainStep step[kMaxChainSteps];
  float* partial;               // split-K slots (layer_chain_scratch_elems)
  size_t partial_elems;
  int* counters;                // tile counters, zero between launches
  size_t counters_elems;
  int* err;
  int* bar;                     // grid barrier: arrivals so far (wrapping int)
  int bar_base;                 // its value before this launch; it ends at bar_base + (nsteps - 1) · grid
};
bool layer_chain_applicable(const ChainArgs& a);
size_t layer_chain_scratch_elems();
int layer_chain_grid();         // CTAs of a launch (one per SM)
cudaError_t launch_layer_chain(const ChainArgs& a, cudaStream_t s);

}  // namespace mg
