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

}  // namespace mg
