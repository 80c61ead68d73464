// Prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
#pragma once

#include "kernels.h"

namespace mg {

bool linear_tc_applicable(int dtype, int M, int N, int K);
size_t linear_tc_scratch_elems(int M, int N, int K, int epilogue);
cudaError_t launch_linear_tc(const LinearArgs& a, cudaStream_t s);

}  // namespace mg
