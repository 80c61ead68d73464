"""Direct access to single kernels of the stage (the C ABI's ``mg_linear``).

The stage runs these inside ``mg_stage_forward``; exposing the linear layer
lets callers and tests drive one GEMM path at a time: the weight-streaming
GEMV (<= 32 rows), the tcgen05 GEMM (more rows, bf16) and the SIMT kernel
(fp32).
"""
from __future__ import annotations

import torch

from gpu_mesh_b200 import _lib

EPILOGUES = {"store": 0, "resid": 1, "swiglu": 2}
_DT = {torch.float32: _lib.MG_DTYPE_F32, torch.bfloat16: _lib.MG_DTYPE_BF16}


def linear(x: torch.Tensor, w: torch.Tensor, *, epilogue: str = "store",
           residual: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """epilogue(x @ w.T) on the device; ``swiglu`` takes w = [gate; up]."""
    if x.dtype not in _DT or w.dtype != x.dtype or x.device.type != "cuda":
        raise ValueError("linear needs CUDA fp32 or bf16 tensors of one dtype")
    if x.stride(-1) != 1 or w.stride(-1) != 1 or not w.is_contiguous():
        raise ValueError("x rows and w must be contiguous")
    M, K = x.shape
    N = w.shape[0] // 2 if epilogue == "swiglu" else w.shape[0]
    if w.shape[1] != K:
        raise ValueError("x and w disagree on K")
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    code = EPILOGUES[epilogue]
    lib = _lib.lib()
    n_scr = lib.mg_linear_scratch(_DT[x.dtype], M, N, K, code)
    scratch = torch.empty(max(int(n_scr), 1), dtype=torch.float32, device=x.device)
    r = residual if residual is not None else None
    with torch.cuda.device(x.device):  # the kernel runs on x's GPU, on its current stream
        _lib.check(lib.mg_linear(
            _DT[x.dtype], x.data_ptr(), x.stride(0), w.data_ptr(), M, N, K, code,
            None if r is None else r.data_ptr(), 0 if r is None else r.stride(0),
            out.data_ptr(), out.stride(0), scratch.data_ptr(), scratch.numel(),
            torch.cuda.current_stream(x.device).cuda_stream,
        ))
    return out
