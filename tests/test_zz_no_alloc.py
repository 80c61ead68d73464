"""mg_linear_noalloc: the linear layer for callers that cannot allocate device
memory (a process whose device memory belongs to another allocator, or a
loop that cannot take cudaMalloc's device-wide synchronisation).  It keeps
its split-K scratch in a fixed array inside the library.

The test calls it through the C ABI on bf16 decode shapes that use split-K
(and one fp32 shape, whose kernel needs no scratch) and checks each of two
consecutive calls against mg_linear (caller-provided scratch).  Both run the
same kernels with the same plan, so the bar is the tightest tolerance the
kernel tests use: identical outputs.  This file is collected last so that a
run which stops at its first failure has already run every other test.
"""
from __future__ import annotations

import re

import pytest
import torch

from gpu_mesh_b200 import _lib
from tests.conftest import ROOT

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
EPI = {"store": 0, "resid": 1, "swiglu": 2}


def _call(fn: str, x, w, n, epi, r, y, scratch=None):
    lib = _lib.lib()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    dt = _lib.MG_DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.MG_DTYPE_F32
    args = [dt, x.data_ptr(), x.stride(0), w.data_ptr(), x.shape[0], n, x.shape[1],
            EPI[epi], None if r is None else r.data_ptr(), 0 if r is None else r.stride(0),
            y.data_ptr(), y.stride(0)]
    if fn == "mg_linear":
        args += [scratch.data_ptr(), scratch.numel()]
    _lib.check(getattr(lib, fn)(*args, stream))


@pytest.mark.parametrize("M,N,K,epi,dtype", [
    (8, 4096, 4096, "resid", torch.bfloat16),     # o_proj, split-K 10 ways
    (16, 4096, 14336, "resid", torch.bfloat16),   # down_proj at 16 rows
    (5, 6144, 4096, "store", torch.bfloat16),     # fused q/k/v
    (16, 14336, 4096, "swiglu", torch.bfloat16),  # gate/up
    (4, 1536, 512, "resid", torch.float32),       # fp32 kernel: no split-K scratch at all
])
def test_noalloc_matches_mg_linear_twice(M, N, K, epi, dtype):
    lib = _lib.lib()
    dt = _lib.MG_DTYPE_BF16 if dtype == torch.bfloat16 else _lib.MG_DTYPE_F32
    need = int(lib.mg_linear_scratch(dt, M, N, K, EPI[epi]))
    if dtype == torch.bfloat16:
        assert 0 < need <= lib_limit(), "the shape should exercise the split-K scratch"
    else:
        assert need == 0
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    rows = 2 * N if epi == "swiglu" else N
    for call in range(2):  # the array keeps the previous call's partial sums
        x = torch.randn(M, K, generator=g, device=DEV).to(dtype)
        w = (torch.randn(rows, K, generator=g, device=DEV) * 0.02).to(dtype)
        r = torch.randn(M, N, generator=g, device=DEV).to(dtype) if epi == "resid" else None
        want = r.clone() if r is not None else torch.empty(M, N, dtype=dtype, device=DEV)
        got = r.clone() if r is not None else torch.empty(M, N, dtype=dtype, device=DEV)
        scratch = torch.empty(max(need, 1), dtype=torch.float32, device=DEV)
        _call("mg_linear", x, w, N, epi, want, want, scratch)
        _call("mg_linear_noalloc", x, w, N, epi, got, got)
        _lib.check(lib.mg_linear_check_device(torch.cuda.current_stream(DEV).cuda_stream))
        assert torch.equal(got, want), (call, float((got.float() - want.float()).abs().max()))


def lib_limit() -> int:
    """MG_LINEAR_NOALLOC_SCRATCH, read from the header that defines it."""
    text = (ROOT / "include" / "meshgpu_b200.h").read_text()
    m = re.search(r"#define MG_LINEAR_NOALLOC_SCRATCH \((\d+)u \* (\d+)u\)", text)
    assert m, "MG_LINEAR_NOALLOC_SCRATCH not found in the header"
    return int(m.group(1)) * int(m.group(2))


def test_noalloc_rejects_shapes_beyond_its_array():
    # o_proj at 32 token rows needs more split-K scratch than the fixed
    # array holds: the call must refuse before launching anything.
    lib = _lib.lib()
    M, N, K = 32, 4096, 4096
    need = int(lib.mg_linear_scratch(_lib.MG_DTYPE_BF16, M, N, K, 1))
    assert need > lib_limit()
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(N, K, dtype=torch.bfloat16, device=DEV)
    y = torch.zeros(M, N, dtype=torch.bfloat16, device=DEV)
    rc = lib.mg_linear_noalloc(_lib.MG_DTYPE_BF16, x.data_ptr(), K, w.data_ptr(), M, N, K, 1,
                               y.data_ptr(), N, y.data_ptr(), N, None)
    assert rc == _lib.MG_EINVAL
    assert "mg_linear_noalloc holds" in _lib.last_error()
