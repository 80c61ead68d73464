"""mg_linear_noalloc: the linear layer for callers that cannot allocate device
memory (a process whose device memory belongs to another allocator, or a
loop that cannot take cudaMalloc's device-wide synchronisation).  It keeps
its split-K scratch in a fixed array inside the library.

The test calls it through the C ABI on decode shapes that use split-K and
checks each of two consecutive calls against mg_linear (caller-provided
scratch).  Both run the same split-K kernels with the same plan, so the bar
is the tightest tolerance the kernel tests use: identical bf16 outputs.  This file is collected last so that a run which stops
at its first failure has already run every other test.
"""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
EPI = {"store": 0, "resid": 1, "swiglu": 2}


def _call(fn: str, x, w, n, epi, r, y, scratch=None):
    lib = _lib.lib()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    args = [_lib.MG_DTYPE_BF16, x.data_ptr(), x.stride(0), w.data_ptr(), x.shape[0], n, x.shape[1],
            EPI[epi], None if r is None else r.data_ptr(), 0 if r is None else r.stride(0),
            y.data_ptr(), y.stride(0)]
    if fn == "mg_linear":
        args += [scratch.data_ptr(), scratch.numel()]
    _lib.check(getattr(lib, fn)(*args, stream))


@pytest.mark.parametrize("M,N,K,epi", [
    (8, 4096, 4096, "resid"),     # o_proj, split-K 10 ways
    (16, 4096, 14336, "resid"),   # down_proj at 16 rows
    (5, 6144, 4096, "store"),     # fused q/k/v
    (16, 14336, 4096, "swiglu"),  # gate/up
])
def test_noalloc_matches_mg_linear_twice(M, N, K, epi):
    lib = _lib.lib()
    need = int(lib.mg_linear_scratch(_lib.MG_DTYPE_BF16, M, N, K, EPI[epi]))
    assert 0 < need <= lib_limit(), "the shape should exercise the split-K scratch"
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    rows = 2 * N if epi == "swiglu" else N
    for call in range(2):  # the array keeps the previous call's partial sums
        x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
        w = (torch.randn(rows, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
        r = torch.randn(M, N, generator=g, device=DEV).to(torch.bfloat16) if epi == "resid" else None
        want = r.clone() if r is not None else torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        got = r.clone() if r is not None else torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        scratch = torch.empty(need, dtype=torch.float32, device=DEV)
        _call("mg_linear", x, w, N, epi, want, want, scratch)
        _call("mg_linear_noalloc", x, w, N, epi, got, got)
        torch.cuda.synchronize()
        assert torch.equal(got, want), (call, float((got.float() - want.float()).abs().max()))


def lib_limit() -> int:
    return 1024 * 1024  # MG_LINEAR_NOALLOC_SCRATCH


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
