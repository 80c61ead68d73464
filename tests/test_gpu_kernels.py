"""Single-kernel numerics: the stage's linear layer (``mg_linear``) on each of
its paths against a plain PyTorch fp32 reference of the same op.

Paths: the weight-streaming GEMV (bf16, <= 32 rows, with and without split-K),
the tcgen05 GEMM (bf16, > 32 rows) and the SIMT kernel (fp32).

Tolerances: the reference applies the same rounding points (round the
product to bf16; round again after the residual add; round gate, up,
silu(gate) and the product for SwiGLU) to an fp32 accumulation.  Two fp32
accumulations in different orders differ by a few fp32 units of the sum of
|x_k * w_k|, which can move a bf16 rounding by one unit in the last place.
The bar per element is therefore
    1 ulp (plain product), 2 ulp (after the residual add), 3 ulp (SwiGLU)
    + 3e-5 * sum_k |x_k * w_k|   (the accumulation-order term, which matters
                                   only where the result nearly cancels).
fp32: 1e-5 relative to the output's largest magnitude.
"""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200.kernels import linear

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def bf16_ulp(t: torch.Tensor) -> torch.Tensor:
    a = t.float().abs().clamp(min=2.0**-100)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


def reference(x, w, epilogue, residual=None):
    """(expected output, accumulation-order error term) in fp32."""
    torch.backends.cuda.matmul.allow_tf32 = False
    rt = (lambda v: v.to(x.dtype).float())
    xa = x.float().abs()
    if epilogue == "swiglu":
        n = w.shape[0] // 2
        g = rt(x.float() @ w[:n].float().T)
        u = rt(x.float() @ w[n:].float().T)
        sg = rt(g / (1 + torch.exp(-g)))
        dg = xa @ w[:n].float().abs().T
        du = xa @ w[n:].float().abs().T
        # one-ulp moves of the rounded gate, up and silu(gate) carried to the product
        flips = 1.1 * bf16_ulp(g) * u.abs() + bf16_ulp(u) * sg.abs() + bf16_ulp(sg) * u.abs()
        return rt(sg * u), 3e-5 * (dg * (u.abs() + 1) + du * (sg.abs() + 1)) + flips
    acc = x.float() @ w.float().T
    slack = 3e-5 * (xa @ w.float().abs().T)
    if epilogue == "resid":
        # a one-ulp move of round(acc) survives the add even where R cancels it
        return rt(residual.float() + rt(acc)), slack + bf16_ulp(rt(acc))
    return rt(acc), slack


def check(y, ref, dtype, ulps):
    ref, slack = ref
    if dtype == torch.float32:
        assert (y.float() - ref).abs().max() <= 1e-5 * ref.abs().max()
        return
    err = (y.float() - ref).abs()
    bad = err > ulps * bf16_ulp(ref) + slack
    worst = float((err / bf16_ulp(ref)).max())
    assert not bad.any(), f"{int(bad.sum())} elements beyond the bar (worst {worst:.1f} ulp)"


SHAPES = [
    # (M, N, K): decode GEMV shapes (split-K when N is narrow) ...
    (1, 4096, 4096), (5, 6144, 4096), (8, 4096, 14336), (16, 28672 // 2, 4096), (17, 512, 1408),
    (32, 128256, 4096), (32, 4096, 4096),
    # ... and prefill shapes on the tcgen05 GEMM, including ragged M.
    (33, 4096, 4096), (100, 688, 256), (128, 6144, 4096), (300, 4096, 14336), (1024, 1024, 2560),
    # several tiles per CTA of the persistent GEMM, both tile orders, ragged N
    (2048, 4096, 4096), (4096, 1024, 2048), (1500, 2000, 512),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("epilogue", ["store", "resid", "swiglu"])
def test_linear_bf16_matches_fp32_reference(M, N, K, epilogue):
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N + K)
    x = (torch.randn(M, K, generator=g, device=DEV) * 1.0).to(torch.bfloat16)
    rows = 2 * N if epilogue == "swiglu" else N
    w = (torch.randn(rows, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    r = torch.randn(M, N, generator=g, device=DEV).to(torch.bfloat16) if epilogue == "resid" else None
    ref = reference(x, w, epilogue, r)
    y = linear(x, w, epilogue=epilogue, residual=None if r is None else r.clone(),
               out=None if r is None else r.clone())
    torch.cuda.synchronize()
    check(y, ref, torch.bfloat16, {"store": 1, "resid": 2, "swiglu": 3}[epilogue])


@pytest.mark.parametrize(
    "M,N,K,epilogue",
    [(8192, 6144, 4096, "store"), (8192, 4096, 14336, "resid"), (8192, 14336, 4096, "swiglu")],
    ids=["qkv", "down", "gate_up"],
)
def test_linear_full_prefill_shapes_match_fp32_reference(M, N, K, epilogue):
    """The Llama-3-8B prefill GEMMs at the benchmark's 8192 token rows: the
    only sizes at which the CTA-pair kernel walks its tiles in more than one
    L2 band."""
    test_linear_bf16_matches_fp32_reference(M, N, K, epilogue)


@pytest.mark.parametrize("M,N,K", [(33, 4096, 4096), (300, 688, 256), (1500, 2000, 512), (2048, 4096, 4096)])
@pytest.mark.parametrize("epilogue", ["store", "resid", "swiglu"])
def test_linear_single_sm_kernel_matches_fp32_reference(M, N, K, epilogue, monkeypatch):
    """The single-SM persistent GEMM that stands in where a device cannot
    co-schedule CTA pairs (selected here by its environment switch)."""
    monkeypatch.setenv("MESHGPU_GEMM_SINGLE_SM", "1")
    test_linear_bf16_matches_fp32_reference(M, N, K, epilogue)


def test_linear_in_place_residual():
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(64, 512, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(256, 512, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    r = torch.randn(64, 256, generator=g, device=DEV).to(torch.bfloat16)
    ref = reference(x, w, "resid", r)
    linear(x, w, epilogue="resid", residual=r, out=r)  # Y aliases R, as in the stage
    check(r, ref, torch.bfloat16, 2)


@pytest.mark.parametrize("M,N,K", [(1, 64, 64), (7, 1408, 512), (64, 512, 1408), (200, 96, 40)])
@pytest.mark.parametrize("epilogue", ["store", "resid", "swiglu"])
def test_linear_fp32_matches_reference(M, N, K, epilogue):
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g, device=DEV)
    rows = 2 * N if epilogue == "swiglu" else N
    w = torch.randn(rows, K, generator=g, device=DEV) * 0.02
    r = torch.randn(M, N, generator=g, device=DEV) if epilogue == "resid" else None
    ref = reference(x, w, epilogue, r)
    y = linear(x, w, epilogue=epilogue, residual=r)
    check(y, ref, torch.float32, 0)


def test_linear_rejects_bad_arguments():
    x = torch.zeros(4, 60, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(64, 60, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError, match="multiples of 16 bytes"):
        linear(x, w)
    with pytest.raises(ValueError, match="residual"):
        linear(torch.zeros(4, 64, dtype=torch.bfloat16, device=DEV),
               torch.zeros(64, 64, dtype=torch.bfloat16, device=DEV), epilogue="resid")
