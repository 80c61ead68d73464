"""The stage-RPC tensor codec (wire format of backends/portable/rpc.py:240-271
and protocol/schema.py:23-77) on the host: bytes identical to the format's
definition (the contiguous tensor's bytes in C order), round trips for every
wire dtype, and the reference's error messages."""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200.wire import WireMeta, tensor_from_wire, tensor_wire_parts

DTYPES = [torch.float32, torch.float16, torch.bfloat16, torch.int8, torch.int32, torch.int64]


@pytest.mark.parametrize("dtype", DTYPES)
def test_round_trip_and_bytes_on_host(dtype):
    g = torch.Generator().manual_seed(1)
    t = (torch.randn(3, 5, 7, generator=g) * 50).to(dtype)
    view = t.transpose(0, 2)  # non-contiguous: serialised in C order of the view
    meta, raw = tensor_wire_parts(view, "hidden")
    assert meta == WireMeta("hidden", {torch.float32: "float32", torch.float16: "float16",
                                       torch.bfloat16: "bfloat16", torch.int8: "int8",
                                       torch.int32: "int32", torch.int64: "int64"}[dtype], (7, 5, 3))
    assert raw == view.contiguous().view(torch.uint8).numpy().tobytes()
    back = tensor_from_wire(meta, raw)
    assert back.dtype == dtype and torch.equal(back, view)


def test_reference_style_metadata_is_accepted():
    class DType:  # the reference's DType is a str enum: .value holds the name
        value = "bfloat16"

    class Meta:
        tensor_id, dtype, shape, layout = "x", DType(), (2, 4), "contiguous"

    t = torch.arange(8, dtype=torch.float32).to(torch.bfloat16).view(2, 4)
    raw = t.view(torch.uint8).numpy().tobytes()
    assert torch.equal(tensor_from_wire(Meta(), raw), t)


def test_errors_match_the_reference():
    with pytest.raises(TypeError, match="RPC tensor must be torch.Tensor"):
        tensor_wire_parts([1, 2], "x")
    with pytest.raises(ValueError, match="non-empty and at most 256"):
        tensor_wire_parts(torch.zeros(2), "")
    with pytest.raises(ValueError, match="non-empty and at most 256"):
        tensor_wire_parts(torch.zeros(2), "x" * 257)
    with pytest.raises(ValueError, match="unsupported RPC tensor dtype"):
        tensor_wire_parts(torch.zeros(2, dtype=torch.float64), "x")
    with pytest.raises(ValueError, match="has 3 bytes; expected 8"):
        tensor_from_wire(WireMeta("x", "float32", (2,)), b"abc")
    with pytest.raises(ValueError, match="INT4"):
        tensor_from_wire(WireMeta("x", "int4", (2,)), b"ab")
    with pytest.raises(ValueError, match="shape dimension must be positive"):
        tensor_from_wire(WireMeta("x", "float32", (0,)), b"")
    with pytest.raises(ValueError, match="exceeds limit"):
        WireMeta("x", "float32", (1 << 28,)).validate()
