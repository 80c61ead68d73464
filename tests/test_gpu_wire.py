"""The stage-RPC tensor codec with CUDA tensors: the pinned-memory path sends
the same bytes as the host path and restores the tensor on the device, for a
decode boundary (8 rows x 4096) and a prefill boundary (8 x 1024 x 4096)."""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200.wire import tensor_from_wire, tensor_wire_parts

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("shape", [(8, 1, 4096), (8, 1024, 4096)], ids=["decode", "prefill"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.int64])
def test_device_round_trip_matches_host_bytes(shape, dtype):
    g = torch.Generator(device=DEV).manual_seed(5)
    t = (torch.randn(*shape, generator=g, device=DEV) * 100).to(dtype)
    meta, raw = tensor_wire_parts(t, "hidden")
    assert raw == t.cpu().view(torch.uint8).numpy().tobytes()
    back = tensor_from_wire(meta, raw, device=DEV)
    assert back.device == t.device and back.dtype == dtype
    assert torch.equal(back, t)
    for _ in range(3):  # pooled buffers are reused, copies stay ordered
        t2 = t + 1
        m2, r2 = tensor_wire_parts(t2, "hidden")
        assert torch.equal(tensor_from_wire(m2, r2, device=DEV), t2)
