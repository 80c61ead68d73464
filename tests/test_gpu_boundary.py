"""Stage boundaries between two GPUs of one process (gpu_mesh_b200.boundary):
a side-stream peer copy ordered by events lands exactly the bytes sent, in
both directions, while both devices' streams keep working on other tensors."""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200.boundary import Link, move_to_stage

pytestmark = pytest.mark.gpu


def _two():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    return torch.device("cuda", 0), torch.device("cuda", 1)


@pytest.mark.parametrize("direction", ["0to1", "1to0"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.int64, torch.float32])
def test_link_delivers_the_bytes_in_order(direction, dtype):
    a, b = _two()
    src, dst = (a, b) if direction == "0to1" else (b, a)
    link = Link.between(src, dst)
    g = torch.Generator(device=src).manual_seed(3)
    outs, wants = [], []
    for i in range(8):  # a chain of hand-offs, each written just before it is sent
        x = torch.randint(-1000, 1000, (8, 3, 512), generator=g, device=src).to(dtype)
        x.mul_(2)  # the producer's last kernel, on the source's current stream
        wants.append(x.cpu())
        y = link.send(x)
        y.add_(0)  # a consumer kernel on the destination's current stream
        outs.append(y)
        del x  # the allocator may reuse the memory at once: record_stream keeps it safe
    torch.cuda.synchronize(src)
    torch.cuda.synchronize(dst)
    for y, want in zip(outs, wants):
        assert y.device == dst and torch.equal(y.cpu(), want)


def test_move_to_stage_on_one_device_is_free():
    a, _ = _two()
    x = torch.ones(4, 4, device=a)
    assert move_to_stage(x, a, transport="local_cuda") is x
