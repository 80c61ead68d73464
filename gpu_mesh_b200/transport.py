"""Stage-boundary transport between GPUs of one host.

Mirrors the reference's ``move_boundary`` / ``probe_cuda_path``
(src/meshgpu/transport/local_cuda.py:27-90): ``cpu`` forces a host hop,
``local_cuda`` keeps the tensor on device and uses a peer copy over NVLink
when the pair has peer access (every B200 pair on an NVSwitch box), else an
explicit host staging copy.  Multi-process pipelines move boundaries with
NCCL instead (``gpu_mesh_b200.dist``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class CudaPath:
    source: torch.device
    destination: torch.device
    mode: str  # same_device, peer, host_fallback, non_cuda
    peer_access: bool = False


def _resolve(device: torch.device) -> torch.device:
    if device.type != "cuda" or device.index is not None:
        return device
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return device


def probe_cuda_path(source: torch.device, destination: torch.device) -> CudaPath:
    source = _resolve(torch.device(source))
    destination = _resolve(torch.device(destination))
    if source == destination:
        return CudaPath(source, destination, "same_device", peer_access=True)
    if source.type != "cuda" or destination.type != "cuda":
        return CudaPath(source, destination, "non_cuda", peer_access=False)
    if not torch.cuda.is_available():
        return CudaPath(source, destination, "host_fallback", peer_access=False)
    try:
        peer = bool(torch.cuda.can_device_access_peer(source.index or 0, destination.index or 0))
    except (RuntimeError, TypeError, AttributeError):
        peer = False
    return CudaPath(source, destination, "peer" if peer else "host_fallback", peer_access=peer)


def move_boundary(tensor: torch.Tensor, destination: torch.device, *, transport: str = "cpu") -> torch.Tensor:
    destination = _resolve(torch.device(destination))
    if transport not in {"cpu", "local_cuda"}:
        raise ValueError(f"unsupported local boundary transport: {transport!r}")
    if tensor.device == destination:
        return tensor
    if transport == "cpu":
        return tensor.detach().to("cpu").to(destination)
    path = probe_cuda_path(tensor.device, destination)
    if path.mode == "peer":
        return tensor.to(destination, non_blocking=True)
    if path.mode == "host_fallback":
        return tensor.detach().to("cpu").to(destination)
    return tensor.to(destination)


def boundary_transport_name(source: torch.device, destination: torch.device) -> str:
    return probe_cuda_path(source, destination).mode
