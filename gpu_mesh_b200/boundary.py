"""Stage boundaries between GPUs of one process.

The reference hands a stage's output to the next stage with ``Tensor.to``
on the caller's stream (transport/local_cuda.py:27-90), so the copy sits in
the compute stream of both devices.  Here every (producer device, receiver
device) pair has a ``Link`` with a side stream on the producer's device, and
a hand-off never blocks a compute stream or the host:

1. an event on the producer's stream marks the output as written;
2. the receive buffer comes from the receiver's allocator on the receiver's
   stream, and an event on that stream marks its memory free of earlier users;
3. the side stream waits for both events and queues ``mg_peer_copy``
   (cudaMemcpyPeerAsync: straight over NVLink once the library has enabled
   peer access for the pair);
4. the receiver's stream waits for an event recorded after the copy;
5. the producer's tensor is marked in use by the side stream
   (``record_stream``), so its allocator cannot hand the memory out again
   before the copy has read it.

``transport="cpu"`` keeps the reference's forced host hop.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from gpu_mesh_b200 import _lib

TRANSPORTS = ("cpu", "local_cuda")


def _resolve(device: torch.device | str | int) -> torch.device:
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        return torch.device("cuda", torch.cuda.current_device())
    return device


class Link:
    """One direction of a boundary between two GPUs of this process."""

    _links: dict[tuple[int, int], "Link"] = {}
    _lock = threading.Lock()

    def __init__(self, src: torch.device, dst: torch.device) -> None:
        self.src, self.dst = src, dst
        self.stream = torch.cuda.Stream(device=src)
        enabled = ctypes.c_int32()
        _lib.check(_lib.lib().mg_peer_access(src.index, dst.index, ctypes.byref(enabled)))
        if enabled.value:  # the copy engine of either side may touch the other's memory
            back = ctypes.c_int32()
            _lib.check(_lib.lib().mg_peer_access(dst.index, src.index, ctypes.byref(back)))
        self.peer = bool(enabled.value)

    @classmethod
    def between(cls, src: torch.device, dst: torch.device) -> "Link":
        key = (src.index, dst.index)
        with cls._lock:
            link = cls._links.get(key)
            if link is None:
                link = cls._links[key] = cls(src, dst)
            return link

    def send(self, tensor: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Queue ``tensor`` (on ``src``) into a buffer on ``dst``; the result is
        ready for work queued later on ``dst``'s current stream."""
        src_stream = torch.cuda.current_stream(self.src)
        dst_stream = torch.cuda.current_stream(self.dst)
        tensor = tensor.detach().contiguous()
        written = torch.cuda.Event()
        written.record(src_stream)
        if out is None:
            with torch.cuda.device(self.dst):
                out = torch.empty(tensor.shape, dtype=tensor.dtype, device=self.dst)
        elif out.shape != tensor.shape or out.dtype != tensor.dtype or not out.is_contiguous():
            raise ValueError("receive buffer does not match the tensor sent")
        free = torch.cuda.Event()
        free.record(dst_stream)
        self.stream.wait_event(written)
        self.stream.wait_event(free)
        _lib.check(_lib.lib().mg_peer_copy(
            out.data_ptr(), self.dst.index, tensor.data_ptr(), self.src.index,
            tensor.numel() * tensor.element_size(), self.stream.cuda_stream,
        ))
        tensor.record_stream(self.stream)
        arrived = torch.cuda.Event()
        arrived.record(self.stream)
        dst_stream.wait_event(arrived)
        return out


def move_to_stage(tensor: torch.Tensor, device: torch.device | str, *, transport: str = "cpu") -> torch.Tensor:
    """Hand a boundary tensor to the stage on ``device``.

    ``cpu`` hops through host memory as the reference's portable transport
    does; ``local_cuda`` keeps it on the GPUs: a link's side-stream copy
    between two devices, no copy on the same device.
    """
    if transport not in TRANSPORTS:
        raise ValueError(f"unsupported local boundary transport: {transport!r}")
    device = _resolve(device)
    if tensor.device == device:
        return tensor
    if transport == "cpu" or tensor.device.type != "cuda" or device.type != "cuda":
        return tensor.detach().to("cpu").to(device)
    return Link.between(tensor.device, device).send(tensor)
