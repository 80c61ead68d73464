"""Stage-boundary tensors to and from the stage-RPC wire format through pinned memory.

The wire format is the reference's (backends/portable/rpc.py:240-271,
protocol/schema.py:23-77): a tensor travels as metadata (tensor id, dtype
name, shape, contiguous layout) plus its bytes in C order.  The reference
moves a CUDA tensor to pageable host memory (``.to("cpu")``) and serialises
that, and on receipt builds a CPU tensor that the stage then copies to its
GPU.  Here the sender copies device memory straight into a pinned staging
buffer (one asynchronous copy on a side stream, ordered after the producing
stream by an event), and the receiver copies the bytes into a pinned buffer
and from there to the device without blocking the host.  Staging buffers are
pooled per size, so a decode loop does not allocate pinned memory per
message.  The bytes on the wire are identical to the reference's.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

MAX_ID_LENGTH = 256                    # backends/portable/rpc.py:69
MAX_TENSOR_BYTES = 512 * 1024 * 1024   # protocol/schema.py:11

_DTYPES = {
    "float32": torch.float32,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "int8": torch.int8,
    "int32": torch.int32,
    "int64": torch.int64,
}
_NAMES = {v: k for k, v in _DTYPES.items()}
_ITEMSIZE = {"float32": 4, "float16": 2, "bfloat16": 2, "int8": 1, "int4": 1, "int32": 4, "int64": 8}


@dataclass(frozen=True)
class WireMeta:
    """Tensor metadata of the wire format (protocol/schema.py:49-77)."""

    tensor_id: str
    dtype: str
    shape: tuple[int, ...]
    layout: str = "contiguous"

    @property
    def byte_length(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n * _ITEMSIZE[self.dtype]

    def validate(self) -> None:
        if not isinstance(self.tensor_id, str) or not self.tensor_id:
            raise ValueError("tensor_id must not be empty")
        if self.dtype not in _ITEMSIZE:
            raise TypeError(f"dtype must be a DType, got {self.dtype!r}")
        if self.dtype == "int4":
            raise ValueError(
                "INT4 wire tensors are unsupported until an explicit packed-byte encoding is implemented"
            )
        if not self.shape:
            raise ValueError("shape must not be empty")
        for d in self.shape:
            if isinstance(d, bool) or not isinstance(d, int):
                raise TypeError(f"shape dimensions must be integers, got {type(d).__name__}")
            if d <= 0:
                raise ValueError(f"shape dimension must be positive, got {d}")
        if self.byte_length > MAX_TENSOR_BYTES:
            raise ValueError(f"tensor byte_length {self.byte_length} exceeds limit {MAX_TENSOR_BYTES}")
        if self.layout != "contiguous":
            raise ValueError(f"unsupported layout: {self.layout!r}")

    @classmethod
    def of(cls, meta: Any) -> WireMeta:
        """This type from itself or from the reference's TensorMeta (whose
        dtype is a str enum)."""
        if isinstance(meta, WireMeta):
            return meta
        dtype = getattr(meta.dtype, "value", meta.dtype)
        return cls(meta.tensor_id, str(dtype), tuple(meta.shape), getattr(meta, "layout", "contiguous"))


class PinnedPool:
    """Reusable pinned host buffers, one free list per power-of-two size.

    A buffer still read by an asynchronous copy is returned with the event
    that completes the copy and becomes free once the event has.
    """

    def __init__(self) -> None:
        self._free: dict[int, list[torch.Tensor]] = {}
        self._busy: list[tuple[torch.cuda.Event, torch.Tensor]] = []
        self._lock = threading.Lock()

    def take(self, nbytes: int) -> torch.Tensor:
        size = 1 << max(12, (nbytes - 1).bit_length())
        with self._lock:
            still = []
            for ev, buf in self._busy:
                if ev.query():
                    self._free.setdefault(buf.numel(), []).append(buf)
                else:
                    still.append((ev, buf))
            self._busy = still
            free = self._free.get(size)
            if free:
                return free.pop()
        return torch.empty(size, dtype=torch.uint8, pin_memory=True)

    def give(self, buf: torch.Tensor, after: torch.cuda.Event | None = None) -> None:
        with self._lock:
            if after is None:
                self._free.setdefault(buf.numel(), []).append(buf)
            else:
                self._busy.append((after, buf))


_POOL = PinnedPool()
_STREAMS: dict[int, torch.cuda.Stream] = {}


def _side_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _STREAMS:
        _STREAMS[idx] = torch.cuda.Stream(device=idx)
    return _STREAMS[idx]


def tensor_wire_parts(tensor: torch.Tensor, tensor_id: str, *, pool: PinnedPool | None = None) -> tuple[WireMeta, bytes]:
    """(metadata, bytes) of a tensor for the wire (rpc.py:240-258).

    A CUDA tensor is copied device -> pinned host on a side stream that first
    waits for the current stream's work on it; the bytes are then read out of
    the pinned buffer.
    """
    if not isinstance(tensor, torch.Tensor):
        raise TypeError(f"RPC tensor must be torch.Tensor, got {type(tensor).__name__}")
    if not tensor_id or len(tensor_id) > MAX_ID_LENGTH:
        raise ValueError("RPC tensor_id must be non-empty and at most 256 characters")
    if tensor.dtype not in _NAMES:
        raise ValueError(f"unsupported RPC tensor dtype: {tensor.dtype}")
    t = tensor.detach()
    meta = WireMeta(tensor_id, _NAMES[t.dtype], tuple(int(d) for d in t.shape))
    meta.validate()
    n = meta.byte_length
    if t.device.type != "cuda":
        raw = t.contiguous().view(torch.uint8).numpy().tobytes()
    else:
        pool = pool or _POOL
        src = t.contiguous().view(-1).view(torch.uint8)
        buf = pool.take(n)
        try:
            side = _side_stream(t.device)
            side.wait_stream(torch.cuda.current_stream(t.device))
            with torch.cuda.stream(side):
                buf[:n].copy_(src, non_blocking=True)
            src.record_stream(side)
            side.synchronize()
            raw = buf[:n].numpy().tobytes()
        finally:
            pool.give(buf)
    if len(raw) != n:
        raise RuntimeError(f"serialized tensor has {len(raw)} bytes; metadata declares {n}")
    return meta, raw


def tensor_from_wire(meta: Any, raw: bytes | bytearray | memoryview, *, device: torch.device | str | None = None,
                     pool: PinnedPool | None = None) -> torch.Tensor:
    """The tensor a (metadata, bytes) pair describes (rpc.py:261-271), on
    ``device`` (default CPU).

    For a CUDA device the bytes go into a pinned buffer and are copied to the
    device asynchronously on the current stream; the pinned buffer returns to
    the pool once that copy has completed.
    """
    meta = WireMeta.of(meta)
    meta.validate()
    n = meta.byte_length
    if len(raw) != n:
        raise ValueError(f"tensor {meta.tensor_id!r} has {len(raw)} bytes; expected {n}")
    dtype = _DTYPES[meta.dtype]
    dev = torch.device(device) if device is not None else torch.device("cpu")
    if dev.type != "cuda":
        return torch.frombuffer(bytearray(raw), dtype=dtype).reshape(meta.shape).clone()
    pool = pool or _POOL
    buf = pool.take(n)
    buf[:n].numpy()[:] = np.frombuffer(raw, dtype=np.uint8, count=n)
    out = torch.empty(n, dtype=torch.uint8, device=dev)
    out.copy_(buf[:n], non_blocking=True)
    done = torch.cuda.Event()
    done.record(torch.cuda.current_stream(dev))
    pool.give(buf, after=done)
    return out.view(dtype).reshape(meta.shape)
