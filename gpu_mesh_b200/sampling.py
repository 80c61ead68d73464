"""Token sampling on the device (inference/sampling.py of the reference).

``greedy_sample`` and ``top_p_sample`` take CUDA logits [..., V] and run the
library's kernels; they accept exactly the reference's arguments.  Top-p
draws one uniform number per row from ``generator`` (a seeded CPU generator
gives reproducible tokens on any device) and returns the token at which the
renormalised nucleus's cumulative probability first exceeds it, with tied
probabilities ordered by token index.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from gpu_mesh_b200 import _lib

_DT = {torch.float32: _lib.MG_DTYPE_F32, torch.bfloat16: _lib.MG_DTYPE_BF16}


@dataclass
class SamplingParams:
    """Sampling parameters with the reference's validation (sampling.py:11-42)."""

    temperature: float = 0.0
    top_p: float = 1.0
    eos_token_id: int | None = None
    seed: int | None = None

    def __post_init__(self) -> None:
        if (
            isinstance(self.temperature, bool)
            or not isinstance(self.temperature, (int, float))
            or not math.isfinite(float(self.temperature))
            or self.temperature < 0
        ):
            raise ValueError("temperature must be a finite non-negative number")
        if (
            isinstance(self.top_p, bool)
            or not isinstance(self.top_p, (int, float))
            or not math.isfinite(float(self.top_p))
            or not 0 <= self.top_p <= 1
        ):
            raise ValueError("top_p must be a finite number in [0, 1]")
        if self.eos_token_id is not None and (
            isinstance(self.eos_token_id, bool)
            or not isinstance(self.eos_token_id, int)
            or self.eos_token_id < 0
        ):
            raise ValueError("eos_token_id must be a non-negative integer or None")
        if self.seed is not None and (isinstance(self.seed, bool) or not isinstance(self.seed, int)):
            raise TypeError("seed must be an integer or None")


def make_sampling_generator(params: SamplingParams, *, device: torch.device | str = "cpu") -> torch.Generator | None:
    if params.seed is None:
        return None
    generator = torch.Generator(device=device)
    generator.manual_seed(params.seed)
    return generator


def _rows(logits: torch.Tensor) -> tuple[torch.Tensor, tuple[int, ...]]:
    if logits.device.type != "cuda":
        raise ValueError("B200 sampling needs CUDA logits")
    if logits.dtype not in _DT:
        logits = logits.float()
    lead = tuple(logits.shape[:-1])
    flat = logits.reshape(-1, logits.shape[-1])
    if flat.stride(-1) != 1:
        flat = flat.contiguous()
    return flat, lead


def greedy_sample(logits: torch.Tensor) -> torch.Tensor:
    """Argmax over the last dimension, lowest index on ties (sampling.py:58-60)."""
    flat, lead = _rows(logits)
    ids = torch.empty(flat.shape[0], dtype=torch.int64, device=flat.device)
    with torch.cuda.device(flat.device):  # the kernel runs on the logits' GPU, on its current stream
        _lib.check(
            _lib.lib().mg_sample_greedy(
                flat.data_ptr(), _DT[flat.dtype], flat.shape[0], flat.shape[1], flat.stride(0),
                ids.data_ptr(), torch.cuda.current_stream(flat.device).cuda_stream,
            )
        )
    return ids.reshape(lead)


def top_p_sample(
    logits: torch.Tensor,
    temperature: float,
    top_p: float,
    *,
    generator: torch.Generator | None = None,
    uniforms: torch.Tensor | None = None,
) -> torch.Tensor:
    """Nucleus sampling (sampling.py:63-95); ``uniforms`` overrides the draw."""
    if not math.isfinite(temperature) or temperature < 0:
        raise ValueError("temperature must be a finite non-negative number")
    if not math.isfinite(top_p) or not 0 <= top_p <= 1:
        raise ValueError("top_p must be a finite number in [0, 1]")
    if temperature <= 0:
        return greedy_sample(logits)
    flat, lead = _rows(logits)
    rows = flat.shape[0]
    if uniforms is None:
        gen_device = generator.device if generator is not None else torch.device("cpu")
        uniforms = torch.rand(rows, generator=generator, device=gen_device)
    uniforms = uniforms.to(device=flat.device, dtype=torch.float32).reshape(rows).contiguous()
    ids = torch.empty(rows, dtype=torch.int64, device=flat.device)
    with torch.cuda.device(flat.device):
        _lib.check(
            _lib.lib().mg_sample_top_p(
                flat.data_ptr(), _DT[flat.dtype], rows, flat.shape[1], flat.stride(0),
                float(temperature), float(top_p), uniforms.data_ptr(), ids.data_ptr(),
                torch.cuda.current_stream(flat.device).cuda_stream,
            )
        )
    return ids.reshape(lead)
