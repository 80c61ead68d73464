"""Stage weights: state-dict key names, seeded synthetic weights, RoPE tables.

Key names are those of the reference's stage modules: ``LlamaStage``
(models/llama_dense.py:325-337, layer indices local to the stage) and
``Qwen3Stage`` (models/qwen3_hf.py:107-135, which adds
``self_attn.q_norm`` / ``self_attn.k_norm``).  A full-model state dict uses
the same names with global layer indices.

Synthetic weights follow the benchmark recipe: every matrix N(0, 0.02), every
RMSNorm weight one.  Each tensor has its own generator, seeded from the seed
and the tensor's global name, so any stage's slice of a model is identical to
the same slice generated as part of the whole model, on any host.
"""
from __future__ import annotations

import os
import zlib
from collections.abc import Iterator

import torch

from gpu_mesh_b200.config import LlamaConfig

LAYER_MATRICES = (
    "self_attn.q_proj.weight",
    "self_attn.k_proj.weight",
    "self_attn.v_proj.weight",
    "self_attn.o_proj.weight",
    "mlp.gate_proj.weight",
    "mlp.up_proj.weight",
    "mlp.down_proj.weight",
)
LAYER_NORMS = ("input_layernorm.weight", "post_attention_layernorm.weight")
QK_NORMS = ("self_attn.q_norm.weight", "self_attn.k_norm.weight")


def layer_shapes(cfg: LlamaConfig) -> dict[str, tuple[int, ...]]:
    H, I, D = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    shapes = {
        "self_attn.q_proj.weight": (nq * D, H),
        "self_attn.k_proj.weight": (nkv * D, H),
        "self_attn.v_proj.weight": (nkv * D, H),
        "self_attn.o_proj.weight": (H, nq * D),
        "mlp.gate_proj.weight": (I, H),
        "mlp.up_proj.weight": (I, H),
        "mlp.down_proj.weight": (H, I),
        "input_layernorm.weight": (H,),
        "post_attention_layernorm.weight": (H,),
    }
    if cfg.qk_norm:
        shapes["self_attn.q_norm.weight"] = (D,)
        shapes["self_attn.k_norm.weight"] = (D,)
    return shapes


def stage_keys(
    cfg: LlamaConfig, layer_start: int, layer_end: int, has_embedding: bool, has_lm_head: bool
) -> Iterator[tuple[str, str, tuple[int, ...]]]:
    """Yield (local key, global key, shape) for one stage."""
    V, H = cfg.vocab_size, cfg.hidden_size
    if has_embedding:
        yield "embed_tokens.weight", "embed_tokens.weight", (V, H)
    for g in range(layer_start, layer_end):
        for name, shape in layer_shapes(cfg).items():
            yield f"layers.{g - layer_start}.{name}", f"layers.{g}.{name}", shape
    if has_lm_head:
        yield "norm.weight", "norm.weight", (H,)
        head = "embed_tokens.weight" if cfg.tie_word_embeddings else "lm_head.weight"
        yield "lm_head.weight", head, (V, H)


def _seed_for(seed: int, global_key: str) -> int:
    return (seed * 1_000_003 + zlib.crc32(global_key.encode())) % (2**63 - 1)


def synthetic_tensor(
    global_key: str,
    shape: tuple[int, ...],
    *,
    seed: int = 0,
    dtype: torch.dtype = torch.float32,
    device: torch.device | str = "cpu",
    std: float = 0.02,
) -> torch.Tensor:
    device = torch.device(device)
    if len(shape) == 1:
        return torch.ones(shape, dtype=dtype, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(_seed_for(seed, global_key))
    t = torch.empty(shape, dtype=torch.float32, device=device)
    t.normal_(0.0, std, generator=gen)
    return t.to(dtype)


# ---------------------------------------------------------------------------
# Device-independent N(0, std) weights
# ---------------------------------------------------------------------------
# torch's CPU and CUDA generators draw different normal streams, and drawing
# billions of normals on a host takes minutes.  The "portable" weights are a
# pure function of (seed, tensor name, element index) in integer arithmetic:
# a bijective 32-bit hash of the index picks one of 65536 equiprobable normal
# quantiles, so the same tensor comes out bit-identical on any host or GPU, and
# a GPU draws a whole model in well under a second.  The hash is two rounds of
# a xorshift-multiply finalizer (constants from Wellons' hash-prospector
# search); every step is a bijection mod 2^32.

_M32 = 0xFFFFFFFF
_MUL1, _MUL2 = 0x21F0AAAD, 0x735A2D97
_QUANTILES = 65536
_CHUNK = 1 << 24


def _portable_keys(seed: int, global_key: str) -> tuple[int, int]:
    h = zlib.crc32(global_key.encode())
    return (h + seed * 0x9E3779B9) & _M32, zlib.crc32(f"{seed}/{global_key}".encode()) & _M32


def _quantile_table(std: float, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    p = (torch.arange(_QUANTILES, dtype=torch.float64) + 0.5) / _QUANTILES
    return (torch.special.ndtri(p) * std).to(torch.float32).to(dtype).to(device)


def _mix_torch(x: torch.Tensor) -> torch.Tensor:
    # int64 holding values < 2^32; constants < 2^31, so products stay < 2^63
    x = x ^ (x >> 16)
    x = (x * _MUL1) & _M32
    x = x ^ (x >> 15)
    x = (x * _MUL2) & _M32
    return x ^ (x >> 15)


def _mix_numpy(x, tmp) -> None:
    import numpy as np

    np.right_shift(x, 16, out=tmp)
    x ^= tmp
    x *= np.uint32(_MUL1)  # uint32 arithmetic wraps mod 2^32
    np.right_shift(x, 15, out=tmp)
    x ^= tmp
    x *= np.uint32(_MUL2)
    np.right_shift(x, 15, out=tmp)
    x ^= tmp


def _portable_index_torch(n: int, k1: int, k2: int, device: torch.device) -> Iterator[tuple[int, torch.Tensor]]:
    for s in range(0, n, _CHUNK):
        m = min(_CHUNK, n - s)
        x = (torch.arange(s, s + m, dtype=torch.int64, device=device) + k1) & _M32
        yield s, _mix_torch(_mix_torch(x) ^ k2) >> 16


def _portable_cpu(n: int, k1: int, k2: int, table_bits):
    """Hash and table lookup in numpy uint32 arithmetic, chunks spread over threads."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    out = np.empty(n, dtype=table_bits.dtype)
    step, per_task = 1 << 18, 1 << 22

    def run(lo: int) -> None:
        x = np.empty(step, dtype=np.uint32)
        tmp = np.empty(step, dtype=np.uint32)
        base = np.arange(step, dtype=np.uint32)
        for s in range(lo, min(lo + per_task, n), step):
            m = min(step, n - s, lo + per_task - s)
            np.add(base[:m], np.uint32((s + k1) & _M32), out=x[:m])
            _mix_numpy(x[:m], tmp[:m])
            x[:m] ^= np.uint32(k2)
            _mix_numpy(x[:m], tmp[:m])
            np.right_shift(x[:m], 16, out=tmp[:m])
            np.take(table_bits, tmp[:m], out=out[s : s + m])

    with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as pool:
        list(pool.map(run, range(0, n, per_task)))
    return out


def portable_quantile_index(n: int, seed: int, global_key: str, device: torch.device | str = "cpu") -> torch.Tensor:
    """The 16-bit quantile index of elements 0..n-1 of a tensor (int64 [n])."""
    device = torch.device(device)
    if n >= 1 << 32:
        raise ValueError("portable weights cover tensors of fewer than 2^32 elements")
    k1, k2 = _portable_keys(seed, global_key)
    if device.type == "cpu":
        import numpy as np

        return torch.from_numpy(_portable_cpu(n, k1, k2, np.arange(_QUANTILES, dtype=np.int64)))
    out = torch.empty(n, dtype=torch.int64, device=device)
    for s, idx in _portable_index_torch(n, k1, k2, device):
        out[s : s + idx.numel()] = idx
    return out


def portable_tensor(
    global_key: str,
    shape: tuple[int, ...],
    *,
    seed: int = 0,
    dtype: torch.dtype = torch.float32,
    device: torch.device | str = "cpu",
    std: float = 0.02,
) -> torch.Tensor:
    """N(0, std) weights (norm vectors one) that are bit-identical on every device."""
    device = torch.device(device)
    if len(shape) == 1:
        return torch.ones(shape, dtype=dtype, device=device)
    n = 1
    for d in shape:
        n *= d
    if n >= 1 << 32:
        raise ValueError("portable weights cover tensors of fewer than 2^32 elements")
    k1, k2 = _portable_keys(seed, global_key)
    table = _quantile_table(std, dtype, torch.device("cpu"))
    if device.type == "cpu":
        bits = {2: torch.int16, 4: torch.int32, 8: torch.int64}[table.element_size()]
        got = _portable_cpu(n, k1, k2, table.view(bits).numpy())
        return torch.from_numpy(got).view(dtype).view(shape)
    table = table.to(device)
    out = torch.empty(n, dtype=dtype, device=device)
    for s, idx in _portable_index_torch(n, k1, k2, device):
        out[s : s + idx.numel()] = table[idx]
    return out.view(shape)


def synthetic_stage_state(
    cfg: LlamaConfig,
    layer_start: int,
    layer_end: int,
    *,
    has_embedding: bool,
    has_lm_head: bool,
    seed: int = 0,
    dtype: torch.dtype = torch.float32,
    device: torch.device | str = "cpu",
    method: str = "normal",
) -> dict[str, torch.Tensor]:
    """Seeded synthetic weights of one stage, with the stage's local key names.

    ``method="normal"`` draws every matrix from torch's generator on
    ``device``; ``"portable"`` uses the device-independent quantile weights
    (``portable_tensor``), identical on any host or GPU.
    """
    make = {"normal": synthetic_tensor, "portable": portable_tensor}.get(method)
    if make is None:
        raise ValueError(f"unknown synthetic weight method {method!r}")
    out: dict[str, torch.Tensor] = {}
    cache: dict[str, torch.Tensor] = {}
    for local, global_key, shape in stage_keys(cfg, layer_start, layer_end, has_embedding, has_lm_head):
        if global_key not in cache:
            cache[global_key] = make(global_key, shape, seed=seed, dtype=dtype, device=device)
        out[local] = cache[global_key]
    return out


def synthetic_model_state(
    cfg: LlamaConfig, *, seed: int = 0, dtype: torch.dtype = torch.float32, device="cpu",
    method: str = "normal",
) -> dict[str, torch.Tensor]:
    """Whole-model weights with global key names (a one-stage state dict)."""
    return synthetic_stage_state(
        cfg, 0, cfg.num_hidden_layers, has_embedding=True, has_lm_head=True,
        seed=seed, dtype=dtype, device=device, method=method,
    )


def slice_stage_state(
    full: dict[str, torch.Tensor], layer_start: int, layer_end: int, *,
    has_embedding: bool, has_lm_head: bool, tie_word_embeddings: bool = False,
) -> dict[str, torch.Tensor]:
    """Cut one stage out of a whole-model state dict (global names -> local names)."""
    out: dict[str, torch.Tensor] = {}
    for g in range(layer_start, layer_end):
        prefix = f"layers.{g}."
        for key, value in full.items():
            if key.startswith(prefix):
                out[f"layers.{g - layer_start}." + key[len(prefix):]] = value
    if has_embedding:
        out["embed_tokens.weight"] = full["embed_tokens.weight"]
    if has_lm_head:
        out["norm.weight"] = full["norm.weight"]
        if "lm_head.weight" in full:
            out["lm_head.weight"] = full["lm_head.weight"]
        elif tie_word_embeddings:
            out["lm_head.weight"] = full["embed_tokens.weight"]
    return out


def rope_tables(
    head_dim: int, max_positions: int, theta: float, dtype: torch.dtype, *, round_inv_freq: bool = False
) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_positions, head_dim/2] on the host, cast to the activation dtype.

    Formula of _precompute_freqs (models/llama_dense.py:96-104), which HF's
    default Qwen3 rotary embedding shares; the cast matches
    ``self.rope_cos.to(x.dtype)`` (llama_dense.py:431-432).
    ``round_inv_freq``: the HF Qwen3 stage keeps the inverse frequencies as a
    module buffer, and Qwen3Stage casts the whole module to the stage dtype
    (models/qwen3_hf.py:139-140), so a bf16 Qwen3 stage rotates with
    frequencies rounded to bf16 (the angles are then formed in fp32,
    Qwen3RotaryEmbedding.forward).
    """
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    if round_inv_freq:
        inv = inv.to(dtype).float()
    t = torch.arange(max_positions).float()
    freqs = torch.outer(t, inv)
    return freqs.cos().to(dtype), freqs.sin().to(dtype)
