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
) -> dict[str, torch.Tensor]:
    """Seeded synthetic weights of one stage, with the stage's local key names."""
    out: dict[str, torch.Tensor] = {}
    cache: dict[str, torch.Tensor] = {}
    for local, global_key, shape in stage_keys(cfg, layer_start, layer_end, has_embedding, has_lm_head):
        if global_key not in cache:
            cache[global_key] = synthetic_tensor(global_key, shape, seed=seed, dtype=dtype, device=device)
        out[local] = cache[global_key]
    return out


def synthetic_model_state(
    cfg: LlamaConfig, *, seed: int = 0, dtype: torch.dtype = torch.float32, device="cpu"
) -> dict[str, torch.Tensor]:
    """Whole-model weights with global key names (a one-stage state dict)."""
    return synthetic_stage_state(
        cfg, 0, cfg.num_hidden_layers, has_embedding=True, has_lm_head=True,
        seed=seed, dtype=dtype, device=device,
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
    head_dim: int, max_positions: int, theta: float, dtype: torch.dtype
) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_positions, head_dim/2] on the host, cast to the activation dtype.

    Formula of _precompute_freqs (models/llama_dense.py:96-104), which HF's
    default Qwen3 rotary embedding shares; the cast matches
    ``self.rope_cos.to(x.dtype)`` (llama_dense.py:431-432).
    """
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    t = torch.arange(max_positions).float()
    freqs = torch.outer(t, inv)
    return freqs.cos().to(dtype), freqs.sin().to(dtype)
