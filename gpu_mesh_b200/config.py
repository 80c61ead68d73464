"""Model configuration of a stage.

``LlamaConfig`` keeps the field names, defaults and validation messages of the
reference's config (src/meshgpu/models/llama_dense.py:20-78), so code written
against the reference constructs it unchanged.  Two fields are added for the
Qwen3 architecture (models/qwen3_hf.py): ``qk_norm`` (per-head RMSNorm on q
and k before RoPE) and ``mask_policy`` (HF's cache-index causal mask).
:func:`config_from` converts a reference ``LlamaConfig`` or an HF
``Qwen3Config`` into this type.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

from gpu_mesh_b200 import _lib


@dataclass
class LlamaConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    max_position_embeddings: int
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    tie_word_embeddings: bool = False
    attention_implementation: str = "sdpa"
    qk_norm: bool = False
    mask_policy: str = "llama"  # "llama" (position-based) or "cache" (HF Qwen3)

    def __post_init__(self) -> None:
        positive = {
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim,
            "max_position_embeddings": self.max_position_embeddings,
        }
        for name, value in positive.items():
            if isinstance(value, bool) or not isinstance(value, int):
                raise TypeError(f"{name} must be an integer, got {type(value).__name__}")
            if value < 1:
                raise ValueError(f"{name} must be positive, got {value}")
        if self.num_attention_heads % self.num_key_value_heads != 0:
            raise ValueError(
                "num_attention_heads must be divisible by num_key_value_heads "
                f"({self.num_attention_heads} % {self.num_key_value_heads} != 0)"
            )
        if self.num_key_value_heads > self.num_attention_heads:
            raise ValueError("num_key_value_heads must not exceed num_attention_heads")
        if self.head_dim % 2 != 0:
            raise ValueError(f"head_dim must be even for rotary embeddings, got {self.head_dim}")
        for name in ("rms_norm_eps", "rope_theta"):
            value = getattr(self, name)
            if (
                isinstance(value, bool)
                or not isinstance(value, (int, float))
                or not math.isfinite(float(value))
                or value <= 0
            ):
                raise ValueError(f"{name} must be positive")
        if self.attention_implementation not in {"eager", "sdpa"}:
            raise ValueError(
                "attention_implementation must be 'eager' or 'sdpa', got "
                f"{self.attention_implementation!r}"
            )
        if self.mask_policy not in {"llama", "cache"}:
            raise ValueError(f"mask_policy must be 'llama' or 'cache', got {self.mask_policy!r}")

    @property
    def attention_impl_code(self) -> int:
        if self.mask_policy == "cache":
            return _lib.MG_ATTN_CACHE_CAUSAL
        if self.attention_implementation == "eager":
            return _lib.MG_ATTN_EAGER
        return _lib.MG_ATTN_SDPA


def _rope_theta(cfg: Any) -> float:
    theta = getattr(cfg, "rope_theta", None)
    if theta is None:
        params = getattr(cfg, "rope_parameters", None) or getattr(cfg, "rope_scaling", None) or {}
        rope_type = params.get("rope_type", "default")
        if rope_type != "default":
            raise ValueError(f"only default RoPE is supported, got rope_type={rope_type!r}")
        theta = params.get("rope_theta")
    if theta is None:
        raise ValueError("config has no rope_theta")
    return float(theta)


def config_from(cfg: Any) -> LlamaConfig:
    """Accept this package's config, the reference's LlamaConfig or an HF Qwen3Config."""
    if isinstance(cfg, LlamaConfig):
        return cfg
    model_type = getattr(cfg, "model_type", None)
    if model_type == "qwen3":
        if getattr(cfg, "attention_bias", False):
            raise ValueError("Qwen3 attention bias is not supported")
        if getattr(cfg, "use_sliding_window", False):
            raise ValueError("Qwen3 sliding-window attention is not supported")
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        return LlamaConfig(
            vocab_size=int(cfg.vocab_size),
            hidden_size=int(cfg.hidden_size),
            intermediate_size=int(cfg.intermediate_size),
            num_hidden_layers=int(cfg.num_hidden_layers),
            num_attention_heads=int(cfg.num_attention_heads),
            num_key_value_heads=int(cfg.num_key_value_heads),
            head_dim=int(head_dim),
            max_position_embeddings=int(cfg.max_position_embeddings),
            rms_norm_eps=float(cfg.rms_norm_eps),
            rope_theta=_rope_theta(cfg),
            tie_word_embeddings=bool(getattr(cfg, "tie_word_embeddings", False)),
            qk_norm=True,
            mask_policy="cache",
        )
    return LlamaConfig(
        vocab_size=cfg.vocab_size,
        hidden_size=cfg.hidden_size,
        intermediate_size=cfg.intermediate_size,
        num_hidden_layers=cfg.num_hidden_layers,
        num_attention_heads=cfg.num_attention_heads,
        num_key_value_heads=cfg.num_key_value_heads,
        head_dim=cfg.head_dim,
        max_position_embeddings=cfg.max_position_embeddings,
        rms_norm_eps=cfg.rms_norm_eps,
        rope_theta=cfg.rope_theta,
        tie_word_embeddings=getattr(cfg, "tie_word_embeddings", False),
        attention_implementation=getattr(cfg, "attention_implementation", "sdpa"),
    )


def split_layers(n_layers: int, n_stages: int) -> list[tuple[int, int]]:
    """Contiguous [start, end) ranges, remainder to the first stages.

    Same partition as build_pipeline (backends/portable/pipeline.py:67-74) and
    split_layers (artifacts/hf_import.py:231-248).
    """
    if n_stages < 1 or n_stages > n_layers:
        raise ValueError(f"num_stages must be in [1, {n_layers}], got {n_stages}")
    base, rem = divmod(n_layers, n_stages)
    ranges = []
    start = 0
    for i in range(n_stages):
        end = start + base + (1 if i < rem else 0)
        ranges.append((start, end))
        start = end
    return ranges


def balanced_layer_ranges(
    cfg: "LlamaConfig", n_stages: int, *, rows: int, context: int, bytes_per_elem: int = 2
) -> list[tuple[int, int]]:
    """Contiguous layer ranges that even out what each stage streams per decode
    step, for ``build_pipeline(layer_ranges=...)`` (the planner's ranges in the
    reference's artifacts, hf_import.py:860-1050, are honoured the same way).

    A layer costs its weights plus the K and V its ``rows`` read at ``context``
    cached positions; the last stage also streams the lm_head (the embedding
    is a gather and costs nothing).  The split minimises the largest stage
    (exact dynamic programme over the contiguous splits)."""
    L = cfg.num_hidden_layers
    if n_stages < 1 or n_stages > L:
        raise ValueError(f"num_stages must be in [1, {L}], got {n_stages}")
    H, I, D = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    layer = (H * (nq + 2 * nkv) * D + nq * D * H + 3 * H * I + 2 * rows * context * nkv * D) * bytes_per_elem
    head = cfg.vocab_size * H * bytes_per_elem
    inf = float("inf")
    # best[s][j]: the smallest possible largest stage when stages 0..s-1 hold layers [0, j)
    best = [[inf] * (L + 1) for _ in range(n_stages + 1)]
    cut = [[0] * (L + 1) for _ in range(n_stages + 1)]
    best[0][0] = 0.0
    for s in range(1, n_stages + 1):
        for j in range(s, L - (n_stages - s) + 1):
            for i in range(s - 1, j):
                cost = (j - i) * layer + (head if s == n_stages else 0)
                v = max(best[s - 1][i], cost)
                if v < best[s][j]:
                    best[s][j], cut[s][j] = v, i
    ranges, j = [], L
    for s in range(n_stages, 0, -1):
        i = cut[s][j]
        ranges.append((i, j))
        j = i
    return ranges[::-1]
