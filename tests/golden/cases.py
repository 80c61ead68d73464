"""Golden-vector cases shared by the generator (make_golden.py) and the tests.

Each case fixes a model geometry, a stage split, a dtype and a seeded prompt.
Weights are the seeded synthetic weights of ``gpu_mesh_b200.weights`` (every
matrix N(0, 0.02), norms one), generated on the CPU, so the reference, the
oracle and the CUDA path all see identical tensors.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from gpu_mesh_b200.config import LlamaConfig

SKETCH_STRIDE = 101  # logits[..., ::101] is stored for every step
TOPK = 8


@dataclass
class Case:
    name: str
    arch: str  # "llama" or "qwen3"
    cfg: dict
    stages: int
    dtype: torch.dtype
    batch: int
    prompt: int
    steps: int
    seed: int = 0
    extra: dict = field(default_factory=dict)

    def config(self) -> LlamaConfig:
        if self.arch == "qwen3":
            return LlamaConfig(**self.cfg, qk_norm=True, mask_policy="cache")
        return LlamaConfig(**self.cfg)

    def prompt_ids(self) -> torch.Tensor:
        g = torch.Generator().manual_seed(1000 + self.seed)
        return torch.randint(0, self.cfg["vocab_size"], (self.batch, self.prompt), generator=g)


# The reference's own CPU-runnable case: the tiny Llama, fp32, 2 stages, B=1,
# 64-token prompt, 32 greedy decode steps.
C1 = Case(
    name="llama_c1_fp32",
    arch="llama",
    cfg=dict(
        vocab_size=32000, hidden_size=512, intermediate_size=1408, num_hidden_layers=4,
        num_attention_heads=8, num_key_value_heads=4, head_dim=64, max_position_embeddings=2048,
        rms_norm_eps=1e-5, rope_theta=10000.0,
    ),
    stages=2, dtype=torch.float32, batch=1, prompt=64, steps=32,
)

# A scaled-down TinyLlama geometry (32q/4kv ratio kept at 8) in bf16.
LLAMA_BF16 = Case(
    name="llama_small_bf16",
    arch="llama",
    cfg=dict(
        vocab_size=4096, hidden_size=256, intermediate_size=688, num_hidden_layers=4,
        num_attention_heads=8, num_key_value_heads=1, head_dim=32, max_position_embeddings=512,
        rms_norm_eps=1e-5, rope_theta=10000.0,
    ),
    stages=2, dtype=torch.bfloat16, batch=2, prompt=48, steps=16,
)

# Qwen3 geometry (QK-norm, head_dim 128 > hidden/heads, tied embeddings, theta 1e6).
QWEN_CFG = dict(
    vocab_size=2048, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
    num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=512,
    rms_norm_eps=1e-6, rope_theta=1_000_000.0, tie_word_embeddings=True,
)
QWEN_FP32 = Case(
    name="qwen3_small_fp32", arch="qwen3", cfg=QWEN_CFG, stages=2, dtype=torch.float32,
    batch=2, prompt=32, steps=8,
)
QWEN_BF16 = Case(
    name="qwen3_small_bf16", arch="qwen3", cfg=QWEN_CFG, stages=2, dtype=torch.bfloat16,
    batch=2, prompt=32, steps=8,
)

# Packed multi-token decode after a prefill (positions T..T+2 with a mask):
# the reference's test_multi_token_decode_matches_single_token_decode shape.
MULTI = Case(
    name="llama_multi_token_fp32",
    arch="llama",
    cfg=dict(
        vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
        num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=64,
        rms_norm_eps=1e-5,
    ),
    stages=2, dtype=torch.float32, batch=1, prompt=3, steps=0,
    extra={"future": [[15, 16, 17]]},
)

CASES = [C1, LLAMA_BF16, QWEN_FP32, QWEN_BF16, MULTI]


def sketch(logits: torch.Tensor) -> dict[str, torch.Tensor]:
    """Compact fingerprint of a logits tensor [..., V] (fp32)."""
    x = logits.float()
    vals, idx = x.topk(TOPK, dim=-1)
    return {
        "sub": x[..., ::SKETCH_STRIDE].contiguous(),
        "top_v": vals,
        "top_i": idx,
        "mean": x.mean(-1),
        "std": x.std(-1),
    }


# ---------------------------------------------------------------------------
# Whole models at the benchmark geometries, bf16, with the device-independent
# ("portable") synthetic weights so that a GPU regenerates the identical model
# in a second.  The reference runs the prompt and a free-running greedy stream;
# the fixtures keep the tokens, every step's top logits and a fixed subsample
# of the vocabulary, and the same logits from the oracle under float64
# accumulation (teacher-forced on the reference's tokens), which measures the
# reference's own rounding noise.
# ---------------------------------------------------------------------------

MODEL_SUB_STRIDE = 997  # logits[..., ::997] per row and step
MODEL_TOPK = 8


@dataclass
class ModelCase:
    name: str
    arch: str
    cfg: dict
    stages: int
    batch: int
    prompt: int
    steps: int
    seed: int = 0
    dtype: torch.dtype = torch.bfloat16

    def config(self) -> LlamaConfig:
        if self.arch == "qwen3":
            return LlamaConfig(**self.cfg, qk_norm=True, mask_policy="cache")
        return LlamaConfig(**self.cfg)

    def prompt_ids(self) -> torch.Tensor:
        g = torch.Generator().manual_seed(5000 + self.seed)
        return torch.randint(0, self.cfg["vocab_size"], (self.batch, self.prompt), generator=g)


# Llama-3-8B: one 8-row micro-batch of the decode benchmark, its 1024-token prompts.
LLAMA3_8B = ModelCase(
    name="model_llama3_8b_bf16",
    arch="llama",
    cfg=dict(
        vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=2048,
        rms_norm_eps=1e-5, rope_theta=500000.0,
    ),
    stages=2, batch=8, prompt=1024, steps=32,
)

# TinyLlama-1.1B: batch 8, 512-token prompts, 2 stages.
TINYLLAMA_1B = ModelCase(
    name="model_tinyllama_1b_bf16",
    arch="llama",
    cfg=dict(
        vocab_size=32000, hidden_size=2048, intermediate_size=5632, num_hidden_layers=22,
        num_attention_heads=32, num_key_value_heads=4, head_dim=64, max_position_embeddings=2048,
        rms_norm_eps=1e-5, rope_theta=10000.0,
    ),
    stages=2, batch=8, prompt=512, steps=32,
)

# Qwen3-4B: QK-norm, tied embeddings, theta 1e6; 2048-token prompts (4 rows).
QWEN3_4B = ModelCase(
    name="model_qwen3_4b_bf16",
    arch="qwen3",
    cfg=dict(
        vocab_size=151936, hidden_size=2560, intermediate_size=9728, num_hidden_layers=36,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=4096,
        rms_norm_eps=1e-6, rope_theta=1_000_000.0, tie_word_embeddings=True,
    ),
    stages=2, batch=4, prompt=2048, steps=32,
)

MODEL_CASES = [LLAMA3_8B, TINYLLAMA_1B, QWEN3_4B]


def model_indices(top_i: torch.Tensor, vocab: int) -> torch.Tensor:
    """Vocabulary indices kept per row: the reference's top-k, then the fixed subsample."""
    sub = torch.arange(0, vocab, MODEL_SUB_STRIDE).expand(*top_i.shape[:-1], -1)
    return torch.cat([top_i, sub], dim=-1)
