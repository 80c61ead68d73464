"""The decode layer chain (one persistent launch for o_proj, norm, gate/up,
down and the next layer's norm + qkv, or the final norm + lm_head) against
the kernel-by-kernel path: the chain reuses the same GEMM split, fix-up
order and norm reduction order, so outputs and KV caches must be identical
bit for bit.  The kernel-by-kernel path is itself held to the oracle by
test_gpu_stage.py.
"""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200 import B200Stage
from gpu_mesh_b200.config import LlamaConfig
from gpu_mesh_b200.weights import synthetic_model_state

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)

SMALL = LlamaConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=3,
                    num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=256)
# Llama-3-8B layer geometry with a small vocabulary (the lm_head shape only
# changes the tile count).
WIDE = LlamaConfig(vocab_size=8192, hidden_size=4096, intermediate_size=14336, num_hidden_layers=2,
                   num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=2048,
                   rope_theta=500000.0)
QWEN = LlamaConfig(vocab_size=4096, hidden_size=2560, intermediate_size=9728, num_hidden_layers=2,
                   num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=2048,
                   rope_theta=1e6, rms_norm_eps=1e-6, qk_norm=True, mask_policy="cache")


def _stage_pair(monkeypatch, cfg, first: bool, last: bool, state):
    stages = []
    for chain in ("0", "1"):
        monkeypatch.setenv("MESHGPU_LAYER_CHAIN", chain)
        stages.append(B200Stage(cfg, 0, cfg.num_hidden_layers, has_embedding=first, has_lm_head=last,
                                device=DEV, dtype=torch.bfloat16, state_dict=state))
    monkeypatch.delenv("MESHGPU_LAYER_CHAIN")
    return stages


def _stage_state(full, first: bool, last: bool):
    drop = ()
    if not first:
        drop += ("embed_tokens",)
    if not last:
        drop += ("norm", "lm_head")
    return {k: v for k, v in full.items() if not k.startswith(drop)}


@pytest.mark.parametrize("cfg", [SMALL, WIDE, QWEN], ids=["small", "llama3-8b-width", "qwen3-4b-width"])
@pytest.mark.parametrize("first,last", [(True, True), (False, False)], ids=["whole", "middle"])
def test_chain_matches_kernel_by_kernel_bitwise(monkeypatch, cfg, first, last):
    full = synthetic_model_state(cfg, seed=9, dtype=torch.bfloat16)
    state = _stage_state(full, first, last)
    plain, chain = _stage_pair(monkeypatch, cfg, first, last, state)
    g = torch.Generator().manual_seed(3)
    slots = {0: 8, 1: 24}  # 8 rows alone (16-row tiles) and 32 rows together (32-row tiles)
    for slot, rows in slots.items():
        for st in (plain, chain):
            st.kv_reserve(slot, rows, 80)
        if first:
            ids = torch.randint(0, cfg.vocab_size, (rows, 33), generator=g)
            outs = [st.forward_slot(slot, None, input_ids=ids, logits="last") for st in (plain, chain)]
        else:
            x = (torch.randn(rows, 33, cfg.hidden_size, generator=g) * 0.5).to(torch.bfloat16)
            outs = [st.forward_slot(slot, x) for st in (plain, chain)]
        assert torch.equal(outs[0], outs[1])  # prefill runs kernel by kernel in both
    for step in range(3):
        if first:
            ids = torch.randint(0, cfg.vocab_size, (8, 1), generator=g)
            a = plain.forward_slot(0, None, input_ids=ids, logits="last")
            b = chain.forward_slot(0, None, input_ids=ids, logits="last")
            ids32 = torch.randint(0, cfg.vocab_size, (32, 1), generator=g)
            c = plain.decode_multi([0, 1], None, input_ids=ids32)
            d = chain.decode_multi([0, 1], None, input_ids=ids32)
        else:
            x = (torch.randn(8, 1, cfg.hidden_size, generator=g) * 0.5).to(torch.bfloat16)
            a = plain.forward_slot(0, x)
            b = chain.forward_slot(0, x)
            x32 = (torch.randn(32, 1, cfg.hidden_size, generator=g) * 0.5).to(torch.bfloat16)
            c = plain.decode_multi([0, 1], x32)
            d = chain.decode_multi([0, 1], x32)
        assert torch.isfinite(a.float()).all()
        assert torch.equal(a, b), f"step {step}, 8 rows"
        assert torch.equal(c, d), f"step {step}, 32 rows"
    for slot, rows in slots.items():
        T = plain.kv_length(slot)
        assert T == chain.kv_length(slot)
        for (ka, va), (kb, vb) in zip(plain.kv_export(slot), chain.kv_export(slot)):
            assert torch.equal(ka, kb) and torch.equal(va, vb)
    chain.check_device()
    plain.close()
    chain.close()
