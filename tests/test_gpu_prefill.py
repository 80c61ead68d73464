"""Prefill / multi-token attention on tcgen05 against the oracle: query
tiles of 128 rows (128 / G tokens x G heads) over caches pre-filled with
N(0, 1) keys and values, with and without a cached prefix, at lengths that
are not multiples of the tile or of the 128-key chunk, every G the tile
supports, head_dim 64 and 128.  The bar is the one for full-width bf16
layers: no further from exactly-rounded arithmetic than the reference's own
bf16 computation."""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200 import B200Stage
from gpu_mesh_b200.config import LlamaConfig
from gpu_mesh_b200.weights import synthetic_model_state
from oracle import stage_ref as R
from tests.test_gpu_stage import _exact_bar

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


CASES = [(D, nq, nkv, T, S)
         for D, nq, nkv in [(128, 32, 8), (64, 32, 4), (128, 8, 8), (64, 16, 8)]
         for T, S in [(0, 8), (0, 200), (5, 33), (130, 77), (1000, 129)]]
# Several work items per CTA (more than 148 items), tiles of up to 10 chunks.
CASES += [(128, 32, 8, 0, 1100), (128, 32, 8, 300, 600), (64, 32, 4, 700, 400)]


@pytest.mark.parametrize("D,nq,nkv,T,S", CASES,
                         ids=[f"d{c[0]}-g{c[1] // c[2]}-T{c[3]}-S{c[4]}" for c in CASES])
def test_prefill_attention_matches_oracle(D, nq, nkv, T, S):
    cfg = LlamaConfig(vocab_size=256, hidden_size=512, intermediate_size=1024, num_hidden_layers=1,
                      num_attention_heads=nq, num_key_value_heads=nkv, head_dim=D,
                      max_position_embeddings=4096, rope_theta=500000.0)
    full = synthetic_model_state(cfg, seed=3, dtype=torch.bfloat16)
    state = {k: v for k, v in full.items() if not k.startswith(("norm", "lm_head"))}
    stage = B200Stage(cfg, 0, 1, has_embedding=True, has_lm_head=False, device=DEV,
                      dtype=torch.bfloat16, state_dict=state)
    oracle = R.OracleStage(cfg, 0, 1, True, False, state, torch.bfloat16)
    exact = R.OracleStage(cfg, 0, 1, True, False, state, torch.bfloat16)
    g = torch.Generator().manual_seed(T * 7 + S + D)
    stage.kv_reserve(3, 2, T + S + 40)  # room past the end: never-written rows
    if T:
        k = torch.randn(2, nkv, T, D, generator=g).to(torch.bfloat16)
        v = torch.randn(2, nkv, T, D, generator=g).to(torch.bfloat16)
        stage.kv_import(3, 0, k, v)
        oracle.caches["c"] = [(k, v)]
        exact.caches["c"] = [(k, v)]
    ids = torch.randint(0, cfg.vocab_size, (2, S), generator=g)
    got = stage.forward_slot(3, None, input_ids=ids).float().cpu()
    ref = oracle.forward(input_ids=ids, key="c").float()
    with R.exact_rounding():
        ex = exact.forward(input_ids=ids, key="c").float()
    _exact_bar(got, ref, ex, f"T={T} S={S}")
    assert stage.kv_length(3) == T + S
    stage.check_device()
    stage.close()
