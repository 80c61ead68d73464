"""Greedy selection on the device (mg_stage_decode_greedy): fused into the
lm_head decode GEMM for bf16, after the logits otherwise.  The ids must be
exactly greedy_sample of the logits the plain decode returns (the
reference's argmax, inference/sampling.py:45-56: the lowest index among equal
maxima), and the logits themselves must not change."""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200 import build_pipeline, greedy_sample, pipeline_prefill
from gpu_mesh_b200.config import LlamaConfig
from gpu_mesh_b200.pipeline import pipeline_decode_greedy, pipeline_decode_multi
from gpu_mesh_b200.weights import synthetic_model_state

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
SMALL = LlamaConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                    num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=256)
# A vocabulary of 1000 tiles of 128 rows plus a ragged one, over the 148 CTAs.
WIDE_VOCAB = LlamaConfig(vocab_size=128000 + 64, hidden_size=256, intermediate_size=512, num_hidden_layers=1,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=128)


def pair(cfg, dtype, state, n=1):
    return [build_pipeline(cfg, n, [DEV] * n, transport="local_cuda", dtype=dtype, state_dict=state)
            for _ in range(2)]


def prefill_both(pipes, groups, cfg, seed=0):
    g = torch.Generator().manual_seed(seed)
    for i, rows in enumerate(groups):
        p = torch.randint(0, cfg.vocab_size, (rows, 5 + 3 * i), generator=g)
        for workers in pipes:
            pipeline_prefill(workers, p, cache_key=f"k{i}", logits="last")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16_fused", "fp32_after_logits"])
@pytest.mark.parametrize("groups", [(3,), (8, 8), (16, 16)], ids=["3rows", "16rows", "32rows"])
def test_ids_equal_argmax_of_unchanged_logits(dtype, groups):
    state = synthetic_model_state(SMALL, seed=21)
    plain, fused = pair(SMALL, dtype, state)
    prefill_both((plain, fused), groups, SMALL)
    keys = [f"k{i}" for i in range(len(groups))]
    rows = sum(groups)
    g = torch.Generator().manual_seed(5)
    for step in range(4):
        nxt = torch.randint(0, SMALL.vocab_size, (rows, 1), generator=g)
        logits = pipeline_decode_multi(plain, nxt, cache_keys=keys)
        ids, logits2 = pipeline_decode_greedy(fused, nxt, cache_keys=keys, return_logits=True)
        assert torch.equal(logits, logits2), step
        assert torch.equal(ids.cpu(), greedy_sample(logits[:, -1]).cpu()), step
        # the other way round at the next position (logits not requested)
        ids_only, none = pipeline_decode_greedy(plain, nxt, cache_keys=keys)
        logits3 = pipeline_decode_multi(fused, nxt, cache_keys=keys)
        assert none is None and torch.equal(ids_only.cpu(), greedy_sample(logits3[:, -1]).cpu()), step
    for workers in (plain, fused):
        for w in workers:
            w._model.check_device()
            w.close()


def test_exact_ties_resolve_to_the_lowest_index_across_tiles_and_ctas():
    """lm_head rows repeat with period 7, so every logit value occurs ~18k
    times across ~1000 tiles split over all CTAs: the pick must be the first."""
    state = synthetic_model_state(WIDE_VOCAB, seed=3, dtype=torch.bfloat16)
    head = state["lm_head.weight"]
    state["lm_head.weight"] = head[:7].repeat((head.shape[0] + 6) // 7, 1)[: head.shape[0]].contiguous()
    plain, fused = pair(WIDE_VOCAB, torch.bfloat16, state)
    prefill_both((plain, fused), (16, 16), WIDE_VOCAB, seed=1)
    keys = ["k0", "k1"]
    g = torch.Generator().manual_seed(9)
    for _ in range(3):
        nxt = torch.randint(0, WIDE_VOCAB.vocab_size, (32, 1), generator=g)
        logits = pipeline_decode_multi(plain, nxt, cache_keys=keys)
        ids, _ = pipeline_decode_greedy(fused, nxt, cache_keys=keys)
        want = greedy_sample(logits[:, -1]).cpu()
        assert torch.all(want < 7)
        assert torch.equal(ids.cpu(), want)
    for workers in (plain, fused):
        for w in workers:
            w._model.check_device()
            w.close()


def test_two_stage_pipeline_and_middle_stage_rejection():
    state = synthetic_model_state(SMALL, seed=4)
    plain, fused = pair(SMALL, torch.bfloat16, state, n=2)
    prefill_both((plain, fused), (4,), SMALL)
    nxt = torch.tensor([[1], [2], [3], [4]])
    logits = pipeline_decode_multi(plain, nxt, cache_keys=["k0"])
    ids, _ = pipeline_decode_greedy(fused, nxt, cache_keys=["k0"])
    assert torch.equal(ids.cpu(), greedy_sample(logits[:, -1]).cpu())
    assert [w.kv_cache_length("k0") for w in fused] == [6, 6]
    with pytest.raises(ValueError, match="last stage"):
        fused[0]._model.decode_greedy([fused[0].slot_of("k0")], None, input_ids=nxt)
    for workers in (plain, fused):
        for w in workers:
            w.close()
