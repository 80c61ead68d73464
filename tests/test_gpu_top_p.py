"""Top-p drawn inside the last stage (mg_stage_decode_top_p): the lm_head's
epilogue counts each row's bf16 logits by value, one selection kernel draws.

Checked against (a) the oracle's restatement of top_p_sample
(inference/sampling.py:63-95) on the stage's own logits: the token is one a
correct fp32 sampler may return for that uniform (exact except within 2e-5 of
a CDF boundary), and (b) the standalone mg_sample_top_p on the same logits and
uniforms, which builds the same histogram with its own kernel: identical.
"""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200 import build_pipeline, pipeline_prefill
from gpu_mesh_b200.config import LlamaConfig
from gpu_mesh_b200.pipeline import pipeline_decode_top_p
from gpu_mesh_b200.sampling import top_p_sample
from gpu_mesh_b200.weights import synthetic_model_state
from oracle import stage_ref as R

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("temperature,top_p", [(0.7, 0.9), (1.0, 0.5), (0.3, 0.95), (1.3, 0.0), (1.0, 1.0)])
def test_fused_top_p_matches_the_sampler_on_the_stage_logits(temperature, top_p):
    cfg = LlamaConfig(vocab_size=151936, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=64, max_position_embeddings=256,
                      tie_word_embeddings=True)
    full = synthetic_model_state(cfg, seed=5, dtype=torch.bfloat16)
    workers = build_pipeline(cfg, 2, [DEV, DEV], transport="local_cuda", dtype=torch.bfloat16, state_dict=full)
    g = torch.Generator().manual_seed(int(100 * temperature + 10 * top_p))
    keys = ["a", "b"]
    prompts = [torch.randint(0, cfg.vocab_size, (n, 12), generator=g) for n in (3, 5)]
    with torch.no_grad():
        for k, p in zip(keys, prompts):
            pipeline_prefill(workers, p, cache_key=k, logits="last")
        ids = torch.randint(0, cfg.vocab_size, (8, 1), generator=g)
        for step in range(3):
            u = torch.rand(8, generator=g)
            tok, logits = pipeline_decode_top_p(workers, ids.to(DEV), cache_keys=keys, temperature=temperature,
                                                top_p=top_p, uniforms=u)
            lg = logits[:, -1]
            alone = top_p_sample(lg, temperature, top_p, uniforms=u.to(DEV))
            assert torch.equal(tok.cpu(), alone.cpu()), step
            host = lg.float().cpu().to(torch.bfloat16)
            for r in range(8):
                ok = R.top_p_acceptable(host[r], temperature, top_p, float(u[r]), eps=2e-5)
                assert int(tok[r]) in ok, (step, r)
            ids = tok.view(-1, 1)
        for w in workers:
            w.check_device()
    for w in workers:
        w.close()
