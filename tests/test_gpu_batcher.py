"""The continuous batcher on B200 workers: several requests of different
lengths decoded together (one weight pass per iteration) stream the same
greedy tokens as decoding each request alone with pipeline_decode_step."""
from __future__ import annotations

import asyncio

import pytest
import torch

from gpu_mesh_b200 import build_pipeline, greedy_sample, pipeline_decode_step, pipeline_prefill
from gpu_mesh_b200.batcher import ContinuousBatcher
from gpu_mesh_b200.config import LlamaConfig
from gpu_mesh_b200.sampling import SamplingParams
from gpu_mesh_b200.weights import synthetic_model_state

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
CFG = LlamaConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=4,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=256)


def alone(workers, prompt, n):
    logits = pipeline_prefill(workers, torch.tensor([prompt]), cache_key="alone")
    out = [int(greedy_sample(logits[0, -1]))]
    for step in range(n - 1):
        logits = pipeline_decode_step(workers, torch.tensor([[out[-1]]]), operation_id=step + 2,
                                      cache_key="alone")
        out.append(int(greedy_sample(logits[0, -1])))
    for w in workers:
        w.clear_kv("alone")
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_batched_streams_match_single_request_decoding(dtype):
    full = synthetic_model_state(CFG, seed=13, dtype=dtype)
    workers = build_pipeline(CFG, 2, [DEV, DEV], transport="local_cuda", dtype=dtype, state_dict=full)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, CFG.vocab_size, (n,), generator=g).tolist() for n in (5, 17, 1, 33, 9)]
    want = [alone(workers, p, 10) for p in prompts]

    async def main():
        b = ContinuousBatcher(workers, max_batch_size=4)
        b.start()
        ids = [await b.submit(p, SamplingParams(), 10) for p in prompts]
        got = await asyncio.gather(*[_tokens(b, i) for i in ids])
        b.stop()
        await b.wait_stopped()
        return got, b, ids

    async def _tokens(b, sid):
        return [r.token_id async for r in b.stream(sid)]

    got, b, ids = asyncio.run(main())
    assert got == want
    assert b.decode_passes < 5 * 9  # requests shared decode passes
    for w in workers:
        assert all(w.kv_cache_length(f"seq:{k}") == 0 for k in ids)
        w.close()
