"""Host-side logic that needs no GPU: config validation, layer splits, stage
context, synthetic weights, RoPE tables, and the pipeline coordinator's
protocol (sync check, rollback, async drain) driven with fake workers.

Mirrors the reference's unit tests (tests/unit/test_model.py:39-61,
tests/unit/test_inference.py:196-233 rollback, :39-61 drain)."""
from __future__ import annotations

import asyncio
import threading

import pytest
import torch

from gpu_mesh_b200 import pipeline as P
from gpu_mesh_b200.config import LlamaConfig, config_from, split_layers
from gpu_mesh_b200.sampling import SamplingParams, make_sampling_generator
from gpu_mesh_b200.stage_worker import StageContext
from gpu_mesh_b200.weights import (
    rope_tables,
    slice_stage_state,
    synthetic_model_state,
    synthetic_stage_state,
)

TINY = dict(
    vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
    num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=64,
)


def test_config_rejects_invalid_numeric_values():
    with pytest.raises(TypeError, match="num_hidden_layers"):
        LlamaConfig(**{**TINY, "num_hidden_layers": 2.0})
    with pytest.raises(ValueError, match="rms_norm_eps"):
        LlamaConfig(**TINY, rms_norm_eps=float("nan"))
    with pytest.raises(ValueError, match="divisible"):
        LlamaConfig(**{**TINY, "num_attention_heads": 3})
    with pytest.raises(ValueError, match="even"):
        LlamaConfig(**{**TINY, "head_dim": 15})
    with pytest.raises(ValueError, match="attention_implementation"):
        LlamaConfig(**TINY, attention_implementation="flash")


def test_config_from_hf_qwen3():
    from transformers import Qwen3Config

    hf = Qwen3Config(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                     max_position_embeddings=128, tie_word_embeddings=True,
                     rope_parameters={"rope_type": "default", "rope_theta": 1e6})
    cfg = config_from(hf)
    assert cfg.qk_norm and cfg.mask_policy == "cache" and cfg.tie_word_embeddings
    assert cfg.rope_theta == 1e6 and cfg.head_dim == 32 and cfg.rms_norm_eps == hf.rms_norm_eps


def test_split_layers_matches_reference_rule():
    assert split_layers(32, 1) == [(0, 32)]
    assert split_layers(22, 4) == [(0, 6), (6, 12), (12, 17), (17, 22)]
    assert split_layers(36, 8)[0] == (0, 5) and split_layers(36, 8)[-1] == (32, 36)
    with pytest.raises(ValueError):
        split_layers(4, 5)


def test_stage_context_validation():
    with pytest.raises(ValueError, match="non-empty layer range"):
        StageContext(0, 2, 2, "cpu", True, True, "j", "a")
    with pytest.raises(ValueError, match="transport"):
        StageContext(0, 0, 2, "cpu", True, True, "j", "a", transport="tcp")
    with pytest.raises(TypeError):
        StageContext(True, 0, 2, "cpu", True, True, "j", "a")


def test_synthetic_weights_are_sliceable_and_deterministic():
    cfg = LlamaConfig(**TINY)
    full = synthetic_model_state(cfg, seed=3)
    again = synthetic_model_state(cfg, seed=3)
    assert all(torch.equal(full[k], again[k]) for k in full)
    stage = synthetic_stage_state(cfg, 2, 4, has_embedding=False, has_lm_head=True, seed=3)
    cut = slice_stage_state(full, 2, 4, has_embedding=False, has_lm_head=True)
    assert stage.keys() == cut.keys()
    assert all(torch.equal(stage[k], cut[k]) for k in stage)
    w = full["layers.0.self_attn.q_proj.weight"]
    assert abs(float(w.std()) - 0.02) < 2e-3 and torch.all(full["norm.weight"] == 1)


def test_tied_lm_head_is_the_embedding():
    cfg = LlamaConfig(**TINY, tie_word_embeddings=True)
    sd = synthetic_stage_state(cfg, 0, 4, has_embedding=True, has_lm_head=True)
    assert sd["lm_head.weight"] is sd["embed_tokens.weight"]


def test_rope_tables_match_hf_qwen3_rotary_embedding():
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    hf = Qwen3Config(head_dim=128, hidden_size=256, num_attention_heads=2, max_position_embeddings=64,
                     rope_parameters={"rope_type": "default", "rope_theta": 1e6})
    emb = Qwen3RotaryEmbedding(hf)
    pos = torch.arange(64).unsqueeze(0)
    cos_hf, sin_hf = emb(torch.zeros(1, dtype=torch.bfloat16), pos)
    cos, sin = rope_tables(128, 64, 1e6, torch.bfloat16)
    assert torch.equal(cos_hf[0, :, :64], cos) and torch.equal(sin_hf[0, :, :64], sin)
    # A bf16 Qwen3Stage casts the rotary module to bf16 (qwen3_hf.py:139-140),
    # rounding its inverse frequencies; at long positions that moves the angles.
    emb.to(torch.bfloat16)
    pos = torch.arange(4096).unsqueeze(0)
    hf.max_position_embeddings = 4096
    cos_hf, sin_hf = emb(torch.zeros(1, dtype=torch.bfloat16), pos)
    cos, sin = rope_tables(128, 4096, 1e6, torch.bfloat16, round_inv_freq=True)
    assert torch.equal(cos_hf[0, :, :64], cos) and torch.equal(sin_hf[0, :, :64], sin)
    plain, _ = rope_tables(128, 4096, 1e6, torch.bfloat16)
    assert not torch.equal(plain, cos)


def test_sampling_params_validation():
    with pytest.raises(ValueError, match="temperature"):
        SamplingParams(temperature=-1)
    with pytest.raises(ValueError, match="top_p"):
        SamplingParams(top_p=1.5)
    with pytest.raises(TypeError):
        SamplingParams(seed=1.5)
    assert make_sampling_generator(SamplingParams()) is None
    g1 = make_sampling_generator(SamplingParams(seed=5))
    g2 = make_sampling_generator(SamplingParams(seed=5))
    assert torch.equal(torch.rand(3, generator=g1), torch.rand(3, generator=g2))


# ---------------------------------------------------------------------------
# Coordinator protocol with fake workers (no GPU).
# ---------------------------------------------------------------------------

class FakeWorker:
    """Records calls and keeps a per-key length like a stage would."""

    def __init__(self, name, fail_on=None, delay_event=None):
        self.name = name
        self.len = {}
        self.fail_on = fail_on
        self.calls = []
        self.delay_event = delay_event

    def clear_kv(self, key=None):
        self.calls.append(("clear", key))
        self.len.pop(key, None)

    def kv_cache_length(self, key=None):
        return self.len.get(key, 0)

    def trim_kv(self, length, key=None):
        self.calls.append(("trim", key, length))
        self.len[key] = length

    def forward_inference(self, hidden, *, input_ids=None, position_ids=None, operation_id, attempt_id,
                          reset_kv=False, cache_key=None, attention_mask=None):
        if self.delay_event is not None:
            self.delay_event.wait(5)
        src = input_ids if input_ids is not None else hidden
        self.len[cache_key] = self.len.get(cache_key, 0) + src.shape[1]
        self.calls.append(("fwd", cache_key, None if position_ids is None else position_ids[0].tolist()))
        if self.fail_on == operation_id:
            raise RuntimeError(f"{self.name} failed")

        class R:
            output = torch.zeros(src.shape[0], src.shape[1], 4)

        return R()


def test_decode_checks_sync_and_prefill():
    a, b = FakeWorker("a"), FakeWorker("b")
    with pytest.raises(RuntimeError, match="requires a prefilled KV cache"):
        P.pipeline_decode_step([a, b], torch.zeros(1, 1, dtype=torch.long), operation_id=2)
    a.len[None], b.len[None] = 3, 2
    with pytest.raises(RuntimeError, match="out of sync"):
        P.pipeline_decode_step([a, b], torch.zeros(1, 1, dtype=torch.long), operation_id=2)


def test_decode_feeds_positions_and_rolls_back_on_failure():
    a, b = FakeWorker("a"), FakeWorker("b", fail_on=3)
    ids = torch.zeros(1, 4, dtype=torch.long)
    P.pipeline_prefill([a, b], ids, cache_key="k")
    P.pipeline_decode_step([a, b], torch.zeros(1, 2, dtype=torch.long), operation_id=2, cache_key="k")
    assert a.calls[-1] == ("fwd", "k", [4, 5])
    with pytest.raises(RuntimeError, match="b failed"):
        P.pipeline_decode_step([a, b], torch.zeros(1, 1, dtype=torch.long), operation_id=3, cache_key="k")
    assert a.len["k"] == 6 and b.len["k"] == 6  # trimmed back to the pre-step lengths
    assert ("trim", "k", 6) in a.calls


def test_prefill_failure_clears_every_stage():
    a, b = FakeWorker("a"), FakeWorker("b", fail_on=1)
    with pytest.raises(RuntimeError):
        P.pipeline_prefill([a, b], torch.zeros(1, 4, dtype=torch.long), cache_key="k")
    assert a.kv_cache_length("k") == 0 and b.kv_cache_length("k") == 0


def test_prefill_rejects_bad_shapes():
    with pytest.raises(ValueError, match="batch, sequence"):
        P.pipeline_prefill([FakeWorker("a")], torch.zeros(4, dtype=torch.long))
    with pytest.raises(ValueError, match="non-empty"):
        P.pipeline_prefill([FakeWorker("a")], torch.zeros(1, 0, dtype=torch.long))
    with pytest.raises(ValueError, match="workers"):
        P.pipeline_prefill([], torch.zeros(1, 2, dtype=torch.long))


def test_async_call_drains_on_cancel():
    gate = threading.Event()
    w = FakeWorker("slow", delay_event=gate)

    async def main():
        task = asyncio.create_task(P.pipeline_prefill_async([w], torch.zeros(1, 2, dtype=torch.long)))
        await asyncio.sleep(0.05)
        task.cancel()
        await asyncio.sleep(0.05)
        gate.set()
        with pytest.raises(asyncio.CancelledError):
            await task

    asyncio.run(main())
    # the running stage call finished before cancellation propagated
    assert any(c[0] == "fwd" for c in w.calls)


class FakeRemoteWorker(FakeWorker):
    """A stage reached over RPC: coroutine methods, as the reference's remote workers."""

    async def clear_kv(self, key=None):
        FakeWorker.clear_kv(self, key)

    async def kv_cache_length(self, key=None):
        return FakeWorker.kv_cache_length(self, key)

    async def trim_kv(self, length, key=None):
        FakeWorker.trim_kv(self, length, key)

    async def forward_inference(self, hidden, **kw):
        await asyncio.sleep(0)
        return FakeWorker.forward_inference(self, hidden, **kw)


def test_async_plans_drive_remote_stages_and_roll_back():
    a, b = FakeRemoteWorker("a"), FakeRemoteWorker("b", fail_on=3)

    async def main():
        out = await P.pipeline_prefill_async([a, b], torch.zeros(2, 3, dtype=torch.long), cache_key="r")
        assert out.shape == (2, 3, 4)
        await P.pipeline_decode_step_async([a, b], torch.zeros(2, 1, dtype=torch.long), operation_id=2,
                                           cache_key="r")
        assert a.calls[-1] == ("fwd", "r", [3])
        with pytest.raises(RuntimeError, match="b failed"):
            await P.pipeline_decode_step_async([a, b], torch.zeros(2, 1, dtype=torch.long), operation_id=3,
                                               cache_key="r")
        with pytest.raises(RuntimeError, match="pipeline_decode_step_async requires a prefilled"):
            await P.pipeline_decode_step_async([a, b], torch.zeros(1, 1, dtype=torch.long), operation_id=4,
                                               cache_key="other")

    asyncio.run(main())
    assert a.len["r"] == 4 and b.len["r"] == 4  # the failed step was trimmed away on both stages


def test_cancelled_async_prefill_rolls_back_after_the_drain():
    gate = threading.Event()
    a, b = FakeWorker("a"), FakeWorker("b", delay_event=gate)

    async def main():
        task = asyncio.create_task(P.pipeline_prefill_async([a, b], torch.zeros(1, 2, dtype=torch.long),
                                                            cache_key="c"))
        await asyncio.sleep(0.05)
        task.cancel()
        await asyncio.sleep(0.05)
        gate.set()
        with pytest.raises(asyncio.CancelledError):
            await task

    asyncio.run(main())
    assert a.kv_cache_length("c") == 0 and b.kv_cache_length("c") == 0


def test_rollback_failures_are_logged_not_raised(caplog):
    class Stubborn(FakeWorker):
        def trim_kv(self, length, key=None):
            raise RuntimeError("cannot trim")

    a, b = Stubborn("a"), FakeWorker("b", fail_on=2)
    P.pipeline_prefill([a, b], torch.zeros(1, 2, dtype=torch.long), cache_key="s")
    with pytest.raises(RuntimeError, match="b failed"):
        P.pipeline_decode_step([a, b], torch.zeros(1, 1, dtype=torch.long), operation_id=2, cache_key="s")
    assert "rollback step trim_kv failed" in caplog.text
    assert b.len["s"] == 2


def test_portable_weights_are_the_same_on_every_code_path():
    from gpu_mesh_b200 import weights as W

    n = 1_000_003
    k1, k2 = W._portable_keys(7, "layers.3.mlp.down_proj.weight")
    host = W.portable_quantile_index(n, 7, "layers.3.mlp.down_proj.weight")
    torch_path = torch.cat([i for _, i in W._portable_index_torch(n, k1, k2, torch.device("cpu"))])
    assert torch.equal(host, torch_path)  # the numpy kernel (hosts) and the torch kernel (GPUs) agree
    w = W.portable_tensor("layers.3.mlp.down_proj.weight", (1000, 1000), seed=7, dtype=torch.bfloat16)
    table = W._quantile_table(0.02, torch.bfloat16, torch.device("cpu"))
    assert torch.equal(w.flatten(), table[host[:1_000_000]])
    assert abs(float(w.float().std()) - 0.02) < 2e-4 and abs(float(w.float().mean())) < 2e-4
    again = W.portable_tensor("layers.3.mlp.down_proj.weight", (1000, 1000), seed=7, dtype=torch.bfloat16)
    other = W.portable_tensor("layers.3.mlp.down_proj.weight", (1000, 1000), seed=8, dtype=torch.bfloat16)
    assert torch.equal(w, again) and not torch.equal(w, other)
    cfg = LlamaConfig(**TINY)
    full = synthetic_model_state(cfg, seed=1, method="portable")
    stage = synthetic_stage_state(cfg, 2, 4, has_embedding=False, has_lm_head=True, seed=1, method="portable")
    assert torch.equal(stage["layers.0.self_attn.q_proj.weight"], full["layers.2.self_attn.q_proj.weight"])
    with pytest.raises(ValueError, match="unknown synthetic weight method"):
        synthetic_model_state(cfg, method="uniform")


def test_boundary_transports_on_the_host():
    from gpu_mesh_b200.boundary import move_to_stage

    x = torch.arange(6.0).view(1, 2, 3)
    assert move_to_stage(x, "cpu", transport="cpu") is x
    assert move_to_stage(x, "cpu", transport="local_cuda") is x
    with pytest.raises(ValueError, match="unsupported local boundary transport"):
        move_to_stage(x, "cpu", transport="rdma")


def test_balanced_layer_ranges_even_out_the_streamed_bytes():
    from gpu_mesh_b200.config import balanced_layer_ranges

    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=8192)
    for n in (1, 2, 4, 8):
        r = balanced_layer_ranges(cfg, n, rows=32, context=1100)
        assert r[0][0] == 0 and r[-1][1] == 32 and all(a[1] == b[0] and a[0] < a[1] for a, b in zip(r, r[1:]))
    r8 = balanced_layer_ranges(cfg, 8, rows=32, context=1100)
    sizes = [b - a for a, b in r8]
    assert sizes[-1] < min(sizes[:-1])  # the lm_head stage holds fewer layers
    assert max(sizes) == 5  # 32 layers + lm_head cannot spread thinner than 5 layers on some stage
    assert balanced_layer_ranges(cfg, 1, rows=1, context=1) == [(0, 32)]
    with pytest.raises(ValueError):
        balanced_layer_ranges(cfg, 33, rows=1, context=1)
