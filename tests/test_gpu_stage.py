"""CUDA stage behaviour through the C ABI: KV-slot semantics, error paths,
multi-slot decode, sampling kernels, and full-width (Llama-3-8B / Qwen3-4B)
layer geometry against the CPU oracle.

Tolerances: fp32 1e-4 relative to the logits' max magnitude; bf16 2e-2
absolute on logits (the parity bar); sampling is exact (integer ids).
"""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200 import B200Stage, build_pipeline, greedy_sample, pipeline_decode_step, pipeline_prefill, top_p_sample
from gpu_mesh_b200._lib import DeviceRangeError
from gpu_mesh_b200.config import LlamaConfig
from gpu_mesh_b200.weights import synthetic_model_state, synthetic_stage_state
from oracle import stage_ref as R

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
TINY = LlamaConfig(
    vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
    num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=64,
)


def tiny_workers(n=2, dtype=torch.float32, cfg=TINY):
    full = synthetic_model_state(cfg, seed=11)
    return build_pipeline(cfg, n, [DEV] * n, transport="local_cuda", dtype=dtype, state_dict=full), full


def test_kv_lengths_trim_clear_and_errors():
    workers, _ = tiny_workers()
    ids = torch.tensor([[1, 2, 3, 4]])
    pipeline_prefill(workers, ids, cache_key="a")
    assert [w.kv_cache_length("a") for w in workers] == [4, 4]
    assert workers[0].kv_cache_length("b") == 0
    pipeline_decode_step(workers, torch.tensor([[5]]), operation_id=2, cache_key="a")
    assert workers[1].kv_cache_length("a") == 5
    workers[0].trim_kv(3, "a")
    assert workers[0].kv_cache_length("a") == 3
    with pytest.raises(RuntimeError, match="out of sync"):
        pipeline_decode_step(workers, torch.tensor([[5]]), operation_id=3, cache_key="a")
    with pytest.raises(RuntimeError, match="shorter than requested"):
        workers[0].trim_kv(9, "a")
    with pytest.raises(RuntimeError, match="empty cache"):
        workers[0].trim_kv(1, "zzz")
    with pytest.raises(ValueError, match="non-negative"):
        workers[0].trim_kv(-1, "a")
    workers[0].clear_kv("a")
    assert workers[0].kv_cache_length("a") == 0
    workers[0].clear_all_kv()
    for w in workers:
        w.close()


def test_stage_argument_errors_match_reference_messages():
    workers, _ = tiny_workers(1)
    w = workers[0]
    with pytest.raises(ValueError, match="requires input_ids"):
        w.forward_inference(None, operation_id=1, attempt_id="a")
    with pytest.raises(ValueError, match="outside"):
        w.forward_inference(None, input_ids=torch.tensor([[TINY.vocab_size, 1]]), operation_id=1, attempt_id="a")
    with pytest.raises(ValueError, match="outside"):
        w.forward_inference(None, input_ids=torch.tensor([[1, 2]]),
                            position_ids=torch.tensor([[0, TINY.max_position_embeddings]]),
                            operation_id=1, attempt_id="a")
    with pytest.raises(ValueError, match="int32 or int64"):
        w.forward_inference(None, input_ids=torch.tensor([[1.0]]), operation_id=1, attempt_id="a")
    with pytest.raises(ValueError, match="would reach"):
        w.forward_inference(None, input_ids=torch.zeros(1, 65, dtype=torch.long), operation_id=1, attempt_id="a")
    # the failed calls left no cache behind
    assert w.kv_cache_length() == 0
    w.close()


def test_device_clamps_and_reports_unchecked_ids():
    workers, _ = tiny_workers(1)
    w = workers[0]
    w.check_values = False
    w.forward_inference(None, input_ids=torch.tensor([[TINY.vocab_size + 5]]), operation_id=1, attempt_id="a")
    with pytest.raises(DeviceRangeError, match="input_ids"):
        w.check_device()
    w.check_device()  # the error word was cleared
    w.close()


def test_causal_prefill_and_multi_token_decode():
    workers, full = tiny_workers()
    ids = torch.tensor([[3, 7, 11, 13]])
    full_logits = pipeline_prefill(workers, ids, cache_key="c").float().cpu()
    first = pipeline_prefill(workers, ids[:, :1], cache_key="d").float().cpu()
    torch.testing.assert_close(full_logits[:, :1], first, atol=1e-4, rtol=1e-3)
    # packed multi-token decode equals sequential single-token decode
    prompt, fut = torch.tensor([[4, 8, 12]]), torch.tensor([[15, 16, 17]])
    pipeline_prefill(workers, prompt, cache_key="pk")
    pipeline_prefill(workers, prompt, cache_key="sq")
    packed = pipeline_decode_step(workers, fut, operation_id=2, cache_key="pk").float().cpu()
    seq = torch.cat([
        pipeline_decode_step(workers, fut[:, i : i + 1], operation_id=3 + i, cache_key="sq").float().cpu()
        for i in range(3)
    ], 1)
    torch.testing.assert_close(packed, seq, atol=1e-4, rtol=1e-3)
    for w in workers:
        w.close()


def test_explicit_positions_follow_the_mask_policy():
    workers, full = tiny_workers(1)
    oracle = R.build_stages(TINY, 1, full)
    ids = torch.tensor([[5, 6, 7, 8, 9]])
    pos = torch.tensor([[0, 1, 1, 3, 2]])  # non-standard positions -> masked path
    got = workers[0].forward_inference(None, input_ids=ids, position_ids=pos, operation_id=1,
                                       attempt_id="a", cache_key="e").output.float().cpu()
    exp = oracle[0].forward(input_ids=ids, position_ids=pos, key="e").float()
    assert (got - exp).abs().max() <= 1e-4 * exp.abs().max()
    workers[0].close()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_multi_equals_per_slot_decode(dtype):
    cfg = LlamaConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=256)
    full = synthetic_model_state(cfg, seed=5)
    a = build_pipeline(cfg, 1, [DEV], transport="local_cuda", dtype=dtype, state_dict=full)[0]
    b = build_pipeline(cfg, 1, [DEV], transport="local_cuda", dtype=dtype, state_dict=full)[0]
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 512, (2, 9), generator=g), torch.randint(0, 512, (3, 17), generator=g)]
    for i, p in enumerate(prompts):
        a.forward_inference(None, input_ids=p, operation_id=1, attempt_id="a", cache_key=f"s{i}")
        b.forward_inference(None, input_ids=p, operation_id=1, attempt_id="a", cache_key=f"s{i}")
    nxt = torch.randint(0, 512, (5, 1), generator=g)
    multi = a.decode_multi(None, ["s0", "s1"], input_ids=nxt).float().cpu()
    sep = torch.cat([
        b.forward_inference(None, input_ids=nxt[:2], operation_id=2, attempt_id="a", cache_key="s0",
                            logits="last").output,
        b.forward_inference(None, input_ids=nxt[2:], operation_id=2, attempt_id="a", cache_key="s1",
                            logits="last").output,
    ]).float().cpu()
    assert torch.equal(multi, sep)
    assert a.kv_cache_length("s0") == 10 and a.kv_cache_length("s1") == 18
    a.close()
    b.close()


def test_kv_import_export_round_trip_and_decode():
    workers, full = tiny_workers(1)
    w = workers[0]
    oracle = R.build_stages(TINY, 1, full)
    ids = torch.randint(0, 256, (2, 12), generator=torch.Generator().manual_seed(3))
    oracle[0].forward(input_ids=ids, key="o")
    w.import_kv("imp", [(k, v) for k, v in oracle[0].caches["o"]])
    assert w.kv_cache_length("imp") == 12
    out = w._model.kv_export(w.slot_of("imp"))
    for (k, v), (ko, vo) in zip(out, oracle[0].caches["o"]):
        assert torch.equal(k.cpu(), ko) and torch.equal(v.cpu(), vo)
    nxt = torch.tensor([[1], [2]])
    got = w.forward_inference(None, input_ids=nxt, operation_id=2, attempt_id="a", cache_key="imp").output
    exp = oracle[0].forward(input_ids=nxt, key="o")
    assert (got.float().cpu() - exp).abs().max() <= 1e-4 * exp.abs().max()
    w.close()


def test_kv_growth_keeps_contents():
    workers, full = tiny_workers(1)
    w = workers[0]
    oracle = R.build_stages(TINY, 1, full)
    ids = torch.randint(0, 256, (1, 5), generator=torch.Generator().manual_seed(9))
    w.forward_inference(None, input_ids=ids, operation_id=1, attempt_id="a", cache_key="g")
    oracle[0].forward(input_ids=ids, key="g")
    for t in range(40):  # forces several capacity doublings
        nxt = torch.tensor([[t % 256]])
        got = w.forward_inference(None, input_ids=nxt, operation_id=2, attempt_id="a", cache_key="g").output
        exp = oracle[0].forward(input_ids=nxt, key="g")
    assert (got.float().cpu() - exp).abs().max() <= 1e-4 * exp.abs().max()
    w.close()


# ---------------------------------------------------------------------------
# Sampling kernels (exact integer parity with the oracle)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_greedy_sample_ties_and_lowest_index(dtype):
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(37, 128256, generator=g).to(dtype)
    logits[3, 100] = logits[3, 5000] = 50.0  # exact tie -> index 100
    got = greedy_sample(logits.to(DEV)).cpu()
    assert torch.equal(got, R.greedy(logits))
    assert got[3] == 100


@pytest.mark.parametrize("temperature,top_p", [(0.7, 0.9), (1.0, 0.5), (0.3, 0.95), (1.3, 0.0), (1.0, 1.0)])
def test_top_p_matches_oracle_inverse_cdf(temperature, top_p):
    g = torch.Generator().manual_seed(int(temperature * 100 + top_p * 10))
    logits = (torch.randn(16, 151936, generator=g) * 1.5).to(torch.bfloat16)
    u = torch.rand(16, generator=g)
    got = top_p_sample(logits.to(DEV), temperature, top_p, uniforms=u).cpu()
    exact = R.top_p_with_uniforms(logits, temperature, top_p, u)
    for r in range(16):
        ok = R.top_p_acceptable(logits[r], temperature, top_p, float(u[r]), eps=2e-5)
        assert int(got[r]) in ok, (r, int(got[r]), int(exact[r]))
    # away from boundaries the draw is the oracle's exact token
    assert (got == exact).float().mean() >= 0.75


def test_top_p_reference_nucleus_golden():
    from tests.conftest import load_golden

    t = load_golden("top_p")
    for r, row in enumerate(t["rows"]):
        lg = t["logits"][r : r + 1]
        for uval in (0.0, 0.25, 0.5, 0.75, 0.999):
            u = torch.tensor([uval])
            got = top_p_sample(lg.to(DEV), row["temperature"], row["top_p"], uniforms=u).cpu()
            ok = R.top_p_acceptable(lg[0], row["temperature"], row["top_p"], uval, eps=2e-5)
            assert int(got[0]) in ok
            # the drawn token is inside the reference's own nucleus
            sp, si = R.top_p_nucleus(lg, row["temperature"], row["top_p"])
            assert int(got[0]) in set(si[0, : row["kept"]].tolist())


# ---------------------------------------------------------------------------
# Full-width layers (the benchmark geometries) against the oracle
# ---------------------------------------------------------------------------

LLAMA3_8B_2L = LlamaConfig(
    vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=2,
    num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=4096,
    rope_theta=500000.0,
)
QWEN3_4B_2L = LlamaConfig(
    vocab_size=151936, hidden_size=2560, intermediate_size=9728, num_hidden_layers=2,
    num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=4096,
    rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=True, qk_norm=True, mask_policy="cache",
)


def _exact_bar(got: torch.Tensor, ref: torch.Tensor, exact: torch.Tensor, what: str) -> None:
    """The full-width bf16 bar (oracle.stage_ref.exact_bar)."""
    R.exact_bar(got, ref, exact, what)


@pytest.mark.parametrize("cfg", [LLAMA3_8B_2L, QWEN3_4B_2L], ids=["llama3-8b", "qwen3-4b"])
def test_full_width_layers_match_oracle(cfg):
    """Two full-width layers of the benchmark geometries (prefill on the
    tcgen05 GEMM, decode on the split-K GEMV and the split attention)."""
    torch.set_num_threads(max(torch.get_num_threads(), 8))
    full = synthetic_model_state(cfg, seed=2, dtype=torch.bfloat16)
    w = build_pipeline(cfg, 1, [DEV], transport="local_cuda", dtype=torch.bfloat16, state_dict=full)[0]
    oracle = R.build_stages(cfg, 1, full, dtype=torch.bfloat16)
    exact = R.build_stages(cfg, 1, full, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, cfg.vocab_size, (8, 40), generator=g)
    got = w.forward_inference(None, input_ids=ids, operation_id=1, attempt_id="a", cache_key="f",
                              logits="last").output.float().cpu()
    ref = oracle[0].forward(input_ids=ids, key="f")[:, -1:].float()
    with R.exact_rounding():
        ex = exact[0].forward(input_ids=ids, key="f")[:, -1:].float()
    _exact_bar(got, ref, ex, "prefill")
    for step in range(3):  # decode: GEMV path, split-K, attention over the cache
        nxt = torch.randint(0, cfg.vocab_size, (8, 1), generator=g)
        got = w.forward_inference(None, input_ids=nxt, operation_id=2, attempt_id="a", cache_key="f").output
        ref = oracle[0].forward(input_ids=nxt, key="f").float()
        with R.exact_rounding():
            ex = exact[0].forward(input_ids=nxt, key="f").float()
        _exact_bar(got.float().cpu(), ref, ex, f"decode {step}")
    w.close()


@pytest.mark.parametrize("D,nq,nkv", [(128, 32, 8), (64, 32, 4)], ids=["d128-g4", "d64-g8"])
@pytest.mark.parametrize("T", [1, 31, 129, 1000, 4100])
def test_attention_over_imported_cache_matches_oracle(D, nq, nkv, T):
    """Decode attention (tensor-core path for bf16 head_dim 64/128) over a
    cache pre-filled with N(0, 1) keys and values, at lengths that are not
    multiples of the 32-key boxes or 128-key chunks."""
    cfg = LlamaConfig(vocab_size=256, hidden_size=512, intermediate_size=1024, num_hidden_layers=1,
                      num_attention_heads=nq, num_key_value_heads=nkv, head_dim=D,
                      max_position_embeddings=8192, rope_theta=500000.0)
    full = synthetic_model_state(cfg, seed=7, dtype=torch.bfloat16)
    state = {k: v for k, v in full.items() if not k.startswith(("norm", "lm_head"))}
    stage = B200Stage(cfg, 0, 1, has_embedding=True, has_lm_head=False, device=DEV,
                      dtype=torch.bfloat16, state_dict=state)
    oracle = R.OracleStage(cfg, 0, 1, True, False, state, torch.bfloat16)
    exact = R.OracleStage(cfg, 0, 1, True, False, state, torch.bfloat16)
    g = torch.Generator().manual_seed(T + D)
    k = torch.randn(2, nkv, T, D, generator=g).to(torch.bfloat16)
    v = torch.randn(2, nkv, T, D, generator=g).to(torch.bfloat16)
    stage.kv_reserve(3, 2, T + 8)
    stage.kv_import(3, 0, k, v)
    oracle.caches["c"] = [(k, v)]
    exact.caches["c"] = [(k, v)]
    ids = torch.tensor([[5], [77]])
    got = stage.forward_slot(3, None, input_ids=ids).float().cpu()
    ref = oracle.forward(input_ids=ids, key="c").float()
    with R.exact_rounding():
        ex = exact.forward(input_ids=ids, key="c").float()
    _exact_bar(got, ref, ex, f"T={T}")
    stage.close()


# RoPE / QK-norm / KV append kernels (every variant) against the oracle
# ---------------------------------------------------------------------------

@pytest.mark.parametrize(
    "dtype,D,nq,nkv,qk_norm,S",
    [
        (torch.float32, 128, 4, 2, True, 40),    # a CTA per token, 32 lanes per head
        (torch.float32, 64, 8, 2, False, 40),    # 16 lanes per head
        (torch.bfloat16, 128, 12, 4, True, 40),  # 16 lanes per head, two rounds of the row
        (torch.bfloat16, 64, 5, 1, False, 40),   # 8 lanes per head, 7 heads: partial warps and groups
        (torch.bfloat16, 32, 4, 2, False, 40),   # head_dim outside the vector kernels
        (torch.bfloat16, 128, 8, 2, False, 300), # more tokens than resident CTAs: each CTA takes several
    ],
    ids=["f32-d128-qkn", "f32-d64", "bf16-d128-qkn", "bf16-d64-odd", "bf16-d32", "bf16-d128-600tok"],
)
def test_rope_kv_append_matches_oracle(dtype, D, nq, nkv, qk_norm, S):
    """Prefill of 2 x S tokens (the many-token kernel) then two decode
    steps (the decode-row kernel, reading the projection's pieces in bf16):
    the exported K / V cache and the logits against the oracle.  Cache bar:
    max |cuda - oracle| <= 1e-4 (fp32) or 2e-2 (bf16) x max |oracle|."""
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=nq, num_key_value_heads=nkv, head_dim=D,
                      max_position_embeddings=512, rope_theta=500000.0,
                      **({"qk_norm": True, "mask_policy": "cache"} if qk_norm else {}))
    full = synthetic_model_state(cfg, seed=21, dtype=dtype)
    stage = B200Stage(cfg, 0, 2, has_embedding=True, has_lm_head=True, device=DEV, dtype=dtype, state_dict=full)
    oracle = R.OracleStage(cfg, 0, 2, True, True, full, dtype)
    rel = 1e-4 if dtype == torch.float32 else 2e-2
    g = torch.Generator().manual_seed(D + nq)
    stage.kv_reserve(1, 2, S + 8)
    ids = torch.randint(0, cfg.vocab_size, (2, S), generator=g)
    steps = [ids] + [torch.randint(0, cfg.vocab_size, (2, 1), generator=g) for _ in range(2)]
    for i, x in enumerate(steps):
        got = stage.forward_slot(1, None, input_ids=x).float().cpu()
        ref = oracle.forward(input_ids=x, key="c").float()
        assert (got - ref).abs().max() <= tol_logits(dtype, ref), i
        for layer, ((gk, gv), (rk, rv)) in enumerate(zip(stage.kv_export(1), oracle.caches["c"])):
            for name, a, b in (("k", gk, rk), ("v", gv, rv)):
                b = b.float()
                err = float((a.float().cpu() - b).abs().max())
                assert err <= rel * float(b.abs().max()), (i, layer, name, err)
    stage.close()


def tol_logits(dtype, ref: torch.Tensor) -> float:
    return 1e-4 * float(ref.abs().max()) if dtype == torch.float32 else 2e-2


def test_decode_norm_cluster_kernel_is_bit_identical_to_one_cta(monkeypatch):
    """The decode residual + RMSNorm spreads each row over a cluster of four
    CTAs; it keeps the one-CTA kernel's reduction order, so two stages with
    the same weights, one per kernel (MESHGPU_NORM_ONE_CTA=1 selects the
    one-CTA kernel), give identical logits at the Llama-3-8B width."""
    cfg = LlamaConfig(vocab_size=2048, hidden_size=4096, intermediate_size=14336, num_hidden_layers=2,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=512,
                      rope_theta=500000.0)
    full = synthetic_model_state(cfg, seed=7, dtype=torch.bfloat16, device=DEV, method="portable")
    a = build_pipeline(cfg, 1, [DEV], transport="local_cuda", dtype=torch.bfloat16, state_dict=full)[0]
    b = build_pipeline(cfg, 1, [DEV], transport="local_cuda", dtype=torch.bfloat16, state_dict=full)[0]
    del full
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (8, 40), generator=g).to(DEV)
    with torch.no_grad():
        a.forward_inference(None, input_ids=ids, operation_id=1, attempt_id="a", cache_key="k")
        b.forward_inference(None, input_ids=ids, operation_id=1, attempt_id="a", cache_key="k")
        tok = torch.randint(0, cfg.vocab_size, (8, 1), generator=g).to(DEV)
        for step in range(3):
            la = a.forward_inference(None, input_ids=tok, operation_id=2 + step, attempt_id="a",
                                     cache_key="k").output.float().cpu()
            monkeypatch.setenv("MESHGPU_NORM_ONE_CTA", "1")
            lb = b.forward_inference(None, input_ids=tok, operation_id=2 + step, attempt_id="a",
                                     cache_key="k").output.float().cpu()
            monkeypatch.delenv("MESHGPU_NORM_ONE_CTA")
            assert torch.equal(la, lb), step
            tok = la[:, -1].argmax(-1, keepdim=True).to(DEV)
    a.check_device()
    b.check_device()
    a.close()
    b.close()
