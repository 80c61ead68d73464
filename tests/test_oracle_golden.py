"""Pin the CPU oracle to golden vectors produced by the reference itself.

The fixtures were written by tests/golden/make_golden.py, which ran the
reference's portable pipeline (LlamaStage / HF Qwen3 stages, pipeline_prefill,
pipeline_decode_step, top_p_sample) on the same seeded weights and prompts.

Tolerances (the parity bar of the build):
  * fp32: max |oracle - reference| <= 1e-4 * max |reference| on the logits;
  * bf16: max |oracle - reference| <= 2e-2 on the logits;
  * greedy tokens identical (teacher-forced), except where the reference's
    own top-2 logit margin is within the bf16 tolerance (a near-tie).
"""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200.weights import synthetic_model_state
from oracle import stage_ref as R
from tests.conftest import load_golden
from tests.golden.cases import CASES, sketch

FP32_REL = 1e-4
BF16_ABS = 2e-2


def _tol(case, ref: torch.Tensor) -> float:
    if case.dtype == torch.float32:
        return FP32_REL * float(ref.abs().max())
    return BF16_ABS


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_oracle_matches_reference_golden(case):
    torch.set_num_threads(max(torch.get_num_threads(), 4))
    g = load_golden(case.name)
    cfg = case.config()
    stages = R.build_stages(cfg, case.stages, synthetic_model_state(cfg, seed=case.seed), dtype=case.dtype)
    assert torch.equal(g["prompt"], case.prompt_ids())
    with torch.no_grad():
        logits = R.prefill(stages, g["prompt"])
        s = sketch(logits)
        ref = g["prefill"]["sub"]
        assert (s["sub"] - ref).abs().max() <= _tol(case, ref)
        if "future" in g:
            packed = R.decode_step(stages, g["future"])
            assert (packed.float() - g["packed"]).abs().max() <= _tol(case, g["packed"])
            return
        toks = g["tokens"]
        assert torch.equal(logits[:, -1].argmax(-1), toks[:, 0])
        for k in range(case.steps):
            logits = R.decode_step(stages, toks[:, k : k + 1])
            ref = g["steps"]["sub"][k]
            assert (sketch(logits[:, -1])["sub"] - ref).abs().max() <= _tol(case, ref)
            got = logits[:, -1].argmax(-1)
            top = g["steps"]["top_v"][k]
            margin = top[:, 0] - top[:, 1]
            near_tie = margin <= (0.0 if case.dtype == torch.float32 else BF16_ABS)
            assert torch.all((got == toks[:, k + 1]) | near_tie), (k, got, toks[:, k + 1], margin)
        assert stages[0].cache_length() == g["kv_len"]


def test_oracle_kv_contents_match_reference():
    case = CASES[0]
    g = load_golden(case.name)
    cfg = case.config()
    stages = R.build_stages(cfg, case.stages, synthetic_model_state(cfg, seed=case.seed), dtype=case.dtype)
    toks = g["tokens"]
    with torch.no_grad():
        R.prefill(stages, g["prompt"])
        for k in range(case.steps):
            R.decode_step(stages, toks[:, k : k + 1])
    k0, v0 = stages[0].caches[None][0]
    torch.testing.assert_close(k0[..., :4].float(), g["kv0_sketch"]["k"], atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(v0[..., :4].float(), g["kv0_sketch"]["v"], atol=1e-5, rtol=1e-4)


def test_oracle_top_p_nucleus_matches_reference():
    t = load_golden("top_p")
    for r, row in enumerate(t["rows"]):
        sp, _ = R.top_p_nucleus(t["logits"][r : r + 1], row["temperature"], row["top_p"])
        kept = int((sp > 0).sum())
        assert kept == row["kept"]
        torch.testing.assert_close(sp[0, :kept], row["probs"], atol=1e-7, rtol=1e-6)


def test_oracle_top_p_inverse_cdf_edges():
    logits = torch.tensor([[2.0, 1.0, 1.0, 0.0]])
    sp, si = R.top_p_nucleus(logits, 1.0, 1.0)
    assert si[0].tolist() == [0, 1, 2, 3]  # ties ordered by index
    cum = torch.cumsum(sp[0], 0)
    assert R.top_p_with_uniforms(logits, 1.0, 1.0, torch.tensor([0.0])).item() == 0
    assert R.top_p_with_uniforms(logits, 1.0, 1.0, torch.tensor([float(cum[0])])).item() == 1
    assert R.top_p_with_uniforms(logits, 1.0, 1.0, torch.tensor([0.999999])).item() == 3
    # top_p = 0 keeps only the best token
    assert R.top_p_with_uniforms(logits, 1.0, 0.0, torch.tensor([0.9])).item() == 0
    # temperature 0 is greedy
    assert R.top_p_with_uniforms(logits, 0.0, 0.5, torch.tensor([0.9])).item() == 0


def test_oracle_exposes_the_parity_helpers_the_gpu_tests_use():
    """The GPU tests and smoke() call these; a missing one would only show on a GPU."""
    from oracle import stage_ref as R

    for name in ("exact_bar", "exact_rounding", "top_p_acceptable", "top_p_with_uniforms", "top_p_nucleus",
                 "build_stages", "prefill", "decode_step", "greedy"):
        assert callable(getattr(R, name)), name
    z = torch.zeros(4)
    assert R.exact_bar(z, z, z)["max_got"] == 0.0
