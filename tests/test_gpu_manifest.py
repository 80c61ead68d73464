"""B200 stages loaded from reference-written artifacts reproduce the
reference's own loaders (build_pipeline_from_manifest on the CPU, outputs in
tests/golden/manifests/*.expected.pt).

Tolerances (the parity bar of the stage path):
  * fp32 artifacts: max |cuda - ref| <= 1e-4 * max |ref| over the logits,
    and the free-running greedy stream identical;
  * bf16 artifacts: max |cuda - ref| <= 2e-2 over the logits, greedy tokens
    identical except where the reference's top-2 margin is within that.
"""
from __future__ import annotations

import pytest
import torch

from gpu_mesh_b200 import pipeline_decode_step, pipeline_prefill
from gpu_mesh_b200.manifest import build_pipeline_from_manifest, build_stage_from_manifest
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
MANIFESTS = GOLDEN / "manifests"
NAMES = ["llama_gqa_bf16", "llama_tied_fp32", "llama_tiny_fp32", "qwen3_tiny_fp32"]


def expected(name):
    return torch.load(MANIFESTS / f"{name}.expected.pt", weights_only=True)


def tol(exp, ref):
    return 2e-2 if exp["dtype"] == "bfloat16" else 1e-4 * float(ref.abs().max())


@pytest.mark.parametrize("name", NAMES)
def test_loaded_pipeline_matches_reference_loader(name):
    exp = expected(name)
    n = exp["stages"]
    workers = build_pipeline_from_manifest(MANIFESTS / name, devices=[DEV] * n, transport="local_cuda")
    assert [w._ctx.is_first for w in workers] == [True] + [False] * (n - 1)
    assert [w._ctx.is_last for w in workers] == [False] * (n - 1) + [True]
    assert workers[0]._model.meshgpu_adapter == ("qwen3_hf_v1" if name.startswith("qwen3") else "llama_dense_v1")
    ids = exp["prompt"]
    with torch.no_grad():
        got = pipeline_prefill(workers, ids, cache_key="m").float().cpu()
        assert (got - exp["prefill"]).abs().max() <= tol(exp, exp["prefill"])
        tok = exp["tokens"][:, :1]
        if exp["dtype"] == "float32":
            assert torch.equal(got[:, -1].argmax(-1, keepdim=True), tok)
        for k in range(exp["steps"].shape[1]):
            out = pipeline_decode_step(workers, tok, operation_id=2 + k, cache_key="m").float().cpu()[:, -1]
            ref = exp["steps"][:, k]
            assert (out - ref).abs().max() <= tol(exp, ref), k
            nxt = out.argmax(-1, keepdim=True)
            want = exp["tokens"][:, k + 1 : k + 2]
            if exp["dtype"] == "float32":
                assert torch.equal(nxt, want), k  # free running
            else:
                top = ref.topk(2, -1).values
                assert torch.all((nxt == want).squeeze(1) | ((top[:, 0] - top[:, 1]) <= tol(exp, ref))), k
                nxt = want  # teacher-forced on the reference's stream
            tok = nxt
    for w in workers:
        w.close()


@pytest.mark.parametrize("name", NAMES)
def test_planner_resplit_matches_reference(name):
    exp = expected(name)
    ranges = exp["planned_ranges"]
    workers = build_pipeline_from_manifest(MANIFESTS / name, devices=[DEV] * len(ranges),
                                           layer_ranges=ranges, transport="local_cuda")
    assert [(w._ctx.layer_start, w._ctx.layer_end) for w in workers] == [tuple(r) for r in ranges]
    with torch.no_grad():
        got = pipeline_prefill(workers, exp["prompt"]).float().cpu()
    assert (got - exp["planned_prefill"]).abs().max() <= tol(exp, exp["planned_prefill"])
    for w in workers:
        w.close()


def test_single_stage_entry_point_loads_only_its_shard():
    w = build_stage_from_manifest(MANIFESTS / "llama_gqa_bf16", 1, device=DEV)
    assert (w._ctx.stage_id, w._ctx.layer_start, w._ctx.layer_end) == (1, 2, 3)
    assert not w._ctx.is_first and not w._ctx.is_last
    assert w._model.dtype == torch.bfloat16
    w.close()
