"""Generate the golden vectors by running the REFERENCE implementation.

Run where a checkout of the reference (hungtrab/gpu_mesh) is available:

    python tests/golden/make_golden.py --reference <checkout>

It imports the reference's own portable pipeline (``build_pipeline``,
``pipeline_prefill``, ``pipeline_decode_step``, ``LlamaStage``,
``Qwen3Stage``, ``StageWorker``, ``top_p_sample``), loads the seeded synthetic
weights of each case in ``cases.py`` into it, and writes one small ``.pt``
fixture per case next to this script: prompt ids, greedy tokens and compact
logits sketches of the prefill and of every decode step.  For top-p it
captures the distribution the reference hands to ``torch.multinomial``.
The fixtures are committed; nothing at test time reads the reference.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from gpu_mesh_b200.weights import slice_stage_state, synthetic_model_state  # noqa: E402
from tests.golden.cases import CASES, LLAMA_BF16, sketch  # noqa: E402


def _llama_workers(ref, case, full):
    from meshgpu.backends.portable.pipeline import build_pipeline
    from meshgpu.models.llama_dense import LlamaConfig

    cfg = LlamaConfig(**case.cfg)
    torch.manual_seed(0)
    workers = build_pipeline(cfg, case.stages, [torch.device("cpu")] * case.stages)
    for w in workers:
        m = w._model
        sd = slice_stage_state(full, m.layer_start, m.layer_end, has_embedding=m.has_embedding,
                               has_lm_head=m.has_lm_head)
        missing, unexpected = m.load_state_dict(sd, strict=False)
        assert not unexpected and all("rope" in k for k in missing), (missing, unexpected)
        m.to(case.dtype)
    return workers


def _qwen_workers(ref, case, full):
    from transformers import Qwen3Config

    from meshgpu.backends.portable.pipeline import build_pipeline  # noqa: F401  (import check)
    from meshgpu.backends.portable.stage_worker import StageContext, StageWorker
    from meshgpu.models.qwen3_hf import Qwen3Stage

    c = dict(case.cfg)
    theta = c.pop("rope_theta")
    hf = Qwen3Config(**c, rope_parameters={"rope_type": "default", "rope_theta": theta})
    ranges = []
    base, rem = divmod(hf.num_hidden_layers, case.stages)
    start = 0
    for i in range(case.stages):
        end = start + base + (1 if i < rem else 0)
        ranges.append((start, end))
        start = end
    workers = []
    for i, (a, b) in enumerate(ranges):
        first, last = i == 0, i == len(ranges) - 1
        stage = Qwen3Stage(hf, a, b, has_embedding=first, has_lm_head=last, device="cpu",
                           dtype=case.dtype, attn_implementation="sdpa")
        sd = slice_stage_state(full, a, b, has_embedding=first, has_lm_head=last,
                               tie_word_embeddings=True)
        missing, unexpected = stage.load_state_dict({k: v.to(case.dtype) for k, v in sd.items()},
                                                    strict=False)
        assert not unexpected, unexpected
        assert all("rotary" in k for k in missing), missing
        ctx = StageContext(stage_id=i, layer_start=a, layer_end=b, device=torch.device("cpu"),
                           is_first=first, is_last=last, job_id="golden", attempt_id="local")
        workers.append(StageWorker(stage, ctx))
    return workers


def run_case(case) -> dict:
    from meshgpu.backends.portable.pipeline import pipeline_decode_step, pipeline_prefill

    cfg = case.config()
    full = synthetic_model_state(cfg, seed=case.seed, dtype=torch.float32)
    workers = (_qwen_workers if case.arch == "qwen3" else _llama_workers)(None, case, full)
    ids = case.prompt_ids()
    out = {"case": case.name, "prompt": ids, "torch": str(torch.__version__)}
    with torch.no_grad():
        logits = pipeline_prefill(workers, ids, operation_id=1, attempt_id="g", cache_key="g")
        out["prefill"] = sketch(logits)
        out["prefill_last"] = logits[:, -1].float().clone()
        if "future" in case.extra:
            fut = torch.tensor(case.extra["future"])
            packed = pipeline_decode_step(workers, fut, operation_id=2, attempt_id="g", cache_key="g")
            out["future"] = fut
            out["packed"] = packed.float().clone()
            return out
        tok = logits[:, -1].argmax(-1, keepdim=True)
        tokens = [tok]
        steps = []
        for k in range(case.steps):
            logits = pipeline_decode_step(workers, tok, operation_id=2 + k, attempt_id="g", cache_key="g")
            steps.append(sketch(logits[:, -1]))
            tok = logits[:, -1].argmax(-1, keepdim=True)
            tokens.append(tok)
        out["tokens"] = torch.cat(tokens, dim=1)
        out["steps"] = {k: torch.stack([s[k] for s in steps]) for k in steps[0]} if steps else {}
        out["kv_len"] = workers[0].kv_cache_length("g")
        if case.arch == "llama":
            k0, v0 = workers[0]._kv_caches_by_key["g"][0]
            out["kv0_sketch"] = {"k": k0[..., :4].float().clone(), "v": v0[..., :4].float().clone()}
    return out


def run_top_p() -> dict:
    """Capture the nucleus the reference samples from (sampling.py:82-94)."""
    from meshgpu.inference import sampling

    g = torch.Generator().manual_seed(7)
    rows = []
    # bf16 logits of the small Llama's scale: many exact ties.
    logits = (torch.randn(4, LLAMA_BF16.cfg["vocab_size"], generator=g) * 1.5).to(torch.bfloat16)
    params = [(0.7, 0.9), (1.0, 0.5), (0.3, 0.95), (1.3, 0.0)]
    captured = []
    real = torch.multinomial

    def spy(probs, num_samples, generator=None, **kw):
        captured.append(probs.detach().clone())
        return real(probs, num_samples, generator=generator, **kw)

    torch.multinomial = spy
    try:
        for r, (t, p) in enumerate(params):
            captured.clear()
            sampling.top_p_sample(logits[r : r + 1], t, p, generator=torch.Generator().manual_seed(r))
            probs = captured[0][0]
            kept = int((probs > 0).sum())
            rows.append({"temperature": t, "top_p": p, "kept": kept, "probs": probs[:kept].clone()})
    finally:
        torch.multinomial = real
    return {"logits": logits, "rows": rows}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a reference checkout (its src/ is imported)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    torch.set_num_threads(8)
    import meshgpu  # noqa: F401

    for case in CASES:
        data = run_case(case)
        torch.save(data, HERE / f"{case.name}.pt")
        print(case.name, "ok")
    torch.save(run_top_p(), HERE / "top_p.pt")
    print("top_p ok")


if __name__ == "__main__":
    main()
