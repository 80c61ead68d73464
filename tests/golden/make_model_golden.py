"""Generate the whole-model golden vectors by running the REFERENCE.

Run where a checkout of the reference (hungtrab/gpu_mesh) is available:

    python tests/golden/make_model_golden.py --reference <checkout> [--case NAME ...]

For every case of ``cases.MODEL_CASES`` (Llama-3-8B, TinyLlama-1.1B and
Qwen3-4B at full depth, bf16, with the device-independent synthetic weights)
it builds the reference's own pipeline on the CPU (``build_pipeline`` for the
Llama geometry, ``Qwen3Stage`` + ``StageWorker`` for Qwen3), loads the
weights, runs ``pipeline_prefill`` on the case's prompt and then a
free-running greedy stream of ``pipeline_decode_step`` calls (argmax of the
bf16 logits, lowest index on ties, as ``greedy_sample`` does).  It then runs
the oracle with float64 accumulation (``oracle.stage_ref.exact_rounding``),
teacher-forced on the reference's tokens, to measure how far the reference's
own bf16 arithmetic sits from the exactly-rounded computation.

Each fixture ``model_<name>.pt`` holds the prompt, the reference's tokens,
and per step and row the logits at a fixed set of vocabulary indices (the
reference's top 8, then every 997th id) from the reference and from the
exact oracle.  Weights are regenerated, not stored.  Nothing at test time
reads the reference.
"""
from __future__ import annotations

import argparse
import contextlib
import sys
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from gpu_mesh_b200.weights import slice_stage_state, synthetic_model_state  # noqa: E402
from oracle import stage_ref as R  # noqa: E402
from tests.golden.cases import MODEL_CASES, MODEL_TOPK, model_indices  # noqa: E402


@contextlib.contextmanager
def _construct_without_init(dtype: torch.dtype):
    """Build modules directly in ``dtype`` and skip their random init: every
    parameter is overwritten by ``load_state_dict`` right after."""
    names = ["kaiming_uniform_", "uniform_", "normal_", "trunc_normal_", "zeros_", "ones_"]
    saved = {n: getattr(torch.nn.init, n) for n in names}
    old = torch.get_default_dtype()
    for n in names:
        setattr(torch.nn.init, n, lambda t, *a, **k: t)
    torch.set_default_dtype(dtype)
    try:
        yield
    finally:
        torch.set_default_dtype(old)
        for n, f in saved.items():
            setattr(torch.nn.init, n, f)


def _split(n_layers: int, n_stages: int) -> list[tuple[int, int]]:
    base, rem = divmod(n_layers, n_stages)
    out, start = [], 0
    for i in range(n_stages):
        end = start + base + (1 if i < rem else 0)
        out.append((start, end))
        start = end
    return out


def reference_workers(case, full):
    if case.arch == "llama":
        from meshgpu.backends.portable.pipeline import build_pipeline
        from meshgpu.models.llama_dense import LlamaConfig

        cfg = LlamaConfig(**case.cfg)
        with _construct_without_init(case.dtype):
            workers = build_pipeline(cfg, case.stages, [torch.device("cpu")] * case.stages)
        for w in workers:
            m = w._model
            sd = slice_stage_state(full, m.layer_start, m.layer_end, has_embedding=m.has_embedding,
                                   has_lm_head=m.has_lm_head)
            missing, unexpected = m.load_state_dict(sd, strict=False)
            assert not unexpected and all("rope" in k for k in missing), (missing, unexpected)
            m.to(case.dtype)
        return workers

    from transformers import Qwen3Config

    from meshgpu.backends.portable.stage_worker import StageContext, StageWorker
    from meshgpu.models.qwen3_hf import Qwen3Stage

    c = dict(case.cfg)
    theta = c.pop("rope_theta")
    hf = Qwen3Config(**c, rope_parameters={"rope_type": "default", "rope_theta": theta})
    workers = []
    ranges = _split(hf.num_hidden_layers, case.stages)
    for i, (a, b) in enumerate(ranges):
        first, last = i == 0, i == len(ranges) - 1
        with _construct_without_init(case.dtype):
            stage = Qwen3Stage(hf, a, b, has_embedding=first, has_lm_head=last, device="cpu",
                               dtype=case.dtype, attn_implementation="sdpa")
        sd = slice_stage_state(full, a, b, has_embedding=first, has_lm_head=last, tie_word_embeddings=True)
        missing, unexpected = stage.load_state_dict(sd, strict=False)
        assert not unexpected, unexpected
        assert all("rotary" in k for k in missing), missing
        ctx = StageContext(stage_id=i, layer_start=a, layer_end=b, device=torch.device("cpu"),
                           is_first=first, is_last=last, job_id="golden", attempt_id="local")
        workers.append(StageWorker(stage, ctx))
    return workers


def run_reference(case, full, ids):
    """Prefill + free-running greedy stream through the reference pipeline."""
    from meshgpu.backends.portable.pipeline import pipeline_decode_step, pipeline_prefill
    from meshgpu.inference.sampling import greedy_sample

    workers = reference_workers(case, full)
    V = case.cfg["vocab_size"]
    rows, tokens = [], []
    with torch.no_grad():
        t0 = time.time()
        logits = pipeline_prefill(workers, ids, operation_id=1, attempt_id="g", cache_key="g")[:, -1].float()
        print(f"  reference prefill {time.time() - t0:.1f}s", flush=True)
        for k in range(case.steps + 1):
            top_v, top_i = logits.topk(MODEL_TOPK, dim=-1)
            idx = model_indices(top_i, V)
            tok = greedy_sample(logits)
            rows.append({
                "index": idx.to(torch.int32),
                "ref": logits.gather(-1, idx),
                "margin": top_v[:, 0] - top_v[:, 1],
                "argmax": tok.clone(),
            })
            tokens.append(tok)
            if k == case.steps:
                break
            logits = pipeline_decode_step(workers, tok.view(-1, 1), operation_id=2 + k, attempt_id="g",
                                          cache_key="g")[:, -1].float()
        print(f"  reference decode done {time.time() - t0:.1f}s", flush=True)
    del workers
    return torch.stack(tokens, dim=1), rows


def run_exact(case, full, ids, tokens, rows):
    """The oracle under float64 accumulation, teacher-forced on the reference's tokens."""
    cfg = case.config()
    stages = R.build_stages(cfg, case.stages, full, dtype=case.dtype)
    out = []
    with torch.no_grad(), R.exact_rounding():
        t0 = time.time()
        logits = R.prefill(stages, ids, key="g", last_only=True)[:, -1].float()
        print(f"  exact prefill {time.time() - t0:.1f}s", flush=True)
        for k in range(case.steps + 1):
            out.append(logits.gather(-1, rows[k]["index"].long()))
            if k == case.steps:
                break
            logits = R.decode_step(stages, tokens[:, k : k + 1], key="g")[:, -1].float()
        print(f"  exact decode done {time.time() - t0:.1f}s", flush=True)
    return out


def run_case(case) -> dict:
    import transformers

    cfg = case.config()
    t0 = time.time()
    full = synthetic_model_state(cfg, seed=case.seed, dtype=case.dtype, method="portable")
    print(f"  weights {time.time() - t0:.1f}s", flush=True)
    ids = case.prompt_ids()
    tokens, rows = run_reference(case, full, ids)
    exact = run_exact(case, full, ids, tokens, rows)
    stack = lambda key: torch.stack([r[key] for r in rows])  # noqa: E731
    ref, ex = stack("ref"), torch.stack(exact)
    noise = (ref - ex).abs()
    print(f"  |ref - exact| max {float(noise.max()):.4f} mean {float(noise.mean()):.5f}; "
          f"argmax(ref)==argmax(exact) on top-8: "
          f"{float((ref[..., :MODEL_TOPK].argmax(-1) == ex[..., :MODEL_TOPK].argmax(-1)).float().mean()):.3f}",
          flush=True)
    return {
        "case": case.name,
        "weights": "portable",
        "seed": case.seed,
        "prompt": ids,
        "tokens": tokens,
        "index": stack("index"),
        "ref": ref,
        "exact": ex,
        "margin": stack("margin"),
        "torch": str(torch.__version__),
        "transformers": str(transformers.__version__),
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a reference checkout (its src/ is imported)")
    ap.add_argument("--case", action="append", help="case name(s); default: all")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import meshgpu  # noqa: F401

    for case in MODEL_CASES:
        if args.case and case.name not in args.case:
            continue
        print(case.name, flush=True)
        data = run_case(case)
        torch.save(data, HERE / f"{case.name}.pt")
        print(case.name, "ok", flush=True)


if __name__ == "__main__":
    main()
