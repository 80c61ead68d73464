"""Generate model-artifact fixtures with the REFERENCE's own importers.

Run in a container that has the reference checkout (hungtrab/gpu_mesh):

    python tests/golden/make_manifest_fixtures.py --reference <checkout>

The reference's artifact package (``meshgpu.artifacts``) ships only inside
its source tarball (kaggle/meshgpu-source-20260914/meshgpu-kaggle-smoke.tar.gz),
so this script copies the checkout's ``src/`` to a scratch directory and
extracts ``src/meshgpu/{artifacts,checkpoints}`` from the tarball beside it.

For each case a small HF model is initialised from a fixed seed and saved
with ``save_pretrained``, then split by the reference's ``import_from_hf``
(Llama) or ``import_qwen_from_hf`` (Qwen3) into ``manifests/<case>/``
(manifest.json, config.json, one shard per stage).  The reference's
``build_pipeline_from_manifest`` then loads the artifact on the CPU, and its
``pipeline_prefill`` / ``pipeline_decode_step`` outputs are stored in
``manifests/<case>.expected.pt``: prefill logits, a free-running greedy
stream with the last-position logits of every step, and the prefill logits
of a planner re-split of the same artifact.  Everything is committed;
nothing at test time reads the reference.

One shim: the reference's ``hf_config_to_llama`` (artifacts/hf_import.py:195-228)
predates transformers 5, which always reports a ``rope_scaling`` dict
(``{'rope_type': 'default', 'rope_theta': ...}``) and keeps ``rope_theta``
only there.  The script hands it a view of the HF config with the default
(unscaled) RoPE entry folded back into ``rope_theta``; any other RoPE type
still goes to the reference function unchanged, which rejects it.
"""
from __future__ import annotations

import argparse
import shutil
import sys
import tarfile
import tempfile
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "manifests"
TARBALL = "kaggle/meshgpu-source-20260914/meshgpu-kaggle-smoke.tar.gz"
STEPS = 8

# name -> (family, HF config kwargs, stages, artifact dtype, seed, prompt, planner ranges)
CASES = {
    "llama_tiny_fp32": (
        "llama",
        dict(vocab_size=64, hidden_size=16, intermediate_size=32, num_hidden_layers=4,
             num_attention_heads=2, num_key_value_heads=2, max_position_embeddings=64),
        2, "float32", 7, [[1, 5, 9, 13, 2, 60, 33]], [(0, 1), (1, 3), (3, 4)],
    ),
    "llama_tied_fp32": (
        "llama",
        dict(vocab_size=64, hidden_size=16, intermediate_size=32, num_hidden_layers=4,
             num_attention_heads=2, num_key_value_heads=2, max_position_embeddings=64,
             tie_word_embeddings=True),
        2, "float32", 11, [[1, 5, 9, 13]], [(0, 4)],
    ),
    "llama_gqa_bf16": (
        "llama",
        dict(vocab_size=256, hidden_size=128, intermediate_size=192, num_hidden_layers=4,
             num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=128,
             rope_theta=500000.0),
        3, "bfloat16", 5, [[3, 17, 99, 250, 7, 7, 128, 64, 1], [200, 4, 4, 8, 15, 16, 23, 42, 0]],
        [(0, 3), (3, 4)],
    ),
    "qwen3_tiny_fp32": (
        "qwen3",
        dict(vocab_size=97, hidden_size=32, intermediate_size=64, num_hidden_layers=4,
             num_attention_heads=4, num_key_value_heads=2, head_dim=8, max_position_embeddings=64,
             rms_norm_eps=1e-6, tie_word_embeddings=False, use_sliding_window=False),
        2, "float32", 23, [[4, 8, 15, 16, 23, 42]], [(0, 1), (1, 3), (3, 4)],
    ),
}


def reference_on_path(reference: Path, scratch: Path) -> None:
    src = scratch / "src"
    shutil.copytree(reference / "src", src)
    with tarfile.open(reference / TARBALL) as tar:
        keep = [m for m in tar.getmembers()
                if m.name.lstrip("./").startswith(("src/meshgpu/artifacts/", "src/meshgpu/checkpoints/"))]
        tar.extractall(scratch, members=keep, filter="data")
    sys.path.insert(0, str(src))


def shim_rope_config() -> None:
    from types import SimpleNamespace

    from meshgpu.artifacts import hf_import

    original = hf_import.hf_config_to_llama

    def hf_config_to_llama(hf_cfg):
        params = getattr(hf_cfg, "rope_parameters", None) or getattr(hf_cfg, "rope_scaling", None) or {}
        if params.get("rope_type", "default") != "default":
            return original(hf_cfg)
        names = ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
                 "num_key_value_heads", "head_dim", "max_position_embeddings", "rms_norm_eps",
                 "tie_word_embeddings", "hidden_act", "attention_bias", "mlp_bias")
        view = SimpleNamespace(**{k: getattr(hf_cfg, k) for k in names if hasattr(hf_cfg, k)})
        view.rope_scaling = None
        view.rope_theta = params.get("rope_theta", getattr(hf_cfg, "rope_theta", 10000.0))
        return original(view)

    hf_import.hf_config_to_llama = hf_config_to_llama


def greedy(workers, ids, steps):
    from meshgpu.backends.portable.pipeline import pipeline_decode_step, pipeline_prefill

    logits = pipeline_prefill(workers, ids, cache_key="g")
    prefill = logits.float().clone()
    tok = logits[:, -1].argmax(-1, keepdim=True)
    tokens, step_logits = [tok], []
    for k in range(steps):
        logits = pipeline_decode_step(workers, tok, operation_id=2 + k, cache_key="g")
        step_logits.append(logits[:, -1].float().clone())
        tok = logits[:, -1].argmax(-1, keepdim=True)
        tokens.append(tok)
    return prefill, torch.cat(tokens, 1), torch.stack(step_logits, 1)


def make(name: str, scratch: Path) -> None:
    from meshgpu.artifacts.hf_import import build_pipeline_from_manifest, import_from_hf
    from meshgpu.artifacts.qwen_import import import_qwen_from_hf
    from meshgpu.backends.portable.pipeline import pipeline_prefill

    family, kwargs, stages, dtype, seed, prompt, planned = CASES[name]
    torch.manual_seed(seed)
    if family == "qwen3":
        from transformers import Qwen3Config, Qwen3ForCausalLM

        model = Qwen3ForCausalLM(Qwen3Config(**kwargs)).eval()
    else:
        from transformers import LlamaConfig, LlamaForCausalLM

        model = LlamaForCausalLM(LlamaConfig(**kwargs)).eval()
    hf_dir = scratch / f"hf_{name}"
    model.save_pretrained(hf_dir, safe_serialization=True)
    out = OUT / name
    if out.exists():
        shutil.rmtree(out)
    importer = import_qwen_from_hf if family == "qwen3" else import_from_hf
    importer(str(hf_dir), stages, out, dtype=dtype, include_tokenizer=False)
    workers = build_pipeline_from_manifest(out)
    ids = torch.tensor(prompt)
    with torch.no_grad():
        prefill, tokens, steps = greedy(workers, ids, STEPS)
        planned_workers = build_pipeline_from_manifest(out, devices=[torch.device("cpu")] * len(planned),
                                                       layer_ranges=planned)
        planned_logits = pipeline_prefill(planned_workers, ids).float().clone()
    torch.save({
        "case": name, "family": family, "dtype": dtype, "stages": stages, "prompt": ids,
        "prefill": prefill, "tokens": tokens, "steps": steps,
        "planned_ranges": planned, "planned_prefill": planned_logits, "torch": str(torch.__version__),
    }, OUT / f"{name}.expected.pt")
    print(name, "ok", sorted(p.name for p in out.iterdir()))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a reference checkout")
    args = ap.parse_args()
    torch.set_num_threads(8)
    OUT.mkdir(exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:
        reference_on_path(Path(args.reference), Path(tmp))
        shim_rope_config()
        for name in CASES:
            make(name, Path(tmp))


if __name__ == "__main__":
    main()
