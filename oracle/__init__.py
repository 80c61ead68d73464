"""CPU oracle of the stage path — TEST INFRASTRUCTURE ONLY.

A restatement, in plain PyTorch CPU ops, of the reference's per-stage decoder
execution (hungtrab/gpu_mesh: src/meshgpu/models/llama_dense.py,
models/qwen3_hf.py via HF transformers' Qwen3 layers,
backends/portable/pipeline.py, inference/sampling.py).  Only the tests,
``__graft_entry__.smoke()`` and the CPU-baseline leg of bench.py may import it; the
product (``gpu_mesh_b200``) never does.  It is pinned against golden vectors
produced by running the reference itself (tests/golden/make_golden.py).
"""
