"""Decode throughput of the B200 stage executor (Llama-3-8B architecture).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload: Llama-3-8B geometry (32 layers, hidden 4096, 32 q / 8 KV heads,
head_dim 128, intermediate 14336, vocab 128256, RoPE theta 5e5), bf16,
synthetic random-init N(0, 0.02) weights, batch 32 as 4 micro-batches (request
contexts) of 8, prompts of 1024 uniform-random ids, greedy decode.  A step is
one decode token for all 32 rows.  N > 1 runs one pipeline stage per GPU
(launched by torchrun), layers split evenly, hidden states between stages over
NCCL, micro-batches in flight across stages.

The JSON line reports decode tok/s (device-timed, inputs resident), the same
metric end to end through the public API with host buffers (``e2e``), the
roofline of the dominant kernel (the weight-streaming decode GEMMs) and of
decode attention against the measured HBM copy bandwidth, and the CPU oracle
timed on the host cores as a baseline.  ``--impl reference`` times only that
CPU path (the reference's algorithm restated by the oracle; the reference
itself is Python code that does not travel to the GPU host).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from gpu_mesh_b200.clocks import ClockSampler  # noqa: E402

METRIC = "decode tok/s (Llama-3-8B arch, 1/2/4/8 B200 stages); attn-decode HBM % of peak"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0  # the same measurement held for seconds under the power cap

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one
# `ncu --set full` capture of the same kernels on the 2-layer case of this
# workload (identical per-layer shapes), next to the algorithmic bytes of the
# same launches.  gemv_tc: o_proj, gate/up, down of layer 0 in the first decode
# step (mean of the three); attn_tc: layers 0 and 1 of that step.
NCU_TRAFFIC = {
    "gemv_tc": {"dram_bytes": (33.84e6 + 244.04e6 + 123.12e6) / 3,
                "algorithmic_bytes": (34.07e6 + 236.06e6 + 118.88e6) / 3,
                "launches": "o_proj, gate/up, down of one layer at 32 rows"},
    "attn_tc": {"dram_bytes": (140.61e6 + 144.39e6) / 2,
                "algorithmic_bytes": 134.87e6,
                "launches": "decode attention of one layer, 32 rows x 8 KV heads x 1025 keys"},
}


def llama3_8b(layers: int = 32):
    from gpu_mesh_b200.config import LlamaConfig

    return LlamaConfig(
        vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=layers,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=8192,
        rms_norm_eps=1e-5, rope_theta=500000.0,
    )


# The scope's other benchmark architectures (--model): batch, prompt and
# sampling of their configurations; a step is one decode token for every row.
MODELS = {
    "llama3-8b": dict(arch="Llama-3-8B", layers=32, micro=8, micro_batches=4, prompt=1024, sampling="greedy"),
    "tinyllama-1.1b": dict(arch="TinyLlama-1.1B", layers=22, micro=8, micro_batches=1, prompt=512,
                           sampling="greedy"),
    "qwen3-4b": dict(arch="Qwen3-4B", layers=36, micro=16, micro_batches=1, prompt=2048,
                     sampling="top-p (T 0.7, p 0.9, seeded)"),
}
TOP_P = (0.7, 0.9)


def model_config(name: str, layers: int | None = None):
    from gpu_mesh_b200.config import LlamaConfig

    n = layers or MODELS[name]["layers"]
    if name == "llama3-8b":
        return llama3_8b(n)
    if name == "tinyllama-1.1b":
        return LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632, num_hidden_layers=n,
                           num_attention_heads=32, num_key_value_heads=4, head_dim=64,
                           max_position_embeddings=4096, rms_norm_eps=1e-5, rope_theta=10000.0)
    return LlamaConfig(vocab_size=151936, hidden_size=2560, intermediate_size=9728, num_hidden_layers=n,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=8192,
                       rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=True, qk_norm=True,
                       mask_policy="cache")


def other_configs(world: int) -> list[dict]:
    """The scope's configurations that name this stage count, measured beside
    the headline line of an N-GPU run: TinyLlama-1.1B on 2 stages; Qwen3-4B
    (top-p) on 2 and 4; the long-context Llama-3-8B stress (64 rows, caches
    pre-filled to 8192 positions) on 8."""
    out = []
    if world == 2:
        out.append({"name": "tinyllama-1.1b", "cfg": model_config("tinyllama-1.1b"), "rows": 8, "prompt": 512,
                    "note": "TinyLlama-1.1B arch, bf16, batch 8, 512-token prompts, greedy"})
    if world in (2, 4):
        out.append({"name": "qwen3-4b", "cfg": model_config("qwen3-4b"), "rows": 16, "prompt": 2048,
                    "top_p": TOP_P, "note": "Qwen3-4B arch, bf16, batch 16, 2048-token prompts, top-p "
                                            "(T 0.7, p 0.9, seeded)"})
    if world == 8:
        cfg = llama3_8b(32)
        cfg.max_position_embeddings = 8192 + 256
        out.append({"name": "llama3-8b-long-context", "cfg": cfg, "rows": 64, "context": 8192,
                    "note": "Llama-3-8B arch, bf16, batch 64, every stage's caches pre-filled to 8192 "
                            "positions with N(0,1), greedy"})
    return out


def metric_for(args) -> str:
    if args.model == "llama3-8b":
        return METRIC
    return f"decode tok/s ({MODELS[args.model]['arch']} arch, B200 stages)"


def peaks() -> tuple[float, float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def sustained_bf16_tflops() -> float:
    """The measured bf16 GEMM rate held for seconds under the power cap (a
    prefill is seconds of back-to-back GEMMs), else the fallback figure."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"])
    return FALLBACK_BF16_TFLOPS_SUSTAINED


def prefill_flops(cfg, rows: int, prompt: int) -> float:
    """Algorithmic FLOPs of a prefill of `rows` prompts of `prompt` tokens:
    the four projections of every layer, causal attention (QK^T and PV over
    the visible keys) and the lm_head of the last position."""
    H, I, D = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    nq, nkv, L = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.num_hidden_layers
    M = rows * prompt
    linear = 2.0 * M * H * (nq + 2 * nkv) * D + 2.0 * M * nq * D * H + 2.0 * M * H * 2 * I + 2.0 * M * I * H
    attn = 4.0 * rows * nq * D * (prompt * (prompt + 1) / 2)
    return L * (linear + attn) + 2.0 * rows * H * cfg.vocab_size


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (the reference's algorithm) on the host cores
# ---------------------------------------------------------------------------

def cpu_baseline(cfg, *, micro: int, micro_batches: int, context: int, steps: int, warmup: int = 1,
                 weights_from=None) -> dict:
    """Time the CPU oracle on the decode workload's own step.

    One step decodes one token for every row: ``micro_batches`` request
    contexts of ``micro`` rows, each a separate KV cache, decoded one context
    after the other through all layers and the lm_head, as the reference's
    pipeline_decode_step does per cache_key.  Every layer's cache is
    pre-filled to ``context`` positions with N(0, 1) bf16 values (the cost of
    a decode step does not depend on how the prefix was produced, and a CPU
    prefill of the prompts would take hours).  ``warmup`` untimed steps, then
    exactly ``steps`` timed steps.
    """
    from oracle import stage_ref as R

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from gpu_mesh_b200.weights import synthetic_tensor, stage_keys

    state = {}
    for local, global_key, shape in stage_keys(cfg, 0, cfg.num_hidden_layers, True, True):
        if weights_from is not None and local in weights_from:
            state[local] = weights_from[local]
        else:
            dev = "cuda" if torch.cuda.is_available() else "cpu"
            state[local] = synthetic_tensor(global_key, shape, seed=0, dtype=torch.bfloat16, device=dev).cpu()
    st = R.OracleStage(cfg, 0, cfg.num_hidden_layers, True, True, state, torch.bfloat16)
    g = torch.Generator().manual_seed(0)
    keys = [f"mb{i}" for i in range(micro_batches)]
    ids = {}
    for key in keys:
        kv = []
        for _ in range(cfg.num_hidden_layers):
            shape = (micro, cfg.num_key_value_heads, context, cfg.head_dim)
            kv.append((torch.randn(shape, generator=g).to(torch.bfloat16),
                       torch.randn(shape, generator=g).to(torch.bfloat16)))
        st.caches[key] = kv
        ids[key] = torch.randint(0, cfg.vocab_size, (micro, 1), generator=g)

    def step() -> None:
        for key in keys:
            logits = st.forward(input_ids=ids[key], key=key)
            ids[key] = R.greedy(logits[:, -1]).unsqueeze(-1)

    with torch.no_grad():
        for _ in range(warmup):
            step()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        dt = time.perf_counter() - t0
    rows = micro * micro_batches
    return {
        "value": rows * steps / dt,
        "unit": "tok/s",
        "cores": threads,
        "kind": "port",
        "sample": (f"oracle (CPU restatement of the reference stage), {cfg.num_hidden_layers} layers bf16, "
                   f"{rows} rows as {micro_batches} request contexts of {micro} decoded one after the other, "
                   f"KV pre-filled to {context} positions with N(0,1), {warmup} untimed + {steps} timed "
                   f"greedy decode steps, {threads} threads"),
        "steps": steps,
        "seconds": dt,
    }


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = model_config(args.model, args.layers)
    # The reference's algorithm on the host cores: exactly --steps timed steps of
    # the full batch (all rows, every context), after one untimed step.
    base = cpu_baseline(cfg, micro=args.micro, micro_batches=args.micro_batches, context=args.prompt,
                        steps=args.steps, warmup=1)
    rows = args.micro * args.micro_batches
    line = {
        "impl": "reference",
        "metric": metric_for(args),
        "value": base["value"],
        "unit": "tok/s",
        "n_gpus": args.gpus,
        "steps": base["steps"],
        "warmup": 1,
        "ms_per_step": 1000.0 * base["seconds"] / base["steps"],
        "rows_per_step": rows,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": workload_config(args),
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args) -> dict:
    m = MODELS[args.model]
    layers = "" if args.layers == m["layers"] else f" cut to {args.layers} layers (profiling case)"
    sampling = "greedy" if m["sampling"] == "greedy" else m["sampling"]
    return {
        "workload": f"{m['arch']}-architecture{layers} bf16 {sampling} decode, batch "
                    f"{args.micro * args.micro_batches} as {args.micro_batches} micro-batches of "
                    f"{args.micro}, {args.prompt}-token prompts",
        "layers": args.layers,
        "batch": args.micro * args.micro_batches,
        "micro_batches": args.micro_batches,
        "prompt": args.prompt,
        "stages": args.gpus,
        "parallelism": f"pp{args.gpus}",
        "l2": "inputs larger than L2: every step streams all weights and the KV caches",
    }


# ---------------------------------------------------------------------------
# Long-context decode attention (one of eight 4-layer stages)
# ---------------------------------------------------------------------------

def long_context(hbm: float, *, rows: int = 64, context: int = 8192, layers: int = 4, steps: int = 8) -> dict:
    """Decode through one middle stage of the Llama-3-8B geometry (4 layers,
    what each GPU of an 8-stage pipeline holds) for 64 rows whose KV caches
    are pre-filled to 8192 positions with N(0, 1) values: attention streams
    2.15 GB of keys and values per layer per step against 0.44 GB of weights.
    Returns decode tok/s of the stage and the attention kernels' HBM rate
    from the per-launch CUDA events."""
    from gpu_mesh_b200 import B200Stage
    from gpu_mesh_b200.weights import synthetic_stage_state

    cfg = llama3_8b(layers)
    cfg.max_position_embeddings = context + 2 * steps + 64  # the cache plus the decoded tokens
    dev = torch.device("cuda", 0)
    state = synthetic_stage_state(cfg, 0, layers, has_embedding=False, has_lm_head=False, seed=0,
                                  dtype=torch.bfloat16, device=dev)
    stage = B200Stage(cfg, 0, layers, has_embedding=False, has_lm_head=False, device=dev,
                      dtype=torch.bfloat16, state_dict=state)
    del state
    g = torch.Generator(device=dev).manual_seed(5)
    nkv, D = cfg.num_key_value_heads, cfg.head_dim
    stage.kv_reserve(0, rows, context + steps + 8)
    for layer in range(layers):
        k = torch.randn(rows, nkv, context, D, generator=g, device=dev, dtype=torch.bfloat16)
        v = torch.randn(rows, nkv, context, D, generator=g, device=dev, dtype=torch.bfloat16)
        stage.kv_import(0, layer, k, v)
        del k, v
    x = (torch.randn(rows, 1, cfg.hidden_size, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    for _ in range(2):  # warm-up
        stage.forward_slot(0, x)
    stage.kv_trim(0, context)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        stage.forward_slot(0, x)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    stage.kv_trim(0, context)
    stage.profile(True)
    for _ in range(steps):
        stage.forward_slot(0, x)
    prof = stage.profile_read()
    stage.profile(False)
    stage.close()
    att = prof["attention"]
    att_gbs = att["bytes"] / (att["ms"] / 1000.0) / 1e9 if att["ms"] else 0.0
    return {
        "workload": (f"one middle stage of 4 Llama-3-8B layers, {rows} rows, KV pre-filled to {context} "
                     "positions with N(0,1), single-token decode"),
        "stage_tok_s": rows / (ms / 1000.0),
        "ms_per_step": ms,
        "attention": {"achieved": att_gbs, "peak": hbm, "unit": "GB/s", "frac": att_gbs / hbm,
                      "bytes_per_step": att["bytes"] / steps, "share_of_step": att["ms"] / sum(
                          p["ms"] for p in prof.values())},
    }


def prefill_attention_rate(worker, cfg, prompt) -> dict:
    """Causal prefill attention of one micro-batch: this stage's tcgen05
    kernel (every layer's launch bracketed by CUDA events during a prefill of
    ``prompt`` into a scratch context) next to the library path the
    reference would reach on this GPU, torch's scaled_dot_product_attention
    (bf16, causal, GQA) on the same shape.  Reported only; the library is
    not on the stage's path."""
    stage = worker._model
    B, S = prompt.shape
    stage.profile(True)
    worker.forward_inference(None, input_ids=prompt, operation_id=1, attempt_id="pa", cache_key="pa",
                             logits="last")
    att = stage.profile_read()["attention"]
    stage.profile(False)
    worker.clear_kv("pa")
    ours = att["flops"] / (att["ms"] / 1000.0) / 1e12 if att["ms"] else None
    nq, nkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    g = torch.Generator(device=prompt.device).manual_seed(9)
    q = torch.randn(B, nq, S, D, generator=g, device=prompt.device, dtype=torch.bfloat16)
    k = torch.randn(B, nkv, S, D, generator=g, device=prompt.device, dtype=torch.bfloat16)
    v = torch.randn(B, nkv, S, D, generator=g, device=prompt.device, dtype=torch.bfloat16)
    sdpa = torch.nn.functional.scaled_dot_product_attention
    for _ in range(3):
        sdpa(q, k, v, is_causal=True, enable_gqa=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record()
    for _ in range(reps):
        sdpa(q, k, v, is_causal=True, enable_gqa=True)
    e1.record()
    torch.cuda.synchronize()
    flops = 4.0 * B * nq * D * (S * (S + 1) / 2)
    lib = flops / (e0.elapsed_time(e1) / reps / 1000.0) / 1e12
    return {"shape": f"{B} rows x {S} tokens, {nq} q / {nkv} KV heads, head_dim {D}, causal",
            "b200_tflops": ours, "sdpa_tflops": lib, "unit": "TFLOP/s",
            "note": "b200: attn_prefill_tc per layer, event-bracketed; sdpa: torch's default backend, "
                    "reported for comparison only"}


# ---------------------------------------------------------------------------
# B200 arm, one GPU
# ---------------------------------------------------------------------------

def run_single(args) -> None:
    from gpu_mesh_b200 import _lib, build_pipeline, greedy_sample
    from gpu_mesh_b200.pipeline import pipeline_decode_greedy, pipeline_decode_top_p

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = model_config(args.model, args.layers)
    greedy = MODELS[args.model]["sampling"] == "greedy"
    sample_gen = torch.Generator(device=dev).manual_seed(1234)
    hbm, tflops, peak_kind = peaks()
    workers = build_pipeline(cfg, 1, [dev], transport="local_cuda", dtype=torch.bfloat16, check_values=False)
    w = workers[0]
    stage = w._model
    keys = [f"mb{i}" for i in range(args.micro_batches)]
    cap = args.prompt + args.warmup + 3 * args.steps + 16
    for k in keys:
        w.reserve_kv(k, args.micro, cap)
    g = torch.Generator().manual_seed(1000)
    prompts = [torch.randint(0, cfg.vocab_size, (args.micro, args.prompt), generator=g) for _ in keys]

    # Prefill every micro-batch (timed for the report, not the headline).
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    first = []
    for k, p in zip(keys, prompts):
        logits = w.forward_inference(None, input_ids=p.to(dev), operation_id=1, attempt_id="b",
                                     cache_key=k, logits="last").output
        first.append(greedy_sample(logits[:, -1]))
    t1.record()
    torch.cuda.synchronize()
    prefill_ms = t0.elapsed_time(t1)
    stage.check_device()  # a kernel that gave up waiting would make every number below meaningless
    ids = torch.cat(first).unsqueeze(-1)

    # The CPU baseline runs here, between the prefill and the decode region:
    # under the prefill's GEMMs the power controller lowers the SM clock
    # (1.44 GHz measured right after it), and it takes about 100 ms of decode
    # to climb back to the 1.965 GHz a decode loop holds.  With the GPU idle
    # while the host cores time the oracle, the decode region is measured at
    # the clock decode runs at, not during that recovery.
    base = None
    if not args.no_cpu_baseline:
        # bounded sample: 3 steps of the full batch (about 10 s of CPU work)
        base = cpu_baseline(cfg, micro=args.micro, micro_batches=args.micro_batches, context=args.prompt,
                            steps=3, warmup=1)

    rows_all = args.micro * args.micro_batches

    def step(ids):
        if greedy:
            tokens, _ = w.decode_greedy(None, keys, input_ids=ids)  # selection fused into lm_head
        else:  # top-p drawn from the value histograms counted in lm_head's epilogue
            u = torch.rand(rows_all, generator=sample_gen, device=dev)
            tokens, _ = w.decode_top_p(None, keys, input_ids=ids, temperature=TOP_P[0], top_p=TOP_P[1],
                                       uniforms=u)
        return tokens.unsqueeze(-1)

    for _ in range(args.warmup):
        ids = step(ids)
    torch.cuda.synchronize()
    launches0 = _lib.lib().mg_launch_count()
    with ClockSampler(0) as clocks:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            ids = step(ids)
        e1.record()
        torch.cuda.synchronize()
    launches = _lib.lib().mg_launch_count() - launches0
    ms = e0.elapsed_time(e1)
    rows = args.micro * args.micro_batches
    value = rows * args.steps / (ms / 1000.0)

    # The same K steps again with every launch group bracketed by CUDA events
    # on the stage's stream: per-kernel-class device time for the roofline.
    stage.profile(True)
    for _ in range(args.steps):
        ids = step(ids)
    prof = stage.profile_read()
    stage.profile(False)

    # End to end through the public API: host ids in, host tokens out, every step.
    host_ids = ids.cpu().pin_memory()
    host_out = torch.empty_like(host_ids).pin_memory()
    torch.cuda.synchronize()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record()
    for _ in range(args.steps):
        d_ids = host_ids.to(dev, non_blocking=True)
        if greedy:
            tok, _ = pipeline_decode_greedy(workers, d_ids, cache_keys=keys)
        else:
            tok, _ = pipeline_decode_top_p(workers, d_ids, cache_keys=keys, temperature=TOP_P[0],
                                           top_p=TOP_P[1], generator=sample_gen)
        tok = tok.unsqueeze(-1)
        host_out.copy_(tok, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        host_ids.copy_(host_out)
    e3.record()
    torch.cuda.synchronize()
    e2e_ms = e2.elapsed_time(e3)
    stage.check_device()
    # Prefill attention beside torch's SDPA (GEMM-heavy: after the decode region).
    prefill_attention = prefill_attention_rate(w, cfg, prompts[0].to(dev))

    lin = prof["linear_decode"]
    att = prof["attention"]
    lin_gbs = lin["bytes"] / (lin["ms"] / 1000.0) / 1e9 if lin["ms"] else 0.0
    att_gbs = att["bytes"] / (att["ms"] / 1000.0) / 1e9 if att["ms"] else 0.0
    step_bytes = sum(p["bytes"] for p in prof.values()) / args.steps
    prof_ms = sum(p["ms"] for p in prof.values())

    # Free the 8B stage before the long-context stage.
    for k in keys:
        w.clear_kv(k)
    for wk in workers:
        wk.close()
    del workers, w, stage
    torch.cuda.empty_cache()
    longctx = None if args.no_long_context or args.model != "llama3-8b" else long_context(hbm)

    traffic = NCU_TRAFFIC if args.model == "llama3-8b" else {
        k: {"dram_bytes": None, "algorithmic_bytes": None, "launches": None} for k in NCU_TRAFFIC}
    line = {
        "metric": metric_for(args),
        "value": value,
        "unit": "tok/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights, uniform-random prompt ids)",
        "config": workload_config(args),
        "roofline": {
            "bound": "hbm",
            "kernel": "gemv_tc (stream-K tcgen05 decode GEMM: qkv, o, gate/up, down, lm_head)",
            "achieved": lin_gbs,
            "peak": hbm,
            "unit": "GB/s",
            "frac": lin_gbs / hbm,
            "traffic": traffic["gemv_tc"]["dram_bytes"],
            "traffic_algorithmic": traffic["gemv_tc"]["algorithmic_bytes"],
            "traffic_launches": traffic["gemv_tc"]["launches"],
            "peak_kind": peak_kind,
            "share_of_step": lin["ms"] / prof_ms if prof_ms else None,
        },
        "attention_roofline": {
            "bound": "hbm",
            "kernel": "attn_tc (persistent decode attention over the stage-owned KV)",
            "achieved": att_gbs,
            "peak": hbm,
            "unit": "GB/s",
            "frac": att_gbs / hbm,
            "traffic": traffic["attn_tc"]["dram_bytes"],
            "traffic_algorithmic": traffic["attn_tc"]["algorithmic_bytes"],
            "traffic_launches": traffic["attn_tc"]["launches"],
            "share_of_step": att["ms"] / prof_ms if prof_ms else None,
        },
        "step_roofline": {
            "bytes_per_step": step_bytes,
            "achieved_gbs": step_bytes / (ms / args.steps / 1000.0) / 1e9,
            "frac": step_bytes / (ms / args.steps / 1000.0) / 1e9 / hbm,
        },
        "e2e": {
            "value": rows * args.steps / (e2e_ms / 1000.0),
            "unit": "tok/s",
            "h2d_bytes_per_step": rows * 8,
            "d2h_bytes_per_step": rows * 8,
        },
        "prefill": {
            "tok_s": rows * args.prompt / (prefill_ms / 1000.0),
            "ms": prefill_ms,
            "tflops": prefill_flops(cfg, rows, args.prompt) / (prefill_ms / 1000.0) / 1e12,
            "sustained_peak_tflops": sustained_bf16_tflops(),
            "frac_of_sustained": prefill_flops(cfg, rows, args.prompt) / (prefill_ms / 1000.0) / 1e12
            / sustained_bf16_tflops(),
        },
        "gpu_launches": int(launches),
        "prefill_attention": prefill_attention,
        "profile": prof,
        "clocks": clocks.summary(),
    }
    if longctx is not None:
        line["long_context"] = longctx
    if base is not None:
        line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--model", choices=sorted(MODELS), default="llama3-8b",
                    help="architecture and its configuration (batch, prompt, sampling)")
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--micro", type=int, default=None)
    ap.add_argument("--micro-batches", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder layers (default: the model's; fewer only for profiling captures)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-weak", action="store_true",
                    help="N > 1: skip the weak-scaling measurement (N groups of 32 rows in flight)")
    ap.add_argument("--nccl-sms", type=int, default=8,
                    help="N > 1: SMs each GPU leaves out of its persistent kernels for NCCL's kernels")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="N > 1: skip the other configurations named at this stage count")
    ap.add_argument("--even-split", action="store_true",
                    help="N > 1: the reference's even layer split instead of ranges that even out the "
                         "bytes each stage streams")
    ap.add_argument("--no-long-context", action="store_true",
                    help="skip the long-context attention measurement (64 rows x 8192 positions)")
    args = ap.parse_args()
    for k in ("prompt", "micro", "micro_batches", "layers"):
        if getattr(args, k) is None:
            setattr(args, k, MODELS[args.model][k])
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference_arm(args)
        return
    if args.gpus == 1 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        run_single(args)
        return
    from gpu_mesh_b200.dist import run_pipeline_bench

    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    run_pipeline_bench(args, model_config(args.model, args.layers), metric_for(args), workload_config(args), peaks(),
                       NCU_TRAFFIC if args.model == "llama3-8b" else None,
                       top_p=None if MODELS[args.model]["sampling"] == "greedy" else TOP_P,
                       other_configs=[] if args.no_other_configs or args.model != "llama3-8b"
                       else other_configs(world))


if __name__ == "__main__":
    main()
