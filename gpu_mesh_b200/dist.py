"""Multi-GPU pipeline: one stage per process/GPU, hidden states over NCCL.

The reference runs its stages strictly in sequence for one request batch
(backends/portable/pipeline.py:210-228) and moves boundaries with
``Tensor.to`` (transport/local_cuda.py:57-90).  Here each GPU is one
process (torchrun), each stage owns its layers and the KV of every group,
and G groups of request contexts are in flight so that stage s works on one
group while stage s+1 works on the previous one.  The only exchanges are
point-to-point: the hidden state of a group to the next stage, and the
sampled token ids from the last stage back to stage 0.

``decode_loop`` is the schedule.  It is device-agnostic (the compute and
sampling functions are arguments) so the same code runs on NCCL/GPU in the
benchmark and on gloo/CPU in the tests.  Hidden states and returning ids
use two communicators, so the return path never queues behind the forward
path.
"""
from __future__ import annotations

import json
import os
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist


@dataclass
class Ring:
    rank: int
    world: int

    @property
    def first(self) -> bool:
        return self.rank == 0

    @property
    def last(self) -> bool:
        return self.rank == self.world - 1


def decode_loop(
    ring: Ring,
    n_groups: int,
    n_steps: int,
    first_inputs: Sequence[torch.Tensor] | None,
    forward: Callable[[int, int, torch.Tensor], torch.Tensor],
    sample: Callable[[int, int, torch.Tensor], torch.Tensor],
    recv_hidden: Callable[[int, int], torch.Tensor],
    recv_ids: Callable[[int], torch.Tensor],
    *,
    fwd_group=None,
    ret_group=None,
) -> list[torch.Tensor] | None:
    """Run ``n_steps`` pipeline steps for ``n_groups`` groups.

    Iterations are (step k, group g) in order k-major.  Stage 0's input for
    (k, g) is ``first_inputs[g]`` at k = 0 and the ids sampled for (k-1, g)
    afterwards; other stages receive the previous stage's output.  The last
    stage samples every iteration and sends the ids to stage 0, which
    receives the ids of the final step after the loop and returns them (the
    inputs of the next call).  ``recv_hidden(k, g)`` / ``recv_ids(g)`` give
    receive buffers.

    Hidden states travel on ``fwd_group`` (a chain: stage r -> r + 1) and ids
    on ``ret_group`` (last stage -> stage 0), two communicators with their own
    ordering, so the return path never queues behind the forward path (one
    shared channel deadlocks as soon as more groups than stages are in
    flight).  Receives are posted non-blocking as soon as their buffer is
    free; every send is waited for at the end of its iteration.  Returns the
    final ids on stage 0, else None.
    """
    it = [(k, g) for k in range(n_steps) for g in range(n_groups)]
    world, rank = ring.world, ring.rank
    pending_in = None
    if not ring.first and it:
        buf = recv_hidden(*it[0])
        pending_in = (buf, dist.irecv(buf, src=rank - 1, group=fwd_group))
    returning: dict[int, tuple[torch.Tensor, object]] = {}
    for i, (k, g) in enumerate(it):
        if ring.first:
            if k == 0:
                x = first_inputs[g]
            else:
                x, work = returning.pop(g)
                work.wait()
        else:
            x, work = pending_in
            work.wait()
        out = forward(k, g, x)
        sends = []
        if ring.last:
            ids = sample(k, g, out)
            if world > 1:
                sends.append(dist.isend(ids, dst=0, group=ret_group))
        else:
            sends.append(dist.isend(out, dst=rank + 1, group=fwd_group))
        if ring.first and world > 1:
            buf = recv_ids(g)
            returning[g] = (buf, dist.irecv(buf, src=world - 1, group=ret_group))
        if not ring.first and i + 1 < len(it):
            buf = recv_hidden(*it[i + 1])
            pending_in = (buf, dist.irecv(buf, src=rank - 1, group=fwd_group))
        for work in sends:
            work.wait()
    if ring.first and world > 1:
        finals = []
        for g in range(n_groups):
            buf, work = returning.pop(g)
            work.wait()
            finals.append(buf.clone())
        return finals
    return None


# ---------------------------------------------------------------------------
# Benchmark on N GPUs (torchrun)
# ---------------------------------------------------------------------------

def run_pipeline_bench(args, cfg, metric: str, workload: dict, peaks: tuple[float, float, str],
                       traffic: dict | None = None, top_p: tuple[float, float] | None = None) -> None:
    """``top_p`` = (temperature, p): the last stage samples with a seeded device
    generator instead of selecting greedily inside its lm_head."""
    from gpu_mesh_b200 import greedy_sample
    from gpu_mesh_b200.sampling import top_p_sample
    from gpu_mesh_b200.config import split_layers
    from gpu_mesh_b200.stage import B200Stage
    from gpu_mesh_b200.weights import synthetic_stage_state

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    ring = Ring(rank, world)
    try:
        hbm, _, peak_kind = peaks
        ls, le = split_layers(cfg.num_hidden_layers, world)[rank]
        sd = synthetic_stage_state(cfg, ls, le, has_embedding=ring.first, has_lm_head=ring.last,
                                   seed=0, dtype=torch.bfloat16, device=dev)
        stage = B200Stage(cfg, ls, le, has_embedding=ring.first, has_lm_head=ring.last, device=dev,
                          dtype=torch.bfloat16, state_dict=sd)
        del sd
        torch.cuda.empty_cache()

        rows_total = args.micro * args.micro_batches
        n_groups = max(world, 1)
        if rows_total % n_groups:
            raise ValueError(f"{rows_total} rows do not split into {n_groups} groups")
        rows = rows_total // n_groups
        H = cfg.hidden_size
        slots = list(range(1, n_groups + 1))
        cap = args.prompt + args.warmup + 3 * args.steps + 16
        for sl in slots:
            stage.kv_reserve(sl, rows, cap)

        g = torch.Generator().manual_seed(1000)
        prompts = [torch.randint(0, cfg.vocab_size, (rows, args.prompt), generator=g).to(dev)
                   for _ in range(n_groups)]
        hid_prefill = [torch.empty(rows, args.prompt, H, dtype=torch.bfloat16, device=dev)
                       for _ in range(n_groups)]
        hid_decode = [torch.empty(rows, 1, H, dtype=torch.bfloat16, device=dev) for _ in range(n_groups)]
        ids_bufs = [torch.empty(rows, 1, dtype=torch.int64, device=dev) for _ in range(n_groups)]

        def forward_prefill(k, grp, x):
            if ring.first:
                return stage.forward_slot(slots[grp], None, input_ids=x, logits="last", check_values=False)
            return stage.forward_slot(slots[grp], x, logits="last", check_values=False)

        sample_gen = torch.Generator(device=dev).manual_seed(1234)

        def decode_on(slot_ids, x):
            # the last stage selects the greedy tokens inside its lm_head
            if ring.last and top_p is None:
                return stage.decode_greedy(slot_ids, None if ring.first else x,
                                           input_ids=x if ring.first else None)[0]
            if ring.first:
                return stage.decode_multi(slot_ids, None, input_ids=x, logits="last")
            return stage.decode_multi(slot_ids, x, logits="last")

        def forward_decode(k, grp, x):
            return decode_on([slots[grp]], x)

        def tokens_of(out):
            if out.dtype == torch.int64:  # already selected by decode_greedy
                return out.view(-1, 1)
            if top_p is not None:
                return top_p_sample(out[:, -1], *top_p, generator=sample_gen).unsqueeze(-1)
            return greedy_sample(out[:, -1]).unsqueeze(-1)

        def sample(k, grp, out):
            return tokens_of(out).contiguous()

        host_ids = torch.empty(rows, 1, dtype=torch.int64).pin_memory()

        def sample_host(k, grp, out):
            ids = tokens_of(out)
            host_ids.copy_(ids, non_blocking=True)  # the server reads every token
            torch.cuda.current_stream().synchronize()
            return host_ids.to(dev, non_blocking=True)

        ret_group = dist.new_group(list(range(world)))

        def run(n_steps, inputs, fwd, smp, hid):
            return decode_loop(ring, n_groups, n_steps, inputs, fwd, smp,
                               lambda k, grp: hid[grp], lambda grp: ids_bufs[grp],
                               ret_group=ret_group)

        def timed(fn):
            dist.barrier()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn()
            e1.record()
            torch.cuda.synchronize()
            ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            return out, float(ms.item())

        # One untimed prefill first (the communicators connect and every kernel
        # is configured on first use), then the caches are rolled back.
        timed(lambda: run(1, prompts, forward_prefill, sample, hid_prefill))
        for sl in slots:
            stage.kv_trim(sl, 0)
        ids, prefill_ms = timed(lambda: run(1, prompts, forward_prefill, sample, hid_prefill))
        ids, _ = timed(lambda: run(args.warmup, ids, forward_decode, sample, hid_decode))
        launches0 = _launches()
        from contextlib import nullcontext

        from gpu_mesh_b200.clocks import ClockSampler

        with (ClockSampler(local) if ring.first else nullcontext()) as clocks:
            ids, ms = timed(lambda: run(args.steps, ids, forward_decode, sample, hid_decode))
        launches = _launches() - launches0
        stage.profile(True)
        ids, _ = timed(lambda: run(args.steps, ids, forward_decode, sample, hid_decode))
        prof = stage.profile_read()
        stage.profile(False)
        ids, e2e_ms = timed(lambda: run(args.steps, ids, forward_decode, sample_host, hid_decode))

        # Weak scaling: the same per-GPU work at a batch that grows with N
        # (N groups of 32 rows in flight: every GPU streams its weights N
        # times per step, as one GPU streams all weights once for 32 rows).
        weak = None
        if world > 1 and not getattr(args, "no_weak", False):
            for sl in slots:
                stage.kv_free(sl)
            torch.cuda.empty_cache()
            rows_w = rows_total
            slots_w = list(range(101, 101 + n_groups))
            for sl in slots_w:
                stage.kv_reserve(sl, rows_w, cap)
            gw = torch.Generator().manual_seed(2000)
            prompts_w = [torch.randint(0, cfg.vocab_size, (rows_w, args.prompt), generator=gw).to(dev)
                         for _ in range(n_groups)]
            hid_pw = [torch.empty(rows_w, args.prompt, H, dtype=torch.bfloat16, device=dev)
                      for _ in range(n_groups)]
            hid_dw = [torch.empty(rows_w, 1, H, dtype=torch.bfloat16, device=dev) for _ in range(n_groups)]
            ids_w = [torch.empty(rows_w, 1, dtype=torch.int64, device=dev) for _ in range(n_groups)]

            def fwd_pw(k, grp, x):
                if ring.first:
                    return stage.forward_slot(slots_w[grp], None, input_ids=x, logits="last", check_values=False)
                return stage.forward_slot(slots_w[grp], x, logits="last", check_values=False)

            def fwd_dw(k, grp, x):
                return decode_on([slots_w[grp]], x)

            def run_w(n_steps, inputs, fwd, hid):
                return decode_loop(ring, n_groups, n_steps, inputs, fwd, sample,
                                   lambda k, grp: hid[grp], lambda grp: ids_w[grp], ret_group=ret_group)

            idw, _ = timed(lambda: run_w(1, prompts_w, fwd_pw, hid_pw))
            idw, _ = timed(lambda: run_w(args.warmup, idw, fwd_dw, hid_dw))
            idw, ms_w = timed(lambda: run_w(args.steps, idw, fwd_dw, hid_dw))
            weak = {
                "scaling": "weak",
                "rows": rows_w * n_groups,
                "groups_in_flight": n_groups,
                "rows_per_group": rows_w,
                "value": rows_w * n_groups * args.steps / (ms_w / 1000.0),
                "unit": "tok/s",
                "ms_per_step": ms_w / args.steps,
                "note": "per-GPU work of the one-GPU workload (32 rows through every layer once per step)",
            }

        profs = [None] * world
        dist.all_gather_object(profs, prof)
        counts = [0] * world
        dist.all_gather_object(counts, launches)
        if ring.first:
            lin = [p["linear_decode"] for p in profs]
            att = [p["attention"] for p in profs]
            lin_b, lin_ms = sum(p["bytes"] for p in lin), sum(p["ms"] for p in lin)
            att_b, att_ms = sum(p["bytes"] for p in att), sum(p["ms"] for p in att)
            lin_gbs = lin_b / (lin_ms / 1000) / 1e9 if lin_ms else 0.0
            att_gbs = att_b / (att_ms / 1000) / 1e9 if att_ms else 0.0
            line = {
                "metric": metric,
                "value": rows_total * args.steps / (ms / 1000.0),
                "unit": "tok/s",
                "n_gpus": world,
                "steps": args.steps,
                "warmup": args.warmup,
                "ms_per_step": ms / args.steps,
                "higher_is_better": True,
                "scaling": "strong",
                "vs_baseline": None,
                "dtype": "bf16",
                "data": "synthetic (random-init N(0,0.02) weights, uniform-random prompt ids)",
                "config": {**workload, "stages": world, "parallelism": f"pp{world}",
                           "groups_in_flight": n_groups, "rows_per_group": rows},
                # Bytes and kernel time are summed over the stages, each on its
                # own GPU, so the ratios are per-GPU rates.
                "roofline": {
                    "bound": "hbm",
                    "kernel": "gemv_tc (stream-K tcgen05 decode GEMM), mean over stages",
                    "achieved": lin_gbs,
                    "peak": hbm,
                    "unit": "GB/s",
                    "frac": lin_gbs / hbm,
                    "traffic": (traffic or {}).get("gemv_tc", {}).get("dram_bytes"),
                    "traffic_algorithmic": (traffic or {}).get("gemv_tc", {}).get("algorithmic_bytes"),
                    "peak_kind": peak_kind,
                },
                "attention_roofline": {
                    "bound": "hbm",
                    "kernel": "attn_tc + attn_combine, mean over stages",
                    "achieved": att_gbs,
                    "peak": hbm,
                    "unit": "GB/s",
                    "frac": att_gbs / hbm,
                    "traffic": (traffic or {}).get("attn_tc", {}).get("dram_bytes"),
                    "traffic_algorithmic": (traffic or {}).get("attn_tc", {}).get("algorithmic_bytes"),
                },
                "e2e": {
                    "value": rows_total * args.steps / (e2e_ms / 1000.0),
                    "unit": "tok/s",
                    "h2d_bytes_per_step": rows_total * 8,
                    "d2h_bytes_per_step": rows_total * 8,
                },
                "prefill": {"tok_s": rows_total * args.prompt / (prefill_ms / 1000.0), "ms": prefill_ms},
                "gpu_launches": int(sum(counts)),
                "per_stage_profile": profs,
                "clocks": clocks.summary(),
            }
            if weak is not None:
                line["weak_scaling"] = weak
            print(json.dumps(line), flush=True)
        stage.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _launches() -> int:
    from gpu_mesh_b200 import _lib

    return int(_lib.lib().mg_launch_count())
