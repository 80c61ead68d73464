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
sampling functions are arguments) so the same code runs on NCCL/GPU and on
gloo/CPU in the tests.  Hidden states and returning ids use two
communicators, so the return path never queues behind the forward path.

``PipelineRank`` is the public entry: this process's stage of an N-process
pipeline, with ``prefill`` and ``decode`` over groups of request contexts in
flight (greedy inside the last stage's lm_head, or top-p), optional host
round trips of the sampled ids, and a record of every id the last stage
produced.  ``verify_one_gpu`` replays a recorded run on one GPU with the
whole model, teacher-forced on the pipeline's own ids, and reports every
token where the two differ with the one-GPU top-2 margin there.
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
# One stage of an N-process pipeline
# ---------------------------------------------------------------------------

class PipelineRank:
    """This process's pipeline stage (one process per GPU, torch.distributed
    initialised with one rank per stage).

    ``layer_ranges`` is the split of the model (default: the reference's even
    split, ``config.split_layers``; ``config.balanced_layer_ranges`` evens
    out the bytes each stage streams).  Weights are the seeded synthetic ones
    (``weights.synthetic_stage_state``) unless ``state_dict`` gives this
    stage's.  ``groups`` is the number of request contexts in flight, each of
    ``rows`` rows; every stage holds one KV slot per group.
    """

    def __init__(self, cfg, *, groups: int, rows: int, capacity: int, layer_ranges=None,
                 dtype: torch.dtype = torch.bfloat16, seed: int = 0, method: str = "portable",
                 state_dict=None, top_p: tuple[float, float] | None = None, sample_seed: int = 1234,
                 nccl_sms: int = 8) -> None:
        from gpu_mesh_b200 import _lib
        from gpu_mesh_b200.config import split_layers
        from gpu_mesh_b200.stage import B200Stage
        from gpu_mesh_b200.weights import synthetic_stage_state

        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.ring = Ring(self.rank, self.world)
        self.device = torch.device("cuda", torch.cuda.current_device())
        # NCCL's send/receive kernels run beside the stage's persistent kernels
        # for most of a step: leave them SMs of their own, so no CTA of a
        # stream-K GEMM or of the attention waits for one.
        _lib.check(_lib.lib().mg_reserve_sms(self.device.index, nccl_sms if self.world > 1 else 0))
        self.cfg = cfg
        self.ranges = list(layer_ranges or split_layers(cfg.num_hidden_layers, self.world))
        ls, le = self.ranges[self.rank]
        first, last = self.ring.first, self.ring.last
        if state_dict is None:
            state_dict = synthetic_stage_state(cfg, ls, le, has_embedding=first, has_lm_head=last, seed=seed,
                                               dtype=dtype, device=self.device, method=method)
        self.stage = B200Stage(cfg, ls, le, has_embedding=first, has_lm_head=last, device=self.device,
                               dtype=dtype, state_dict=state_dict)
        del state_dict
        torch.cuda.empty_cache()
        self.dtype = dtype
        self.groups, self.rows = groups, rows
        self.slots = list(range(1, groups + 1))
        for sl in self.slots:
            self.stage.kv_reserve(sl, rows, capacity)
        self.top_p = top_p
        self.sample_gen = torch.Generator(device=self.device).manual_seed(sample_seed)
        self.ret_group = dist.new_group(list(range(self.world)))
        self._ids = [torch.empty(rows, 1, dtype=torch.int64, device=self.device) for _ in range(groups)]
        self._hidden: dict[int, list[torch.Tensor]] = {}
        self._host = torch.empty(rows, 1, dtype=torch.int64).pin_memory()
        self.record: list[tuple[int, torch.Tensor]] | None = None  # (group, ids) per last-stage iteration

    def _hidden_bufs(self, S: int) -> list[torch.Tensor]:
        if S not in self._hidden:
            self._hidden[S] = [torch.empty(self.rows, S, self.cfg.hidden_size, dtype=self.dtype,
                                           device=self.device) for _ in range(self.groups)]
        return self._hidden[S]

    def _tokens(self, out: torch.Tensor) -> torch.Tensor:
        from gpu_mesh_b200.sampling import greedy_sample, top_p_sample

        if out.dtype == torch.int64:  # already chosen inside the lm_head
            return out.view(-1, 1)
        if self.top_p is not None:
            return top_p_sample(out[:, -1], *self.top_p, generator=self.sample_gen).unsqueeze(-1)
        return greedy_sample(out[:, -1]).unsqueeze(-1)

    def _run(self, n_steps: int, inputs, forward, S: int, host_tokens: bool):
        def sample(k, g, out):
            ids = self._tokens(out).contiguous()
            if self.record is not None:
                self.record.append((g, ids.clone()))
            if host_tokens:  # a server reads every token on the host
                self._host.copy_(ids, non_blocking=True)
                torch.cuda.current_stream().synchronize()
                ids = self._host.to(self.device, non_blocking=True)
            return ids

        bufs = self._hidden_bufs(S)
        return decode_loop(self.ring, self.groups, n_steps, inputs, forward, sample,
                           lambda k, g: bufs[g], lambda g: self._ids[g], ret_group=self.ret_group)

    def prefill(self, prompts: list[torch.Tensor] | None, prompt_len: int, *, host_tokens: bool = False):
        """One prefill pass of every group's prompt [rows, prompt_len] (given on
        rank 0, None elsewhere: the other ranks size their receive buffers from
        ``prompt_len``); returns the first sampled ids per group on rank 0."""
        st = self.stage

        def forward(k, g, x):
            if self.ring.first:
                return st.forward_slot(self.slots[g], None, input_ids=x, logits="last", check_values=False)
            return st.forward_slot(self.slots[g], x, logits="last", check_values=False)

        return self._run(1, prompts, forward, prompt_len, host_tokens)

    def decode(self, ids: list[torch.Tensor] | None, n_steps: int, *, host_tokens: bool = False):
        """``n_steps`` decode steps of every group from ``ids`` (rank 0);
        returns the last step's ids per group on rank 0."""
        st = self.stage
        greedy_inside = self.ring.last and self.top_p is None
        top_p_inside = self.ring.last and self.top_p is not None

        def forward(k, g, x):
            slot = [self.slots[g]]
            if greedy_inside:
                return st.decode_greedy(slot, None if self.ring.first else x,
                                        input_ids=x if self.ring.first else None)[0]
            if top_p_inside:  # drawn from the histograms counted in the lm_head's epilogue
                u = torch.rand(self.rows, generator=self.sample_gen, device=self.device)
                return st.decode_top_p(slot, None if self.ring.first else x, temperature=self.top_p[0],
                                       top_p=self.top_p[1], uniforms=u,
                                       input_ids=x if self.ring.first else None)[0]
            if self.ring.first:
                return st.decode_multi(slot, None, input_ids=x, logits="last")
            return st.decode_multi(slot, x, logits="last")

        return self._run(n_steps, ids, forward, 1, host_tokens)

    def reset(self) -> None:
        for sl in self.slots:
            self.stage.kv_trim(sl, 0)

    def import_random_kv(self, context: int, seed: int = 5) -> None:
        """Fill every group's cache on this stage to ``context`` positions with
        N(0, 1) keys and values (a long-context decode without a prefill)."""
        cfg = self.cfg
        g = torch.Generator(device=self.device).manual_seed(seed + self.rank)
        shape = (self.rows, cfg.num_key_value_heads, context, cfg.head_dim)
        for sl in self.slots:
            for layer in range(self.stage.layer_end - self.stage.layer_start):
                k = torch.randn(shape, generator=g, device=self.device, dtype=self.dtype)
                v = torch.randn(shape, generator=g, device=self.device, dtype=self.dtype)
                self.stage.kv_import(sl, layer, k, v)
                del k, v

    def close(self) -> None:
        self.stage.close()


def verify_one_gpu(cfg, prompts: list[torch.Tensor], record: list[tuple[int, torch.Tensor]], groups: int,
                   *, dtype: torch.dtype = torch.bfloat16, seed: int = 0, method: str = "portable",
                   device: torch.device | None = None) -> dict:
    """Replay a recorded pipeline run with the whole model on one GPU.

    ``record`` is the last stage's ids in iteration order (the prefill's
    groups, then every decode step's groups).  The replay prefills the same
    prompts, then decodes every group in ONE pass per step (the one-GPU
    path: all rows through each weight once), teacher-forced on the
    pipeline's previous ids so a difference never propagates.  Returns the
    count of differing tokens and, for each, the one-GPU logit margin between
    its own choice and the pipeline's."""
    from gpu_mesh_b200.stage import B200Stage
    from gpu_mesh_b200.weights import synthetic_stage_state

    device = device or torch.device("cuda", torch.cuda.current_device())
    L = cfg.num_hidden_layers
    state = synthetic_stage_state(cfg, 0, L, has_embedding=True, has_lm_head=True, seed=seed, dtype=dtype,
                                  device=device, method=method)
    stage = B200Stage(cfg, 0, L, has_embedding=True, has_lm_head=True, device=device, dtype=dtype,
                      state_dict=state)
    del state
    try:
        rows = prompts[0].shape[0]
        n_iters = len(record) // groups
        cap = prompts[0].shape[1] + n_iters + 8
        slots = list(range(1, groups + 1))
        for sl in slots:
            stage.kv_reserve(sl, rows, cap)
        steps = [[record[k * groups + g][1].view(-1) for g in range(groups)] for k in range(n_iters)]
        mismatches, margins = 0, []
        from gpu_mesh_b200.sampling import greedy_sample

        mine = []
        for g, p in enumerate(prompts):
            logits = stage.forward_slot(slots[g], None, input_ids=p.to(device), logits="last", check_values=False)
            mine.append(greedy_sample(logits[:, -1]))
        compare = [(0, torch.cat(mine), torch.cat(steps[0]), None)]
        for k in range(1, n_iters):
            prev = torch.cat(steps[k - 1]).view(-1, 1)
            ids, logits = stage.decode_greedy(slots, None, input_ids=prev, return_logits=True)
            compare.append((k, ids, torch.cat(steps[k]), logits[:, -1]))
        for k, one, pipe, logits in compare:
            diff = torch.nonzero(one != pipe).flatten().tolist()
            mismatches += len(diff)
            for r in diff:
                m = None if logits is None else float(logits[r, one[r]].float() - logits[r, pipe[r]].float())
                margins.append({"step": k, "row": r, "one_gpu": int(one[r]), "pipeline": int(pipe[r]),
                                "margin": m})
        stage.check_device()
        return {"tokens_compared": sum(int(c[1].numel()) for c in compare), "token_mismatches": mismatches,
                "mismatch_margins": margins[:16], "reference": "one GPU, whole model, one pass for all rows, "
                "teacher-forced on the pipeline's ids"}
    finally:
        stage.close()


# ---------------------------------------------------------------------------
# Benchmark on N GPUs (torchrun)
# ---------------------------------------------------------------------------

def run_pipeline_bench(args, cfg, metric: str, workload: dict, peaks: tuple[float, float, str],
                       traffic: dict | None = None, top_p: tuple[float, float] | None = None,
                       other_configs: list[dict] | None = None) -> None:
    """``top_p`` = (temperature, p): the last stage samples with a seeded device
    generator instead of selecting greedily inside its lm_head.
    ``other_configs``: the scope's configurations named at this stage count,
    measured after the headline one (``run_other_config``)."""
    from contextlib import nullcontext

    from gpu_mesh_b200.clocks import ClockSampler
    from gpu_mesh_b200.config import balanced_layer_ranges, split_layers

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    ring = Ring(rank, world)
    try:
        hbm, _, peak_kind = peaks
        rows_total = args.micro * args.micro_batches
        n_groups = max(world, 1)
        if rows_total % n_groups:
            raise ValueError(f"{rows_total} rows do not split into {n_groups} groups")
        rows = rows_total // n_groups
        mean_ctx = args.prompt + args.warmup + args.steps
        ranges = (split_layers(cfg.num_hidden_layers, world) if getattr(args, "even_split", False) else
                  balanced_layer_ranges(cfg, world, rows=rows_total, context=mean_ctx))
        cap = args.prompt + args.warmup + 3 * args.steps + 16
        nccl_sms = getattr(args, "nccl_sms", 8)
        pr = PipelineRank(cfg, groups=n_groups, rows=rows, capacity=cap, layer_ranges=ranges, top_p=top_p,
                          nccl_sms=nccl_sms)
        g = torch.Generator().manual_seed(1000)
        prompts_host = [torch.randint(0, cfg.vocab_size, (rows, args.prompt), generator=g)
                        for _ in range(n_groups)]
        prompts = [p.to(dev) for p in prompts_host] if ring.first else None

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
        timed(lambda: pr.prefill(prompts, args.prompt))
        pr.reset()
        pr.record = [] if top_p is None else None  # ids of every iteration, for the one-GPU check
        ids, prefill_ms = timed(lambda: pr.prefill(prompts, args.prompt))
        ids, _ = timed(lambda: pr.decode(ids, args.warmup))
        launches0 = _launches()
        with (ClockSampler(local) if ring.first else nullcontext()) as clocks:
            ids, ms = timed(lambda: pr.decode(ids, args.steps))
        launches = _launches() - launches0
        pr.stage.profile(True)
        ids, _ = timed(lambda: pr.decode(ids, args.steps))
        prof = pr.stage.profile_read()
        pr.stage.profile(False)
        ids, e2e_ms = timed(lambda: pr.decode(ids, args.steps, host_tokens=True))
        record, pr.record = pr.record, None

        # Weak scaling: the same per-GPU work at a batch that grows with N
        # (N groups of 32 rows in flight: every GPU streams its weights N
        # times per step, as one GPU streams all weights once for 32 rows).
        weak = None
        if world > 1 and not getattr(args, "no_weak", False):
            pr.close()
            torch.cuda.empty_cache()
            ranges_w = (split_layers(cfg.num_hidden_layers, world) if getattr(args, "even_split", False) else
                        balanced_layer_ranges(cfg, world, rows=rows_total * n_groups, context=mean_ctx))
            pw = PipelineRank(cfg, groups=n_groups, rows=rows_total, capacity=cap, layer_ranges=ranges_w,
                              top_p=top_p, nccl_sms=nccl_sms)
            gw = torch.Generator().manual_seed(2000)
            prompts_w = [torch.randint(0, cfg.vocab_size, (rows_total, args.prompt), generator=gw).to(dev)
                         for _ in range(n_groups)] if ring.first else None
            idw, _ = timed(lambda: pw.prefill(prompts_w, args.prompt))
            idw, _ = timed(lambda: pw.decode(idw, args.warmup))
            idw, ms_w = timed(lambda: pw.decode(idw, args.steps))
            pw.close()
            weak = {
                "scaling": "weak",
                "rows": rows_total * n_groups,
                "groups_in_flight": n_groups,
                "rows_per_group": rows_total,
                "layer_ranges": ranges_w,
                "value": rows_total * n_groups * args.steps / (ms_w / 1000.0),
                "unit": "tok/s",
                "ms_per_step": ms_w / args.steps,
                "note": "per-GPU work of the one-GPU workload (32 rows through every layer once per step)",
            }
        else:
            pr.close()
        torch.cuda.empty_cache()

        # Token check: the last stage replays the run with the whole model on
        # its own GPU (the one-GPU path), teacher-forced on the pipeline's ids.
        check = None
        if ring.last and record is not None:
            check = verify_one_gpu(cfg, prompts_host, record, n_groups, device=dev)
        checks = [None] * world
        dist.all_gather_object(checks, check)
        check = checks[-1]

        others = {}
        for spec in other_configs or []:
            others[spec["name"]] = run_other_config(spec, args, timed)

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
            stage_ms = [sum(c["ms"] for c in p.values()) / args.steps for p in profs]
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
                           "groups_in_flight": n_groups, "rows_per_group": rows, "layer_ranges": ranges,
                           "sms_left_to_nccl": nccl_sms},
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
                    "kernel": "attn_tc, mean over stages",
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
                "per_stage_ms_per_step": stage_ms,
                "per_stage_profile": profs,
                "clocks": clocks.summary(),
            }
            if check is not None:
                line["token_check"] = check
            if others:
                line["other_configs"] = others
            if weak is not None:
                line["weak_scaling"] = weak
            print(json.dumps(line), flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def run_other_config(spec: dict, args, timed) -> dict:
    """One of the scope's other configurations on this pipeline (every rank
    calls it): ``spec`` = {name, cfg, rows, prompt | context, top_p, note}.
    Greedy (or seeded top-p) decode with the N ranks' groups in flight; a
    ``context`` spec starts from caches pre-filled with N(0, 1) instead of a
    prefill.  Returns tok/s, ms per step and the prefill rate."""
    from gpu_mesh_b200.config import balanced_layer_ranges

    world = dist.get_world_size()
    cfg, rows_total = spec["cfg"], spec["rows"]
    groups = world
    if rows_total % groups:
        raise ValueError(f"{rows_total} rows do not split into {groups} groups")
    rows = rows_total // groups
    start = spec.get("context") or spec["prompt"]
    cap = start + args.warmup + args.steps + 8
    ranges = balanced_layer_ranges(cfg, world, rows=rows_total, context=start)
    pr = PipelineRank(cfg, groups=groups, rows=rows, capacity=cap, layer_ranges=ranges, top_p=spec.get("top_p"),
                      nccl_sms=getattr(args, "nccl_sms", 8))
    try:
        dev = pr.device
        out = {"config": spec["note"], "stages": world, "rows": rows_total, "groups_in_flight": groups,
               "layer_ranges": ranges}
        g = torch.Generator().manual_seed(3000)
        if spec.get("context"):
            pr.import_random_kv(spec["context"])
            ids = ([torch.randint(0, cfg.vocab_size, (rows, 1), generator=g).to(dev) for _ in range(groups)]
                   if pr.ring.first else None)
        else:
            prompts = ([torch.randint(0, cfg.vocab_size, (rows, spec["prompt"]), generator=g).to(dev)
                        for _ in range(groups)] if pr.ring.first else None)
            ids, pf_ms = timed(lambda: pr.prefill(prompts, spec["prompt"]))
            out["prefill_tok_s"] = rows_total * spec["prompt"] / (pf_ms / 1000.0)
        ids, _ = timed(lambda: pr.decode(ids, args.warmup))
        ids, ms = timed(lambda: pr.decode(ids, args.steps))
        out.update({"decode_tok_s": rows_total * args.steps / (ms / 1000.0), "ms_per_step": ms / args.steps,
                    "steps": args.steps})
        pr.stage.check_device()
        return out
    finally:
        pr.close()
        torch.cuda.empty_cache()


def _launches() -> int:
    from gpu_mesh_b200 import _lib

    return int(_lib.lib().mg_launch_count())
