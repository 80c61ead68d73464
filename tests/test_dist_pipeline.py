"""The multi-GPU pipeline schedule, run as gloo ranks on the CPU.

``decode_loop`` drives N stages with G groups in flight: hidden states go
stage to stage, sampled ids return from the last stage to stage 0.  Here the
stages are fake (stage r adds a known function to the hidden state, the last
stage "samples" a deterministic id), and every rank's results are checked
against the same computation run sequentially in one process.  Also covers
a stage that raises mid-run: the other ranks see the failure through the
process group's timeout instead of hanging.
"""
from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gpu_mesh_b200.dist import Ring, decode_loop

ROWS, H = 3, 4


def stage_fn(rank: int, x: torch.Tensor) -> torch.Tensor:
    if rank == 0:  # "embedding": ids [rows, 1] -> hidden [rows, 1, H]
        return (x.float().unsqueeze(-1) + torch.arange(H).float()).contiguous()
    return (x * 1.5 + rank).contiguous()


def sample_fn(k: int, g: int, out: torch.Tensor) -> torch.Tensor:
    return ((out.sum(-1).round().long() * 7 + k + 3 * g) % 101).reshape(ROWS, 1).contiguous()


def sequential(world: int, groups: int, steps: int, first: list[torch.Tensor],
               per_call: int) -> list[list[torch.Tensor]]:
    """Every step of every group in order; steps are numbered per call of
    ``decode_loop`` (``per_call`` steps each), as the schedule numbers them."""
    ids = list(first)
    history = []
    for step in range(steps):
        k = step % per_call
        row = []
        for g in range(groups):
            x = ids[g]
            for r in range(world):
                x = stage_fn(r, x)
            ids[g] = sample_fn(k, g, x)
            row.append(ids[g].clone())
        history.append(row)
    return history


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, groups: int, steps: int, fail_rank: int, q) -> None:
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        ret_group = dist.new_group(list(range(world)), timeout=timedelta(seconds=20))
        ring = Ring(rank, world)
        first = [torch.tensor([[g + 1], [g + 2], [g + 5]]) for g in range(groups)]
        seen = []

        def forward(k, g, x):
            if rank == fail_rank and k == 1:
                raise RuntimeError(f"stage {rank} failed")
            return stage_fn(rank, x)

        def sample(k, g, out):
            ids = sample_fn(k, g, out)
            seen.append((k, g, ids.clone()))
            return ids

        hid = {}
        ids_buf = {}
        finals = first
        for _ in range(2):  # two calls, carrying stage 0's ids across them
            finals = decode_loop(
                ring, groups, steps, finals if rank == 0 else None, forward, sample,
                lambda k, g: hid.setdefault((k, g), torch.empty(ROWS, 1, H)),
                lambda g: ids_buf.setdefault(g, torch.empty(ROWS, 1, dtype=torch.long)),
                ret_group=ret_group,
            )
        # plain lists: tensors would be shared through descriptors that die with this process
        q.put((rank, "ok", [(k, g, t.tolist()) for k, g, t in seen],
               None if finals is None else [t.tolist() for t in finals]))
    except Exception:
        q.put((rank, "error", traceback.format_exc(), None))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(world: int, groups: int, steps: int, fail_rank: int = -1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, groups, steps, fail_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, a, b = q.get(timeout=120)
        results[rank] = (status, a, b)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world,groups", [(2, 2), (3, 3), (3, 1), (2, 4)])
def test_pipeline_schedule_matches_sequential(world, groups):
    steps = 3
    res = _run(world, groups, steps)
    for r, (status, a, _) in res.items():
        assert status == "ok", a
    first = [torch.tensor([[g + 1], [g + 2], [g + 5]]) for g in range(groups)]
    ref = sequential(world, groups, 2 * steps, first, steps)
    last = res[world - 1][1]
    assert len(last) == 2 * steps * groups
    for i, (k, g, ids) in enumerate(last):
        call, kk = divmod(i // groups, steps)
        assert ids == ref[call * steps + kk][g].tolist(), (i, k, g)
    finals = res[0][2]
    for g in range(groups):
        assert finals[g] == ref[-1][g].tolist()


def test_failing_stage_surfaces_on_every_rank():
    res = _run(2, 2, 3, fail_rank=1)
    assert res[1][0] == "error" and "stage 1 failed" in res[1][1]
    # rank 0 does not hang: its next exchange with the dead stage errors out
    assert res[0][0] == "error"
