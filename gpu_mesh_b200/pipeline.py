"""Pipeline coordinator over B200 stages.

The contract is the reference's portable coordinator
(src/meshgpu/backends/portable/pipeline.py): ``build_pipeline`` splits layers
evenly with the remainder to the first stages (:48-103); ``pipeline_prefill``
clears the context on every stage, runs the stages in order and clears again
on failure (:110-163); ``pipeline_decode_step`` requires every stage to hold
the same cached length, feeds positions arange(T, T+S) and trims back on
failure (:166-233); the async variants drain a running stage call before a
cancellation propagates (:240-377).  Arguments, results, messages and
exception types are the reference's; the functions are duck-typed and drive
reference workers and B200 workers alike.

How a call runs is this module's own.  Each coordinator function is a *plan*:
a generator that validates its arguments, yields the stage calls it needs
(``_Call``) one at a time, receives their results, and on failure yields its
rollback calls before re-raising.  One plan serves both drivers:
``_run_plan`` calls the stages directly, and ``_run_plan_async`` either runs
the whole synchronous driver in one worker thread (every stage local) or
awaits the calls one by one (remote stages with coroutine methods).  Between
B200 stages on different GPUs the boundary tensor moves through
``gpu_mesh_b200.boundary`` (a side-stream peer copy ordered by events), and
``gpu_mesh_b200.schedule.MicroBatchPipeline`` keeps several micro-batches in
flight across the stages.
"""
from __future__ import annotations

import asyncio
import inspect
import logging
import threading
from collections.abc import Generator, Sequence
from dataclasses import dataclass, field
from typing import Any

import torch

from gpu_mesh_b200.config import LlamaConfig, config_from, split_layers
from gpu_mesh_b200.stage import B200Stage
from gpu_mesh_b200.stage_worker import B200StageWorker, StageContext
from gpu_mesh_b200.weights import slice_stage_state, synthetic_stage_state

log = logging.getLogger(__name__)


def build_pipeline(
    cfg: Any,
    num_stages: int,
    devices: list[torch.device],
    job_id: str = "local",
    transport: str = "cpu",
    activation_checkpointing: bool = False,
    *,
    dtype: torch.dtype = torch.float32,
    state_dict: dict[str, torch.Tensor] | None = None,
    layer_ranges: Sequence[tuple[int, int]] | None = None,
    seed: int = 0,
    check_values: bool = True,
) -> list[B200StageWorker]:
    """B200 workers for ``cfg`` split into ``num_stages`` stages.

    ``state_dict`` is a whole-model state dict with global layer names
    (``layers.{i}....``); without one, seeded synthetic weights are used.
    ``layer_ranges`` overrides the even split (the manifest/planner ranges).
    """
    del activation_checkpointing  # training-only in the reference
    cfg = config_from(cfg)
    if num_stages < 1 or num_stages > cfg.num_hidden_layers:
        raise ValueError(f"num_stages must be in [1, {cfg.num_hidden_layers}], got {num_stages}")
    if len(devices) != num_stages:
        raise ValueError(f"need {num_stages} devices, got {len(devices)}")
    ranges = list(layer_ranges) if layer_ranges is not None else split_layers(cfg.num_hidden_layers, num_stages)
    if len(ranges) != num_stages or ranges[0][0] != 0 or ranges[-1][1] != cfg.num_hidden_layers or any(
        a[1] != b[0] for a, b in zip(ranges, ranges[1:])
    ):
        raise ValueError(f"layer ranges {ranges} do not tile [0, {cfg.num_hidden_layers})")
    workers = []
    for i, (ls, le) in enumerate(ranges):
        is_first, is_last = i == 0, i == num_stages - 1
        if state_dict is not None:
            sd = slice_stage_state(
                state_dict, ls, le, has_embedding=is_first, has_lm_head=is_last,
                tie_word_embeddings=cfg.tie_word_embeddings,
            )
        else:
            sd = synthetic_stage_state(
                cfg, ls, le, has_embedding=is_first, has_lm_head=is_last, seed=seed,
                dtype=dtype, device=devices[i],
            )
        stage = B200Stage(
            cfg, ls, le, has_embedding=is_first, has_lm_head=is_last,
            device=devices[i], dtype=dtype, state_dict=sd,
        )
        del sd
        ctx = StageContext(
            stage_id=i, layer_start=ls, layer_end=le, device=devices[i],
            is_first=is_first, is_last=is_last, job_id=job_id, attempt_id="local",
            transport=transport,
        )
        workers.append(B200StageWorker(stage, ctx, check_values=check_values))
        log.debug("stage %d: layers [%d, %d) on %s", i, ls, le, devices[i])
    return workers


def from_reference_workers(
    workers: Sequence[Any],
    devices: Sequence[torch.device] | None = None,
    *,
    dtype: torch.dtype | None = None,
    transport: str | None = None,
) -> list[B200StageWorker]:
    """Convert already-built reference ``StageWorker`` objects (LlamaStage or
    Qwen3Stage models) into B200 workers with the same weights and ranges."""
    out = []
    for i, w in enumerate(workers):
        model, ctx = w._model, w._ctx
        cfg = config_from(getattr(model, "cfg", None) or model.config)
        sd = {k: v for k, v in model.state_dict().items()}
        dev = torch.device(devices[i]) if devices is not None else torch.device("cuda", i)
        dt = dtype or next(iter(sd.values())).dtype
        stage = B200Stage(
            cfg, model.layer_start, model.layer_end, has_embedding=model.has_embedding,
            has_lm_head=model.has_lm_head, device=dev, dtype=dt, state_dict=sd,
        )
        new_ctx = StageContext(
            stage_id=ctx.stage_id, layer_start=ctx.layer_start, layer_end=ctx.layer_end, device=dev,
            is_first=ctx.is_first, is_last=ctx.is_last, job_id=ctx.job_id, attempt_id=ctx.attempt_id,
            transport=transport or ctx.transport,
        )
        out.append(B200StageWorker(stage, new_ctx))
    return out


# ---------------------------------------------------------------------------
# Plans and their drivers
# ---------------------------------------------------------------------------

@dataclass
class _Call:
    """One stage method call a plan needs; ``best_effort`` calls are rollback
    steps whose failure is logged and answered with ``None``."""

    worker: Any
    method: str
    args: tuple = ()
    kwargs: dict = field(default_factory=dict)
    best_effort: bool = False


Plan = Generator[_Call, Any, Any]


def _invoke(call: _Call) -> Any:
    return getattr(call.worker, call.method)(*call.args, **call.kwargs)


def _run_plan(plan: Plan, cancelled: threading.Event | None = None) -> Any:
    """Drive a plan with direct (blocking) stage calls.  Once ``cancelled`` is
    set, the plan gets a CancelledError at its next stage-call boundary, so it
    rolls back the way an awaited plan does."""
    try:
        call = next(plan)
        while True:
            try:
                result = _invoke(call)
            except Exception as exc:
                if not call.best_effort:
                    call = plan.throw(exc)
                    continue
                log.warning("rollback step %s failed: %s", call.method, exc)
                result = None
            except BaseException as exc:  # KeyboardInterrupt and the like: roll back, then re-raise
                call = plan.throw(exc)
                continue
            if cancelled is not None and cancelled.is_set() and not call.best_effort:
                call = plan.throw(asyncio.CancelledError())
                continue
            call = plan.send(result)
    except StopIteration as done:
        return done.value


def _has_coroutines(workers: Sequence[Any]) -> bool:
    return any(
        inspect.iscoroutinefunction(getattr(w, name, None))
        for w in workers
        for name in ("forward_inference", "clear_kv", "trim_kv", "kv_cache_length")
    )


async def _drained(fn, *args, cancelled: threading.Event | None = None) -> Any:
    """Run a blocking function in a worker thread.  A cancellation sets
    ``cancelled`` and waits for the function to finish before it propagates,
    so nothing that follows races a stage call still running on the GPU."""
    task = asyncio.ensure_future(asyncio.to_thread(fn, *args))
    try:
        return await asyncio.shield(task)
    except asyncio.CancelledError:
        if cancelled is not None:
            cancelled.set()
        await asyncio.wait([task])
        raise


async def _run_plan_async(plan: Plan, workers: Sequence[Any]) -> Any:
    if not _has_coroutines(workers):
        # Every stage is in this process: one thread hop for the whole call; a
        # cancellation reaches the plan at its next stage-call boundary.
        cancelled = threading.Event()
        return await _drained(_run_plan, plan, cancelled, cancelled=cancelled)
    try:
        call = next(plan)
        while True:
            try:
                fn = getattr(call.worker, call.method)
                if inspect.iscoroutinefunction(fn):
                    result = await fn(*call.args, **call.kwargs)
                else:
                    result = await _drained(_invoke, call)
            except Exception as exc:
                if not call.best_effort:
                    call = plan.throw(exc)
                    continue
                log.warning("rollback step %s failed: %s", call.method, exc)
                result = None
            except BaseException as exc:  # cancellation: roll back, then propagate
                call = plan.throw(exc)
                continue
            call = plan.send(result)
    except StopIteration as done:
        return done.value


# ---------------------------------------------------------------------------
# Argument checks (the reference's messages)
# ---------------------------------------------------------------------------

def _max_positions(worker: Any) -> int | None:
    model = getattr(worker, "_model", None)
    cfg = getattr(model, "cfg", None)
    if cfg is not None:
        return getattr(cfg, "max_position_embeddings", None)
    return getattr(worker, "max_position_embeddings", None)


def _check_prompt(workers: Sequence[Any], input_ids: torch.Tensor) -> None:
    if input_ids.ndim != 2:
        raise ValueError("input_ids must have shape [batch, sequence]")
    if input_ids.shape[0] < 1 or input_ids.shape[1] < 1:
        raise ValueError("input_ids must have a non-empty batch and sequence")
    if not workers:
        raise ValueError("workers must not be empty")
    limit = _max_positions(workers[0])
    if limit is not None and input_ids.shape[1] > limit:
        raise ValueError(f"prefill sequence length {input_ids.shape[1]} exceeds model context {limit}")


def _check_next(workers: Sequence[Any], next_token: torch.Tensor) -> None:
    if next_token.ndim != 2 or next_token.shape[0] < 1 or next_token.shape[1] < 1:
        raise ValueError("next_token must have shape [batch, sequence] with sequence >= 1")
    if not workers:
        raise ValueError("workers must not be empty")


def _checked_lengths(
    lengths: list[int], query_len: int, max_positions: int | None, name: str, prefill_name: str
) -> list[int]:
    """Every stage must hold the same non-empty context with room for the query."""
    for i, kv_len in enumerate(lengths):
        if kv_len != lengths[0]:
            raise RuntimeError(
                "pipeline KV caches are out of sync: "
                f"stage 0 has {lengths[0]} tokens, stage {i} has {kv_len}"
            )
        if kv_len == 0:
            raise RuntimeError(f"{name} requires a prefilled KV cache; call {prefill_name} first")
        if max_positions is not None and kv_len + query_len > max_positions:
            raise ValueError(
                f"decode would reach position {kv_len + query_len - 1}, "
                f"beyond model context {max_positions}"
            )
    return lengths


def _logits_kw(worker: Any, logits: str) -> dict[str, Any]:
    return {"logits": logits} if logits != "all" and isinstance(worker, B200StageWorker) else {}


def _restore(workers: Sequence[Any], lengths: Sequence[int], cache_key: str | None) -> Plan:
    """Rollback: every stage back to its length before the failed call."""
    for worker, length in zip(workers, lengths):
        if length == 0:
            yield _Call(worker, "clear_kv", (cache_key,), best_effort=True)
        else:
            yield _Call(worker, "trim_kv", (length, cache_key), best_effort=True)


# ---------------------------------------------------------------------------
# The coordinator's plans
# ---------------------------------------------------------------------------

def _prefill_plan(workers, input_ids, operation_id, attempt_id, cache_key, logits="all") -> Plan:
    _check_prompt(workers, input_ids)
    for worker in workers:
        yield _Call(worker, "clear_kv", (cache_key,))
    hidden = None
    try:
        for i, worker in enumerate(workers):
            kw = dict(input_ids=input_ids if i == 0 else None, operation_id=operation_id,
                      attempt_id=attempt_id, reset_kv=False, cache_key=cache_key)
            if i == len(workers) - 1:
                kw.update(_logits_kw(worker, logits))
            hidden = (yield _Call(worker, "forward_inference", (hidden,), kw)).output
    except BaseException:
        yield from _restore(workers, [0] * len(workers), cache_key)
        raise
    return hidden


def _decode_plan(workers, next_token, operation_id, attempt_id, cache_key, logits="all",
                 names=("pipeline_decode_step", "pipeline_prefill")) -> Plan:
    _check_next(workers, next_token)
    batch, query_len = next_token.shape
    lengths = []
    for worker in workers:
        lengths.append(int((yield _Call(worker, "kv_cache_length", (cache_key,)))))
    _checked_lengths(lengths, query_len, _max_positions(workers[0]), *names)
    hidden = None
    try:
        for i, worker in enumerate(workers):
            positions = torch.arange(lengths[i], lengths[i] + query_len, dtype=torch.long,
                                     device=next_token.device).unsqueeze(0).expand(batch, -1)
            kw = dict(input_ids=next_token if i == 0 else None, position_ids=positions,
                      operation_id=operation_id, attempt_id=attempt_id, reset_kv=False,
                      cache_key=cache_key)
            if i == len(workers) - 1:
                kw.update(_logits_kw(worker, logits))
            hidden = (yield _Call(worker, "forward_inference", (hidden,), kw)).output
    except BaseException:
        yield from _restore(workers, lengths, cache_key)
        raise
    return hidden


def _multi_plan(workers, next_tokens, cache_keys, name, last_call) -> Plan:
    """One decode token for several contexts in one pass per stage; the last
    stage runs ``last_call`` (``decode_multi`` or ``decode_greedy``)."""
    if next_tokens.ndim != 2 or next_tokens.shape[1] != 1:
        raise ValueError("next_tokens must have shape [rows, 1]")
    if not workers:
        raise ValueError("workers must not be empty")
    limit = _max_positions(workers[0])
    lengths = {}
    for key in cache_keys:
        lengths[key] = _checked_lengths([w.kv_cache_length(key) for w in workers], 1, limit, name,
                                        "pipeline_prefill")
    keys = list(cache_keys)
    hidden = None
    try:
        for i, worker in enumerate(workers):
            ids = next_tokens if i == 0 else None
            if i == len(workers) - 1:
                return (yield last_call(worker, hidden, keys, ids))
            hidden = yield _Call(worker, "decode_multi", (hidden, keys), dict(input_ids=ids))
    except BaseException:
        for key, lens in lengths.items():
            yield from _restore(workers, lens, key)
        raise


# ---------------------------------------------------------------------------
# Public coordinator functions
# ---------------------------------------------------------------------------

@torch.no_grad()
def pipeline_prefill(
    workers: list[Any],
    input_ids: torch.Tensor,
    *,
    operation_id: int = 1,
    attempt_id: str = "a0",
    cache_key: str | None = None,
    logits: str = "all",
) -> torch.Tensor:
    """Prefill through all stages in order; logits [B, S, V] (or [B, 1, V]
    with ``logits="last"``)."""
    return _run_plan(_prefill_plan(workers, input_ids, operation_id, attempt_id, cache_key, logits))


@torch.no_grad()
def pipeline_decode_step(
    workers: list[Any],
    next_token: torch.Tensor,
    *,
    operation_id: int,
    attempt_id: str = "a0",
    cache_key: str | None = None,
    logits: str = "all",
) -> torch.Tensor:
    """One decode step over prefilled caches; logits [B, S, V]."""
    return _run_plan(_decode_plan(workers, next_token, operation_id, attempt_id, cache_key, logits))


@torch.no_grad()
def pipeline_decode_multi(
    workers: list[B200StageWorker],
    next_tokens: torch.Tensor,
    *,
    cache_keys: Sequence[str | None],
    logits: str = "last",
) -> torch.Tensor:
    """One decode token for several request contexts in one pass per stage.

    Rows of ``next_tokens`` [sum of batches, 1] are the contexts' rows stacked
    in ``cache_keys`` order; each row attends to its own context's cache, and
    every weight is read once for all of them.  Equivalent to one
    ``pipeline_decode_step`` per context (the reference drives one context at
    a time, inference/batcher.py:229-247).  Rolls every context back on failure.
    """
    def last(worker, hidden, keys, ids):
        return _Call(worker, "decode_multi", (hidden, keys), dict(input_ids=ids, logits=logits))

    return _run_plan(_multi_plan(workers, next_tokens, cache_keys, "pipeline_decode_multi", last))


@torch.no_grad()
def pipeline_decode_greedy(
    workers: list[B200StageWorker],
    next_tokens: torch.Tensor,
    *,
    cache_keys: Sequence[str | None],
    return_logits: bool = False,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``pipeline_decode_multi`` whose last stage also picks every row's
    greedy token on the device (fused into its lm_head): returns (token ids
    int64 [rows], logits [rows, 1, V] or None).  The ids equal
    ``greedy_sample`` of the logits (inference/sampling.py:45-56), which is
    what the reference's decode loops apply to the returned logits
    (session.py:245-259, batcher.py:356-388)."""
    def last(worker, hidden, keys, ids):
        return _Call(worker, "decode_greedy", (hidden, keys), dict(input_ids=ids, return_logits=return_logits))

    return _run_plan(_multi_plan(workers, next_tokens, cache_keys, "pipeline_decode_greedy", last))


@torch.no_grad()
def pipeline_decode_top_p(
    workers: list[B200StageWorker],
    next_tokens: torch.Tensor,
    *,
    cache_keys: Sequence[str | None],
    temperature: float,
    top_p: float,
    generator: torch.Generator | None = None,
    uniforms: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``pipeline_decode_multi`` whose last stage also draws every row's
    top-p token on the device (counted in its lm_head): returns (token ids
    int64 [rows], logits [rows, 1, V]).  The draw of row r is ``uniforms[r]``
    (default: ``torch.rand`` with ``generator``), as ``top_p_sample`` draws
    (inference/sampling.py:63-95; the reference hands the nucleus to
    ``torch.multinomial``).  Temperature 0 is greedy, as the reference's."""
    if temperature <= 0:
        ids, logits = pipeline_decode_greedy(workers, next_tokens, cache_keys=cache_keys, return_logits=True)
        return ids, logits
    rows = next_tokens.shape[0]
    if uniforms is None:
        dev = generator.device if generator is not None else torch.device("cpu")
        uniforms = torch.rand(rows, generator=generator, device=dev)

    def last(worker, hidden, keys, ids):
        return _Call(worker, "decode_top_p", (hidden, keys),
                     dict(input_ids=ids, temperature=temperature, top_p=top_p, uniforms=uniforms))

    return _run_plan(_multi_plan(workers, next_tokens, cache_keys, "pipeline_decode_top_p", last))


async def pipeline_prefill_async(
    workers: list[Any],
    input_ids: torch.Tensor,
    *,
    operation_id: int = 1,
    attempt_id: str = "a0",
    cache_key: str | None = None,
) -> torch.Tensor:
    """``pipeline_prefill`` for local or remote (coroutine) stages."""
    with torch.no_grad():
        return await _run_plan_async(
            _prefill_plan(workers, input_ids, operation_id, attempt_id, cache_key), workers)


async def pipeline_decode_step_async(
    workers: list[Any],
    next_token: torch.Tensor,
    *,
    operation_id: int,
    attempt_id: str = "a0",
    cache_key: str | None = None,
) -> torch.Tensor:
    """``pipeline_decode_step`` for local or remote (coroutine) stages."""
    with torch.no_grad():
        return await _run_plan_async(
            _decode_plan(workers, next_token, operation_id, attempt_id, cache_key,
                         names=("pipeline_decode_step_async", "pipeline_prefill_async")),
            workers)


__all__ = [
    "LlamaConfig",
    "build_pipeline",
    "from_reference_workers",
    "pipeline_prefill",
    "pipeline_decode_step",
    "pipeline_decode_multi",
    "pipeline_decode_greedy",
    "pipeline_decode_top_p",
    "pipeline_prefill_async",
    "pipeline_decode_step_async",
]
