"""Pipeline coordinator over B200 stages.

Same contract as the reference's portable coordinator
(src/meshgpu/backends/portable/pipeline.py):
  * ``build_pipeline`` splits layers evenly, remainder to the first stages,
    stage 0 with the embedding and the last stage with norm + lm_head (:48-103);
  * ``pipeline_prefill`` clears the context on every stage, runs stages in
    order and clears again on failure (:110-163);
  * ``pipeline_decode_step`` checks that every stage holds the same cached
    length, feeds positions arange(T, T+S) and trims back on failure (:166-233);
  * async variants run local stage calls in a worker thread and drain them on
    cancellation (:240-377).
The coordinator functions are duck-typed: they drive reference workers and
B200 workers alike.
"""
from __future__ import annotations

import asyncio
import inspect
import logging
from collections.abc import Sequence
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
# In-process pipeline inference
# ---------------------------------------------------------------------------

def _max_positions(worker: Any) -> int | None:
    model = getattr(worker, "_model", None)
    cfg = getattr(model, "cfg", None)
    if cfg is not None:
        return getattr(cfg, "max_position_embeddings", None)
    return getattr(worker, "max_position_embeddings", None)


def _extra(worker: Any, logits: str) -> dict[str, Any]:
    return {"logits": logits} if logits != "all" and isinstance(worker, B200StageWorker) else {}


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
    if input_ids.ndim != 2:
        raise ValueError("input_ids must have shape [batch, sequence]")
    B, S = input_ids.shape
    if B < 1 or S < 1:
        raise ValueError("input_ids must have a non-empty batch and sequence")
    if not workers:
        raise ValueError("workers must not be empty")
    max_positions = _max_positions(workers[0])
    if max_positions is not None and S > max_positions:
        raise ValueError(f"prefill sequence length {S} exceeds model context {max_positions}")
    for w in workers:
        w.clear_kv(cache_key)
    hidden = None
    try:
        for i, worker in enumerate(workers):
            result = worker.forward_inference(
                hidden,
                input_ids=input_ids if i == 0 else None,
                operation_id=operation_id,
                attempt_id=attempt_id,
                reset_kv=False,
                cache_key=cache_key,
                **(_extra(worker, logits) if i == len(workers) - 1 else {}),
            )
            hidden = result.output
    except BaseException:
        _clear_kv_best_effort(workers, cache_key)
        raise
    assert hidden is not None
    return hidden


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
    if next_token.ndim != 2 or next_token.shape[0] < 1 or next_token.shape[1] < 1:
        raise ValueError("next_token must have shape [batch, sequence] with sequence >= 1")
    batch_size, query_len = next_token.shape
    if not workers:
        raise ValueError("workers must not be empty")
    max_positions = _max_positions(workers[0])
    cache_lengths = _checked_lengths(
        [w.kv_cache_length(cache_key) for w in workers], query_len, max_positions, "pipeline_decode_step",
        "pipeline_prefill",
    )
    hidden = None
    try:
        for i, worker in enumerate(workers):
            kv_len = cache_lengths[i]
            position_ids = torch.arange(
                kv_len, kv_len + query_len, dtype=torch.long, device=next_token.device
            ).unsqueeze(0).expand(batch_size, -1)
            result = worker.forward_inference(
                hidden,
                input_ids=next_token if i == 0 else None,
                position_ids=position_ids,
                operation_id=operation_id,
                attempt_id=attempt_id,
                reset_kv=False,
                cache_key=cache_key,
                **(_extra(worker, logits) if i == len(workers) - 1 else {}),
            )
            hidden = result.output
    except BaseException:
        _restore_kv_lengths_best_effort(workers, cache_lengths, cache_key)
        raise
    assert hidden is not None
    return hidden


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
    if next_tokens.ndim != 2 or next_tokens.shape[1] != 1:
        raise ValueError("next_tokens must have shape [rows, 1]")
    if not workers:
        raise ValueError("workers must not be empty")
    max_positions = _max_positions(workers[0])
    lengths = {}
    for key in cache_keys:
        lengths[key] = _checked_lengths(
            [w.kv_cache_length(key) for w in workers], 1, max_positions,
            "pipeline_decode_multi", "pipeline_prefill",
        )
    hidden = None
    try:
        for i, worker in enumerate(workers):
            hidden = worker.decode_multi(
                hidden, list(cache_keys), input_ids=next_tokens if i == 0 else None,
                logits=logits,
            )
    except BaseException:
        for key, lens in lengths.items():
            _restore_kv_lengths_best_effort(workers, lens, key)
        raise
    assert hidden is not None
    return hidden


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
    if next_tokens.ndim != 2 or next_tokens.shape[1] != 1:
        raise ValueError("next_tokens must have shape [rows, 1]")
    if not workers:
        raise ValueError("workers must not be empty")
    max_positions = _max_positions(workers[0])
    lengths = {}
    for key in cache_keys:
        lengths[key] = _checked_lengths(
            [w.kv_cache_length(key) for w in workers], 1, max_positions,
            "pipeline_decode_greedy", "pipeline_prefill",
        )
    hidden = None
    try:
        for i, worker in enumerate(workers[:-1]):
            hidden = worker.decode_multi(
                hidden, list(cache_keys), input_ids=next_tokens if i == 0 else None,
            )
        return workers[-1].decode_greedy(
            hidden, list(cache_keys), input_ids=next_tokens if len(workers) == 1 else None,
            return_logits=return_logits,
        )
    except BaseException:
        for key, lens in lengths.items():
            _restore_kv_lengths_best_effort(workers, lens, key)
        raise


def _checked_lengths(
    lengths: list[int], query_len: int, max_positions: int | None, name: str, prefill_name: str
) -> list[int]:
    expected = None
    for i, kv_len in enumerate(lengths):
        if expected is None:
            expected = kv_len
        elif kv_len != expected:
            raise RuntimeError(
                "pipeline KV caches are out of sync: "
                f"stage 0 has {expected} tokens, stage {i} has {kv_len}"
            )
        if kv_len == 0:
            raise RuntimeError(
                f"{name} requires a prefilled KV cache; call {prefill_name} first"
            )
        if max_positions is not None and kv_len + query_len > max_positions:
            raise ValueError(
                f"decode would reach position {kv_len + query_len - 1}, "
                f"beyond model context {max_positions}"
            )
    return lengths


# ---------------------------------------------------------------------------
# Async variants (local or remote stages)
# ---------------------------------------------------------------------------

async def pipeline_prefill_async(
    workers: list[Any],
    input_ids: torch.Tensor,
    *,
    operation_id: int = 1,
    attempt_id: str = "a0",
    cache_key: str | None = None,
) -> torch.Tensor:
    if input_ids.ndim != 2:
        raise ValueError("input_ids must have shape [batch, sequence]")
    if input_ids.shape[0] < 1 or input_ids.shape[1] < 1:
        raise ValueError("input_ids must have a non-empty batch and sequence")
    if not workers:
        raise ValueError("workers must not be empty")
    max_positions = _max_positions(workers[0])
    if max_positions is not None and input_ids.shape[1] > max_positions:
        raise ValueError(
            f"prefill sequence length {input_ids.shape[1]} exceeds model context {max_positions}"
        )
    for worker in workers:
        await _async_stage_call(worker, "clear_kv", cache_key)
    hidden = None
    try:
        for index, worker in enumerate(workers):
            result = await _async_stage_call(
                worker, "forward_inference", hidden,
                input_ids=input_ids if index == 0 else None,
                operation_id=operation_id, attempt_id=attempt_id, reset_kv=False, cache_key=cache_key,
            )
            hidden = result.output
    except BaseException:
        await _clear_kv_async_best_effort(workers, cache_key)
        raise
    assert hidden is not None
    return hidden


async def pipeline_decode_step_async(
    workers: list[Any],
    next_token: torch.Tensor,
    *,
    operation_id: int,
    attempt_id: str = "a0",
    cache_key: str | None = None,
) -> torch.Tensor:
    if next_token.ndim != 2 or next_token.shape[0] < 1 or next_token.shape[1] < 1:
        raise ValueError("next_token must have shape [batch, sequence] with sequence >= 1")
    if not workers:
        raise ValueError("workers must not be empty")
    batch_size, query_len = next_token.shape
    max_positions = _max_positions(workers[0])
    lengths = [int(await _async_stage_call(w, "kv_cache_length", cache_key)) for w in workers]
    cache_lengths = _checked_lengths(
        lengths, query_len, max_positions, "pipeline_decode_step_async", "pipeline_prefill_async"
    )
    hidden = None
    try:
        for index, worker in enumerate(workers):
            kv_len = cache_lengths[index]
            position_ids = torch.arange(
                kv_len, kv_len + query_len, dtype=torch.long, device=next_token.device
            ).unsqueeze(0).expand(batch_size, -1)
            result = await _async_stage_call(
                worker, "forward_inference", hidden,
                input_ids=next_token if index == 0 else None, position_ids=position_ids,
                operation_id=operation_id, attempt_id=attempt_id, reset_kv=False, cache_key=cache_key,
            )
            hidden = result.output
    except BaseException:
        await _restore_kv_lengths_async_best_effort(workers, cache_lengths, cache_key)
        raise
    assert hidden is not None
    return hidden


async def _async_stage_call(worker: Any, method_name: str, *args: Any, **kwargs: Any) -> Any:
    """Run a synchronous stage method in a thread; on cancellation wait for it
    to finish before propagating, so cleanup never races a running call."""
    method = getattr(worker, method_name)
    if inspect.iscoroutinefunction(method):
        return await method(*args, **kwargs)
    task = asyncio.create_task(asyncio.to_thread(method, *args, **kwargs))
    try:
        return await asyncio.shield(task)
    except asyncio.CancelledError:
        try:
            await asyncio.shield(task)
        except BaseException:
            pass
        raise


def _clear_kv_best_effort(workers: Sequence[Any], cache_key: str | None) -> None:
    for worker in workers:
        try:
            worker.clear_kv(cache_key)
        except Exception as exc:
            log.warning("could not roll back stage KV cache: %s", exc)


def _restore_kv_lengths_best_effort(
    workers: Sequence[Any], lengths: Sequence[int], cache_key: str | None
) -> None:
    for worker, length in zip(workers, lengths):
        try:
            if length == 0:
                worker.clear_kv(cache_key)
            else:
                worker.trim_kv(length, cache_key)
        except Exception as exc:
            log.warning("could not roll back stage KV cache to %d: %s", length, exc)


async def _clear_kv_async_best_effort(workers: Sequence[Any], cache_key: str | None) -> None:
    for worker in workers:
        try:
            await _async_stage_call(worker, "clear_kv", cache_key)
        except Exception as exc:
            log.warning("could not roll back remote stage KV cache: %s", exc)


async def _restore_kv_lengths_async_best_effort(
    workers: Sequence[Any], lengths: Sequence[int], cache_key: str | None
) -> None:
    for worker, length in zip(workers, lengths):
        try:
            if length == 0:
                await _async_stage_call(worker, "clear_kv", cache_key)
            else:
                await _async_stage_call(worker, "trim_kv", length, cache_key)
        except Exception as exc:
            log.warning("could not roll back remote stage KV cache to %d: %s", length, exc)


__all__ = [
    "LlamaConfig",
    "build_pipeline",
    "from_reference_workers",
    "pipeline_prefill",
    "pipeline_decode_step",
    "pipeline_prefill_async",
    "pipeline_decode_step_async",
]
