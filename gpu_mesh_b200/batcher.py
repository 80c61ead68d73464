"""Continuous batching over the stage-owned KV (inference/batcher.py of the reference).

Same public surface as the reference's ``ContinuousBatcher`` (batcher.py:56-426):
``start`` / ``stop`` / ``wait_stopped`` / ``submit`` / ``stream`` /
``active_count`` / ``pending_count``, the same validation messages, the same
``SessionResult`` stream (``seq_num`` monotone, ``is_last`` on EOS or
``max_new_tokens``, ``token_id = -1`` on failure or cancellation) and the same
cache ownership (one ``seq:<id>`` context per request, cleared on finish,
failure, cancellation and stop).

The decode loop is what changes. The reference decodes its active sequences
one after another (batcher.py:229-247), each step a full pass over every
stage's weights for one context. Here one iteration is a single
``pipeline_decode_multi`` call for all active sequences: every stage reads
its weights once for the batch, and each row attends to its own context's
cache at its own length. Sampling follows the reference's ``_sample``
(session.py:245-259): greedy at temperature 0, else top-p with the request's
seeded generator. If the batched step fails, the loop retries the step one
sequence at a time, so a failing context is isolated the way the reference
isolates it (its own ``-1`` result, its cache cleared).
"""
from __future__ import annotations

import asyncio
import logging
import time
import uuid
from dataclasses import dataclass, field
from typing import Any

import torch

from gpu_mesh_b200.pipeline import (
    pipeline_decode_greedy,
    pipeline_decode_multi,
    pipeline_decode_step,
    pipeline_prefill,
)
from gpu_mesh_b200.sampling import SamplingParams, greedy_sample, make_sampling_generator, top_p_sample

log = logging.getLogger(__name__)


@dataclass
class SessionResult:
    """One streamed token (inference/session.py:32-37)."""

    token_id: int
    seq_num: int  # monotone; the client dedupes replayed tokens by it
    is_last: bool
    text: str = ""


@dataclass
class _Sequence:
    seq_id: str
    prompt_ids: list[int]
    sampling: SamplingParams
    max_new_tokens: int
    result_queue: asyncio.Queue
    generator: torch.Generator | None = None
    generator_device: torch.device | None = None
    generated: list[int] = field(default_factory=list)
    seq_num: int = 0
    finished: bool = False
    cancelled: bool = False
    started_at: float = field(default_factory=time.time)

    def last_token(self) -> int:
        return self.generated[-1] if self.generated else self.prompt_ids[-1]

    @property
    def total_generated(self) -> int:
        return len(self.generated)

    @property
    def cache_key(self) -> str:
        return f"seq:{self.seq_id}"


class ContinuousBatcher:
    """Drives one batched decode loop across the active sequences.

    Usage (as the reference)::

        batcher = ContinuousBatcher(workers, max_batch_size=8)
        batcher.start()
        seq_id = await batcher.submit(prompt_ids, sampling, max_new_tokens)
        async for result in batcher.stream(seq_id):
            ...
        batcher.stop()
    """

    def __init__(self, workers: list[Any], max_batch_size: int = 8) -> None:
        if not workers:
            raise ValueError("workers must not be empty")
        if max_batch_size < 1:
            raise ValueError("max_batch_size must be positive")
        self._workers = workers
        self._max_batch = max_batch_size
        self._active: dict[str, _Sequence] = {}
        self._pending: asyncio.Queue[_Sequence] = asyncio.Queue()
        self._pending_by_id: dict[str, _Sequence] = {}
        self._queues: dict[str, asyncio.Queue] = {}
        self._stream_consumers: set[str] = set()
        self._lock = asyncio.Lock()
        self._running = False
        self._stopping = False
        self._loop_task: asyncio.Task | None = None
        self._inflight: set[asyncio.Task] = set()
        self._op_seq = 0
        self.decode_passes = 0  # batched decode calls made (one weight pass each)

    def _next_op(self) -> int:
        self._op_seq += 1
        return self._op_seq

    # ------------------------------------------------------------------
    # Public API (batcher.py:104-219)
    # ------------------------------------------------------------------

    def start(self) -> None:
        if self._running:
            return
        if self._loop_task is not None and not self._loop_task.done():
            raise RuntimeError("batcher is still stopping; await wait_stopped() before restarting")
        self._running = True
        self._stopping = False
        self._loop_task = asyncio.ensure_future(self._decode_loop())

    def stop(self) -> None:
        self._running = False
        if self._loop_task is not None and not self._loop_task.done():
            self._stopping = True
        for seq in list(self._active.values()):
            if not seq.finished:
                seq.finished = True
                seq.cancelled = True
                seq.result_queue.put_nowait(SessionResult(token_id=-1, seq_num=seq.seq_num, is_last=True))
        while True:
            try:
                seq = self._pending.get_nowait()
            except asyncio.QueueEmpty:
                break
            seq.finished = True
            seq.cancelled = True
            self._pending_by_id.pop(seq.seq_id, None)
            seq.result_queue.put_nowait(SessionResult(token_id=-1, seq_num=seq.seq_num, is_last=True))
        if self._loop_task:
            self._loop_task.cancel()

    async def wait_stopped(self) -> None:
        """Wait until a canceled decode loop has drained its worker threads."""
        task = self._loop_task
        if task is None:
            return
        try:
            await task
        except asyncio.CancelledError:
            pass

    async def submit(self, prompt_ids: list[int], sampling: SamplingParams, max_new_tokens: int) -> str:
        """Submit a new request; returns seq_id for streaming."""
        if not self._running:
            raise RuntimeError("batcher is not running; call start() first")
        if not prompt_ids:
            raise ValueError("prompt_ids must not be empty")
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be positive")
        model_cfg = getattr(getattr(self._workers[0], "_model", None), "cfg", None)
        vocab_size = getattr(model_cfg, "vocab_size", None)
        prompt_ids = list(prompt_ids)
        if vocab_size is not None and any(token < 0 or token >= vocab_size for token in prompt_ids):
            raise ValueError("prompt contains an out-of-vocabulary token")
        max_positions = getattr(model_cfg, "max_position_embeddings", None)
        if max_positions is not None and len(prompt_ids) + max_new_tokens > max_positions:
            raise ValueError(
                f"prompt ({len(prompt_ids)}) + max_new_tokens ({max_new_tokens}) "
                f"exceeds model context {max_positions}"
            )
        seq_id = uuid.uuid4().hex[:12]
        q: asyncio.Queue = asyncio.Queue()
        seq = _Sequence(seq_id=seq_id, prompt_ids=prompt_ids, sampling=sampling,
                        max_new_tokens=max_new_tokens, result_queue=q)
        async with self._lock:
            if not self._running:
                raise RuntimeError("batcher is not running; call start() first")
            self._queues[seq_id] = q
            self._pending_by_id[seq_id] = seq
            await self._pending.put(seq)
        return seq_id

    async def stream(self, seq_id: str):
        """Async generator: yields SessionResult for each generated token."""
        q = self._queues.get(seq_id)
        if q is None:
            raise RuntimeError(f"seq {seq_id} not found — call submit() first")
        async with self._lock:
            if seq_id in self._stream_consumers:
                raise RuntimeError(f"seq {seq_id} already has an active stream consumer")
            self._stream_consumers.add(seq_id)
        completed = False
        try:
            while True:
                result: SessionResult = await q.get()
                yield result
                if result.is_last:
                    completed = True
                    self._queues.pop(seq_id, None)
                    break
        finally:
            if not completed:
                await self._cancel_sequence(seq_id)
                self._queues.pop(seq_id, None)
            async with self._lock:
                self._stream_consumers.discard(seq_id)

    @property
    def active_count(self) -> int:
        return len(self._active)

    @property
    def pending_count(self) -> int:
        return self._pending.qsize()

    # ------------------------------------------------------------------
    # Decode loop
    # ------------------------------------------------------------------

    async def _decode_loop(self) -> None:
        try:
            while self._running:
                await self._admit_pending()
                if not self._active:
                    await asyncio.sleep(0.01)
                    continue
                batch = [s for s in self._active.values() if not s.finished]
                if batch:
                    results = await self._run_sync(self._decode_batch_sync, batch)
                    for seq, result in zip(batch, results):
                        if result is not None and not seq.cancelled:
                            await seq.result_queue.put(result)
                async with self._lock:
                    for sid in [sid for sid, s in self._active.items() if s.finished]:
                        finished_seq = self._active.pop(sid)
                        self._clear_sequence_cache(finished_seq)
        finally:
            try:
                if self._inflight:
                    await asyncio.gather(*tuple(self._inflight), return_exceptions=True)
                for seq in list(self._active.values()):
                    self._clear_sequence_cache(seq)
                self._active.clear()
            finally:
                self._running = False
                self._stopping = False

    async def _admit_pending(self) -> None:
        for _ in range(self._max_batch):
            async with self._lock:
                if len(self._active) >= self._max_batch:
                    break
                try:
                    seq = self._pending.get_nowait()
                except asyncio.QueueEmpty:
                    break
                self._pending_by_id.pop(seq.seq_id, None)
                if seq.cancelled:
                    continue
                self._active[seq.seq_id] = seq
            result = await self._run_sync(self._prefill_sync, seq)
            if result is not None and not seq.cancelled:
                await seq.result_queue.put(result)

    async def _cancel_sequence(self, seq_id: str) -> None:
        async with self._lock:
            sequence = self._active.get(seq_id) or self._pending_by_id.get(seq_id)
            if sequence is None:
                return
            sequence.cancelled = True
            sequence.finished = True
            self._pending_by_id.pop(seq_id, None)

    async def _run_sync(self, function, *args):
        """Run a blocking stage operation and retain it across cancellation."""
        task = asyncio.create_task(asyncio.to_thread(function, *args))
        self._inflight.add(task)
        task.add_done_callback(self._inflight.discard)
        try:
            return await asyncio.shield(task)
        finally:
            if task.done():
                self._inflight.discard(task)

    # ------------------------------------------------------------------
    # Blocking steps (run in a worker thread)
    # ------------------------------------------------------------------

    def _sample_row(self, seq: _Sequence, logits: torch.Tensor) -> int:
        """The reference's ``_sample`` for one row of logits [V]."""
        if seq.sampling.temperature == 0.0:
            return int(greedy_sample(logits))
        return int(top_p_sample(logits, seq.sampling.temperature, seq.sampling.top_p,
                                generator=self._generator_for(seq, logits)))

    def _advance(self, seq: _Sequence, next_id: int) -> SessionResult:
        seq.generated.append(next_id)
        seq.seq_num += 1
        eos = seq.sampling.eos_token_id
        is_last = (eos is not None and next_id == eos) or seq.total_generated >= seq.max_new_tokens
        seq.finished = is_last
        if is_last:
            self._clear_sequence_cache(seq)
        return SessionResult(token_id=next_id, seq_num=seq.seq_num, is_last=is_last)

    def _fail(self, seq: _Sequence, seq_num: int) -> SessionResult:
        self._clear_sequence_cache(seq)
        seq.finished = True
        return SessionResult(token_id=-1, seq_num=seq_num, is_last=True)

    def _prefill_sync(self, seq: _Sequence) -> SessionResult | None:
        try:
            input_ids = torch.tensor([seq.prompt_ids], dtype=torch.long)
            logits = pipeline_prefill(self._workers, input_ids, operation_id=self._next_op(),
                                      attempt_id=f"pf_{seq.seq_id}", cache_key=seq.cache_key)
            return self._advance(seq, self._sample_row(seq, logits[0, -1, :]))
        except Exception:
            log.exception("prefill failed for seq %s", seq.seq_id)
            return self._fail(seq, 0)

    def _decode_batch_sync(self, batch: list[_Sequence]) -> list[SessionResult | None]:
        live = [s for s in batch if not s.finished]
        if not live:
            return [None] * len(batch)
        try:
            ids = torch.tensor([[s.last_token()] for s in live], dtype=torch.long)
            keys = [s.cache_key for s in live]
            greedy = [i for i, s in enumerate(live) if s.sampling.temperature == 0.0]
            if len(greedy) == len(live) and hasattr(self._workers[-1], "decode_greedy"):
                # every row greedy: the last stage selects on the device, no logits leave it
                chosen, _ = pipeline_decode_greedy(self._workers, ids, cache_keys=keys)
                self.decode_passes += 1
                out = {id(s): self._advance(s, int(t)) for s, t in zip(live, chosen.tolist())}
                return [out.get(id(s)) for s in batch]
            logits = pipeline_decode_multi(self._workers, ids, cache_keys=keys)
            self.decode_passes += 1
            tokens: dict[int, int] = {}
            if greedy:
                sel = torch.tensor(greedy, device=logits.device)
                for i, t in zip(greedy, greedy_sample(logits[sel, -1, :]).tolist()):
                    tokens[i] = int(t)
            for i, s in enumerate(live):
                if i not in tokens:
                    tokens[i] = self._sample_row(s, logits[i, -1, :])
            out = {id(s): self._advance(s, tokens[i]) for i, s in enumerate(live)}
        except Exception:
            log.exception("batched decode failed; retrying %d sequences one by one", len(live))
            out = {id(s): self._decode_one_sync(s) for s in live}
        return [out.get(id(s)) for s in batch]

    def _decode_one_sync(self, seq: _Sequence) -> SessionResult | None:
        if seq.finished:
            return None
        try:
            next_input = torch.tensor([[seq.last_token()]], dtype=torch.long)
            logits = pipeline_decode_step(self._workers, next_input, operation_id=self._next_op(),
                                          attempt_id=f"dc_{seq.seq_id}", cache_key=seq.cache_key)
            return self._advance(seq, self._sample_row(seq, logits[0, -1, :]))
        except Exception:
            log.exception("decode failed for seq %s", seq.seq_id)
            return self._fail(seq, seq.seq_num)

    def _clear_sequence_cache(self, seq: _Sequence) -> None:
        for worker in self._workers:
            try:
                worker.clear_kv(seq.cache_key)
            except Exception as exc:
                log.warning("could not clear batcher cache for seq %s on stage: %s", seq.seq_id, exc)

    @staticmethod
    def _generator_for(seq: _Sequence, logits: torch.Tensor) -> torch.Generator | None:
        """One request RNG on the device where its logits are sampled."""
        if seq.sampling.seed is None:
            return None
        device = torch.device(logits.device)
        if seq.generator is None:
            seq.generator = make_sampling_generator(seq.sampling, device=device)
            seq.generator_device = device
        elif seq.generator_device != device:
            raise RuntimeError(
                "sampling logits changed device during one sequence: "
                f"{seq.generator_device} -> {device}"
            )
        return seq.generator
