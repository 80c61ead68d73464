"""Continuous batching over the stage-owned KV cache.

Public surface of the reference's ``ContinuousBatcher``
(inference/batcher.py:56-426), kept so its callers work unchanged:
``start`` / ``stop`` / ``wait_stopped`` / ``submit`` / ``stream`` /
``active_count`` / ``pending_count``, the same validation messages, the same
``SessionResult`` stream (``seq_num`` counts tokens from 1, ``is_last`` on EOS
or ``max_new_tokens``, one ``token_id = -1`` result on failure, cancellation
or stop) and one ``seq:<id>`` context per request, cleared when it ends.

The engine is this module's own.  The reference runs its loop as an asyncio
task that hands each stage call to a thread and decodes its active sequences
one after another (batcher.py:229-247), a full pass over every weight per
sequence and token.  Here one engine thread owns every stage call:

* each iteration admits pending requests up to ``max_batch_size`` (one
  prefill each, its first token sampled from the prefill's last position),
  then runs ONE batched decode over every active request:
  ``pipeline_decode_greedy`` when all rows are greedy (the token is chosen
  inside the last stage's lm_head and only ids leave the GPU), else
  ``pipeline_decode_multi`` and per-row sampling.  Every request keeps its own
  KV slot and length; each weight is read once per iteration for all of them;
* results go to each request's asyncio queue through
  ``loop.call_soon_threadsafe``; the event loop never blocks on the GPU;
* a request ends exactly once (``_finish``, under a lock): by EOS or its
  token budget, by a failure, by its stream being closed, or by ``stop``;
* if a batched decode fails, every context is rolled back by the pipeline and
  the iteration is retried one request at a time, so only the failing
  request ends with ``-1`` (the reference's isolation).

Sampling follows the reference's ``_sample`` (inference/session.py:245-259):
greedy at temperature 0, else top-p with the request's seeded generator.
"""
from __future__ import annotations

import asyncio
import logging
import threading
import uuid
from collections import deque
from dataclasses import dataclass
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


class _Request:
    """One request as the engine sees it."""

    __slots__ = ("rid", "prompt", "sampling", "budget", "tokens", "queue", "loop", "generator",
                 "generator_device", "ended", "cancel")

    def __init__(self, rid: str, prompt: list[int], sampling: SamplingParams, budget: int,
                 queue: asyncio.Queue, loop: asyncio.AbstractEventLoop) -> None:
        self.rid = rid
        self.prompt = prompt
        self.sampling = sampling
        self.budget = budget
        self.tokens: list[int] = []
        self.queue = queue
        self.loop = loop
        self.generator: torch.Generator | None = None
        self.generator_device: torch.device | None = None
        self.ended = False     # its terminal result has been queued
        self.cancel = False    # its stream was closed: end it at the next iteration

    @property
    def key(self) -> str:
        return f"seq:{self.rid}"

    @property
    def next_input(self) -> int:
        return self.tokens[-1] if self.tokens else self.prompt[-1]


class ContinuousBatcher:
    """Batched decode of concurrent requests over shared stage workers.

    Usage (as the reference)::

        batcher = ContinuousBatcher(workers, max_batch_size=8)
        batcher.start()
        seq_id = await batcher.submit(prompt_ids, sampling, max_new_tokens)
        async for result in batcher.stream(seq_id):
            ...
        batcher.stop()
        await batcher.wait_stopped()
    """

    def __init__(self, workers: list[Any], max_batch_size: int = 8) -> None:
        if not workers:
            raise ValueError("workers must not be empty")
        if max_batch_size < 1:
            raise ValueError("max_batch_size must be positive")
        self._workers = workers
        self._max_batch = max_batch_size
        self._lock = threading.Lock()
        self._wake = threading.Condition(self._lock)
        self._pending: deque[_Request] = deque()
        self._active: list[_Request] = []
        self._requests: dict[str, _Request] = {}  # until their stream has read the last result
        self._streaming: set[str] = set()
        self._thread: threading.Thread | None = None
        self._stopped: asyncio.Future | None = None
        self._running = False
        self._op = 0
        self.decode_passes = 0  # batched decode calls made (one weight pass each)

    # ------------------------------------------------------------------
    # Front end (event loop side)
    # ------------------------------------------------------------------

    def start(self) -> None:
        if self._running:
            return
        if self._thread is not None and self._thread.is_alive():
            raise RuntimeError("batcher is still stopping; await wait_stopped() before restarting")
        loop = asyncio.get_event_loop()
        self._stopped = loop.create_future()
        self._running = True
        self._thread = threading.Thread(target=self._engine, args=(loop, self._stopped),
                                        name="b200-batcher", daemon=True)
        self._thread.start()

    def stop(self) -> None:
        """End every pending and active request with a ``-1`` result and let
        the engine release their contexts and exit."""
        with self._lock:
            self._running = False
            for req in list(self._pending) + self._active:
                self._finish(req, -1)
            self._wake.notify_all()

    async def wait_stopped(self) -> None:
        """Wait until the engine thread has released every context and exited."""
        if self._stopped is not None:
            await asyncio.shield(self._stopped)

    async def submit(self, prompt_ids: list[int], sampling: SamplingParams, max_new_tokens: int) -> str:
        """Queue a request; returns its seq_id for ``stream``."""
        if not self._running:
            raise RuntimeError("batcher is not running; call start() first")
        if not prompt_ids:
            raise ValueError("prompt_ids must not be empty")
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be positive")
        cfg = getattr(getattr(self._workers[0], "_model", None), "cfg", None)
        prompt = [int(t) for t in prompt_ids]
        vocab = getattr(cfg, "vocab_size", None)
        if vocab is not None and any(t < 0 or t >= vocab for t in prompt):
            raise ValueError("prompt contains an out-of-vocabulary token")
        limit = getattr(cfg, "max_position_embeddings", None)
        if limit is not None and len(prompt) + max_new_tokens > limit:
            raise ValueError(
                f"prompt ({len(prompt)}) + max_new_tokens ({max_new_tokens}) exceeds model context {limit}"
            )
        req = _Request(uuid.uuid4().hex[:12], prompt, sampling, max_new_tokens, asyncio.Queue(),
                       asyncio.get_running_loop())
        with self._lock:
            if not self._running:
                raise RuntimeError("batcher is not running; call start() first")
            self._requests[req.rid] = req
            self._pending.append(req)
            self._wake.notify_all()
        return req.rid

    async def stream(self, seq_id: str):
        """Async generator of the request's SessionResults.  Closing it before
        the last result cancels the request and releases its context."""
        with self._lock:
            req = self._requests.get(seq_id)
            if req is None:
                raise RuntimeError(f"seq {seq_id} not found — call submit() first")
            if seq_id in self._streaming:
                raise RuntimeError(f"seq {seq_id} already has an active stream consumer")
            self._streaming.add(seq_id)
        done = False
        try:
            while True:
                result: SessionResult = await req.queue.get()
                yield result
                if result.is_last:
                    done = True
                    break
        finally:
            with self._lock:
                self._streaming.discard(seq_id)
                if not done and not req.ended:
                    req.cancel = True
                    if req in self._pending:  # never admitted: end it here
                        self._pending.remove(req)
                        self._finish(req, -1)
                    self._wake.notify_all()
                if req.ended:
                    self._requests.pop(seq_id, None)

    @property
    def active_count(self) -> int:
        return len(self._active)

    @property
    def pending_count(self) -> int:
        return len(self._pending)

    # ------------------------------------------------------------------
    # Results
    # ------------------------------------------------------------------

    def _finish(self, req: _Request, token: int) -> None:
        """Queue the terminal result of ``req`` once (call with the lock held)."""
        if req.ended:
            return
        req.ended = True
        self._emit(req, SessionResult(token_id=token, seq_num=len(req.tokens), is_last=True))

    @staticmethod
    def _emit(req: _Request, result: SessionResult) -> None:
        try:
            req.loop.call_soon_threadsafe(req.queue.put_nowait, result)
        except RuntimeError:  # the event loop has closed; nobody is listening
            pass

    def _take(self, req: _Request, token: int) -> None:
        """Record a sampled token; the request ends on EOS or its budget."""
        with self._lock:
            if req.ended:
                return
            req.tokens.append(token)
            eos = req.sampling.eos_token_id
            last = (eos is not None and token == eos) or len(req.tokens) >= req.budget
            if last:
                req.ended = True
            self._emit(req, SessionResult(token_id=token, seq_num=len(req.tokens), is_last=last))

    # ------------------------------------------------------------------
    # Engine (its own thread; every stage call happens here)
    # ------------------------------------------------------------------

    def _engine(self, loop: asyncio.AbstractEventLoop, stopped: asyncio.Future) -> None:
        try:
            while True:
                with self._lock:
                    while self._running and not self._pending and not self._active:
                        self._wake.wait(timeout=0.05)
                    if not self._running:
                        break
                    room = self._max_batch - len(self._active)
                    admitted = [self._pending.popleft() for _ in range(min(room, len(self._pending)))]
                    self._active.extend(admitted)
                for req in admitted:
                    if not req.cancel:
                        self._prefill(req)
                self._decode([r for r in self._active if not r.ended and not r.cancel and r.tokens])
                self._retire()
        except Exception:
            log.exception("batcher engine failed")
        finally:
            with self._lock:
                self._running = False
                leftovers = list(self._pending) + self._active
                self._pending.clear()
                self._active = []
                for req in leftovers:
                    self._finish(req, -1)
            for req in leftovers:
                self._release(req)
            try:
                loop.call_soon_threadsafe(lambda: stopped.done() or stopped.set_result(None))
            except RuntimeError:
                pass

    def _retire(self) -> None:
        """Drop ended or cancelled requests from the batch and free their contexts."""
        with self._lock:
            gone = [r for r in self._active if r.ended or r.cancel]
            self._active = [r for r in self._active if not (r.ended or r.cancel)]
            for r in gone:
                self._finish(r, -1)  # no-op for a request that already ended
        for r in gone:
            self._release(r)

    def _release(self, req: _Request) -> None:
        for w in self._workers:
            try:
                w.clear_kv(req.key)
            except Exception as exc:
                log.warning("could not clear the context of seq %s: %s", req.rid, exc)

    def _next_op(self) -> int:
        self._op += 1
        return self._op

    def _prefill(self, req: _Request) -> None:
        try:
            logits = pipeline_prefill(self._workers, torch.tensor([req.prompt], dtype=torch.long),
                                      operation_id=self._next_op(), attempt_id=f"pf_{req.rid}",
                                      cache_key=req.key)
            self._take(req, self._sample(req, logits[0, -1]))
        except Exception:
            log.exception("prefill failed for seq %s", req.rid)
            with self._lock:
                self._finish(req, -1)

    def _decode(self, batch: list[_Request]) -> None:
        if not batch:
            return
        ids = torch.tensor([[r.next_input] for r in batch], dtype=torch.long)
        keys = [r.key for r in batch]
        try:
            if all(r.sampling.temperature == 0.0 for r in batch) and hasattr(self._workers[-1], "decode_greedy"):
                chosen, _ = pipeline_decode_greedy(self._workers, ids, cache_keys=keys)
                self.decode_passes += 1
                picks = [int(t) for t in chosen.tolist()]
            else:
                logits = pipeline_decode_multi(self._workers, ids, cache_keys=keys)
                self.decode_passes += 1
                picks = self._sample_rows(batch, logits[:, -1])
        except Exception:
            log.exception("batched decode failed; retrying %d requests one at a time", len(batch))
            for req in batch:
                self._decode_alone(req)
            return
        for req, token in zip(batch, picks):
            self._take(req, token)

    def _decode_alone(self, req: _Request) -> None:
        try:
            logits = pipeline_decode_step(self._workers, torch.tensor([[req.next_input]], dtype=torch.long),
                                          operation_id=self._next_op(), attempt_id=f"dc_{req.rid}",
                                          cache_key=req.key)
            self._take(req, self._sample(req, logits[0, -1]))
        except Exception:
            log.exception("decode failed for seq %s", req.rid)
            with self._lock:
                self._finish(req, -1)

    # ------------------------------------------------------------------
    # Sampling
    # ------------------------------------------------------------------

    def _sample_rows(self, batch: list[_Request], logits: torch.Tensor) -> list[int]:
        """Greedy rows in one argmax launch, the rest with their own generators."""
        picks: list[int | None] = [None] * len(batch)
        greedy = [i for i, r in enumerate(batch) if r.sampling.temperature == 0.0]
        if greedy:
            rows = torch.tensor(greedy, device=logits.device)
            for i, t in zip(greedy, greedy_sample(logits[rows]).tolist()):
                picks[i] = int(t)
        for i, r in enumerate(batch):
            if picks[i] is None:
                picks[i] = self._sample(r, logits[i])
        return picks

    def _sample(self, req: _Request, logits: torch.Tensor) -> int:
        """The reference's ``_sample`` for one row of logits [V]."""
        if req.sampling.temperature == 0.0:
            return int(greedy_sample(logits))
        return int(top_p_sample(logits, req.sampling.temperature, req.sampling.top_p,
                                generator=self._generator(req, logits.device)))

    @staticmethod
    def _generator(req: _Request, device: torch.device) -> torch.Generator | None:
        """One RNG per seeded request, on the device its logits are sampled on."""
        if req.sampling.seed is None:
            return None
        device = torch.device(device)
        if req.generator is None:
            req.generator = make_sampling_generator(req.sampling, device=device)
            req.generator_device = device
        elif req.generator_device != device:
            raise RuntimeError(
                f"sampling logits changed device during one sequence: {req.generator_device} -> {device}"
            )
        return req.generator
