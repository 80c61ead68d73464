"""Stage executor: the drop-in for the reference's ``StageWorker``.

``B200StageWorker`` has the methods and attributes callers of
``StageWorker`` use (backends/portable/stage_worker.py:103-453):
``forward_inference``, ``clear_kv``, ``clear_all_kv``, ``kv_cache_length``,
``trim_kv``, ``_model`` (with ``cfg``), ``_ctx`` and ``_saved``.  The KV cache
of every request context (``cache_key``) is a slot in the stage's HBM, owned
by the stage and never sent across the boundary (stage_worker.py:103-107).
Calls are serialised per stage by a re-entrant lock (stage_worker.py:117-121).
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Any

import torch

from gpu_mesh_b200.stage import B200Stage
from gpu_mesh_b200.boundary import move_to_stage


@dataclass
class StageContext:
    """Stage identity (stage_worker.py:30-63), with the same validation."""

    stage_id: int
    layer_start: int
    layer_end: int
    device: torch.device
    is_first: bool
    is_last: bool
    job_id: str
    attempt_id: str
    transport: str = "cpu"

    def __post_init__(self) -> None:
        for name, value in (
            ("stage_id", self.stage_id),
            ("layer_start", self.layer_start),
            ("layer_end", self.layer_end),
        ):
            if isinstance(value, bool) or not isinstance(value, int):
                raise TypeError(f"{name} must be an integer")
        if self.stage_id < 0:
            raise ValueError("stage_id must be non-negative")
        if self.layer_start < 0 or self.layer_end <= self.layer_start:
            raise ValueError("StageContext must own a non-empty layer range")
        self.device = torch.device(self.device)
        if self.transport not in {"cpu", "local_cuda"}:
            raise ValueError(f"unsupported stage transport: {self.transport!r}")
        if not self.job_id:
            raise ValueError("job_id must not be empty")
        if not self.attempt_id:
            raise ValueError("attempt_id must not be empty")


@dataclass
class ForwardResult:
    """Result of one stage forward (stage_worker.py:66-74)."""

    stage_id: int
    operation_id: int
    attempt_id: str
    output: torch.Tensor
    kv_caches: Any
    _boundary_tensor: torch.Tensor | None = field(default=None, repr=False)


class KVSlotRef:
    """Handle to a stage-owned KV slot; ``export()`` copies it out as the
    reference's list of per-layer (k, v) tensors."""

    def __init__(self, stage: B200Stage, slot: int) -> None:
        self.stage = stage
        self.slot = slot

    def __len__(self) -> int:
        return self.stage.layer_end - self.stage.layer_start

    def export(self) -> list[tuple[torch.Tensor, torch.Tensor]]:
        return self.stage.kv_export(self.slot)


class B200StageWorker:
    """Owns one ``B200Stage`` and its per-request KV slots."""

    def __init__(self, model: B200Stage, ctx: StageContext, *, check_values: bool = True) -> None:
        self._model = model
        self._ctx = ctx
        self._inference_lock = threading.RLock()
        self._saved: dict[int, dict[str, Any]] = {}
        # cache_key -> slot id; ``None`` is the legacy default context.
        self._slots: dict[str | None, int] = {None: 0}
        self._next_slot = 1
        self.check_values = check_values

    # ------------------------------------------------------------------
    def _slot(self, cache_key: str | None) -> int:
        slot = self._slots.get(cache_key)
        if slot is None:
            slot = self._next_slot
            self._next_slot += 1
            self._slots[cache_key] = slot
        return slot

    def slot_of(self, cache_key: str | None) -> int:
        with self._inference_lock:
            return self._slot(cache_key)

    @torch.no_grad()
    def forward_inference(
        self,
        hidden: torch.Tensor | None,
        *,
        input_ids: torch.Tensor | None = None,
        position_ids: torch.Tensor | None = None,
        attention_mask: torch.Tensor | None = None,
        operation_id: int,
        attempt_id: str,
        reset_kv: bool = False,
        cache_key: str | None = None,
        logits: str = "all",
    ) -> ForwardResult:
        """StageWorker.forward_inference (stage_worker.py:129-170).

        ``logits="last"`` (an addition) makes the last stage return only the
        final position's logits, which is all a sampler needs.
        """
        if attention_mask is not None:
            raise ValueError(
                "explicit attention masks are not supported by the B200 stage; "
                "the causal policy is derived from position_ids"
            )
        with self._inference_lock:
            if reset_kv:
                self.clear_kv(cache_key)
            x = None
            if hidden is not None and hidden.numel() > 0:
                x = self._move_input(hidden)
            slot = self._slot(cache_key)
            out = self._model.forward_slot(
                slot,
                x,
                input_ids=input_ids,
                position_ids=position_ids,
                logits=logits,
                check_values=self.check_values,
            )
        return ForwardResult(
            stage_id=self._ctx.stage_id,
            operation_id=operation_id,
            attempt_id=attempt_id,
            output=self._boundary_output(out),
            kv_caches=KVSlotRef(self._model, slot),
        )

    def decode_multi(
        self,
        hidden: torch.Tensor | None,
        cache_keys: list[str | None],
        *,
        input_ids: torch.Tensor | None = None,
        logits: str = "last",
    ) -> torch.Tensor:
        """One decode token for several request contexts in one weight pass."""
        with self._inference_lock:
            slots = [self._slot(k) for k in cache_keys]
            x = None
            if hidden is not None:
                x = self._move_input(hidden)
            out = self._model.decode_multi(slots, x, input_ids=input_ids, logits=logits)
        return self._boundary_output(out)

    def decode_greedy(
        self,
        hidden: torch.Tensor | None,
        cache_keys: list[str | None],
        *,
        input_ids: torch.Tensor | None = None,
        return_logits: bool = False,
    ) -> tuple[torch.Tensor, torch.Tensor | None]:
        """``decode_multi`` on the last stage returning each row's greedy token
        (int64 [rows], on the host for transport "cpu") and, if asked, the
        logits."""
        with self._inference_lock:
            slots = [self._slot(k) for k in cache_keys]
            x = None
            if hidden is not None:
                x = self._move_input(hidden)
            tokens, logits = self._model.decode_greedy(slots, x, input_ids=input_ids,
                                                       return_logits=return_logits)
        return self._boundary_output(tokens), (None if logits is None else self._boundary_output(logits))

    def decode_top_p(
        self,
        hidden: torch.Tensor | None,
        cache_keys: list[str | None],
        *,
        temperature: float,
        top_p: float,
        uniforms: torch.Tensor,
        input_ids: torch.Tensor | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """``decode_multi`` on the last stage returning each row's top-p token
        for ``uniforms`` (drawn on the device) and the logits."""
        with self._inference_lock:
            slots = [self._slot(k) for k in cache_keys]
            x = None
            if hidden is not None:
                x = self._move_input(hidden)
            tokens, logits = self._model.decode_top_p(slots, x, temperature=temperature, top_p=top_p,
                                                      uniforms=uniforms, input_ids=input_ids)
        return self._boundary_output(tokens), self._boundary_output(logits)

    # ------------------------------------------------------------------
    # KV ownership (stage_worker.py:358-416)
    # ------------------------------------------------------------------
    def clear_kv(self, cache_key: str | None = None) -> None:
        with self._inference_lock:
            slot = self._slots.get(cache_key)
            if slot is not None:
                self._model.kv_free(slot)
                if cache_key is not None:
                    del self._slots[cache_key]

    @property
    def _kv_caches_by_key(self) -> dict[str | None, KVSlotRef]:
        """The named request contexts this stage holds, as the reference
        worker's dict of the same name lists them (stage_worker.py:112-116,
        358-381; the unnamed default context is not in it)."""
        with self._inference_lock:
            return {k: KVSlotRef(self._model, s) for k, s in self._slots.items() if k is not None}

    def clear_all_kv(self) -> None:
        with self._inference_lock:
            self._model.kv_free_all()
            self._slots = {None: 0}

    def kv_cache_length(self, cache_key: str | None = None) -> int:
        with self._inference_lock:
            slot = self._slots.get(cache_key)
            return 0 if slot is None else self._model.kv_length(slot)

    def trim_kv(self, length: int, cache_key: str | None = None) -> None:
        if length < 0:
            raise ValueError("cache length must be non-negative")
        with self._inference_lock:
            slot = self._slots.get(cache_key)
            if slot is None or self._model.kv_length(slot) == 0:
                if length:
                    raise RuntimeError("cannot trim an empty cache to a non-zero length")
                return
            self._model.kv_trim(slot, length)

    def reserve_kv(self, cache_key: str | None, batch: int, capacity: int) -> None:
        """Pre-size a context's slot so decode never regrows it."""
        with self._inference_lock:
            self._model.kv_reserve(self._slot(cache_key), batch, capacity)

    def import_kv(self, cache_key: str | None, caches: list[tuple[torch.Tensor, torch.Tensor]]) -> None:
        """Load a context from the reference's list of per-layer (k, v) tensors."""
        with self._inference_lock:
            slot = self._slot(cache_key)
            if len(caches) != self._model.layer_end - self._model.layer_start:
                raise ValueError(
                    f"expected {self._model.layer_end - self._model.layer_start} KV cache entries, "
                    f"got {len(caches)}"
                )
            for layer, (k, v) in enumerate(caches):
                self._model.kv_import(slot, layer, k, v)

    def check_device(self) -> None:
        self._model.check_device()

    def clear_saved(self, operation_id: int | None = None) -> None:
        if operation_id is None:
            self._saved.clear()
        else:
            self._saved.pop(operation_id, None)

    def close(self) -> None:
        self._model.close()

    # ------------------------------------------------------------------
    def _move_input(self, hidden: torch.Tensor) -> torch.Tensor:
        return move_to_stage(hidden, self._ctx.device, transport=self._ctx.transport)

    def _boundary_output(self, output: torch.Tensor) -> torch.Tensor:
        """Detached output; CPU for transport "cpu" (stage_worker.py:436-442)."""
        if self._ctx.transport == "local_cuda":
            return output.detach()
        if self._ctx.transport == "cpu":
            return output.detach().cpu()
        raise ValueError(f"unsupported stage transport: {self._ctx.transport!r}")
