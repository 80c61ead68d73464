"""Micro-batches in flight across pipeline stages on the GPUs of one process.

The reference runs one request batch through its stages strictly in order
(backends/portable/pipeline.py:210-228): while stage s works, every other
stage idles.  ``MicroBatchPipeline`` splits the work into micro-batches, one
request context (``cache_key``, its own KV slot on every stage) each, and
queues (step k, micro-batch m, stage s) in k-major, then m, then s order.
Nothing in the loop waits on the host: each stage's kernels go to its own
device's stream, a boundary tensor moves by a side-stream peer copy ordered
by events (``gpu_mesh_b200.boundary.Link``), and the greedy token of the last
stage returns to stage 0's device the same way.  So stage s runs
micro-batch m while stage s+1 runs m-1, and with at least as many
micro-batches as stages every GPU is busy.  The host reads the generated ids
once, at the end.

Stages on the same device hand tensors over directly; one device holding
every stage is the plain sequential pipeline.
"""
from __future__ import annotations

from collections.abc import Sequence

import torch

from gpu_mesh_b200.boundary import Link
from gpu_mesh_b200.sampling import greedy_sample
from gpu_mesh_b200.stage_worker import B200StageWorker


class MicroBatchPipeline:
    """Greedy generation over B200 stages with micro-batches in flight."""

    def __init__(self, workers: Sequence[B200StageWorker]) -> None:
        if not workers:
            raise ValueError("workers must not be empty")
        if not all(isinstance(w, B200StageWorker) for w in workers):
            raise TypeError("MicroBatchPipeline drives B200 stage workers")
        self.workers = list(workers)
        self.stages = [w._model for w in self.workers]
        self.devices = [s.device for s in self.stages]
        if not self.stages[0].has_embedding or not self.stages[-1].has_lm_head:
            raise ValueError("the first stage must hold the embedding and the last the lm_head")

    def _hop(self, tensor: torch.Tensor, src: int, dst: int) -> torch.Tensor:
        a, b = self.devices[src], self.devices[dst]
        return tensor if a == b else Link.between(a, b).send(tensor)

    @torch.no_grad()
    def generate_greedy(
        self,
        prompts: Sequence[torch.Tensor],
        cache_keys: Sequence[str],
        max_new_tokens: int,
    ) -> list[torch.Tensor]:
        """Prefill every micro-batch's prompt [rows_m, S_m], then decode
        greedily until each has ``max_new_tokens`` tokens.  Returns one int64
        [rows_m, max_new_tokens] host tensor per micro-batch; the contexts stay
        cached under ``cache_keys`` (prompt + max_new_tokens - 1 positions).

        The tokens are the ones ``pipeline_prefill`` + ``pipeline_decode_step``
        with ``greedy_sample`` would produce for each context alone."""
        if len(prompts) != len(cache_keys) or not prompts:
            raise ValueError("need one cache key per prompt")
        if len(set(cache_keys)) != len(cache_keys):
            raise ValueError("cache keys must be distinct")
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be positive")
        cfg = self.stages[0].cfg
        for p in prompts:
            if p.ndim != 2 or p.shape[0] < 1 or p.shape[1] < 1:
                raise ValueError("each prompt must have shape [batch, sequence] and be non-empty")
            if p.shape[1] + max_new_tokens - 1 > cfg.max_position_embeddings:
                raise ValueError(
                    f"prompt ({p.shape[1]}) + max_new_tokens ({max_new_tokens}) exceeds model context "
                    f"{cfg.max_position_embeddings}"
                )
            lo, hi = int(p.min()), int(p.max())
            if lo < 0 or hi >= cfg.vocab_size:
                raise ValueError(f"input_ids contain a value outside [0, {cfg.vocab_size})")
        last = len(self.stages) - 1
        dev0 = self.devices[0]
        slots = []
        for key, p in zip(cache_keys, prompts):
            row = []
            for w in self.workers:
                w.clear_kv(key)
                w.reserve_kv(key, p.shape[0], p.shape[1] + max_new_tokens)
                row.append(w.slot_of(key))
            slots.append(row)
        try:
            ids = []
            for m, p in enumerate(prompts):  # prefill: micro-batches in flight across the stages
                h = p.to(dev0, non_blocking=True)
                for i, st in enumerate(self.stages):
                    if i == 0:
                        h = st.forward_slot(slots[m][0], None, input_ids=h, logits="last", check_values=False)
                    else:
                        h = st.forward_slot(slots[m][i], self._hop(h, i - 1, i), logits="last",
                                            check_values=False)
                ids.append(greedy_sample(h[:, -1]))
            out = [[t] for t in ids]
            for _ in range(max_new_tokens - 1):
                for m in range(len(prompts)):
                    x = self._hop(ids[m].view(-1, 1), last, 0)
                    for i, st in enumerate(self.stages):
                        if i > 0:
                            x = self._hop(x, i - 1, i)
                        inp = dict(input_ids=x) if i == 0 else {}
                        if i == last:
                            ids[m], _ = st.decode_greedy([slots[m][i]], None if i == 0 else x, **inp)
                        else:
                            x = st.decode_multi([slots[m][i]], None if i == 0 else x, **inp)
                    out[m].append(ids[m])
            result = [torch.stack(toks, dim=1).cpu() for toks in out]
            for st in self.stages:
                st.check_device()
            return result
        except BaseException:
            for key in cache_keys:
                for w in self.workers:
                    try:
                        w.clear_kv(key)
                    except Exception:
                        pass
            raise
