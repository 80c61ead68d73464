"""Continuous batcher scheduling on the host (no GPU): the reference's
ContinuousBatcher contract (inference/batcher.py) with one batched decode
pass per iteration, over fake stage workers whose "model" is a fixed map
from the last token to the next, and argmax sampling on the CPU."""
from __future__ import annotations

import asyncio
from types import SimpleNamespace

import pytest
import torch

import gpu_mesh_b200.batcher as B
from gpu_mesh_b200.sampling import SamplingParams

V = 50


def next_token(t: int) -> int:
    return (3 * t + 1) % V


class FakeWorker:
    """One stage with per-key caches; logits put all mass on next_token(x)."""

    def __init__(self, fail_key_prefix: str | None = None) -> None:
        self._model = SimpleNamespace(cfg=SimpleNamespace(vocab_size=V, max_position_embeddings=64))
        self.caches: dict[str | None, list[int]] = {}
        self.fail = fail_key_prefix
        self.multi_rows: list[int] = []

    def _logits(self, ids: list[list[int]]) -> torch.Tensor:
        out = torch.full((len(ids), len(ids[0]), V), -1.0)
        for b, row in enumerate(ids):
            for s, t in enumerate(row):
                out[b, s, next_token(t)] = 1.0
        return out

    def forward_inference(self, hidden, *, input_ids=None, position_ids=None, attention_mask=None,
                          operation_id, attempt_id, reset_kv=False, cache_key=None, logits="all"):
        if self.fail and cache_key and cache_key.startswith(self.fail):
            raise RuntimeError("stage failure")
        ids = input_ids.tolist()
        self.caches.setdefault(cache_key, []).extend(ids[0])
        return SimpleNamespace(output=self._logits(ids))

    def decode_multi(self, hidden, cache_keys, *, input_ids=None, logits="last"):
        if self.fail and any(k and k.startswith(self.fail) for k in cache_keys):
            raise RuntimeError("stage failure")
        ids = input_ids.tolist()
        for k, row in zip(cache_keys, ids):
            self.caches[k].extend(row)
        self.multi_rows.append(len(ids))
        return self._logits(ids)

    def kv_cache_length(self, cache_key=None) -> int:
        return len(self.caches.get(cache_key, []))

    def trim_kv(self, length, cache_key=None) -> None:
        self.caches[cache_key] = self.caches.get(cache_key, [])[:length]

    def clear_kv(self, cache_key=None) -> None:
        self.caches.pop(cache_key, None)


@pytest.fixture(autouse=True)
def cpu_sampling(monkeypatch):
    monkeypatch.setattr(B, "greedy_sample", lambda logits: logits.argmax(-1))


def expected(prompt: list[int], n: int, eos: int | None = None) -> list[int]:
    out, t = [], prompt[-1]
    for _ in range(n):
        t = next_token(t)
        out.append(t)
        if eos is not None and t == eos:
            break
    return out


async def _collect(batcher, seq_id):
    return [r async for r in batcher.stream(seq_id)]


def test_batched_decode_streams_the_reference_tokens():
    async def main():
        w = FakeWorker()
        b = B.ContinuousBatcher([w], max_batch_size=4)
        b.start()
        prompts = [[1, 2, 3], [7], [4, 5], [9, 9, 9, 9], [11]]
        ids = [await b.submit(p, SamplingParams(), 6) for p in prompts]
        results = await asyncio.gather(*[_collect(b, i) for i in ids])
        b.stop()
        await b.wait_stopped()
        return w, b, prompts, results

    w, b, prompts, results = asyncio.run(main())
    for p, res in zip(prompts, results):
        assert [r.token_id for r in res] == expected(p, 6)
        assert [r.seq_num for r in res] == list(range(1, 7))
        assert [r.is_last for r in res] == [False] * 5 + [True]
    assert max(w.multi_rows) == 4  # sequences share decode passes, up to the batch limit
    assert b.decode_passes < sum(5 for _ in prompts)  # fewer passes than per-sequence decode steps
    assert w.caches == {}  # every context released


def test_eos_and_validation_messages():
    async def main():
        w = FakeWorker()
        b = B.ContinuousBatcher([w], max_batch_size=2)
        with pytest.raises(RuntimeError, match="not running"):
            await b.submit([1], SamplingParams(), 3)
        b.start()
        with pytest.raises(ValueError, match="must not be empty"):
            await b.submit([], SamplingParams(), 3)
        with pytest.raises(ValueError, match="must be positive"):
            await b.submit([1], SamplingParams(), 0)
        with pytest.raises(ValueError, match="out-of-vocabulary"):
            await b.submit([V], SamplingParams(), 3)
        with pytest.raises(ValueError, match="exceeds model context"):
            await b.submit([1] * 60, SamplingParams(), 10)
        eos = expected([2], 3)[2]
        sid = await b.submit([2], SamplingParams(eos_token_id=eos), 10)
        res = await _collect(b, sid)
        b.stop()
        await b.wait_stopped()
        return res, eos

    res, eos = asyncio.run(main())
    assert [r.token_id for r in res] == expected([2], 10, eos=eos)
    assert res[-1].is_last and res[-1].token_id == eos


def test_a_failing_context_is_isolated():
    async def main():
        w = FakeWorker(fail_key_prefix="seq:")
        b = B.ContinuousBatcher([w], max_batch_size=4)
        b.start()
        sid = await b.submit([1, 2], SamplingParams(), 4)
        res = await _collect(b, sid)
        b.stop()
        await b.wait_stopped()
        return res

    res = asyncio.run(main())
    assert res == [B.SessionResult(token_id=-1, seq_num=0, is_last=True)]


def test_cancelled_stream_releases_its_context():
    async def main():
        w = FakeWorker()
        b = B.ContinuousBatcher([w], max_batch_size=2)
        b.start()
        sid = await b.submit([3], SamplingParams(), 20)
        agen = b.stream(sid)
        first = await agen.__anext__()
        await agen.aclose()
        for _ in range(50):
            await asyncio.sleep(0.01)
            if b.active_count == 0:
                break
        b.stop()
        await b.wait_stopped()
        return w, first, b

    w, first, b = asyncio.run(main())
    assert first.token_id == next_token(3)
    assert b.active_count == 0 and w.caches == {}


def test_a_failing_request_does_not_end_the_others():
    import threading

    class Flaky(FakeWorker):
        def __init__(self):
            super().__init__()
            self.bad = None
            self.armed = threading.Event()

        def decode_multi(self, hidden, cache_keys, **kw):
            self.armed.wait(5)  # the test names the failing context before any decode
            if self.bad in cache_keys:
                raise RuntimeError("stage failure")
            return super().decode_multi(hidden, cache_keys, **kw)

        def forward_inference(self, hidden, **kw):
            if self.bad is not None and kw.get("cache_key") == self.bad:
                raise RuntimeError("stage failure")
            return super().forward_inference(hidden, **kw)

    async def main():
        w = Flaky()
        b = B.ContinuousBatcher([w], max_batch_size=4)
        b.start()
        bad = await b.submit([1], SamplingParams(), 6)
        good = await b.submit([2], SamplingParams(), 6)
        w.bad = f"seq:{bad}"
        w.armed.set()
        res_bad, res_good = await asyncio.gather(_collect(b, bad), _collect(b, good))
        b.stop()
        await b.wait_stopped()
        return w, res_bad, res_good

    w, res_bad, res_good = asyncio.run(main())
    assert [r.token_id for r in res_good] == expected([2], 6)
    assert res_bad[-1].token_id == -1 and res_bad[-1].is_last  # at its prefill or its first decode
    assert w.caches == {}


def test_stop_ends_running_requests_and_releases_them():
    async def main():
        w = FakeWorker()
        b = B.ContinuousBatcher([w], max_batch_size=2)
        b.start()
        sid = await b.submit([5], SamplingParams(), 60)
        agen = b.stream(sid)
        first = await agen.__anext__()
        b.stop()
        rest = [r async for r in agen]
        await b.wait_stopped()
        with pytest.raises(RuntimeError, match="not running"):
            await b.submit([1], SamplingParams(), 1)
        return w, first, rest

    w, first, rest = asyncio.run(main())
    assert first.seq_num == 1
    assert rest[-1].token_id == -1 and rest[-1].is_last
    assert w.caches == {}
