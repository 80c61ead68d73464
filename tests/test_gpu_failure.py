"""Failure detection on the device, tested without a fault.

Every wait inside the stage's kernels is bounded: on expiry the kernel
records code 3 in the stage's error word, lets what it issued finish, and
returns; ``check_device`` then raises and resets the stage's counters.  Here
a wait is made to run out the allowed way: ``probe_wait`` waits, with the
kernels' own bounded wait, for a flag that nothing sets, under a limit of a
few milliseconds.  The test checks that the timeout is reported once, that a
wait whose flag is set reports nothing, and that the stage's next forwards
are correct against the CPU oracle.  (The reference tests failures on the
host only: tests/unit/test_inference.py:196-233; host-side failures are
covered in test_host_logic.py and test_dist_pipeline.py.)
"""
from __future__ import annotations

import time

import pytest
import torch

from gpu_mesh_b200 import B200Stage
from gpu_mesh_b200._lib import DeviceTimeoutError
from gpu_mesh_b200.config import LlamaConfig
from gpu_mesh_b200.weights import synthetic_model_state
from oracle import stage_ref as R

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_bounded_wait_expiry_is_reported_and_the_stage_recovers():
    cfg = LlamaConfig(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=64, max_position_embeddings=256)
    full = synthetic_model_state(cfg, seed=31, dtype=torch.bfloat16)
    stage = B200Stage(cfg, 0, 2, has_embedding=True, has_lm_head=True, device=DEV, dtype=torch.bfloat16,
                      state_dict=full)
    oracle = R.OracleStage(cfg, 0, 2, True, True, full, torch.bfloat16)
    g = torch.Generator().manual_seed(8)
    try:
        stage.kv_reserve(1, 2, 64)
        ids = torch.randint(0, cfg.vocab_size, (2, 24), generator=g)
        got = stage.forward_slot(1, None, input_ids=ids).float().cpu()
        ref = oracle.forward(input_ids=ids, key="c").float()
        assert (got - ref).abs().max() <= 2e-2
        stage.check_device()

        stage.probe_wait(2000, flag_set=True)   # the flag is set: the wait ends at once
        stage.check_device()

        torch.cuda.synchronize(DEV)
        t0 = time.perf_counter()
        stage.probe_wait(3000)                   # nothing sets the flag: runs out after 3 ms
        torch.cuda.synchronize(DEV)
        assert time.perf_counter() - t0 >= 2.5e-3
        with pytest.raises(DeviceTimeoutError, match="bounded wait"):
            stage.check_device()
        stage.check_device()                     # reported once, then cleared

        for _ in range(2):                       # the stage still decodes correctly
            nxt = torch.randint(0, cfg.vocab_size, (2, 1), generator=g)
            got = stage.forward_slot(1, None, input_ids=nxt).float().cpu()
            ref = oracle.forward(input_ids=nxt, key="c").float()
            assert (got - ref).abs().max() <= 2e-2
        stage.check_device()
        with pytest.raises(ValueError, match="limit_us"):
            stage.probe_wait(0)
    finally:
        stage.close()
