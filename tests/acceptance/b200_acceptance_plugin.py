"""pytest plugin: the reference's own unit tests, with B200 stage workers.

Loaded into a pytest run over the reference checkout's tests/unit/test_model.py
and tests/unit/test_inference.py (``tests/test_gpu_reference_suites.py``
starts that run).  It replaces the reference's
``meshgpu.backends.portable.pipeline.build_pipeline`` before the test modules
import it: the replacement builds the reference's workers exactly as the
original would (same seeding, same init), then converts them with
``gpu_mesh_b200.from_reference_workers`` into B200 workers holding the same
weights on cuda:0 with the reference's default "cpu" transport, so every test
sees CPU tensors as before.  Everything else (the reference's coordinator,
sessions, sampling, its monolithic CPU stages used as the expected values) is
the reference's own code.

Tests of the training step (pipeline_train_step, gradient scaling) are
skipped: the B200 stage executor serves inference only.  The reference runs
its coroutine tests with pytest-asyncio, which this image lacks; the
``pytest_pyfunc_call`` hook below runs them on a fresh event loop instead.
"""
from __future__ import annotations

import asyncio
import inspect

import pytest
import torch

TRAINING_TESTS = ("test_training_", "test_pipeline_gradient_scaler_")


def pytest_configure(config):
    config.addinivalue_line("markers", "asyncio: coroutine test, run on a fresh event loop")
    from meshgpu.backends.portable import pipeline as ref_pipeline

    from gpu_mesh_b200.pipeline import from_reference_workers

    reference_build = ref_pipeline.build_pipeline

    def build_pipeline_b200(cfg, num_stages, devices, *args, **kwargs):
        workers = reference_build(cfg, num_stages, devices, *args, **kwargs)
        dtype = next(workers[0]._model.parameters()).dtype
        return from_reference_workers(workers, [torch.device("cuda", 0)] * num_stages, dtype=dtype,
                                      transport="cpu")

    ref_pipeline.build_pipeline = build_pipeline_b200


def pytest_collection_modifyitems(config, items):
    skip = pytest.mark.skip(reason="training step: the B200 stage executor serves inference only")
    for item in items:
        if item.name.startswith(TRAINING_TESTS):
            item.add_marker(skip)


@pytest.hookimpl(tryfirst=True)
def pytest_pyfunc_call(pyfuncitem):
    if inspect.iscoroutinefunction(pyfuncitem.obj):
        args = {name: pyfuncitem.funcargs[name] for name in pyfuncitem._fixtureinfo.argnames}
        asyncio.run(pyfuncitem.obj(**args))
        return True
    return None
