"""The drop-in acceptance check: the reference's own unit tests pass when its
``build_pipeline`` returns B200 workers.

Runs the reference checkout's tests/unit/test_model.py and
tests/unit/test_inference.py in a child pytest with
``tests/acceptance/b200_acceptance_plugin.py`` loaded (see there for what it
swaps in and which training tests it skips).  The reference is looked up in
``$MESHGPU_REFERENCE_CHECKOUT``, else in ``baseline/_ref`` at the repository
root (a plain copy of the checkout's ``src/`` and those two test files); the
test is skipped where neither holds it.  Tolerances are the reference's own
(fp32, atol 1e-4 / rtol 1e-3 against its monolithic CPU stage).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu

SUITES = ["tests/unit/test_model.py", "tests/unit/test_inference.py"]


def _checkout() -> Path:
    return Path(os.environ.get("MESHGPU_REFERENCE_CHECKOUT") or ROOT / "baseline" / "_ref")


@pytest.mark.parametrize("suite", SUITES)
def test_reference_suite_passes_with_b200_workers(suite):
    checkout = _checkout()
    if not (checkout / "src" / "meshgpu").is_dir() or not (checkout / suite).is_file():
        pytest.skip(f"reference checkout with {suite} not available here")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(checkout / "src"), str(ROOT), str(ROOT / "tests" / "acceptance")])
    cmd = [sys.executable, "-m", "pytest", "-q", "-rs", "--import-mode=importlib", "-p", "no:cacheprovider",
           "-p", "b200_acceptance_plugin", str(checkout / suite)]
    res = subprocess.run(cmd, cwd=checkout, env=env, capture_output=True, text=True, timeout=1200)
    print(res.stdout[-4000:])
    assert res.returncode == 0, res.stdout[-6000:] + res.stderr[-3000:]
