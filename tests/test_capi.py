"""The C-ABI library loads and exports every entry point the header declares.

No compute runs here: only calls that fail validation before touching a GPU.
"""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from gpu_mesh_b200 import _lib
from tests.conftest import ROOT

HEADER = ROOT / "include" / "meshgpu_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(mg_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in (
        "mg_stage_create", "mg_stage_destroy", "mg_stage_forward", "mg_stage_decode_multi",
        "mg_kv_alloc", "mg_kv_free", "mg_kv_length", "mg_kv_trim", "mg_kv_import", "mg_kv_export",
        "mg_sample_greedy", "mg_sample_top_p", "mg_last_error",
    ):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True)
    exported = set(re.findall(r"\bT (mg_[a-z_0-9]+)", out.stdout))
    for name in declared_functions():
        assert name in exported, name
        assert hasattr(lib, name)
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_calls_without_gpu():
    lib = _lib.lib()
    assert b"sm_100a" in lib.mg_version()
    rc = lib.mg_stage_create(None, None, None)
    assert rc == _lib.MG_EINVAL
    assert "null" in _lib.last_error()
    with pytest.raises(ValueError, match="null"):
        _lib.check(lib.mg_kv_trim(None, 0, 0))
    n = ctypes.c_int32(7)
    assert lib.mg_kv_length(None, 0, ctypes.byref(n)) == _lib.MG_EINVAL


def test_invalid_config_is_rejected_before_any_allocation():
    lib = _lib.lib()
    cfg = _lib.StageConfig(
        vocab_size=64, hidden_size=16, intermediate_size=32, num_hidden_layers=2,
        num_attention_heads=3, num_key_value_heads=2, head_dim=8, max_position_embeddings=32,
        rms_norm_eps=1e-5, dtype=_lib.MG_DTYPE_F32, layer_start=0, layer_end=2,
    )
    w = _lib.StageWeights()
    h = ctypes.c_void_p()
    assert lib.mg_stage_create(ctypes.byref(cfg), ctypes.byref(w), ctypes.byref(h)) == _lib.MG_EINVAL
    assert "divisible" in _lib.last_error()
    cfg.num_attention_heads = 4
    cfg.layer_end = 3
    assert lib.mg_stage_create(ctypes.byref(cfg), ctypes.byref(w), ctypes.byref(h)) == _lib.MG_EINVAL
    assert "invalid layer range" in _lib.last_error()
    cfg.layer_end = 2
    cfg.head_dim = 24
    assert lib.mg_stage_create(ctypes.byref(cfg), ctypes.byref(w), ctypes.byref(h)) == _lib.MG_EINVAL
    assert "head_dim" in _lib.last_error()


def test_sampling_argument_checks_without_gpu():
    lib = _lib.lib()
    assert lib.mg_sample_top_p(1, 0, 1, 4, 4, -1.0, 0.5, None, 1, None) == _lib.MG_EINVAL
    assert "temperature" in _lib.last_error()
    assert lib.mg_sample_top_p(1, 0, 1, 4, 4, 1.0, 1.5, None, 1, None) == _lib.MG_EINVAL
    assert "top_p" in _lib.last_error()
    assert lib.mg_sample_top_p(1, 0, 1, 4, 4, 1.0, 0.5, None, 1, None) == _lib.MG_EINVAL
    assert "uniforms" in _lib.last_error()
