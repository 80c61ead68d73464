"""ctypes binding of ``libmeshgpu_b200.so`` (the C ABI in ``include/meshgpu_b200.h``).

The library is loaded from ``gpu_mesh_b200/lib``.  There is no fallback: if
the library is missing, :func:`lib` raises, so a stage can never silently run
on another implementation.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

# MESHGPU_LIB names a build of the library made elsewhere (for example with other
# compile-time tuning macros); by default the in-tree build is loaded.
LIB_PATH = Path(os.environ.get("MESHGPU_LIB") or Path(__file__).resolve().parent / "lib" / "libmeshgpu_b200.so")

MG_OK = 0
MG_EINVAL = 1
MG_ESTATE = 2
MG_ECUDA = 3
MG_ENOMEM = 4
MG_EDEVICE = 5
MG_ETIMEOUT = 6

MG_DTYPE_F32 = 0
MG_DTYPE_BF16 = 1

MG_OUT_HIDDEN = 0
MG_OUT_LOGITS_ALL = 1
MG_OUT_LOGITS_LAST = 2

(MG_W_EMBED, MG_W_NORM, MG_W_LM_HEAD, MG_W_INPUT_NORM, MG_W_QKV, MG_W_Q_NORM, MG_W_K_NORM, MG_W_O,
 MG_W_POST_NORM, MG_W_GATE_UP, MG_W_DOWN) = range(11)

MG_ATTN_SDPA = 0
MG_ATTN_EAGER = 1
MG_ATTN_CACHE_CAUSAL = 2

# Every function the header declares, with its ctypes signature.
_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_u64p = ctypes.POINTER(ctypes.c_uint64)
_i32p = ctypes.POINTER(ctypes.c_int32)


class StageConfig(ctypes.Structure):
    _fields_ = [
        ("vocab_size", _i32),
        ("hidden_size", _i32),
        ("intermediate_size", _i32),
        ("num_hidden_layers", _i32),
        ("num_attention_heads", _i32),
        ("num_key_value_heads", _i32),
        ("head_dim", _i32),
        ("max_position_embeddings", _i32),
        ("rms_norm_eps", _f32),
        ("qk_norm", _i32),
        ("attention_impl", _i32),
        ("dtype", _i32),
        ("layer_start", _i32),
        ("layer_end", _i32),
        ("has_embedding", _i32),
        ("has_lm_head", _i32),
        ("device", _i32),
    ]


class LayerWeights(ctypes.Structure):
    _fields_ = [
        ("input_layernorm", _vp),
        ("q_proj", _vp),
        ("k_proj", _vp),
        ("v_proj", _vp),
        ("q_norm", _vp),
        ("k_norm", _vp),
        ("o_proj", _vp),
        ("post_attention_layernorm", _vp),
        ("gate_proj", _vp),
        ("up_proj", _vp),
        ("down_proj", _vp),
    ]


class StageWeights(ctypes.Structure):
    _fields_ = [
        ("embed_tokens", _vp),
        ("norm", _vp),
        ("lm_head", _vp),
        ("rope_cos", _vp),
        ("rope_sin", _vp),
        ("layers", ctypes.POINTER(LayerWeights)),
    ]


MG_PROF_CLASSES = 4
PROF_NAMES = ("linear_decode", "linear_prefill", "attention", "other")


class Profile(ctypes.Structure):
    _fields_ = [
        ("ms", ctypes.c_double * MG_PROF_CLASSES),
        ("bytes", ctypes.c_double * MG_PROF_CLASSES),
        ("flops", ctypes.c_double * MG_PROF_CLASSES),
        ("launches", ctypes.c_uint64 * MG_PROF_CLASSES),
    ]

    def as_dict(self) -> dict[str, dict[str, float]]:
        return {
            name: {"ms": self.ms[i], "bytes": self.bytes[i], "flops": self.flops[i],
                   "launches": int(self.launches[i])}
            for i, name in enumerate(PROF_NAMES)
        }


SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "mg_version": (ctypes.c_char_p, []),
    "mg_last_error": (ctypes.c_char_p, []),
    "mg_stage_create": (
        ctypes.c_int,
        [ctypes.POINTER(StageConfig), ctypes.POINTER(StageWeights), ctypes.POINTER(_vp)],
    ),
    "mg_stage_destroy": (ctypes.c_int, [_vp]),
    "mg_stage_memory": (ctypes.c_int, [_vp, _u64p, _u64p, _u64p]),
    "mg_kv_alloc": (ctypes.c_int, [_vp, _i32, _i32, _i32]),
    "mg_kv_free": (ctypes.c_int, [_vp, _i32]),
    "mg_kv_free_all": (ctypes.c_int, [_vp]),
    "mg_kv_length": (ctypes.c_int, [_vp, _i32, _i32p]),
    "mg_kv_batch": (ctypes.c_int, [_vp, _i32, _i32p]),
    "mg_kv_trim": (ctypes.c_int, [_vp, _i32, _i32]),
    "mg_kv_import": (ctypes.c_int, [_vp, _i32, _i32, _vp, _vp, _i32, _vp]),
    "mg_kv_export": (ctypes.c_int, [_vp, _i32, _i32, _vp, _vp, _vp]),
    "mg_stage_forward": (ctypes.c_int, [_vp, _i32, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp]),
    "mg_stage_decode_multi": (ctypes.c_int, [_vp, _i32p, _i32, _vp, _vp, _i32, _vp, _vp]),
    "mg_stage_decode_greedy": (ctypes.c_int, [_vp, _i32p, _i32, _vp, _vp, _vp, _vp, _vp]),
    "mg_stage_check_device": (ctypes.c_int, [_vp, _vp]),
    "mg_stage_profile": (ctypes.c_int, [_vp, _i32]),
    "mg_stage_profile_read": (ctypes.c_int, [_vp, ctypes.POINTER(Profile)]),
    "mg_launch_count": (ctypes.c_uint64, []),
    "mg_sample_greedy": (ctypes.c_int, [_vp, _i32, _i32, _i32, _i64, _vp, _vp]),
    "mg_sample_top_p": (ctypes.c_int, [_vp, _i32, _i32, _i32, _i64, _f32, _f32, _vp, _vp, _vp]),
}

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None


class MeshGpuError(RuntimeError):
    """A CUDA or allocation failure reported by the stage library."""


class DeviceRangeError(ValueError):
    """A kernel met an out-of-range token id or position (reported lazily)."""


class DeviceTimeoutError(MeshGpuError):
    """A kernel gave up a bounded wait; the outputs since the last check are invalid."""


def lib() -> ctypes.CDLL:
    """Load the stage library once; raise if it has not been built."""
    global _LIB
    with _LOCK:
        if _LIB is None:
            if not LIB_PATH.exists():
                raise MeshGpuError(
                    f"{LIB_PATH} is missing: build it with `python -m gpu_mesh_b200.build`"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _LIB = handle
        return _LIB


def last_error() -> str:
    msg = lib().mg_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    """Map a status code to the reference's exception types."""
    if status == MG_OK:
        return
    msg = last_error()
    if status == MG_EINVAL:
        raise ValueError(msg)
    if status == MG_ESTATE:
        raise RuntimeError(msg)
    if status == MG_EDEVICE:
        raise DeviceRangeError(msg)
    if status == MG_ETIMEOUT:
        raise DeviceTimeoutError(msg)
    raise MeshGpuError(msg)


SIGNATURES["mg_linear"] = (
    ctypes.c_int,
    [_i32, _vp, _i64, _vp, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, ctypes.c_uint64, _vp],
)
SIGNATURES["mg_linear_scratch"] = (ctypes.c_uint64, [_i32, _i32, _i32, _i32, _i32])
SIGNATURES["mg_linear_check_device"] = (ctypes.c_int, [_vp])
SIGNATURES["mg_stage_decode_top_p"] = (
    ctypes.c_int, [_vp, _i32p, _i32, _vp, _vp, ctypes.c_float, ctypes.c_float, _vp, _vp, _vp, _vp])
SIGNATURES["mg_stage_probe_wait"] = (ctypes.c_int, [_vp, ctypes.c_uint32, _i32, _vp])
SIGNATURES["mg_stage_weight"] = (ctypes.c_int, [_vp, _i32, _i32, ctypes.POINTER(ctypes.c_void_p)])
SIGNATURES["mg_reserve_sms"] = (ctypes.c_int, [_i32, _i32])
SIGNATURES["mg_peer_access"] = (ctypes.c_int, [_i32, _i32, ctypes.POINTER(ctypes.c_int32)])
SIGNATURES["mg_peer_copy"] = (ctypes.c_int, [_vp, _i32, _vp, _i32, ctypes.c_uint64, _vp])
SIGNATURES["mg_linear_noalloc"] = (
    ctypes.c_int,
    [_i32, _vp, _i64, _vp, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp],
)
