"""B200 stages loaded from a MeshGPU model artifact (manifest.json + shards).

The artifact format is the reference's: ``manifest.json`` as written by
``ModelManifest.save`` (artifacts/manifest.py:14-260) from the importers
(artifacts/hf_import.py:294-535, artifacts/qwen_import.py:169-320), a
``config.json`` beside it, and one ``torch.save``'d state dict per shard with
stage-local key names.  :class:`ModelManifest` here parses that file with the
same validation rules; a reference ``ModelManifest`` object is accepted too.

:func:`build_pipeline_from_manifest` and :func:`build_stage_from_manifest`
keep the reference loaders' contract (hf_import.py:638-858, with the Qwen3
dispatch of qwen_import.py:393-616): the same order of checks and error
messages, a size and sha256 check of every shard before it is deserialised,
strict key matching, and planner ranges recombined from the overlapping
shards (hf_import.py:860-1050).  What differs is where the weights go.  The
reference builds a CPU module, loads the shard into it, then moves the module
to the GPU.  Here a shard is memory-mapped (``torch.load(mmap=True)``), and
each tensor is copied once from the page cache into the stage's own HBM
layout; the shards of a pipeline are hashed concurrently.
"""
from __future__ import annotations

import hashlib
import json
import logging
import os
from collections.abc import Sequence
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path
from types import SimpleNamespace
from typing import Any

import torch

from gpu_mesh_b200.config import LlamaConfig, config_from
from gpu_mesh_b200.stage import B200Stage
from gpu_mesh_b200.stage_worker import B200StageWorker, StageContext
from gpu_mesh_b200.weights import stage_keys

log = logging.getLogger(__name__)

_HASH_CHUNK = 16 << 20
_HEX = set("0123456789abcdefABCDEF")
_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
# Fields of the reference LlamaConfig (models/llama_dense.py:20-32): the
# manifest's config_hash is taken over exactly these.
_LLAMA_FIELDS = (
    "vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
    "num_key_value_heads", "head_dim", "max_position_embeddings", "rms_norm_eps", "rope_theta",
    "tie_word_embeddings", "attention_implementation",
)
LLAMA_ADAPTER = ("llama_dense", "llama_dense_v1")
QWEN3_ADAPTER = ("qwen3", "qwen3_hf_v1")


def _strict_int(value: Any, what: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError(f"{what} must be integers")
    return value


def _contained(value: str, what: str) -> str:
    path = Path(value)
    if not value or path == Path(".") or path.is_absolute() or ".." in path.parts:
        raise ValueError(f"{what} must be relative and contained in the artifact")
    return value


@dataclass(frozen=True)
class ShardEntry:
    """One stage shard (artifacts/manifest.py:14-73)."""

    shard_id: str
    path: str
    byte_length: int
    sha256: str
    layer_start: int
    layer_end: int
    tensor_names: tuple[str, ...]

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> ShardEntry:
        sid = d["shard_id"]
        if not isinstance(sid, str) or not sid or Path(sid).name != sid or sid in {".", ".."}:
            raise ValueError("shard_id must be a non-empty path component")
        path = _contained(d["path"], "shard path")
        n = _strict_int(d["byte_length"], "shard sizes and layer bounds")
        ls = _strict_int(d["layer_start"], "shard sizes and layer bounds")
        le = _strict_int(d["layer_end"], "shard sizes and layer bounds")
        if n < 0:
            raise ValueError("shard byte_length must be non-negative")
        names = d["tensor_names"]
        if not names or any(not isinstance(x, str) or not x for x in names):
            raise ValueError("shard tensor_names must contain non-empty strings")
        if len(set(names)) != len(names):
            raise ValueError("shard tensor_names must be unique")
        if ls < 0:
            raise ValueError("shard layer_start must be non-negative")
        if le <= ls:
            raise ValueError("shard layer_end must be greater than layer_start")
        sha = d.get("sha256", "")
        if sha and (len(sha) != 64 or any(c not in _HEX for c in sha)):
            raise ValueError("shard sha256 must be a 64-character hexadecimal digest")
        return cls(sid, path, n, sha, ls, le, tuple(names))


@dataclass(frozen=True)
class ManifestMeta:
    """Model identity and geometry (artifacts/manifest.py:76-146)."""

    model_family: str
    model_id: str
    adapter: str
    num_layers: int
    hidden_size: int
    num_attention_heads: int
    num_kv_heads: int
    head_dim: int
    vocab_size: int
    max_position_embeddings: int
    compute_dtype: str
    weight_format: str
    tied_embeddings: bool = False
    extra: dict[str, Any] = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> ManifestMeta:
        for k in ("model_family", "model_id", "adapter"):
            if not isinstance(d.get(k), str) or not d[k].strip():
                raise ValueError("manifest model identity fields must be non-empty strings")
        dims = {}
        for k in ("num_layers", "hidden_size", "num_attention_heads", "num_kv_heads", "head_dim",
                  "vocab_size", "max_position_embeddings"):
            v = _strict_int(d[k], "manifest dimensions")
            if v < 1:
                raise ValueError("manifest dimensions must be positive")
            dims[k] = v
        if d["compute_dtype"] not in _DTYPES:
            raise ValueError(f"unsupported manifest compute_dtype: {d['compute_dtype']!r}")
        if d["weight_format"] not in {"safetensors", "pytorch", "pt"}:
            raise ValueError(f"unsupported manifest weight_format: {d['weight_format']!r}")
        if dims["num_attention_heads"] % dims["num_kv_heads"]:
            raise ValueError("manifest num_attention_heads must be divisible by num_kv_heads")
        if dims["head_dim"] % 2:
            raise ValueError("manifest head_dim must be even for rotary embeddings")
        return cls(
            model_family=d["model_family"], model_id=d["model_id"], adapter=d["adapter"], **dims,
            compute_dtype=d["compute_dtype"], weight_format=d["weight_format"],
            tied_embeddings=bool(d.get("tied_embeddings", False)), extra=dict(d.get("extra") or {}),
        )


@dataclass(frozen=True)
class ModelManifest:
    """A sharded model artifact (artifacts/manifest.py:149-260)."""

    manifest_id: str
    meta: ManifestMeta
    shards: tuple[ShardEntry, ...]
    schema_version: int = 1
    tokenizer_path: str | None = None
    config_path: str | None = None
    config_hash: str = ""

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> ModelManifest:
        version = d.get("schema_version", 1)
        if isinstance(version, bool) or not isinstance(version, int) or version < 1:
            raise ValueError("schema_version must be a positive integer")
        mid = d["manifest_id"]
        if not isinstance(mid, str) or not mid or mid in {".", ".."} or Path(mid).name != mid:
            raise ValueError("manifest_id must be a single relative path component")
        chash = d.get("config_hash", "") or ""
        if chash and (len(chash) % 2 or any(c not in _HEX for c in chash)):
            raise ValueError("config_hash must be hexadecimal")
        shards = tuple(ShardEntry.from_dict(s) for s in d["shards"])
        if not shards:
            raise ValueError("manifest must have at least one shard")
        if len({s.shard_id for s in shards}) != len(shards):
            raise ValueError("manifest shard IDs must be unique")
        if len({s.path for s in shards}) != len(shards):
            raise ValueError("manifest shard paths must be unique")
        opt = {}
        for k in ("tokenizer_path", "config_path"):
            v = d.get(k)
            if v is not None:
                if not v:
                    raise ValueError("artifact paths must not be empty")
                _contained(v, "artifact paths")
            opt[k] = v
        meta = ManifestMeta.from_dict(d["meta"])
        end = 0
        for s in sorted(shards, key=lambda s: s.layer_start):
            if s.layer_start != end:
                raise ValueError("manifest shards must cover contiguous layer ranges from zero")
            end = s.layer_end
        if end != meta.num_layers:
            raise ValueError(f"manifest shards cover {end} layers, expected {meta.num_layers}")
        return cls(mid, meta, shards, version, opt["tokenizer_path"], opt["config_path"], chash)

    @classmethod
    def load(cls, path: str | Path) -> ModelManifest:
        return cls.from_dict(json.loads(Path(path).read_text()))

    def shards_for_layers(self, layer_start: int, layer_end: int) -> list[ShardEntry]:
        """Shards overlapping [layer_start, layer_end) (manifest.py:212-217)."""
        return [s for s in self.shards if s.layer_end > layer_start and s.layer_start < layer_end]


def compute_config_hash(config: dict[str, Any]) -> str:
    """First 16 hex digits of sha256 over the sorted-key JSON (manifest.py:257-260)."""
    return hashlib.sha256(json.dumps(config, sort_keys=True).encode()).hexdigest()[:16]


def as_manifest(obj: Any) -> ModelManifest:
    """This module's manifest from itself or from a reference ``ModelManifest``."""
    if isinstance(obj, ModelManifest):
        return obj
    if hasattr(obj, "model_dump"):
        return ModelManifest.from_dict(obj.model_dump())
    raise TypeError(f"expected a ModelManifest, got {type(obj).__name__}")


def _open(manifest_or_dir: Any, artifact_root: str | Path | None) -> tuple[ModelManifest, Path]:
    if isinstance(manifest_or_dir, (str, Path)):
        root = Path(manifest_or_dir)
        return ModelManifest.load(root / "manifest.json"), root
    return as_manifest(manifest_or_dir), Path(artifact_root) if artifact_root is not None else Path(".")


def resolve_artifact_path(root: Path, relative_path: str) -> Path:
    """A manifest path inside the artifact root (hf_import.py:1164-1175)."""
    candidate = Path(relative_path)
    if candidate.is_absolute() or ".." in candidate.parts:
        raise ValueError(f"manifest path must be relative and contained: {relative_path!r}")
    base = root.resolve()
    resolved = (base / candidate).resolve()
    try:
        resolved.relative_to(base)
    except ValueError as exc:
        raise ValueError(f"manifest path escapes artifact root: {relative_path!r}") from exc
    return resolved


# ---------------------------------------------------------------------------
# Configs
# ---------------------------------------------------------------------------

def _qwen_config(values: dict[str, Any]) -> LlamaConfig:
    try:
        from transformers import Qwen3Config
    except ImportError:  # the geometry fields are all this stage needs
        return config_from(SimpleNamespace(**{"model_type": "qwen3", "rms_norm_eps": 1e-6, **values}))
    return config_from(Qwen3Config(**{k: v for k, v in values.items() if k != "model_type"}))


def load_stage_config(manifest_or_dir: Any, *, artifact_root: str | Path | None = None) -> LlamaConfig:
    """The execution config of an artifact, checked against its manifest.

    Llama artifacts: ``config.json`` holds the reference LlamaConfig fields, or,
    without it, ``meta.extra`` supplies them (hf_import.py:537-568).  Qwen3
    artifacts: ``config.json`` is the HF Qwen3Config dict (qwen_import.py:322-349).
    The config hash, when the manifest carries one, must match
    (hf_import.py:1070-1076).
    """
    manifest, root = _open(manifest_or_dir, artifact_root)
    meta = manifest.meta
    config_path = resolve_artifact_path(root, manifest.config_path or "config.json")
    if meta.adapter == QWEN3_ADAPTER[1]:  # dispatched on the adapter (hf_import.py:661-672)
        if meta.model_family != QWEN3_ADAPTER[0]:
            raise ValueError("manifest is not a qwen3_hf_v1 artifact")
        if not config_path.exists():
            raise FileNotFoundError(f"Qwen3 config not found: {config_path}")
        values = json.loads(config_path.read_text())
        if not isinstance(values, dict):
            raise ValueError("Qwen3 config file must contain an object")
        actual = compute_config_hash(values)
        if manifest.config_hash and actual != manifest.config_hash:
            raise ValueError(f"Qwen3 config hash mismatch: expected {manifest.config_hash}, got {actual}")
        cfg = _qwen_config(values)
        _check_geometry(manifest, cfg)
        return cfg
    if config_path.exists():
        values = json.loads(config_path.read_text())
        cfg = LlamaConfig(**values)
    else:
        extra = meta.extra
        cfg = LlamaConfig(
            vocab_size=meta.vocab_size,
            hidden_size=meta.hidden_size,
            intermediate_size=extra.get("intermediate_size", meta.hidden_size * 4),
            num_hidden_layers=meta.num_layers,
            num_attention_heads=meta.num_attention_heads,
            num_key_value_heads=meta.num_kv_heads,
            head_dim=meta.head_dim,
            max_position_embeddings=meta.max_position_embeddings,
            rms_norm_eps=extra.get("rms_norm_eps", 1e-5),
            rope_theta=extra.get("rope_theta", 10000.0),
            tie_word_embeddings=meta.tied_embeddings,
            attention_implementation=extra.get("attn_implementation", "sdpa"),
        )
    if manifest.config_hash:
        actual = compute_config_hash({k: getattr(cfg, k) for k in _LLAMA_FIELDS})
        if actual != manifest.config_hash:
            raise ValueError(
                "artifact config hash mismatch: the referenced config does not match "
                f"manifest (expected {manifest.config_hash}, got {actual})"
            )
    validate_manifest_config(manifest, cfg)
    return cfg


def _check_geometry(manifest: ModelManifest, cfg: LlamaConfig) -> None:
    meta = manifest.meta
    expected = {
        "num_layers": cfg.num_hidden_layers,
        "hidden_size": cfg.hidden_size,
        "num_attention_heads": cfg.num_attention_heads,
        "num_kv_heads": cfg.num_key_value_heads,
        "head_dim": cfg.head_dim,
        "vocab_size": cfg.vocab_size,
        "max_position_embeddings": cfg.max_position_embeddings,
    }
    bad = [f"{k}: manifest={getattr(meta, k)!r}, config={v!r}" for k, v in expected.items()
           if getattr(meta, k) != v]
    if meta.tied_embeddings != cfg.tie_word_embeddings:
        bad.append(f"tied_embeddings: manifest={meta.tied_embeddings!r}, config={cfg.tie_word_embeddings!r}")
    if bad:
        raise ValueError("manifest/config mismatch: " + "; ".join(bad))


def validate_manifest_config(manifest: ModelManifest, cfg: LlamaConfig) -> None:
    """Manifest metadata and execution config describe one Llama model
    (hf_import.py:592-631)."""
    _check_geometry(manifest, cfg)
    meta = manifest.meta
    if (meta.model_family, meta.adapter) != LLAMA_ADAPTER:
        raise ValueError(f"unsupported manifest adapter: family={meta.model_family!r}, adapter={meta.adapter!r}")
    if meta.weight_format not in {"pt", "pytorch"}:
        raise ValueError(f"unsupported manifest weight format: {meta.weight_format!r}")
    attn = meta.extra.get("attn_implementation")
    if attn is not None and attn != cfg.attention_implementation:
        raise ValueError(
            "manifest/config mismatch: "
            f"attn_implementation: manifest={attn!r}, config={cfg.attention_implementation!r}"
        )


def validate_manifest_layout(manifest: ModelManifest) -> list[ShardEntry]:
    """Shards sorted by layer, contiguous from zero to num_layers (hf_import.py:571-589)."""
    ordered = sorted(manifest.shards, key=lambda s: s.layer_start)
    end = 0
    for i, s in enumerate(ordered):
        if s.layer_start != end:
            raise ValueError(f"manifest stage {i} starts at layer {s.layer_start}; expected {end}")
        end = s.layer_end
    if end != manifest.meta.num_layers:
        raise ValueError(
            f"manifest covers layers [0, {end}), but config declares {manifest.meta.num_layers} layers"
        )
    return ordered


def validate_requested_ranges(layer_ranges: Sequence[tuple[int, int]], num_layers: int) -> list[tuple[int, int]]:
    """A planner partition: non-empty, contiguous from zero, covering every
    layer (hf_import.py:860-898)."""
    if isinstance(layer_ranges, (str, bytes)) or len(layer_ranges) == 0:
        raise ValueError("layer_ranges must contain at least one range")
    if len(layer_ranges) > num_layers:
        raise ValueError("layer_ranges cannot contain more stages than model layers")
    out: list[tuple[int, int]] = []
    end = 0
    for i, r in enumerate(layer_ranges):
        if (not isinstance(r, (tuple, list)) or len(r) != 2
                or any(isinstance(v, bool) or not isinstance(v, int) for v in r)):
            raise TypeError(f"layer_ranges[{i}] must be a pair of integers")
        a, b = r
        if a != end or b <= a or b > num_layers:
            raise ValueError(
                "layer_ranges must be non-empty and contiguous from zero; "
                f"range {i} was [{a}, {b}) after {end}"
            )
        out.append((a, b))
        end = b
    if end != num_layers:
        raise ValueError(f"layer_ranges cover [0, {end}), expected [0, {num_layers})")
    return out


# ---------------------------------------------------------------------------
# Shards
# ---------------------------------------------------------------------------

def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb", buffering=0) as f:
        buf = bytearray(_HASH_CHUNK)
        view = memoryview(buf)
        while n := f.readinto(buf):
            h.update(view[:n])
    return h.hexdigest()


def verify_shard(root: Path, shard: ShardEntry) -> Path:
    """The shard's file, after its size and sha256 match the manifest."""
    path = resolve_artifact_path(root, shard.path)
    if not path.exists():
        raise FileNotFoundError(f"shard not found: {path}")
    size = path.stat().st_size
    if size != shard.byte_length:
        raise ValueError(f"shard {shard.shard_id} size mismatch: expected {shard.byte_length}, got {size}")
    actual = sha256_file(path)
    if actual != shard.sha256:
        raise ValueError(f"shard {shard.shard_id} hash mismatch: expected {shard.sha256}, got {actual}")
    return path


def _verify_all(root: Path, shards: Sequence[ShardEntry]) -> dict[str, Path]:
    """Verify distinct shards concurrently (sha256 releases the GIL)."""
    unique = list({s.shard_id: s for s in shards}.values())
    if len(unique) == 1:
        return {unique[0].shard_id: verify_shard(root, unique[0])}
    with ThreadPoolExecutor(max_workers=min(len(unique), os.cpu_count() or 1, 8)) as pool:
        paths = list(pool.map(lambda s: verify_shard(root, s), unique))
    return {s.shard_id: p for s, p in zip(unique, paths)}


def _load_state(path: Path, shard: ShardEntry) -> dict[str, torch.Tensor]:
    try:
        state = torch.load(path, map_location="cpu", weights_only=True, mmap=True)
    except RuntimeError:  # legacy (non-zip) serialisation cannot be mapped
        state = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(state, dict) or any(not isinstance(k, str) for k in state):
        raise ValueError(f"shard {shard.shard_id} must contain a string-keyed state dict")
    return state


def stage_state_for_range(
    manifest: ModelManifest, root: Path, layer_start: int, layer_end: int, *,
    is_first: bool, is_last: bool, verified: dict[str, Path] | None = None,
) -> dict[str, torch.Tensor]:
    """One stage's state (local names) from the shards overlapping its range:
    layer keys renumbered, the embedding kept on the first stage and the
    final norm / head on the last (hf_import.py:926-974)."""
    overlapping = manifest.shards_for_layers(layer_start, layer_end)
    if not overlapping:
        raise ValueError(f"no artifact shard overlaps requested range [{layer_start}, {layer_end})")
    state: dict[str, torch.Tensor] = {}
    for shard in overlapping:
        path = (verified or {}).get(shard.shard_id) or verify_shard(root, shard)
        for key, value in _load_state(path, shard).items():
            if key.startswith("layers."):
                parts = key.split(".", 2)
                if len(parts) < 3:
                    raise ValueError(f"invalid layer key in shard {shard.shard_id}: {key!r}")
                try:
                    local = int(parts[1])
                except ValueError as exc:
                    raise ValueError(f"invalid local layer index in shard {shard.shard_id}: {key!r}") from exc
                g = shard.layer_start + local
                if not layer_start <= g < layer_end:
                    continue
                target = f"layers.{g - layer_start}.{parts[2]}"
            elif key == "embed_tokens.weight":
                if not is_first:
                    continue
                target = key
            elif key in {"norm.weight", "lm_head.weight"}:
                if not is_last:
                    continue
                target = key
            else:
                raise ValueError(f"unexpected tensor key in shard {shard.shard_id}: {key!r}")
            if target in state:
                raise ValueError(f"duplicate tensor {target!r} while combining requested stage")
            state[target] = value
    return state


def check_stage_state(
    cfg: LlamaConfig, state: dict[str, torch.Tensor], stage_id: int, layer_start: int, layer_end: int, *,
    is_first: bool, is_last: bool,
) -> None:
    """Strict key and shape match, as ``load_state_dict(strict=True)``."""
    want = {local: shape for local, _, shape in stage_keys(cfg, layer_start, layer_end, is_first, is_last)}
    missing = sorted(set(want) - set(state))
    unexpected = sorted(set(state) - set(want))
    if missing or unexpected:
        raise RuntimeError(f"Stage {stage_id} weight mismatch — missing={missing}, unexpected={unexpected}")
    bad = [f"{k}: expected {want[k]}, got {tuple(state[k].shape)}" for k in sorted(want)
           if tuple(state[k].shape) != tuple(want[k])]
    if bad:
        raise RuntimeError(f"Stage {stage_id} weight shape mismatch: " + "; ".join(bad))


# ---------------------------------------------------------------------------
# Builders
# ---------------------------------------------------------------------------

def _stage_dtype(manifest: ModelManifest, dtype: torch.dtype | None) -> torch.dtype:
    if dtype is not None:
        return dtype
    try:
        return _DTYPES[manifest.meta.compute_dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported artifact compute_dtype: {manifest.meta.compute_dtype!r}") from exc


def _config_for(manifest: ModelManifest, root: Path) -> LlamaConfig:
    return load_stage_config(manifest, artifact_root=root)


def _make_worker(
    manifest: ModelManifest, cfg: LlamaConfig, state: dict[str, torch.Tensor], stage_id: int,
    layer_start: int, layer_end: int, *, is_first: bool, is_last: bool, device: Any, dtype: torch.dtype,
    job_id: str, transport: str, check_values: bool,
) -> B200StageWorker:
    check_stage_state(cfg, state, stage_id, layer_start, layer_end, is_first=is_first, is_last=is_last)
    if is_first and is_last and cfg.tie_word_embeddings:
        head, embed = state["lm_head.weight"], state["embed_tokens.weight"]
        if head.untyped_storage().data_ptr() == embed.untyped_storage().data_ptr():
            state["lm_head.weight"] = embed  # one HBM copy for the tied pair
    device = torch.device("cuda") if device is None else torch.device(device)
    stage = B200Stage(cfg, layer_start, layer_end, has_embedding=is_first, has_lm_head=is_last,
                      device=device, dtype=dtype, state_dict=state)
    stage.meshgpu_adapter = manifest.meta.adapter
    ctx = StageContext(
        stage_id=stage_id, layer_start=layer_start, layer_end=layer_end, device=stage.device,
        is_first=is_first, is_last=is_last, job_id=job_id, attempt_id="local", transport=transport,
    )
    log.info("loaded stage %d layers [%d, %d) on %s", stage_id, layer_start, layer_end, stage.device)
    return B200StageWorker(stage, ctx, check_values=check_values)


def build_stage_from_manifest(
    manifest_or_dir: Any,
    stage_id: int,
    *,
    device: torch.device | str | None = None,
    job_id: str = "local",
    artifact_root: str | Path | None = None,
    transport: str = "cpu",
    activation_checkpointing: bool = False,
    dtype: torch.dtype | None = None,
    check_values: bool = True,
) -> B200StageWorker:
    """Load exactly one shard's stage (hf_import.py:729-857): the entry point
    of a stage process, which never touches the other shards.

    ``device`` defaults to the current CUDA device; the stage dtype defaults
    to the manifest's ``compute_dtype``.
    """
    del activation_checkpointing  # training-only in the reference
    manifest, root = _open(manifest_or_dir, artifact_root)
    cfg = _config_for(manifest, root)
    ordered = validate_manifest_layout(manifest)
    if stage_id < 0 or stage_id >= len(ordered):
        raise IndexError(f"stage_id {stage_id} out of range [0, {len(ordered)})")
    st_dtype = _stage_dtype(manifest, dtype)
    shard = ordered[stage_id]
    is_first, is_last = stage_id == 0, stage_id == len(ordered) - 1
    state = _load_state(verify_shard(root, shard), shard)
    return _make_worker(manifest, cfg, state, stage_id, shard.layer_start, shard.layer_end,
                        is_first=is_first, is_last=is_last, device=device, dtype=st_dtype,
                        job_id=job_id, transport=transport, check_values=check_values)


def build_pipeline_from_manifest(
    manifest_or_dir: Any,
    *,
    artifact_root: str | Path | None = None,
    devices: list[torch.device] | None = None,
    job_id: str = "local",
    transport: str = "cpu",
    activation_checkpointing: bool = False,
    layer_ranges: Sequence[tuple[int, int]] | None = None,
    dtype: torch.dtype | None = None,
    check_values: bool = True,
) -> list[B200StageWorker]:
    """B200 workers for a saved artifact (hf_import.py:638-726).

    One stage per shard, or one per ``layer_ranges`` entry (a planner's
    partition, recombined from the overlapping shards).  ``devices`` defaults
    to the current CUDA device for every stage.
    """
    del activation_checkpointing
    manifest, root = _open(manifest_or_dir, artifact_root)
    cfg = _config_for(manifest, root)
    ordered = validate_manifest_layout(manifest)
    ranges = (validate_requested_ranges(layer_ranges, cfg.num_hidden_layers) if layer_ranges is not None
              else [(s.layer_start, s.layer_end) for s in ordered])
    n = len(ranges)
    if devices is None:
        devices = [None] * n
    if len(devices) != n:
        raise ValueError(f"need {n} devices for {n} stages, got {len(devices)}")
    st_dtype = _stage_dtype(manifest, dtype)
    verified = _verify_all(root, [s for a, b in ranges for s in manifest.shards_for_layers(a, b)])
    workers: list[B200StageWorker] = []
    try:
        for i, (a, b) in enumerate(ranges):
            first, last = i == 0, i == n - 1
            if layer_ranges is None:
                shard = ordered[i]
                state = _load_state(verified[shard.shard_id], shard)
            else:
                state = stage_state_for_range(manifest, root, a, b, is_first=first, is_last=last,
                                              verified=verified)
            workers.append(_make_worker(manifest, cfg, state, i, a, b, is_first=first, is_last=last,
                                        device=devices[i], dtype=st_dtype, job_id=job_id,
                                        transport=transport, check_values=check_values))
            del state
    except BaseException:
        for w in workers:
            w.close()
        raise
    return workers
