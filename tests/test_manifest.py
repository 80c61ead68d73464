"""The artifact loader's host side (no GPU): manifest parsing, config and
shard verification, planner re-splits and the reference loaders' error
behaviour (artifacts/manifest.py, artifacts/hf_import.py:537-1050, and the
reference tests tests/unit/test_hf_import.py:309-442).  The fixtures under
tests/golden/manifests were written by the reference's own importers
(make_manifest_fixtures.py)."""
from __future__ import annotations

import json
import shutil

import pytest
import torch

from gpu_mesh_b200.manifest import (
    ModelManifest,
    build_pipeline_from_manifest,
    build_stage_from_manifest,
    compute_config_hash,
    load_stage_config,
    stage_state_for_range,
    validate_manifest_layout,
    validate_requested_ranges,
)
from tests.conftest import GOLDEN

MANIFESTS = GOLDEN / "manifests"
NAMES = sorted(p.name for p in MANIFESTS.iterdir() if p.is_dir())


def copy(name, tmp_path):
    out = tmp_path / name
    shutil.copytree(MANIFESTS / name, out)
    return out


def manifest_json(root):
    return json.loads((root / "manifest.json").read_text())


def write_manifest(root, data):
    (root / "manifest.json").write_text(json.dumps(data))


def test_fixture_set():
    assert NAMES == ["llama_gqa_bf16", "llama_tied_fp32", "llama_tiny_fp32", "qwen3_tiny_fp32"]


@pytest.mark.parametrize("name", NAMES)
def test_reference_artifacts_parse_and_their_configs_hash(name):
    m = ModelManifest.load(MANIFESTS / name / "manifest.json")
    cfg = load_stage_config(MANIFESTS / name)  # raises on a config-hash mismatch
    assert m.config_hash
    assert cfg.num_hidden_layers == m.meta.num_layers == 4
    assert cfg.qk_norm == (m.meta.adapter == "qwen3_hf_v1")
    ordered = validate_manifest_layout(m)
    assert ordered[0].layer_start == 0 and ordered[-1].layer_end == 4
    exp = torch.load(MANIFESTS / f"{name}.expected.pt", weights_only=True)
    assert exp["stages"] == len(ordered)
    assert exp["prefill"].shape[-1] == cfg.vocab_size


@pytest.mark.parametrize("name", NAMES)
def test_planner_ranges_recombine_the_shards(name):
    root = MANIFESTS / name
    m = ModelManifest.load(root / "manifest.json")
    whole = stage_state_for_range(m, root, 0, 4, is_first=True, is_last=True)
    mid = stage_state_for_range(m, root, 1, 3, is_first=False, is_last=False)
    assert not any(k.startswith(("embed_tokens", "norm", "lm_head")) for k in mid)
    for k, v in mid.items():
        i, rest = k.split(".", 2)[1:]
        assert torch.equal(v, whole[f"layers.{int(i) + 1}.{rest}"])
    assert {k.split(".")[1] for k in mid if k.startswith("layers.")} == {"0", "1"}


def test_compute_config_hash_is_sorted_json_sha256_prefix():
    assert compute_config_hash({"b": 1, "a": 2.0}) == compute_config_hash({"a": 2.0, "b": 1})
    assert len(compute_config_hash({})) == 16


def test_missing_selected_shard_reports_not_found(tmp_path):
    root = copy("llama_tiny_fp32", tmp_path)
    shard = ModelManifest.load(root / "manifest.json").shards[1]
    (root / shard.path).unlink()
    with pytest.raises(FileNotFoundError, match="shard not found"):
        build_stage_from_manifest(root, 1)
    with pytest.raises(FileNotFoundError):
        build_pipeline_from_manifest(root)


def test_tampered_shard_fails_the_hash_check(tmp_path):
    root = copy("llama_tiny_fp32", tmp_path)
    shard = ModelManifest.load(root / "manifest.json").shards[0]
    data = bytearray((root / shard.path).read_bytes())
    data[-100] ^= 1
    (root / shard.path).write_bytes(bytes(data))
    with pytest.raises(ValueError, match="hash mismatch"):
        build_stage_from_manifest(root, 0)


def test_truncated_shard_fails_the_size_check(tmp_path):
    root = copy("llama_tiny_fp32", tmp_path)
    shard = ModelManifest.load(root / "manifest.json").shards[0]
    data = (root / shard.path).read_bytes()
    (root / shard.path).write_bytes(data[:-1])
    with pytest.raises(ValueError, match="size mismatch"):
        build_pipeline_from_manifest(root)


def test_edited_config_fails_the_config_hash(tmp_path):
    root = copy("llama_tiny_fp32", tmp_path)
    cpath = root / manifest_json(root)["config_path"]
    values = json.loads(cpath.read_text())
    values["rope_theta"] = 20000.0
    cpath.write_text(json.dumps(values))
    with pytest.raises(ValueError, match="config hash mismatch"):
        load_stage_config(root)


def test_config_falls_back_to_manifest_meta_without_config_json(tmp_path):
    root = copy("llama_tiny_fp32", tmp_path)
    want = load_stage_config(root)
    (root / manifest_json(root)["config_path"]).unlink()
    assert load_stage_config(root) == want  # meta.extra carries eps / theta / attention


def test_manifest_paths_must_stay_inside_the_artifact(tmp_path):
    root = copy("llama_tiny_fp32", tmp_path)
    data = manifest_json(root)
    data["shards"][0]["path"] = "../escape.pt"
    write_manifest(root, data)
    with pytest.raises(ValueError, match="relative and contained"):
        ModelManifest.load(root / "manifest.json")


def test_shards_must_cover_contiguous_layers(tmp_path):
    root = copy("llama_tiny_fp32", tmp_path)
    data = manifest_json(root)
    data["shards"][1]["layer_start"] = 3
    write_manifest(root, data)
    with pytest.raises(ValueError, match="contiguous"):
        ModelManifest.load(root / "manifest.json")


def test_unsupported_adapter_is_rejected(tmp_path):
    root = copy("llama_tiny_fp32", tmp_path)
    data = manifest_json(root)
    data["meta"]["adapter"] = "mixtral_v1"
    write_manifest(root, data)
    with pytest.raises(ValueError, match="unsupported manifest adapter"):
        load_stage_config(root)


def test_geometry_mismatch_is_rejected(tmp_path):
    root = copy("qwen3_tiny_fp32", tmp_path)
    data = manifest_json(root)
    data["meta"]["vocab_size"] = 98
    write_manifest(root, data)
    with pytest.raises(ValueError, match="manifest/config mismatch: vocab_size"):
        load_stage_config(root)


def test_requested_ranges_validation_messages():
    assert validate_requested_ranges([(0, 1), (1, 4)], 4) == [(0, 1), (1, 4)]
    with pytest.raises(ValueError, match="contiguous"):
        validate_requested_ranges([(0, 1), (2, 4)], 4)
    with pytest.raises(ValueError, match="cover"):
        validate_requested_ranges([(0, 1), (1, 3)], 4)
    with pytest.raises(ValueError, match="at least one"):
        validate_requested_ranges([], 4)
    with pytest.raises(TypeError, match="pair of integers"):
        validate_requested_ranges([(0, 1.0)], 4)
    with pytest.raises(ValueError, match="more stages"):
        validate_requested_ranges([(0, 1)] * 5, 4)


def test_pipeline_needs_one_device_per_stage():
    with pytest.raises(ValueError, match="need 2 devices for 2 stages"):
        build_pipeline_from_manifest(MANIFESTS / "llama_tiny_fp32", devices=[torch.device("cuda", 0)])


def test_stages_never_fall_back_to_the_cpu():
    with pytest.raises(ValueError, match="CUDA device"):
        build_stage_from_manifest(MANIFESTS / "llama_tiny_fp32", 0, device=torch.device("cpu"))


def test_reference_manifest_objects_are_accepted():
    class PydanticLike:  # a reference ModelManifest exposes model_dump()
        def model_dump(self):
            return manifest_json(MANIFESTS / "qwen3_tiny_fp32")

    cfg = load_stage_config(PydanticLike(), artifact_root=MANIFESTS / "qwen3_tiny_fp32")
    assert cfg.qk_norm and cfg.vocab_size == 97
