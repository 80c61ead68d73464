"""B200-native stage executor for MeshGPU-style pipeline inference.

Dense decoder stages (Llama and Qwen3 architectures) run on hand-written
sm_100a CUDA kernels behind a C ABI (``include/meshgpu_b200.h``); this package
is the Python host side with the reference's stage / pipeline API.
"""
from gpu_mesh_b200.batcher import ContinuousBatcher, SessionResult
from gpu_mesh_b200.config import LlamaConfig, config_from, split_layers
from gpu_mesh_b200.manifest import ModelManifest, build_pipeline_from_manifest, build_stage_from_manifest
from gpu_mesh_b200.pipeline import (
    build_pipeline,
    from_reference_workers,
    pipeline_decode_step,
    pipeline_decode_step_async,
    pipeline_prefill,
    pipeline_prefill_async,
)
from gpu_mesh_b200.sampling import SamplingParams, greedy_sample, make_sampling_generator, top_p_sample
from gpu_mesh_b200.stage import B200Stage
from gpu_mesh_b200.stage_worker import B200StageWorker, ForwardResult, StageContext
from gpu_mesh_b200.wire import tensor_from_wire, tensor_wire_parts

__all__ = [
    "B200Stage",
    "B200StageWorker",
    "ContinuousBatcher",
    "ForwardResult",
    "LlamaConfig",
    "ModelManifest",
    "SamplingParams",
    "SessionResult",
    "StageContext",
    "build_pipeline",
    "build_pipeline_from_manifest",
    "build_stage_from_manifest",
    "config_from",
    "from_reference_workers",
    "greedy_sample",
    "make_sampling_generator",
    "pipeline_decode_step",
    "pipeline_decode_step_async",
    "pipeline_prefill",
    "pipeline_prefill_async",
    "split_layers",
    "tensor_from_wire",
    "tensor_wire_parts",
    "top_p_sample",
]
