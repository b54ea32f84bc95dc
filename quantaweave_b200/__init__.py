"""QuantaWeave-B200: a sparse Mixture-of-Experts language-model framework for NVIDIA B200 (sm_100a).

Public API (names kept from jorgenep/QuantaWeave):

* model: ``QuantaWeaveConfig``, ``QuantaWeaveMoEForCausalLM``, ``QuantaWeaveBlock``, ``TopKMoE``, ``SparseSwiGLU``;
* data: ``CharTokenizer``, ``BPETokenizer``, ``SentencePieceTokenizer``, ``load_tokenizer``;
* training: ``run_training``, ``default_args``, ``build_parser``, ``save_checkpoint``, ``load_checkpoint``,
  ``TrainingController``, ``ScheduleConfig``, ``MetricsLogger``;
* inference and adaptation: ``FastDecoder``, ``QuantizedLinear``, ``quantize_model``, ``save_quantized``,
  ``load_quantized``, ``add_lora``, ``CPUOffloadAdamW``;
* parallelism: ``init_expert_parallel``, ``ShardedAdamW``, ``PipelineEngine``, ``consolidate_checkpoint``,
  ``reshard_checkpoint``.
"""

from .config import PRESETS, QuantaWeaveConfig, preset
from .models import QuantaWeaveBlock, QuantaWeaveMoEForCausalLM, SparseSwiGLU, TopKMoE

__version__ = "0.1.0"

_LAZY = {
    "run_training": ("training.trainer", "run_training"),
    "default_args": ("training.trainer", "default_args"),
    "build_parser": ("training.trainer", "build_parser"),
    "save_checkpoint": ("training.trainer", "save_checkpoint"),
    "load_checkpoint": ("training.trainer", "load_checkpoint"),
    "TrainingController": ("training.schedules", "TrainingController"),
    "ScheduleConfig": ("training.schedules", "ScheduleConfig"),
    "MetricsLogger": ("training.metrics", "MetricsLogger"),
    "CharTokenizer": ("data.pipeline", "CharTokenizer"),
    "BPETokenizer": ("data.pipeline", "BPETokenizer"),
    "SentencePieceTokenizer": ("data.pipeline", "SentencePieceTokenizer"),
    "load_tokenizer": ("data.pipeline", "load_tokenizer"),
    "FastDecoder": ("inference.fast_decode", "FastDecoder"),
    "save_quantized": ("inference.quantization", "save_quantized"),
    "load_quantized": ("inference.quantization", "load_quantized"),
    "add_lora": ("tools.lora", "add_lora"),
    "CPUOffloadAdamW": ("optim.cpu_offload", "CPUOffloadAdamW"),
    "QuantizedLinear": ("inference.quantization", "QuantizedLinear"),
    "quantize_model": ("inference.quantization", "quantize_model"),
    "init_expert_parallel": ("parallel.expert_parallel", "init_expert_parallel"),
    "ShardedAdamW": ("parallel.sharded_optimizer", "ShardedAdamW"),
    "PipelineEngine": ("parallel.pipeline_parallel", "PipelineEngine"),
    "consolidate_checkpoint": ("parallel.checkpoint", "consolidate_checkpoint"),
    "reshard_checkpoint": ("parallel.checkpoint", "reshard_checkpoint"),
}


def __getattr__(name):
    if name in _LAZY:
        import importlib

        module, attr = _LAZY[name]
        return getattr(importlib.import_module(f".{module}", __name__), attr)
    raise AttributeError(name)


__all__ = ["PRESETS", "QuantaWeaveConfig", "preset", "QuantaWeaveBlock", "QuantaWeaveMoEForCausalLM", "SparseSwiGLU",
           "TopKMoE", *_LAZY]
