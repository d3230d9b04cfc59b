"""ElasticMegatron-B200: an elastic LLM training framework for NVIDIA B200.

Public surface (the reference exports the same four names from ``elastic_megatron/__init__.py``):
``ElasticMegatronManager``, ``apply_hetero_dp``, ``meta_device_context``, ``nccl_group_recreate``; plus the
building blocks ``ParallelStrategy``, ``TrainingState``, ``train_step``.  Imports are lazy so that
``import elasticmegatron_b200`` stays cheap and never touches CUDA.
"""
__version__ = "0.1.0"

_EXPORTS = {
    "ElasticMegatronManager": ("runtime.manager", "ElasticMegatronManager"),
    "apply_hetero_dp": ("runtime.hetero_dp", "apply_hetero_dp"),
    "meta_device_context": ("runtime.meta", "meta_device_context"),
    "nccl_group_recreate": ("parallel.process_groups", "nccl_group_recreate"),
    "global_barrier_by_gloo": ("parallel.process_groups", "global_barrier_by_gloo"),
    "build_nccl_connection_context": ("runtime.manager", "build_nccl_connection_context"),
    "ParallelStrategy": ("parallel.strategy", "ParallelStrategy"),
    "TrainingState": ("runtime.training_state", "TrainingState"),
    "train_step": ("runtime.train", "train_step"),
    "ModelConfig": ("config", "ModelConfig"),
    "TrainConfig": ("config", "TrainConfig"),
}

__all__ = sorted(_EXPORTS)


def __getattr__(name):
    if name in _EXPORTS:
        import importlib

        mod, attr = _EXPORTS[name]
        return getattr(importlib.import_module(f"{__name__}.{mod}"), attr)
    raise AttributeError(name)
