"""Model definitions."""
from .qwen_moe import MoEConfig, Partition, QwenMoE, param_specs  # noqa: F401
