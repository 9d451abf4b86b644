"""B200-native (sm_100a) rebuild of the reference's transformer forward pass.

Public surface, mirroring torch_transformer_benchmark.py:
    TransformerConfig, BaselineTransformer (parameter layout),
    UserOptimizedTransformer (the drop-in forward on B200 kernels),
    copy_model_weights, count_dense_flops.
Kernel-level wrappers are in `transformer_optimization_b200.kernels`; the C
ABI they call is declared in include/tfb200.h.
"""

from .config import NAMED_CONFIGS, TransformerConfig, count_causal_flops, count_dense_flops
from .model import (
    BaselineSelfAttention,
    BaselineTransformer,
    BaselineTransformerBlock,
    UserOptimizedTransformer,
    copy_model_weights,
)

__all__ = [
    "TransformerConfig",
    "NAMED_CONFIGS",
    "count_dense_flops",
    "count_causal_flops",
    "BaselineSelfAttention",
    "BaselineTransformerBlock",
    "BaselineTransformer",
    "UserOptimizedTransformer",
    "copy_model_weights",
]
