"""B200-native (sm_100a) forward pass of the TikTokTechJam2026 causal Transformer.

Public surface (mirrors the reference's mixed_precision package):

* ``MixedPrecisionTransformer`` / ``B200Transformer`` -- drop-in model
* ``copy_mixed_model_weights``                       -- baseline -> packed weights
* ``PreallocatedMicrobatchModel``                    -- the reference runner's microbatch wrapper
* ``TransformerConfig``                              -- same fields as the reference's
* ``ops``                                            -- single-op wrappers of the C ABI
* ``sharding``                                       -- batch sharding across GPUs
"""

from .model import (  # noqa: F401
    B200Transformer,
    MixedPrecisionTransformer,
    PreallocatedMicrobatchModel,
    TransformerConfig,
    copy_mixed_model_weights,
)

__all__ = ["B200Transformer", "MixedPrecisionTransformer", "PreallocatedMicrobatchModel", "TransformerConfig",
           "copy_mixed_model_weights"]
