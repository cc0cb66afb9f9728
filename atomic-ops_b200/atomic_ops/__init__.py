"""Legacy `atomic_ops` API (atomic_ops/__init__.py, fallback.py:16-22) on the B200 operator.

The reference's legacy package exposes a (batch, seq_len, heads, d_head) ("BLHD") interface,
`gdn2_forward(q, k, v, w, b, g, scale, h0=None, config=None)` and its differentiable twin
`gdn2_forward_trainable`, configured by `KernelConfig` presets.  Here both run the atomic_gdn2
CUDA operator: the inputs are relaid out to (B, H, L, D), all products run in the fp32-faithful
"highest" mode (the legacy kernels use Precision.HIGHEST throughout), the operator's chunk is
128 tokens whatever `config.bt` says (the chunked-WY result does not depend on the chunk length;
`config.bt` still decides which sequence lengths are accepted, as in the reference), and the
whole sequence is one call (the legacy API has no segmentation).  o comes back as (B, L, H, D)
fp32, h_final as (B, H, D, D) fp32; gradients in the input dtypes.  There is no CPU path.
"""
from .configs import (DEFAULT_CONFIG, KAGGLE_LARGE, KAGGLE_MEDIUM, KAGGLE_SMALL, KernelConfig, sanitize,
                      validate_inputs)
from .fallback import gdn2_forward, gdn2_forward_trainable
from .utils import estimate_memory, get_recommended_config, is_tpu_available

gdn2_pallas_forward = gdn2_forward
gdn2_pallas_forward_trainable = gdn2_forward_trainable

__all__ = ["KernelConfig", "KAGGLE_SMALL", "KAGGLE_MEDIUM", "KAGGLE_LARGE", "DEFAULT_CONFIG", "is_tpu_available",
           "estimate_memory", "get_recommended_config", "gdn2_forward", "gdn2_forward_trainable",
           "gdn2_pallas_forward", "gdn2_pallas_forward_trainable", "sanitize", "validate_inputs"]
