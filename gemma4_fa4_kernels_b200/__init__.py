"""B200-native (sm_100a) Gemma-4 attention backend.

Drop-in for the operator surface of the reference ``gemma4_fa4`` package:
the fixed-BSHD and packed-THD local-d256 / global-d512 adapters, the exact
mask builders and the geometry contract, and a Transformers attention backend
(``register_gemma4_fa4_b200``), and the fused Q/K/V preparation (RMS norm +
rotary, with its adjoint).  Compute runs in
``libgemma4_b200.so`` (hand-written tcgen05/TMA kernels); there is no CPU or
library fallback on the attention path.
"""

from .b200 import (
    fa4_global_forward_only,
    fa4_global_text_forward,
    fa4_global_varlen_forward,
    fa4_global_varlen_forward_only,
    fa4_local_forward,
    fa4_local_text_forward,
    fa4_local_varlen_forward,
)
from .errors import GlobalBackwardBudgetExceeded, UnsupportedB200Path, UnsupportedH100Path
from .masks import additive_mask, gemma4_attention_mask
from .model_spec import (
    GEMMA4_31B,
    GLOBAL_ATTENTION,
    SLIDING_ATTENTION,
    AttentionLayerSpec,
    Gemma4ModelSpec,
)
from .prep import (
    prepare_global_kv_from_projection_source,
    prepare_rotary_operand,
    prepare_shared_kv,
    prepare_value,
)
from .transformers_backend import (
    BACKEND_NAME,
    Gemma4DispatchResult,
    Gemma4MaskPlan,
    gemma4_fa4_b200_attention_forward,
    gemma4_fa4_b200_mask,
    gemma4_fa4_b200_prepared,
    register_gemma4_fa4_b200,
)

__all__ = [
    "AttentionLayerSpec",
    "Gemma4ModelSpec",
    "GEMMA4_31B",
    "SLIDING_ATTENTION",
    "GLOBAL_ATTENTION",
    "fa4_local_forward",
    "fa4_local_text_forward",
    "fa4_local_varlen_forward",
    "fa4_global_text_forward",
    "fa4_global_forward_only",
    "fa4_global_varlen_forward",
    "fa4_global_varlen_forward_only",
    "GlobalBackwardBudgetExceeded",
    "UnsupportedB200Path",
    "UnsupportedH100Path",
    "gemma4_attention_mask",
    "additive_mask",
    "BACKEND_NAME",
    "Gemma4DispatchResult",
    "Gemma4MaskPlan",
    "gemma4_fa4_b200_attention_forward",
    "gemma4_fa4_b200_mask",
    "gemma4_fa4_b200_prepared",
    "register_gemma4_fa4_b200",
    "prepare_global_kv_from_projection_source",
    "prepare_rotary_operand",
    "prepare_shared_kv",
    "prepare_value",
]
