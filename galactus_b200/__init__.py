"""galactus_b200: the routed-expert FFN of a quantized MoE layer on B200 (sm_100a).

The product is the C-ABI library libgalactus_b200.so (include/galactus_b200.h);
this package is its Python binding plus the model shapes used by the tests and
the benchmark. Importing it loads the library and fails loudly if it is absent.
"""
from ._lib import (  # noqa: F401
    ACT_SWIGLU, ACT_SWIGLU_OAI, BLOCK_BYTES, BLOCK_ELEMS, GX_OK, GxError,
    GX_ERR_ALIGN, GX_ERR_BATCH, GX_ERR_COMM, GX_ERR_COPY, GX_ERR_CUDA, GX_ERR_DEVICE, GX_ERR_DOMAIN, GX_ERR_INVALID,
    GX_ERR_NOMEM, GX_ERR_SLOTS, GX_ERR_STATE, GX_ERR_TIMEOUT, GX_ERR_TYPE,
    POLICY_AUTO, POLICY_FREQUENCY, POLICY_LRU, POLICY_PLAN, POLICY_UNIFORM,
    TYPE_IQ1_S, TYPE_MXFP4, TYPE_NAMES, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, TYPE_Q8_K,
    check, declared_symbols, lib, row_bytes, vec_dot_type,
)
from .moe import Arena, LayerShape, SlotPolicy, mul_mat_id, record_layout  # noqa: F401
from .models import MODELS, ModelShape  # noqa: F401

__all__ = [
    "Arena", "LayerShape", "SlotPolicy", "mul_mat_id", "record_layout", "MODELS", "ModelShape", "lib", "check",
    "GxError",
]
