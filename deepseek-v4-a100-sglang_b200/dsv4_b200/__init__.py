"""B200 (sm_100a) MXFP4-weight / INT8-activation MoE hot path.

Public API mirrors the reference's op layer (``triton_kernels``) and JIT op
layer (``sglang_jit_patches``); see ``mxfp4_int8_moe`` and ``jit_ops``.
"""

from .mxfp4_int8_moe import (  # noqa: F401
    Mxfp4Int8DenseWeight,
    Mxfp4Int8MoeWeights,
    max_mxfp4_int8_moe_block_m,
    moe_align_block_size,
    mxfp4_int8_dense_forward,
    mxfp4_int8_moe_forward,
    prepare_mxfp4_int8_dense_weight,
    prepare_mxfp4_int8_moe,
    quantize_per_token_int8,
    remap_mxfp4_weight_for_int8,
    select_mxfp4_int8_moe_tile_shape,
    select_sorted_block_m,
    router_topk,
    router_align,
    mxfp4_int8_moe_forward_from_logits,
    Mxfp4Int8MoeGraph,
)
from .jit_ops import (  # noqa: F401
    mxfp4_int8_dense_gemm,
    mxfp4_int8_dense_gemm_i32,
    mxfp4_int8_moe_gemm,
    mxfp4_int8_moe_gemm_swiglu,
    mxfp4_int8_moe_reduce,
    moe_sort_rows,
    quantize_scatter_int8,
    quantize_sorted_int8,
    mxfp4_int8_moe_gemm_sorted,
    mxfp4_int8_moe_gemm_swiglu_sorted,
    prewarm_mxfp4_int8_dense_jit_module,
    prewarm_mxfp4_int8_moe_jit_modules,
)
from ._native import DeviceTimeoutError, check_device_status  # noqa: F401,E402
