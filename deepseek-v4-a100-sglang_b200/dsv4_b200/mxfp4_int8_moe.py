"""MXFP4-weight / INT8-activation MoE and dense ops for B200 (sm_100a).

Drop-in mirror of the reference's op layer
``dsv4_a100_patch/triton_kernels/mxfp4_int8_moe.py`` (PYMOE): the same public
names, arguments, returned layouts and error types, backed by the C ABI of
``libdsv4_b200.so`` (hand-written sm_100a kernels).  There is no CPU path: a
CPU tensor or a missing library raises.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
from torch.nn import Parameter

from . import _native as N
from .jit_ops import (
    mxfp4_int8_moe_gemm_swiglu,
    mxfp4_int8_moe_gemm,
    mxfp4_int8_moe_reduce,
    mxfp4_int8_dense_gemm,
    prewarm_mxfp4_int8_moe_jit_modules,
    moe_sort_rows,
    quantize_scatter_int8,
    quantize_sort_int8,
    quantize_sorted_int8,
    mxfp4_int8_moe_gemm_swiglu_sorted,
    mxfp4_int8_moe_gemm_sorted,
    use_cm_tile,
    quantize_per_token_int8_cm,
    dense_gemm_cm,
)

_VALID_BLOCK_M = {16, 32, 64, 128}
_VALID_BLOCK_N = {32, 64, 128}
_MAX_BLOCK_M = 128
# The B200 kernel computes 128 output channels per CTA; block_n is kept in the
# API for compatibility and does not change the tile.
_B200_BLOCK_N = 128


@dataclass
class Mxfp4Int8MoeWeights:
    """PYMOE:34-43."""
    w13_mxfp4: torch.Tensor
    w13_shift2: torch.Tensor
    w13_channel_scale: torch.Tensor
    w2_mxfp4: torch.Tensor
    w2_shift2: torch.Tensor
    w2_channel_scale: torch.Tensor
    headroom_bits: int


@dataclass
class Mxfp4Int8DenseWeight:
    """PYMOE:46-50."""
    weight_mxfp4: torch.Tensor
    weight_shift2: torch.Tensor
    weight_channel_scale: torch.Tensor
    headroom_bits: int


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor on an sm_100a device (no CPU path)")


_DTYPES = {torch.float32: N.DTYPE_F32, torch.float16: N.DTYPE_F16, torch.bfloat16: N.DTYPE_BF16}


def quantize_per_token_int8(a: torch.Tensor, clamp_abs: float = 0.0):
    """PYMOE:95-126: ``(q int8 [M,K], scale fp32 [M])``."""
    if a.dim() != 2:
        raise ValueError(f"a must have shape [M, K], got {tuple(a.shape)}")
    if a.dtype not in _DTYPES:
        raise TypeError(f"a must be fp32, fp16, or bf16, got {a.dtype}")
    _require_cuda(a, "a")
    a = a.contiguous()
    m, k = a.shape
    a_q = torch.empty((m, k), device=a.device, dtype=torch.int8)
    a_scale = torch.empty((m,), device=a.device, dtype=torch.float32)
    N.call("dsv4_b200_quantize_per_token_int8", a.data_ptr(), _DTYPES[a.dtype], m, k, k,
           float(clamp_abs), a_q.data_ptr(), a_scale.data_ptr(), N.stream_of(a))
    return a_q, a_scale


def _as_uint8_storage(tensor: torch.Tensor) -> torch.Tensor:
    """PYMOE:269-279."""
    data = tensor.data if hasattr(tensor, "data") else tensor
    if data.dtype == torch.uint8:
        return data.contiguous()
    if data.dtype == torch.int8:
        return data.view(torch.uint8).contiguous()
    if data.dtype == torch.float8_e8m0fnu:
        return data.view(torch.uint8).contiguous()
    if data.dtype in (torch.float16, torch.bfloat16, torch.float32):
        return data.to(torch.float8_e8m0fnu).view(torch.uint8).contiguous()
    raise TypeError(f"unsupported MXFP4 scale dtype: {data.dtype}")


def remap_mxfp4_weight_for_int8(weight: torch.Tensor, scale: torch.Tensor, *, headroom_bits: int = 3,
                                use_triton: bool = True):
    """PYMOE:607-667.  ``use_triton=True`` selects the production rounding of
    the reference's Triton repack (half-up), ``False`` its torch repack
    (half-even); both run on the GPU here."""
    if headroom_bits < 0 or headroom_bits > 7:
        raise ValueError(f"invalid headroom_bits={headroom_bits}")
    w_u8 = weight.data if hasattr(weight, "data") else weight
    w_u8 = w_u8.view(torch.uint8).contiguous()
    scale_u8 = _as_uint8_storage(scale)
    if w_u8.dim() != 3 or scale_u8.dim() != 3:
        raise ValueError(
            f"expected expert weight/scale shapes [E, N, K/2] and [E, N, K/32], "
            f"got {tuple(w_u8.shape)} and {tuple(scale_u8.shape)}")
    if w_u8.shape[0] != scale_u8.shape[0] or w_u8.shape[1] != scale_u8.shape[1]:
        raise ValueError(f"weight/scale shape mismatch: {tuple(w_u8.shape)} vs {tuple(scale_u8.shape)}")
    if w_u8.shape[2] * 2 != scale_u8.shape[2] * 32:
        raise ValueError(f"K mismatch: {tuple(w_u8.shape)} vs {tuple(scale_u8.shape)}")
    _require_cuda(w_u8, "weight")
    e, n, pk = w_u8.shape
    k = pk * 2
    kb = k // 32
    ng8 = (n + 7) // 8
    ss = (kb + 3) // 4
    b_mxfp4 = torch.empty((e, kb, ng8, 128), device=w_u8.device, dtype=torch.uint8)
    b_shift2 = torch.empty((e, ss, ng8, 8), device=w_u8.device, dtype=torch.uint8)
    cs = torch.empty((e, n), device=w_u8.device, dtype=torch.float32)
    N.call("dsv4_b200_remap_mxfp4_weight_for_int8", w_u8.data_ptr(), scale_u8.data_ptr(), e, n, k,
           headroom_bits, 0 if use_triton else 1, b_mxfp4.data_ptr(), b_shift2.data_ptr(),
           cs.data_ptr(), N.stream_of(w_u8))
    return b_mxfp4, b_shift2, cs


def prepare_mxfp4_int8_dense_weight(weight: torch.Tensor, scale: torch.Tensor, *,
                                    headroom_bits: int = 3) -> Mxfp4Int8DenseWeight:
    """PYMOE:670-686."""
    b, sh, cs = remap_mxfp4_weight_for_int8(weight.unsqueeze(0), scale.unsqueeze(0),
                                            headroom_bits=headroom_bits)
    return Mxfp4Int8DenseWeight(b[0].contiguous(), sh[0].contiguous(), cs[0].contiguous(),
                                headroom_bits)


def mxfp4_int8_dense_forward(hidden_states: torch.Tensor, weight: Mxfp4Int8DenseWeight,
                             bias: torch.Tensor | None = None) -> torch.Tensor:
    """PYMOE:689-740 (bias unsupported, as in the reference)."""
    if bias is not None:
        raise NotImplementedError("MXFP4-int8 dense JIT path does not support bias")
    hidden_states = hidden_states.contiguous()
    n = weight.weight_channel_scale.shape[0]
    m, k = hidden_states.shape
    out = torch.empty((m, n), device=hidden_states.device, dtype=torch.bfloat16)
    if (use_cm_tile(m, k, n) and hidden_states.dtype in (torch.bfloat16, torch.float16)
            and k <= 8192):
        # large M: quantise straight into the K-chunk-major layout of the
        # 256-token tile (same numbers as the row-major quantiser)
        _require_cuda(hidden_states, "hidden_states")
        a_cm, a_scale, rs = quantize_per_token_int8_cm(hidden_states)
        dense_gemm_cm(a_cm, a_scale, rs, weight.weight_mxfp4, weight.weight_shift2,
                      weight.weight_channel_scale, out)
        return out
    a_q, a_scale = quantize_per_token_int8(hidden_states, 0.0)
    partial = (torch.empty((4, m, (n + 31) // 32 * 32), device=hidden_states.device, dtype=torch.int32)
               if m <= 128 else torch.empty((0,), device=hidden_states.device, dtype=torch.int32))
    mxfp4_int8_dense_gemm(a_q, a_scale, weight.weight_mxfp4, weight.weight_shift2,
                          weight.weight_channel_scale, out, partial)
    return out


def prepare_mxfp4_int8_moe(layer: torch.nn.Module, *, headroom_bits: int = 3,
                           topk: int | None = None) -> None:
    """PYMOE:743-788: repack W13/W2, prewarm, free the original Parameters."""
    backend = os.environ.get("SGLANG_DSV4_MXFP4_INT8_REPACK_BACKEND", "triton").strip().lower()
    if backend not in {"triton", "torch"}:
        raise ValueError("SGLANG_DSV4_MXFP4_INT8_REPACK_BACKEND must be 'triton' or 'torch'")
    use_triton = backend == "triton"
    w13 = remap_mxfp4_weight_for_int8(layer.w13_weight.data, layer.w13_weight_scale_inv.data,
                                      headroom_bits=headroom_bits, use_triton=use_triton)
    w2 = remap_mxfp4_weight_for_int8(layer.w2_weight.data, layer.w2_weight_scale_inv.data,
                                     headroom_bits=headroom_bits, use_triton=use_triton)
    layer._dsv4_mxfp4_int8_weights = Mxfp4Int8MoeWeights(*w13, *w2, headroom_bits)
    if topk is None:
        topk = int(getattr(layer, "top_k", 0) or getattr(layer, "topk", 0) or 8)
    hidden_size = int(w2[2].shape[1])
    intermediate_size = int(w2[0].shape[1] * 32)
    prewarm_mxfp4_int8_moe_jit_modules(hidden_size=hidden_size,
                                       intermediate_size=intermediate_size, topk=topk)
    empty_u8 = torch.empty(0, device=w13[0].device, dtype=torch.uint8)
    empty_i8 = empty_u8.view(torch.int8)
    layer.w13_weight = Parameter(empty_i8, requires_grad=False)
    layer.w2_weight = Parameter(empty_i8, requires_grad=False)
    layer.w13_weight_scale_inv = Parameter(empty_u8, requires_grad=False)
    layer.w2_weight_scale_inv = Parameter(empty_u8, requires_grad=False)


def max_mxfp4_int8_moe_block_m(m: int, topk: int, experts: int) -> int:
    """PYMOE:799-801."""
    avg = max(1, (m * topk + max(experts, 1) - 1) // max(experts, 1))
    return min(_MAX_BLOCK_M, max(16, 1 << (avg - 1).bit_length()))


def _select_moe_tile_shape(m: int, topk: int, experts: int) -> tuple[int, int]:
    """B200 tile policy with the reference's env overrides and cap
    (PYMOE:816-839).  The token tile equals block_m and one decoded weight
    tile serves all of its tokens, so the largest block_m under the cap
    (the average routed tokens per expert, rounded up to a power of two)
    is chosen."""
    max_block_m = max_mxfp4_int8_moe_block_m(m, topk, experts)
    bm_env = os.environ.get("SGLANG_DSV4_MXFP4_INT8_BLOCK_M", "").strip()
    bn_env = os.environ.get("SGLANG_DSV4_MXFP4_INT8_BLOCK_N", "").strip()
    if bm_env or bn_env:
        block_m = int(bm_env) if bm_env else 16
        block_n = int(bn_env) if bn_env else 128
        if block_m not in _VALID_BLOCK_M:
            raise ValueError("SGLANG_DSV4_MXFP4_INT8_BLOCK_M must be 16, 32, 64, or 128")
        if block_n not in _VALID_BLOCK_N:
            raise ValueError("SGLANG_DSV4_MXFP4_INT8_BLOCK_N must be 32, 64, or 128")
        if block_m > max_block_m:
            raise ValueError(f"SGLANG_DSV4_MXFP4_INT8_BLOCK_M={block_m} exceeds cap "
                             f"{max_block_m} for m={m}, topk={topk}, experts={experts}")
        return block_m, block_n
    return max_block_m, _B200_BLOCK_N


def select_mxfp4_int8_moe_tile_shape(m: int, topk: int, experts: int) -> tuple[int, int]:
    """PYMOE:795-796."""
    return _select_moe_tile_shape(m, topk, experts)


def select_sorted_block_m(m: int, topk: int, experts: int) -> int:
    """Token tile of the expert-sorted fast path: the tile policy above,
    widened to 256 tokens (N=256 MMAs: one weight decode and one MMA
    instruction per 256 tokens) when the average routed tokens per expert
    reach 256 and no tile is forced through the environment.
    ``DSV4_B200_WIDE_TILE=192`` picks the 192-token tile instead (two
    accumulators, so the epilogue overlaps the next item's MMAs; measured
    slower overall at M=8192: W2 -5 %, W13 +12 %)."""
    block_m, _ = _select_moe_tile_shape(m, topk, experts)
    forced = os.environ.get("SGLANG_DSV4_MXFP4_INT8_BLOCK_M", "").strip()
    avg = (m * topk + max(experts, 1) - 1) // max(experts, 1)
    if block_m == _MAX_BLOCK_M and not forced and avg >= 256:
        return int(os.environ.get("DSV4_B200_WIDE_TILE", "256"))
    return block_m


def router_topk(router_logits: torch.Tensor, topk: int, *, bias: torch.Tensor | None = None,
                renormalize: bool = True, scale: float = 1.0):
    """DeepSeek routing on the GPU (what SGLang computes before the MoE call,
    PATCH:505-507): sigmoid scores, top-``topk`` experts by score + ``bias``
    (selection only), weights = chosen scores renormalised (and scaled).
    Returns ``(topk_ids int32 [M, topk], topk_weights fp32 [M, topk])`` in
    descending order, ready for :func:`moe_align_block_size`."""
    if router_logits.dim() != 2 or router_logits.dtype not in _DTYPES:
        raise ValueError("router_logits must be a 2-D fp32/fp16/bf16 tensor")
    _require_cuda(router_logits, "router_logits")
    logits = router_logits.contiguous()
    m, e = logits.shape
    b = None
    if bias is not None:
        b = bias.to(device=logits.device, dtype=torch.float32).contiguous()
        if b.shape != (e,):
            raise ValueError(f"bias must have shape [{e}], got {tuple(b.shape)}")
    ids = torch.empty((m, topk), device=logits.device, dtype=torch.int32)
    w = torch.empty((m, topk), device=logits.device, dtype=torch.float32)
    N.call("dsv4_b200_router_topk", logits.data_ptr(), _DTYPES[logits.dtype], m, e,
           b.data_ptr() if b is not None else None, topk, 1 if renormalize else 0, float(scale),
           ids.data_ptr(), w.data_ptr(), N.stream_of(logits))
    return ids, w


def router_align(router_logits: torch.Tensor, topk: int, block_size: int, *,
                 bias: torch.Tensor | None = None, renormalize: bool = True,
                 scale: float = 1.0, return_slot_pos: bool = False):
    """:func:`router_topk` and :func:`moe_align_block_size` in one launch
    (a cooperative kernel; same results bit for bit).  Returns
    ``(topk_ids, topk_weights, sorted_token_ids, expert_ids,
    num_tokens_post_pad)``, plus ``slot_pos`` (the sorted position of each
    routed slot) with ``return_slot_pos``."""
    if router_logits.dim() != 2 or router_logits.dtype not in _DTYPES:
        raise ValueError("router_logits must be a 2-D fp32/fp16/bf16 tensor")
    _require_cuda(router_logits, "router_logits")
    logits = router_logits.contiguous()
    m, e = logits.shape
    dev = logits.device
    b = None
    if bias is not None:
        b = bias.to(device=dev, dtype=torch.float32).contiguous()
        if b.shape != (e,):
            raise ValueError(f"bias must have shape [{e}], got {tuple(b.shape)}")
    ids = torch.empty((m, topk), device=dev, dtype=torch.int32)
    w = torch.empty((m, topk), device=dev, dtype=torch.float32)
    cap = align_capacity(m * topk, e, block_size)
    sorted_ids = torch.empty((cap,), dtype=torch.int32, device=dev)
    n_blocks = (cap + block_size - 1) // block_size
    expert_ids = torch.empty((n_blocks,), dtype=torch.int32, device=dev)
    ntpp = torch.empty((1,), dtype=torch.int32, device=dev)
    import ctypes
    words = ctypes.c_int64(0)
    N.call("dsv4_b200_router_align_workspace_words", m, e, ctypes.byref(words))
    ws = torch.empty((max(words.value, 1),), dtype=torch.int32, device=dev)
    slot_pos = (torch.empty((m * topk,), dtype=torch.int32, device=dev)
                if return_slot_pos else None)
    N.call("dsv4_b200_router_align", logits.data_ptr(), _DTYPES[logits.dtype], m, e,
           b.data_ptr() if b is not None else None, topk, 1 if renormalize else 0, float(scale),
           block_size, ids.data_ptr(), w.data_ptr(), sorted_ids.data_ptr(), cap,
           expert_ids.data_ptr(), n_blocks, ntpp.data_ptr(), ws.data_ptr(), ws.numel(),
           slot_pos.data_ptr() if slot_pos is not None else None, N.stream_of(logits))
    if return_slot_pos:
        return ids, w, sorted_ids, expert_ids, ntpp, slot_pos
    return ids, w, sorted_ids, expert_ids, ntpp


def align_capacity(numel: int, num_experts: int, block_size: int) -> int:
    """PYMOE:848-851."""
    if numel < num_experts + 1:
        return numel * block_size
    return numel + (num_experts + 1) * (block_size - 1)


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int, *,
                         return_slot_pos: bool = False):
    """Native replacement of ``_moe_align_block_size`` (PYMOE:842-869):
    ``(sorted_token_ids, expert_ids, num_tokens_post_pad)``.  Stable order
    inside each expert; padding value ``numel``; ids outside [0, E) dropped.
    With ``return_slot_pos`` a fourth tensor, int32 ``[numel]``: the sorted
    position of each id (-1 when dropped), the inverse permutation."""
    _require_cuda(topk_ids, "topk_ids")
    ids = topk_ids.to(torch.int32).contiguous()
    numel = ids.numel()
    cap = align_capacity(numel, num_experts, block_size)
    dev = ids.device
    sorted_ids = torch.empty((cap,), dtype=torch.int32, device=dev)
    n_blocks = (cap + block_size - 1) // block_size
    expert_ids = torch.empty((n_blocks,), dtype=torch.int32, device=dev)
    ntpp = torch.empty((1,), dtype=torch.int32, device=dev)
    if numel >= _ALIGN_COOP_MIN_IDS or return_slot_pos:
        # many ids: the multi-CTA align (same outputs); it also records the
        # inverse permutation
        import ctypes
        words = ctypes.c_int64(0)
        N.call("dsv4_b200_moe_align_workspace_words", numel, num_experts, ctypes.byref(words))
        ws = torch.empty((max(words.value, 1),), dtype=torch.int32, device=dev)
        slot_pos = (torch.empty((max(numel, 1),), dtype=torch.int32, device=dev)
                    if return_slot_pos else None)
        N.call("dsv4_b200_moe_align_block_size_ws", ids.data_ptr() if numel else None, numel,
               num_experts, block_size, sorted_ids.data_ptr(), cap, expert_ids.data_ptr(),
               n_blocks, ntpp.data_ptr(), None, ws.data_ptr(), ws.numel(),
               slot_pos.data_ptr() if slot_pos is not None else None, N.stream_of(ids))
        if return_slot_pos:
            return sorted_ids, expert_ids, ntpp, slot_pos[:numel]
        return sorted_ids, expert_ids, ntpp
    N.call("dsv4_b200_moe_align_block_size", ids.data_ptr() if numel else None, numel, num_experts,
           block_size, sorted_ids.data_ptr(), cap, expert_ids.data_ptr(), n_blocks,
           ntpp.data_ptr(), None, N.stream_of(ids))
    return sorted_ids, expert_ids, ntpp


# tokens up to which the layer quantises by sorted position (every routed
# copy quantised again); above it each token is quantised once and scattered
# through the align's inverse map.  The scatter measured faster at every M
# from 16 to 8192 on B200 (12.2 vs 14.2 us at M=16, 117 vs 566 us at 8192),
# so the per-position form is left to explicit callers.
_FUSED_QUANT_SORT_MAX_TOKENS = 0

# ids from which moe_align_block_size runs the multi-CTA kernel
_ALIGN_COOP_MIN_IDS = 8192


_moe_align_block_size = moe_align_block_size


def mxfp4_int8_moe_forward(hidden_states: torch.Tensor, weights: Mxfp4Int8MoeWeights,
                           topk_ids: torch.Tensor, topk_weights: torch.Tensor, *, hidden_size: int,
                           intermediate_size: int, routed_scaling_factor: float | None = None,
                           clamp_limit: float | None = None,
                           apply_router_weight_on_input: bool = False) -> torch.Tensor:
    """PYMOE:880-959.  Launches: align, quant fused with the sort into expert
    order, W13 GEMM with fused SwiGLU,
    quant, W2 GEMM, top-k combine with the routed scaling fused."""
    if apply_router_weight_on_input:
        raise NotImplementedError(
            "mxfp4_int8 MoE only supports router weights in the W2 reduce path")
    if hidden_states.dtype != torch.bfloat16:
        hidden_states = hidden_states.to(torch.bfloat16)
    hidden_states = hidden_states.contiguous()
    _require_cuda(hidden_states, "hidden_states")
    topk_ids_i32 = topk_ids.to(torch.int32).contiguous()
    topk_weights_f32 = topk_weights.to(torch.float32).contiguous()
    m = hidden_states.shape[0]
    topk = topk_ids_i32.shape[1]
    experts = weights.w13_mxfp4.shape[0]
    _, block_n = _select_moe_tile_shape(m, topk, experts)
    block_m = select_sorted_block_m(m, topk, experts)
    slot_pos = None
    if m > _FUSED_QUANT_SORT_MAX_TOKENS:
        sorted_ids, expert_ids, ntpp, slot_pos = moe_align_block_size(
            topk_ids_i32, block_m, experts, return_slot_pos=True)
    else:
        sorted_ids, expert_ids, ntpp = moe_align_block_size(topk_ids_i32, block_m, experts)
    return _moe_core(None, None, weights, topk_ids_i32, topk_weights_f32, sorted_ids,
                     expert_ids, ntpp, block_m=block_m, block_n=block_n, hidden_size=hidden_size,
                     intermediate_size=intermediate_size,
                     routed_scaling_factor=routed_scaling_factor, clamp_limit=clamp_limit,
                     masked=False, hidden=hidden_states, slot_pos=slot_pos)


def mxfp4_int8_moe_forward_from_logits(hidden_states: torch.Tensor,
                                       weights: Mxfp4Int8MoeWeights,
                                       router_logits: torch.Tensor, topk: int, *,
                                       hidden_size: int, intermediate_size: int,
                                       router_bias: torch.Tensor | None = None,
                                       renormalize: bool = True,
                                       routed_scaling_factor: float | None = None,
                                       clamp_limit: float | None = None):
    """The MoE layer from router logits: routing and expert align in one fused
    launch (:func:`router_align`), then the same launches as
    :func:`mxfp4_int8_moe_forward`.  Returns ``(out, topk_ids, topk_weights)``."""
    if hidden_states.dtype != torch.bfloat16:
        hidden_states = hidden_states.to(torch.bfloat16)
    hidden_states = hidden_states.contiguous()
    _require_cuda(hidden_states, "hidden_states")
    m = hidden_states.shape[0]
    experts = weights.w13_mxfp4.shape[0]
    _, block_n = _select_moe_tile_shape(m, topk, experts)
    block_m = select_sorted_block_m(m, topk, experts)
    scatter = m > _FUSED_QUANT_SORT_MAX_TOKENS
    ids, w, sorted_ids, expert_ids, ntpp, *rest = router_align(
        router_logits, topk, block_m, bias=router_bias, renormalize=renormalize,
        return_slot_pos=scatter)
    out = _moe_core(None, None, weights, ids, w, sorted_ids, expert_ids, ntpp,
                    block_m=block_m, block_n=block_n, hidden_size=hidden_size,
                    intermediate_size=intermediate_size,
                    routed_scaling_factor=routed_scaling_factor, clamp_limit=clamp_limit,
                    masked=False, hidden=hidden_states, slot_pos=rest[0] if rest else None)
    return out, ids, w


def _moe_core(a13_q, a13_scale, weights, topk_ids_i32, topk_weights_f32, sorted_ids, expert_ids,
              ntpp, *, block_m, block_n, hidden_size, intermediate_size, routed_scaling_factor,
              clamp_limit, masked, hidden=None, slot_pos=None):
    """W13 + SwiGLU, requantisation and W2 of mxfp4_int8_moe_forward
    (PYMOE:904-958) on expert-sorted rows: the routed token rows are copied
    once into the order of the aligned permutation (K-chunk-major), so each
    GEMM stage loads its token tile with one tensor-map copy.  Same results as
    the slot-addressed JIT entry points, bit for bit."""
    m = (hidden if hidden is not None else a13_q).shape[0]
    topk = topk_ids_i32.shape[1]
    dev = topk_ids_i32.device
    nv = m * topk
    kw = dict(hidden_size=hidden_size, intermediate_size=intermediate_size, topk=topk,
              block_m=block_m, num_valid_tokens=nv)
    if hidden is not None and m <= _FUSED_QUANT_SORT_MAX_TOKENS:
        # few tokens: quantise and sort in one launch (each routed copy of a
        # token is quantised again; cheap at decode, not at prefill)
        a13, s13, r13 = quantize_sort_int8(hidden, sorted_ids, ntpp, topk=topk,
                                           num_valid_tokens=nv)
    elif hidden is not None and slot_pos is not None:
        # many tokens: quantise each token once and scatter its routed copies
        # to their sorted positions (the inverse map from the align)
        a13, s13, r13 = quantize_scatter_int8(hidden, slot_pos, sorted_ids.numel(), topk=topk,
                                              num_valid_tokens=nv)
    else:
        if hidden is not None:
            a13_q, a13_scale = quantize_per_token_int8(hidden, 0.0)
        a13, s13, r13 = moe_sort_rows(a13_q, a13_scale, sorted_ids, ntpp, topk=topk,
                                      num_valid_tokens=nv)
    inter = torch.empty((sorted_ids.numel(), intermediate_size), device=dev, dtype=torch.bfloat16)
    mxfp4_int8_moe_gemm_swiglu_sorted(a13, s13, r13, weights.w13_mxfp4, weights.w13_shift2,
                                      weights.w13_channel_scale, inter, sorted_ids, expert_ids,
                                      ntpp, clamp_limit=clamp_limit, **kw)
    a2, s2, r2 = quantize_sorted_int8(inter, sorted_ids, ntpp, num_valid_tokens=nv)
    out = torch.empty((m, hidden_size), device=dev, dtype=torch.bfloat16)
    routed_out = torch.empty((nv, hidden_size), device=dev, dtype=torch.bfloat16)
    mxfp4_int8_moe_gemm_sorted(a2, s2, r2, weights.w2_mxfp4, weights.w2_shift2,
                               weights.w2_channel_scale, routed_out, sorted_ids, expert_ids, ntpp,
                               **kw)
    if masked:
        apply = routed_scaling_factor is not None and routed_scaling_factor != 1.0
        N.call("dsv4_b200_mxfp4_int8_moe_reduce_masked", routed_out.data_ptr(),
               topk_weights_f32.data_ptr(), topk_ids_i32.data_ptr(), out.data_ptr(), m,
               hidden_size, topk, m * topk, 1 if apply else 0,
               float(routed_scaling_factor) if apply else 1.0, N.stream_of(out))
    else:
        mxfp4_int8_moe_reduce(routed_out, topk_weights_f32, out, hidden_size=hidden_size,
                              intermediate_size=intermediate_size, topk=topk,
                              block_m=min(block_m, _MAX_BLOCK_M),  # validated only
                              block_n=block_n, num_valid_tokens=m * topk,
                              routed_scaling_factor=routed_scaling_factor)
    return out


def mxfp4_int8_moe_forward_quantized(a_q: torch.Tensor, a_scale: torch.Tensor,
                                     weights: Mxfp4Int8MoeWeights, topk_ids: torch.Tensor,
                                     topk_weights: torch.Tensor, *, hidden_size: int,
                                     intermediate_size: int,
                                     routed_scaling_factor: float | None = None,
                                     clamp_limit: float | None = None,
                                     expected_routes: int | None = None) -> torch.Tensor:
    """MoE layer on rows that are already INT8-quantised (``a_q``, ``a_scale``),
    as they arrive from the expert-parallel dispatch.  ``topk_ids`` index the
    local experts of ``weights``; negative ids (experts held by other ranks)
    contribute nothing.  Same arithmetic as mxfp4_int8_moe_forward.
    ``expected_routes``: the number of valid (id >= 0) routes the caller
    expects, for the token-tile choice when many rows are padding (the exact
    count would need a host synchronisation); default: every route."""
    _require_cuda(a_q, "a_q")
    ids = topk_ids.to(torch.int32).contiguous()
    w = topk_weights.to(torch.float32).contiguous()
    m, topk = ids.shape
    experts = weights.w13_mxfp4.shape[0]
    if m == 0:
        return torch.empty((0, hidden_size), device=a_q.device, dtype=torch.bfloat16)
    m_sel = m if expected_routes is None else max(1, -(-int(expected_routes) // topk))
    _, block_n = _select_moe_tile_shape(m_sel, topk, experts)
    block_m = select_sorted_block_m(m_sel, topk, experts)
    sorted_ids, expert_ids, ntpp = moe_align_block_size(ids, block_m, experts)
    return _moe_core(a_q, a_scale, weights, ids, w, sorted_ids,
                     expert_ids, ntpp, block_m=block_m, block_n=block_n, hidden_size=hidden_size,
                     intermediate_size=intermediate_size,
                     routed_scaling_factor=routed_scaling_factor, clamp_limit=clamp_limit,
                     masked=True)


class Mxfp4Int8MoeGraph:
    """:func:`mxfp4_int8_moe_forward` for a fixed token count, captured once
    into a CUDA graph and replayed: the serving form of the decode layer (the
    reference runs under SGLang's CUDA-graph decode, where the layer's host
    work is paid at capture, not per step).  The launches, kernels and
    results are those of :func:`mxfp4_int8_moe_forward`, bit for bit.

    Inputs live in static device buffers (``hidden_states``, ``topk_ids``,
    ``topk_weights``): write them, or pass tensors to :meth:`__call__`, which
    copies them in on the current stream.  The output is the static tensor
    ``out``, overwritten by the next replay."""

    def __init__(self, weights: Mxfp4Int8MoeWeights, num_tokens: int, topk: int, *,
                 hidden_size: int, intermediate_size: int,
                 routed_scaling_factor: float | None = None,
                 clamp_limit: float | None = None, device=None):
        if num_tokens < 1:
            raise ValueError("num_tokens must be positive")
        dev = torch.device(device) if device is not None else weights.w13_mxfp4.device
        _require_cuda(weights.w13_mxfp4, "weights")
        self.num_tokens, self.topk = num_tokens, topk
        self.hidden_states = torch.zeros((num_tokens, hidden_size), dtype=torch.bfloat16,
                                         device=dev)
        # any valid routing for the capture (the graph holds no routing)
        experts = weights.w13_mxfp4.shape[0]
        self.topk_ids = (torch.arange(num_tokens * topk, device=dev, dtype=torch.int32)
                         % experts).view(num_tokens, topk)
        self.topk_weights = torch.full((num_tokens, topk), 1.0 / topk, dtype=torch.float32,
                                       device=dev)
        kw = dict(hidden_size=hidden_size, intermediate_size=intermediate_size,
                  routed_scaling_factor=routed_scaling_factor, clamp_limit=clamp_limit)

        def fwd():
            return mxfp4_int8_moe_forward(self.hidden_states, weights, self.topk_ids,
                                          self.topk_weights, **kw)

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):  # loads the library, warms the allocator
                fwd()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = fwd()

    def __call__(self, hidden_states: torch.Tensor | None = None,
                 topk_ids: torch.Tensor | None = None,
                 topk_weights: torch.Tensor | None = None) -> torch.Tensor:
        if hidden_states is not None:
            self.hidden_states.copy_(hidden_states, non_blocking=True)
        if topk_ids is not None:
            self.topk_ids.copy_(topk_ids, non_blocking=True)
        if topk_weights is not None:
            self.topk_weights.copy_(topk_weights, non_blocking=True)
        self.graph.replay()
        return self.out
