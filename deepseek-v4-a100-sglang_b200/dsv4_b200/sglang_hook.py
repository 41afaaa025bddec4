"""SGLang MoE-method hook: routes ``Mxfp4MarlinMoEMethod`` through the B200
MXFP4 x INT8 kernels.

Mirrors the reference's ``_patch_dsv4_mxfp4_moe_a100`` (PATCH:450-581): at
weight-load time the layer's MXFP4 experts are repacked once
(``prepare_mxfp4_int8_moe``); at run time ``apply`` runs the whole routed-MoE
layer (``mxfp4_int8_moe_forward``) on the dispatcher's hidden states and
standard top-k output and hands the result back as a
``StandardCombineInput``.  There is no silent fallback: a layer that was not
prepared, a non-standard top-k format or another backend raises.

Usage inside an SGLang process (before the model is built)::

    from dsv4_b200 import sglang_hook
    sglang_hook.install()

SGLang itself is imported only inside ``install`` / ``apply`` so that the
module can be imported (and tested) without it.
"""

from __future__ import annotations

import os
from collections import namedtuple

import torch

from ._native import check_device_status
from .mxfp4_int8_moe import mxfp4_int8_moe_forward, prepare_mxfp4_int8_moe

BACKEND_TAG = "b200_mxfp4_int8"
_BACKEND_ENV = "SGLANG_DSV4_MXFP4_MOE_BACKEND"
_HEADROOM_ENV = "SGLANG_DSV4_MXFP4_INT8_HEADROOM_BITS"

# Used when SGLang's StandardCombineInput cannot be imported (tests, tools).
CombineInput = namedtuple("CombineInput", ["hidden_states"])


def _backend() -> str:
    """PATCH:455 (``mxfp4_int8`` default; ``int8`` / ``cutlass`` are aliases).
    The reference's ``ogs`` comparison backend is not provided here."""
    name = os.environ.get(_BACKEND_ENV, "mxfp4_int8").strip().lower()
    if name not in {"mxfp4_int8", "int8", "cutlass"}:
        raise ValueError(f"{_BACKEND_ENV} must be 'mxfp4_int8' on B200 "
                         f"(the OGS backend is not provided), got {name!r}")
    return name


def _config(method):
    runner = getattr(method, "runner", None)
    return getattr(runner, "config", None)


def process_weights_after_loading(method, layer: torch.nn.Module) -> None:
    """PATCH:457-499: let the wrapped FP8/marlin method finish its own
    post-processing, then repack W13/W2 for the INT8 tensor-core kernels."""
    _backend()
    inner = getattr(method, "_fp8", None)
    if inner is not None:
        inner.process_weights_after_loading(layer)
    if getattr(layer, "_mega_moe_weights_built", False):
        raise RuntimeError("the B200 MXFP4 MoE hook does not support prebuilt MegaMoE weights")
    layer.w13_weight.data = layer.w13_weight.data.view(torch.int8)
    layer.w2_weight.data = layer.w2_weight.data.view(torch.int8)
    headroom_bits = int(os.environ.get(_HEADROOM_ENV, "3"))
    cfg = _config(method)
    topk = int(cfg.num_experts_per_tok) if hasattr(cfg, "num_experts_per_tok") else None
    prepare_mxfp4_int8_moe(layer, headroom_bits=headroom_bits, topk=topk)
    layer._dsv4_mxfp4_backend = BACKEND_TAG


def _is_standard_topk(topk_output) -> bool:
    try:
        from sglang.srt.layers.moe.topk import TopKOutputChecker
    except ImportError:
        fmt = getattr(topk_output, "format", None)
        return fmt is None or getattr(fmt, "name", str(fmt)).lower().endswith("standard")
    return TopKOutputChecker.format_is_standard(topk_output)


def _combine_input(hidden_states):
    try:
        from sglang.srt.layers.moe.token_dispatcher.standard import StandardCombineInput
    except ImportError:
        return CombineInput(hidden_states=hidden_states)
    return StandardCombineInput(hidden_states=hidden_states)


def apply(method, layer: torch.nn.Module, dispatch_output):
    """PATCH:501-565: the routed-MoE layer for one dispatched batch."""
    topk_output = dispatch_output.topk_output
    if not _is_standard_topk(topk_output):
        raise ValueError(f"Unsupported topk output format: {getattr(topk_output, 'format', None)}")
    if getattr(layer, "_dsv4_mxfp4_backend", None) != BACKEND_TAG:
        raise RuntimeError("the B200 MXFP4 MoE layer was not prepared by this hook; "
                           "refusing to fall back to another path")
    weights = layer._dsv4_mxfp4_int8_weights
    hidden_size = int(weights.w2_channel_scale.shape[1])
    intermediate_size = int(weights.w2_mxfp4.shape[1] * 32)
    cfg = _config(method)
    out = mxfp4_int8_moe_forward(
        hidden_states=dispatch_output.hidden_states,
        weights=weights,
        topk_ids=topk_output.topk_ids,
        topk_weights=topk_output.topk_weights,
        hidden_size=hidden_size,
        intermediate_size=intermediate_size,
        routed_scaling_factor=getattr(cfg, "routed_scaling_factor", None),
        clamp_limit=getattr(cfg, "swiglu_limit", None),
        apply_router_weight_on_input=bool(getattr(cfg, "apply_router_weight_on_input", False)),
    )
    if os.environ.get("DSV4_B200_CHECK_STATUS", "0") == "1":
        # synchronises: raises DeviceTimeoutError if a kernel gave up a wait
        check_device_status()
    return _combine_input(out)


def install(method_cls=None) -> type:
    """Replace ``process_weights_after_loading`` and ``apply`` of SGLang's
    ``Mxfp4MarlinMoEMethod`` (or of ``method_cls``) with this hook; the
    original ``apply`` is kept as ``_sglang_original_apply`` (PATCH:567-576).
    Idempotent.  Raises ImportError when SGLang is absent and no class is
    given."""
    if method_cls is None:
        from sglang.srt.layers.quantization import mxfp4_marlin_moe
        method_cls = mxfp4_marlin_moe.Mxfp4MarlinMoEMethod
    _backend()
    if not hasattr(method_cls, "_sglang_original_apply"):
        method_cls._sglang_original_apply = method_cls.apply
    method_cls.process_weights_after_loading = process_weights_after_loading
    method_cls.apply = apply
    return method_cls
