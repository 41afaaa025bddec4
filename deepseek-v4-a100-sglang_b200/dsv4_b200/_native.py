"""ctypes binding of the C ABI in include/dsv4_b200.h (libdsv4_b200.so).

The library is the only compute path: there is no CPU or eager fallback.
Loading fails loudly if the shared library has not been built.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import os

# DSV4_B200_LIB points at another build of the same library (A/B runs of
# build variants); the in-tree build otherwise.
LIB_PATH = Path(os.environ.get("DSV4_B200_LIB") or Path(__file__).with_name("libdsv4_b200.so"))

DSV4_OK = 0
DSV4_ERR_INVALID_ARGUMENT = 1
DSV4_ERR_UNSUPPORTED = 2
DSV4_ERR_CUDA = 3
DSV4_ERR_DEVICE = 4

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float

# name -> argtypes (restype is int status unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "dsv4_b200_abi_version": [],
    "dsv4_b200_last_error": [],
    "dsv4_b200_init": [_I],
    "dsv4_b200_get_device_status": [_P, _I],
    "dsv4_b200_quantize_per_token_int8": [_P, _I, _I64, _I64, _I64, _F, _P, _P, _P],
    "dsv4_b200_remap_mxfp4_weight_for_int8": [_P, _P, _I64, _I64, _I64, _I, _I, _P, _P, _P, _P],
    "dsv4_b200_router_align_workspace_words": [_I64, _I64, _P],
    "dsv4_b200_router_align": [_P, _I, _I64, _I64, _P, _I64, _I, _F, _I64, _P, _P, _P, _I64, _P,
                               _I64, _P, _P, _I64, _P, _P],
    "dsv4_b200_moe_align_workspace_words": [_I64, _I64, _P],
    "dsv4_b200_moe_align_block_size_ws": [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P,
                                          _I64, _P, _P],
    "dsv4_b200_moe_align_block_size": [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P],
    "dsv4_b200_mxfp4_int8_moe_gemm": [_P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _P,
                                      _I64, _P, _I64, _P, _I64, _I64, _I, _I64, _P],
    "dsv4_b200_mxfp4_int8_moe_gemm_swiglu": [_P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _I64,
                                             _P, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I,
                                             _F, _P],
    "dsv4_b200_router_topk": [_P, _I, _I64, _I64, _P, _I64, _I, _F, _P, _P, _P],
    "dsv4_b200_moe_sort_rows": [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _I64, _I, _I64, _P, _P, _P,
                                _P],
    "dsv4_b200_quantize_sort_int8": [_P, _I, _I64, _I64, _P, _I64, _P, _I64, _I64, _P, _P, _P, _P],
    "dsv4_b200_quantize_scatter_int8": [_P, _I, _I64, _I64, _P, _I64, _I64, _I64, _P, _P, _P, _P],
    "dsv4_b200_quantize_sorted_int8": [_P, _I, _I64, _P, _I64, _P, _I64, _P, _P, _P, _P],
    "dsv4_b200_mxfp4_int8_moe_gemm_sorted": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                                             _P, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _P],
    "dsv4_b200_mxfp4_int8_moe_gemm_swiglu_sorted": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64,
                                                    _I64, _P, _P, _I64, _P, _I64, _P, _I64,
                                                    _I64, _I64, _I, _F, _P],
    "dsv4_b200_mxfp4_int8_moe_reduce": [_P, _P, _P, _I64, _I64, _I64, _I64, _I, _F, _P],
    "dsv4_b200_mxfp4_int8_moe_reduce_masked": [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _F, _P],
    "dsv4_b200_gather_rows": [_P, _I64, _P, _I64, _P, _I64, _P],
    "dsv4_b200_ep_plan_fixed": [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _P,
                                _P],
    "dsv4_b200_ep_combine": [_P, _P, _I64, _P, _I64, _I64, _I, _F, _P],
    "dsv4_b200_mxfp4_int8_dense_gemm": [_P, _P, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _P,
                                        _I64, _I64, _P],
    "dsv4_b200_mxfp4_int8_dense_gemm_i32": [_P, _I64, _I64, _P, _P, _I64, _I64, _P, _P],
    "dsv4_b200_quantize_per_token_int8_cm": [_P, _I, _I64, _I64, _P, _P, _P, _P],
    "dsv4_b200_rows_to_cm": [_P, _I64, _I64, _I64, _P, _P, _P],
    "dsv4_b200_mxfp4_int8_dense_gemm_cm": [_P, _P, _P, _I64, _I64, _P, _P, _I64, _P, _I64, _P,
                                           _P],
    "dsv4_b200_mxfp4_int8_dense_gemm_noalloc": [_P, _P, _I64, _I64, _P, _P, _I64, _P, _I64, _P,
                                                _P],
}
_RESTYPES = {"dsv4_b200_last_error": ctypes.c_char_p}

_lib = None
_lock = threading.Lock()


class DeviceTimeoutError(RuntimeError):
    """A kernel abandoned a bounded wait (device status word set)."""


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run "
                    "deepseek-v4-a100-sglang_b200/csrc/build.py (there is no fallback path)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def last_error() -> str:
    return load().dsv4_b200_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc == DSV4_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == DSV4_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc == DSV4_ERR_DEVICE:
        raise DeviceTimeoutError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def device_status(reset: bool = False) -> int:
    v = ctypes.c_int(0)
    call("dsv4_b200_get_device_status", ctypes.byref(v), 1 if reset else 0)
    return v.value


def check_device_status() -> int:
    """Read (and clear) the device status word; raise DeviceTimeoutError if a
    kernel gave up a bounded wait since the last check (its outputs are then
    garbage).  Synchronises with the device: call it at a sync point, e.g.
    after a step, not inside a captured graph."""
    code = device_status(reset=True)
    if code != 0:
        raise DeviceTimeoutError(
            f"a kernel abandoned a bounded wait (device status 0x{code:x}); "
            "results since the last check are invalid")
    return 0


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t) -> int:
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream
