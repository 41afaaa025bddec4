"""CPU-side checks of the C-ABI library: it loads, exports every symbol that
include/dsv4_b200.h declares, and the host-side validation rejects bad
arguments (no GPU needed: validation runs before any device work)."""

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "dsv4_b200.h"


def declared_symbols():
    return sorted(set(re.findall(r"^DSV4_API\s+[\w\s\*]+?\b(dsv4_b200_\w+)\s*\(", HEADER.read_text(), re.M)))


def test_library_exports_every_declared_symbol():
    from dsv4_b200 import _native as N
    lib = N.load()
    syms = declared_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(N.SIGNATURES), "ctypes table out of sync with the header"
    assert lib.dsv4_b200_abi_version() == 2


def test_no_cpu_fallback_for_cpu_tensors():
    import torch
    import dsv4_b200
    with pytest.raises(RuntimeError, match="CUDA"):
        dsv4_b200.quantize_per_token_int8(torch.zeros(4, 8))


def test_template_validation_mirrors_reference():
    import dsv4_b200.jit_ops as J
    with pytest.raises(ValueError, match="topk"):
        J._validate_template_args(128, 128, 9, 16, 128)
    with pytest.raises(ValueError, match="block_m"):
        J._validate_template_args(128, 128, 2, 8, 128)
    with pytest.raises(ValueError, match="block_n"):
        J._validate_template_args(128, 128, 2, 16, 256)
    with pytest.raises(ValueError, match="divisible by 32"):
        J._validate_dense_template_args(100, 128)


def test_tile_policy():
    import dsv4_b200 as D
    assert D.max_mxfp4_int8_moe_block_m(64, 8, 256) == 16
    assert D.max_mxfp4_int8_moe_block_m(8192, 8, 256) == 128
    assert D.select_mxfp4_int8_moe_tile_shape(13, 2, 4)[0] == 16
