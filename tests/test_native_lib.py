"""CPU-side checks of the C-ABI library: it loads, exports every symbol that
include/dsv4_b200.h declares, and the host-side validation rejects bad
arguments (no GPU needed: validation runs before any device work)."""

import re
from pathlib import Path

import pytest
import torch

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


def test_sorted_tile_policy(monkeypatch):
    import dsv4_b200 as D
    monkeypatch.delenv("SGLANG_DSV4_MXFP4_INT8_BLOCK_M", raising=False)
    # decode: the reference policy's small tile is kept
    assert D.select_sorted_block_m(64, 8, 256) == 16
    # prefill: 8192 x 8 routes over 256 experts = 256 per expert -> 256-token tiles
    assert D.select_sorted_block_m(8192, 8, 256) == 256
    # just below 256 routed tokens per expert: the 128-token tile stays
    assert D.select_sorted_block_m(8160, 8, 256) == 128
    # a forced tile is honoured, never widened
    monkeypatch.setenv("SGLANG_DSV4_MXFP4_INT8_BLOCK_M", "128")
    assert D.select_sorted_block_m(8192, 8, 256) == 128


def test_router_topk_argument_checks():
    import dsv4_b200 as D
    with pytest.raises(ValueError, match="2-D"):
        D.router_topk(torch.zeros(4, dtype=torch.float32), 2)
    with pytest.raises(ValueError, match="2-D"):
        D.router_topk(torch.zeros((4, 8), dtype=torch.int32), 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        D.router_topk(torch.zeros((4, 8), dtype=torch.float32), 2)


@pytest.mark.parametrize("compiler,std,ext", [("gcc", "-std=c99", "c"), ("g++", "-std=c++17", "cpp")])
def test_header_compiles_standalone(tmp_path, compiler, std, ext):
    """include/dsv4_b200.h is a plain C ABI: it compiles on its own as C99
    and as C++17 with every warning an error (what a non-Python host sees)."""
    import shutil
    import subprocess
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} not found")
    src = tmp_path / f"use.{ext}"
    src.write_text('#include "dsv4_b200.h"\nint main(void) { return DSV4_OK; }\n')
    inc = Path(__file__).resolve().parent.parent / "include"
    r = subprocess.run([compiler, std, "-Wall", "-Wextra", "-Werror", "-I", str(inc), "-c",
                        str(src), "-o", str(tmp_path / "use.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
