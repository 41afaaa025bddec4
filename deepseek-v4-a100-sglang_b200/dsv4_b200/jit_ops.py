"""Raw MoE / dense GEMM ops with the reference's JIT-op signatures.

Mirrors ``dsv4_a100_patch/sglang_jit_patches/mxfp4_int8_moe.py`` (JITMOE) and
``.../mxfp4_int8_dense.py`` (JITDENSE): same names, keyword arguments,
template validation (ValueError) and shape checks (RuntimeError, the
reference's RuntimeCheck).  Nothing is JIT-compiled here: the kernels are in
the prebuilt ``libdsv4_b200.so``; "prewarm" sets their attributes.
"""

from __future__ import annotations

import torch

from . import _native as N


def _default_block_n(block_m: int) -> int:
    """JITMOE:29-32."""
    return 64 if block_m in (32, 64) else 128


def _validate_template_args(hidden_size, intermediate_size, topk, block_m, block_n) -> None:
    """JITMOE:40-57."""
    if hidden_size <= 0 or intermediate_size <= 0:
        raise ValueError(f"hidden_size/intermediate_size must be positive, got "
                         f"{hidden_size}/{intermediate_size}")
    if topk <= 0 or topk > 8:
        raise ValueError(f"topk must be in [1, 8], got {topk}")
    if block_m not in {16, 32, 64, 128}:
        raise ValueError(f"block_m must be 16, 32, 64, or 128, got {block_m}")
    if block_n not in {32, 64, 128}:
        raise ValueError(f"block_n must be 32, 64, or 128, got {block_n}")


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_tensor(t: torch.Tensor, name: str, dtype, shape=None, device=None) -> None:
    _check(t.is_cuda, f"{name} must be a CUDA tensor")
    _check(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")
    _check(t.is_contiguous(), f"{name} must be contiguous")
    if shape is not None:
        _check(tuple(t.shape) == tuple(shape), f"{name} must have shape {tuple(shape)}, "
                                               f"got {tuple(t.shape)}")
    if device is not None:
        _check(t.device == device, f"{name} is on {t.device}, expected {device}")


_initialised: set[int] = set()


def _init_device(device: torch.device) -> None:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _initialised:
        N.call("dsv4_b200_init", idx)
        _initialised.add(idx)


@torch.compiler.disable
def prewarm_mxfp4_int8_moe_jit_modules(*, hidden_size: int, intermediate_size: int, topk: int,
                                       block_ms: tuple[int, ...] = (16, 32, 64),
                                       block_n: int | None = None,
                                       tile_shapes: tuple[tuple[int, int], ...] | None = None) -> None:
    """JITMOE:113-139: validate the template args and set kernel attributes
    (dynamic shared memory) on the current device before graph capture."""
    if tile_shapes is None:
        tile_shapes = tuple((bm, _default_block_n(bm) if block_n is None else block_n)
                            for bm in block_ms)
    for bm, bn in tile_shapes:
        _validate_template_args(hidden_size, intermediate_size, topk, bm, bn)
    _init_device(torch.device("cuda", torch.cuda.current_device()))


@torch.compiler.disable
def prewarm_mxfp4_int8_dense_jit_module(*, k: int, n: int) -> None:
    """JITDENSE:65-69."""
    _validate_dense_template_args(k, n)
    _init_device(torch.device("cuda", torch.cuda.current_device()))


def _moe_common_checks(a_q, a_scale, b_mxfp4, b_shift2, b_channel_scale, sorted_token_ids,
                       expert_ids, num_tokens_post_padded, n, k):
    dev = a_q.device
    _check_tensor(a_q, "a_q", torch.int8, device=dev)
    _check(a_q.dim() == 2 and a_q.shape[1] == k, f"a_q must be [m_in, {k}], got {tuple(a_q.shape)}")
    _check_tensor(a_scale, "a_scale", torch.float32, (a_q.shape[0],), dev)
    _check_tensor(b_mxfp4, "b_mxfp4", torch.uint8, device=dev)
    e = b_mxfp4.shape[0]
    _check(b_mxfp4.dim() == 4 and tuple(b_mxfp4.shape[1:]) == (k // 32, (n + 7) // 8, 128),
           f"b_mxfp4 must be [E, {k // 32}, {(n + 7) // 8}, 128], got {tuple(b_mxfp4.shape)}")
    _check_tensor(b_shift2, "b_shift2", torch.uint8, device=dev)
    _check(b_shift2.dim() == 4 and b_shift2.shape[0] == e and b_shift2.shape[2] == (n + 7) // 8
           and b_shift2.shape[3] == 8 and b_shift2.shape[1] >= (k // 32 + 3) // 4,
           f"b_shift2 shape mismatch {tuple(b_shift2.shape)}")
    _check_tensor(b_channel_scale, "b_channel_scale", torch.float32, (e, n), dev)
    _check_tensor(sorted_token_ids, "sorted_token_ids", torch.int32, device=dev)
    _check_tensor(expert_ids, "expert_ids", torch.int32, device=dev)
    _check_tensor(num_tokens_post_padded, "num_tokens_post_padded", torch.int32, (1,), dev)
    _check(k % 128 == 0, "K must be divisible by 128")
    return e


def mxfp4_int8_moe_gemm(a_q, a_scale, b_mxfp4, b_shift2, b_channel_scale, out, topk_weights,
                        sorted_token_ids, expert_ids, num_tokens_post_padded, *, hidden_size: int,
                        intermediate_size: int, topk: int, block_m: int,
                        source_rows_are_slots: bool, num_valid_tokens: int,
                        routed_out: torch.Tensor | None = None, block_n: int | None = None) -> None:
    """JITMOE:143-192 / MOE_ENTRY:146-272.  W13 (``source_rows_are_slots``
    False) writes ``out`` [num_valid, 2I]; W2 writes ``routed_out``
    [num_valid, H] (``out`` is the later reduce target)."""
    bn = _default_block_n(block_m) if block_n is None else block_n
    _validate_template_args(hidden_size, intermediate_size, topk, block_m, bn)
    if routed_out is None:
        routed_out = out
    n = hidden_size if source_rows_are_slots else 2 * intermediate_size
    k = intermediate_size if source_rows_are_slots else hidden_size
    e = _moe_common_checks(a_q, a_scale, b_mxfp4, b_shift2, b_channel_scale, sorted_token_ids,
                           expert_ids, num_tokens_post_padded, n, k)
    _check_tensor(topk_weights, "topk_weights", torch.float32, device=a_q.device)
    _check(topk_weights.dim() == 2 and topk_weights.shape[1] == topk
           and topk_weights.shape[0] * topk >= num_valid_tokens,
           "topk_weights does not cover routed slots")
    _check_tensor(routed_out, "routed_out", torch.bfloat16, (num_valid_tokens, n), a_q.device)
    if source_rows_are_slots:
        _check(out.dim() == 2 and out.shape[1] == n and out.shape[0] * topk >= num_valid_tokens,
               "W2 output rows do not cover routed slots")
    _init_device(a_q.device)
    N.call("dsv4_b200_mxfp4_int8_moe_gemm", a_q.data_ptr(), a_scale.data_ptr(), a_q.shape[0],
           b_mxfp4.data_ptr(), b_shift2.data_ptr(), b_channel_scale.data_ptr(), e, n, k,
           b_shift2.shape[1], routed_out.data_ptr(), sorted_token_ids.data_ptr(),
           sorted_token_ids.numel(), expert_ids.data_ptr(), expert_ids.numel(),
           num_tokens_post_padded.data_ptr(), topk, block_m, 1 if source_rows_are_slots else 0,
           num_valid_tokens, N.stream_of(a_q))


def mxfp4_int8_moe_gemm_swiglu(a_q, a_scale, b_mxfp4, b_shift2, b_channel_scale, out,
                               sorted_token_ids, expert_ids, num_tokens_post_padded, *,
                               hidden_size: int, intermediate_size: int, topk: int, block_m: int,
                               num_valid_tokens: int, clamp_limit: float | None = None) -> None:
    """W13 GEMM with ``_apply_swiglu`` (PYMOE:872-877) fused into the epilogue:
    ``out`` [num_valid, I] bf16 equals ``_apply_swiglu(gate_up)`` of the
    unfused path."""
    _validate_template_args(hidden_size, intermediate_size, topk, block_m, 128)
    n, k = 2 * intermediate_size, hidden_size
    e = _moe_common_checks(a_q, a_scale, b_mxfp4, b_shift2, b_channel_scale, sorted_token_ids,
                           expert_ids, num_tokens_post_padded, n, k)
    _check_tensor(out, "out", torch.bfloat16, (num_valid_tokens, intermediate_size), a_q.device)
    _init_device(a_q.device)
    N.call("dsv4_b200_mxfp4_int8_moe_gemm_swiglu", a_q.data_ptr(), a_scale.data_ptr(),
           a_q.shape[0], b_mxfp4.data_ptr(), b_shift2.data_ptr(), b_channel_scale.data_ptr(), e,
           intermediate_size, k, b_shift2.shape[1], out.data_ptr(), sorted_token_ids.data_ptr(),
           sorted_token_ids.numel(), expert_ids.data_ptr(), expert_ids.numel(),
           num_tokens_post_padded.data_ptr(), topk, block_m, num_valid_tokens,
           0 if clamp_limit is None else 1, 0.0 if clamp_limit is None else float(clamp_limit),
           N.stream_of(a_q))


# ---- expert-sorted row pipeline (B200 fast path; same arithmetic) ----

def _sorted_bm(block_m: int) -> int:
    """The sorted-row GEMMs also take 192- and 256-token tiles; validate the rest as usual."""
    return 128 if block_m in (192, 256) else block_m


def moe_sort_rows(a_q, a_scale, sorted_token_ids, num_tokens_post_padded, *, topk: int,
                  num_valid_tokens: int, source_rows_are_slots: bool = False):
    """Copy the routed INT8 rows into the order of the aligned permutation:
    returns ``(q, scale, rowsum)`` with ``q`` int8 K-chunk-major
    ``[K/128][sorted_capacity][128]`` (flat), ``scale`` fp32 and ``rowsum``
    int32 (sum of the row's int8 values) ``[sorted_capacity]``; position p
    holds row ``sorted_token_ids[p] // topk`` (or the slot itself).  Padding
    positions are left unwritten.  ``a_q`` may be a row-strided view (rows
    16-byte aligned) and ``a_scale`` a strided 1-D view, as when the rows
    arrive packed with their metadata."""
    _check(a_q.is_cuda and a_q.dtype == torch.int8 and a_q.dim() == 2 and a_q.stride(1) == 1,
           "a_q must be a CUDA int8 [M, K] tensor with unit column stride")
    _check(a_scale.is_cuda and a_scale.dtype == torch.float32 and a_scale.dim() == 1
           and a_scale.shape[0] == a_q.shape[0], "a_scale must be a CUDA fp32 [M] tensor")
    m_in, k = a_q.shape
    lda = a_q.stride(0) if m_in > 1 else k
    cap = sorted_token_ids.numel()
    q = torch.empty(cap * k, device=a_q.device, dtype=torch.int8)
    sc = torch.empty(cap, device=a_q.device, dtype=torch.float32)
    rs = torch.empty(cap, device=a_q.device, dtype=torch.int32)
    _init_device(a_q.device)
    N.call("dsv4_b200_moe_sort_rows", a_q.data_ptr(), a_scale.data_ptr(), m_in, k, lda,
           max(a_scale.stride(0), 1), sorted_token_ids.data_ptr(), cap,
           num_tokens_post_padded.data_ptr(), topk, 1 if source_rows_are_slots else 0,
           num_valid_tokens, q.data_ptr(), sc.data_ptr(), rs.data_ptr(), N.stream_of(a_q))
    return q, sc, rs


def quantize_sort_int8(a, sorted_token_ids, num_tokens_post_padded, *, topk: int,
                       num_valid_tokens: int):
    """Per-token INT8 quantisation of the bf16/fp16 token rows ``a`` [M, K]
    fused with :func:`moe_sort_rows`: position p receives token
    ``sorted_token_ids[p] // topk`` quantised, with its scale and row sum,
    in the K-chunk-major layout.  One launch instead of two."""
    _check(a.dim() == 2 and a.dtype in (torch.bfloat16, torch.float16) and a.is_contiguous(),
           "a must be a contiguous 2-D bf16/fp16 tensor")
    _check(a.is_cuda, "a must be a CUDA tensor (no CPU path)")
    m, k = a.shape
    cap = sorted_token_ids.numel()
    q = torch.empty(cap * k, device=a.device, dtype=torch.int8)
    sc = torch.empty(cap, device=a.device, dtype=torch.float32)
    rs = torch.empty(cap, device=a.device, dtype=torch.int32)
    _init_device(a.device)
    N.call("dsv4_b200_quantize_sort_int8", a.data_ptr(),
           N.DTYPE_BF16 if a.dtype == torch.bfloat16 else N.DTYPE_F16, m, k,
           sorted_token_ids.data_ptr(), cap, num_tokens_post_padded.data_ptr(), topk,
           num_valid_tokens, q.data_ptr(), sc.data_ptr(), rs.data_ptr(), N.stream_of(a))
    return q, sc, rs


def quantize_scatter_int8(a, slot_pos, sorted_capacity: int, *, topk: int,
                          num_valid_tokens: int):
    """Same outputs as :func:`quantize_sort_int8`, computed from the token
    side: each row of ``a`` [M, K] is quantised once and written to the sorted
    position ``slot_pos[t * topk + j]`` of each routed slot (``slot_pos`` from
    :func:`moe_align_block_size` / :func:`router_align` with
    ``return_slot_pos=True``).  For many tokens, where quantising every routed
    copy again would cost topk times the arithmetic."""
    _check(a.dim() == 2 and a.dtype in (torch.bfloat16, torch.float16) and a.is_contiguous(),
           "a must be a contiguous 2-D bf16/fp16 tensor")
    _check(a.is_cuda, "a must be a CUDA tensor (no CPU path)")
    m, k = a.shape
    _check(slot_pos.dtype == torch.int32 and slot_pos.is_contiguous() and
           slot_pos.numel() >= num_valid_tokens, "slot_pos must be int32 [>= num_valid_tokens]")
    cap = int(sorted_capacity)
    q = torch.empty(cap * k, device=a.device, dtype=torch.int8)
    sc = torch.empty(cap, device=a.device, dtype=torch.float32)
    rs = torch.empty(cap, device=a.device, dtype=torch.int32)
    _init_device(a.device)
    N.call("dsv4_b200_quantize_scatter_int8", a.data_ptr(),
           N.DTYPE_BF16 if a.dtype == torch.bfloat16 else N.DTYPE_F16, m, k,
           slot_pos.data_ptr(), topk, num_valid_tokens, cap, q.data_ptr(), sc.data_ptr(),
           rs.data_ptr(), N.stream_of(a))
    return q, sc, rs


def quantize_sorted_int8(a, sorted_token_ids, num_tokens_post_padded, *, num_valid_tokens: int):
    """Per-token INT8 quantisation of sorted-position rows ``a``
    ``[sorted_capacity, K]`` (bf16/fp16) into ``(q, scale, rowsum)`` as
    returned by :func:`moe_sort_rows`."""
    _check(a.dim() == 2 and a.dtype in (torch.bfloat16, torch.float16) and a.is_contiguous(),
           "a must be a contiguous 2-D bf16/fp16 tensor")
    _check(a.is_cuda, "a must be a CUDA tensor (no CPU path)")
    cap, k = a.shape
    _check(cap == sorted_token_ids.numel(), "a must have one row per sorted position")
    q = torch.empty(cap * k, device=a.device, dtype=torch.int8)
    sc = torch.empty(cap, device=a.device, dtype=torch.float32)
    rs = torch.empty(cap, device=a.device, dtype=torch.int32)
    _init_device(a.device)
    N.call("dsv4_b200_quantize_sorted_int8", a.data_ptr(),
           N.DTYPE_BF16 if a.dtype == torch.bfloat16 else N.DTYPE_F16, k,
           sorted_token_ids.data_ptr(), cap, num_tokens_post_padded.data_ptr(),
           num_valid_tokens, q.data_ptr(), sc.data_ptr(), rs.data_ptr(), N.stream_of(a))
    return q, sc, rs


def mxfp4_int8_moe_gemm_swiglu_sorted(a_sorted, a_scale, a_rowsum, b_mxfp4, b_shift2,
                                      b_channel_scale, out,
                                      sorted_token_ids, expert_ids, num_tokens_post_padded, *,
                                      hidden_size: int, intermediate_size: int, topk: int,
                                      block_m: int, num_valid_tokens: int,
                                      clamp_limit: float | None = None) -> None:
    """:func:`mxfp4_int8_moe_gemm_swiglu` on sorted rows: ``out``
    ``[sorted_capacity, I]`` bf16 by sorted position."""
    _validate_template_args(hidden_size, intermediate_size, topk, _sorted_bm(block_m), 128)
    n, k = 2 * intermediate_size, hidden_size
    cap = sorted_token_ids.numel()
    e = _moe_common_checks(a_sorted.view(cap, k), a_scale, b_mxfp4, b_shift2, b_channel_scale,
                           sorted_token_ids, expert_ids, num_tokens_post_padded, n, k)
    _check_tensor(out, "out", torch.bfloat16, (cap, intermediate_size), a_sorted.device)
    _init_device(a_sorted.device)
    _check_tensor(a_rowsum, "a_rowsum", torch.int32, (cap,), a_sorted.device)
    N.call("dsv4_b200_mxfp4_int8_moe_gemm_swiglu_sorted", a_sorted.data_ptr(), a_scale.data_ptr(),
           a_rowsum.data_ptr(), b_mxfp4.data_ptr(), b_shift2.data_ptr(), b_channel_scale.data_ptr(), e,
           intermediate_size, k, b_shift2.shape[1], out.data_ptr(), sorted_token_ids.data_ptr(),
           cap, expert_ids.data_ptr(), expert_ids.numel(), num_tokens_post_padded.data_ptr(), topk,
           block_m, num_valid_tokens, 0 if clamp_limit is None else 1,
           0.0 if clamp_limit is None else float(clamp_limit), N.stream_of(a_sorted))


def mxfp4_int8_moe_gemm_sorted(a_sorted, a_scale, a_rowsum, b_mxfp4, b_shift2, b_channel_scale,
                               routed_out,
                               sorted_token_ids, expert_ids, num_tokens_post_padded, *,
                               hidden_size: int, intermediate_size: int, topk: int, block_m: int,
                               num_valid_tokens: int) -> None:
    """W2 of :func:`mxfp4_int8_moe_gemm` (``source_rows_are_slots``) on
    sorted rows: ``routed_out`` ``[num_valid, H]`` by routed slot."""
    _validate_template_args(hidden_size, intermediate_size, topk, _sorted_bm(block_m), 128)
    n, k = hidden_size, intermediate_size
    cap = sorted_token_ids.numel()
    e = _moe_common_checks(a_sorted.view(cap, k), a_scale, b_mxfp4, b_shift2, b_channel_scale,
                           sorted_token_ids, expert_ids, num_tokens_post_padded, n, k)
    _check_tensor(routed_out, "routed_out", torch.bfloat16, device=a_sorted.device)
    _check(routed_out.dim() == 2 and routed_out.shape[1] == n
           and routed_out.shape[0] >= num_valid_tokens, "routed_out does not cover routed slots")
    _init_device(a_sorted.device)
    _check_tensor(a_rowsum, "a_rowsum", torch.int32, (cap,), a_sorted.device)
    N.call("dsv4_b200_mxfp4_int8_moe_gemm_sorted", a_sorted.data_ptr(), a_scale.data_ptr(),
           a_rowsum.data_ptr(), b_mxfp4.data_ptr(), b_shift2.data_ptr(), b_channel_scale.data_ptr(), e, n, k,
           b_shift2.shape[1], routed_out.data_ptr(), sorted_token_ids.data_ptr(), cap,
           expert_ids.data_ptr(), expert_ids.numel(), num_tokens_post_padded.data_ptr(), topk,
           block_m, num_valid_tokens, N.stream_of(a_sorted))


def mxfp4_int8_moe_reduce(routed_out, topk_weights, out, *, hidden_size: int,
                          intermediate_size: int, topk: int, block_m: int, num_valid_tokens: int,
                          block_n: int | None = None,
                          routed_scaling_factor: float | None = None) -> None:
    """JITMOE:196-225 / MOE_ENTRY:274-321; ``routed_scaling_factor`` fuses the
    ``out.mul_(rsf)`` of PYMOE:957-958."""
    bn = _default_block_n(block_m) if block_n is None else block_n
    _validate_template_args(hidden_size, intermediate_size, topk, block_m, bn)
    n = hidden_size
    _check_tensor(routed_out, "routed_out", torch.bfloat16, device=routed_out.device)
    _check(routed_out.dim() == 2 and routed_out.shape[1] == n
           and routed_out.shape[0] >= num_valid_tokens, "routed_out does not cover valid routed slots")
    _check_tensor(topk_weights, "topk_weights", torch.float32, device=routed_out.device)
    _check(topk_weights.dim() == 2 and topk_weights.shape[1] == topk
           and topk_weights.shape[0] * topk >= num_valid_tokens,
           "topk_weights does not cover routed slots")
    _check_tensor(out, "out", torch.bfloat16, device=routed_out.device)
    _check(out.dim() == 2 and out.shape[1] == n and out.shape[0] * topk >= num_valid_tokens,
           "out rows do not cover routed slots")
    _check(n % 16 == 0, "W2 reduce requires N divisible by 16")
    apply = routed_scaling_factor is not None and routed_scaling_factor != 1.0
    _init_device(out.device)
    N.call("dsv4_b200_mxfp4_int8_moe_reduce", routed_out.data_ptr(), topk_weights.data_ptr(),
           out.data_ptr(), out.shape[0], n, topk, num_valid_tokens, 1 if apply else 0,
           float(routed_scaling_factor) if apply else 1.0, N.stream_of(out))


def _validate_dense_template_args(k: int, n: int) -> None:
    """JITDENSE:29-34."""
    if k <= 0 or n <= 0:
        raise ValueError(f"k/n must be positive, got {k}/{n}")
    if k % 32 != 0:
        raise ValueError(f"k must be divisible by 32, got {k}")
    if k > 64 and k % 64 != 0:
        raise ValueError(f"k must be <= 64 or divisible by 64, got {k}")


def mxfp4_int8_dense_gemm(a_q, a_scale, b_mxfp4, b_shift2, b_channel_scale, out,
                          partial: torch.Tensor | None = None) -> None:
    """JITDENSE:73-108 / DENSE_ENTRY:334-433.  ``partial`` int32
    [splits, M, ceil32(N)] is the split-K workspace used when M <= 128."""
    if a_q.dim() != 2:
        raise ValueError(f"a_q must have shape [M, K], got {tuple(a_q.shape)}")
    m, k = int(a_q.shape[0]), int(a_q.shape[1])
    n = int(b_channel_scale.shape[0])
    _validate_dense_template_args(k, n)
    dev = a_q.device
    _check_tensor(a_q, "a_q", torch.int8, device=dev)
    _check_tensor(a_scale, "a_scale", torch.float32, (m,), dev)
    _check_tensor(b_mxfp4, "b_mxfp4", torch.uint8, (k // 32, (n + 7) // 8, 128), dev)
    _check_tensor(b_shift2, "b_shift2", torch.uint8, device=dev)
    _check(b_shift2.dim() == 3 and b_shift2.shape[1] == (n + 7) // 8 and b_shift2.shape[2] == 8
           and b_shift2.shape[0] >= (k // 32 + 3) // 4, "b_shift2 stride mismatch")
    _check_tensor(b_channel_scale, "b_channel_scale", torch.float32, (n,), dev)
    _check_tensor(out, "out", torch.bfloat16, (m, n), dev)
    acc_ld = (n + 31) // 32 * 32
    if partial is None:
        partial = (torch.empty((4, m, acc_ld), device=dev, dtype=torch.int32) if m <= 128
                   else torch.empty((0,), device=dev, dtype=torch.int32))
    use_partial = m <= 128 and partial.numel() > 0
    if use_partial:
        _check_tensor(partial, "partial", torch.int32, device=dev)
        _check(partial.dim() == 3 and partial.shape[1] == m and partial.shape[2] == acc_ld,
               f"partial must be [splits, {m}, {acc_ld}], got {tuple(partial.shape)}")
    _init_device(dev)
    if use_cm_tile(m, k, n):
        a_cm, rs = rows_to_cm(a_q)
        dense_gemm_cm(a_cm, a_scale, rs, b_mxfp4, b_shift2, b_channel_scale, out)
        return
    N.call("dsv4_b200_mxfp4_int8_dense_gemm", a_q.data_ptr(), a_scale.data_ptr(), m, k,
           b_mxfp4.data_ptr(), b_shift2.data_ptr(), b_shift2.shape[0], b_channel_scale.data_ptr(),
           n, out.data_ptr(), partial.data_ptr() if use_partial else None,
           partial.shape[0] if use_partial else 0, acc_ld, N.stream_of(a_q))


def use_cm_tile(m: int, k: int, n: int) -> bool:
    """Large M runs on the 256-token K-chunk-major tile (above
    ``DSV4_B200_DENSE_CM_MIN_M`` rows, default 128)."""
    import os
    lim = int(os.environ.get("DSV4_B200_DENSE_CM_MIN_M", "128"))
    return m > lim and k % 128 == 0 and n % 128 == 0


def rows_to_cm(a_q):
    """Row-major int8 [M, K] -> (K-chunk-major int8 [K/128 * M * 128], int32 row sums [M])."""
    m, k = a_q.shape
    a_cm = torch.empty(m * k, device=a_q.device, dtype=torch.int8)
    rs = torch.empty(m, device=a_q.device, dtype=torch.int32)
    N.call("dsv4_b200_rows_to_cm", a_q.data_ptr(), m, k, a_q.stride(0), a_cm.data_ptr(),
           rs.data_ptr(), N.stream_of(a_q))
    return a_cm, rs


def quantize_per_token_int8_cm(a):
    """Per-token INT8 quantisation of bf16/fp16 ``a`` [M, K] straight into the
    K-chunk-major layout: ``(a_cm, scale [M], rowsum [M])``."""
    _check(a.dim() == 2 and a.dtype in (torch.bfloat16, torch.float16) and a.is_contiguous(),
           "a must be a contiguous 2-D bf16/fp16 tensor")
    m, k = a.shape
    a_cm = torch.empty(m * k, device=a.device, dtype=torch.int8)
    sc = torch.empty(m, device=a.device, dtype=torch.float32)
    rs = torch.empty(m, device=a.device, dtype=torch.int32)
    _init_device(a.device)
    N.call("dsv4_b200_quantize_per_token_int8_cm", a.data_ptr(),
           N.DTYPE_BF16 if a.dtype == torch.bfloat16 else N.DTYPE_F16, m, k, a_cm.data_ptr(),
           sc.data_ptr(), rs.data_ptr(), N.stream_of(a))
    return a_cm, sc, rs


def dense_gemm_cm(a_cm, a_scale, a_rowsum, b_mxfp4, b_shift2, b_channel_scale, out) -> None:
    """Dense GEMM on K-chunk-major activations (256-token tiles)."""
    m = a_scale.shape[0]
    n = b_channel_scale.shape[0]
    k = b_mxfp4.shape[0] * 32
    _check_tensor(out, "out", torch.bfloat16, (m, n), a_scale.device)
    N.call("dsv4_b200_mxfp4_int8_dense_gemm_cm", a_cm.data_ptr(), a_scale.data_ptr(),
           a_rowsum.data_ptr(), m, k, b_mxfp4.data_ptr(), b_shift2.data_ptr(), b_shift2.shape[0],
           b_channel_scale.data_ptr(), n, out.data_ptr(), N.stream_of(out))


def mxfp4_int8_dense_gemm_i32(a_q, b_mxfp4, b_shift2, n: int) -> torch.Tensor:
    """Raw int32 accumulators ``a_q @ W^T`` of the tensor-core path."""
    m, k = a_q.shape
    acc = torch.empty((m, n), device=a_q.device, dtype=torch.int32)
    _init_device(a_q.device)
    N.call("dsv4_b200_mxfp4_int8_dense_gemm_i32", a_q.data_ptr(), m, k, b_mxfp4.data_ptr(),
           b_shift2.data_ptr(), b_shift2.shape[0], n, acc.data_ptr(), N.stream_of(a_q))
    return acc
