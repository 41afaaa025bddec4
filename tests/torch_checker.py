"""Device-side checker for parity at production shapes.

TEST INFRASTRUCTURE ONLY.  The numpy oracle (oracle/mxfp4_int8_oracle.py)
decodes and multiplies on the host; at the benchmarked shapes (256 experts of
7168 x 4096, 65,536 routed rows) that takes far too long.  This module restates
the same integer algorithm in torch so it runs on whichever device holds the
tensors (the GPU in the `-m gpu` tests):

* ``decode_repacked``    the repacked MXFP4 -> int8 decode
                          (reference CORE:36-70, PYMOE:290-333),
* ``moe_gemm_bf16``      per-expert int8 x int8 GEMM, exact in float64
                          (|acc| < 2^31 << 2^53), then the reference epilogue
                          ``bf16((f32(acc) * a_scale) * cs)`` (MOE_CORE:229-237),
* ``quantize_rows``      per-token INT8 quant (PYMOE:53-126),
* ``swiglu_bf16``        PYMOE:872-877 with the reference's bf16 rounding points,
* ``moe_reduce_bf16``    the k-ordered fma combine (MOE_ENTRY:71-126) + rsf.

It is pinned against the numpy oracle on small inputs by
``tests/test_torch_checker.py`` (runs on CPU), so a bit-exact match against it
at full size is a bit-exact match against the oracle's algorithm.
It is never the thing measured and the product never imports it.
"""

from __future__ import annotations

import torch

_MAG_X2 = (0, 1, 2, 3, 4, 6, 8, 12)


def decode_repacked(b_mxfp4: torch.Tensor, b_shift2: torch.Tensor, n: int) -> torch.Tensor:
    """[E, KB, NG8, 128] codes + [E, SS, NG8, 8] shifts -> int8 weights [E, N, K]."""
    b = b_mxfp4.to(torch.int32)
    e, kb, ng8, _ = b.shape
    k = kb * 32
    lanes = b.view(e, kb, ng8, 8, 4, 4)  # [E, KB, NG8, r, t, j]
    codes = torch.zeros((e, kb, ng8, 8, 32), dtype=torch.int32, device=b.device)
    for t in range(4):
        for j in range(4):
            kk = (4 * t if j < 2 else 16 + 4 * t) + 2 * (j & 1)
            byte = lanes[..., t, j]
            codes[..., kk] = byte & 15
            codes[..., kk + 1] = byte >> 4
    codes = codes.permute(0, 2, 3, 1, 4).reshape(e, ng8 * 8, k)[:, :n]
    sh = b_shift2.to(torch.int32)
    kbi = torch.arange(kb, device=b.device)
    sb = sh[:, kbi // 4]  # [E, KB, NG8, 8]
    shifts = (sb >> ((kbi % 4) * 2).view(1, kb, 1, 1)) & 3
    shifts = shifts.permute(0, 2, 3, 1).reshape(e, ng8 * 8, kb)[:, :n]
    lut = torch.tensor(_MAG_X2, dtype=torch.int32, device=b.device)
    mag = lut[codes & 7] << shifts.repeat_interleave(32, dim=2)
    return torch.where((codes & 8) != 0, -mag, mag).to(torch.int8)


def _bf16_epilogue(acc_f64: torch.Tensor, a_scale: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
    v = acc_f64.to(torch.float32) * a_scale.to(torch.float32)
    v = v * cs.to(torch.float32)
    return v.to(torch.bfloat16)


def moe_gemm_bf16(a_q, a_scale, b_mxfp4, b_shift2, cs, sorted_ids, expert_ids, ntpp, *,
                  block_m, topk, num_valid, source_rows_are_slots, out_rows=None,
                  by_position=False):
    """Grouped GEMM of the aligned permutation, one expert at a time.

    Rows: ``a_q[src]`` with src = slot (W2), slot // topk (W13), or, with
    ``by_position``, the sorted position itself (``a_q`` then holds one row per
    position of ``sorted_ids``, as the expert-sorted pipeline lays it out).
    Output row = slot, or the sorted position when ``by_position``.  Returns
    bf16 [out_rows, N] (rows nobody writes stay 0) and a bool mask of written rows.
    """
    dev = a_q.device
    n = cs.shape[1]
    total = int(ntpp.reshape(-1)[0].item())
    nb = total // block_m
    ids = sorted_ids[:nb * block_m].to(torch.int64)
    blk_e = expert_ids[:nb].to(torch.int64).repeat_interleave(block_m)
    pos = torch.arange(nb * block_m, device=dev)
    ok = (ids >= 0) & (ids < num_valid) & (blk_e >= 0)
    if out_rows is None:
        out_rows = sorted_ids.numel() if by_position else num_valid
    out = torch.zeros((out_rows, n), dtype=torch.bfloat16, device=dev)
    written = torch.zeros((out_rows,), dtype=torch.bool, device=dev)
    for e in torch.unique(blk_e[ok]).tolist():
        sel = ok & (blk_e == e)
        slots, p = ids[sel], pos[sel]
        if by_position:
            src = p
        else:
            src = slots if source_rows_are_slots else slots // topk
        w = decode_repacked(b_mxfp4[e:e + 1], b_shift2[e:e + 1], n)[0].to(torch.float64)
        acc = a_q[src].to(torch.float64) @ w.T
        assert acc.abs().max().item() < 2 ** 31
        row = p if by_position else slots
        out[row] = _bf16_epilogue(acc, a_scale[src][:, None], cs[e][None, :])
        written[row] = True
    return out, written


def dense_gemm_i32(a_q, b_mxfp4, b_shift2, n):
    w = decode_repacked(b_mxfp4[None], b_shift2[None], n)[0].to(torch.float64)
    acc = a_q.to(torch.float64) @ w.T
    assert acc.abs().max().item() < 2 ** 31
    return acc.to(torch.int64)


def dense_gemm_bf16(a_q, a_scale, b_mxfp4, b_shift2, cs):
    acc = dense_gemm_i32(a_q, b_mxfp4, b_shift2, cs.shape[0]).to(torch.float64)
    return _bf16_epilogue(acc, a_scale[:, None], cs[None, :])


def quantize_rows(x: torch.Tensor):
    """scale = max|x| / 127 (0 -> 1), q = clamp(rne(x / scale), -127, 127)."""
    xf = x.to(torch.float32)
    amax = xf.abs().amax(dim=1)
    # a tensor divisor: torch turns division by a Python scalar into a
    # multiplication by its reciprocal on CUDA, which is not IEEE division
    scale = amax / torch.full_like(amax, 127.0)
    scale = torch.where(amax == 0, torch.ones_like(scale), scale)
    q = torch.round(xf / scale[:, None]).clamp(-127, 127).to(torch.int8)
    return q, scale


def swiglu_bf16(gate_up: torch.Tensor, inter: int) -> torch.Tensor:
    g = gate_up[:, :inter].to(torch.float32)
    u = gate_up[:, inter:2 * inter].to(torch.float32)
    s = (g / (1.0 + torch.exp(-g))).to(torch.bfloat16).to(torch.float32)
    return (s * u).to(torch.bfloat16)


def _fma_f32(a, b, c):
    return (a.to(torch.float64) * b.to(torch.float64) + c.to(torch.float64)).to(torch.float32)


def moe_reduce_bf16(routed: torch.Tensor, topk_weights: torch.Tensor, m_out: int, topk: int,
                    num_valid: int, rsf=None) -> torch.Tensor:
    r = routed.to(torch.float32)
    w = topk_weights.reshape(-1).to(torch.float32)
    acc = torch.zeros((m_out, r.shape[1]), dtype=torch.float32, device=r.device)
    t = torch.arange(m_out, device=r.device)
    for k in range(topk):
        slots = t * topk + k
        okk = slots < num_valid
        sl = slots.clamp(max=max(num_valid - 1, 0))
        acc = torch.where(okk[:, None], _fma_f32(r[sl], w[sl][:, None], acc), acc)
    out = acc.to(torch.bfloat16)
    if rsf is not None and rsf != 1.0:
        out = (out.to(torch.float32) * rsf).to(torch.bfloat16)
    return out
