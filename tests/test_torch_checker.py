"""Pins the torch checker used by the full-shape GPU parity tests to the numpy
oracle (CPU, small inputs): every function bit for bit."""

import numpy as np
import torch

from oracle import mxfp4_int8_oracle as O
import gen_inputs as G
import torch_checker as TC


def _bits(t):
    return t.view(torch.int16).numpy().view(np.uint16)


def _weights(e, n, k, seed):
    w, s = G.make_random_packed_mxfp4(e, n, k, seed, exp_range=(-8, -4))
    b, sh, cs = O.remap_mxfp4_weight_for_int8(w.numpy(), s.numpy())
    return (b, sh, cs), tuple(torch.from_numpy(x) for x in (b, sh, cs))


def test_decode_matches_oracle():
    (b, sh, cs), (tb, tsh, _) = _weights(3, 72, 320, 5)
    np.testing.assert_array_equal(TC.decode_repacked(tb, tsh, 72).numpy(),
                                  O.decode_repacked(b, sh, 72))


def test_quant_matches_oracle():
    x = G.randn_bf16((37, 512), 3)
    x[0] = 0
    q, s = TC.quantize_rows(x)
    oq, os_ = O.quantize_per_token_int8(x.float().numpy())
    np.testing.assert_array_equal(q.numpy(), oq)
    np.testing.assert_array_equal(s.numpy().view(np.uint32), os_.view(np.uint32))


def test_dense_matches_oracle():
    (b, sh, cs), (tb, tsh, tcs) = _weights(1, 256, 1024, 9)
    x = G.randn_bf16((19, 1024), 4)
    q, s = O.quantize_per_token_int8(x.float().numpy())
    tq, ts = torch.from_numpy(q), torch.from_numpy(s)
    np.testing.assert_array_equal(TC.dense_gemm_i32(tq, tb[0], tsh[0], 256).numpy(),
                                  O.dense_gemm_i32(q, b[0], sh[0], 256))
    np.testing.assert_array_equal(_bits(TC.dense_gemm_bf16(tq, ts, tb[0], tsh[0], tcs[0])),
                                  O.dense_gemm(q, s, b[0], sh[0], cs[0]))


def test_moe_chain_matches_oracle():
    e, t, h, i, topk, bm = 8, 40, 256, 128, 4, 16
    (b13, sh13, cs13), d13 = _weights(e, 2 * i, h, 11)
    (b2, sh2, cs2), d2 = _weights(e, h, i, 12)
    ids, tw = G.routing_sigmoid_bias_topk(t, e, topk, 13)
    x = G.randn_bf16((t, h), 14)
    nv = t * topk
    s_ids, e_ids, ntp, _ = O.moe_align_block_size(ids.numpy(), bm, e)
    ts, te, tn = (torch.from_numpy(np.asarray(v)) for v in (s_ids, e_ids, ntp))
    q, qs = O.quantize_per_token_int8(x.float().numpy())
    gu, _ = TC.moe_gemm_bf16(torch.from_numpy(q), torch.from_numpy(qs), *d13, ts, te, tn,
                             block_m=bm, topk=topk, num_valid=nv, source_rows_are_slots=False)
    ref_gu = O.moe_gemm(q, qs, b13, sh13, cs13, s_ids, e_ids, ntp, block_m=bm, topk=topk,
                        num_valid=nv, source_rows_are_slots=False)
    np.testing.assert_array_equal(_bits(gu), ref_gu)
    inter = TC.swiglu_bf16(gu, i)
    ref_inter = O.swiglu_bf16(ref_gu, i)
    diff = np.abs(_bits(inter).astype(np.int32) - ref_inter.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() <= 0.005
    q2, qs2 = TC.quantize_rows(torch.from_numpy(ref_inter.view(np.int16)).view(torch.bfloat16))
    oq2, oqs2 = O.quantize_per_token_int8(O.bf16_bits_to_f32(ref_inter))
    np.testing.assert_array_equal(q2.numpy(), oq2)
    routed, _ = TC.moe_gemm_bf16(q2, qs2, *d2, ts, te, tn, block_m=bm, topk=topk, num_valid=nv,
                                 source_rows_are_slots=True)
    ref_routed = O.moe_gemm(oq2, oqs2, b2, sh2, cs2, s_ids, e_ids, ntp, block_m=bm, topk=topk,
                            num_valid=nv, source_rows_are_slots=True)
    np.testing.assert_array_equal(_bits(routed), ref_routed)
    out = TC.moe_reduce_bf16(routed, tw, t, topk, nv, 2.5)
    np.testing.assert_array_equal(_bits(out), O.moe_reduce(ref_routed, tw.numpy(), t, topk, nv, 2.5))
