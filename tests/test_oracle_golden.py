"""Pins the CPU oracle against outputs of the reference's own code
(tests/golden/*.npz, made by tests/golden/make_golden.py)."""

import numpy as np
import pytest
import torch

from oracle import mxfp4_int8_oracle as O
import gen_inputs as G


@pytest.mark.parametrize("name", ["quant_f32", "quant_f16", "quant_bf16", "quant_clamp"])
def test_quant_matches_reference(golden, name):
    g = golden(name)
    q, s = O.quantize_per_token_int8(g["a"], float(g["clamp"]))
    np.testing.assert_array_equal(q, g["q"])
    np.testing.assert_array_equal(s.view(np.uint32), g["scale"].view(np.uint32))


@pytest.mark.parametrize("name", ["repack_span3", "repack_baseline", "repack_wide"])
@pytest.mark.parametrize("variant", ["tri", "torch"])
def test_repack_matches_reference(golden, name, variant):
    g = golden(name)
    rounding = "half_up" if variant == "tri" else "half_even"
    b, sh, cs = O.remap_mxfp4_weight_for_int8(g["weight"], g["scale"], 3, rounding)
    np.testing.assert_array_equal(b, g[f"{variant}_b"])
    np.testing.assert_array_equal(sh, g[f"{variant}_shift"])
    np.testing.assert_array_equal(cs.view(np.uint32), g[f"{variant}_cs"].view(np.uint32))


def test_repack_variants_diverge_only_for_wide_spans(golden):
    g = golden("repack_span3")
    assert (g["tri_b"] == g["torch_b"]).all()
    g = golden("repack_baseline")
    assert (g["tri_b"] != g["torch_b"]).any()


def test_remap_stats_match_reference(golden):
    g = golden("remap_stats")
    st = O.compute_remap_stats(g["weight"], g["scale"], 3)
    assert st["overflow_count"] == int(g["overflow_count"]) == 0
    assert st["row_span_max"] == int(g["row_span_max"])
    assert abs(st["exact_rate_nonzero"] - float(g["exact_rate_nonzero"])) < 1e-9
    assert abs(st["mean_rel_err_nonzero"] - float(g["mean_rel_err_nonzero"])) < 1e-6
    assert st["exact_rate_nonzero"] > 0.98 and st["mean_rel_err_nonzero"] < 0.02


def test_decode_roundtrip_tracks_original():
    """Decoding the repack reproduces the remapped weights exactly, and the
    remap tracks the original MXFP4 (TEST_MOE:111-120 thresholds)."""
    w, s = G.make_random_packed_mxfp4(2, 24, 128, 3)
    b, sh, cs = O.remap_mxfp4_weight_for_int8(w.numpy(), s.numpy())
    q = O.decode_repacked(b, sh, 24).astype(np.float64) * cs[:, :, None]
    orig = O.dequant_mxfp4_torch(w, s).reshape(2, 24, 128).double().numpy()
    nz = orig != 0
    assert (q[nz] == orig[nz]).mean() > 0.98


def test_float_reference_matches_reference_small(golden):
    g = golden("moe_ref_small")
    x = torch.from_numpy(g["hidden_bits"]).view(torch.bfloat16)
    out = O.mxfp4_moe_reference_torch(
        x, torch.from_numpy(g["w13"]), torch.from_numpy(g["s13"]), torch.from_numpy(g["w2"]),
        torch.from_numpy(g["s2"]), torch.from_numpy(g["topk_ids"]), torch.from_numpy(g["topk_weights"]))
    ref = torch.from_numpy(g["out_bits"]).view(torch.bfloat16)
    assert O.relative_l2(out.float().numpy(), ref.float().numpy()) < 1e-2


def test_oracle_moe_forward_within_reference_tolerance(golden):
    """Integer-path oracle vs the reference's float MoE: rel-L2 < 0.08 (TEST_MOE:258)."""
    g = golden("moe_ref_small")
    weights = {}
    for name, wk, sk in (("w13", "w13", "s13"), ("w2", "w2", "s2")):
        b, sh, cs = O.remap_mxfp4_weight_for_int8(g[wk], g[sk])
        weights[f"{name}_mxfp4"], weights[f"{name}_shift2"], weights[f"{name}_channel_scale"] = b, sh, cs
    out = O.moe_forward(g["hidden_bits"].view(np.uint16), weights, g["topk_ids"], g["topk_weights"],
                        block_m=16)
    ref = O.bf16_bits_to_f32(g["out_bits"].view(np.uint16))
    assert O.relative_l2(O.bf16_bits_to_f32(out), ref) < 0.08


def test_config1_inputs_reproducible_and_oracle_close(golden):
    g = golden("moe_ref_config1")
    e, t, h, i, topk = 8, 16, 1024, 512, 2
    w13, s13 = G.make_random_packed_mxfp4(e, 2 * i, h, 101, exp_range=(-8, -4))
    w2, s2 = G.make_random_packed_mxfp4(e, h, i, 102, exp_range=(-8, -4))
    ids, tw = G.routing_softmax_topk(t, e, topk, 103)
    x = G.randn_bf16((t, h), 104, 1.0)
    import hashlib
    hsh = hashlib.sha256()
    for a in (w13.numpy(), s13.numpy(), w2.numpy(), s2.numpy(), ids.numpy(), tw.numpy(),
              x.view(torch.int16).numpy()):
        hsh.update(np.ascontiguousarray(a).tobytes())
    assert hsh.hexdigest() == str(g["input_sha"])
    weights = {}
    for name, w, s in (("w13", w13, s13), ("w2", w2, s2)):
        b, sh, cs = O.remap_mxfp4_weight_for_int8(w.numpy(), s.numpy())
        weights[f"{name}_mxfp4"], weights[f"{name}_shift2"], weights[f"{name}_channel_scale"] = b, sh, cs
    out = O.moe_forward(x.view(torch.int16).numpy().view(np.uint16), weights, ids.numpy(),
                        tw.numpy(), block_m=16)
    ref = O.bf16_bits_to_f32(g["out_bits"].view(np.uint16))
    assert O.relative_l2(O.bf16_bits_to_f32(out), ref) < 0.08


def test_dense_oracle_within_reference_tolerance(golden):
    g = golden("dense_ref")
    b, sh, cs = O.remap_mxfp4_weight_for_int8(g["weight"][None], g["scale"][None])
    x = O.bf16_bits_to_f32(g["x_bits"].view(np.uint16))
    q, s = O.quantize_per_token_int8(x)
    out = O.dense_gemm(q, s, b[0], sh[0], cs[0])
    ref = O.bf16_bits_to_f32(g["out_bits"].view(np.uint16))
    assert O.relative_l2(O.bf16_bits_to_f32(out), ref) < 0.04


def test_align_oracle_properties():
    rng = np.random.default_rng(0)
    for numel_tokens, e, topk, bm in ((13, 4, 2, 16), (64, 256, 8, 16), (300, 8, 2, 64)):
        ids = rng.integers(0, e, (numel_tokens, topk))
        s, ex, ntp, cum = O.moe_align_block_size(ids, bm, e)
        flat = ids.reshape(-1)
        assert ntp[0] % bm == 0
        for b in range(ntp[0] // bm):
            blk = s[b * bm:(b + 1) * bm]
            v = blk[blk < flat.size]
            assert (flat[v] == ex[b]).all()
            assert (np.diff(v) > 0).all()
        assert sorted(s[s < flat.size].tolist()) == list(range(flat.size))


def test_fma_emulation_known_cases():
    # 1 + 2^-24 is a float32 tie; the exact fma of (1+2^-23)*(1) + 2^-24*(1+eps) rounds up
    a = np.array([1.0], np.float32)
    b = np.array([1.0], np.float32)
    c = np.array([np.float32(2.0**-24)], np.float32)
    assert O.fma_f32(a, b, c)[0] == np.float32(1.0)  # tie to even
    b2 = np.array([np.float32(1.0 + 2.0**-23)], np.float32)
    c2 = np.array([np.float32(-2.0**-24) * np.float32(1.0 - 2.0**-23)], np.float32)
    # exact: 1 + 2^-23 - 2^-24 + 2^-47 -> just above the midpoint -> 1 + 2^-23
    r = O.fma_f32(a, b2, c2)[0]
    exact = 1.0 + 2.0**-23 - 2.0**-24 * (1.0 - 2.0**-23)
    assert r == np.float32(1.0 + 2.0**-23) and exact > 1.0 + 2.0**-24
