"""The fused router top-k + expert align (one cooperative launch) against the
two separate launches it replaces: every output bit for bit."""

import pytest
import torch

import gen_inputs as G

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import dsv4_b200 as D

DEV = "cuda"


def _logits(m, e, seed, dtype, zipf):
    gen = torch.Generator()
    gen.manual_seed(seed)
    x = torch.randn(m, e, generator=gen)
    if zipf:
        p = torch.arange(1, e + 1, dtype=torch.float32).pow(-1.1)
        x = x + torch.log(p / p.sum())[torch.randperm(e, generator=gen)]
    return x.to(dtype)


@pytest.mark.parametrize("m,e,topk,bm,dtype,zipf,use_bias", [
    (1, 256, 8, 16, torch.float32, False, True),
    (64, 256, 8, 16, torch.float32, False, True),
    (64, 256, 8, 16, torch.bfloat16, False, False),
    (8192, 256, 8, 256, torch.float32, True, True),
    (5000, 64, 4, 64, torch.float16, False, True),
    (300, 1024, 8, 128, torch.float32, False, True),
    (20000, 256, 8, 128, torch.bfloat16, True, True),
    (0, 256, 8, 16, torch.float32, False, True),
])
def test_router_align_matches_separate_launches(m, e, topk, bm, dtype, zipf, use_bias):
    logits = _logits(max(m, 1), e, 7 + m, dtype, zipf)[:m].to(DEV)
    bias = (torch.randn(e, generator=torch.Generator().manual_seed(3)) * 0.1).to(DEV) \
        if use_bias else None
    ids, w, s, eid, n = D.router_align(logits, topk, bm, bias=bias)
    rids, rw = D.router_topk(logits, topk, bias=bias)
    rs, reid, rn = D.moe_align_block_size(rids, bm, e)
    torch.cuda.synchronize()
    assert torch.equal(ids, rids)
    assert torch.equal(w.view(torch.int32), rw.view(torch.int32))
    assert int(n.item()) == int(rn.item())
    assert torch.equal(s, rs)
    assert torch.equal(eid, reid)
    assert D.check_device_status() == 0


def test_forward_from_logits_matches_forward():
    e, t, h, i, topk = 16, 300, 256, 128, 8
    ws = []
    for n_, k_, seed in ((2 * i, h, 5), (h, i, 6)):
        w, sc = G.make_random_packed_mxfp4(e, n_, k_, seed, exp_range=(-8, -4))
        ws.extend(D.remap_mxfp4_weight_for_int8(w.to(DEV), sc.to(DEV)))
    wts = D.Mxfp4Int8MoeWeights(*ws, 3)
    logits = _logits(t, e, 11, torch.float32, False).to(DEV)
    x = G.randn_bf16((t, h), 12).to(DEV)
    out, ids, w = D.mxfp4_int8_moe_forward_from_logits(x, wts, logits, topk, hidden_size=h,
                                                       intermediate_size=i,
                                                       routed_scaling_factor=2.5)
    ref = D.mxfp4_int8_moe_forward(x, wts, ids, w, hidden_size=h, intermediate_size=i,
                                   routed_scaling_factor=2.5)
    assert torch.equal(out, ref)
