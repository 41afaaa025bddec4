"""The inverse permutation recorded by the multi-CTA align and the fused
router + align, and the quantise-scatter that uses it: the same K-chunk-major
rows, scales and row sums as the quantise-and-sort (per sorted position),
bit for bit, with ragged sizes, dropped ids and num_valid below m * topk."""

import pytest
import torch

import gen_inputs as G

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import dsv4_b200 as D
    import dsv4_b200.jit_ops as J

DEV = "cuda"


def _ids(m, e, topk, seed, drop):
    gen = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(e, generator=gen)[:topk] for _ in range(m)]) \
        if m else torch.empty((0, topk), dtype=torch.int64)
    ids = ids.to(torch.int32)
    if drop and m:
        ids[::7, 0] = -1          # outside [0, E): dropped by the align
        ids[1::11, -1] = e + 3
    return ids


def _check_inverse(sorted_ids, ntpp, slot_pos, numel):
    n = int(ntpp.item())
    s = sorted_ids[:n].long()
    placed = s < numel
    inv = torch.full((numel,), -1, dtype=torch.int64, device=DEV)
    inv[s[placed]] = torch.nonzero(placed).reshape(-1)
    assert torch.equal(slot_pos.long(), inv)


@pytest.mark.parametrize("m,e,topk,k,bm,dtype,drop,nv_cut", [
    (1, 8, 2, 128, 16, torch.bfloat16, False, 0),
    (37, 16, 4, 256, 32, torch.float16, True, 0),
    (513, 256, 8, 7168, 256, torch.bfloat16, False, 0),
    (3000, 256, 8, 2048, 128, torch.bfloat16, True, 5),
    (1200, 64, 6, 7168, 192, torch.float16, False, 3),
    (2048, 1024, 8, 4096, 64, torch.bfloat16, True, 0),
])
def test_quantize_scatter_matches_quantize_sort(m, e, topk, k, bm, dtype, drop, nv_cut):
    ids = _ids(m, e, topk, 100 + m, drop).to(DEV)
    x = G.randn_bf16((m, k), 200 + m).to(dtype).to(DEV)
    numel = m * topk
    nv = numel - nv_cut
    s, eid, n, spos = D.moe_align_block_size(ids, bm, e, return_slot_pos=True)
    rs, reid, rn = D.moe_align_block_size(ids.to(torch.int32), bm, e)
    torch.cuda.synchronize()
    assert torch.equal(s, rs) and torch.equal(eid, reid) and torch.equal(n, rn)
    _check_inverse(s, n, spos, numel)
    cap = s.numel()
    q, sc, rsum = J.quantize_scatter_int8(x, spos, cap, topk=topk, num_valid_tokens=nv)
    fq, fsc, frs = J.quantize_sort_int8(x, s, n, topk=topk, num_valid_tokens=nv)
    torch.cuda.synchronize()
    sl = s.long()
    valid = (torch.arange(cap, device=DEV) < int(n.item())) & (sl < nv)
    rows = q.view(k // 128, cap, 128).permute(1, 0, 2).reshape(cap, k)
    frows = fq.view(k // 128, cap, 128).permute(1, 0, 2).reshape(cap, k)
    assert int(valid.sum()) > 0
    assert torch.equal(rows[valid], frows[valid])
    assert torch.equal(sc[valid].view(torch.int32), fsc[valid].view(torch.int32))
    assert torch.equal(rsum[valid], frs[valid])
    assert D.check_device_status() == 0


@pytest.mark.parametrize("m,e,topk,bm", [(1, 256, 8, 16), (700, 256, 8, 64), (9000, 64, 4, 256)])
def test_router_align_slot_pos_is_inverse(m, e, topk, bm):
    gen = torch.Generator().manual_seed(m)
    logits = torch.randn(m, e, generator=gen).to(DEV)
    ids, w, s, eid, n, spos = D.router_align(logits, topk, bm, return_slot_pos=True)
    ids2, w2, s2, eid2, n2 = D.router_align(logits, topk, bm)
    torch.cuda.synchronize()
    assert torch.equal(s, s2) and torch.equal(ids, ids2) and torch.equal(n, n2)
    _check_inverse(s, n, spos, m * topk)


def test_forward_paths_agree_around_scatter_threshold():
    """The layer's two ways in: quantise by sorted position (tokens up to
    _FUSED_QUANT_SORT_MAX_TOKENS) and quantise once + scatter (above it, the
    default for every M): the same output bit for bit."""
    import dsv4_b200.mxfp4_int8_moe as MM
    e, t, h, i, topk = 16, 600, 256, 128, 8
    ws = []
    for n_, k_, seed in ((2 * i, h, 5), (h, i, 6)):
        w, sc = G.make_random_packed_mxfp4(e, n_, k_, seed, exp_range=(-8, -4))
        ws.extend(D.remap_mxfp4_weight_for_int8(w.to(DEV), sc.to(DEV)))
    wts = D.Mxfp4Int8MoeWeights(*ws, 3)
    x = G.randn_bf16((t, h), 12).to(DEV)
    ids = _ids(t, e, topk, 9, False).to(DEV)
    tw = torch.softmax(torch.randn(t, topk, generator=torch.Generator().manual_seed(4)), 1).to(DEV)
    out = D.mxfp4_int8_moe_forward(x, wts, ids, tw, hidden_size=h, intermediate_size=i)
    old = MM._FUSED_QUANT_SORT_MAX_TOKENS
    try:
        MM._FUSED_QUANT_SORT_MAX_TOKENS = 1 << 30
        ref = D.mxfp4_int8_moe_forward(x, wts, ids, tw, hidden_size=h, intermediate_size=i)
    finally:
        MM._FUSED_QUANT_SORT_MAX_TOKENS = old
    assert torch.equal(out, ref)
