"""The CUDA-graph form of the MoE layer (Mxfp4Int8MoeGraph): replays with new
inputs give mxfp4_int8_moe_forward's output bit for bit, at a decode size
(quantise-scatter, single-CTA paths) and a prefill-like size (256-token
tiles, multi-CTA align)."""

import pytest
import torch

import gen_inputs as G

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import dsv4_b200 as D

DEV = "cuda"


@pytest.mark.parametrize("e,t,h,i,topk,rsf", [(16, 64, 512, 256, 8, 2.5),
                                              (8, 1500, 256, 128, 4, None)])
def test_graph_replay_matches_forward(e, t, h, i, topk, rsf):
    ws = []
    for n_, k_, seed in ((2 * i, h, 21), (h, i, 22)):
        w, sc = G.make_random_packed_mxfp4(e, n_, k_, seed, exp_range=(-8, -4))
        ws.extend(D.remap_mxfp4_weight_for_int8(w.to(DEV), sc.to(DEV)))
    wts = D.Mxfp4Int8MoeWeights(*ws, 3)
    runner = D.Mxfp4Int8MoeGraph(wts, t, topk, hidden_size=h, intermediate_size=i,
                                 routed_scaling_factor=rsf)
    for step in range(3):
        gen = torch.Generator().manual_seed(50 + step)
        ids = torch.stack([torch.randperm(e, generator=gen)[:topk] for _ in range(t)])
        ids = ids.to(torch.int32).to(DEV)
        tw = torch.softmax(torch.randn(t, topk, generator=gen), 1).to(DEV)
        x = G.randn_bf16((t, h), 60 + step).to(DEV)
        out = runner(x, ids, tw).clone()
        ref = D.mxfp4_int8_moe_forward(x, wts, ids, tw, hidden_size=h, intermediate_size=i,
                                       routed_scaling_factor=rsf)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), step
    assert D.check_device_status() == 0
