"""Seeded synthetic inputs shared by the golden-fixture script, the tests and
bench.py.  Everything is drawn from CPU ``torch.Generator`` streams so the
same seed gives the same bytes here and on the GPU box.

``make_random_packed_mxfp4`` restates the reference fixture generator
(tests/test_mxfp4_int8_moe.py:25-38: uniform code bytes, UE8M0 scales
``row_base in [122,127] - delta in [0,3]``) and adds the BASELINE form
(exponents uniform in [exp_lo, exp_hi] per 32-K group).
"""

from __future__ import annotations

import torch


def make_random_packed_mxfp4(experts, n, k, seed, *, exp_range=None):
    gen = torch.Generator()
    gen.manual_seed(seed)
    packed = torch.randint(0, 256, (experts, n, k // 2), dtype=torch.uint8, generator=gen)
    if exp_range is None:
        row_base = torch.randint(122, 128, (experts, n, 1), dtype=torch.uint8, generator=gen)
        delta = torch.randint(0, 4, (experts, n, k // 32), dtype=torch.uint8, generator=gen)
        scale = row_base - delta
    else:
        lo, hi = exp_range
        scale = torch.randint(127 + lo, 127 + hi + 1, (experts, n, k // 32),
                              dtype=torch.uint8, generator=gen)
    return packed, scale


def randn_bf16(shape, seed, scale=1.0):
    gen = torch.Generator()
    gen.manual_seed(seed)
    return (torch.randn(shape, generator=gen) * scale).to(torch.bfloat16)


def routing_softmax_topk(tokens, experts, topk, seed):
    """Config-1 routing: top-k of softmax over N(0,1) logits; weights are the
    chosen softmax probabilities (not renormalised)."""
    gen = torch.Generator()
    gen.manual_seed(seed)
    logits = torch.randn(tokens, experts, generator=gen)
    probs = torch.softmax(logits, dim=-1)
    w, ids = torch.topk(probs, topk, dim=-1)
    return ids.to(torch.int32), w.to(torch.float32)


def routing_sigmoid_bias_topk(tokens, experts, topk, seed, *, zipf_s=None, model_seed=None):
    """DeepSeek-style routing: sigmoid scores, per-expert bias N(0, 0.1) used
    for selection only, weights = chosen sigmoid scores renormalised to sum 1.
    With ``zipf_s`` the logits get ``log p_e`` added, ``p_e ~ rank^-s`` over a
    seeded expert permutation (skewed expert popularity).  With
    ``model_seed`` the bias and the popularity permutation (properties of the
    model, shared by every rank) come from that seed and only the logits from
    ``seed``."""
    gen = torch.Generator()
    gen.manual_seed(seed)
    logits = torch.randn(tokens, experts, generator=gen)
    mgen = gen
    if model_seed is not None:
        mgen = torch.Generator()
        mgen.manual_seed(model_seed)
    bias = torch.randn(experts, generator=mgen) * 0.1
    if zipf_s is not None:
        perm = torch.randperm(experts, generator=mgen)
        ranks = torch.empty(experts)
        ranks[perm] = torch.arange(1, experts + 1, dtype=torch.float32)
        p = ranks.pow(-zipf_s)
        p = p / p.sum()
        logits = logits + torch.log(p)[None, :] * 1.0
    scores = torch.sigmoid(logits)
    _, ids = torch.topk(scores + bias[None, :], topk, dim=-1)
    w = torch.gather(scores, 1, ids)
    w = w / w.sum(dim=-1, keepdim=True)
    return ids.to(torch.int32), w.to(torch.float32)


def routing_uniform_topk(tokens, experts, topk, seed):
    """Uniform routing: top-k of sigmoid(N(0,1)) logits with no bias or skew
    (every expert equally likely), weights renormalised to sum 1."""
    gen = torch.Generator()
    gen.manual_seed(seed)
    scores = torch.sigmoid(torch.randn(tokens, experts, generator=gen))
    _, ids = torch.topk(scores, topk, dim=-1)
    w = torch.gather(scores, 1, ids)
    return ids.to(torch.int32), (w / w.sum(dim=-1, keepdim=True)).to(torch.float32)


def round_robin_routing(tokens, experts, topk):
    """Reference test routing (tests/test_mxfp4_int8_moe.py:177-183 for topk=2)."""
    t = torch.arange(tokens, dtype=torch.int32)
    cols = [t % experts, (t * 3 + 1) % experts]
    for j in range(2, topk):
        cols.append((t * (2 * j + 1) + j) % experts)
    return torch.stack(cols[:topk], dim=1)
