"""Expert-parallel protocol on CPU: world_size 2 over gloo.

The plan, the count/row/metadata/partial all_to_alls and the rank-ordered
combine of dsv4_b200.ep run unchanged; only the per-rank compute uses the CPU
oracle (test-only ops) instead of the CUDA kernels.  The EP output is
compared with the single-process oracle MoE on the union of all ranks'
tokens (BF16 partial sums make it close, not bit-identical), and the plan's
bookkeeping is checked exactly.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mxfp4_int8_oracle as O
import gen_inputs as G

E, H, I, TOPK, M = 8, 128, 128, 4, 12


def _weights():
    out = {}
    for nm, (n, k, seed) in (("w13", (2 * I, H, 71)), ("w2", (H, I, 72))):
        w, s = G.make_random_packed_mxfp4(E, n, k, seed, exp_range=(-8, -4))
        b, sh, cs = O.remap_mxfp4_weight_for_int8(w.numpy(), s.numpy())
        out[f"{nm}_mxfp4"], out[f"{nm}_shift2"], out[f"{nm}_channel_scale"] = b, sh, cs
    return out


def _inputs(rank):
    x = G.randn_bf16((M, H), 300 + rank)
    ids, w = G.routing_softmax_topk(M, E, TOPK, 400 + rank)
    return x, ids, w


class CpuOracleOps:
    """Test-only stand-in for ep.GpuOps, computing with the CPU oracle."""

    def __init__(self, weights_local):
        self.w = weights_local

    def quantize(self, hidden):
        q, s = O.quantize_per_token_int8(hidden.float().numpy())
        return torch.from_numpy(q), torch.from_numpy(s)

    def gather_rows(self, rows, idx):
        return rows.index_select(0, idx).contiguous()

    def local_moe(self, a_q, a_scale, lids, w, expected_routes=None):
        m, topk = lids.shape
        if m == 0:
            return torch.empty((0, H), dtype=torch.bfloat16)
        q, s, ids, wn = a_q.numpy(), a_scale.numpy(), lids.numpy(), w.numpy()
        e_loc = self.w["w13_mxfp4"].shape[0]
        srt, eid, ntp, _ = O.moe_align_block_size(ids, 16, e_loc)
        nv = m * topk
        gu = O.moe_gemm(q, s, self.w["w13_mxfp4"], self.w["w13_shift2"], self.w["w13_channel_scale"],
                        srt, eid, ntp, block_m=16, topk=topk, num_valid=nv, source_rows_are_slots=False)
        inter = O.swiglu_bf16(gu, I)
        q2, s2 = O.quantize_per_token_int8(O.bf16_bits_to_f32(inter))
        routed = O.moe_gemm(q2, s2, self.w["w2_mxfp4"], self.w["w2_shift2"], self.w["w2_channel_scale"],
                            srt, eid, ntp, block_m=16, topk=topk, num_valid=nv, source_rows_are_slots=True)
        out = O.moe_reduce(routed, wn, m, topk, nv)
        return torch.from_numpy(out.view(np.int16)).view(torch.bfloat16)

    def combine(self, partial, pos, m, rsf):
        p = O.bf16_bits_to_f32(partial.view(torch.int16).numpy().view(np.uint16)) if partial.numel() else None
        acc = np.zeros((m, H), np.float32)
        for r in range(pos.shape[1]):
            for t in range(m):
                j = int(pos[t, r])
                if j >= 0:
                    acc[t] = (acc[t] + p[j]).astype(np.float32)
        return torch.from_numpy(O.f32_to_bf16_bits(acc).view(np.int16)).view(torch.bfloat16)


def _worker(rank, world, port, q, mode="fixed", zero_rank=-1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from dsv4_b200.ep import ExpertParallelMoE
        full = _weights()
        e_loc = E // world
        local = {k: v[rank * e_loc:(rank + 1) * e_loc] for k, v in full.items()}
        ep = ExpertParallelMoE(CpuOracleOps(local), num_experts=E, hidden_size=H,
                               capacity_tokens=M if mode == "fixed" else None,
                               exact_sizes=(mode == "exact"))
        x, ids, w = _inputs(rank)
        if rank == zero_rank:  # this rank has no tokens this step
            x, ids, w = x[:0], ids[:0], w[:0]
        out = ep.forward(x, ids, w)
        q.put((rank, out.view(torch.int16).numpy().copy(), ep.last_stats))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_plan_bookkeeping_exact():
    from dsv4_b200.ep import plan_dispatch
    _, ids, w = _inputs(0)
    ids[0, 1] = -1  # a masked route is dropped
    plan = plan_dispatch(ids, w, E, 2)
    seen = set()
    for row in range(plan.send_token.numel()):
        t, r = int(plan.send_token[row]), int(plan.send_rank[row])
        assert plan.pos[t, r] == row
        for k in range(TOPK):
            lid = int(plan.send_lids[row, k])
            if lid >= 0:
                assert int(ids[t, k]) == r * (E // 2) + lid
                assert float(plan.send_w[row, k]) == float(w[t, k])
                seen.add((t, k))
    expect = {(t, k) for t in range(M) for k in range(TOPK) if int(ids[t, k]) >= 0}
    assert seen == expect
    assert int(plan.send_counts.sum()) == plan.send_token.numel()
    assert (plan.send_rank.diff() >= 0).all()


@pytest.mark.parametrize("mode,zero_rank", [("exact", -1), ("fixed", -1), ("implicit", -1),
                                            ("exact", 1), ("fixed", 1), ("fixed", 0)])
def test_ep_world2_matches_single_process_oracle(mode, zero_rank):
    """Packed single-exchange dispatch in every size mode; a rank with zero
    tokens still takes part in every collective (ranks that get no rows)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode, zero_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, out, stats = q.get(timeout=300)
        res[rank] = (out, stats)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = _weights()
    for rank in range(world):
        if rank == zero_rank:
            assert res[rank][0].shape == (0, H)
            continue
        x, ids, w = _inputs(rank)
        ref = O.moe_forward(x.view(torch.int16).numpy().view(np.uint16), full, ids.numpy(), w.numpy(),
                            block_m=16)
        got = O.bf16_bits_to_f32(res[rank][0].view(np.uint16))
        assert O.relative_l2(got, O.bf16_bits_to_f32(ref)) < 1e-2
