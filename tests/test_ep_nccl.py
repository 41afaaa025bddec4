"""Expert-parallel MoE on 2+ GPUs over NCCL (skipped with fewer GPUs).

Each rank holds E/R experts; the EP output for its tokens is compared with
a single-GPU forward of the same tokens on the full expert set."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import gen_inputs as G

pytestmark = pytest.mark.gpu

E, H, I, TOPK, M = 16, 256, 256, 4, 40


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, mode, zero_rank):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "deepseek-v4-a100-sglang_b200"), os.path.join(root, "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import dsv4_b200 as D
    from dsv4_b200.ep import ExpertParallelMoE, GpuOps
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        dev = torch.device("cuda", rank)
        full = []
        for n, k, seed in ((2 * I, H, 81), (H, I, 82)):
            w, s = G.make_random_packed_mxfp4(E, n, k, seed, exp_range=(-8, -4))
            full.extend(D.remap_mxfp4_weight_for_int8(w.to(dev), s.to(dev)))
        fw = D.Mxfp4Int8MoeWeights(*full, 3)
        e_loc = E // world
        lw = D.Mxfp4Int8MoeWeights(*[t[rank * e_loc:(rank + 1) * e_loc].contiguous() for t in full], 3)
        x = G.randn_bf16((M, H), 500 + rank).to(dev)
        ids, tw = G.routing_sigmoid_bias_topk(M, E, TOPK, 600 + rank)
        ep = ExpertParallelMoE(GpuOps(lw, H, I), num_experts=E, hidden_size=H, routed_scaling_factor=2.0,
                               capacity_tokens=M if mode == "fixed" else None,
                               exact_sizes=(mode == "exact"), timing=True)
        if rank == zero_rank:  # no tokens on this rank this step
            x, ids, tw = x[:0], ids[:0], tw[:0]
        out = ep.forward(x, ids.to(dev), tw.to(dev))
        phases = ep.phase_ms()
        assert set(phases) == set(ep.PHASES)
        D.check_device_status()
        if rank == zero_rank:
            q.put((rank, 0.0 if out.shape == (0, H) else 1.0))
            return
        ref = D.mxfp4_int8_moe_forward(x, fw, ids.to(dev), tw.to(dev), hidden_size=H,
                                       intermediate_size=I, routed_scaling_factor=2.0)
        rel = float((out.float() - ref.float()).norm() / ref.float().norm())
        q.put((rank, rel))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode,zero_rank", [("exact", -1), ("fixed", -1), ("implicit", -1),
                                            ("fixed", 1), ("exact", 0)])
def test_ep_nccl_matches_single_gpu(mode, zero_rank):
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode, zero_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    rels = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, rel in rels:
        assert rel < 1e-2, (rank, rel)
