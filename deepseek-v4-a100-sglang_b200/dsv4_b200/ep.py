"""Expert-parallel (EP) MXFP4/INT8 MoE across the GPUs of one node.

The reference shards the MoE by tensor parallelism inside SGLang and has no
expert parallelism; this module adds it.  One process per GPU, experts split
contiguously (rank r holds experts [r*E/R, (r+1)*E/R)), tokens owned by the
rank that produced them.  One forward:

1. quantise the local tokens to INT8 (per-token scale);
2. plan: for every token, the set of ranks that hold at least one of its
   top-k experts; one row is sent per (token, destination rank) pair, ordered
   by destination then token, carrying the INT8 row, its scale, the local
   expert ids on that rank (-1 elsewhere) and the matching router weights;
3. NCCL all_to_all of the counts, then of the rows and of the metadata;
4. every rank runs the grouped MoE on what it received (negative ids are
   skipped), producing one BF16 partial per received row, already summed over
   that rank's experts (router weights applied);
5. NCCL all_to_all of the partials back to their owners;
6. combine: out[t] = bf16(sum over ranks, in rank order, of f32(partial)),
   then the routed scaling.  Deterministic for a fixed world size.

Collective traffic per step: H + 4 + 8*topk bytes per dispatched row and 2*H
bytes per returned partial.  The plan (index bookkeeping) is plain torch on
the device; row packing and the combine are CUDA kernels of libdsv4_b200.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native as N


@dataclass
class DispatchPlan:
    send_token: torch.Tensor   # int64 [S]: token of each sent row (dest-major order)
    send_rank: torch.Tensor    # int64 [S]: destination rank of each sent row
    send_counts: torch.Tensor  # int64 [R]
    send_lids: torch.Tensor    # int32 [S, topk]: local expert ids on the destination, -1 = none
    send_w: torch.Tensor       # float32 [S, topk]: router weights (0 where lid < 0)
    pos: torch.Tensor          # int64 [M, R]: row of (token, rank) in the send order, -1 = none


def plan_dispatch(topk_ids: torch.Tensor, topk_weights: torch.Tensor, num_experts: int,
                  world: int) -> DispatchPlan:
    """Routing plan of one rank (device-agnostic torch index logic)."""
    if num_experts % world != 0:
        raise ValueError(f"num_experts={num_experts} must be divisible by world={world}")
    e_loc = num_experts // world
    ids = topk_ids.to(torch.int64)
    m, topk = ids.shape
    valid = (ids >= 0) & (ids < num_experts)
    dest = torch.where(valid, ids // e_loc, torch.full_like(ids, world))
    has = torch.zeros((m, world + 1), dtype=torch.bool, device=ids.device)
    has.scatter_(1, dest, True)
    has = has[:, :world]
    r_idx, t_idx = has.t().nonzero(as_tuple=True)  # dest-major, token ascending
    send_counts = has.sum(dim=0).to(torch.int64)
    mine = dest[t_idx] == r_idx[:, None]
    send_lids = torch.where(mine, ids[t_idx] - r_idx[:, None] * e_loc,
                            torch.full_like(ids[t_idx], -1)).to(torch.int32)
    send_w = torch.where(mine, topk_weights.to(torch.float32)[t_idx],
                         torch.zeros((), dtype=torch.float32, device=ids.device))
    pos = torch.full((m, world), -1, dtype=torch.int64, device=ids.device)
    pos[t_idx, r_idx] = torch.arange(t_idx.numel(), dtype=torch.int64, device=ids.device)
    return DispatchPlan(t_idx, r_idx, send_counts, send_lids.contiguous(), send_w.contiguous(), pos)


def pad_plan(plan: DispatchPlan, world: int, capacity: int) -> torch.Tensor:
    """Fixed-capacity layout: the row for (token, dest) goes to dest*capacity +
    its index among the rows for dest.  Returns the padded position of every
    sent row (int64 [S]); plan.pos is rewritten to padded positions."""
    starts = torch.cumsum(plan.send_counts, 0) - plan.send_counts
    within = torch.arange(plan.send_token.numel(), device=plan.send_token.device) - starts[plan.send_rank]
    padded = plan.send_rank * capacity + within
    valid = plan.pos >= 0
    plan.pos = torch.where(valid, padded[plan.pos.clamp_min(0)], plan.pos)
    return padded


def _meta_width(topk: int) -> int:
    """int32 words per metadata row: scale, topk ids, topk weights, padded to 16 B."""
    w = 1 + 2 * topk
    return (w + 3) // 4 * 4


def pack_meta(scale: torch.Tensor, lids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    n, topk = lids.shape
    meta = torch.zeros((n, _meta_width(topk)), dtype=torch.int32, device=lids.device)
    meta[:, 0] = scale.to(torch.float32).view(torch.int32)
    meta[:, 1:1 + topk] = lids
    meta[:, 1 + topk:1 + 2 * topk] = w.to(torch.float32).view(torch.int32)
    return meta


def unpack_meta(meta: torch.Tensor, topk: int):
    scale = meta[:, 0].contiguous().view(torch.float32)
    lids = meta[:, 1:1 + topk].contiguous()
    w = meta[:, 1 + topk:1 + 2 * topk].contiguous().view(torch.float32)
    return scale, lids, w


class GpuOps:
    """The CUDA data path (libdsv4_b200)."""

    def __init__(self, weights, hidden_size: int, intermediate_size: int, clamp_limit=None):
        self.weights = weights
        self.h = hidden_size
        self.i = intermediate_size
        self.clamp = clamp_limit

    def quantize(self, hidden):
        from .mxfp4_int8_moe import quantize_per_token_int8
        if hidden.dtype != torch.bfloat16:
            hidden = hidden.to(torch.bfloat16)
        return quantize_per_token_int8(hidden.contiguous(), 0.0)

    def gather_rows(self, rows: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        n = idx.numel()
        out = torch.empty((n, rows.shape[1]), dtype=rows.dtype, device=rows.device)
        if n:
            N.call("dsv4_b200_gather_rows", rows.data_ptr(), rows.shape[1] * rows.element_size(),
                   idx.contiguous().data_ptr(), n, out.data_ptr(), N.stream_of(rows))
        return out

    def local_moe(self, a_q, a_scale, lids, w):
        from .mxfp4_int8_moe import mxfp4_int8_moe_forward_quantized
        return mxfp4_int8_moe_forward_quantized(a_q, a_scale, self.weights, lids, w,
                                                hidden_size=self.h, intermediate_size=self.i,
                                                clamp_limit=self.clamp)

    def plan_fixed(self, topk_ids, topk_weights, a_scale, num_experts, world, capacity):
        """Device-side plan of the fixed-capacity exchange (no host sync):
        (send_src int64 [world*cap], send_meta int32 [world*cap, W], pos [m, world])."""
        m, topk = topk_ids.shape
        dev = topk_ids.device
        ids = topk_ids.to(torch.int32).contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        n = world * capacity
        send_src = torch.empty((n,), dtype=torch.int64, device=dev)
        meta = torch.empty((n, _meta_width(topk)), dtype=torch.int32, device=dev)
        pos = torch.empty((m, world), dtype=torch.int64, device=dev)
        N.call("dsv4_b200_ep_plan_fixed", ids.data_ptr() if m else None, w.data_ptr() if m else None,
               a_scale.data_ptr() if m else None, m, topk, num_experts, world, capacity,
               send_src.data_ptr(), meta.data_ptr(), meta.shape[1], pos.data_ptr(), N.stream_of(pos))
        return send_src, meta, pos

    def combine(self, partial, pos, m, rsf):
        out = torch.empty((m, self.h), dtype=torch.bfloat16, device=pos.device)
        apply = rsf is not None and rsf != 1.0
        if m:
            ptr = partial.data_ptr() if partial.numel() else 0
            N.call("dsv4_b200_ep_combine", ptr, pos.contiguous().data_ptr(), pos.shape[1],
                   out.data_ptr(), m, self.h, 1 if apply else 0, float(rsf) if apply else 1.0,
                   N.stream_of(out))
        return out


class ExpertParallelMoE:
    """One rank's share of an expert-parallel MoE layer."""

    def __init__(self, ops, *, num_experts: int, hidden_size: int, group=None,
                 routed_scaling_factor: float | None = None, capacity_tokens: int | None = None):
        """``capacity_tokens``: if set (>= the tokens per call), every rank sends
        exactly that many rows to every peer (padding rows carry expert id -1),
        so the all_to_alls have fixed sizes and need no host synchronisation;
        suited to small decode batches.  Otherwise sizes are exact and the
        counts are read back to the host once per call."""
        self.ops = ops
        self.capacity = capacity_tokens
        self.num_experts = num_experts
        self.h = hidden_size
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rsf = routed_scaling_factor
        self.last_stats: dict = {}

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                               input_split_sizes=in_splits, group=self.group)

    def forward(self, hidden: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor) -> torch.Tensor:
        m, topk = topk_ids.shape
        a_q, a_scale = self.ops.quantize(hidden)
        dev = a_q.device
        send_list = recv_list = None
        if self.capacity is not None:
            if m > self.capacity:
                raise ValueError(f"{m} tokens exceed capacity_tokens={self.capacity}")
            cap = self.capacity
            n_send = n_recv = self.world * cap
            if hasattr(self.ops, "plan_fixed"):
                # device-side plan (one kernel): no host synchronisation in the step
                send_src, meta, pos = self.ops.plan_fixed(topk_ids, topk_weights, a_scale,
                                                          self.num_experts, self.world, cap)
                send_rows = self.ops.gather_rows(a_q, send_src)
            else:
                plan = plan_dispatch(topk_ids, topk_weights, self.num_experts, self.world)
                padded = pad_plan(plan, self.world, cap)
                send_rows = torch.zeros((n_send, a_q.shape[1]), dtype=a_q.dtype, device=dev)
                send_rows[padded] = self.ops.gather_rows(a_q, plan.send_token)
                meta = torch.zeros((n_send, _meta_width(topk)), dtype=torch.int32, device=dev)
                meta[:, 1:1 + topk] = -1
                meta[padded] = pack_meta(a_scale[plan.send_token], plan.send_lids, plan.send_w)
                pos = plan.pos
        else:
            plan = plan_dispatch(topk_ids, topk_weights, self.num_experts, self.world)
            # 1. counts (read back to size the exchange)
            recv_counts = torch.empty_like(plan.send_counts)
            self._a2a(recv_counts, plan.send_counts, None, None)
            send_list = plan.send_counts.tolist()
            recv_list = recv_counts.tolist()
            n_recv = int(sum(recv_list))
            n_send = plan.send_token.numel()
            send_rows = self.ops.gather_rows(a_q, plan.send_token)
            meta = pack_meta(a_scale[plan.send_token], plan.send_lids, plan.send_w)
            pos = plan.pos
        # 2. rows + metadata
        recv_rows = torch.empty((n_recv, a_q.shape[1]), dtype=a_q.dtype, device=dev)
        recv_meta = torch.empty((n_recv, meta.shape[1]), dtype=meta.dtype, device=dev)
        self._a2a(recv_rows, send_rows, recv_list, send_list)
        self._a2a(recv_meta, meta, recv_list, send_list)
        r_scale, r_lids, r_w = unpack_meta(recv_meta, topk)
        # 3. local experts
        partial = self.ops.local_moe(recv_rows, r_scale, r_lids, r_w)
        # 4. partials back to their owners, same order as sent
        back = torch.empty((n_send, self.h), dtype=torch.bfloat16, device=dev)
        self._a2a(back, partial.contiguous(), send_list, recv_list)
        self.last_stats = {"sent_rows": int(n_send), "recv_rows": n_recv,
                           "dispatch_bytes": int(send_rows.numel() + meta.numel() * 4),
                           "combine_bytes": int(back.numel() * 2)}
        return self.ops.combine(back, pos, m, self.rsf)
