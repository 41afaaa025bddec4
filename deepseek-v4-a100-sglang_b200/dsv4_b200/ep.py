"""Expert-parallel (EP) MXFP4/INT8 MoE across the GPUs of one node.

The reference shards the MoE by tensor parallelism inside SGLang and has no
expert parallelism; this module adds it.  One process per GPU, experts split
contiguously (rank r holds experts [r*E/R, (r+1)*E/R)), tokens owned by the
rank that produced them.  One forward:

1. quantise the local tokens to INT8 (per-token scale);
2. plan and pack (two kernels): for every token, the set of ranks that hold
   at least one of its top-k experts; one packed row is sent per (token,
   destination rank) pair, ordered by destination then token: the INT8 row,
   then its scale, the local expert ids on that rank (-1 elsewhere) and the
   matching router weights;
3. one NCCL all_to_all of the packed rows: fixed-size (every peer gets
   ``capacity`` rows, padding rows carry ids -1; no host synchronisation), or
   exact-size after an all_to_all of the counts read back to the host;
4. every rank runs the grouped MoE on what it received (negative ids are
   skipped), producing one BF16 partial per received row, already summed over
   that rank's experts (router weights applied);
5. NCCL all_to_all of the partials back to their owners;
6. combine: out[t] = bf16(sum over ranks, in rank order, of f32(partial)),
   then the routed scaling.  Deterministic for a fixed world size.

Collective traffic per step: H + 80 bytes per dispatched row (top-8) and 2*H
bytes per returned partial.  Plan, packing and combine are CUDA kernels of
libdsv4_b200; the torch bookkeeping (plan_dispatch, pad_plan) serves the
exact-size mode and test ops without those kernels.
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


def packed_row_bytes(hidden: int, topk: int) -> int:
    """Bytes per packed dispatch row: the int8 row, then the metadata words,
    padded to 16 bytes."""
    return (hidden + 4 * _meta_width(topk) + 15) // 16 * 16


def unpack_rows(buf: torch.Tensor, hidden: int, topk: int):
    """Views of a packed dispatch buffer: (int8 rows [n, H] with the buffer's
    row stride, scale fp32 [n] strided, local ids int32 [n, topk], weights
    fp32 [n, topk]); the ids and weights are small contiguous copies."""
    a_q = buf[:, :hidden].view(torch.int8)
    meta = buf[:, hidden:hidden + 4 * _meta_width(topk)].view(torch.int32)
    scale = meta[:, 0].view(torch.float32)
    lids = meta[:, 1:1 + topk].contiguous()
    w = meta[:, 1 + topk:1 + 2 * topk].contiguous().view(torch.float32)
    return a_q, scale, lids, w


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
            rb = rows.shape[1] * rows.element_size()
            N.call("dsv4_b200_gather_rows", rows.data_ptr() if rows.numel() else None, rb,
                   idx.contiguous().data_ptr(), n, out.data_ptr(), rb, N.stream_of(out))
        return out

    def local_moe(self, a_q, a_scale, lids, w, expected_routes=None):
        from .mxfp4_int8_moe import mxfp4_int8_moe_forward_quantized
        return mxfp4_int8_moe_forward_quantized(a_q, a_scale, self.weights, lids, w,
                                                hidden_size=self.h, intermediate_size=self.i,
                                                clamp_limit=self.clamp,
                                                expected_routes=expected_routes)

    def dispatch_pack(self, a_q, a_scale, topk_ids, topk_weights, num_experts, world, capacity):
        """Device-side plan and packing of the fixed-capacity exchange (two
        kernels, no host synchronisation).  Returns the send buffer uint8
        [world*capacity, row_bytes] (int8 row | metadata words | pad; padding
        rows are zero with expert ids -1) and pos int64 [m, world]."""
        m, topk = topk_ids.shape
        dev = a_q.device
        h = a_q.shape[1]
        row_bytes = packed_row_bytes(h, topk)
        n = world * capacity
        buf = torch.empty((n, row_bytes), dtype=torch.uint8, device=dev)
        send_src = torch.empty((n,), dtype=torch.int64, device=dev)
        pos = torch.empty((m, world), dtype=torch.int64, device=dev)
        ids = topk_ids.to(torch.int32).contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        st = N.stream_of(buf)
        N.call("dsv4_b200_ep_plan_fixed", ids.data_ptr() if m else None,
               w.data_ptr() if m else None, a_scale.data_ptr() if m else None, m, topk,
               num_experts, world, capacity, send_src.data_ptr(), buf.data_ptr() + h,
               _meta_width(topk), row_bytes // 4, pos.data_ptr() if m else None, st)
        if n:
            N.call("dsv4_b200_gather_rows", a_q.data_ptr() if m else None, h, send_src.data_ptr(),
                   n, buf.data_ptr(), row_bytes, st)
        return buf, pos

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

    PHASES = ("pack", "dispatch", "local_moe", "return", "combine")

    def __init__(self, ops, *, num_experts: int, hidden_size: int, group=None,
                 routed_scaling_factor: float | None = None, capacity_tokens: int | None = None,
                 exact_sizes: bool = False, timing: bool = False):
        """Row exchange sizes:

        * default (``exact_sizes=False``): every rank sends ``capacity`` packed
          rows to every peer (padding rows carry expert id -1), so both
          all_to_alls have fixed sizes and the step has no host
          synchronisation.  ``capacity_tokens`` must be >= the tokens of any
          rank's call; ``None`` means this call's token count, which every
          rank must then share.
        * ``exact_sizes=True``: the counts are exchanged first and read back
          to the host, and exactly the needed rows move.

        ``timing=True`` records CUDA events around the phases (pack, dispatch
        all_to_all, local MoE, return all_to_all, combine); see
        :meth:`phase_ms`."""
        self.ops = ops
        self.capacity = capacity_tokens
        self.exact = exact_sizes
        self.num_experts = num_experts
        self.h = hidden_size
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rsf = routed_scaling_factor
        self.timing = timing
        self._events: list = []
        self.last_stats: dict = {}

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                               input_split_sizes=in_splits, group=self.group)

    def _mark(self, evs):
        if evs is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append(e)

    def phase_ms(self, reset: bool = True) -> dict:
        """Mean milliseconds per phase over the timed calls since the last reset."""
        torch.cuda.synchronize()
        out = {k: 0.0 for k in self.PHASES}
        for evs in self._events:
            for k, a, b in zip(self.PHASES, evs[:-1], evs[1:]):
                out[k] += a.elapsed_time(b)
        n = max(len(self._events), 1)
        if reset:
            self._events = []
        return {k: v / n for k, v in out.items()}

    def _pack(self, a_q, a_scale, topk_ids, topk_weights, cap):
        """Packed send rows (int8 row | metadata) and pos [m, world]; exact
        sizes when cap is None (then also the per-peer counts)."""
        m, topk = topk_ids.shape
        if cap is not None and hasattr(self.ops, "dispatch_pack"):
            buf, pos = self.ops.dispatch_pack(a_q, a_scale, topk_ids, topk_weights,
                                              self.num_experts, self.world, cap)
            return buf, pos, None
        # torch bookkeeping (exact sizes, or ops without the packing kernels)
        plan = plan_dispatch(topk_ids, topk_weights, self.num_experts, self.world)
        rb = packed_row_bytes(self.h, topk)
        meta = pack_meta(a_scale[plan.send_token], plan.send_lids, plan.send_w)
        rows = self.ops.gather_rows(a_q, plan.send_token)
        dev = a_q.device
        if cap is None:
            buf = torch.zeros((plan.send_token.numel(), rb), dtype=torch.uint8, device=dev)
            at = slice(None)
        else:
            padded = pad_plan(plan, self.world, cap)
            buf = torch.zeros((self.world * cap, rb), dtype=torch.uint8, device=dev)
            pad_meta = torch.zeros((1, meta.shape[1]), dtype=torch.int32, device=dev)
            pad_meta[:, 1:1 + topk] = -1
            buf[:, self.h:self.h + 4 * meta.shape[1]] = pad_meta.view(torch.uint8)
            at = padded
        buf[at, :self.h] = rows.view(torch.uint8)
        buf[at, self.h:self.h + 4 * meta.shape[1]] = meta.view(torch.uint8)
        return buf, plan.pos, plan.send_counts

    def forward(self, hidden: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor) -> torch.Tensor:
        m, topk = topk_ids.shape
        evs = [] if self.timing else None
        self._mark(evs)
        a_q, a_scale = self.ops.quantize(hidden)
        dev = a_q.device
        cap = None
        if not self.exact:
            cap = self.capacity if self.capacity is not None else m
            if m > cap:
                raise ValueError(f"{m} tokens exceed capacity_tokens={cap}")
        buf, pos, counts = self._pack(a_q, a_scale, topk_ids, topk_weights, cap)
        send_list = recv_list = None
        if cap is None:
            recv_counts = torch.empty_like(counts)
            self._a2a(recv_counts, counts, None, None)
            send_list = counts.tolist()
            recv_list = recv_counts.tolist()
            n_recv = int(sum(recv_list))
        else:
            n_recv = self.world * cap
        n_send = buf.shape[0]
        self._mark(evs)
        # 1. packed rows (int8 row + scale + local ids + weights) in one exchange
        recv = torch.empty((n_recv, buf.shape[1]), dtype=torch.uint8, device=dev)
        self._a2a(recv, buf, recv_list, send_list)
        self._mark(evs)
        r_q, r_scale, r_lids, r_w = unpack_rows(recv, self.h, topk)
        # 2. local experts: one bf16 partial per received row
        # a balanced rank receives about its own token count's worth of routes
        partial = self.ops.local_moe(r_q, r_scale, r_lids, r_w, expected_routes=m * topk)
        self._mark(evs)
        # 3. partials back to their owners, same order as sent
        back = torch.empty((n_send, self.h), dtype=torch.bfloat16, device=dev)
        self._a2a(back, partial.contiguous(), send_list, recv_list)
        self._mark(evs)
        out = self.ops.combine(back, pos, m, self.rsf)
        self._mark(evs)
        if evs is not None:
            self._events.append(evs)
        self.last_stats = {"sent_rows": int(n_send), "recv_rows": int(n_recv),
                           "dispatch_bytes": int(buf.numel()),
                           "combine_bytes": int(back.numel() * 2)}
        return out
