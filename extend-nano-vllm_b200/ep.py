"""Expert-parallel exchange for ExpertParallelMoE.

``forward_global_dp`` keeps the reference's cross-DP contract
(nanovllm/layers/moe.py:942-1018: every replica's tokens are exchanged,
every rank routes the global batch, partial outputs are reduced).

``forward_all_to_all_nvlink`` (backend "all_to_all_nvlink") is the B200
replacement: each rank routes only its own tokens and moves rows over NVLink
peer memory (``NvlinkExchange``, kernels in csrc/nvl.cu):
  1. capacity: per-expert route counts of every rank reach every rank, so
     each route's capacity position is its position in the global
     (rank-major, token-major, slot-minor) order the reference uses, and the
     dropped set is the reference's;
  2. dispatch: each token row once per destination rank that owns one of its
     kept routes, plus one 16-byte record per kept route;
  3. the destination runs the packed local pipeline over received routes;
  4. return: one bf16 row per route, written into the source's buffer at the
     route's own index;
  5. the source combines its routes in slot order, the same arithmetic as
     EP=1 (so the output does not depend on the EP size).
Every size that varies stays on the device, so the exchange can be captured
in a CUDA graph.

``_exchange`` is the same algorithm over NCCL all_to_all_single with
variable splits (host-read sizes); the reference's rank-0 experiments
("all_to_all", "all_to_all_reduce", moe.py:1020-1216) run on it.
"""

from __future__ import annotations

import itertools

import torch
import torch.distributed as dist

from . import _lib
from . import dist_env


def _prefix(values: list[int]) -> list[int]:
    return [0] + list(itertools.accumulate(values))[:-1]


def _replica_rows(counts, slot_rows: int, device) -> torch.Tensor:
    """Rows of the gathered buffer that hold real tokens: replica r owns rows
    [r * slot_rows, r * slot_rows + counts[r])."""
    starts = [r * slot_rows for r in range(len(counts))]
    return torch.cat([torch.arange(s, s + c, device=device, dtype=torch.int64)
                      for s, c in zip(starts, counts)])


def forward_global_dp(layer, hidden_states: torch.Tensor, reduce_scatter_output: bool
                      ) -> torch.Tensor:
    """Cross-DP backends "allgather_reduce" / "allgather_reducescatter".

    Contract (nanovllm/layers/moe.py:942-1018, pinned by the reference's
    tests/test_moe_dp_padding.py): every DP replica's tokens are exchanged in
    equal-sized slots (the largest replica's count, at least 1 row; the
    coordinated counts come from the forward context), every rank routes the
    concatenation of all replicas' real tokens (slot padding never takes part
    in routing, so it consumes no expert capacity), computes its local
    experts, and the per-slot partial outputs are summed over the MoE group:
    all-reduce and keep this replica's slot, or reduce-scatter (then an
    all-gather inside the TP group when TP > 1).  A dummy replica (count 0,
    one placeholder row) receives zeros.
    """
    tp_size = dist_env.get_tp_world_size()
    if layer.ep_size % tp_size:
        raise RuntimeError("global DP MoE group must contain complete TP replicas")
    dp_size = layer.ep_size // tp_size
    dp_rank = layer.ep_rank // tp_size
    local_tokens = hidden_states.size(0)
    ctx = dist_env.get_context()
    counts = ctx.moe_token_counts
    if counts is not None:
        if len(counts) != dp_size or any(type(c) is not int or c < 0 for c in counts):
            raise ValueError("MoE token counts must cover every DP replica")
        dummy = counts[dp_rank] == 0 and ctx.is_dummy and local_tokens == 1
        if local_tokens != counts[dp_rank] and not dummy:
            raise ValueError("MoE local token count does not match coordinated batch")
        slot_rows = max(1, max(counts))
    else:
        counts = [local_tokens] * dp_size
        slot_rows = local_tokens
    hidden = layer.hidden_size
    device = hidden_states.device
    group = dist_env.get_moe_group()

    # One slot per MoE rank (TP ranks of a replica send identical slots).
    send = torch.zeros((slot_rows, hidden), dtype=hidden_states.dtype, device=device)
    send[:min(local_tokens, slot_rows)] = hidden_states[:slot_rows]
    slots = torch.empty((layer.ep_size * slot_rows, hidden), dtype=hidden_states.dtype,
                        device=device)
    dist.all_gather_into_tensor(slots, send, group=group)
    layer.ep_all_gather_count += 1
    # Replica r's slot is MoE rank r * tp_size's slot.
    replica_slots = slots.view(dp_size, tp_size, slot_rows, hidden)[:, 0].reshape(-1, hidden)
    rows = _replica_rows(counts, slot_rows, device)
    routed = layer._forward_local(replica_slots.index_select(0, rows))
    partial = torch.zeros((dp_size * slot_rows, hidden), dtype=routed.dtype, device=device)
    partial.index_copy_(0, rows, routed)

    if reduce_scatter_output:
        if partial.numel() % layer.ep_size:
            raise RuntimeError("MoE output cannot be split across global EP ranks")
        piece = torch.empty(partial.numel() // layer.ep_size, dtype=partial.dtype, device=device)
        dist.reduce_scatter_tensor(piece, partial.view(-1), group=group)
        layer.ep_reduce_scatter_count += 1
        if tp_size > 1:
            whole = torch.empty(piece.numel() * tp_size, dtype=partial.dtype, device=device)
            dist.all_gather_into_tensor(whole, piece, group=dist_env.get_tp_group())
            layer.ep_all_gather_count += 1
            piece = whole
        mine = piece.view(slot_rows, hidden)
    else:
        dist.all_reduce(partial, group=group)
        layer.ep_all_reduce_count += 1
        mine = partial.view(dp_size, slot_rows, hidden)[dp_rank]
    if counts[dp_rank] == 0:
        return torch.zeros_like(hidden_states)
    return mine[:local_tokens]


def _exchange(layer, x: torch.Tensor) -> torch.Tensor:
    """Route this rank's tokens and run them through the all-to-all exchange."""
    ops = layer._ops
    group = dist_env.get_moe_group()
    n = layer.ep_size
    num_experts = layer.num_experts
    top_k = layer.top_k
    tokens = x.size(0)
    device = x.device
    hidden = layer.hidden_size

    if tokens:
        layer._check_inputs(x)
        logits = layer.gate(x)
        weights, ids = ops.route_topk(logits, top_k, layer.norm_topk_prob)
    else:
        weights = torch.empty((0, top_k), device=device, dtype=torch.bfloat16)
        ids = torch.empty((0, top_k), device=device, dtype=torch.int64)

    stats = layer._device_stats(device)
    capacity = None
    expert_base = None
    if layer.expert_capacity is not None or layer.expert_capacity_factor is not None:
        # Global capacity positions: routes of lower EP ranks come first.
        hist = torch.zeros(num_experts + 1, device=device, dtype=torch.int32)
        if tokens:
            hist[:num_experts] = ops.expert_histogram(ids, num_experts)
        hist[num_experts] = tokens
        table = torch.empty((n, num_experts + 1), device=device, dtype=torch.int32)
        dist.all_gather_into_tensor(table.view(-1), hist, group=group)
        layer.ep_all_gather_count += 1
        table_host = table.tolist()
        global_tokens = sum(row[num_experts] for row in table_host)
        capacity = layer._capacity(global_tokens)
        rank = layer.ep_rank
        expert_base = table[:rank, :num_experts].sum(dim=0, dtype=torch.int32).contiguous()
    if tokens:
        if capacity is not None:
            # Capacity pass over this rank's routes: rewrites dropped routes in place.
            packed_src = layer._pack(ids.view(-1), weights.view(-1), capacity=capacity,
                                     expert_base=expert_base)
            if stats is not None:
                stats[1] += packed_src.counters[_lib.CNT_DROPPED].to(torch.int64)
        send_token_slot, route_dest_slot, counts = ops.ep_plan(ids, layer._owner_i32, n,
                                                               num_experts)
    else:
        send_token_slot = torch.empty((0, n), device=device, dtype=torch.int32)
        route_dest_slot = torch.empty(0, device=device, dtype=torch.int32)
        counts = torch.zeros(2 * n, device=device, dtype=torch.int32)

    # Counts per destination -> counts per source.
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts.view(n, 2), counts.view(2, n).t().contiguous(),
                           group=group)
    layer.ep_all_to_all_count += 1
    # One device-to-host read for both count vectors.
    host = torch.cat([counts, recv_counts]).tolist()
    send_tok, send_rt = host[:n], host[n:2 * n]
    recv_host = host[2 * n:]
    recv_tok = recv_host[0::2]
    recv_rt = recv_host[1::2]

    # One payload per peer: its token rows, then its 16-byte route records
    # padded to whole rows, so a single all-to-all carries both.
    per_row = hidden * x.element_size() // 16  # route records per row
    send_rows = [send_tok[d] + -(-send_rt[d] // per_row) for d in range(n)]
    recv_rows = [recv_tok[s] + -(-recv_rt[s] // per_row) for s in range(n)]
    send_row0, recv_row0 = _prefix(send_rows), _prefix(recv_rows)
    send_buf = torch.empty((sum(send_rows), hidden), device=device, dtype=x.dtype)
    if tokens:
        ops.ep_pack(x, ids, weights, layer._owner_i32, n, num_experts, send_token_slot,
                    route_dest_slot, send_row0,
                    [(send_row0[d] + send_tok[d]) * per_row for d in range(n)], send_buf,
                    send_buf.view(torch.int32).view(-1, 4))
    recv_buf = torch.empty((sum(recv_rows), hidden), device=device, dtype=x.dtype)
    dist.all_to_all_single(recv_buf, send_buf, recv_rows, send_rows, group=group)
    layer.ep_all_to_all_count += 1
    layer.total_dispatch_token_count += sum(send_tok)

    num_recv = sum(recv_rt)
    if num_recv:
        r_ids, token_of_route, r_w = ops.ep_unpack_routes(
            recv_buf.view(torch.int32).view(-1, 4), n, _prefix(recv_rt) + [num_recv],
            recv_row0, [(recv_row0[s] + recv_tok[s]) * per_row for s in range(n)],
            num_records=num_recv)
        packed = layer._pack(r_ids, None, stats=stats)
        y_local = layer._run_experts(recv_buf, r_w, packed, 1, token_of_route)
    else:
        y_local = torch.empty((0, hidden), device=device, dtype=torch.bfloat16)
    returned = torch.empty((sum(send_rt), hidden), device=device, dtype=torch.bfloat16)
    dist.all_to_all_single(returned, y_local, send_rt, recv_rt, group=group)
    layer.ep_all_to_all_count += 1
    layer.total_assignment_count += ids.numel()
    if not tokens:
        return torch.zeros_like(x)
    combine_rows = ops.ep_return_rows(ids, layer._owner_i32, n, num_experts, route_dest_slot,
                                      _prefix(send_rt), returned.size(0))
    return layer._combine_expert_routes(returned, combine_rows, tokens, top_k)


class NvlinkExchange:
    """One EP rank's part of one layer call over the NVLink peer-memory
    exchange (csrc/nvl.cu), split into the phases of the collective step.

    Within a phase a rank only signals its peers or waits for signals that
    every rank sends in an earlier phase, so the ranks of an exchange can run
    as processes on their own GPUs (forward_all_to_all_nvlink calls the
    phases back to back) or all on one GPU, phase by phase across the ranks.

    Sizes stay on the device under CUDA-graph capture: the received route
    count bounds the packing kernels, and temporaries are sized by the
    host-known bound (the coordinated token counts of the forward context, or
    ep_size times this rank's count: the reference's own contract when no
    counts are given).  Eager calls read the received count once to size
    them exactly.
    """

    def __init__(self, layer, x: torch.Tensor, bufs) -> None:
        self.layer = layer
        self.x = x
        self.bufs = bufs
        self.tokens = x.size(0)
        if self.tokens > bufs.max_tokens:
            raise ValueError(
                f"{self.tokens} tokens exceed the NVLink exchange's max_tokens "
                f"{bufs.max_tokens} (set ExpertParallelMoE.nvl_max_tokens)")
        self.capacity_mode = (layer.expert_capacity is not None
                              or layer.expert_capacity_factor is not None)
        self.capturing = torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()
        self.stats = layer._device_stats(x.device)

    # Phase 1: local routing; with a capacity limit, counts to every peer.
    def route(self) -> None:
        layer, x = self.layer, self.x
        k = layer.top_k
        if self.tokens:
            layer._check_inputs(x)
            self.weights, self.ids = layer._ops.route_topk(layer.gate(x), k,
                                                           layer.norm_topk_prob)
        else:
            self.weights = torch.empty((0, k), device=x.device, dtype=torch.bfloat16)
            self.ids = torch.empty((0, k), device=x.device, dtype=torch.int64)
        if self.capacity_mode:
            layer._ops.nvl_histogram_send(self.ids, self.tokens, k, layer.ep_rank, self.bufs)

    # Phase 2: capacity positions of the global route order, then the
    # per-destination plan and the dispatch of rows and route records.
    def dispatch(self) -> None:
        layer, ops, bufs = self.layer, self.layer._ops, self.bufs
        n, num_experts = layer.ep_size, layer.num_experts
        if self.capacity_mode:
            base, _, cap_dev = ops.nvl_histogram_wait(layer.top_k, layer.ep_rank, bufs,
                                                      layer.expert_capacity_factor)
            if self.tokens:
                fixed = layer.expert_capacity
                packed = layer._pack(self.ids.view(-1), self.weights.view(-1),
                                     capacity=fixed, expert_base=base,
                                     capacity_dev=None if fixed is not None else cap_dev)
                if self.stats is not None:
                    self.stats[1] += packed.counters[_lib.CNT_DROPPED].to(torch.int64)
        if self.tokens:
            slots, route_slots, counts = ops.ep_plan(self.ids, layer._owner_i32, n, num_experts)
            if self.stats is not None:
                self.stats[2] += counts[:n].sum(dtype=torch.int64)
        else:
            slots = route_slots = counts = None
        self.combine_rows = ops.nvl_dispatch(self.x, self.ids, self.weights, layer._owner_i32,
                                             layer.ep_rank, bufs, slots, route_slots, counts,
                                             bump_epoch=not self.capacity_mode)
        layer.ep_all_to_all_count += 1
        layer.total_assignment_count += self.ids.numel()

    def _route_bound(self, assume_equal: bool = True) -> int:
        """Host bound on the routes this rank can receive in this call.
        ``assume_equal``: without coordinated counts or a per-peer bound,
        assume every peer holds as many tokens as this rank (the captured
        graphs' contract); otherwise fall back to the buffer's capacity."""
        layer = self.layer
        counts = dist_env.get_context().moe_token_counts
        peer_cap = getattr(layer, "nvl_graph_peer_tokens", None)
        if counts is not None and len(counts) == layer.ep_size:
            tokens = sum(counts)
        elif peer_cap is not None:
            tokens = self.tokens + (layer.ep_size - 1) * max(int(peer_cap), self.tokens)
        elif assume_equal:
            tokens = layer.ep_size * self.tokens
        else:
            return self.bufs.max_routes
        per_token = min(layer.top_k, layer.num_local_experts)
        return max(1, min(self.bufs.max_routes, tokens * per_token))

    # Phase 3: receive, local expert GEMMs, rows back to their sources.
    def compute(self) -> None:
        layer, ops, bufs = self.layer, self.layer._ops, self.bufs
        ids, token_of_route, weights, src_rank, src_route, count = ops.nvl_receive(
            layer.ep_rank, bufs)
        # Device-side sizes (no host read) under capture, and eagerly when
        # the layer asks for them: the host then never waits for the exchange.
        device_sizes = self.capturing or (getattr(layer, "nvl_eager_device_sizes", False)
                                          and getattr(ops, "NVL_DIRECT_RETURN", False))
        if device_sizes:
            bound = self._route_bound(assume_equal=self.capturing)
            packed = layer._pack(ids[:bound], None, stats=self.stats, route_count=count)
            hint = self.tokens * layer.top_k
            weights = weights[:bound]
            token_of_route = token_of_route[:bound]
        else:
            received = int(count.item())  # one host read per eager call: exact sizes
            packed = layer._pack(ids[:received], None, stats=self.stats)
            hint = None
            weights = weights[:received]
            token_of_route = token_of_route[:received]
        if packed.num_routes and getattr(ops, "NVL_DIRECT_RETURN", False):
            # Rows go to the sources from the down GEMM's epilogue.
            layer._run_experts(bufs.tokens_view(), weights, packed, 1, token_of_route,
                               routes_hint=hint, scatter=(src_rank, src_route, bufs))
            ops.nvl_return_signal(layer.ep_rank, bufs)
        else:
            if packed.num_routes:
                y = layer._run_experts(bufs.tokens_view(), weights, packed, 1, token_of_route,
                                       routes_hint=hint)
            else:
                y = torch.empty((0, layer.hidden_size), device=self.x.device,
                                dtype=torch.bfloat16)
            ops.nvl_return(y, src_rank, src_route, count, layer.ep_rank, bufs)
        layer.ep_all_to_all_count += 1

    # Phase 4: wait for this rank's rows, combine them in slot order.
    def finish(self) -> torch.Tensor:
        layer = self.layer
        layer._ops.nvl_wait_return(layer.ep_rank, self.bufs)
        if not self.tokens:
            return torch.zeros_like(self.x)
        rows = self.tokens * layer.top_k
        return layer._combine_expert_routes(self.bufs.returned_view(rows), self.combine_rows,
                                            self.tokens, layer.top_k)


def forward_all_to_all_nvlink(layer, hidden_states: torch.Tensor) -> torch.Tensor:
    """Backend "all_to_all_nvlink": every rank routes its own tokens and the
    rows move over NVLink peer memory (graph-safe, no host synchronisation
    under capture)."""
    bufs = layer._ops.nvl_buffers(layer, hidden_states.device, dist_env.get_moe_group())
    step = NvlinkExchange(layer, hidden_states, bufs)
    step.route()
    step.dispatch()
    step.compute()
    output = step.finish()
    return output if output.dtype == hidden_states.dtype else output.to(hidden_states.dtype)


def forward_rank0_all_to_all(layer, hidden_states: torch.Tensor, reduce_output: bool
                             ) -> torch.Tensor:
    """The reference's 'all_to_all' / 'all_to_all_reduce' backends
    (moe.py:1020-1216): EP rank 0 routes its tokens, experts run where they
    live, and every rank receives rank 0's result."""
    group = dist_env.get_ep_group()
    source = hidden_states if layer.ep_rank == 0 else hidden_states[:0]
    output = _exchange(layer, source)
    if layer.ep_rank != 0:
        output = torch.empty_like(hidden_states)
    if reduce_output:
        if layer.ep_rank != 0:
            output.zero_()
        dist.all_reduce(output, group=group)
        layer.ep_all_reduce_count += 1
    else:
        dist.broadcast(output, src=dist_env.get_ep_group_ranks()[0], group=group)
        layer.ep_broadcast_count += 1
    return output
