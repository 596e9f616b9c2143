"""Expert-parallel exchange for ExpertParallelMoE.

``forward_global_dp`` keeps the reference's cross-DP algorithm
(nanovllm/layers/moe.py:942-1018: all-gather every replica's tokens, route the
global batch on every rank, reduce partial outputs) with the native kernels.

``forward_all_to_all_nvlink`` is the B200 replacement: each rank routes only
its own tokens, then
  1. capacity: per-expert route counts of every rank are all-gathered so each
     route's capacity position is its position in the global (rank-major,
     token-major, slot-minor) order the reference uses, and the dropped set
     is the reference's;
  2. dispatch: NCCL all-to-all of each token once per destination rank that
     owns one of its kept routes, plus one 16-byte record per kept route;
  3. the destination runs the packed local pipeline over received routes;
  4. return: NCCL all-to-all of one bf16 row per route, in received order;
  5. the source combines its routes in slot order, the same arithmetic as
     EP=1 (so the output does not depend on the EP size).
Split sizes need host values, so this path synchronises; under CUDA-graph
capture it switches to the graph-safe all-gather exchange.
"""

from __future__ import annotations

import itertools

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _lib
from . import dist_env


def _prefix(values: list[int]) -> list[int]:
    return [0] + list(itertools.accumulate(values))[:-1]


def forward_global_dp(layer, hidden_states: torch.Tensor, reduce_scatter_output: bool
                      ) -> torch.Tensor:
    tp_size = dist_env.get_tp_world_size()
    if layer.ep_size % tp_size:
        raise RuntimeError("global DP MoE group must contain complete TP replicas")
    local_tokens = hidden_states.size(0)
    ctx = dist_env.get_context()
    counts = ctx.moe_token_counts
    dp_rank = layer.ep_rank // tp_size
    if counts is not None:
        if (len(counts) != layer.ep_size // tp_size
                or any(type(c) is not int or c < 0 for c in counts)):
            raise ValueError("MoE token counts must cover every DP replica")
        if local_tokens != counts[dp_rank] and not (
                counts[dp_rank] == 0 and ctx.is_dummy and local_tokens == 1):
            raise ValueError("MoE local token count does not match coordinated batch")
    padded = max(1, max(counts)) if counts is not None else local_tokens
    payload = (hidden_states if padded == local_tokens
               else F.pad(hidden_states, (0, 0, 0, padded - local_tokens)))
    group = dist_env.get_moe_group()
    gathered = torch.empty((layer.ep_size * padded, layer.hidden_size),
                           dtype=hidden_states.dtype, device=hidden_states.device)
    dist.all_gather_into_tensor(gathered, payload.contiguous(), group=group)
    layer.ep_all_gather_count += 1
    replicas = gathered.view(layer.ep_size, padded, layer.hidden_size)[::tp_size]
    # Padding is transport-only: dummy rows must not consume expert capacity.
    all_tokens = (replicas.reshape(-1, layer.hidden_size) if counts is None
                  else torch.cat([r[:c] for r, c in zip(replicas, counts)]))
    output = layer._forward_local(all_tokens)
    if counts is not None:
        output = torch.cat([F.pad(part, (0, 0, 0, padded - c))
                            for part, c in zip(output.split(list(counts)), counts)])
    if reduce_scatter_output:
        if output.numel() % layer.ep_size:
            raise RuntimeError("MoE output cannot be split across global EP ranks")
        shard = torch.empty(output.numel() // layer.ep_size, dtype=output.dtype,
                            device=output.device)
        dist.reduce_scatter_tensor(shard, output.contiguous().view(-1), group=group)
        layer.ep_reduce_scatter_count += 1
        if tp_size == 1:
            result = shard.view(padded, layer.hidden_size)
        else:
            replica = torch.empty(tp_size * shard.numel(), dtype=output.dtype,
                                  device=output.device)
            dist.all_gather_into_tensor(replica, shard, group=dist_env.get_tp_group())
            layer.ep_all_gather_count += 1
            result = replica.view(padded, layer.hidden_size)
    else:
        dist.all_reduce(output, group=group)
        layer.ep_all_reduce_count += 1
        result = output.narrow(0, dp_rank * padded, padded)
    if counts is not None and counts[dp_rank] == 0:
        return torch.zeros_like(hidden_states)
    return result[:local_tokens]


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


def forward_all_to_all_nvlink(layer, hidden_states: torch.Tensor) -> torch.Tensor:
    if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
        # Variable split sizes need host values; capture uses the fixed-shape exchange.
        return forward_global_dp(layer, hidden_states, reduce_scatter_output=True)
    output = _exchange(layer, hidden_states)
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
