"""CPU stand-in for ``extend_nano_vllm_b200.ops`` -- TEST INFRASTRUCTURE ONLY.

Implements the same functions with the same tensor contracts on CPU tensors,
using the oracle in ``moe_oracle``, so the layer's host logic (expert-parallel
exchange over gloo, counters, placement) can be tested without a GPU by
assigning an instance to ``layer._ops``.  The product never imports it.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import moe_oracle as mo

ENGINE_STREAM, ENGINE_TCGEN05 = 0, 1


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach()
    if t.dtype == torch.bfloat16:
        return t.float().numpy()
    return t.numpy()


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(mo.bf16_round(a)).to(torch.bfloat16)


@dataclass
class PackedRoutes:
    num_routes: int
    row_capacity: int
    max_mtiles: int
    row_route: torch.Tensor
    route_row: torch.Tensor
    combine_rows: torch.Tensor
    tile_expert: torch.Tensor
    expert_offsets: torch.Tensor
    expert_counts: torch.Tensor
    mtiles: torch.Tensor
    counters: torch.Tensor
    local_ids: np.ndarray
    chunks: torch.Tensor | None = None


class CpuOps:
    """Drop-in for the ops module on CPU tensors (oracle arithmetic)."""

    def route_topk(self, logits, top_k, renormalize):
        w, ids = mo.route_topk(logits.detach().float().numpy(), top_k, renormalize)
        return torch.from_numpy(w).to(torch.bfloat16), torch.from_numpy(ids)

    def pack_routes(self, expert_ids, route_weights, num_experts, num_local_experts, *,
                    local_index=None, expert_start=0, expert_base=None, capacity=None,
                    stats=None, route_count=None, capacity_dev=None):
        flat = expert_ids.view(-1)
        if route_count is not None:
            flat = flat[:int(route_count.reshape(-1)[0])]
            route_weights = None if route_weights is None else route_weights.view(-1)[:flat.numel()]
        if capacity_dev is not None:
            capacity = int(capacity_dev.reshape(-1)[0])
            capacity = None if capacity < 0 else capacity
        dropped = 0
        if capacity is not None:
            w = (route_weights.float().numpy() if route_weights is not None
                 else np.zeros(flat.numel(), dtype=np.float32))
            base = None if expert_base is None else expert_base.numpy()
            w2, ids2, keep = mo.apply_capacity(w, flat.numpy(), num_experts, capacity, base)
            dropped = int((~keep).sum())
            flat.copy_(torch.from_numpy(ids2))
            if route_weights is not None:
                route_weights.copy_(torch.from_numpy(w2).to(torch.bfloat16))
        li = None if local_index is None else local_index.numpy()
        lay = mo.pack(flat.numpy(), num_experts, num_local_experts, expert_start, li)
        R = flat.numel()
        counters = torch.tensor([lay["padded_rows"], len(lay["mtiles"]), lay["local_kept"],
                                 dropped, len(lay["chunks"])], dtype=torch.int32)
        if stats is not None:
            stats[0] += lay["local_kept"]
            stats[1] += dropped
        i32 = lambda a: torch.from_numpy(np.asarray(a, dtype=np.int32))  # noqa: E731
        return PackedRoutes(R, mo.row_capacity(R, num_local_experts), max(1, len(lay["mtiles"])),
                            i32(lay["row_route"]), i32(lay["route_row"]),
                            i32(lay["combine_rows"]), i32(lay["tile_expert"]),
                            i32(lay["expert_offsets"]), i32(lay["expert_counts"]),
                            i32(lay["mtiles"]), counters,
                            mo.local_ids(flat.numpy(), num_experts, num_local_experts,
                                         expert_start, li), i32(lay["chunks"]))

    def expert_histogram(self, expert_ids, num_experts):
        flat = expert_ids.reshape(-1).numpy()
        flat = flat[(flat >= 0) & (flat < num_experts)]
        return torch.from_numpy(np.bincount(flat, minlength=num_experts).astype(np.int32))

    def gather_rows(self, x, packed, top_k, token_of_route=None):
        return None  # the CPU stand-in reads x directly in expert_gate_up

    def expert_gate_up(self, engine, x, x_packed, w13, packed, top_k, token_of_route=None):
        inter = w13.shape[1] // 2
        act = torch.zeros((packed.row_capacity, inter), dtype=torch.bfloat16)
        rows = np.nonzero(packed.row_route.numpy() < packed.num_routes)[0]
        routes = packed.row_route.numpy()[rows]
        toks = (token_of_route.numpy()[routes] if token_of_route is not None
                else routes // top_k)
        experts = packed.local_ids[routes]
        xs = _np(x)
        w = _np(w13)
        for e in np.unique(experts):
            sel = experts == e
            gu = (torch.from_numpy(xs[toks[sel]]) @ torch.from_numpy(w[e]).T).numpy()
            g = mo.bf16_round(gu[:, :inter])
            u = mo.bf16_round(gu[:, inter:])
            s = mo.bf16_round(g / (1.0 + np.exp(-g, dtype=np.float32)))
            act[torch.from_numpy(rows[sel])] = _bf16(s * u)
        return act

    def expert_down(self, engine, act, w2, packed, route_weights, max_expert_rows=0):
        H = w2.shape[1]
        y = torch.zeros((packed.num_routes, H), dtype=torch.bfloat16)
        rows = np.nonzero(packed.row_route.numpy() < packed.num_routes)[0]
        routes = packed.row_route.numpy()[rows]
        experts = packed.local_ids[routes]
        a = _np(act)
        w = _np(w2)
        rw = route_weights.float().numpy()
        for e in np.unique(experts):
            sel = experts == e
            d = (torch.from_numpy(a[rows[sel]]) @ torch.from_numpy(w[e]).T).numpy()
            y[torch.from_numpy(routes[sel])] = _bf16(d * rw[routes[sel]][:, None])
        return y

    def combine(self, y, route_rows, num_tokens, top_k, out_dtype=torch.bfloat16,
                accum_f64=False):
        rows = (np.arange(num_tokens * top_k) if route_rows is None
                else route_rows.numpy().astype(np.int64))
        acc = mo.combine(y.float().numpy(), rows, num_tokens, top_k,
                         np.float64 if accum_f64 else np.float32)
        out = torch.from_numpy(acc)
        return out.to(out_dtype)

    # ---- expert-parallel exchange --------------------------------------
    @staticmethod
    def _dest(ids, owner, n, num_experts):
        ids = ids.reshape(-1)
        valid = (ids >= 0) & (ids < num_experts)
        d = np.where(valid, owner[np.clip(ids, 0, num_experts - 1)], -1)
        return np.where((d >= 0) & (d < n), d, -1)

    def ep_plan(self, expert_ids, owner, ep_size, num_experts):
        T, k = expert_ids.shape
        dest = self._dest(expert_ids.numpy(), owner.numpy(), ep_size, num_experts)
        route_slot = np.full(T * k, -1, dtype=np.int32)
        tok_slot = np.full((T, ep_size), -1, dtype=np.int32)
        rt_counts = np.zeros(ep_size, dtype=np.int32)
        tok_counts = np.zeros(ep_size, dtype=np.int32)
        for r in range(T * k):
            if dest[r] >= 0:
                route_slot[r] = rt_counts[dest[r]]
                rt_counts[dest[r]] += 1
        for t in range(T):
            for d in sorted(set(dest[t * k:(t + 1) * k]) - {-1}):
                tok_slot[t, d] = tok_counts[d]
                tok_counts[d] += 1
        return (torch.from_numpy(tok_slot), torch.from_numpy(route_slot),
                torch.from_numpy(np.concatenate([tok_counts, rt_counts])))

    def ep_pack(self, x, expert_ids, route_weights, owner, ep_size, num_experts,
                send_token_slot, route_dest_slot, token_offsets, route_offsets, send_x,
                send_meta):
        T, k = expert_ids.shape
        dest = self._dest(expert_ids.numpy(), owner.numpy(), ep_size, num_experts)
        tok_slot = send_token_slot.numpy()
        for t in range(T):
            for d in range(ep_size):
                if tok_slot[t, d] >= 0:
                    send_x[token_offsets[d] + tok_slot[t, d]] = x[t]
        bits = route_weights.reshape(-1).view(torch.int16).numpy().astype(np.int32) & 0xFFFF
        ids = expert_ids.reshape(-1).numpy()
        rs = route_dest_slot.numpy()
        for r in range(T * k):
            d = dest[r]
            if d >= 0 and rs[r] >= 0:
                send_meta[route_offsets[d] + rs[r]] = torch.tensor(
                    [int(ids[r]), int(tok_slot[r // k, d]), int(bits[r]), r], dtype=torch.int32)

    def ep_unpack_routes(self, recv_meta, ep_size, recv_route_offsets, recv_token_offsets,
                         recv_meta_starts=None, num_records=None):
        meta = recv_meta.numpy()
        n = meta.shape[0] if num_records is None else int(num_records)
        src = np.searchsorted(np.asarray(recv_route_offsets[1:ep_size]), np.arange(n),
                              side="right")
        if recv_meta_starts is not None:
            pos = (np.asarray(recv_meta_starts)[src]
                   + np.arange(n) - np.asarray(recv_route_offsets)[src])
            meta = meta[pos]
        ids = torch.from_numpy(meta[:, 0].astype(np.int64))
        tor = torch.from_numpy((np.asarray(recv_token_offsets)[src] + meta[:, 1]).astype(np.int32))
        w = torch.from_numpy((meta[:, 2] & 0xFFFF).astype(np.int16)).view(torch.bfloat16)
        return ids, tor, w

    def ep_return_rows(self, expert_ids, owner, ep_size, num_experts, route_dest_slot,
                       route_offsets, num_rows_returned):
        dest = self._dest(expert_ids.numpy(), owner.numpy(), ep_size, num_experts)
        rs = route_dest_slot.numpy()
        off = np.asarray(list(route_offsets) + [0])
        rows = np.where((dest >= 0) & (rs >= 0), off[np.maximum(dest, 0)] + rs, num_rows_returned)
        return torch.from_numpy(rows.astype(np.int32))

    # ---- expert-parallel exchange over peer memory (stand-in transport) ----
    # The NVLink exchange's phases with the same tensor contracts; the rows
    # and records travel through gloo object collectives on the MoE group
    # instead of peer stores, so the layer's host logic runs on CPU ranks.
    def nvl_buffers(self, layer, device, group):
        bufs = getattr(layer, "_cpu_exchange", None)
        if bufs is None:
            bufs = CpuExchange(layer, group)
            layer._cpu_exchange = bufs
        return bufs

    def nvl_histogram_send(self, expert_ids, num_tokens, top_k, rank, bufs):
        import torch.distributed as dist
        flat = expert_ids.reshape(-1).numpy()
        flat = flat[(flat >= 0) & (flat < bufs.num_experts)]
        mine = np.append(np.bincount(flat, minlength=bufs.num_experts), num_tokens)
        everyone = [None] * bufs.ep_size
        dist.all_gather_object(everyone, mine.astype(np.int64), group=bufs.group)
        bufs.hist = np.stack(everyone)

    def nvl_histogram_wait(self, top_k, rank, bufs, capacity_factor):
        import math
        E = bufs.num_experts
        base = torch.from_numpy(bufs.hist[:rank, :E].sum(axis=0).astype(np.int32))
        tokens = int(bufs.hist[:, E].sum())
        cap = (max(1, math.ceil(capacity_factor * tokens * top_k / E))
               if capacity_factor else -1)
        return base, torch.tensor([tokens]), torch.tensor([cap])

    def nvl_dispatch(self, x, expert_ids, route_weights, owner, rank, bufs, send_token_slot,
                     route_dest_slot, counts, bump_epoch):
        import torch.distributed as dist
        T, k = expert_ids.shape
        n = bufs.ep_size
        dest = self._dest(expert_ids.numpy(), owner.numpy(), n, bufs.num_experts)
        payload = {d: ([], []) for d in range(n)}
        combine_rows = np.full(T * k, T * k, dtype=np.int32)
        if T:
            tok_slot = send_token_slot.numpy()
            rs = route_dest_slot.numpy()
            bits = route_weights.reshape(-1).view(torch.int16).numpy().astype(np.int32) & 0xFFFF
            ids = expert_ids.reshape(-1).numpy()
            xs = x.view(torch.int16).numpy()
            for t in range(T):
                for d in range(n):
                    if tok_slot[t, d] >= 0:
                        payload[d][0].append((int(tok_slot[t, d]), xs[t].copy()))
            for r in range(T * k):
                d = dest[r]
                if d >= 0 and rs[r] >= 0:
                    payload[d][1].append((int(rs[r]), int(ids[r]), int(tok_slot[r // k, d]),
                                          int(bits[r]), r))
                    combine_rows[r] = r
        everyone = [None] * n
        dist.all_gather_object(everyone, payload, group=bufs.group)
        bufs.received = []
        for s in range(n):
            rows, records = everyone[s][rank]
            for slot, row in rows:
                bufs.tokens.view(torch.int16)[s * bufs.max_tokens + slot] = torch.from_numpy(row)
            bufs.received.append(sorted(records))
        return torch.from_numpy(combine_rows)

    def nvl_receive(self, rank, bufs):
        m = bufs.max_routes
        ids = torch.full((m,), -1, dtype=torch.int64)
        tor = torch.zeros(m, dtype=torch.int32)
        w = torch.zeros(m, dtype=torch.int16)
        src_rank = torch.zeros(m, dtype=torch.int32)
        src_route = torch.zeros(m, dtype=torch.int32)
        j = 0
        for s, records in enumerate(bufs.received):
            for _, expert, slot, bits, route in records:
                ids[j], tor[j] = expert, s * bufs.max_tokens + slot
                w[j] = np.int16(np.uint16(bits).view(np.int16))
                src_rank[j], src_route[j] = s, route
                j += 1
        return ids, tor, w.view(torch.bfloat16), src_rank, src_route, torch.tensor([j],
                                                                                  dtype=torch.int32)

    def nvl_return(self, y, src_rank, src_route, count, rank, bufs):
        import torch.distributed as dist
        n = int(count.reshape(-1)[0])
        out = {s: [] for s in range(bufs.ep_size)}
        ys = y.view(torch.int16).numpy()
        for j in range(n):
            out[int(src_rank[j])].append((int(src_route[j]), ys[j].copy()))
        everyone = [None] * bufs.ep_size
        dist.all_gather_object(everyone, out, group=bufs.group)
        for d in range(bufs.ep_size):
            for route, row in everyone[d][rank]:
                bufs.returned.view(torch.int16)[route] = torch.from_numpy(row)

    def nvl_wait_return(self, rank, bufs):
        return None


class CpuExchange:
    """CPU stand-in of one rank's NVLink exchange buffer (token rows received
    per source, route rows returned to this rank) and its geometry."""

    def __init__(self, layer, group) -> None:
        self.group = group
        self.ep_size = layer.ep_size
        self.max_tokens = int(getattr(layer, "nvl_max_tokens", None) or 8192)
        self.top_k = layer.top_k
        self.num_experts = layer.num_experts
        self.hidden = layer.hidden_size
        self.route_cap = self.max_tokens * min(layer.top_k, layer.num_local_experts)
        self.max_routes = self.ep_size * self.route_cap
        self.tokens = torch.zeros((self.ep_size * self.max_tokens, self.hidden),
                                  dtype=torch.bfloat16)
        self.returned = torch.zeros((self.max_tokens * self.top_k, self.hidden),
                                    dtype=torch.bfloat16)
        self.received = []
        self.hist = None

    def tokens_view(self):
        return self.tokens

    def returned_view(self, rows):
        return self.returned[:rows]
