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
                    stats=None):
        flat = expert_ids.view(-1)
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
