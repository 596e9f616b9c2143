"""Tensor-level wrappers of the b200moe C ABI.

Every function enqueues its kernels on the current CUDA stream of the
tensors' device and returns without synchronising.  Outputs are allocated
through the PyTorch caching allocator, so the calls can be captured in CUDA
graphs (no host synchronisation happens inside them).
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import call

_DTYPE_CODES = {torch.bfloat16: _lib.BF16, torch.float16: _lib.F16,
                torch.float32: _lib.F32, torch.float64: _lib.F64}


def _p(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("b200moe kernels run on CUDA tensors only (no CPU path)")


def _host_i32(values) -> ctypes.c_void_p:
    """Host int32 array for the C ABI's *_host arguments (kept alive by the caller's frame)."""
    arr = (ctypes.c_int32 * max(1, len(values)))(*[int(v) for v in values])
    _host_i32.keep = arr  # the C call copies it into kernel arguments before returning
    return ctypes.cast(arr, ctypes.c_void_p)


def route_topk(logits: torch.Tensor, top_k: int, renormalize: bool,
               shared_logits: torch.Tensor | None = None
               ) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 softmax + top-k (+ renorm) of [T, E] logits -> (bf16 weights, int64 ids).

    With ``shared_logits`` (bf16 [T] or [T, 1], the shared-expert gate's
    output) the rows have top_k + 1 slots, the last one the shared expert
    (id E, weight sigmoid of its gate logit)."""
    _require_cuda(logits)
    logits = logits.contiguous()
    if logits.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise TypeError(f"router logits must be fp32/bf16/fp16, got {logits.dtype}")
    tokens, experts = logits.shape
    slots = top_k if shared_logits is None else top_k + 1
    weights = torch.empty((tokens, slots), device=logits.device, dtype=torch.bfloat16)
    ids = torch.empty((tokens, slots), device=logits.device, dtype=torch.int64)
    if shared_logits is None:
        call("b200moe_route_topk", _p(logits), _DTYPE_CODES[logits.dtype], tokens, experts,
             top_k, int(bool(renormalize)), _p(weights), _p(ids), _stream(logits))
    else:
        if shared_logits.dtype != torch.bfloat16 or shared_logits.numel() != tokens:
            raise TypeError("shared_logits must be bf16 with one logit per token")
        shared_logits = shared_logits.contiguous()
        call("b200moe_route_topk_shared", _p(logits), _DTYPE_CODES[logits.dtype], tokens,
             experts, top_k, int(bool(renormalize)), _p(shared_logits), _p(weights), _p(ids),
             _stream(logits))
    return weights, ids


# Largest batch b200moe_route_gate_topk takes.
ROUTE_GATE_MAX_TOKENS = 64
_GATE_SYNC: dict[torch.device, torch.Tensor] = {}


def route_gate_topk(x: torch.Tensor, gate_w: torch.Tensor, top_k: int, renormalize: bool
                    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Router projection + softmax top-k (+ renorm) in one launch for
    <= ROUTE_GATE_MAX_TOKENS tokens -> (bf16 weights, int64 ids, bf16 logits)."""
    _require_cuda(x, gate_w)
    if x.dtype != torch.bfloat16 or gate_w.dtype != torch.bfloat16:
        raise TypeError("the fused router projection takes bf16 activations and gate weights")
    x = x.contiguous()
    gate_w = gate_w.contiguous()
    tokens, hidden = x.shape
    experts = gate_w.size(0)
    device = x.device
    sync = _GATE_SYNC.get(device)
    if sync is None:
        sync = torch.zeros(ROUTE_GATE_MAX_TOKENS // 8, device=device, dtype=torch.int32)
        _GATE_SYNC[device] = sync
    logits = torch.empty((tokens, experts), device=device, dtype=torch.bfloat16)
    weights = torch.empty((tokens, top_k), device=device, dtype=torch.bfloat16)
    ids = torch.empty((tokens, top_k), device=device, dtype=torch.int64)
    call("b200moe_route_gate_topk", _p(x), hidden, _p(gate_w), tokens, experts, top_k,
         int(bool(renormalize)), _p(logits), _p(weights), _p(ids), _p(sync), _stream(x))
    return weights, ids, logits


@dataclass
class PackedRoutes:
    """Expert-major layout of a flat route array (see b200moe_pack_routes)."""

    num_routes: int
    row_capacity: int
    max_mtiles: int
    row_route: torch.Tensor      # [row_capacity] int32
    route_row: torch.Tensor      # [num_routes] int32
    combine_rows: torch.Tensor   # [num_routes] int32
    tile_expert: torch.Tensor    # [row_capacity // 16] int32
    expert_offsets: torch.Tensor  # [E_loc + 1] int32
    expert_counts: torch.Tensor  # [E_loc] int32
    mtiles: torch.Tensor         # [max_mtiles, 3] int32
    counters: torch.Tensor       # [5] int32
    chunks: torch.Tensor | None = None  # [max_mtiles, 3] int32 row chunks of <= 256 rows


def _layout_buffers(routes: int, num_experts: int, num_local_experts: int,
                    device: torch.device):
    row_capacity = int(_lib.LIB.b200moe_pack_row_capacity(routes, num_local_experts))
    max_mtiles = int(_lib.LIB.b200moe_pack_max_mtiles(routes, num_local_experts))
    scratch_bytes = int(_lib.LIB.b200moe_pack_scratch_bytes(routes, num_experts))
    i32 = dict(device=device, dtype=torch.int32)
    return (row_capacity, max_mtiles,
            torch.empty(row_capacity, **i32),                                # row_route
            torch.empty(routes, **i32),                                      # route_row
            torch.empty(routes, **i32),                                      # combine_rows
            torch.empty(row_capacity // _lib.BLOCK_ROWS, **i32),             # tile_expert
            torch.empty(num_local_experts + 1, **i32),                       # expert_offsets
            torch.empty(num_local_experts, **i32),                           # expert_counts
            torch.empty((max(1, max_mtiles), _lib.MTILE_WORDS), **i32),      # mtiles
            torch.empty((max(1, max_mtiles), _lib.MTILE_WORDS), **i32),      # chunks
            torch.empty(_lib.NUM_COUNTERS, **i32),                           # counters
            torch.empty(max(1, scratch_bytes // 4), **i32))                  # scratch


# Largest route count b200moe_route_pack takes (one route block).
ROUTE_PACK_MAX_ROUTES = 1024


def route_pack(logits: torch.Tensor, top_k: int, renormalize: bool, num_experts: int,
               num_local_experts: int, *, local_index: torch.Tensor | None = None,
               expert_start: int = 0, capacity: int | None = None,
               stats: torch.Tensor | None = None
               ) -> tuple[torch.Tensor, torch.Tensor, "PackedRoutes"]:
    """route_topk + pack_routes in one launch for <= ROUTE_PACK_MAX_ROUTES
    routes -> (bf16 weights [T, k], int64 ids [T, k], packed layout)."""
    _require_cuda(logits)
    logits = logits.contiguous()
    if logits.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise TypeError(f"router logits must be fp32/bf16/fp16, got {logits.dtype}")
    tokens, experts = logits.shape
    if experts != num_experts:
        raise ValueError("logits must have one column per expert")
    routes = tokens * top_k
    device = logits.device
    weights = torch.empty((tokens, top_k), device=device, dtype=torch.bfloat16)
    ids = torch.empty((tokens, top_k), device=device, dtype=torch.int64)
    (row_capacity, max_mtiles, row_route, route_row, combine_rows, tile_expert, expert_offsets,
     expert_counts, mtiles, chunks, counters, scratch) = _layout_buffers(
        routes, num_experts, num_local_experts, device)
    if local_index is not None and (local_index.dtype != torch.int64
                                    or local_index.numel() != num_experts):
        raise TypeError("local_index must be int64 [num_experts]")
    call("b200moe_route_pack", _p(logits), _DTYPE_CODES[logits.dtype], tokens, experts, top_k,
         int(bool(renormalize)), _p(weights), _p(ids), _p(local_index), int(expert_start),
         num_local_experts, -1 if capacity is None else int(capacity), row_capacity,
         _p(row_route), _p(route_row), _p(combine_rows), _p(tile_expert), _p(expert_offsets),
         _p(expert_counts), _p(mtiles), max_mtiles, _p(chunks), _p(counters), _p(stats),
         _p(scratch), scratch.numel() * 4, _stream(logits))
    return weights, ids, PackedRoutes(routes, row_capacity, max_mtiles, row_route, route_row,
                                      combine_rows, tile_expert, expert_offsets, expert_counts,
                                      mtiles, counters, chunks)


def pack_routes(expert_ids: torch.Tensor, route_weights: torch.Tensor | None,
                num_experts: int, num_local_experts: int, *,
                local_index: torch.Tensor | None = None, expert_start: int = 0,
                expert_base: torch.Tensor | None = None, capacity: int | None = None,
                stats: torch.Tensor | None = None, route_count: torch.Tensor | None = None,
                capacity_dev: torch.Tensor | None = None,
                num_shared_experts: int = 0) -> PackedRoutes:
    """Capacity + expert-major packing of flat int64 routes.

    With ``capacity`` set, dropped routes are rewritten in place in
    ``expert_ids`` (to num_experts) and ``route_weights`` (to 0).
    ``route_count`` (device int32 [1]) packs only the first routes;
    ``capacity_dev`` (device int64 [1]) replaces ``capacity``.
    ``num_shared_experts``: the last experts of ``num_experts`` are shared
    experts (no capacity, not counted as kept routes).
    """
    _require_cuda(expert_ids)
    if expert_ids.dtype != torch.int64 or not expert_ids.is_contiguous():
        raise TypeError("expert_ids must be a contiguous int64 tensor")
    flat = expert_ids.view(-1)
    routes = flat.numel()
    (row_capacity, max_mtiles, row_route, route_row, combine_rows, tile_expert, expert_offsets,
     expert_counts, mtiles, chunks, counters, scratch) = _layout_buffers(
        routes, num_experts, num_local_experts, flat.device)
    if local_index is not None:
        if local_index.dtype != torch.int64 or local_index.numel() != num_experts:
            raise TypeError("local_index must be int64 [num_experts]")
    if expert_base is not None and expert_base.dtype != torch.int32:
        raise TypeError("expert_base must be int32")
    if route_weights is not None and (route_weights.dtype != torch.bfloat16
                                      or route_weights.numel() != routes):
        raise TypeError("route_weights must be bf16 with one weight per route")
    if num_shared_experts:
        if route_count is not None or capacity_dev is not None or expert_base is not None:
            raise ValueError("shared experts are packed with host bounds only")
        call("b200moe_pack_routes_shared", _p(flat), _p(route_weights), routes, num_experts,
             int(num_shared_experts), _p(local_index), int(expert_start), num_local_experts,
             -1 if capacity is None else int(capacity), row_capacity, _p(row_route),
             _p(route_row), _p(combine_rows), _p(tile_expert), _p(expert_offsets),
             _p(expert_counts), _p(mtiles), max_mtiles, _p(chunks), _p(counters), _p(stats),
             _p(scratch), scratch.numel() * 4, _stream(flat))
    elif route_count is None and capacity_dev is None:
        call("b200moe_pack_routes", _p(flat), _p(route_weights), routes, num_experts,
             _p(local_index), int(expert_start), num_local_experts, _p(expert_base),
             -1 if capacity is None else int(capacity), row_capacity, _p(row_route),
             _p(route_row), _p(combine_rows), _p(tile_expert), _p(expert_offsets),
             _p(expert_counts), _p(mtiles), max_mtiles, _p(chunks), _p(counters), _p(stats),
             _p(scratch), scratch.numel() * 4, _stream(flat))
    else:
        if route_count is not None and route_count.dtype != torch.int32:
            raise TypeError("route_count must be a device int32 scalar tensor")
        if capacity_dev is not None and capacity_dev.dtype != torch.int64:
            raise TypeError("capacity_dev must be a device int64 scalar tensor")
        call("b200moe_pack_routes_device_bounds", _p(flat), _p(route_weights), routes,
             _p(route_count), num_experts, _p(local_index), int(expert_start),
             num_local_experts, _p(expert_base), -1 if capacity is None else int(capacity),
             _p(capacity_dev), row_capacity, _p(row_route), _p(route_row), _p(combine_rows),
             _p(tile_expert), _p(expert_offsets), _p(expert_counts), _p(mtiles), max_mtiles,
             _p(chunks), _p(counters), _p(stats), _p(scratch), scratch.numel() * 4,
             _stream(flat))
    return PackedRoutes(routes, row_capacity, max_mtiles, row_route, route_row, combine_rows,
                        tile_expert, expert_offsets, expert_counts, mtiles, counters, chunks)


def expert_histogram(expert_ids: torch.Tensor, num_experts: int) -> torch.Tensor:
    _require_cuda(expert_ids)
    flat = expert_ids.reshape(-1).contiguous()
    counts = torch.empty(num_experts, device=flat.device, dtype=torch.int32)
    call("b200moe_expert_histogram", _p(flat), flat.numel(), num_experts, _p(counts),
         _stream(flat))
    return counts


def gather_rows(x: torch.Tensor, packed: PackedRoutes, top_k: int,
                token_of_route: torch.Tensor | None = None) -> torch.Tensor:
    hidden = x.size(1)
    x_packed = torch.empty((packed.row_capacity, hidden), device=x.device, dtype=x.dtype)
    call("b200moe_gather_rows", _p(x), x.size(0), hidden, _p(packed.row_route),
         _p(token_of_route), top_k, packed.num_routes, packed.row_capacity,
         _p(packed.counters), _p(x_packed), _stream(x))
    return x_packed


def expert_gate_up(engine: int, x: torch.Tensor, x_packed: torch.Tensor | None,
                   w13: torch.Tensor, packed: PackedRoutes, top_k: int,
                   token_of_route: torch.Tensor | None = None) -> torch.Tensor:
    """SwiGLU(x W13^T) per packed row -> act [row_capacity, I] (packed order)."""
    num_local, two_inter, hidden = w13.shape
    inter = two_inter // 2
    act = torch.empty((packed.row_capacity, inter), device=x.device, dtype=torch.bfloat16)
    call("b200moe_expert_gate_up", engine, _p(x), x.size(0), _p(x_packed), hidden, inter,
         _p(w13), num_local, _p(packed.row_route), _p(token_of_route), top_k,
         packed.num_routes, packed.row_capacity, _p(packed.mtiles), packed.max_mtiles,
         _p(packed.chunks), _p(packed.counters), _p(act), _stream(x))
    return act


def expert_down(engine: int, act: torch.Tensor, w2: torch.Tensor, packed: PackedRoutes,
                route_weights: torch.Tensor, max_expert_rows: int = 0) -> torch.Tensor:
    """Route-weighted down projection -> y [num_routes, H] in route order.

    Rows of routes that are not computed here are left unwritten; combine masks
    them through ``packed.combine_rows``.
    """
    num_local, hidden, inter = w2.shape
    y = torch.empty((packed.num_routes, hidden), device=act.device, dtype=torch.bfloat16)
    call("b200moe_expert_down", engine, _p(act), hidden, inter, _p(w2), num_local,
         _p(packed.row_route), _p(route_weights), packed.num_routes, int(max_expert_rows),
         packed.row_capacity, _p(packed.mtiles), packed.max_mtiles, _p(packed.chunks),
         _p(packed.counters), _p(y), _stream(act))
    return y


TINY_MAX_ROUTES = 16


def decode_tiny(logits: torch.Tensor, x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor,
                top_k: int, renormalize: bool, num_experts: int, *,
                local_index: torch.Tensor | None = None, expert_start: int = 0,
                stats: torch.Tensor | None = None) -> torch.Tensor:
    """Whole expert path for <= 16 routes (no capacity) in two launches -> out [T, H]."""
    _require_cuda(logits, x)
    logits = logits.contiguous()
    if logits.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("tiny decode path takes fp32 or bf16 logits")
    tokens, hidden = x.shape
    num_local, two_inter, _ = w13.shape
    inter = two_inter // 2
    act = torch.empty((tokens * top_k, inter), device=x.device, dtype=torch.bfloat16)
    out = torch.empty((tokens, hidden), device=x.device, dtype=torch.bfloat16)
    call("b200moe_decode_tiny", _p(logits), _DTYPE_CODES[logits.dtype], _p(x), tokens, hidden,
         inter, num_experts, top_k, int(bool(renormalize)), _p(w13), _p(w2), num_local,
         _p(local_index), int(expert_start), _p(act), _p(out), _p(stats), _stream(x))
    return out


def combine(y: torch.Tensor, route_rows: torch.Tensor | None, num_tokens: int, top_k: int,
            out_dtype: torch.dtype = torch.bfloat16, accum_f64: bool = False) -> torch.Tensor:
    """out[t] = sum_s y[route_rows[t*k+s]] in slot order (rows >= len(y) are zero)."""
    _require_cuda(y)
    if y.dtype != torch.bfloat16:
        raise TypeError("combine input must be bf16")
    y = y.contiguous()
    hidden = y.size(1)
    out = torch.empty((num_tokens, hidden), device=y.device, dtype=out_dtype)
    if route_rows is not None:
        route_rows = route_rows.to(torch.int32).contiguous()
    call("b200moe_combine", _p(y), y.size(0), _p(route_rows), num_tokens, top_k, hidden,
         int(bool(accum_f64)), _p(out), _DTYPE_CODES[out_dtype], _stream(y))
    return out


# ---------------------------------------------------------------------------
# Expert-parallel exchange helpers.
# ---------------------------------------------------------------------------
def ep_plan(expert_ids: torch.Tensor, owner: torch.Tensor, ep_size: int, num_experts: int):
    tokens, top_k = expert_ids.shape
    device = expert_ids.device
    send_token_slot = torch.empty((tokens, ep_size), device=device, dtype=torch.int32)
    route_dest_slot = torch.empty(tokens * top_k, device=device, dtype=torch.int32)
    counts = torch.empty(2 * ep_size, device=device, dtype=torch.int32)
    call("b200moe_ep_plan", _p(expert_ids), tokens, top_k, num_experts, _p(owner), ep_size,
         _p(send_token_slot), _p(route_dest_slot), _p(counts), _stream(expert_ids))
    return send_token_slot, route_dest_slot, counts


def ep_pack(x, expert_ids, route_weights, owner, ep_size, num_experts, send_token_slot,
            route_dest_slot, token_offsets, route_offsets, send_x, send_meta) -> None:
    tokens, top_k = expert_ids.shape
    call("b200moe_ep_pack", _p(x), x.size(1), _p(expert_ids), _p(route_weights), tokens, top_k,
         num_experts, _p(owner), ep_size, _p(send_token_slot), _p(route_dest_slot),
         _host_i32(token_offsets), _host_i32(route_offsets), _p(send_x), _p(send_meta),
         _stream(x))


def ep_unpack_routes(recv_meta, ep_size, recv_route_offsets, recv_token_offsets,
                     recv_meta_starts=None, num_records=None):
    """recv_meta: [n, 4] int32 records, or (with recv_meta_starts) any buffer
    holding each source's records at those 16-byte record indices."""
    n = recv_meta.size(0) if num_records is None else int(num_records)
    device = recv_meta.device
    ids = torch.empty(n, device=device, dtype=torch.int64)
    token_of_route = torch.empty(n, device=device, dtype=torch.int32)
    weights = torch.empty(n, device=device, dtype=torch.bfloat16)
    call("b200moe_ep_unpack_routes", _p(recv_meta), n, ep_size, _host_i32(recv_route_offsets),
         _host_i32(recv_token_offsets),
         None if recv_meta_starts is None else _host_i32(recv_meta_starts), _p(ids),
         _p(token_of_route), _p(weights), _stream(recv_meta))
    return ids, token_of_route, weights


def ep_return_rows(expert_ids, owner, ep_size, num_experts, route_dest_slot, route_offsets,
                   num_rows_returned) -> torch.Tensor:
    flat = expert_ids.reshape(-1)
    rows = torch.empty(flat.numel(), device=flat.device, dtype=torch.int32)
    call("b200moe_ep_return_rows", _p(flat), _p(owner), flat.numel(), num_experts, ep_size,
         _p(route_dest_slot), _host_i32(route_offsets), int(num_rows_returned), _p(rows),
         _stream(flat))
    return rows


# ---------------------------------------------------------------------------
# Expert-parallel exchange over NVLink peer memory (see nvl.py for the buffers).
# ---------------------------------------------------------------------------
def nvl_buffers(layer, device: torch.device, group):
    """The NVLink exchange buffer for this layer's shape on `group` (nvl.py)."""
    from . import nvl
    return nvl.buffers_for(layer, device, group)


def nvl_histogram_send(expert_ids: torch.Tensor, num_tokens: int, top_k: int, rank: int,
                       bufs) -> None:
    """This rank's per-expert route counts and token count to every peer."""
    call("b200moe_nvl_histogram_send", _p(expert_ids) if num_tokens else None, num_tokens,
         top_k, bufs.num_experts, rank, bufs.ep_size, bufs.peer_bases, bufs.layout_ptr,
         bufs.stream_ptr())


def nvl_histogram_wait(top_k: int, rank: int, bufs, capacity_factor: float | None):
    """-> (expert_base int32 [E], global_tokens int64 [1], capacity int64 [1]) on device."""
    device = bufs.device
    base = torch.empty(bufs.num_experts, device=device, dtype=torch.int32)
    global_tokens = torch.empty(1, device=device, dtype=torch.int64)
    capacity = torch.full((1,), -1, device=device, dtype=torch.int64)
    call("b200moe_nvl_histogram_wait", top_k, bufs.num_experts, rank, bufs.ep_size,
         bufs.peer_bases, bufs.layout_ptr, ctypes.c_double(float(capacity_factor or 0.0)),
         _p(base), _p(global_tokens), _p(capacity), bufs.stream_ptr())
    return base, global_tokens, capacity


def nvl_dispatch(x: torch.Tensor, expert_ids: torch.Tensor, route_weights: torch.Tensor,
                 owner: torch.Tensor, rank: int, bufs, send_token_slot, route_dest_slot, counts,
                 bump_epoch: bool) -> torch.Tensor:
    """Send this rank's tokens and route records; -> combine_rows int32 [T*k]."""
    tokens, top_k = expert_ids.shape
    combine_rows = torch.empty(tokens * top_k, device=bufs.device, dtype=torch.int32)
    call("b200moe_nvl_dispatch", _p(x) if tokens else None, bufs.hidden,
         _p(expert_ids) if tokens else None, _p(route_weights) if tokens else None, tokens,
         top_k, bufs.num_experts, _p(owner), rank, bufs.ep_size,
         _p(send_token_slot) if tokens else None, _p(route_dest_slot) if tokens else None,
         _p(counts) if tokens else None, bufs.peer_bases, bufs.layout_ptr, bufs.max_tokens,
         int(bool(bump_epoch)), _p(combine_rows) if tokens else None, bufs.stream_ptr())
    return combine_rows


def nvl_receive(rank: int, bufs):
    """-> (ids int64, token_of_route int32, weights bf16, src_rank int32, src_route int32)
    of length bufs.max_routes, and the received count (device int32 [1])."""
    n = bufs.max_routes
    device = bufs.device
    ids = torch.empty(n, device=device, dtype=torch.int64)
    token_of_route = torch.empty(n, device=device, dtype=torch.int32)
    weights = torch.empty(n, device=device, dtype=torch.bfloat16)
    src_rank = torch.empty(n, device=device, dtype=torch.int32)
    src_route = torch.empty(n, device=device, dtype=torch.int32)
    count = torch.empty(1, device=device, dtype=torch.int32)
    call("b200moe_nvl_receive", rank, bufs.ep_size, bufs.peer_bases, bufs.layout_ptr,
         bufs.max_tokens, _p(ids), _p(token_of_route), _p(weights), _p(src_rank),
         _p(src_route), _p(count), bufs.stream_ptr())
    return ids, token_of_route, weights, src_rank, src_route, count


def nvl_return(y: torch.Tensor, src_rank: torch.Tensor, src_route: torch.Tensor,
               count: torch.Tensor, rank: int, bufs) -> None:
    """Rows of the received routes back to their sources' return buffers."""
    call("b200moe_nvl_return", _p(y), bufs.hidden, _p(src_rank), _p(src_route), _p(count),
         y.size(0), bufs.max_tokens * bufs.top_k, rank, bufs.ep_size, bufs.peer_bases,
         bufs.layout_ptr, bufs.stream_ptr())


def nvl_return_signal(rank: int, bufs) -> None:
    """Publish the return phase after expert_down_scatter wrote the rows."""
    call("b200moe_nvl_return_signal", rank, bufs.ep_size, bufs.peer_bases, bufs.layout_ptr,
         bufs.stream_ptr())


# The NVLink exchange writes each received route's down-projection row
# straight into its source's return buffer from the GEMM epilogue
# (expert_down_scatter) instead of copying y afterwards (nvl_return).
# B200MOE_NVL_DIRECT_RETURN=0 keeps the copy.
NVL_DIRECT_RETURN = os.environ.get("B200MOE_NVL_DIRECT_RETURN", "1") != "0"


def expert_down_scatter(engine: int, act: torch.Tensor, w2: torch.Tensor, packed: PackedRoutes,
                        route_weights: torch.Tensor, src_rank: torch.Tensor,
                        src_route: torch.Tensor, bufs) -> None:
    """Route-weighted down projection whose route rows go to the sources'
    return buffers (rank src_rank[r], row src_route[r]) of the exchange."""
    num_local, hidden, inter = w2.shape
    call("b200moe_expert_down_scatter", engine, _p(act), hidden, inter, _p(w2), num_local,
         _p(packed.row_route), _p(route_weights), packed.num_routes, packed.row_capacity,
         _p(packed.mtiles), packed.max_mtiles, _p(packed.counters), bufs.peer_bases,
         bufs.ep_size, bufs.layout["returned"], _p(src_rank), _p(src_route),
         bufs.max_tokens * bufs.top_k, _stream(act))


def nvl_wait_return(rank: int, bufs) -> None:
    call("b200moe_nvl_wait_return", rank, bufs.ep_size, bufs.peer_bases, bufs.layout_ptr,
         bufs.stream_ptr())
