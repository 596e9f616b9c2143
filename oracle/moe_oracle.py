"""CPU oracle of the Qwen3-MoE expert path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module; the product path never does.

It restates, in numpy (integer/routing work) and torch-CPU fp32 (expert
math), the algorithm of ``nanovllm.layers.moe.ExpertParallelMoE`` from
kagami4243/extend-nano-vLLM 0.3.0.  Each function cites the reference lines
it follows.  Parity pinning: ``tests/test_oracle_golden.py`` checks these
functions against golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference on CPU and records
its outputs).

Conventions shared with the CUDA library:
  * the router reproduces torch's CUDA softmax, top-k (including the order
    of equal probabilities) and renormalisation sum, the reference's GPU
    path (moe.py:872-878);
  * rounding points of the reference's GPU path (moe.py:742-746, :848-858):
    gate/up stored in bf16, silu and the product rounded to bf16, the route
    weight applied to the fp32 down accumulator before the bf16 store, the
    combine summed in fp32 in slot order (moe.py:164-192).
"""

from __future__ import annotations

import math

import numpy as np
import torch

BLOCK_ROWS = 16      # reference _MOE_BLOCK_M, moe.py:36
MTILE_ROWS = 128     # work-tile rows of the CUDA library
CHUNK_ROWS = 256     # row-chunk limit of the CUDA library's two-SM engine


# ---------------------------------------------------------------------------
# bf16 helpers
# ---------------------------------------------------------------------------
def bf16_round(a) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out)


def bf16_bits(a) -> np.ndarray:
    return (bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# Router (moe.py:870-878): the arithmetic and selection order of
#   F.softmax(logits, -1, dtype=float32); torch.topk(probs, k);
#   w /= w.sum(-1, keepdim=True); w.to(bf16)
# as torch 2.x computes them on a CUDA device (the reference's GPU path).
# ---------------------------------------------------------------------------
def softmax_f32(logits: np.ndarray) -> np.ndarray:
    """torch's persistent warp softmax for rows of <= 1024 fp32 values:
    with P = next power of two >= E and L = min(P, 32) lanes, lane l holds
    elements l + L*i; p = exp(v - max); each lane sums its elements in i
    order, a butterfly (xor L/2 ... 1) sums the lanes; out = p / sum.
    numpy's float32 exp stands in for CUDA's expf (they agree to within an
    ulp; the tie-order tests feed probabilities recorded on a GPU instead)."""
    logits = np.asarray(logits, dtype=np.float32)
    rows, experts = logits.shape
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - m, dtype=np.float32)
    width = 1
    while width < experts:
        width *= 2
    lanes = min(width, 32)
    padded = np.zeros((rows, width), dtype=np.float32)
    padded[:, :experts] = e
    lane_sum = np.zeros((rows, lanes), dtype=np.float32)
    for i in range(width // lanes):
        lane_sum = (lane_sum + padded[:, i * lanes:(i + 1) * lanes]).astype(np.float32)
    off = lanes // 2
    idx = np.arange(lanes)
    while off:
        lane_sum = (lane_sum + lane_sum[:, idx ^ off]).astype(np.float32)
        off //= 2
    return (e / lane_sum[:, :1]).astype(np.float32)


def _bitonic_exchange(key, ids, lo, hi, direction):
    """One compare-exchange of torch's bitonic sort (descending comparator
    a > b): exchange when ((key[lo] > key[hi] and lo valid) or hi invalid)
    equals the direction.  ids < 0 mark invalid padding."""
    ka, kb = key[:, lo], key[:, hi]
    va, vb = ids[:, lo] >= 0, ids[:, hi] >= 0
    swap = ((ka > kb) & va) | ~vb
    ex = swap == direction
    key[ex, lo], key[ex, hi] = kb[ex], ka[ex]
    ia, ib = ids[:, lo].copy(), ids[:, hi].copy()
    ids[ex, lo], ids[ex, hi] = ib[ex], ia[ex]


def topk_from_probs(probs: np.ndarray, top_k: int) -> tuple[np.ndarray, np.ndarray]:
    """torch.topk(probs, k) (largest, sorted) on a CUDA device, k <= 32.

    The selection kernel writes the elements above the k-th largest value in
    ascending index order, then the first elements equal to it (ascending
    index); the k pairs are then sorted by a 32-wide bitonic network whose
    exchange is not stable, which fixes the order of equal values."""
    probs = np.asarray(probs, dtype=np.float32)
    rows, experts = probs.shape
    if not 1 <= top_k <= min(32, experts):
        raise ValueError("top_k must be in [1, min(32, num_experts)]")
    order = np.lexsort((np.broadcast_to(np.arange(experts), probs.shape), -probs))[:, :top_k]
    kth = np.take_along_axis(probs, order[:, -1:], axis=1)
    gathered = np.empty((rows, top_k), dtype=np.int64)
    for r in range(rows):
        above = np.sort(order[r][probs[r, order[r]] > kth[r, 0]])
        equal = np.nonzero(probs[r] == kth[r, 0])[0][: top_k - above.size]
        gathered[r] = np.concatenate([above, equal])
    key = np.zeros((rows, 32), dtype=np.float32)
    ids = np.full((rows, 32), -1, dtype=np.int64)
    key[:, :top_k] = np.take_along_axis(probs, gathered, axis=1)
    ids[:, :top_k] = gathered
    if top_k > 1:
        pos = np.arange(32)
        size = 2
        while size < 32:
            stride = size // 2
            while stride:
                lo = pos[(pos & stride) == 0]
                for a in lo:
                    _bitonic_exchange(key, ids, a, a + stride, bool(a & size))
                stride //= 2
            size *= 2
        stride = 16
        while stride:
            for a in pos[(pos & stride) == 0]:
                _bitonic_exchange(key, ids, a, a + stride, False)
            stride //= 2
    return key[:, :top_k].copy(), ids[:, :top_k].copy()


def renorm_sum(w: np.ndarray) -> np.ndarray:
    """torch's sum over the last dim of a [T, k] fp32 tensor on CUDA: thread
    t < W (W = largest power of two <= k) adds slots t and t + W, then a
    shuffle-down tree with offsets W/2 ... 1."""
    w = np.asarray(w, dtype=np.float32)
    k = w.shape[1]
    width = 1
    while width * 2 <= k:
        width *= 2
    acc = w[:, :width].copy()
    for t in range(width):
        if t + width < k:
            acc[:, t] = (acc[:, t] + w[:, t + width]).astype(np.float32)
    off = width // 2
    while off:
        acc[:, :off] = (acc[:, :off] + acc[:, off:2 * off]).astype(np.float32)
        off //= 2
    return acc[:, 0]


def route_from_probs(probs: np.ndarray, top_k: int, renormalize: bool
                     ) -> tuple[np.ndarray, np.ndarray]:
    """top-k + optional renorm + bf16 cast of given fp32 probabilities."""
    w, ids = topk_from_probs(probs, top_k)
    if renormalize:
        w = (w / renorm_sum(w)[:, None]).astype(np.float32)
    return bf16_round(w), ids


def route_topk(logits: np.ndarray, top_k: int, renormalize: bool
               ) -> tuple[np.ndarray, np.ndarray]:
    """softmax(fp32) -> top-k -> optional renorm -> bf16 (moe.py:871-878).

    Returns (weights as bf16-rounded float32 [T, k], ids int64 [T, k]).
    """
    return route_from_probs(softmax_f32(logits), top_k, renormalize)


def tie_tokens(logits: np.ndarray, top_k: int) -> np.ndarray:
    """Tokens whose top-(k+1) logits contain a tie (order there is unspecified
    in the reference)."""
    logits = np.asarray(logits, dtype=np.float32)
    top = -np.sort(-logits, axis=-1)[:, : top_k + 1]
    return np.any(top[:, 1:] == top[:, :-1], axis=-1)


# ---------------------------------------------------------------------------
# Capacity (moe.py:879-919)
# ---------------------------------------------------------------------------
def capacity_of(num_tokens: int, top_k: int, num_experts: int,
                expert_capacity: int | None, capacity_factor: float | None) -> int | None:
    """moe.py:880-886, same float expression order."""
    if expert_capacity is not None:
        return int(expert_capacity)
    if capacity_factor is not None:
        return max(1, math.ceil(capacity_factor * num_tokens * top_k / num_experts))
    return None


def expert_positions(flat_ids: np.ndarray, num_experts: int) -> np.ndarray:
    """Position of each route among earlier routes to the same expert (stable
    argsort + group offsets, moe.py:887-909).  Invalid ids get their own key."""
    flat = np.asarray(flat_ids, dtype=np.int64).reshape(-1)
    keys = np.where((flat >= 0) & (flat < num_experts), flat, num_experts)
    order = np.argsort(keys, kind="stable")
    sorted_keys = keys[order]
    idx = np.arange(flat.size)
    start = np.ones(flat.size, dtype=bool)
    start[1:] = sorted_keys[1:] != sorted_keys[:-1]
    first = np.maximum.accumulate(np.where(start, idx, 0)) if flat.size else idx
    pos = np.empty(flat.size, dtype=np.int64)
    pos[order] = idx - first
    return pos


def apply_capacity(weights: np.ndarray, ids: np.ndarray, num_experts: int,
                   capacity: int | None, expert_base: np.ndarray | None = None):
    """keep = base[e] + position < capacity; dropped -> weight 0, id E
    (moe.py:910-919).  Returns (weights, ids, keep) as new arrays."""
    ids = np.array(ids, dtype=np.int64, copy=True)
    weights = np.array(weights, dtype=np.float32, copy=True)
    if capacity is None:
        return weights, ids, np.ones(ids.shape, dtype=bool)
    flat = ids.reshape(-1)
    pos = expert_positions(flat, num_experts)
    valid = (flat >= 0) & (flat < num_experts)
    base = np.zeros(flat.size, dtype=np.int64)
    if expert_base is not None:
        base[valid] = np.asarray(expert_base, dtype=np.int64)[flat[valid]]
    keep = ~valid | (base + pos < capacity)
    keep = keep.reshape(ids.shape)
    dropped = valid.reshape(ids.shape) & ~keep
    weights[dropped] = 0.0
    ids[dropped] = num_experts
    return weights, ids, ~dropped


# ---------------------------------------------------------------------------
# Local-route mapping and packing (moe.py:491-517, :698-740, :783-847)
# ---------------------------------------------------------------------------
def local_ids(flat_ids: np.ndarray, num_experts: int, num_local: int,
              expert_start: int = 0, local_index: np.ndarray | None = None) -> np.ndarray:
    """Local expert id of each route or -1 (moe.py:494-517)."""
    flat = np.asarray(flat_ids, dtype=np.int64).reshape(-1)
    valid = (flat >= 0) & (flat < num_experts)
    if local_index is None:
        local = flat - expert_start
        ok = valid & (local >= 0) & (local < num_local)
    else:
        li = np.asarray(local_index, dtype=np.int64)
        local = np.where(valid, li[np.clip(flat, 0, num_experts - 1)], -1)
        ok = valid & (local >= 0)
    return np.where(ok, local, -1)


def row_capacity(num_routes: int, num_local: int) -> int:
    """moe.py:793-797."""
    active = min(num_routes, num_local)
    rows = num_routes + active * (BLOCK_ROWS - 1)
    return (rows + BLOCK_ROWS - 1) // BLOCK_ROWS * BLOCK_ROWS


def pack(flat_ids: np.ndarray, num_experts: int, num_local: int, expert_start: int = 0,
         local_index: np.ndarray | None = None) -> dict:
    """Expert-major 16-aligned layout of the local routes.

    Keys: row_route (reference static row_ids with sentinel = num_routes,
    moe.py:828-846), tile_expert (reference expert_ids, :833-844),
    padded_rows (num_tokens_post_padded, :807), route_row (dynamic-path
    route_rows with sentinel = row_capacity, :763-767), expert_offsets,
    expert_counts, combine_rows (route id if local else num_routes), mtiles
    (128-row work tiles of the CUDA library), chunks (the library's row chunks
    of <= 256 rows: ceil(n/256) equal 16-row multiples per expert, the last
    one shorter).
    """
    flat = np.asarray(flat_ids, dtype=np.int64).reshape(-1)
    R = flat.size
    cap_rows = row_capacity(R, num_local)
    local = local_ids(flat, num_experts, num_local, expert_start, local_index)
    counts = np.bincount(local[local >= 0], minlength=num_local).astype(np.int64)
    padded = (counts + BLOCK_ROWS - 1) // BLOCK_ROWS * BLOCK_ROWS
    starts = np.cumsum(padded) - padded
    total = int(padded.sum())
    row_route = np.full(cap_rows, R, dtype=np.int64)
    route_row = np.full(R, cap_rows, dtype=np.int64)
    combine_rows = np.full(R, R, dtype=np.int64)
    # Stable expert-major order of local routes (moe.py:808-832).
    sel = np.nonzero(local >= 0)[0]
    order = sel[np.argsort(local[sel], kind="stable")]
    within = np.arange(order.size) - (np.cumsum(counts) - counts)[local[order]]
    positions = starts[local[order]] + within
    row_route[positions] = order
    route_row[order] = positions
    combine_rows[order] = order
    tile_expert = np.zeros(cap_rows // BLOCK_ROWS, dtype=np.int64)
    for e in range(num_local):
        tile_expert[starts[e] // BLOCK_ROWS:(starts[e] + padded[e]) // BLOCK_ROWS] = e
    mtiles = []
    for e in range(num_local):
        for i in range(0, int(counts[e]), MTILE_ROWS):
            mtiles.append((e, int(starts[e] + i), int(starts[e] + min(counts[e], i + MTILE_ROWS))))
    chunks = []
    for e in range(num_local):
        n = int(counts[e])
        if n == 0:
            continue
        nc = -(-n // CHUNK_ROWS)
        q = -(-(-(-n // nc)) // BLOCK_ROWS) * BLOCK_ROWS
        for i in range(nc):
            chunks.append((e, int(starts[e] + i * q), int(starts[e] + min(n, (i + 1) * q))))
    return dict(row_route=row_route, tile_expert=tile_expert, padded_rows=total,
                route_row=route_row, combine_rows=combine_rows,
                expert_offsets=np.append(starts, total), expert_counts=counts,
                mtiles=np.array(mtiles, dtype=np.int64).reshape(-1, 3),
                chunks=np.array(chunks, dtype=np.int64).reshape(-1, 3),
                local_kept=int(counts.sum()))


# ---------------------------------------------------------------------------
# Expert math (Triton path numerics, moe.py:63-139, :742-770, :848-863)
# ---------------------------------------------------------------------------
def _t32(a) -> torch.Tensor:
    """fp32 CPU tensor of a numpy array or a torch tensor (any device, bf16
    allowed), so that large bf16 weights are widened one expert at a time."""
    if isinstance(a, torch.Tensor):
        return a.detach().to(device="cpu", dtype=torch.float32)
    return torch.as_tensor(np.asarray(a, dtype=np.float32))


def expert_rows(x: np.ndarray, w13: np.ndarray, w2: np.ndarray, flat_ids: np.ndarray,
                flat_weights: np.ndarray, tokens_of_route: np.ndarray, num_experts: int,
                num_local: int, expert_start: int = 0,
                local_index: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Per-route expert output y [R, H] (bf16-valued float32) and a mask of the
    routes computed here.  x, w13, w2, flat_weights hold bf16 values; w13 and
    w2 may be numpy arrays or (bf16) torch tensors."""
    flat = np.asarray(flat_ids, dtype=np.int64).reshape(-1)
    local = local_ids(flat, num_experts, num_local, expert_start, local_index)
    H = x.shape[1]
    inter = w13.shape[1] // 2
    y = np.zeros((flat.size, H), dtype=np.float32)
    xt = _t32(x)
    for e in np.unique(local[local >= 0]):
        routes = np.nonzero(local == e)[0]
        a = xt[torch.as_tensor(tokens_of_route[routes])]
        gu = a @ _t32(w13[e]).T                       # fp32 accumulate
        g = bf16_round(gu[:, :inter].numpy())
        u = bf16_round(gu[:, inter:].numpy())
        s = bf16_round(g / (1.0 + np.exp(-g, dtype=np.float32)))
        act = bf16_round(s * u)
        d = (_t32(act) @ _t32(w2[e]).T).numpy()       # fp32 accumulate
        w = np.asarray(flat_weights, dtype=np.float32)[routes][:, None]
        y[routes] = bf16_round(d * w)
    return y, local >= 0


def combine(y: np.ndarray, route_rows: np.ndarray, num_tokens: int, top_k: int,
            accum=np.float32) -> np.ndarray:
    """out[t] = sum_s Y[route_rows[t*k+s]] in slot order, rows >= len(Y) are 0
    (moe.py:164-192).  Returns the accumulator dtype; round with bf16_round."""
    rows = np.asarray(route_rows, dtype=np.int64).reshape(num_tokens, top_k)
    padded = np.concatenate([np.asarray(y, dtype=accum), np.zeros((1, y.shape[1]), dtype=accum)])
    safe = np.where((rows >= 0) & (rows < y.shape[0]), rows, y.shape[0])
    out = np.zeros((num_tokens, y.shape[1]), dtype=accum)
    for s in range(top_k):
        out = (out + padded[safe[:, s]]).astype(accum)
    return out


def moe_forward(x: np.ndarray, logits: np.ndarray, w13: np.ndarray, w2: np.ndarray,
                top_k: int, renormalize: bool, *, capacity: int | None = None,
                num_local: int | None = None, expert_start: int = 0,
                local_index: np.ndarray | None = None, probs: np.ndarray | None = None
                ) -> dict:
    """Full layer on one rank: route, capacity, local experts, combine.

    ``probs`` (optional) are softmax probabilities computed elsewhere (a GPU
    test passes torch's CUDA softmax so that exp rounding cannot differ);
    selection, renormalisation and everything after run here."""
    num_tokens, num_experts = logits.shape
    num_local = w13.shape[0] if num_local is None else num_local
    if probs is None:
        weights, ids = route_topk(logits, top_k, renormalize)
    else:
        weights, ids = route_from_probs(probs, top_k, renormalize)
    weights, ids, keep = apply_capacity(weights, ids, num_experts, capacity)
    flat = ids.reshape(-1)
    tokens = np.arange(flat.size) // top_k
    y, computed = expert_rows(x, w13, w2, flat, weights.reshape(-1), tokens, num_experts,
                              num_local, expert_start, local_index)
    rows = np.where(computed, np.arange(flat.size), flat.size)
    out = bf16_round(combine(y, rows, num_tokens, top_k))
    return dict(weights=weights, ids=ids, keep=keep, y=y, output=out)


# ---------------------------------------------------------------------------
# The reference's own CPU path, restated for the CPU baseline timing:
# _route + _forward_reference (moe.py:870-920, :546-580), bf16 torch ops.
# ---------------------------------------------------------------------------
def forward_reference_torch(x: torch.Tensor, gate_w: torch.Tensor, w13: torch.Tensor,
                            w2: torch.Tensor, top_k: int, renormalize: bool,
                            logits: torch.Tensor | None = None) -> torch.Tensor:
    """Per-expert torch loop on CPU tensors (bf16), as the reference computes on CPU."""
    if logits is None:
        logits = torch.nn.functional.linear(x, gate_w)
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    w, ids = torch.topk(probs, top_k, dim=-1)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    w = w.to(x.dtype)
    out = torch.zeros_like(x)
    inter = w13.shape[1] // 2
    for e in ids.unique().tolist():
        tok, slot = torch.where(ids == e)
        gu = torch.nn.functional.linear(x[tok], w13[e])
        h = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
        o = torch.nn.functional.linear(h, w2[e]) * w[tok, slot, None]
        out.index_add_(0, tok, o)
    return out


def shared_expert_torch(x: torch.Tensor, w13_s: torch.Tensor, w2_s: torch.Tensor,
                        gate_s: torch.Tensor) -> torch.Tensor:
    """The shared expert term the reference adds after the routed output
    (moe.py:1259-1262): sigmoid(x gate_s^T) * down(silu(gate) * up), with the
    MLP of moe.py:231-234; bf16 torch operations as on the reference's path."""
    gate, up = torch.nn.functional.linear(x, w13_s).chunk(2, dim=-1)
    projected = torch.nn.functional.linear(torch.nn.functional.silu(gate) * up, w2_s)
    return torch.sigmoid(torch.nn.functional.linear(x, gate_s)) * projected
