"""The packing entry point for callers that cannot provide scratch memory.

b200moe_pack_routes_static_scratch serves hosts that have no device memory
to spare or no allocator to call (the library keeps its own fixed scratch
array per GPU).  It must produce exactly what b200moe_pack_routes produces
with a caller buffer, call after call, because every call reuses the same
array.  Packing results are integers, so the comparison is bit-exact.

This file is collected last so that a failing run still executes every
other test first.
"""

import ctypes

import numpy as np
import pytest
import torch

import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _pack_static(ids, weights, num_experts, num_local, capacity, local_index=None,
                 expert_start=0):
    """Same outputs as ops.pack_routes, through the no-scratch entry point."""
    flat = ids.view(-1)
    routes = flat.numel()
    dev = flat.device
    row_capacity = int(_lib.LIB.b200moe_pack_row_capacity(routes, num_local))
    max_mtiles = int(_lib.LIB.b200moe_pack_max_mtiles(routes, num_local))
    i32 = dict(device=dev, dtype=torch.int32)
    out = dict(
        row_route=torch.empty(row_capacity, **i32), route_row=torch.empty(routes, **i32),
        combine_rows=torch.empty(routes, **i32),
        tile_expert=torch.empty(row_capacity // _lib.BLOCK_ROWS, **i32),
        expert_offsets=torch.empty(num_local + 1, **i32),
        expert_counts=torch.empty(num_local, **i32),
        mtiles=torch.empty((max_mtiles, _lib.MTILE_WORDS), **i32),
        counters=torch.empty(_lib.NUM_COUNTERS, **i32))
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.call("b200moe_pack_routes_static_scratch", _p(flat), _p(weights.view(-1)), routes,
              num_experts, _p(local_index), expert_start, num_local, None,
              -1 if capacity is None else capacity,
              row_capacity, _p(out["row_route"]), _p(out["route_row"]), _p(out["combine_rows"]),
              _p(out["tile_expert"]), _p(out["expert_offsets"]), _p(out["expert_counts"]),
              _p(out["mtiles"]), max_mtiles, _p(out["counters"]), None, stream)
    return out


@pytest.mark.parametrize("tokens,capacity", [(512, None), (8192, 640)])
def test_static_scratch_pack_matches_caller_scratch_pack_twice(tokens, capacity):
    dev = torch.device("cuda")
    for call in range(2):  # consecutive calls reuse the library's scratch array
        logits = wl.zipf_logits(tokens, 128, seed=70 + 10 * call + tokens).to(dev)
        weights, ids = ops.route_topk(logits, 8, True)
        ids_a, w_a = ids.clone(), weights.clone()
        ids_b, w_b = ids.clone(), weights.clone()
        ref = ops.pack_routes(ids_a.view(-1), w_a.view(-1), 128, 128, capacity=capacity)
        got = _pack_static(ids_b, w_b, 128, 128, capacity)
        torch.cuda.synchronize()
        assert torch.equal(ids_a, ids_b)
        assert torch.equal(w_a, w_b)
        for name, tensor in got.items():
            expect = getattr(ref, name)
            if name == "mtiles":
                n = int(ref.counters[_lib.CNT_MTILES])
                tensor, expect = tensor[:n], expect[:n]
            if name == "counters":
                # This variant writes no row-chunk list and reports zero chunks.
                assert int(tensor[_lib.CNT_CHUNKS]) == 0
                tensor, expect = tensor[:_lib.CNT_CHUNKS], expect[:_lib.CNT_CHUNKS]
            np.testing.assert_array_equal(tensor.cpu().numpy(), expect.cpu().numpy(),
                                          err_msg=f"{name} (call {call})")
    assert _lib.device_status(clear=True) == 0


def _compare(ref, got, tag):
    for name, tensor in got.items():
        expect = getattr(ref, name)
        if name == "mtiles":
            n = int(ref.counters[_lib.CNT_MTILES])
            tensor, expect = tensor[:n], expect[:n]
        if name == "counters":
            assert int(tensor[_lib.CNT_CHUNKS]) == 0
            tensor, expect = tensor[:_lib.CNT_CHUNKS], expect[:_lib.CNT_CHUNKS]
        np.testing.assert_array_equal(tensor.cpu().numpy(), expect.cpu().numpy(),
                                      err_msg=f"{name} ({tag})")


@pytest.mark.parametrize("placement", ["shard", "round_robin"])
def test_static_scratch_pack_expert_parallel_placements(placement):
    """An EP rank's view: 32 of 128 experts local, either the contiguous
    shard starting at expert 64 or every fourth expert through local_index."""
    dev = torch.device("cuda")
    local_index = None
    expert_start = 0
    if placement == "shard":
        expert_start = 64
    else:
        local_index = torch.tensor([(e // 4 if e % 4 == 1 else -1) for e in range(128)],
                                   dtype=torch.int64, device=dev)
    for call in range(2):
        logits = wl.uniform_logits(2048, 128, seed=90 + call).to(dev)
        weights, ids = ops.route_topk(logits, 8, True)
        ref = ops.pack_routes(ids.clone().view(-1), weights.clone().view(-1), 128, 32,
                              local_index=local_index, expert_start=expert_start)
        got = _pack_static(ids.clone(), weights.clone(), 128, 32, None, local_index,
                           expert_start)
        torch.cuda.synchronize()
        _compare(ref, got, f"{placement}, call {call}")
    assert _lib.device_status(clear=True) == 0


def test_static_scratch_rejects_oversized_calls():
    cap = int(_lib.LIB.b200moe_pack_static_scratch_capacity())
    assert cap == 256 * 1024
    # 16 histogram blocks x 4097 counters x 4 bytes is just over the array.
    routes, experts = 16 * 1024, 4096
    assert int(_lib.LIB.b200moe_pack_scratch_bytes(routes, experts)) > cap
    assert int(_lib.LIB.b200moe_pack_scratch_bytes(65536, 1023)) <= cap
    with pytest.raises(ValueError, match="static scratch"):
        _lib.call("b200moe_pack_routes_static_scratch", None, None, routes, experts, None, 0,
                  experts, None, -1, 0, None, None, None, None, None, None, None, 0, None, None,
                  None)
