"""b200moe_route_pack: router and packing in one launch for small batches.

Its outputs must equal, bit for bit, b200moe_route_topk followed by
b200moe_pack_routes on the same logits (the layer's two-launch form, whose
routing is pinned to torch's CUDA kernels in test_gpu_router.py and whose
packing is pinned to the reference layouts in test_gpu_kernels.py): ids,
bf16 weights (drops rewritten in place), and every layout array within the
packed length.
"""

import pytest
import torch

import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def clean_status():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0


def _layout(p):
    n = int(p.counters[_lib.CNT_PADDED_ROWS])
    m = int(p.counters[_lib.CNT_MTILES])
    c = int(p.counters[_lib.CNT_CHUNKS])
    return {"counters": p.counters, "row_route": p.row_route[:n], "route_row": p.route_row,
            "combine_rows": p.combine_rows, "tile_expert": p.tile_expert[:n // 16],
            "expert_offsets": p.expert_offsets, "expert_counts": p.expert_counts,
            "mtiles": p.mtiles[:m], "chunks": p.chunks[:c]}


CASES = [  # tokens, experts, top_k, dtype, capacity, placement
    (1, 128, 8, torch.float32, None, "all"), (3, 128, 8, torch.bfloat16, None, "all"),
    (8, 128, 8, torch.float32, None, "all"), (16, 128, 8, torch.bfloat16, 1, "all"),
    (16, 128, 8, torch.float32, None, "shard"), (12, 40, 6, torch.float32, 2, "roundrobin"),
    (128, 128, 8, torch.float32, 9, "all"), (5, 1024, 8, torch.float32, None, "all"),
    (32, 64, 32, torch.bfloat16, None, "all")]


@pytest.mark.parametrize("tokens,experts,top_k,dtype,capacity,placement", CASES)
def test_route_pack_equals_route_then_pack(tokens, experts, top_k, dtype, capacity, placement):
    g = torch.Generator(device="cpu").manual_seed(tokens * 131 + experts)
    logits = torch.randn((tokens, experts), generator=g).to(dtype).to(DEV)
    if dtype == torch.bfloat16:
        logits[:, : experts // 4] = logits[:, :1]  # equal logits: the tie order must agree
    local_index, start, num_local = None, 0, experts
    if placement == "shard":
        num_local, start = experts // 4, experts // 2
    elif placement == "roundrobin":
        num_local = experts // 2
        local_index = torch.tensor([e // 2 if e % 2 == 0 else -1 for e in range(experts)],
                                   dtype=torch.int64, device=DEV)
    w1, ids1, p1 = ops.route_pack(logits, top_k, True, experts, num_local,
                                  local_index=local_index, expert_start=start,
                                  capacity=capacity)
    w2, ids2 = ops.route_topk(logits, top_k, True)
    p2 = ops.pack_routes(ids2.view(-1), w2.view(-1), experts, num_local,
                         local_index=local_index, expert_start=start, capacity=capacity)
    torch.cuda.synchronize()
    assert torch.equal(ids1, ids2)
    assert torch.equal(w1.view(torch.int16), w2.view(torch.int16))
    a, b = _layout(p1), _layout(p2)
    for key in a:
        assert torch.equal(a[key], b[key]), key
    if capacity is not None:
        assert int(p1.counters[_lib.CNT_DROPPED]) > 0


def test_route_pack_in_the_layer_matches_two_launch_form():
    """The layer takes the fused launch for <= 16 tokens; its output equals
    the same layer forced onto the two-launch form."""
    from extend_nano_vllm_b200 import moe as moe_mod
    from extend_nano_vllm_b200.moe import ExpertParallelMoE

    shape = wl.QWEN3_30B_A3B
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              True).to(device=DEV, dtype=torch.bfloat16)
    w13, w2 = wl.expert_weights(shape, seed=3, device=DEV, on_device=True)
    with torch.no_grad():
        layer.gate.weight.copy_(wl.gate_weight(shape, seed=4).to(DEV))
        layer.gate_up_proj.copy_(w13)
        layer.down_proj.copy_(w2)
    for tokens in (3, 8, 16):
        x = wl.hidden_states(tokens, shape.hidden, seed=tokens).to(DEV)
        logits = wl.uniform_logits(tokens, shape.num_experts, seed=tokens + 1).to(DEV)
        launches = dict(_lib.CALL_COUNTS)
        fused = layer._forward_from_logits(x, logits)
        assert _lib.CALL_COUNTS.get("b200moe_route_pack", 0) == \
            launches.get("b200moe_route_pack", 0) + 1
        limit = moe_mod.ROUTE_PACK_MAX_TOKENS
        moe_mod.ROUTE_PACK_MAX_TOKENS = 0
        try:
            split = layer._forward_from_logits(x, logits)
        finally:
            moe_mod.ROUTE_PACK_MAX_TOKENS = limit
        torch.cuda.synchronize()
        assert torch.equal(fused, split), tokens
