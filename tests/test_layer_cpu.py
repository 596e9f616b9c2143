"""ExpertParallelMoE keeps the reference layer's contract (constructor checks,
parameters, placement, seams, counters).  Runs on CPU: the kernel entry
points are replaced by the oracle-backed CpuOps where numbers are needed."""

import math

import numpy as np
import pytest
import torch

import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import MOE_MAX_GRAPH_TOKENS_PER_RANK
from extend_nano_vllm_b200.moe import ExpertParallelMoE
from oracle import moe_oracle as mo
from oracle.cpu_ops import CpuOps


def test_constructor_validation_matches_reference_messages():
    with pytest.raises(ValueError, match="divide evenly"):
        ExpertParallelMoE(16, 32, 6, 2, True, ep_size=4)
    with pytest.raises(ValueError, match="top_k"):
        ExpertParallelMoE(16, 32, 4, 5, True)
    with pytest.raises(ValueError, match="unknown MoE dispatch backend"):
        ExpertParallelMoE(16, 32, 4, 2, True, dispatch_backend="nope")
    with pytest.raises(ValueError, match="capacity"):
        ExpertParallelMoE(16, 32, 4, 2, True, expert_capacity=0)
    for factor in (0.0, -1.0, float("inf"), float("nan"), True):
        with pytest.raises(ValueError, match="capacity factor"):
            ExpertParallelMoE(16, 32, 4, 2, True, expert_capacity_factor=factor)
    with pytest.raises(ValueError, match="mutually exclusive"):
        ExpertParallelMoE(16, 32, 4, 2, True, expert_capacity=2, expert_capacity_factor=1.0)
    with pytest.raises(ValueError, match="graph-safe dispatch"):
        ExpertParallelMoE(128, 256, 8, 2, True, dispatch_backend="all_to_all",
                          graph_safe_decode=True)
    with pytest.raises(ValueError, match="equal experts"):
        ExpertParallelMoE(16, 32, 4, 2, True, ep_size=2, expert_owners=[0, 0, 0, 1])
    with pytest.raises(ValueError, match="shared expert"):
        ExpertParallelMoE(16, 32, 4, 2, True, shared_expert_intermediate_size=0)
    # The new NCCL all-to-all backend is accepted, also for graph-safe decode.
    ExpertParallelMoE(16, 32, 4, 2, True, dispatch_backend="all_to_all_nvlink",
                      graph_safe_decode=True)


def test_parameters_state_dict_and_placement():
    layer = ExpertParallelMoE(16, 32, 8, 2, True, ep_rank=1, ep_size=2)
    shapes = {k: tuple(v.shape) for k, v in layer.state_dict().items()}
    assert shapes == {"gate.weight": (8, 16), "gate_up_proj": (4, 64, 16),
                      "down_proj": (4, 16, 32)}
    assert layer.local_expert_ids == (4, 5, 6, 7)
    assert layer.owns_expert(5) and not layer.owns_expert(3)
    assert layer.expert_parameter_bytes == (4 * 64 * 16 + 4 * 16 * 32) * 4
    layer.load_expert_weight(6, "up_proj", torch.ones(32, 16))
    assert torch.equal(layer.gate_up_proj.data[2, 32:], torch.ones(32, 16))
    layer.load_expert_weight(1, "down_proj", torch.ones(16, 32))  # not local: ignored
    with pytest.raises(ValueError, match="unknown expert projection"):
        layer.load_expert_weight(4, "bad", torch.ones(1))
    other = ExpertParallelMoE(16, 32, 8, 2, True, ep_rank=1, ep_size=2)
    other.load_state_dict(layer.state_dict())
    assert layer.graph_token_limit == MOE_MAX_GRAPH_TOKENS_PER_RANK
    gathered = ExpertParallelMoE(16, 32, 8, 2, True, ep_rank=1, ep_size=2,
                                 dispatch_backend="allgather_reduce")
    assert gathered.graph_token_limit == 2 * MOE_MAX_GRAPH_TOKENS_PER_RANK


def test_noncontiguous_route_mapping_handles_padding():
    # Same case as the reference's tests/test_moe_placement.py:79-91.
    layer = ExpertParallelMoE(16, 32, 4, 2, True, ep_rank=0, ep_size=2,
                              expert_owners=[0, 1, 1, 0])
    mask, local_ids = layer._local_routes(torch.tensor([-1, 0, 1, 2, 3, 4]))
    assert mask.tolist() == [False, True, False, False, True, False]
    assert local_ids[mask].tolist() == [0, 1]


def test_cpu_tensors_have_no_fallback():
    layer = ExpertParallelMoE(16, 32, 4, 2, True).bfloat16()
    with pytest.raises(RuntimeError, match="CUDA"):
        layer(torch.randn(3, 16, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="no CPU path"):
        layer._execute_local(torch.randn(3, 16, dtype=torch.bfloat16),
                             torch.ones(3, 2, dtype=torch.bfloat16),
                             torch.zeros(3, 2, dtype=torch.int64))


def _layer_with_weights(shape, seed, **kw):
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              shape.norm_topk_prob, **kw).bfloat16()
    w13, w2 = wl.expert_weights(shape, seed=seed)
    gate = wl.gate_weight(shape, seed=seed + 1).bfloat16()
    with torch.no_grad():
        layer.gate.weight.copy_(gate)
        layer.gate_up_proj.copy_(w13)
        layer.down_proj.copy_(w2)
    layer._ops = CpuOps()
    return layer, w13, w2, gate


@pytest.mark.parametrize("kw,tokens", [(dict(), 9), (dict(expert_capacity=1), 9),
                                        (dict(expert_capacity_factor=1.0), 2),
                                        (dict(expert_capacity_factor=1.0), 9)])
def test_host_logic_and_counters_follow_reference(kw, tokens):
    shape = wl.LayerShape("small", 16, 32, 4, 2)
    layer, w13, w2, gate = _layer_with_weights(shape, 31, **kw)
    x = wl.hidden_states(tokens, 16, seed=5)
    out = layer(x)
    logits = torch.nn.functional.linear(x, gate).float().numpy()
    cap = mo.capacity_of(tokens, 2, 4, kw.get("expert_capacity"), kw.get("expert_capacity_factor"))
    ref = mo.moe_forward(x.float().numpy(), logits, w13.float().numpy(), w2.float().numpy(), 2,
                         True, capacity=cap)
    np.testing.assert_array_equal(out.float().numpy(), ref["output"])
    kept = int(ref["keep"].sum())
    assert layer.dispatch_assignment_count == kept
    assert layer.return_assignment_count == kept
    assert layer.total_assignment_count == tokens * 2
    assert layer.dropped_assignment_count == tokens * 2 - kept
    layer.dispatch_assignment_count = 0
    assert layer.dispatch_assignment_count == 0


def test_route_and_execute_local_seams():
    shape = wl.LayerShape("small", 32, 64, 8, 2)
    layer, w13, w2, gate = _layer_with_weights(shape, 41, expert_capacity_factor=0.5)
    x = wl.hidden_states(12, 32, seed=6)
    w, ids = layer._route(x)
    assert (ids == 8).any()  # capacity 0.5 drops some routes
    assert layer.dropped_assignment_count == int((ids == 8).sum())
    out, local = layer._execute_local(x, w, ids)
    assert local == int((ids < 8).sum())
    assert math.isfinite(float(out.float().abs().sum()))


def test_shared_expert_weights_live_behind_the_routed_experts():
    """A shared expert of the routed width is stored as expert E_loc of the
    grouped storage; its parameters stay the reference's names, shapes and
    loaders, and the storage survives dtype moves and state_dict loads."""
    layer = ExpertParallelMoE(16, 32, 8, 2, True, shared_expert_intermediate_size=32)
    shapes = {k: tuple(v.shape) for k, v in layer.state_dict().items()}
    assert shapes == {"gate.weight": (8, 16), "gate_up_proj": (8, 64, 16),
                      "down_proj": (8, 16, 32),
                      "shared_expert.gate_up_proj.weight": (64, 16),
                      "shared_expert.down_proj.weight": (16, 32),
                      "shared_expert_gate.weight": (1, 16)}
    shared = layer.shared_expert
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0, 0.02)
    for dtype in (torch.float32, torch.bfloat16):
        layer = layer.to(dtype)
        w13, w2 = layer._shared_store()
        assert w13.shape == (9, 64, 16) and w2.shape == (9, 16, 32)
        assert w13.data_ptr() == layer.gate_up_proj.data_ptr()
        assert w13[8].data_ptr() == shared.gate_up_proj.weight.data_ptr()
        assert w2[8].data_ptr() == shared.down_proj.weight.data_ptr()
    gate = torch.randn(32, 16).to(torch.bfloat16)
    up = torch.randn(32, 16).to(torch.bfloat16)
    loader = shared.gate_up_proj.weight.weight_loader
    loader(shared.gate_up_proj.weight, gate, 0)
    loader(shared.gate_up_proj.weight, up, 1)
    w13, _ = layer._shared_store()
    assert torch.equal(w13[8, :32], gate) and torch.equal(w13[8, 32:], up)
    other = ExpertParallelMoE(16, 32, 8, 2, True,
                              shared_expert_intermediate_size=32).to(torch.bfloat16)
    other.load_state_dict(layer.state_dict())
    o13, o2 = other._shared_store()
    assert torch.equal(o13, w13) and torch.equal(o2[8], layer.shared_expert.down_proj.weight)
    # A wider shared expert keeps its own storage (it runs after the routed output).
    wide = ExpertParallelMoE(16, 32, 8, 2, True, shared_expert_intermediate_size=64)
    assert not wide._shared_in_store
