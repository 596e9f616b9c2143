"""Layer-level GPU tests of ExpertParallelMoE, modelled on the reference's
layer tests (tests/test_moe_graph_capture.py, test_moe_compact_layout.py,
test_moe_precision_mode.py, test_moe_capacity.py, test_moe_kernel.py).
Tolerances as in test_gpu_kernels.py: layer outputs max|diff| <= 2^-7*max|ref|,
mean <= 2e-4*max|ref|; integer results and combines bit-exact."""

import numpy as np
import pytest
import torch

import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import _lib
from extend_nano_vllm_b200.moe import ExpertParallelMoE
from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def close(got: torch.Tensor, ref, max_rel=2.0 ** -7, mean_rel=2e-4):
    got = got.float().cpu().numpy()
    ref = ref.float().cpu().numpy() if isinstance(ref, torch.Tensor) else ref
    scale = float(np.abs(ref).max()) or 1.0
    diff = np.abs(got.astype(np.float64) - ref)
    assert diff.max() <= max_rel * scale, (diff.max(), scale)
    assert diff.mean() <= mean_rel * scale, (diff.mean(), scale)


def make_layer(shape, seed, **kw):
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              shape.norm_topk_prob, **kw).to(device=DEV, dtype=torch.bfloat16)
    w13, w2 = wl.expert_weights(shape, seed=seed, num_local=layer.num_local_experts,
                                first_expert=max(layer.expert_start, 0))
    gate = wl.gate_weight(shape, seed=seed + 1).to(torch.bfloat16)
    with torch.no_grad():
        layer.gate.weight.copy_(gate)
        layer.gate_up_proj.copy_(w13)
        layer.down_proj.copy_(w2)
    return layer, w13, w2, gate


def gpu_logits(layer, x):
    """The layer's own router logits (bf16 gate GEMM on the GPU) and torch's
    CUDA softmax of them, for the oracle's routing."""
    logits = layer.gate(x.to(DEV))
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    return logits.float().cpu().numpy(), probs.cpu().numpy()


@pytest.fixture(autouse=True)
def clean_status():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0


SMALL = wl.LayerShape("small", 128, 256, 8, 2)
A = wl.QWEN3_30B_A3B


@pytest.mark.parametrize("tokens,engine", [(1, "auto"), (4, "auto"), (16, "auto"), (17, "auto"),
                                           (32, "auto"), (16, "stream"), (32, "stream"),
                                           (16, "tcgen05-wide"), (32, "tcgen05-wide")])
@torch.inference_mode()
def test_decode_cuda_graph_replays_changed_inputs(tokens, engine):
    """A replayed graph runs its kernels back to back with programmatic
    dependent launch, so every kernel's reads of its predecessor's outputs must
    sit behind its dependency wait; eager runs rarely overlap and miss this."""
    layer, *_ = make_layer(SMALL, 17, graph_safe_decode=True)
    layer.expert_engine = engine
    hidden = wl.hidden_states(tokens, 128, seed=1).to(DEV)
    first, second = hidden.clone(), wl.hidden_states(tokens, 128, seed=2).to(DEV)
    expected_first, expected_second = layer(first), layer(second)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        layer(hidden)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        output = layer(hidden)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(output, expected_first)
    hidden.copy_(second)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(output, expected_second)
    assert not torch.equal(expected_first, expected_second)


@torch.inference_mode()
def test_layer_matches_oracle_config1_shape_and_counters():
    layer, w13, w2, gate = make_layer(A, 31)
    x = wl.hidden_states(64, A.hidden, seed=33)
    out = layer(x.to(DEV))
    logits, probs = gpu_logits(layer, x)
    ref = mo.moe_forward(x.float().numpy(), logits, w13.float().numpy(), w2.float().numpy(), 8,
                         True, probs=probs)
    close(out, ref["output"])
    assert layer.dispatch_assignment_count == 64 * 8
    assert layer.total_assignment_count == 64 * 8


@torch.inference_mode()
def test_capacity_counters_match_oracle():
    layer, w13, w2, gate = make_layer(A, 41, expert_capacity_factor=0.5)
    x = wl.hidden_states(256, A.hidden, seed=43)
    out = layer(x.to(DEV))
    logits, probs = gpu_logits(layer, x)
    cap = mo.capacity_of(256, 8, 128, None, 0.5)
    ref = mo.moe_forward(x.float().numpy(), logits, w13.float().numpy(), w2.float().numpy(), 8,
                         True, capacity=cap, probs=probs)
    close(out, ref["output"])
    kept = int(ref["keep"].sum())
    assert layer.dispatch_assignment_count == kept
    assert layer.dropped_assignment_count == 256 * 8 - kept > 0


@pytest.mark.parametrize("tokens", [1, 4, 16, 17, 32])
@torch.inference_mode()
def test_static_decode_matches_dynamic_local_expert_shards(tokens):
    hidden = wl.hidden_states(tokens, 128, seed=100 + tokens).to(DEV)
    shape = wl.LayerShape("shard", 128, 256, 128, 8)
    for ep_rank in range(4):
        module, *_ = make_layer(shape, 5, ep_rank=ep_rank, ep_size=4)
        weights, experts = module._route(hidden)
        dynamic, dynamic_count = module._execute_local(hidden, weights, experts)
        module.graph_safe_decode = True
        static, static_count = module._execute_local(hidden, weights, experts)
        assert static_count == dynamic_count
        assert torch.equal(static, dynamic)


@torch.inference_mode()
def test_ep_shard_partials_sum_to_unsharded_layer():
    # Simulated EP=2 on one GPU (reference tests/test_moe_kernel.py:64-86).
    full, *_ = make_layer(SMALL, 21)
    x = wl.hidden_states(22, 128, seed=23).to(DEV)
    weights, experts = full._route(x)
    reference, count = full._execute_local(x, weights, experts)
    parts, total = [], 0
    for rank in range(2):
        shard = ExpertParallelMoE(128, 256, 8, 2, True, rank, 2).to(device=DEV,
                                                                   dtype=torch.bfloat16)
        with torch.no_grad():
            shard.gate.weight.copy_(full.gate.weight)
            shard.gate_up_proj.copy_(full.gate_up_proj[4 * rank:4 * rank + 4])
            shard.down_proj.copy_(full.down_proj[4 * rank:4 * rank + 4])
        out, n = shard._execute_local(x, weights, experts)
        parts.append(out.float())
        total += n
    assert total == count == 22 * 2
    close(parts[0] + parts[1], reference.float())


@torch.inference_mode()
def test_expert_with_more_than_one_tile_and_graph():
    module, *_ = make_layer(SMALL, 132)
    hidden = wl.hidden_states(300, 128, seed=3).to(DEV)
    selected = torch.tensor([0, 1], device=DEV).expand(300, 2)
    weights = torch.full((300, 2), 0.5, device=DEV, dtype=torch.bfloat16)
    dynamic, _ = module._forward_triton(hidden, weights, selected)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        module._forward_static_decode(hidden, weights, selected)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        replayed, _ = module._forward_static_decode(hidden, weights, selected)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(replayed, dynamic)
    hidden.copy_(wl.hidden_states(300, 128, seed=4).to(DEV))
    expected, _ = module._forward_triton(hidden, weights, selected)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(replayed, expected)


@pytest.mark.parametrize("static_decode", [False, True])
@torch.inference_mode()
def test_moe_combine_is_exactly_repeatable(static_decode):
    module, *_ = make_layer(wl.LayerShape("rep", 128, 256, 8, 8), 17)
    hidden = wl.hidden_states(16, 128, seed=5).to(DEV)
    selected = torch.arange(8, device=DEV).expand(16, 8)
    weights = torch.full((16, 8), 0.125, device=DEV, dtype=torch.bfloat16)
    forward = module._forward_static_decode if static_decode else module._forward_triton
    outputs = [forward(hidden, weights, selected)[0] for _ in range(8)]
    assert all(torch.equal(o, outputs[0]) for o in outputs[1:])


def test_route_order_combine_handles_missing_and_permuted_routes():
    torch.manual_seed(23)
    module = ExpertParallelMoE(32, 64, 8, 4, True)
    packed = torch.randn(9, 32, dtype=torch.bfloat16)
    route_rows = torch.tensor([3, 0, 9, 7, 2, 9, 8, 1, 4, 9, 6, 5], dtype=torch.int32)
    expected = torch.cat((packed, torch.zeros_like(packed[:1])))[route_rows.long()].reshape(
        3, 4, 32).float().sum(dim=1).bfloat16()
    actual = module._combine_expert_routes(packed.to(DEV), route_rows.to(DEV), 3, 4)
    assert torch.equal(actual.cpu(), expected)


def test_fp32_and_fp64_combine_precision_modes(monkeypatch):
    monkeypatch.setenv("NANOVLLM_EXPERIMENTAL_FP32_EP_REDUCE", "1")
    module = ExpertParallelMoE(16, 32, 8, 2, True, ep_rank=0, ep_size=4)
    y = torch.tensor([[1.0] * 16, [0.00390625] * 16], dtype=torch.bfloat16, device=DEV)
    out = module._combine_expert_routes(y, torch.tensor([0, 1], dtype=torch.int32, device=DEV),
                                        1, 2)
    assert out.dtype == torch.float32
    assert torch.equal(out.cpu(), torch.full((1, 16), 1.00390625))
    monkeypatch.delenv("NANOVLLM_EXPERIMENTAL_FP32_EP_REDUCE")
    monkeypatch.setenv("NANOVLLM_EXPERIMENTAL_FP64_MOE_COMBINE", "1")
    module = ExpertParallelMoE(16, 32, 8, 8, True, ep_rank=0, ep_size=4)
    values = torch.tensor([0.043701171875, 0.037109375, -0.0047607421875, -0.00506591796875,
                           -4.423782229423523e-09, -0.001953125, 0.005859375,
                           -0.01068115234375], dtype=torch.bfloat16)
    values = values.unsqueeze(1).expand(8, 16).contiguous()
    out = module._combine_expert_routes(values.to(DEV), torch.arange(8, dtype=torch.int32,
                                                                     device=DEV), 1, 8)
    assert out.dtype == torch.float64
    assert torch.equal(out.cpu(), values.double().sum(dim=0, keepdim=True))


def test_cuda_route_mapping_replays_changed_input():
    layer = ExpertParallelMoE(16, 32, 4, 2, True, ep_rank=0, ep_size=2,
                              expert_owners=[0, 1, 1, 0]).to(DEV)
    routes = torch.tensor([-1, 0, 1, 2, 3, 4], device=DEV)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        mask, local_ids = layer._local_routes(routes)
    for values, expected_mask, expected_ids in (
        ([-1, 0, 1, 2, 3, 4], [False, True, False, False, True, False], [0, 1]),
        ([4, 1, 3, 0, 2, -1], [False, False, True, True, False, False], [1, 0]),
    ):
        routes.copy_(torch.tensor(values, device=DEV))
        graph.replay()
        torch.cuda.synchronize()
        assert mask.tolist() == expected_mask
        assert local_ids[mask].tolist() == expected_ids


@torch.inference_mode()
def test_relocate_experts_single_rank_keeps_storage():
    layer, *_ = make_layer(SMALL, 9, dynamic_placement=True)
    ptr = layer.gate_up_proj.data_ptr()
    x = wl.hidden_states(12, 128, seed=1).to(DEV)
    before = layer(x)
    assert layer.relocate_experts(tuple(range(1)) * 8) == 0
    assert layer.gate_up_proj.data_ptr() == ptr
    assert torch.equal(layer(x), before)


@pytest.mark.parametrize("tokens", [1, 2])
@pytest.mark.parametrize("placement", ["full", "shard", "round_robin"])
@torch.inference_mode()
def test_tiny_decode_path_matches_unfused_streaming_path(tokens, placement):
    kw = {"full": {}, "shard": dict(ep_rank=1, ep_size=2),
          "round_robin": dict(ep_rank=1, ep_size=2,
                              expert_owners=tuple(e % 2 for e in range(128)))}[placement]
    layer = ExpertParallelMoE(A.hidden, A.intermediate, A.num_experts, A.top_k, True,
                              **kw).to(device=DEV, dtype=torch.bfloat16)
    w13, w2 = wl.expert_weights(A, seed=61, device=DEV, on_device=True)
    local = list(layer.local_expert_ids)
    with torch.no_grad():
        layer.gate.weight.copy_(wl.gate_weight(A, seed=62).to(DEV))
        layer.gate_up_proj.copy_(w13[local])
        layer.down_proj.copy_(w2[local])
    x = wl.hidden_states(tokens, A.hidden, seed=63).to(DEV)
    for logits in (layer.gate(x), wl.uniform_logits(tokens, 128, seed=64).to(DEV)):
        calls = dict(_lib.CALL_COUNTS)
        fused = layer._forward_from_logits(x, logits)
        assert _lib.CALL_COUNTS.get("b200moe_decode_tiny", 0) == calls.get(
            "b200moe_decode_tiny", 0) + 1
        layer.expert_engine = "stream"
        unfused = layer._forward_from_logits(x, logits)
        layer.expert_engine = "auto"
        assert torch.equal(fused, unfused)
    routes = tokens * A.top_k
    assert layer.dispatch_assignment_count <= 4 * routes


@pytest.mark.parametrize("top_k,tokens", [(1, 16), (2, 8), (4, 4), (8, 2), (16, 1)])
@torch.inference_mode()
def test_tiny_decode_path_every_token_and_slot(top_k, tokens):
    """More tokens than warps in a CTA (top_k 1 and 2) and up to 16 slots."""
    shape = wl.LayerShape("tiny-k", 256, 512, 32, top_k)
    layer, *_ = make_layer(shape, 80 + top_k)
    x = wl.hidden_states(tokens, shape.hidden, seed=81).to(DEV)
    logits = wl.uniform_logits(tokens, shape.num_experts, seed=82).to(DEV)
    calls = _lib.CALL_COUNTS.get("b200moe_decode_tiny", 0)
    fused = layer._forward_from_logits(x, logits)
    assert _lib.CALL_COUNTS.get("b200moe_decode_tiny", 0) == calls + 1
    layer.expert_engine = "stream"
    assert torch.equal(fused, layer._forward_from_logits(x, logits))


@torch.inference_mode()
def test_tiny_decode_path_graph_replay():
    layer, *_ = make_layer(SMALL, 71, graph_safe_decode=True)
    hidden = wl.hidden_states(2, 128, seed=1).to(DEV)
    second = wl.hidden_states(2, 128, seed=2).to(DEV)
    expected_first, expected_second = layer(hidden.clone()), layer(second)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        layer(hidden)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        output = layer(hidden)
    hidden.copy_(second)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(output, expected_second)
    layer.expert_engine = "stream"
    assert torch.equal(layer(second), expected_second)


@torch.inference_mode()
def test_empty_batch_through_layer_and_every_entry_point():
    """A step with no tokens (an idle data-parallel rank) returns empty outputs
    through the layer on every engine and through each C-ABI call, with no
    kernel error and no device status bit."""
    from extend_nano_vllm_b200 import ops

    layer, *_ = make_layer(SMALL, 91)
    x = torch.empty((0, SMALL.hidden), device=DEV, dtype=torch.bfloat16)
    for engine in ("auto", "stream", "tcgen05-wide", "tcgen05-swap", "tcgen05-pair"):
        layer.expert_engine = engine
        out = layer(x)
        assert out.shape == (0, SMALL.hidden) and out.dtype == torch.bfloat16
    layer.expert_engine = "auto"
    logits = torch.empty((0, SMALL.num_experts), device=DEV)
    w, ids = ops.route_topk(logits, SMALL.top_k, True)
    assert w.shape == (0, SMALL.top_k) and ids.shape == (0, SMALL.top_k)
    packed = ops.pack_routes(ids, w.view(-1), SMALL.num_experts, SMALL.num_experts)
    assert packed.counters.cpu().tolist() == [0] * _lib.NUM_COUNTERS
    assert packed.expert_offsets.cpu().tolist() == [0] * (SMALL.num_experts + 1)
    for engine in (_lib.ENGINE_STREAM, _lib.ENGINE_TCGEN05_WIDE, _lib.ENGINE_TCGEN05_SWAP,
                   _lib.ENGINE_TCGEN05_PAIR):
        act = ops.expert_gate_up(engine, x, None, layer.gate_up_proj, packed, SMALL.top_k)
        y = ops.expert_down(engine, act, layer.down_proj, packed, w.view(-1))
        assert act.shape[0] == packed.row_capacity and y.shape == (0, SMALL.hidden)
    assert ops.combine(torch.empty((0, SMALL.hidden), device=DEV, dtype=torch.bfloat16),
                       None, 0, SMALL.top_k).shape == (0, SMALL.hidden)
    tiny = ops.decode_tiny(logits, x, layer.gate_up_proj, layer.down_proj, SMALL.top_k, True,
                           SMALL.num_experts)
    assert tiny.shape == (0, SMALL.hidden)
    torch.cuda.synchronize()
