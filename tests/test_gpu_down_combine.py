"""The route-order combine inside the swap-AB down GEMM (small batches).

b200moe_expert_down_combine must give the bits of b200moe_expert_down
followed by b200moe_combine (slot order, fp32, bf16 store): the layer's
output with the fused form equals the same layer forced onto the two-launch
form, eagerly and replayed from a CUDA graph, and the arrival counters are
left zero for the next call.
"""

import pytest
import torch

import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import _lib, ops
from extend_nano_vllm_b200.moe import ExpertParallelMoE

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def clean_status():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0


def _layer(shape, **kw):
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              True, **kw).to(device=DEV, dtype=torch.bfloat16)
    w13, w2 = wl.expert_weights(shape, seed=41, device=DEV, on_device=True)
    with torch.no_grad():
        layer.gate.weight.copy_(wl.gate_weight(shape, seed=42).to(DEV))
        layer.gate_up_proj.copy_(w13)
        layer.down_proj.copy_(w2)
    return layer


def _split(layer, x, logits):
    """The same forward with the combine as its own launch."""
    fused = layer._fused_combine
    layer._fused_combine = lambda n: False
    try:
        return layer._forward_from_logits(x, logits)
    finally:
        layer._fused_combine = fused


@pytest.mark.parametrize("shape", [wl.QWEN3_30B_A3B, wl.QWEN3_235B_A22B,
                                   wl.LayerShape("odd", 272, 144, 40, 6)],
                         ids=lambda s: s.name)
@torch.inference_mode()
def test_fused_combine_equals_separate_combine(shape):
    layer = _layer(shape)
    for tokens in (3, 8, 17, 40, 64):
        x = wl.hidden_states(tokens, shape.hidden, seed=tokens).to(DEV)
        logits = wl.uniform_logits(tokens, shape.num_experts, seed=tokens + 1).to(DEV)
        if tokens * shape.top_k <= 16:
            continue  # the two-launch tiny path handles these
        assert layer._fused_combine(tokens)
        calls = _lib.CALL_COUNTS.get("b200moe_expert_down_combine", 0)
        fused = layer._forward_from_logits(x, logits)
        assert _lib.CALL_COUNTS.get("b200moe_expert_down_combine", 0) == calls + 1
        split = _split(layer, x, logits)
        torch.cuda.synchronize()
        assert torch.equal(fused, split), tokens
    assert all(int(t.abs().sum()) == 0 for t in ops._COMBINE_SYNC.values())


@torch.inference_mode()
def test_fused_combine_replays_from_cuda_graph():
    shape = wl.QWEN3_30B_A3B
    layer = _layer(shape, graph_safe_decode=True)
    x = wl.hidden_states(8, shape.hidden, seed=5).to(DEV)
    logits = wl.uniform_logits(8, shape.num_experts, seed=6).to(DEV)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        layer._forward_from_logits(x, logits)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = layer._forward_from_logits(x, logits)
    for seed in (7, 8, 9):
        x.copy_(wl.hidden_states(8, shape.hidden, seed=seed).to(DEV))
        logits.copy_(wl.uniform_logits(8, shape.num_experts, seed=seed + 50).to(DEV))
        graph.replay()
        expected = _split(layer, x, logits)
        torch.cuda.synchronize()
        assert torch.equal(out, expected), seed
    assert all(int(t.abs().sum()) == 0 for t in ops._COMBINE_SYNC.values())
