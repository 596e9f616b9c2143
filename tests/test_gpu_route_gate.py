"""b200moe_route_gate_topk: the router projection fused into the routing launch.

The reference's logits are cuBLAS's bf16 F.linear (moe.py:871, linear.py:51).
The fused kernel accumulates the same products in fp32 in its own fixed order
and rounds once to bf16, so:
* its logits are within half a bf16 unit (plus fp32 summation error) of the
  exact fp64 dot product, and within one unit of cuBLAS's;
* its routing equals b200moe_route_topk of its own logits bit for bit;
* the layer with fuse_router_gate=True equals the layer fed those logits,
  eagerly and replayed from a CUDA graph, and its sync counters stay zero.
The share of tokens routed differently from the cuBLAS logits is measured
here (it is why the fusion is off by default).
"""

import json
import os

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


CASES = [(wl.QWEN3_30B_A3B, 1), (wl.QWEN3_30B_A3B, 8), (wl.QWEN3_30B_A3B, 64),
         (wl.QWEN3_235B_A22B, 5), (wl.QWEN3_235B_A22B, 64),
         (wl.LayerShape("odd", 264, 128, 40, 6), 13)]


@pytest.mark.parametrize("shape,tokens", CASES, ids=[f"{s.name}-T{t}" for s, t in CASES])
def test_fused_router_projection(shape, tokens):
    x = wl.hidden_states(tokens, shape.hidden, seed=tokens + 5).to(DEV)
    gate = wl.gate_weight(shape, seed=9).to(torch.bfloat16).to(DEV)
    w, ids, logits = ops.route_gate_topk(x, gate, shape.top_k, True)
    ref = torch.nn.functional.linear(x, gate)
    exact = (x.double() @ gate.double().T)
    torch.cuda.synchronize()
    # Both round an fp32 sum once: each is within half a bf16 unit (relative
    # 2^-8) of the exact value plus its fp32 summation error, so they are
    # within one unit of each other (fp32 error bounded by 1e-5 of the
    # largest logit; near zero the bf16 unit is tiny and that term dominates).
    noise = 1e-5 * exact.abs().max()
    err = (logits.double() - exact).abs()
    assert bool((err <= exact.abs() * 2.0 ** -8 + noise).all()), float(err.max())
    gap = (logits.double() - ref.double()).abs()
    assert bool((gap <= exact.abs() * 2.0 ** -7 + 2 * noise).all()), float(gap.max())
    w2, ids2 = ops.route_topk(logits, shape.top_k, True)
    assert torch.equal(ids, ids2) and torch.equal(w.view(torch.int16), w2.view(torch.int16))
    _, ids_ref = ops.route_topk(ref, shape.top_k, True)
    differing_logits = float((logits != ref).float().mean())
    differing_tokens = float((ids != ids_ref).any(dim=1).float().mean())
    log = os.environ.get("B200MOE_PARITY_LOG")
    if log:
        with open(log, "a") as f:
            f.write(json.dumps({"test": "route_gate", "shape": shape.name, "tokens": tokens,
                                "logits_differing_from_cublas": differing_logits,
                                "tokens_routed_differently": differing_tokens}) + "\n")
    assert differing_logits < 0.05
    assert all(int(t.abs().sum()) == 0 for t in ops._GATE_SYNC.values())


@torch.inference_mode()
def test_layer_with_fused_router_projection():
    shape = wl.QWEN3_30B_A3B
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              True, graph_safe_decode=True).to(device=DEV, dtype=torch.bfloat16)
    w13, w2 = wl.expert_weights(shape, seed=12, device=DEV, on_device=True)
    with torch.no_grad():
        layer.gate.weight.copy_(wl.gate_weight(shape, seed=13).to(DEV))
        layer.gate_up_proj.copy_(w13)
        layer.down_proj.copy_(w2)
    layer.fuse_router_gate = True
    for tokens in (1, 2, 8, 40):
        x = wl.hidden_states(tokens, shape.hidden, seed=tokens).to(DEV)
        calls = _lib.CALL_COUNTS.get("b200moe_route_gate_topk", 0)
        fused = layer(x)
        assert _lib.CALL_COUNTS.get("b200moe_route_gate_topk", 0) == calls + 1
        _, _, logits = ops.route_gate_topk(x, layer.gate.weight, shape.top_k, True)
        expected = layer._forward_from_logits(x, logits)
        torch.cuda.synchronize()
        assert torch.equal(fused, expected), tokens
    x = wl.hidden_states(8, shape.hidden, seed=100).to(DEV)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        layer(x)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = layer(x)
    for seed in (101, 102):
        x.copy_(wl.hidden_states(8, shape.hidden, seed=seed).to(DEV))
        graph.replay()
        eager = layer(x)
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    assert all(int(t.abs().sum()) == 0 for t in ops._GATE_SYNC.values())
