"""The shared expert inside the grouped expert path (one EP rank).

The reference adds a shared expert after the routed output
(nanovllm/layers/moe.py:1259-1262): output + sigmoid(gate(x)) * MLP(x), the
MLP of moe.py:212-234, each step a bf16 torch operation.  Here the shared
expert is every token's (top_k + 1)-th route, computed by the same grouped
GEMM launches as the routed experts.  Checked on a Qwen3-Next-shaped layer
(512 experts, top-10, shared expert as wide as the routed ones) and a small one:
* routing, capacity drops and counters of the routed experts are unchanged;
* the output agrees with the reference formula within the reference's own
  tolerance for this path (benchmarks/bench_moe_shared.py: rtol 3e-2,
  atol 3e-3), and its distance to the fp32 result exceeds the reference
  formula's own distance by at most one bf16 rounding step (2^-8 of
  max|exact|);
* a captured CUDA graph replays it bit for bit.
"""

import pytest
import torch
import torch.nn.functional as F

import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import _lib
from extend_nano_vllm_b200.moe import ExpertParallelMoE

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
NEXT = wl.QWEN3_NEXT_80B_A3B
SMALL = wl.LayerShape("small-shared", 256, 128, 16, 4, shared_intermediate=128)


@pytest.fixture(autouse=True)
def clean_status():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0


_LAYERS = {}


def make_layer(shape, seed=23, **kw):
    key = (shape.name, seed, tuple(sorted(kw.items())))
    if key in _LAYERS:
        return _LAYERS[key]
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              shape.norm_topk_prob,
                              shared_expert_intermediate_size=shape.shared_intermediate,
                              **kw).to(device=DEV, dtype=torch.bfloat16)
    w13, w2 = wl.expert_weights(shape, seed=seed, device=DEV, on_device=True)
    s13, s2, sg = wl.shared_expert_weights(shape, seed=seed, device=DEV)
    with torch.no_grad():
        layer.gate.weight.copy_(wl.gate_weight(shape, seed=seed + 1).to(DEV))
        layer.gate_up_proj.copy_(w13)
        layer.down_proj.copy_(w2)
        layer.shared_expert.gate_up_proj.weight.copy_(s13)
        layer.shared_expert.down_proj.weight.copy_(s2)
        layer.shared_expert_gate.weight.copy_(sg)
    _LAYERS.clear()
    _LAYERS[key] = layer
    return layer


def reference_formula(layer, x, routed):
    """moe.py:1259-1262 with the MLP of moe.py:231-234, as bf16 torch ops."""
    shared = layer.shared_expert
    gate, up = F.linear(x, shared.gate_up_proj.weight).chunk(2, dim=-1)
    projected = F.linear(F.silu(gate) * up, shared.down_proj.weight)
    return routed + torch.sigmoid(F.linear(x, layer.shared_expert_gate.weight)) * projected


def exact_output(layer, x, weights, ids):
    """fp32 routed experts for the given (post-capacity) routes plus the fp32 shared expert."""
    xf = x.float()
    out = torch.zeros_like(xf)
    inter = layer.intermediate_size
    flat_ids = ids.reshape(-1)
    flat_w = weights.reshape(-1).float()
    tokens = torch.arange(x.size(0), device=DEV).repeat_interleave(ids.size(1))
    for e in torch.unique(flat_ids).tolist():
        if e >= layer.num_experts:
            continue
        sel = flat_ids == e
        gu = xf[tokens[sel]] @ layer.gate_up_proj[e].float().T
        act = F.silu(gu[:, :inter]) * gu[:, inter:]
        y = (act @ layer.down_proj[e].float().T) * flat_w[sel, None]
        out.index_add_(0, tokens[sel], y)
    shared = layer.shared_expert
    gu = xf @ shared.gate_up_proj.weight.float().T
    act = F.silu(gu[:, :shared.intermediate_size]) * gu[:, shared.intermediate_size:]
    gate = torch.sigmoid(xf @ layer.shared_expert_gate.weight.float().T)
    return out + gate * (act @ shared.down_proj.weight.float().T)


def _counts(layer):
    return (layer.dispatch_assignment_count, layer.dropped_assignment_count,
            layer.total_assignment_count)


CASES = [(SMALL, 1, {}), (SMALL, 5, {}), (SMALL, 64, {}), (SMALL, 300, {"expert_capacity": 60}),
         (NEXT, 1, {}), (NEXT, 16, {}), (NEXT, 32, {}), (NEXT, 512, {}),
         (NEXT, 4096, {"expert_capacity_factor": 1.25})]


@pytest.mark.parametrize("shape,tokens,kw", CASES,
                         ids=[f"{s.name}-T{t}-{'cap' if k else 'nocap'}" for s, t, k in CASES])
@torch.inference_mode()
def test_fused_shared_expert_matches_reference_formula(shape, tokens, kw):
    layer = make_layer(shape, **kw)
    x = wl.hidden_states(tokens, shape.hidden, seed=tokens + 7).to(DEV)
    assert layer._fused_shared(x)
    before = _counts(layer)
    fused = layer(x)
    torch.cuda.synchronize()
    mid = _counts(layer)
    # The reference's order: routed output first (bit-exact with the
    # reference's routed path), then the shared expert in torch.
    routed = layer._forward_local(x, shared=False)
    expected = reference_formula(layer, x, routed)
    after = _counts(layer)
    # Routed counters: the fused call counts exactly what the routed-only call counts.
    assert tuple(m - b for m, b in zip(mid, before)) == tuple(a - m for a, m in zip(after, mid))
    if kw:
        assert mid[1] > before[1], "the capacity case must drop routes"
    torch.testing.assert_close(fused, expected, rtol=3e-2, atol=3e-3)
    weights, ids = layer._route(x)
    exact = exact_output(layer, x, weights, ids)
    scale = float(exact.abs().max())
    err_fused = float((fused.float() - exact).abs().max())
    err_ref = float((expected.float() - exact).abs().max())
    assert err_fused <= err_ref + 2.0 ** -8 * scale, (err_fused, err_ref, scale)


@torch.inference_mode()
def test_fused_shared_expert_replays_from_cuda_graph():
    layer = make_layer(NEXT, graph_safe_decode=True)
    x = wl.hidden_states(16, NEXT.hidden, seed=3).to(DEV)
    layer(x)  # eager warm-up (binds the grouped storage)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        layer(x)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = layer(x)
    for seed in (11, 12):
        x.copy_(wl.hidden_states(16, NEXT.hidden, seed=seed).to(DEV))
        graph.replay()
        eager = layer(x)
        torch.cuda.synchronize()
        assert torch.equal(out, eager), seed
