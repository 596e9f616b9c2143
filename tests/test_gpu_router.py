"""Router parity against the reference's own routing arithmetic on the GPU.

The reference routes with F.softmax(fp32) + torch.topk + renormalisation
(nanovllm/layers/moe.py:872-878); on a GPU those are torch's CUDA kernels.
b200moe_route_topk and the fused tiny decode path must return the same ids
(ties included: bf16 logits tie often) and the same bf16 weight bits.
The CPU oracle's selection (oracle.moe_oracle.route_from_probs) is checked
against the same results, fed torch's CUDA probabilities.
Tolerance: none -- ids and weight bits are compared exactly.
"""

import importlib.util
import os

import numpy as np
import pytest
import torch

import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import _lib, ops
from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu
DEV = "cuda"

_spec = importlib.util.spec_from_file_location(
    "make_cuda_route_golden",
    os.path.join(os.path.dirname(__file__), "golden", "make_cuda_route_golden.py"))
route_sets = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(route_sets)


@pytest.fixture(autouse=True)
def clean_status():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0, "a kernel reported a timeout or bad index"


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


def _gate_gemm_logits() -> torch.Tensor:
    """The real model's router input: bf16 gate GEMM on the GPU -> bf16 logits."""
    a = wl.QWEN3_30B_A3B
    x = wl.hidden_states(4096, a.hidden, seed=51).to(DEV)
    gate = wl.gate_weight(a, seed=52).to(DEV).to(torch.bfloat16)
    return torch.nn.functional.linear(x, gate)


# name -> (builder of the logits, top_k); built inside the tests (no CUDA at import).
SETS = {name: (lambda v=v: v[0], v[1]) for name, v in route_sets.logit_sets().items()}
SETS.update({
    "bf16_gate_gemm_4096": (_gate_gemm_logits, 8),
    "f32_uniform_8192": (lambda: wl.uniform_logits(8192, 128, seed=53), 8),
    "f32_zipf_8192": (lambda: wl.zipf_logits(8192, 128, seed=54), 8),
    "bf16_uniform_k1": (lambda: wl.uniform_logits(512, 128, seed=55).to(torch.bfloat16), 1),
    "f16_q_e128_k8": (lambda: ((torch.randn((1024, 128), generator=torch.Generator()
                                            .manual_seed(56)) * 4).round() / 4).half(), 8),
})


@pytest.mark.parametrize("renorm", [True, False])
@pytest.mark.parametrize("name", sorted(SETS))
def test_router_matches_torch_cuda_routing_bit_exact(name, renorm):
    build, k = SETS[name]
    logits = build().to(DEV)
    probs, ref_w, ref_ids = route_sets.cuda_route(logits, k, renorm)
    w, ids = ops.route_topk(logits, k, renorm)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids.cpu().numpy())
    np.testing.assert_array_equal(_bits(w), _bits(ref_w))
    # The oracle's selection, fed the same probabilities, agrees too.
    o_w, o_ids = mo.route_from_probs(probs.cpu().numpy(), k, renorm)
    np.testing.assert_array_equal(o_ids, ref_ids.cpu().numpy())
    np.testing.assert_array_equal(mo.bf16_bits(o_w).astype(np.int16), _bits(ref_w))


def test_bf16_tie_sets_really_tie():
    """The bf16 sets exercise the tie order: a large share of their tokens
    has equal probabilities within the top k + 1."""
    for name in ("bf16_gold256", "bf16_zipf8192", "bf16_gate_gemm_4096"):
        build, k = SETS[name]
        probs = route_sets.cuda_route(build().to(DEV), k)[0].cpu().numpy()
        assert len(route_sets.tie_rows(probs, k)) >= 0.05 * probs.shape[0], name


@pytest.mark.parametrize("tokens", [1, 2])
def test_tiny_decode_routing_matches_torch_cuda_on_ties(tokens):
    """The fused two-launch decode path routes inside its kernels with the same
    routine; on tie-heavy bf16 logits its output equals the unfused path's."""
    shape = wl.LayerShape("tiny-ties", 256, 128, 128, 8)
    w13, w2 = wl.expert_weights(shape, seed=61)
    w13, w2 = w13.to(DEV), w2.to(DEV)
    golden = np.load(os.path.join(os.path.dirname(__file__), "golden", "moe_golden.npz"))
    logits = torch.from_numpy(golden["route_bf16_logits"].astype(np.int16)).view(
        torch.bfloat16).reshape(256, 128)
    probs = route_sets.cuda_route(logits, 8)[0].numpy()
    rows = route_sets.tie_rows(probs, 8)[:tokens]
    lg = logits[torch.as_tensor(rows)].contiguous().to(DEV)
    x = wl.hidden_states(tokens, shape.hidden, seed=62).to(DEV)
    out = ops.decode_tiny(lg, x, w13, w2, 8, True, 128)
    _, ref_w, ref_ids = route_sets.cuda_route(lg, 8)
    p = ops.pack_routes(ref_ids.reshape(-1).contiguous(), None, 128, 128)
    act = ops.expert_gate_up(_lib.ENGINE_STREAM, x, None, w13, p, 8)
    y = ops.expert_down(_lib.ENGINE_STREAM, act, w2, p, ref_w.reshape(-1).contiguous(), tokens)
    ref = ops.combine(y, p.combine_rows, tokens, 8)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
