"""Parity against the reference's own GPU path (its Triton kernels), run on
the same inputs in the same process.

The unmodified reference is installed into baseline/_ref by
baseline/install_reference.sh; without it these tests skip.  For each case:
  * routing: the reference's _route (torch CUDA softmax/top-k, capacity) and
    b200moe_route_topk + b200moe_pack_routes give identical ids, bf16
    weight bits and dropped sets;
  * packed layouts: the row_ids / expert_ids / num_tokens_post_padded that the
    reference's _forward_static_decode (moe.py:783-868) and _forward_triton
    (moe.py:680-771) hand to their grouped GEMM equal this library's
    row_route / tile_expert / padded-row count, bit for bit;
  * outputs: the layer output of this library equals the output of both
    reference Triton paths bit for bit (measured on B200 for every case
    below, the 235B-shaped layer at T=4096 included).  Both are also compared
    with the CPU oracle (same rounding points, fp32 accumulation in another
    order), and the measured differences are logged; the oracle tolerance is
    the reference kernel's own distance to the oracle, which this library
    therefore matches exactly.
"""

import functools
import importlib
import json
import os
import sys

import numpy as np
import pytest
import torch

import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import _lib, ops
from extend_nano_vllm_b200.moe import ExpertParallelMoE
from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(REPO, "baseline", "_ref")


@functools.lru_cache(maxsize=1)
def reference_moe():
    """nanovllm.layers.moe from baseline/_ref, or None when not installed."""
    if not os.path.isdir(os.path.join(REF_DIR, "nanovllm")):
        return None
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    try:
        return importlib.import_module("nanovllm.layers.moe")
    except Exception as exc:  # noqa: BLE001 - report why the reference is unusable
        pytest.skip(f"reference in baseline/_ref does not import: {exc!r}")


@pytest.fixture(autouse=True)
def clean_status():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0


def _layers(shape, seed, **kw):
    ref_moe = reference_moe()
    if ref_moe is None:
        pytest.skip("reference not installed in baseline/_ref (baseline/install_reference.sh)")
    w13, w2 = wl.expert_weights(shape, seed=seed, device=DEV, on_device=True)
    gate = wl.gate_weight(shape, seed=seed + 1).to(torch.bfloat16).to(DEV)
    ours = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                             True, **kw).to(device=DEV, dtype=torch.bfloat16)
    ref = ref_moe.ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts,
                                    shape.top_k, True, **kw).to(device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        for layer in (ours, ref):
            layer.gate.weight.copy_(gate)
            layer.gate_up_proj.copy_(w13)
            layer.down_proj.copy_(w2)
    return ours, ref, w13, w2


def _capture_gemm_args(ref):
    """Record the layout arguments of the reference's grouped GEMM calls."""
    seen = []
    original = ref._run_grouped_gemm

    def spy(a, b, row_ids, expert_ids, routing_weights=None, **kw):
        ntpp = kw.get("num_tokens_post_padded")
        seen.append((row_ids.clone(), expert_ids.clone(),
                     None if ntpp is None else int(ntpp)))
        return original(a, b, row_ids, expert_ids, routing_weights, **kw)

    ref._run_grouped_gemm = spy
    return seen


def _err(got: torch.Tensor, ref: np.ndarray) -> tuple[float, float]:
    d = np.abs(got.float().cpu().numpy().astype(np.float64) - ref.astype(np.float64))
    return float(d.max()), float(d.mean())


def _record(name: str, stats: dict) -> None:
    """Append the measured errors to $B200MOE_PARITY_LOG (a JSON-lines file)."""
    path = os.environ.get("B200MOE_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": name, **stats}) + "\n")


CASES = [
    # (name, shape, tokens, logits kind, capacity factor, our engine)
    ("small_T22", wl.LayerShape("small", 128, 256, 8, 2), 22, "gate", None, "auto"),
    ("a30b_T8", wl.QWEN3_30B_A3B, 8, "gate", None, "auto"),
    ("a30b_T64", wl.QWEN3_30B_A3B, 64, "gate", None, "auto"),
    ("a30b_T512", wl.QWEN3_30B_A3B, 512, "gate", None, "auto"),
    ("a30b_T8192_zipf_cap", wl.QWEN3_30B_A3B, 8192, "zipf", 1.25, "auto"),
    ("d235b_T512_swap", wl.QWEN3_235B_A22B, 512, "gate", None, "tcgen05-swap"),
    ("d235b_T512_pair", wl.QWEN3_235B_A22B, 512, "gate", None, "tcgen05-pair"),
    ("d235b_T4096_wide", wl.QWEN3_235B_A22B, 4096, "gate", None, "auto"),
    ("d235b_T4096_pair", wl.QWEN3_235B_A22B, 4096, "gate", None, "tcgen05-pair"),
    ("d235b_T4096_tall", wl.QWEN3_235B_A22B, 4096, "gate", None, "tcgen05-tall"),
    ("a30b_T8192_zipf_cap_tall", wl.QWEN3_30B_A3B, 8192, "zipf", 1.25, "tcgen05-tall"),
]


@pytest.mark.parametrize("name,shape,tokens,kind,factor,engine", CASES,
                         ids=[c[0] for c in CASES])
@torch.inference_mode()
def test_matches_reference_triton_path(name, shape, tokens, kind, factor, engine):
    kw = {} if factor is None else {"expert_capacity_factor": factor}
    ours, ref, w13, w2 = _layers(shape, 700 + tokens, **kw)
    ours.expert_engine = engine
    x = wl.hidden_states(tokens, shape.hidden, seed=800 + tokens).to(DEV)
    if kind == "zipf":
        logits = wl.zipf_logits(tokens, shape.num_experts, seed=801).to(DEV)
        ref.gate.forward = lambda h, _l=logits: _l  # inject fp32 logits into both
        ours.gate.forward = lambda h, _l=logits: _l
    else:
        logits = ours.gate(x)

    # Routing (with capacity): the reference's _route against ours.
    ref_w, ref_ids = ref._route(x)
    w, ids = ops.route_topk(logits, shape.top_k, True)
    cap = ours._capacity(tokens)
    packed = ops.pack_routes(ids.view(-1), w.view(-1), shape.num_experts, shape.num_experts,
                             capacity=cap)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids.cpu().numpy())
    assert torch.equal(w.view(torch.int16), ref_w.view(torch.int16))

    # Packed layouts of both reference paths.
    seen = _capture_gemm_args(ref)
    ref_static, _ = ref._forward_static_decode(x, ref_w, ref_ids)
    ref_dyn, _ = ref._forward_triton(x, ref_w, ref_ids)
    torch.cuda.synchronize()
    static_rows, static_tiles, ntpp = seen[0]
    dyn_rows, dyn_tiles, _ = seen[2]
    total = int(packed.counters[_lib.CNT_PADDED_ROWS])
    assert ntpp == total
    np.testing.assert_array_equal(packed.row_route[:static_rows.numel()].cpu().numpy(),
                                  static_rows.cpu().numpy())
    np.testing.assert_array_equal(packed.tile_expert[:static_tiles.numel()].cpu().numpy(),
                                  static_tiles.cpu().numpy())
    routes = ids.numel()
    rr = packed.row_route[:total].cpu().numpy()
    np.testing.assert_array_equal(np.where(rr < routes, rr // shape.top_k, tokens),
                                  dyn_rows.cpu().numpy())
    np.testing.assert_array_equal(packed.tile_expert[:total // 16].cpu().numpy(),
                                  dyn_tiles.cpu().numpy())

    # Outputs: ours (through the layer), the reference's two Triton paths,
    # and the CPU oracle over the same routing.
    out = ours(x)
    torch.cuda.synchronize()
    probs = torch.softmax(logits.float(), dim=-1, dtype=torch.float32).cpu().numpy()
    oracle = mo.moe_forward(x.float().cpu().numpy(), logits.float().cpu().numpy(),
                            w13.cpu(), w2.cpu(), shape.top_k, True, capacity=cap,
                            probs=probs)["output"]
    scale = float(np.abs(oracle).max())
    ours_max, ours_mean = _err(out, oracle)
    stat_max, stat_mean = _err(ref_static, oracle)
    dyn_max, dyn_mean = _err(ref_dyn, oracle)
    vs_ref_max, vs_ref_mean = _err(out, ref_static.float().cpu().numpy())
    stats = dict(scale=scale, ours_max=ours_max, ours_mean=ours_mean,
                 triton_static_max=stat_max, triton_static_mean=stat_mean,
                 triton_dyn_max=dyn_max, triton_dyn_mean=dyn_mean,
                 ours_vs_triton_max=vs_ref_max, ours_vs_triton_mean=vs_ref_mean,
                 ours_bits_equal_triton=bool(torch.equal(out, ref_static)))
    _record(name, stats)
    print(name, json.dumps(stats))
    assert torch.equal(out, ref_static), stats
    assert torch.equal(out, ref_dyn), stats
    # And the reference kernel itself sits within 2^-7 of the output scale of
    # the oracle (its bf16 rounding points are the oracle's).
    assert max(stat_max, dyn_max) <= scale * 2.0 ** -7, stats
