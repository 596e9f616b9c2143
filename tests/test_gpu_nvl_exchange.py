"""The NVLink expert-parallel exchange, all ranks on one GPU.

Every rank's exchange buffer lives on this device and every rank's "peer"
pointers are plain local addresses, so the same kernels run as on several
GPUs.  The ranks' phases run in turn (all ranks route, then all dispatch,
then all compute, then all finish): each wait is already satisfied when it
starts, so no kernel ever waits for one launched after it.

Each rank's output must equal, bit for bit, the single-GPU layer applied to
the concatenation of all ranks' tokens (rank-major: the reference's global
routing order), with and without a capacity limit, eagerly and replayed
from one CUDA graph per exchange with changed inputs.
"""

import numpy as np
import pytest
import torch

import extend_nano_vllm_b200.workloads as wl
from extend_nano_vllm_b200 import _lib, dist_env
from extend_nano_vllm_b200.ep import NvlinkExchange
from extend_nano_vllm_b200.moe import ExpertParallelMoE
from extend_nano_vllm_b200.nvl import ExchangeBuffers

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
SHAPE = wl.QWEN3_30B_A3B


@pytest.fixture(autouse=True)
def clean_status():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0, "a kernel reported a timeout or bad index"
    dist_env.set_moe_token_counts(None)


def _layers(world, kw, owners=None):
    full = ExpertParallelMoE(SHAPE.hidden, SHAPE.intermediate, SHAPE.num_experts, SHAPE.top_k,
                             True, **kw).to(device=DEV, dtype=torch.bfloat16)
    w13, w2 = wl.expert_weights(SHAPE, seed=31, device=DEV, on_device=True)
    gate = wl.gate_weight(SHAPE, seed=32).to(DEV)
    with torch.no_grad():
        full.gate.weight.copy_(gate)
        full.gate_up_proj.copy_(w13)
        full.down_proj.copy_(w2)
    ranks = []
    for r in range(world):
        layer = ExpertParallelMoE(SHAPE.hidden, SHAPE.intermediate, SHAPE.num_experts,
                                  SHAPE.top_k, True, ep_rank=r, ep_size=world,
                                  dispatch_backend="all_to_all_nvlink", expert_owners=owners,
                                  **kw).to(device=DEV, dtype=torch.bfloat16)
        local = list(layer.local_expert_ids)
        with torch.no_grad():
            layer.gate.weight.copy_(gate)
            layer.gate_up_proj.copy_(w13[local])
            layer.down_proj.copy_(w2[local])
        ranks.append(layer)
    return full, ranks


def _buffers(ranks, max_tokens):
    bufs = [ExchangeBuffers(ep_size=len(ranks), rank=r, max_tokens=max_tokens,
                            top_k=SHAPE.top_k, num_experts=SHAPE.num_experts,
                            num_local_experts=ranks[0].num_local_experts, hidden=SHAPE.hidden,
                            device=DEV) for r in range(len(ranks))]
    for b in bufs:
        b.connect_local(bufs)
    return bufs


def _exchange(ranks, bufs, xs):
    steps = [NvlinkExchange(layer, x, b) for layer, x, b in zip(ranks, xs, bufs)]
    for s in steps:
        s.route()
    for s in steps:
        s.dispatch()
    for s in steps:
        s.compute()
    return [s.finish() for s in steps]


CASES = [(2, (96, 160), {}), (4, (64, 1, 0, 300), {}), (2, (512, 512), {}),
         (2, (1536, 1024), {}),  # > 4096 received routes per rank: wide tiles
         (4, (200, 100, 50, 25), {"expert_capacity_factor": 1.0}),
         (2, (64, 200), {"expert_capacity": 12}), (8, (16,) * 8, {})]


@pytest.mark.parametrize("mode", ["epilogue-return", "copy-return", "device-sizes"])
@pytest.mark.parametrize("world,counts,kw", CASES)
@torch.inference_mode()
def test_exchange_matches_single_gpu_layer(world, counts, kw, mode, monkeypatch):
    """Returned rows written by the down GEMM into the sources' buffers
    (default) or copied there afterwards; eager temporaries sized exactly
    (default) or from host bounds with the received count on the device."""
    from extend_nano_vllm_b200 import ops
    monkeypatch.setattr(ops, "NVL_DIRECT_RETURN", mode != "copy-return")
    full, ranks = _layers(world, kw)
    for layer in ranks:
        layer.nvl_eager_device_sizes = mode == "device-sizes"
    bufs = _buffers(ranks, max(counts))
    dist_env.set_moe_token_counts(counts)
    for step in range(2):  # the second call reuses the buffers (epoch 2)
        xs = [wl.hidden_states(c, SHAPE.hidden, seed=70 + 10 * step + r).to(DEV)
              for r, c in enumerate(counts)]
        outs = _exchange(ranks, bufs, xs)
        expected = full(torch.cat(xs))
        torch.cuda.synchronize()
        got = torch.cat(outs)
        assert torch.equal(got, expected), float((got.float() - expected.float()).abs().max())
    assert sum(r.dispatch_assignment_count for r in ranks) == full.dispatch_assignment_count
    assert sum(r.dropped_assignment_count for r in ranks) == full.dropped_assignment_count
    if kw:
        assert full.dropped_assignment_count > 0


@torch.inference_mode()
def test_exchange_round_robin_placement():
    world = 4
    owners = tuple(e % world for e in range(SHAPE.num_experts))
    full, ranks = _layers(world, {}, owners)
    bufs = _buffers(ranks, 128)
    xs = [wl.hidden_states(128, SHAPE.hidden, seed=90 + r).to(DEV) for r in range(world)]
    outs = _exchange(ranks, bufs, xs)
    expected = full(torch.cat(xs))
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(outs), expected)


@pytest.mark.parametrize("kw", [{}, {"expert_capacity_factor": 1.25}])
@pytest.mark.parametrize("counts", [(32, 32, 32, 32), (8, 64, 1, 40)])
@torch.inference_mode()
def test_exchange_replays_from_one_cuda_graph(kw, counts):
    """All ranks' phases captured into one graph; replays with new inputs
    (device-side counts, no host reads) equal the single-GPU layer.  Ranks
    may hold different batch sizes in the same captured step: nothing in
    the exchange needs equal sizes, only the coordinated counts that bound
    the temporaries."""
    world = len(counts)
    full, ranks = _layers(world, kw)
    bufs = _buffers(ranks, max(counts))
    dist_env.set_moe_token_counts(counts)
    xs = [torch.empty((c, SHAPE.hidden), device=DEV, dtype=torch.bfloat16) for c in counts]
    for r, x in enumerate(xs):
        x.copy_(wl.hidden_states(counts[r], SHAPE.hidden, seed=5 + r))
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        _exchange(ranks, bufs, xs)  # eager warm-up
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = _exchange(ranks, bufs, xs)
    for step in range(3):
        for r, x in enumerate(xs):
            x.copy_(wl.hidden_states(counts[r], SHAPE.hidden, seed=100 + 10 * step + r).to(DEV))
        graph.replay()
        expected = full(torch.cat(xs))
        torch.cuda.synchronize()
        assert torch.equal(torch.cat(outs), expected), step


@torch.inference_mode()
def test_exchange_graph_sized_by_peer_token_bound():
    """Without coordinated counts, a per-peer token bound
    (nvl_graph_peer_tokens) sizes the captured temporaries, so ranks holding
    different batch sizes replay one step correctly (the ranks' graphs need
    not agree on sizes)."""
    counts = (8, 64, 1, 40)
    world = len(counts)
    full, ranks = _layers(world, {})
    for layer in ranks:
        layer.nvl_graph_peer_tokens = max(counts)
    bufs = _buffers(ranks, max(counts))
    dist_env.set_moe_token_counts(None)
    xs = [wl.hidden_states(c, SHAPE.hidden, seed=7 + r).to(DEV) for r, c in enumerate(counts)]
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        _exchange(ranks, bufs, xs)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = _exchange(ranks, bufs, xs)
    for step in range(2):
        for r, x in enumerate(xs):
            x.copy_(wl.hidden_states(counts[r], SHAPE.hidden, seed=200 + 10 * step + r).to(DEV))
        graph.replay()
        expected = full(torch.cat(xs))
        torch.cuda.synchronize()
        assert torch.equal(torch.cat(outs), expected), step
