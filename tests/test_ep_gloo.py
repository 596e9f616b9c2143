"""Expert-parallel host logic over two gloo ranks on CPU.

Each rank holds half of the experts and its own tokens (5 and 7 tokens); the
kernels are replaced by the oracle-backed CpuOps so only the exchange logic
is under test.  Every backend must reproduce the unsharded layer applied to
the concatenated batch (the reference's global routing order: rank 0's
tokens first), including the capacity drop set.  Modelled on the reference's
tests/test_moe_all_to_all.py and tests/test_moe_dp_padding.py.
"""

import datetime
import multiprocessing as mp
import socket

import numpy as np
import pytest
import torch

SHAPE = dict(hidden=32, inter=64, experts=8, top_k=2)
COUNTS = (5, 7)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    import extend_nano_vllm_b200.workloads as wl
    shape = wl.LayerShape("ep", SHAPE["hidden"], SHAPE["inter"], SHAPE["experts"],
                          SHAPE["top_k"])
    w13, w2 = wl.expert_weights(shape, seed=11)
    gate = wl.gate_weight(shape, seed=12).bfloat16()
    return shape, w13, w2, gate


def _tokens(rank):
    import extend_nano_vllm_b200.workloads as wl
    return wl.hidden_states(COUNTS[rank], SHAPE["hidden"], seed=100 + rank)


def _layer(rank, world, backend, kw):
    from extend_nano_vllm_b200.moe import ExpertParallelMoE
    from oracle.cpu_ops import CpuOps
    shape, w13, w2, gate = _weights()
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              True, ep_rank=rank, ep_size=world, dispatch_backend=backend,
                              **kw).bfloat16()
    local = list(layer.local_expert_ids)
    with torch.no_grad():
        layer.gate.weight.copy_(gate)
        layer.gate_up_proj.copy_(w13[local])
        layer.down_proj.copy_(w2[local])
    layer._ops = CpuOps()
    return layer


def _worker(rank, port, backend, kw, queue):
    import torch.distributed as dist
    from extend_nano_vllm_b200 import dist_env
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=2,
                                rank=rank, timeout=datetime.timedelta(seconds=60))
        dist_env.set_moe_token_counts(COUNTS)
        layer = _layer(rank, 2, backend, kw)
        tokens = (torch.cat([_tokens(0), _tokens(1)]) if backend == "replicated"
                  else _tokens(rank))
        with torch.no_grad():
            out = layer(tokens)
        queue.put((rank, out.float().numpy(), layer.dispatch_assignment_count,
                   layer.dropped_assignment_count, layer.total_assignment_count,
                   layer.ep_all_to_all_count + layer.ep_all_gather_count))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        import traceback
        queue.put((rank, "error", traceback.format_exc(), None, None, None))


def _run(backend, kw):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, backend, kw, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = {}
        for _ in range(2):
            item = queue.get(timeout=120)
            results[item[0]] = item
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    for r in results.values():
        assert not isinstance(r[1], str), r[2]
    return results


@pytest.mark.timeout(300)
@pytest.mark.parametrize("backend", ["all_to_all_nvlink", "allgather_reduce",
                                     "allgather_reducescatter", "replicated"])
@pytest.mark.parametrize("kw", [dict(), dict(expert_capacity_factor=0.6)])
def test_ep_backends_match_unsharded_layer(backend, kw):
    results = _run(backend, kw)
    full = _layer(0, 1, "replicated", kw)
    with torch.no_grad():
        expected = full(torch.cat([_tokens(0), _tokens(1)])).float().numpy()
    if backend == "replicated":
        # Every rank routed the whole batch; both hold the reduced output.
        np.testing.assert_array_equal(results[0][1], results[1][1])
        np.testing.assert_allclose(results[0][1], expected, rtol=2e-2, atol=2e-3)
        assert results[0][2] + results[1][2] == full.dispatch_assignment_count
        return
    got = np.concatenate([results[0][1], results[1][1]])
    if backend == "all_to_all_nvlink":
        # Same per-route arithmetic and slot-order combine as EP=1.
        np.testing.assert_array_equal(got, expected)
    else:
        # Partial outputs are summed in bf16 by the collective.
        np.testing.assert_allclose(got, expected, rtol=2e-2, atol=2e-3)
    kept = results[0][2] + results[1][2]
    dropped = sum(COUNTS) * SHAPE["top_k"] - kept
    assert kept == full.dispatch_assignment_count
    if backend == "all_to_all_nvlink":
        assert results[0][3] + results[1][3] == full.dropped_assignment_count == dropped
        assert results[0][4] + results[1][4] == full.total_assignment_count
    if kw:
        assert dropped > 0
