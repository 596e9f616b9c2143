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


def _rank0_worker(rank, port, backend, queue):
    import torch.distributed as dist
    from extend_nano_vllm_b200 import dist_env
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=2,
                                rank=rank, timeout=datetime.timedelta(seconds=60))
        dist_env.set_moe_token_counts(None)
        layer = _layer(rank, 2, backend, {})
        with torch.no_grad():
            out = layer(_tokens(0))  # every rank holds rank 0's batch
        queue.put((rank, out.float().numpy(), layer.ep_all_to_all_count,
                   layer.ep_broadcast_count + layer.ep_all_reduce_count, None, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - reported to the parent
        import traceback
        queue.put((rank, "error", traceback.format_exc(), None, None, None))


@pytest.mark.timeout(300)
@pytest.mark.parametrize("backend", ["all_to_all", "all_to_all_reduce"])
def test_rank0_all_to_all_backends(backend):
    """The reference's rank-0 experiments (moe.py:1020-1216): EP rank 0 routes
    its tokens, experts run where they live, every rank gets rank 0's result
    (broadcast, or an all-reduce of it with zeros)."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank0_worker, args=(r, port, backend, queue))
             for r in range(2)]
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
    full = _layer(0, 1, "replicated", {})
    with torch.no_grad():
        expected = full(_tokens(0)).float().numpy()
    for r in (0, 1):
        np.testing.assert_array_equal(results[r][1], expected)
        assert results[r][2] == 3  # counts, dispatch and return all-to-alls
        assert results[r][3] == 1


def _relocate_worker(rank, port, queue, disagree):
    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=2,
                                rank=rank, timeout=datetime.timedelta(seconds=60))
        from extend_nano_vllm_b200.moe import ExpertParallelMoE
        from oracle.cpu_ops import CpuOps
        if disagree:
            layer = ExpertParallelMoE(SHAPE["hidden"], SHAPE["inter"], 4, 2, True, ep_rank=rank,
                                      ep_size=2, dynamic_placement=True).bfloat16()
            with pytest.raises(ValueError, match="same expert placement"):
                layer.relocate_experts(((0, 0, 1, 1), (0, 1, 0, 1))[rank])
            queue.put((rank, "ok"))
            dist.destroy_process_group()
            return
        shape, w13, w2, gate = _weights()
        initial = tuple(e // 4 for e in range(8))          # experts 0-3 on rank 0
        target = tuple((e + 1) % 2 for e in range(8))      # odd experts on rank 0
        layer = ExpertParallelMoE(shape.hidden, shape.intermediate, 8, 2, True, ep_rank=rank,
                                  ep_size=2, expert_owners=initial,
                                  dynamic_placement=True).bfloat16()
        local = [e for e, o in enumerate(initial) if o == rank]
        with torch.no_grad():
            layer.gate.weight.copy_(gate)
            layer.gate_up_proj.copy_(w13[local])
            layer.down_proj.copy_(w2[local])
        layer._ops = CpuOps()
        x = torch.cat([_tokens(0), _tokens(1)])
        with torch.no_grad():
            before = layer(x)
        pointers = (layer.gate_up_proj.data_ptr(), layer.down_proj.data_ptr(),
                    layer.expert_owner_tensor.data_ptr())
        with pytest.raises(ValueError, match="equal experts"):
            layer.relocate_experts((0,) * 7 + (1,))
        moved = layer.relocate_experts(target)
        now = [e for e, o in enumerate(target) if o == rank]
        ok = (moved == 4 and list(layer.local_expert_ids) == now
              and pointers == (layer.gate_up_proj.data_ptr(), layer.down_proj.data_ptr(),
                               layer.expert_owner_tensor.data_ptr())
              and torch.equal(layer.gate_up_proj.data, w13[now])
              and torch.equal(layer.down_proj.data, w2[now]))
        with torch.no_grad():
            after = layer(x)
        again = layer.relocate_experts(target)
        back = layer.relocate_experts(initial)
        with torch.no_grad():
            restored = layer(x)
        queue.put((rank, (ok, torch.equal(after, before), again, back,
                          torch.equal(restored, before))))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - reported to the parent
        import traceback
        queue.put((rank, traceback.format_exc()))


@pytest.mark.timeout(300)
@pytest.mark.parametrize("disagree", [False, True])
def test_relocate_experts_moves_rows_between_ranks(disagree):
    """Modelled on the reference's tests/test_moe_dynamic_placement.py:72-202:
    experts move between two ranks in place (same storage), the output stays
    bit-identical, repeating the placement moves nothing, and ranks that
    propose different placements fail without deadlock."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_relocate_worker, args=(r, port, queue, disagree))
             for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = dict(queue.get(timeout=120) for _ in range(2))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    for r in (0, 1):
        if disagree:
            assert results[r] == "ok", results[r]
        else:
            assert results[r] == (True, True, 0, 4, True), results[r]
