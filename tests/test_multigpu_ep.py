"""Expert parallelism on two GPUs over NCCL with the native kernels.

Rank r holds experts [64r, 64r+64) of a 128-expert 30B-A3B-shaped layer and
its own tokens.  With the NVLink exchange backend every route is computed by
the same kernel arithmetic as on one GPU and combined in slot order at its
source, so the sharded output must equal the single-GPU layer bit for bit
(both sides forced onto the tcgen05 engine), eagerly and replayed from a
CUDA graph with new tokens; the all-gather backend sums bf16 partials in the
collective and is compared with the usual tolerance.
Skipped unless two GPUs are visible.
"""

import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
COUNTS = (96, 160)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _build(rank, world, backend, kw, device):
    import extend_nano_vllm_b200.workloads as wl
    from extend_nano_vllm_b200.moe import ExpertParallelMoE
    shape = wl.QWEN3_30B_A3B
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              True, ep_rank=rank, ep_size=world, dispatch_backend=backend,
                              **kw).to(device=device, dtype=torch.bfloat16)
    n = shape.num_experts // world
    w13, w2 = wl.expert_weights(shape, seed=5, num_local=n, first_expert=rank * n,
                                device=device, on_device=True)
    with torch.no_grad():
        layer.gate.weight.copy_(wl.gate_weight(shape, seed=6).to(device))
        layer.gate_up_proj.copy_(w13)
        layer.down_proj.copy_(w2)
    layer.expert_engine = "tcgen05"
    return layer


def _tokens(rank, device, step=0):
    import extend_nano_vllm_b200.workloads as wl
    return wl.hidden_states(COUNTS[rank], 2048, seed=50 + rank + 10 * step, device=device)


def _worker(rank, port, backend, kw, queue):
    import torch.distributed as dist
    from extend_nano_vllm_b200 import dist_env
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        device = torch.device("cuda", rank)
        torch.cuda.set_device(device)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=2,
                                rank=rank, device_id=device,
                                timeout=datetime.timedelta(seconds=120))
        dist_env.set_moe_token_counts(COUNTS)
        layer = _build(rank, 2, backend, kw, device)
        with torch.no_grad():
            out = layer(_tokens(rank, device))
        torch.cuda.synchronize()
        replays = []
        if backend == "all_to_all_nvlink":
            # The exchange captured in a CUDA graph, replayed with new tokens.
            x = _tokens(rank, device).clone()
            graph = torch.cuda.CUDAGraph()
            with torch.no_grad():
                with torch.cuda.graph(graph):
                    static_out = layer(x)
                for step in range(2):
                    x.copy_(_tokens(rank, device, step + 1))
                    graph.replay()
                    torch.cuda.synchronize()
                    replays.append(static_out.float().cpu().numpy())
            del graph
        from extend_nano_vllm_b200 import device_status
        queue.put((rank, out.float().cpu().numpy(), layer.dispatch_assignment_count,
                   layer.dropped_assignment_count, device_status(), replays))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - reported to the parent
        import traceback
        queue.put((rank, "error", traceback.format_exc(), None, None, None))


@pytest.mark.timeout(600)
@pytest.mark.parametrize("backend,kw", [("all_to_all_nvlink", {}),
                                        ("all_to_all_nvlink", {"expert_capacity_factor": 1.0}),
                                        ("allgather_reducescatter", {})])
def test_two_gpu_expert_parallel_matches_one_gpu(backend, kw):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, backend, kw, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            item = queue.get(timeout=300)
            results[item[0]] = item
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    for r in results.values():
        assert not isinstance(r[1], str), r[2]
        assert r[4] == 0
    device = torch.device("cuda", 0)
    full = _build(0, 1, "replicated", kw, device)
    with torch.no_grad():
        expected = full(torch.cat([_tokens(0, device), _tokens(1, device)])).float().cpu().numpy()
    got = np.concatenate([results[0][1], results[1][1]])
    assert results[0][2] + results[1][2] == full.dispatch_assignment_count
    if backend == "all_to_all_nvlink":
        np.testing.assert_array_equal(got, expected)
        assert results[0][3] + results[1][3] == full.dropped_assignment_count
        for step in range(2):
            with torch.no_grad():
                want = full(torch.cat([_tokens(0, device, step + 1),
                                       _tokens(1, device, step + 1)])).float().cpu().numpy()
            np.testing.assert_array_equal(
                np.concatenate([results[0][5][step], results[1][5][step]]), want)
    else:
        scale = float(np.abs(expected).max())
        assert np.abs(got - expected).max() <= 1e-2 * scale
