#!/usr/bin/env python
"""MoE-layer throughput of the B200 expert path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

Headline workload (all N): the Qwen3-235B-A22B-shaped MoE layer (hidden 4096,
128 experts, top-8, moe_intermediate 1536, bf16, weights N(0, 0.02)) with
T = 4096 tokens per GPU; experts sharded over the N GPUs (128/N each) with
the NCCL all-to-all backend for N > 1.  A step is one layer forward (router
projection, softmax top-k, packing, grouped gate/up + SwiGLU, grouped down,
exchange, combine) over that GPU's 4096 tokens.  ``value`` = tokens of all
ranks per second with inputs resident in HBM; ``e2e`` adds, every step, the
pinned host->device copy of the hidden states and the device->host copy of
the output (on copy streams, overlapping the neighbouring steps' compute).
Timing: CUDA events on the launching stream, barrier +
synchronize around the timed region, max over ranks.  Expert weights
(4.83 GB / N per GPU) are larger than L2, so no extra L2 flush is needed.

At N = 1, rank 0 also reports (``sweep``) the decode buckets T in
{1, 8, 32, 64, 128, 256, 512} of the 30B-A3B layer (uniform fp32 logits, one
CUDA graph per bucket, L2 flushed before every replay by writing and then
reading 256 MB buffers) and the T=8192
chunked-prefill batch with Zipf(1.2) expert popularity and capacity factor
1.25, each against its roofline; and a CPU baseline: the reference's own
CPU algorithm (softmax/top-k and the per-expert torch loop of
nanovllm/layers/moe.py:546-580, restated in oracle/) on a bounded sample.

At N = 1 the line also carries ``reference_triton_gpu``: the unmodified
reference's own GPU path (Triton kernels, installed in baseline/_ref) timed
on the same GPU with the same workloads and timing, and the speed-ups over it.
At N > 1 it carries ``reference_ep_gpu``: the reference's all-gather +
reduce-scatter backend on the same ranks and headline workload, and one
CUDA-graph decode replay of the 30B-A3B layer at 8 and 32 tokens per rank,
the reference's all-gather + all-reduce against this library's NVLink
exchange.

``--e2e b200|reference`` runs end-to-end offline generation through the
reference's own engine instead (see e2e()).

``--impl reference`` times that CPU implementation alone on the host cores
(rank 0 only) on the same workload and prints the same line with
"impl": "reference".
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

def load_workloads():
    """extend-nano-vllm_b200/workloads.py as a standalone module: it needs only
    torch, so the reference arm can build the same inputs without importing
    the package (whose import loads the CUDA library)."""
    import importlib.util

    path = os.path.join(REPO, "extend-nano-vllm_b200", "workloads.py")
    name = "b200moe_bench_workloads"
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module  # dataclasses look their module up while the class is built
    spec.loader.exec_module(module)
    return module


METRIC = "MoE-layer tokens/s (Qwen3-235B-A22B-shaped layer, T=4096 tokens per GPU)"
UNIT = "tokens/s"
TOKENS_PER_GPU = 4096
DECODE_BUCKETS = (1, 8, 32, 64, 128, 256, 512)
PREFILL_TOKENS = 8192
# Seconds of timed CPU work the reference arm allows itself (whole steps).
REFERENCE_BUDGET_S = 120.0
# Config 1 of the benchmark list: the CPU oracle on the 30B-A3B layer, T=64.
CPU_CONFIG1_TOKENS = 64
# Timed regions at least this long are compared with the sustained bf16 peak.
SUSTAINED_REGION_S = 2.0
# DRAM bytes of one gate/up launch of the N=1 headline workload, measured by an
# ncu capture of that launch (dram__bytes_read.sum + dram__bytes_write.sum);
# 1.12x the algorithmic 3.59 GB.
GATE_UP_TRAFFIC_EP1 = 3_908_390_400 + 120_817_152


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--no-sweep", action="store_true", help="skip the N=1 decode/prefill sweep")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-reference-triton", action="store_true",
                   help="skip timing the reference's own GPU path (baseline/_ref): its Triton "
                        "path at N=1, its expert-parallel backends at N>1")
    p.add_argument("--profile-case", choices=("gemm-small", "decode", "prefill", "ep-emulated"),
                   default=None,
                   help="run a case for ncu captures and exit (no JSON line): gemm-small = "
                        "235B-shaped experts, 16 experts x 320 routed rows, 604 MB of "
                        "weights (larger than L2), --steps forwards; decode = the 30B-A3B "
                        "decode bucket of --profile-tokens tokens captured in a CUDA graph "
                        "and replayed --steps times; prefill = the T=8192 Zipf prefill "
                        "case, --steps forwards; ep-emulated = the NVLink exchange of "
                        "--profile-ep ranks (235B shape, 4096 tokens each) all on this GPU, "
                        "phase by phase, --steps exchanges")
    p.add_argument("--engine", default="auto",
                   choices=("auto", "tcgen05", "tcgen05-wide", "tcgen05-tall", "tcgen05-pair"),
                   help="expert GEMM engine of the headline layer (default: the library's choice)")
    p.add_argument("--e2e", choices=("b200", "reference"), default=None,
                   help="end-to-end offline generation through the reference's own engine "
                        "(baseline/_ref) with DP x EP = --gpus replicas, its MoE layer "
                        "('reference', all-gather backend) or this one ('b200', NVLink "
                        "exchange); prints one JSON line of decode tokens/s")
    p.add_argument("--e2e-requests", type=int, default=256)
    p.add_argument("--e2e-prompt", type=int, default=1024)
    p.add_argument("--e2e-output", type=int, default=256)
    p.add_argument("--e2e-layers", type=int, default=48)
    p.add_argument("--profile-tokens", type=int, default=1)
    p.add_argument("--profile-ep", type=int, default=8)
    p.add_argument("--profile-engine", default="auto",
                   choices=("auto", "tcgen05-wide", "tcgen05-swap", "tcgen05-pair",
                            "tcgen05-tall"),
                   help="expert engine of the gemm-small profiling case")
    return p.parse_args()


def profile_case(args) -> None:
    """Small workloads for ncu captures (see --profile-case)."""
    import extend_nano_vllm_b200.workloads as wl

    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    if args.profile_case == "decode":
        shape = wl.QWEN3_30B_A3B
        layer = build_layer(shape, 1, 0, device, graph_safe_decode=True)
        t = args.profile_tokens
        x = wl.hidden_states(t, shape.hidden, seed=300 + t, device=device)
        logits = wl.uniform_logits(t, shape.num_experts, seed=400 + t, device=device)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            layer._forward_from_logits(x, logits)
        torch.cuda.current_stream().wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            layer._forward_from_logits(x, logits)
        for _ in range(max(1, args.steps)):
            graph.replay()
        torch.cuda.synchronize()
        print(f"profile case decode T={t}: {args.steps} graph replays", flush=True)
        return
    if args.profile_case == "ep-emulated":
        # Every rank's buffers and layer on this GPU; each phase runs for all
        # ranks before the next phase starts, so every wait is already
        # satisfied (the kernels and per-rank sizes of an EP step without
        # the NVLink transfer times).
        from extend_nano_vllm_b200.ep import NvlinkExchange
        from extend_nano_vllm_b200.nvl import ExchangeBuffers

        shape, world = wl.QWEN3_235B_A22B, args.profile_ep
        ranks = [build_layer(shape, world, r, device) for r in range(world)]
        bufs = [ExchangeBuffers(ep_size=world, rank=r, max_tokens=TOKENS_PER_GPU,
                                top_k=shape.top_k, num_experts=shape.num_experts,
                                num_local_experts=shape.num_experts // world,
                                hidden=shape.hidden, device=device) for r in range(world)]
        for b in bufs:
            b.connect_local(bufs)
        xs = [wl.hidden_states(TOKENS_PER_GPU, shape.hidden, seed=1000 + r, device=device)
              for r in range(world)]
        for _ in range(max(1, args.steps)):
            steps = [NvlinkExchange(layer, x, b) for layer, x, b in zip(ranks, xs, bufs)]
            for phase in ("route", "dispatch", "compute", "finish"):
                for st in steps:
                    getattr(st, phase)()
        torch.cuda.synchronize()
        print(f"profile case ep-emulated: {world} ranks, {args.steps} exchanges", flush=True)
        return
    if args.profile_case == "prefill":
        shape = wl.QWEN3_30B_A3B
        layer = build_layer(shape, 1, 0, device, expert_capacity_factor=1.25)
        x = wl.hidden_states(PREFILL_TOKENS, shape.hidden, seed=500, device=device)
        logits = wl.zipf_logits(PREFILL_TOKENS, shape.num_experts, seed=501, device=device)
        for _ in range(max(1, args.steps)):
            layer._forward_from_logits(x, logits)
        torch.cuda.synchronize()
        print(f"profile case prefill: {args.steps} forwards", flush=True)
        return
    shape = wl.LayerShape("profile-small", 4096, 1536, 16, 8)
    layer = build_layer(shape, 1, 0, device)
    layer.expert_engine = args.profile_engine
    x = wl.hidden_states(640, shape.hidden, seed=3, device=device)
    for _ in range(max(1, args.steps)):
        layer(x)
    torch.cuda.synchronize()
    print(f"profile case {args.profile_case}: {args.steps} forwards, "
          f"{layer.dispatch_assignment_count} routes", flush=True)


def peaks() -> dict:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            data = json.load(f)
        return dict(hbm_gbs=float(data["hbm_gbs"]), bf16_tflops=float(data["bf16_tflops"]),
                    bf16_tflops_sustained=float(data.get("bf16_tflops_sustained",
                                                         data["bf16_tflops"])),
                    source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0,
                source="fallback")


# ---------------------------------------------------------------------------
# Clocks sampled with nvidia-smi during a timed region.
# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi samples every 50 ms; only those stamped inside [begin, end]
    of the timed region count (the sampler starts before the region)."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu_index = gpu_index
        self.proc = None
        self.begin_t = self.end_t = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu_index), "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.5)  # let the sampler come up before the timed region
        except OSError:
            self.proc = None

    def mark_begin(self) -> None:
        self.begin_t = datetime.datetime.now()

    def mark_end(self) -> None:
        self.end_t = datetime.datetime.now()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for line in out.strip().splitlines():
            r = [c.strip() for c in line.split(",")]
            if len(r) < 10:
                continue
            try:
                stamp = datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f")
                rows.append((stamp, float(r[2]), float(r[3]), r[6:10]))
            except ValueError:
                continue
        # Samples stamped inside the timed region; a region shorter than the
        # sampling period takes the samples closest to it (within 100 ms).
        window = "timed region"
        picked = rows
        if self.begin_t and self.end_t:
            slack = datetime.timedelta(milliseconds=20)
            picked = [x for x in rows if self.begin_t - slack <= x[0] <= self.end_t + slack]
            if not picked:
                slack = datetime.timedelta(milliseconds=100)
                picked = [x for x in rows if self.begin_t - slack <= x[0] <= self.end_t + slack]
                window = "within 100 ms of the timed region"
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = {name for x in picked for name, flag in zip(names, x[3])
                   if flag.lower().startswith("active")}
        sm = [x[1] for x in picked]
        mx = [x[2] for x in picked]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm), "window": window}


class KernelTimer:
    """CUDA events around named launches on the current stream."""

    def __init__(self) -> None:
        self.events: dict[str, list] = {}
        self.open: dict[str, torch.cuda.Event] = {}

    def begin(self, name: str) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.open[name] = ev

    def end(self, name: str) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.events.setdefault(name, []).append((self.open.pop(name), ev))

    def mean_ms(self, name: str) -> float:
        pairs = self.events.get(name, [])
        return sum(a.elapsed_time(b) for a, b in pairs) / max(1, len(pairs))

    def count(self, name: str) -> int:
        return len(self.events.get(name, []))


# ---------------------------------------------------------------------------
# Distributed setup.
# ---------------------------------------------------------------------------
def init_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world > 1 or args.gpus > 1:
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun")
    if world > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=300))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------
# Native arm.
# ---------------------------------------------------------------------------
def build_layer(shape, world, rank, device, **kw):
    import extend_nano_vllm_b200.workloads as wl
    from extend_nano_vllm_b200 import ExpertParallelMoE

    backend = "all_to_all_nvlink" if world > 1 else "replicated"
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              shape.norm_topk_prob, ep_rank=rank, ep_size=world,
                              dispatch_backend=backend, **kw)
    layer = layer.to(device=device, dtype=torch.bfloat16)
    num_local = shape.num_experts // world
    w13, w2 = wl.expert_weights(shape, seed=2024, num_local=num_local,
                                first_expert=rank * num_local, device=device, on_device=True)
    with torch.no_grad():
        layer.gate.weight.copy_(wl.gate_weight(shape, seed=2025).to(device))
        layer.gate_up_proj.copy_(w13)
        layer.down_proj.copy_(w2)
    del w13, w2
    return layer


def time_steps(fn, steps: int, warmup: int, world: int) -> float:
    """Seconds for `steps` calls, max over ranks (events on the current stream)."""
    for _ in range(warmup):
        fn()
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    stop.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(start.elapsed_time(stop) / 1e3, world)


def time_e2e(layer, x, steps: int, warmup: int, world: int) -> float:
    """Seconds for `steps` host->device->host layer calls (max over ranks)."""
    x_host = [x.cpu().pin_memory() for _ in range(2)]
    out_host = [torch.empty_like(x, device="cpu").pin_memory() for _ in range(2)]
    x_dev = [torch.empty_like(x) for _ in range(2)]
    compute = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()

    def run(n: int) -> None:
        done = [None, None]  # compute finished with x_dev[b]
        ready = torch.cuda.Event()
        h2d.wait_stream(compute)
        with torch.cuda.stream(h2d):
            x_dev[0].copy_(x_host[0], non_blocking=True)
            ready.record()
        for i in range(n):
            b = i % 2
            compute.wait_event(ready)
            out = layer(x_dev[b])
            ev = torch.cuda.Event()
            ev.record(compute)
            done[b] = ev
            if i + 1 < n:
                nb = (i + 1) % 2
                ready = torch.cuda.Event()
                with torch.cuda.stream(h2d):
                    if done[nb] is not None:
                        h2d.wait_event(done[nb])
                    x_dev[nb].copy_(x_host[nb], non_blocking=True)
                    ready.record()
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev)
                out.record_stream(d2h)
                out_host[b].copy_(out, non_blocking=True)
        compute.wait_stream(d2h)

    run(warmup)
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    run(steps)
    stop.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(start.elapsed_time(stop) / 1e3, world)


def decode_sweep(steps: int, warmup: int, pk: dict) -> list[dict]:
    import extend_nano_vllm_b200.workloads as wl
    from extend_nano_vllm_b200 import STREAM_ENGINE_MAX_ROUTES
    from extend_nano_vllm_b200.ops import TINY_MAX_ROUTES

    shape = wl.QWEN3_30B_A3B
    device = torch.device("cuda")
    layer = build_layer(shape, 1, 0, device, graph_safe_decode=True)
    # L2 flush between replays: write 256 MB (evicts everything), then read
    # another 256 MB, so that the replay starts with none of the layer's data
    # in L2 and with clean lines only.  A write-only flush leaves up to L2's
    # size of dirty lines whose write-back then lands inside the timed replay;
    # that variant is timed too and reported as "ms_dirty_l2".
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    flush_read = torch.ones(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    results = []
    for tokens in DECODE_BUCKETS:
        x = wl.hidden_states(tokens, shape.hidden, seed=300 + tokens, device=device)
        logits = wl.uniform_logits(tokens, shape.num_experts, seed=400 + tokens, device=device)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(3):
                layer._forward_from_logits(x, logits)
        torch.cuda.current_stream().wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            layer._forward_from_logits(x, logits)
        for _ in range(warmup):
            graph.replay()
        times, dirty = [], []
        for clean in (True, False):
            for _ in range(steps):
                flush.fill_(1)  # evict the previous replay's weights from L2
                if clean:
                    flush_read.amax()
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record()
                graph.replay()
                b.record()
                (times if clean else dirty).append((a, b))
        torch.cuda.synchronize()
        ms = statistics.median(a.elapsed_time(b) for a, b in times)
        ms_dirty = statistics.median(a.elapsed_time(b) for a, b in dirty)
        ids = torch.topk(logits, shape.top_k, dim=-1).indices
        active = int(torch.unique(ids).numel())
        bytes_ = (active * shape.expert_bytes + tokens * shape.hidden * 2 * 2
                  + tokens * shape.num_experts * 4)
        achieved = bytes_ / (ms / 1e3) / 1e9
        results.append({"tokens": tokens, "ms": round(ms, 5),
                        "ms_dirty_l2": round(ms_dirty, 5),
                        "tokens_per_s": round(tokens / (ms / 1e3), 1),
                        "active_experts": active, "algorithmic_bytes": bytes_,
                        "achieved_gbs": round(achieved, 1),
                        "hbm_roofline_frac": round(achieved / pk["hbm_gbs"], 4),
                        "engine": ("fused-tiny" if tokens * shape.top_k <= TINY_MAX_ROUTES
                                   else "stream" if tokens * shape.top_k <= STREAM_ENGINE_MAX_ROUTES
                                   else "tcgen05-swap" if tokens * shape.top_k <= 4096
                                   else "tcgen05-wide")})
        del graph
    del layer, flush, flush_read
    torch.cuda.empty_cache()
    return results


# Token counts of the reference's shared-expert benchmark
# (benchmarks/bench_moe_shared.py: --tokens 16 | 32).
SHARED_BUCKETS = (16, 32)


def graph_latency_ms(forward, steps: int, warmup: int, flush, flush_read) -> float:
    """Median device time of one CUDA-graph replay of ``forward()`` with L2
    flushed (write then read 256 MB) before each replay."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.no_grad(), torch.cuda.stream(stream):
        for _ in range(3):
            forward()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.no_grad(), torch.cuda.graph(graph):
        forward()
    for _ in range(warmup):
        graph.replay()
    times = []
    for _ in range(steps):
        flush.fill_(1)
        flush_read.amax()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        times.append((a, b))
    torch.cuda.synchronize()
    del graph
    return statistics.median(a.elapsed_time(b) for a, b in times)


def load_shared_layer(layer, shape, device) -> None:
    import extend_nano_vllm_b200.workloads as wl
    w13, w2 = wl.expert_weights(shape, seed=2024, device=device, on_device=True)
    s13, s2, sg = wl.shared_expert_weights(shape, seed=2024, device=device)
    with torch.no_grad():
        layer.gate.weight.copy_(wl.gate_weight(shape, seed=2025).to(device))
        layer.gate_up_proj.copy_(w13)
        layer.down_proj.copy_(w2)
        layer.shared_expert.gate_up_proj.weight.copy_(s13)
        layer.shared_expert.down_proj.weight.copy_(s2)
        layer.shared_expert_gate.weight.copy_(sg)


def shared_expert_sweep(steps: int, warmup: int, pk: dict) -> dict:
    """Qwen3-Next-shaped layer with a shared expert (512 experts, top-10,
    routed and shared width 512), decode graphs at the reference benchmark's
    token counts: the shared expert inside the grouped expert launches
    ("fused") against the same layer computing it after the routed output
    with torch, as the reference does ("unfused")."""
    import extend_nano_vllm_b200.workloads as wl
    from extend_nano_vllm_b200.moe import ExpertParallelMoE

    shape = wl.QWEN3_NEXT_80B_A3B
    device = torch.device("cuda")
    layer = ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts, shape.top_k,
                              shape.norm_topk_prob, graph_safe_decode=True,
                              shared_expert_intermediate_size=shape.shared_intermediate)
    layer = layer.to(device=device, dtype=torch.bfloat16)
    load_shared_layer(layer, shape, device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    flush_read = torch.ones(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    rows = []
    for tokens in SHARED_BUCKETS:
        x = wl.hidden_states(tokens, shape.hidden, seed=71 + tokens, device=device)
        row = {"tokens": tokens}
        for fused in (True, False):
            layer.fuse_shared_expert = fused
            ms = graph_latency_ms(lambda: layer(x), steps, warmup, flush, flush_read)
            row["ms_fused" if fused else "ms_unfused"] = round(ms, 5)
        ids = torch.topk(layer.gate(x), shape.top_k, dim=-1).indices
        active = int(torch.unique(ids).numel()) + 1
        bytes_ = active * shape.expert_bytes + tokens * shape.hidden * 2 * 2
        row["active_experts_incl_shared"] = active
        row["hbm_roofline_frac_fused"] = round(
            bytes_ / (row["ms_fused"] / 1e3) / 1e9 / pk["hbm_gbs"], 4)
        rows.append(row)
    layer.fuse_shared_expert = True
    del layer, flush, flush_read
    torch.cuda.empty_cache()
    return {"shape": shape.name, "buckets": rows}


def prefill_case(steps: int, warmup: int, pk: dict) -> dict:
    import extend_nano_vllm_b200.workloads as wl

    shape = wl.QWEN3_30B_A3B
    device = torch.device("cuda")
    layer = build_layer(shape, 1, 0, device, expert_capacity_factor=1.25)
    x = wl.hidden_states(PREFILL_TOKENS, shape.hidden, seed=500, device=device)
    logits = wl.zipf_logits(PREFILL_TOKENS, shape.num_experts, seed=501, device=device)
    timer = KernelTimer()
    fn = lambda: layer._forward_from_logits(x, logits)  # noqa: E731
    for _ in range(warmup):
        fn()
    kept0 = layer.dispatch_assignment_count
    layer.kernel_timer = timer
    seconds = time_steps(fn, steps, 0, 1)
    layer.kernel_timer = None
    kept = (layer.dispatch_assignment_count - kept0) / steps
    flops = kept * shape.flops_per_route
    ms = seconds / steps * 1e3
    gu_ms, dn_ms = timer.mean_ms("gate_up"), timer.mean_ms("down")
    gu_flops = kept * 2 * 2 * shape.intermediate * shape.hidden
    out = {"tokens": PREFILL_TOKENS, "capacity": wl.capacity_for(PREFILL_TOKENS, shape, 1.25),
           "kept_routes": int(kept), "ms": round(ms, 4),
           "tokens_per_s": round(PREFILL_TOKENS / (ms / 1e3), 1),
           "layer_tflops": round(flops / (ms / 1e3) / 1e12, 1),
           "layer_tensor_frac": round(flops / (ms / 1e3) / 1e12 / pk["bf16_tflops"], 4),
           # All 128 experts hold kept routes: their weights stream once.
           "roofline_ms": round(max(flops / (pk["bf16_tflops"] * 1e12),
                                    shape.num_experts * shape.expert_bytes
                                    / (pk["hbm_gbs"] * 1e9)) * 1e3, 4),
           "roofline_frac": round(max(flops / (pk["bf16_tflops"] * 1e12),
                                      shape.num_experts * shape.expert_bytes
                                      / (pk["hbm_gbs"] * 1e9)) / (ms / 1e3), 4),
           "gate_up_ms": round(gu_ms, 4), "down_ms": round(dn_ms, 4),
           "gate_up_tflops": round(gu_flops / (gu_ms / 1e3) / 1e12, 1)}
    del layer
    torch.cuda.empty_cache()
    return out


def cpu_config1_baseline(wl, reps: int = 5) -> dict:
    """Config 1: the reference CPU algorithm (router + per-expert torch loop,
    nanovllm/layers/moe.py:870-920 and :546-580, restated in oracle/) on the
    30B-A3B layer, T=64, all host threads, median of `reps` after one warm-up.
    The fp32 gate of the config is cast to bf16 before the router GEMM (the
    reference's F.linear needs matching dtypes; the real model's gate is bf16)."""
    from oracle import moe_oracle as mo

    shape = wl.QWEN3_30B_A3B
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    x = wl.hidden_states(CPU_CONFIG1_TOKENS, shape.hidden, seed=0)
    gate = wl.gate_weight(shape, seed=0).to(torch.bfloat16)
    w13, w2 = wl.expert_weights(shape, seed=0)
    mo.forward_reference_torch(x, gate, w13, w2, shape.top_k, True)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        mo.forward_reference_torch(x, gate, w13, w2, shape.top_k, True)
        times.append(time.perf_counter() - t0)
    ms = statistics.median(times) * 1e3
    return {"value": round(CPU_CONFIG1_TOKENS / (ms / 1e3), 2), "unit": UNIT, "cores": cores,
            "kind": "port", "ms_per_forward": round(ms, 2),
            "sample": f"configs[0]: 30B-A3B layer (H=2048, E=128, k=8, I=768), "
                      f"T={CPU_CONFIG1_TOKENS}, bf16, gate cast to bf16, seed 0; median of "
                      f"{reps} forwards after one warm-up"}


def headline_config(shape, world: int) -> dict:
    """The `config` object of both arms' JSON lines (same workload, same keys)."""
    return {"workload": "configs[3]: Qwen3-235B-A22B-shaped MoE layer, EP over N GPUs",
            "hidden": shape.hidden, "num_experts": shape.num_experts, "top_k": shape.top_k,
            "moe_intermediate": shape.intermediate, "tokens_per_gpu": TOKENS_PER_GPU,
            "global_batch": world * TOKENS_PER_GPU, "parallelism": f"ep{world}",
            "router": "bf16 gate GEMM -> fp32 softmax top-8, renormalised",
            "inputs": "hidden N(0,1) seed 1000+rank, gate N(0,0.02) seed 2025, "
                      "experts N(0,0.02) seed 2024",
            "l2": "inputs larger than L2 (expert weights %.2f GB per GPU)"
                  % (shape.num_experts // world * shape.expert_bytes / 1e9)}


def reference_triton(steps: int, warmup: int) -> dict:
    """The unmodified reference's own GPU path on this GPU, same workloads and
    timing as the native lines: its Triton grouped GEMMs, torch routing and
    packing (nanovllm/layers/moe.py _forward_triton for the 235B headline and
    the Zipf prefill, _forward_static_decode captured in one CUDA graph per
    decode bucket, as its model runner does).  Imported from baseline/_ref
    (baseline/install_reference.sh); a same-box comparison, not the product."""
    import importlib

    import extend_nano_vllm_b200.workloads as wl

    ref_dir = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "nanovllm")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    if ref_dir not in sys.path:
        sys.path.append(ref_dir)
    try:
        ref_moe = importlib.import_module("nanovllm.layers.moe")
    except Exception as exc:  # noqa: BLE001 - reported in the JSON line
        return {"unavailable": f"reference import failed: {exc!r}"[:300]}
    device = torch.device("cuda")

    def make(shape, seed_w, seed_g, **kw):
        layer = ref_moe.ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts,
                                          shape.top_k, shape.norm_topk_prob, **kw)
        layer = layer.to(device=device, dtype=torch.bfloat16)
        w13, w2 = wl.expert_weights(shape, seed=seed_w, device=device, on_device=True)
        with torch.no_grad():
            layer.gate.weight.copy_(wl.gate_weight(shape, seed=seed_g).to(device))
            layer.gate_up_proj.copy_(w13)
            layer.down_proj.copy_(w2)
        return layer

    out = {}
    shape = wl.QWEN3_235B_A22B
    layer = make(shape, 2024, 2025)
    x = wl.hidden_states(TOKENS_PER_GPU, shape.hidden, seed=1000, device=device)
    with torch.no_grad():
        seconds = time_steps(lambda: layer(x), steps, warmup, 1)
    ms = seconds / steps * 1e3
    out["headline_235b_t4096"] = {"ms": round(ms, 4),
                                  "tokens_per_s": round(TOKENS_PER_GPU / (ms / 1e3), 1)}
    del layer, x
    torch.cuda.empty_cache()

    shape = wl.QWEN3_30B_A3B
    layer = make(shape, 2024, 2025, graph_safe_decode=True)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    flush_read = torch.ones(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    decode = []
    for tokens in DECODE_BUCKETS:
        x = wl.hidden_states(tokens, shape.hidden, seed=300 + tokens, device=device)
        logits = wl.uniform_logits(tokens, shape.num_experts, seed=400 + tokens, device=device)
        layer.gate.forward = lambda h, _l=logits: _l  # the same injected fp32 logits
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.no_grad(), torch.cuda.stream(stream):
            for _ in range(3):
                layer(x)
        torch.cuda.current_stream().wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(graph):
            layer(x)
        for _ in range(warmup):
            graph.replay()
        times = []
        for _ in range(max(20, steps // 4)):
            flush.fill_(1)
            flush_read.amax()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            times.append((a, b))
        torch.cuda.synchronize()
        ms = statistics.median(a.elapsed_time(b) for a, b in times)
        decode.append({"tokens": tokens, "ms": round(ms, 5),
                       "tokens_per_s": round(tokens / (ms / 1e3), 1)})
        del graph
    out["decode_30b_a3b"] = decode
    del layer, flush, flush_read
    torch.cuda.empty_cache()

    layer = make(shape, 2024, 2025, expert_capacity_factor=1.25)
    x = wl.hidden_states(PREFILL_TOKENS, shape.hidden, seed=500, device=device)
    logits = wl.zipf_logits(PREFILL_TOKENS, shape.num_experts, seed=501, device=device)
    layer.gate.forward = lambda h: logits
    with torch.no_grad():
        seconds = time_steps(lambda: layer(x), max(10, steps // 10), warmup, 1)
    ms = seconds / max(10, steps // 10) * 1e3
    out["prefill_30b_a3b_zipf"] = {"ms": round(ms, 4),
                                   "tokens_per_s": round(PREFILL_TOKENS / (ms / 1e3), 1)}
    del layer
    torch.cuda.empty_cache()

    # The reference's shared-expert benchmark shape (bench_moe_shared.py):
    # its layer with graph-safe decode and the shared expert, same weights.
    shape = wl.QWEN3_NEXT_80B_A3B
    layer = ref_moe.ExpertParallelMoE(
        shape.hidden, shape.intermediate, shape.num_experts, shape.top_k, shape.norm_topk_prob,
        graph_safe_decode=True, shared_expert_intermediate_size=shape.shared_intermediate)
    layer = layer.to(device=device, dtype=torch.bfloat16)
    load_shared_layer(layer, shape, device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    flush_read = torch.ones(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    rows = []
    for tokens in SHARED_BUCKETS:
        x = wl.hidden_states(tokens, shape.hidden, seed=71 + tokens, device=device)
        ms = graph_latency_ms(lambda: layer(x), max(20, steps // 4), warmup, flush, flush_read)
        rows.append({"tokens": tokens, "ms": round(ms, 5)})
    out["shared_next_decode"] = rows
    del layer, flush, flush_read
    torch.cuda.empty_cache()
    return out


# Decode batch sizes per rank of the expert-parallel latency comparison.
EP_DECODE_TOKENS = (8, 32)


def ep_graph_ms(forward, steps: int, warmup: int, world: int, flush, flush_read) -> float:
    """Median device time of one CUDA-graph replay of ``forward()`` on every
    rank at once (L2 flushed before each replay), max over ranks."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.no_grad(), torch.cuda.stream(stream):
        for _ in range(3):
            forward()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.no_grad(), torch.cuda.graph(graph):
        forward()
    for _ in range(warmup):
        graph.replay()
    barrier(world)
    times = []
    for _ in range(steps):
        flush.fill_(1)
        flush_read.amax()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        times.append((a, b))
    torch.cuda.synchronize()
    barrier(world)
    del graph
    return max_over_ranks(statistics.median(a.elapsed_time(b) for a, b in times), world)


def reference_ep(args, world: int, rank: int, local: int) -> dict:
    """The unmodified reference's expert-parallel backends on the same ranks
    (baseline/_ref, its process groups from initialize_model_parallel):
    all-gather + reduce-scatter at the headline workload, and decode latency
    of one CUDA-graph replay at EP_DECODE_TOKENS tokens per rank on the
    30B-A3B layer against this library's NVLink exchange (same weights)."""
    import importlib

    import extend_nano_vllm_b200.workloads as wl

    ref_dir = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "nanovllm")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    if ref_dir not in sys.path:
        sys.path.append(ref_dir)
    try:
        ref_moe = importlib.import_module("nanovllm.layers.moe")
        ps = importlib.import_module("nanovllm.distributed.parallel_state")
    except Exception as exc:  # noqa: BLE001 - reported in the JSON line
        return {"unavailable": f"reference import failed: {exc!r}"[:300]}
    ps.initialize_model_parallel(1, 1, True, data_parallel_size=world)
    device = torch.device("cuda", local)

    def make_ref(shape, backend, **kw):
        layer = ref_moe.ExpertParallelMoE(shape.hidden, shape.intermediate, shape.num_experts,
                                          shape.top_k, shape.norm_topk_prob, ep_rank=rank,
                                          ep_size=world, dispatch_backend=backend, **kw)
        layer = layer.to(device=device, dtype=torch.bfloat16)
        n = shape.num_experts // world
        w13, w2 = wl.expert_weights(shape, seed=2024, num_local=n, first_expert=rank * n,
                                    device=device, on_device=True)
        with torch.no_grad():
            layer.gate.weight.copy_(wl.gate_weight(shape, seed=2025).to(device))
            layer.gate_up_proj.copy_(w13)
            layer.down_proj.copy_(w2)
        return layer

    out = {}
    shape = wl.QWEN3_235B_A22B
    layer = make_ref(shape, "allgather_reducescatter")
    x = wl.hidden_states(TOKENS_PER_GPU, shape.hidden, seed=1000 + rank, device=device)
    steps = max(5, args.steps // 4)
    with torch.no_grad():
        seconds = time_steps(lambda: layer(x), steps, min(3, args.warmup), world)
    ms = seconds / steps * 1e3
    out["headline_allgather_reducescatter"] = {
        "ms": round(ms, 4), "tokens_per_s": round(world * TOKENS_PER_GPU / (ms / 1e3), 1)}
    del layer, x
    torch.cuda.empty_cache()

    shape = wl.QWEN3_30B_A3B
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    flush_read = torch.ones(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    ref_layer = make_ref(shape, "allgather_reduce", graph_safe_decode=True)
    own_layer = build_layer(shape, world, rank, device, graph_safe_decode=True)
    decode = []
    for tokens in EP_DECODE_TOKENS:
        x = wl.hidden_states(tokens, shape.hidden, seed=300 + tokens + 17 * rank, device=device)
        row = {"tokens_per_rank": tokens}
        row["reference_allgather_reduce_us"] = round(1e3 * ep_graph_ms(
            lambda: ref_layer(x), max(20, args.steps // 4), args.warmup, world, flush,
            flush_read), 2)
        row["nvlink_exchange_us"] = round(1e3 * ep_graph_ms(
            lambda: own_layer(x), max(20, args.steps // 4), args.warmup, world, flush,
            flush_read), 2)
        row["speedup"] = round(row["reference_allgather_reduce_us"]
                               / row["nvlink_exchange_us"], 2)
        decode.append(row)
    out["decode_30b_a3b_graph"] = decode
    del ref_layer, own_layer, flush, flush_read
    torch.cuda.empty_cache()
    return out


def native(args, world, rank, local, json_fd: int = 1) -> None:
    import extend_nano_vllm_b200 as pkg
    import extend_nano_vllm_b200.workloads as wl
    from extend_nano_vllm_b200 import _lib

    pk = peaks()
    shape = wl.QWEN3_235B_A22B
    device = torch.device("cuda", local)
    layer = build_layer(shape, world, rank, device)
    layer.expert_engine = args.engine
    x = wl.hidden_states(TOKENS_PER_GPU, shape.hidden, seed=1000 + rank, device=device)
    step = lambda: layer(x)  # noqa: E731

    for _ in range(args.warmup):
        step()
    barrier(world)
    kept0 = layer.dispatch_assignment_count
    snapshot = dict(_lib.LAUNCH_COUNTS)
    timer = KernelTimer()
    layer.kernel_timer = timer
    clocks = ClockSampler(local)
    clocks.start()
    clocks.mark_begin()
    seconds = time_steps(step, args.steps, 0, world)
    clocks.mark_end()
    clock_info = clocks.stop()
    layer.kernel_timer = None
    launches = _lib.launches_since(snapshot)
    kept_per_step = (layer.dispatch_assignment_count - kept0) / args.steps
    ms_per_step = seconds / args.steps * 1e3
    value = world * TOKENS_PER_GPU * args.steps / seconds

    # Dominant kernel: the tcgen05 gate/up GEMM (2/3 of the FLOPs).
    gu_ms = timer.mean_ms("gate_up")
    gu_flops = kept_per_step * 2 * 2 * shape.intermediate * shape.hidden
    gu_tflops = gu_flops / (gu_ms / 1e3) / 1e12 if gu_ms > 0 else 0.0
    gu_tflops = max_over_ranks(gu_tflops, world) if world > 1 else gu_tflops
    # The burst peak applies while the SM clock stays at its maximum (short
    # timed regions); the sustained one once the 1 kW power cap has pulled the
    # clock down (median sampled clock below 90% of the maximum) or for a
    # region of seconds.
    sampled, sampled_max = clock_info.get("sm_mhz"), clock_info.get("sm_max_mhz")
    capped = bool(sampled and sampled_max and sampled < 0.9 * sampled_max)
    sustained = capped or seconds >= SUSTAINED_REGION_S
    peak_key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    peak = pk[peak_key]
    roofline = {"kernel": "grouped_gemm_kernel<gate_up, 256> (tcgen05 wide)", "bound": "tensor",
                "achieved": round(gu_tflops, 1), "peak": peak,
                "peak_kind": f"{peak_key} ({pk['source']}; timed region {seconds:.3f} s, "
                             f"median SM clock {sampled} of {sampled_max} MHz)",
                "unit": "TFLOP/s", "frac": round(gu_tflops / peak, 4),
                "frac_of_burst": round(gu_tflops / pk["bf16_tflops"], 4),
                "frac_of_sustained": round(gu_tflops / pk["bf16_tflops_sustained"], 4),
                "traffic": GATE_UP_TRAFFIC_EP1 if world == 1 else None,
                "traffic_source": "profiles/grouped_gemm_traffic_ep1_235b.md (ncu dram bytes "
                                  "of one full-size gate/up launch)" if world == 1 else None,
                "flops_per_launch": int(gu_flops),
                "launch_ms": round(gu_ms, 4)}
    # Whole-layer roofline: the slower of the FLOPs at the tensor peak and the
    # expert-weight bytes at the HBM peak.
    layer_flops = kept_per_step * shape.flops_per_route
    layer_bytes = shape.num_experts // world * shape.expert_bytes
    layer_bound_ms = max(layer_flops / (peak * 1e12), layer_bytes / (pk["hbm_gbs"] * 1e9)) * 1e3
    layer_roofline = {"bound_ms": round(layer_bound_ms, 4), "ms": round(ms_per_step, 4),
                      "frac": round(layer_bound_ms / ms_per_step, 4),
                      "tflops": round(layer_flops / (ms_per_step / 1e3) / 1e12, 1)}

    # End to end through the public layer API with pinned host buffers: every
    # step copies its hidden states in from pinned host memory and its output
    # back out.  The copies run on their own streams (PCIe is full duplex), so
    # step i+1's input copy and step i's output copy overlap compute, as a
    # throughput-oriented caller would run it.
    e2e_seconds = time_e2e(layer, x, args.steps, args.warmup, world)
    e2e_value = world * TOKENS_PER_GPU * args.steps / e2e_seconds
    h2d = x.numel() * x.element_size()

    record = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) hidden, N(0,0.02) weights; no checkpoint)",
        "config": headline_config(shape, world),
        "exchange": "NVLink peer memory (CUDA IPC), graph-safe" if world > 1 else "none",
        "kept_routes_per_gpu_step": round(kept_per_step, 1),
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": h2d},
        "gpu_launches": launches,
        "roofline": roofline,
        "layer_roofline": layer_roofline,
        "clocks": clock_info,
        "device_status": pkg.device_status(),
    }
    del layer, x
    torch.cuda.empty_cache()

    if world == 1 and not args.no_sweep:
        record["sweep"] = {"decode_30b_a3b": decode_sweep(max(20, args.steps // 4),
                                                          args.warmup, pk),
                           "prefill_30b_a3b_zipf": prefill_case(max(10, args.steps // 10),
                                                                args.warmup, pk),
                           "shared_expert_next": shared_expert_sweep(max(20, args.steps // 4),
                                                                     args.warmup, pk)}
        if not args.no_reference_triton:
            ref = reference_triton(args.steps, args.warmup)
            record["reference_triton_gpu"] = ref
            if "headline_235b_t4096" in ref:
                sweep = record["sweep"]
                record["speedup_vs_reference_triton_gpu"] = {
                    "headline_235b_t4096": round(ref["headline_235b_t4096"]["ms"]
                                                 / ms_per_step, 2),
                    "prefill_30b_a3b_zipf": round(ref["prefill_30b_a3b_zipf"]["ms"]
                                                  / sweep["prefill_30b_a3b_zipf"]["ms"], 2),
                    "decode_30b_a3b": {str(r["tokens"]): round(r["ms"] / n["ms"], 2)
                                       for r, n in zip(ref["decode_30b_a3b"],
                                                       sweep["decode_30b_a3b"])},
                    "shared_next_decode": {
                        str(r["tokens"]): round(r["ms"] / n["ms_fused"], 2)
                        for r, n in zip(ref.get("shared_next_decode", []),
                                        sweep["shared_expert_next"]["buckets"])}}
    if world > 1 and not args.no_reference_triton:
        ref = reference_ep(args, world, rank, local)
        record["reference_ep_gpu"] = ref
        if "headline_allgather_reducescatter" in ref:
            record["speedup_vs_reference_ep_gpu"] = round(
                ref["headline_allgather_reducescatter"]["ms"] / ms_per_step, 2)
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        record["cpu_baseline"] = cpu_config1_baseline(wl)
    if rank == 0:
        sys.stdout.flush()
        os.write(json_fd, (json.dumps(record) + "\n").encode())


# ---------------------------------------------------------------------------
# Reference arm: the reference's CPU implementation on the host cores.
# ---------------------------------------------------------------------------
def reference(args, world, rank) -> None:
    """The reference's CPU implementation of the path (router + per-expert
    torch loop, nanovllm/layers/moe.py:870-920 and :546-580, restated in
    oracle/) on this host's cores, over the headline workload: full
    4096-token steps with the same routing inputs as the native arm.  Only
    as many steps are timed as fit in about REFERENCE_BUDGET_S seconds (one
    step takes several seconds); the line says how many."""
    if rank != 0:
        return
    wl = load_workloads()
    from oracle import moe_oracle as mo

    shape = wl.QWEN3_235B_A22B
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    x = wl.hidden_states(TOKENS_PER_GPU, shape.hidden, seed=1000)
    gate = wl.gate_weight(shape, seed=2025).to(torch.bfloat16)
    w13, w2 = wl.expert_weights(shape, seed=2024)
    step = lambda: mo.forward_reference_torch(x, gate, w13, w2, shape.top_k, True)  # noqa: E731
    t0 = time.perf_counter()
    step()  # warm-up: one full step
    per_step = time.perf_counter() - t0
    timed = int(max(1, min(args.steps, REFERENCE_BUDGET_S // max(per_step, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(timed):
        step()
    seconds = time.perf_counter() - t0
    value = TOKENS_PER_GPU * timed / seconds
    sample = (f"full {TOKENS_PER_GPU}-token steps of the headline workload (all 128 experts) "
              f"through the reference CPU algorithm, bf16; {timed} timed step(s) after one "
              f"warm-up step, {cores} threads")
    record = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT,
        "n_gpus": world, "steps": timed, "steps_requested": args.steps, "warmup": 1,
        "ms_per_step": round(seconds / timed * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) hidden, N(0,0.02) weights; no checkpoint)",
        "config": headline_config(shape, world),
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(record), flush=True)


# ---------------------------------------------------------------------------
# End-to-end offline generation (the benchmark list's last configuration):
# the reference's unchanged engine (LLM, scheduler, model runner with paged KV
# cache and decode CUDA graphs, data-parallel replicas sharing one MoE group)
# on a random-init Qwen3-30B-A3B-architecture model, with the reference's MoE
# layer or this one swapped in at import time, the way the integration patch
# at the end of nanovllm/layers/moe.py would.
# ---------------------------------------------------------------------------
E2E_MODEL = dict(hidden_size=2048, num_attention_heads=32, num_key_value_heads=4, head_dim=128,
                 num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768,
                 intermediate_size=6144, vocab_size=151936, norm_topk_prob=True,
                 max_position_embeddings=40960, rope_theta=1000000.0, rms_norm_eps=1e-6,
                 tie_word_embeddings=False, decoder_sparse_step=1, mlp_only_layers=[],
                 bos_token_id=151643, eos_token_id=151645)
E2E_SEED = 20251


def e2e_model_dir(root: str, layers: int) -> str:
    """Config-only checkpoint directory (no weights) plus a word-level
    tokenizer over the model's vocabulary ("t<id>"): prompts are token ids and
    generation ignores EOS, so the tokenizer only names the EOS id and turns
    the outputs back into text."""
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast, Qwen3MoeConfig

    config = Qwen3MoeConfig(**{**E2E_MODEL, "num_hidden_layers": layers}, dtype="bfloat16")
    config.save_pretrained(root)
    vocab = {f"t{i}": i for i in range(E2E_MODEL["vocab_size"])}
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="t0"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="t0",
                            eos_token=f"t{E2E_MODEL['eos_token_id']}").save_pretrained(root)
    return root


def e2e_random_init(model, path) -> None:
    """Stands in for nanovllm.utils.loader.load_model (no checkpoint exists):
    every parameter N(0, 0.02) from a generator seeded by its name, norms 1.
    Both arms name and shard their parameters alike, so they get the same
    weights."""
    import zlib

    with torch.no_grad():
        for name, param in model.named_parameters():
            if "norm" in name:
                param.fill_(1.0)
                continue
            g = torch.Generator(device=param.device)
            g.manual_seed(E2E_SEED * 1000003 + zlib.crc32(name.encode()))
            param.normal_(0.0, 0.02, generator=g)


def e2e_install_b200_layer() -> None:
    """Make every nanovllm module that imported the reference's
    ExpertParallelMoE use this repository's class; the engine's cross-DP
    all-gather backend becomes the NVLink exchange."""
    import nanovllm.layers.moe as ref_moe

    from extend_nano_vllm_b200.moe import ExpertParallelMoE as B200MoE

    class EngineMoE(B200MoE):
        def __init__(self, *args, dispatch_backend: str = "replicated", **kwargs):
            if dispatch_backend in ("allgather_reduce", "allgather_reducescatter"):
                dispatch_backend = "all_to_all_nvlink"
            super().__init__(*args, dispatch_backend=dispatch_backend, **kwargs)

    original = ref_moe.ExpertParallelMoE
    for module in list(sys.modules.values()):
        if (getattr(module, "__name__", "").startswith("nanovllm")
                and getattr(module, "ExpertParallelMoE", None) is original):
            module.ExpertParallelMoE = EngineMoE


def e2e_replica(replica_id, dp, model_dir, indexed_prompts, max_tokens, queue, kwargs, impl):
    """One data-parallel replica (the reference's data_parallel._run_replica,
    plus step timing): its own LLM engine on GPU `replica_id`."""
    import traceback

    llm = None
    try:
        ref_dir = os.path.join(REPO, "baseline", "_ref")
        if ref_dir not in sys.path:
            sys.path.insert(0, ref_dir)
        import nanovllm.engine.model_runner as runner_mod
        import nanovllm.utils.loader as loader_mod
        from nanovllm import LLM, SamplingParams
        from nanovllm.engine.llm_engine import LLMEngine

        loader_mod.load_model = e2e_random_init
        runner_mod.load_model = e2e_random_init
        if impl == "b200":
            e2e_install_b200_layer()
        stats = {"prefill_s": 0.0, "prefill_tokens": 0, "decode_s": 0.0, "decode_tokens": 0,
                 "decode_steps": 0}
        step = LLMEngine.step
        step_ms = []
        prefill_ms = []

        def timed_step(self):
            t0 = time.perf_counter()
            outputs, num_tokens = step(self)
            dt = time.perf_counter() - t0
            if num_tokens > 0:
                stats["prefill_s"] += dt
                stats["prefill_tokens"] += num_tokens
                prefill_ms.append(round(dt * 1e3, 2))
            elif num_tokens < 0:
                stats["decode_s"] += dt
                stats["decode_tokens"] += -num_tokens
                stats["decode_steps"] += 1
                step_ms.append(dt * 1e3)
            return outputs, num_tokens

        LLMEngine.step = timed_step
        t0 = time.perf_counter()
        llm = LLM(model_dir, data_parallel_size=dp, data_parallel_rank=replica_id, **kwargs)
        stats["init_s"] = time.perf_counter() - t0
        _, prompts = zip(*indexed_prompts)
        params = SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True)
        t0 = time.perf_counter()
        outputs = llm.generate(list(prompts), params, use_tqdm=False)
        stats["generate_s"] = time.perf_counter() - t0
        stats["output_tokens"] = sum(len(o["token_ids"]) for o in outputs)
        stats["first_tokens"] = [o["token_ids"][:8] for o in outputs[:2]]
        stats["decode_step_ms_median"] = statistics.median(step_ms) if step_ms else None
        stats["decode_step_ms_first"] = [round(v, 2) for v in step_ms[:3]]
        stats["prefill_step_ms"] = prefill_ms
        stats["decode_graph_replays"] = getattr(llm.model_runner, "decode_graph_replay_count",
                                                None)
        queue.put((replica_id, stats, None))
    except Exception:  # noqa: BLE001 - reported to the parent
        queue.put((replica_id, None, traceback.format_exc()))
    finally:
        if llm is not None:
            llm.exit()


def e2e(args) -> None:
    """DP x EP = --gpus replicas of the reference engine (generate_data_parallel's
    launch: one spawned process per replica, a shared MoE group over all of
    them, prompts dealt round-robin, equal max_tokens, EOS ignored)."""
    import multiprocessing as mp
    import shutil
    import socket
    import tempfile
    from queue import Empty

    dp = args.gpus
    gen = torch.Generator().manual_seed(E2E_SEED)
    prompts = torch.randint(0, E2E_MODEL["vocab_size"], (args.e2e_requests, args.e2e_prompt),
                            generator=gen).tolist()
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    per_rank = args.e2e_requests // dp
    kwargs = dict(enable_expert_parallel=dp > 1, master_port=port, max_num_seqs=per_rank,
                  max_model_len=2048, max_num_batched_tokens=8192)
    assignments = [[] for _ in range(dp)]
    for index, prompt in enumerate(prompts):
        assignments[index % dp].append((index, prompt))
    root = tempfile.mkdtemp(prefix="e2e_model_")
    e2e_model_dir(root, args.e2e_layers)
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=e2e_replica, args=(r, dp, root, assignments[r], args.e2e_output,
                                                    queue, kwargs, args.e2e))
             for r in range(dp)]
    t0 = time.perf_counter()
    for p in procs:
        p.start()
    results, errors = {}, []
    for _ in procs:
        try:
            rid, stats, err = queue.get(timeout=900)
        except Empty:
            errors.append("timed out waiting for a replica")
            break
        if err:
            errors.append(f"replica {rid}: {err}")
        else:
            results[rid] = stats
    wall = time.perf_counter() - t0
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
            p.join()
    shutil.rmtree(root, ignore_errors=True)
    record = {"metric": "e2e decode tokens/s (offline generation, DP x EP)", "impl": args.e2e,
              "n_gpus": dp, "unit": "tokens/s", "higher_is_better": True,
              "data": "random-init weights, seeded uniform prompt token ids",
              "config": {"model": f"Qwen3-30B-A3B architecture, {args.e2e_layers} layers",
                         "requests": args.e2e_requests, "prompt_tokens": args.e2e_prompt,
                         "output_tokens": args.e2e_output, "parallelism": f"dp{dp}xep{dp}",
                         "moe_backend": ("replicated, one GPU" if dp == 1 else
                                         "all_to_all_nvlink (this repository)"
                                         if args.e2e == "b200" else
                                         "allgather_reduce (reference)"),
                         "kvcache_block_size": 256, "decode_cuda_graphs": True},
              "wall_s": round(wall, 1)}
    if errors or len(results) != dp:
        record["error"] = "\n".join(errors)[-4000:]
    else:
        decode_s = max(r["decode_s"] for r in results.values())
        prefill_s = max(r["prefill_s"] for r in results.values())
        decode_tokens = sum(r["decode_tokens"] for r in results.values())
        prefill_tokens = sum(r["prefill_tokens"] for r in results.values())
        generate_s = max(r["generate_s"] for r in results.values())
        record.update({
            "value": round(decode_tokens / decode_s, 1),
            "decode_s": round(decode_s, 3), "decode_tokens": decode_tokens,
            "decode_steps": max(r["decode_steps"] for r in results.values()),
            "prefill_tokens_per_s": round(prefill_tokens / prefill_s, 1),
            "generate_s": round(generate_s, 3),
            "output_tokens_per_s": round(sum(r["output_tokens"] for r in results.values())
                                         / generate_s, 1),
            "init_s": round(max(r["init_s"] for r in results.values()), 1),
            "decode_step_ms_median": [round(r["decode_step_ms_median"], 3)
                                      for _, r in sorted(results.items())],
            "decode_step_ms_first": results[0]["decode_step_ms_first"],
            "prefill_step_ms": results[0]["prefill_step_ms"],
            "decode_graph_replays": [r["decode_graph_replays"] for _, r in sorted(results.items())],
            "first_tokens": results[0]["first_tokens"]})
    print(json.dumps(record), flush=True)
    if "error" in record:
        sys.exit(1)


def main() -> None:
    args = parse_args()
    if args.e2e:
        e2e(args)
        return
    if args.profile_case:
        profile_case(args)
        return
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
        return
    # Only the JSON line goes to stdout: anything else written to fd 1 while the
    # benchmark runs (library banners, e.g. NCCL's version line) goes to stderr.
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    world, rank, local = init_dist(args)
    try:
        native(args, world, rank, local, json_fd)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
