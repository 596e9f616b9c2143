"""ExpertParallelMoE on B200: the reference layer API over the b200moe kernels.

This class keeps the constructor, validation errors, parameters
(``gate.weight``, ``gate_up_proj [E_loc, 2I, H]``, ``down_proj [E_loc, H, I]``),
buffers, counters, placement/relocation methods and private seams of
nano-vLLM's ``ExpertParallelMoE`` (nanovllm/layers/moe.py:237-1263), so the
model runner, scheduler, CUDA-graph bucket capture and ``relocate_experts``
keep working when it is substituted.  Every numeric step of the expert path
runs in the CUDA library (router, capacity/packing, grouped gate/up + SwiGLU,
grouped down, route-order combine, EP dispatch/combine packing).  There is no
CPU or Triton path: CPU tensors raise.

Differences from the reference, by design:
  * an additional dispatch backend ``"all_to_all_nvlink"``: every EP rank
    routes its own tokens and exchanges token rows and route results with
    its peers over NVLink peer memory, graph-safe and without host reads
    under capture (the reference all-gathers every replica's tokens);
  * the unfused grouped-GEMM seam ``_run_grouped_gemm`` does not exist (gate/up
    and SwiGLU are one kernel), nor does the per-expert torch loop
    ``_forward_reference`` (correctness oracles live with the tests);
  * bf16 activations and weights only.
"""

from __future__ import annotations

import math
import os

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from . import _lib
from . import dist_env
from . import ops as _native_ops

_MOE_BLOCK_M = _lib.BLOCK_ROWS
MOE_MAX_GRAPH_TOKENS_PER_RANK = 512
# Routes per call up to which the weight-streaming engine runs (decode
# buckets of <= 2 tokens at top-8, measured crossover); above it the tcgen05
# grouped GEMM runs.
STREAM_ENGINE_MAX_ROUTES = 16
# Route counts up to which the tcgen05 gate/up GEMM gathers token rows itself
# (measured: 1-2% faster at 64-256 routes, 4% slower at 4096).
FUSED_GATHER_MAX_ROUTES = 512

DISPATCH_BACKENDS = (
    "replicated", "all_to_all", "all_to_all_reduce",
    "allgather_reduce", "allgather_reducescatter", "all_to_all_nvlink",
)
GRAPH_SAFE_BACKENDS = ("replicated", "allgather_reduce", "allgather_reducescatter",
                       "all_to_all_nvlink")


# Batches of up to this many tokens route and pack in one launch (the packing
# block's 8 warps route two tokens each at most).
ROUTE_PACK_MAX_TOKENS = 16


def _capturing() -> bool:
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


def reduce_fp64_to_bf16(local_output: torch.Tensor, group, output_dtype=torch.bfloat16
                        ) -> torch.Tensor:
    """fp64 reduce-scatter then all-gather in ``output_dtype`` (moe.py:41-58)."""
    flat = local_output.contiguous().view(-1)
    world_size = dist.get_world_size(group)
    if flat.dtype != torch.float64 or flat.numel() % world_size:
        raise ValueError("FP64 EP output must divide evenly across ranks")
    reduced = torch.empty(flat.numel() // world_size, device=flat.device, dtype=torch.float64)
    dist.reduce_scatter_tensor(reduced, flat, group=group)
    gathered = torch.empty(flat.numel(), device=flat.device, dtype=output_dtype)
    dist.all_gather_into_tensor(gathered, reduced.to(output_dtype), group=group)
    return gathered.view_as(local_output)


class ReplicatedGate(nn.Module):
    """Router projection [E, H] (the reference's ReplicatedLinear, linear.py:54-68)."""

    def __init__(self, input_size: int, output_size: int) -> None:
        super().__init__()
        self.input_size = input_size
        self.output_size = output_size
        self.weight = nn.Parameter(torch.empty(output_size, input_size))
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor) -> None:
        param.data.copy_(loaded_weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight)


class SharedMergedGate(ReplicatedGate):
    """The shared expert's merged gate/up projection [2 * I_s, H]: gate rows
    first; its loader takes the shard id (0 gate, 1 up) like the reference's
    SharedMergedReplicatedLinear (moe.py:195-209)."""

    def __init__(self, hidden_size: int, intermediate_size: int) -> None:
        self.intermediate_size = intermediate_size
        super().__init__(hidden_size, 2 * intermediate_size)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor,
                      loaded_shard_id: int | None = None) -> None:
        if loaded_shard_id is None:
            param.data.copy_(loaded_weight)
            return
        param.data.narrow(0, int(loaded_shard_id) * self.intermediate_size,
                          self.intermediate_size).copy_(loaded_weight)


class SharedExpertMLP(nn.Module):
    """Dense shared expert (moe.py:212-234), replicated.  With one EP rank and
    the routed experts' width the layer runs it inside the grouped expert
    kernels; otherwise it is computed as the reference does, after the
    routed output."""

    def __init__(self, hidden_size: int, intermediate_size: int) -> None:
        super().__init__()
        self.intermediate_size = intermediate_size
        self.gate_up_proj = SharedMergedGate(hidden_size, intermediate_size)
        self.down_proj = ReplicatedGate(intermediate_size, hidden_size)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        gate, up = self.gate_up_proj(hidden_states).chunk(2, dim=-1)
        return self.down_proj(F.silu(gate) * up)


class ExpertParallelMoE(nn.Module):
    """Qwen3-MoE sparse block with the reference's constructor and seams."""

    def __init__(
        self,
        hidden_size: int,
        intermediate_size: int,
        num_experts: int,
        top_k: int,
        norm_topk_prob: bool,
        ep_rank: int = 0,
        ep_size: int = 1,
        dispatch_backend: str = "replicated",
        expert_capacity: int | None = None,
        graph_safe_decode: bool = False,
        expert_owners: tuple[int, ...] | list[int] | None = None,
        expert_capacity_factor: float | None = None,
        shared_expert_intermediate_size: int | None = None,
        shared_expert_tp_sharded: bool = False,
        dynamic_placement: bool = False,
    ) -> None:
        super().__init__()
        # Validation mirrors moe.py:258-283 (same messages for the same errors).
        if num_experts % ep_size != 0:
            raise ValueError("num_experts must divide evenly across EP ranks")
        if not 1 <= top_k <= num_experts:
            raise ValueError("top_k must be between 1 and num_experts")
        if dispatch_backend not in DISPATCH_BACKENDS:
            raise ValueError("unknown MoE dispatch backend")
        if expert_capacity is not None and expert_capacity < 1:
            raise ValueError("expert capacity must be positive")
        if expert_capacity_factor is not None:
            if (isinstance(expert_capacity_factor, bool)
                    or not isinstance(expert_capacity_factor, (int, float))
                    or not math.isfinite(expert_capacity_factor)
                    or expert_capacity_factor <= 0):
                raise ValueError("expert capacity factor must be finite and positive")
            if expert_capacity is not None:
                raise ValueError("fixed capacity and capacity factor are mutually exclusive")
        if graph_safe_decode and dispatch_backend not in GRAPH_SAFE_BACKENDS:
            raise ValueError("graph-safe MoE decode requires graph-safe dispatch")
        if (shared_expert_intermediate_size is not None
                and shared_expert_intermediate_size < 1):
            raise ValueError("shared expert intermediate size must be positive")
        if shared_expert_tp_sharded:
            raise NotImplementedError("TP-sharded shared experts are not supported")

        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.ep_rank = ep_rank
        self.ep_size = ep_size
        self.dispatch_backend = dispatch_backend
        self.fp64_combine = (
            dispatch_backend == "replicated"
            and os.environ.get("NANOVLLM_EXPERIMENTAL_FP64_MOE_COMBINE") == "1"
        )
        self.fp64_staged_reduce = (
            self.fp64_combine and ep_size > 1
            and os.environ.get("NANOVLLM_EXPERIMENTAL_FP64_STAGED_REDUCE") == "1"
        )
        self.fp32_reduce = (
            ep_size > 1 and dispatch_backend == "replicated" and not self.fp64_combine
            and os.environ.get("NANOVLLM_EXPERIMENTAL_FP32_EP_REDUCE") == "1"
        )
        self.expert_capacity = expert_capacity
        self.expert_capacity_factor = expert_capacity_factor
        self.graph_safe_decode = graph_safe_decode
        self.dynamic_placement = dynamic_placement
        self.num_local_experts = num_experts // ep_size
        if expert_owners is None and dynamic_placement:
            expert_owners = tuple(e // self.num_local_experts for e in range(num_experts))
        self.expert_owners = (
            tuple(expert_owners) if expert_owners is not None
            else tuple(e // self.num_local_experts for e in range(num_experts))
        )
        if expert_owners is None:
            self.expert_start = ep_rank * self.num_local_experts
            self.expert_end = self.expert_start + self.num_local_experts
            self.local_expert_ids = tuple(range(self.expert_start, self.expert_end))
            self.expert_id_to_local = None
            self.register_buffer("expert_owner_tensor", None, persistent=False)
            self.register_buffer("expert_local_index_tensor", None, persistent=False)
        else:
            owners = list(expert_owners)
            if (len(owners) != num_experts
                    or any(type(o) is not int or not 0 <= o < ep_size for o in owners)
                    or any(owners.count(r) != self.num_local_experts for r in range(ep_size))):
                raise ValueError("expert placement must assign equal experts per EP rank")
            self.expert_start = -1
            self.expert_end = -1
            self.local_expert_ids = tuple(e for e, o in enumerate(owners) if o == ep_rank)
            self.expert_id_to_local = {e: i for i, e in enumerate(self.local_expert_ids)}
            self.register_buffer(
                "expert_owner_tensor", torch.tensor(owners, dtype=torch.int64), persistent=False)
            self.register_buffer(
                "expert_local_index_tensor",
                torch.tensor([self.expert_id_to_local.get(e, -1) for e in range(num_experts)],
                             dtype=torch.int64),
                persistent=False)
        # int32 owner map for the EP exchange kernels (kept in sync by relocate_experts).
        self.register_buffer(
            "_owner_i32", torch.tensor(self.expert_owners, dtype=torch.int32), persistent=False)

        self.gate = ReplicatedGate(hidden_size, num_experts)
        self.gate_up_proj = nn.Parameter(
            torch.empty(self.num_local_experts, 2 * intermediate_size, hidden_size))
        self.down_proj = nn.Parameter(
            torch.empty(self.num_local_experts, hidden_size, intermediate_size))
        self.shared_expert = (
            SharedExpertMLP(hidden_size, shared_expert_intermediate_size)
            if shared_expert_intermediate_size is not None else None)
        self.shared_expert_gate = (
            ReplicatedGate(hidden_size, 1) if shared_expert_intermediate_size is not None
            else None)
        # A shared expert as wide as the routed experts runs as one more
        # expert of the grouped GEMMs: its weights sit right after the local
        # experts' in one storage per projection, and the parameters
        # (gate_up_proj, down_proj, shared_expert.*.weight) are views of it.
        self._shared_in_store = shared_expert_intermediate_size == intermediate_size
        if self._shared_in_store:
            self._bind_shared_store()
        # False: compute the shared expert after the routed output, as the
        # reference does, even where the fused form applies.
        self.fuse_shared_expert = True
        # True: batches of up to ops.ROUTE_GATE_MAX_TOKENS tokens compute the
        # router projection inside the routing kernel (one launch instead of
        # a cuBLAS GEMM plus the router).  Off by default: its fp32
        # accumulation order differs from cuBLAS's, so a bf16 logit can differ
        # by one unit and with it the routing of that token.
        self.fuse_router_gate = False

        # Kernel entry points; tests may substitute an object with the same
        # functions to exercise the host logic without a GPU.
        self._ops = _native_ops
        # "auto" | "stream" | "tcgen05" | "tcgen05-wide" | "tcgen05-swap" |
        # "tcgen05-pair" | "tcgen05-tall": expert GEMM engine ("tcgen05" lets
        # the library pick the variant per call).
        self.expert_engine = "auto"
        # Optional object with begin(name)/end(name) that records CUDA events
        # around the grouped GEMM launches (used by the benchmark).
        self.kernel_timer = None
        self.ep_all_reduce_count = 0
        self.ep_reduce_scatter_count = 0
        self.ep_all_gather_count = 0
        self.ep_all_to_all_count = 0
        self.ep_broadcast_count = 0
        self.total_assignment_count = 0
        # Largest batch (tokens per rank) the NVLink exchange buffers hold
        # ("all_to_all_nvlink"); None: nvl.DEFAULT_MAX_TOKENS.
        self.nvl_max_tokens: int | None = None
        # Under CUDA-graph capture without coordinated per-rank token counts,
        # the exchange sizes its temporaries for every peer holding as many
        # tokens as this rank (the reference's equal-batch contract).  Set to
        # the largest batch any peer may replay with (e.g. the largest decode
        # graph size) to let ranks replay graphs of different batch sizes in
        # the same step.
        self.nvl_graph_peer_tokens: int | None = None
        # Eager calls of the NVLink exchange read the received route count
        # once per layer and size the temporaries exactly.  True (or
        # B200MOE_NVL_EAGER_DEVICE_SIZES=1): size them from host bounds and
        # keep the count on the device, as under graph capture -- no host
        # read per layer, more memory for the temporaries.
        self.nvl_eager_device_sizes = (
            os.environ.get("B200MOE_NVL_EAGER_DEVICE_SIZES", "0") == "1")
        # Counters fed by kernels: host part + device accumulator
        # [local kept routes, dropped routes, dispatched tokens], read
        # (synchronising) on access.
        self._host_counts = {"dispatch": 0, "return": 0, "dropped": 0, "tokens": 0}
        self._stats: torch.Tensor | None = None

    # ------------------------------------------------------------------
    # Shared expert storage.
    # ------------------------------------------------------------------
    def _shared_pairs(self):
        return ((self.gate_up_proj, self.shared_expert.gate_up_proj.weight),
                (self.down_proj, self.shared_expert.down_proj.weight))

    def _shares_store(self, routed: torch.Tensor, shared: torch.Tensor) -> bool:
        if not (routed.is_contiguous() and shared.is_contiguous()
                and routed.device == shared.device and routed.dtype == shared.dtype):
            return False
        if routed.device.type == "meta":
            return False
        if routed.untyped_storage().data_ptr() != shared.untyped_storage().data_ptr():
            return False
        return shared.data_ptr() == routed.data_ptr() + routed.numel() * routed.element_size()

    def _bind_shared_store(self) -> None:
        """Re-home the routed and shared weights into one [E_loc + 1, ...]
        storage per projection (shared expert last) unless they already share
        one; parameters keep their identity (only ``.data`` changes)."""
        num_local = self.num_local_experts
        for routed, shared in self._shared_pairs():
            if self._shares_store(routed, shared):
                continue
            store = torch.empty((num_local + 1, *routed.shape[1:]), device=routed.device,
                                dtype=routed.dtype)
            if routed.device.type != "meta":
                with torch.no_grad():
                    store[:num_local].copy_(routed.detach())
                    store[num_local].copy_(shared.detach())
            routed.data = store[:num_local]
            shared.data = store[num_local]

    def _apply(self, fn, recurse=True):
        # Device and dtype moves rebuild every parameter separately; put the
        # shared expert back behind the routed experts afterwards.
        super()._apply(fn, recurse)
        if getattr(self, "_shared_in_store", False):
            self._bind_shared_store()
        return self

    def _shared_store(self) -> tuple[torch.Tensor, torch.Tensor]:
        """[E_loc + 1, 2I, H] and [E_loc + 1, H, I] views over the routed and
        shared expert weights."""
        if _capturing():
            pairs_ok = all(self._shares_store(r, s) for r, s in self._shared_pairs())
            if not pairs_ok:
                raise RuntimeError("shared-expert storage was split; run one eager forward "
                                   "before capturing")
        else:
            self._bind_shared_store()
        out = []
        for routed, _ in self._shared_pairs():
            size = (routed.size(0) + 1, *routed.shape[1:])
            out.append(routed.detach().as_strided(size, routed.stride(), routed.storage_offset()))
        return out[0], out[1]

    def _fused_shared(self, x: torch.Tensor) -> bool:
        """The shared expert runs inside the grouped expert path: same width
        as the routed experts, one EP rank (with several, the reference adds
        it once per rank after the exchange), the native kernels."""
        return (self.shared_expert is not None and getattr(self, "_shared_in_store", False)
                and self.fuse_shared_expert and self.ep_size == 1 and self._ops is _native_ops and x.is_cuda
                and self.top_k < 32)

    # ------------------------------------------------------------------
    # Counters (moe.py:384-393).  Kernels accumulate local assignments and
    # capacity drops on the device outside graph capture; reading a counter
    # synchronises once.
    # ------------------------------------------------------------------
    def _device_stats(self, device: torch.device) -> torch.Tensor | None:
        if _capturing():
            return None
        if self._stats is None or self._stats.device != device:
            previous = self._read_stats()
            self._host_counts["dispatch"] += previous[0]
            self._host_counts["return"] += previous[0]
            self._host_counts["dropped"] += previous[1]
            self._host_counts["tokens"] += previous[2]
            self._stats = torch.zeros(3, device=device, dtype=torch.int64)
        return self._stats

    def _read_stats(self) -> tuple[int, int, int]:
        if self._stats is None:
            return 0, 0, 0
        kept, dropped, tokens = self._stats.tolist()
        return int(kept), int(dropped), int(tokens)

    @property
    def total_dispatch_token_count(self) -> int:
        return self._host_counts["tokens"] + self._read_stats()[2]

    @total_dispatch_token_count.setter
    def total_dispatch_token_count(self, value: int) -> None:
        self._host_counts["tokens"] = int(value) - self._read_stats()[2]

    @property
    def dispatch_assignment_count(self) -> int:
        return self._host_counts["dispatch"] + self._read_stats()[0]

    @dispatch_assignment_count.setter
    def dispatch_assignment_count(self, value: int) -> None:
        self._host_counts["dispatch"] = int(value) - self._read_stats()[0]

    @property
    def return_assignment_count(self) -> int:
        return self._host_counts["return"] + self._read_stats()[0]

    @return_assignment_count.setter
    def return_assignment_count(self, value: int) -> None:
        self._host_counts["return"] = int(value) - self._read_stats()[0]

    @property
    def dropped_assignment_count(self) -> int:
        return self._host_counts["dropped"] + self._read_stats()[1]

    @dropped_assignment_count.setter
    def dropped_assignment_count(self, value: int) -> None:
        self._host_counts["dropped"] = int(value) - self._read_stats()[1]

    # ------------------------------------------------------------------
    # Placement (moe.py:395-544).
    # ------------------------------------------------------------------
    @property
    def expert_parameter_bytes(self) -> int:
        return sum(p.numel() * p.element_size() for p in (self.gate_up_proj, self.down_proj))

    def owns_expert(self, expert_id: int) -> bool:
        if self.expert_id_to_local is not None:
            return expert_id in self.expert_id_to_local
        return self.expert_start <= expert_id < self.expert_end

    def _local_id(self, expert_id: int) -> int:
        return (expert_id - self.expert_start if self.expert_id_to_local is None
                else self.expert_id_to_local[expert_id])

    def load_expert_weight(self, expert_id: int, projection: str,
                           loaded_weight: torch.Tensor) -> None:
        if not self.owns_expert(expert_id):
            return
        local = self._local_id(expert_id)
        if projection == "gate_proj":
            target = self.gate_up_proj[local, : self.intermediate_size]
        elif projection == "up_proj":
            target = self.gate_up_proj[local, self.intermediate_size:]
        elif projection == "down_proj":
            target = self.down_proj[local]
        else:
            raise ValueError(f"unknown expert projection: {projection}")
        target.data.copy_(loaded_weight)

    @torch.no_grad()
    def relocate_experts(self, expert_owners: tuple[int, ...] | list[int]) -> int:
        """Move expert weights between EP ranks in place (moe.py:407-489).

        Every rank must request the same placement (agreed with
        all_gather_object before any data moves).  Per projection the rows
        that leave are gathered with one index_select, travel with one NCCL
        all_to_all_single and land with one index_copy_ in the existing
        parameter storage, so captured CUDA graphs stay valid.
        """
        if not self.dynamic_placement:
            raise RuntimeError("runtime expert placement was not enabled")
        owners = tuple(expert_owners)
        if (len(owners) != self.num_experts
                or any(type(o) is not int or not 0 <= o < self.ep_size for o in owners)
                or any(owners.count(r) != self.num_local_experts for r in range(self.ep_size))):
            raise ValueError("expert placement must assign equal experts per EP rank")
        group = dist_env.get_moe_group()
        if self.ep_size > 1:
            proposals = [None] * self.ep_size
            dist.all_gather_object(proposals, owners, group=group)
            if any(p != owners for p in proposals):
                raise ValueError("all EP ranks must request the same expert placement")
        if owners == self.expert_owners:
            return 0
        old = self.expert_owners
        new_ids = tuple(e for e, o in enumerate(owners) if o == self.ep_rank)
        new_local = {e: i for i, e in enumerate(new_ids)}
        # Rows leave in destination order, within a destination in expert
        # order; they arrive in source order, within a source in expert order.
        outgoing = [e for d in range(self.ep_size) for e in self.local_expert_ids if owners[e] == d]
        send_counts = [sum(owners[e] == d for e in self.local_expert_ids)
                       for d in range(self.ep_size)]
        incoming = [e for s in range(self.ep_size) for e in new_ids if old[e] == s]
        recv_counts = [sum(old[e] == s for e in new_ids) for s in range(self.ep_size)]
        device = self.gate_up_proj.device
        gather = torch.tensor([self.expert_id_to_local[e] for e in outgoing], device=device)
        scatter = torch.tensor([new_local[e] for e in incoming], device=device)

        def exchange(param: torch.Tensor) -> None:
            # One gather of the rows that leave, one all-to-all, one scatter
            # into the same storage (captured graphs keep their pointers).
            rows = param.index_select(0, gather)
            if self.ep_size > 1:
                received = torch.empty_like(rows)
                row = param[0].numel()
                dist.all_to_all_single(received.view(-1), rows.view(-1),
                                       [c * row for c in recv_counts],
                                       [c * row for c in send_counts], group=group)
            else:
                received = rows
            param.index_copy_(0, scatter, received)

        exchange(self.gate_up_proj)
        exchange(self.down_proj)
        self.expert_owner_tensor.copy_(torch.tensor(owners, device=self.expert_owner_tensor.device))
        self.expert_local_index_tensor.copy_(torch.tensor(
            [new_local.get(e, -1) for e in range(self.num_experts)],
            device=self.expert_local_index_tensor.device))
        self._owner_i32.copy_(torch.tensor(owners, dtype=torch.int32, device=self._owner_i32.device))
        self.local_expert_ids = new_ids
        self.expert_id_to_local = new_local
        self.expert_owners = owners
        return sum(a != b for a, b in zip(old, owners))

    # ------------------------------------------------------------------
    # Seams kept from the reference.
    # ------------------------------------------------------------------
    def _local_routes(self, flat_experts: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Route -> (is local, local expert id) (moe.py:491-517).

        Compatibility seam only: the native path maps routes inside
        b200moe_pack_routes.
        """
        if self.expert_id_to_local is None:
            mask = (flat_experts >= self.expert_start) & (flat_experts < self.expert_end)
            return mask, flat_experts - self.expert_start
        valid = (flat_experts >= 0) & (flat_experts < self.num_experts)
        safe = flat_experts.clamp(0, self.num_experts - 1)
        local = self.expert_local_index_tensor.to(flat_experts.device)[safe]
        mask = valid & (local >= 0)
        return mask, torch.where(valid, local, torch.full_like(local, -1))

    def _can_use_native_kernel(self, hidden_states: torch.Tensor) -> bool:
        return (hidden_states.is_cuda and hidden_states.dtype == torch.bfloat16
                and self.gate_up_proj.dtype == torch.bfloat16
                and self.down_proj.dtype == torch.bfloat16)

    # The reference name of the same check (moe.py:582-589).
    _can_use_triton_kernel = _can_use_native_kernel

    @property
    def graph_token_limit(self) -> int:
        dp_size = (self.ep_size // dist_env.get_tp_world_size()
                   if self.dispatch_backend in ("allgather_reduce", "allgather_reducescatter")
                   else 1)
        return MOE_MAX_GRAPH_TOKENS_PER_RANK * dp_size

    def _capacity(self, num_tokens: int) -> int | None:
        if self.expert_capacity is not None:
            return int(self.expert_capacity)
        if self.expert_capacity_factor is not None:
            # Same float expression and evaluation order as moe.py:882-885.
            return max(1, math.ceil(
                self.expert_capacity_factor * num_tokens * self.top_k / self.num_experts))
        return None

    def _pack(self, flat_ids: torch.Tensor, flat_weights: torch.Tensor | None, *,
              capacity: int | None = None, expert_base: torch.Tensor | None = None,
              stats: torch.Tensor | None = None, route_count: torch.Tensor | None = None,
              capacity_dev: torch.Tensor | None = None):
        local_index = self.expert_local_index_tensor if self.expert_id_to_local is not None else None
        bounds = {}
        if route_count is not None or capacity_dev is not None:
            bounds = dict(route_count=route_count, capacity_dev=capacity_dev)
        return self._ops.pack_routes(
            flat_ids, flat_weights, self.num_experts, self.num_local_experts,
            local_index=local_index, expert_start=max(self.expert_start, 0),
            expert_base=expert_base, capacity=capacity, stats=stats, **bounds)

    def _use_tiny_path(self, num_tokens: int, logits: torch.Tensor) -> bool:
        """Two-launch fused path: tiny buckets, no capacity, plain bf16 combine."""
        return (self.expert_engine == "auto" and self._ops is _native_ops
                and num_tokens * self.top_k <= _native_ops.TINY_MAX_ROUTES
                and self.expert_capacity is None and self.expert_capacity_factor is None
                and not self.fp64_combine and not self.fp32_reduce
                and logits.dtype in (torch.float32, torch.bfloat16))

    def _engine(self, num_routes: int) -> int:
        if self.expert_engine == "stream":
            return _lib.ENGINE_STREAM
        if self.expert_engine == "tcgen05":
            return _lib.ENGINE_TCGEN05
        if self.expert_engine == "tcgen05-wide":
            return _lib.ENGINE_TCGEN05_WIDE
        if self.expert_engine == "tcgen05-swap":
            return _lib.ENGINE_TCGEN05_SWAP
        if self.expert_engine == "tcgen05-pair":
            return _lib.ENGINE_TCGEN05_PAIR
        if self.expert_engine == "tcgen05-tall":
            return _lib.ENGINE_TCGEN05_TALL
        if self.expert_engine != "auto":
            raise ValueError(f"unknown expert engine {self.expert_engine!r}")
        return _lib.ENGINE_STREAM if num_routes <= STREAM_ENGINE_MAX_ROUTES else _lib.ENGINE_TCGEN05

    def _run_experts(self, x: torch.Tensor, flat_weights: torch.Tensor, packed, top_k: int,
                     token_of_route: torch.Tensor | None = None,
                     routes_hint: int | None = None,
                     weights: tuple[torch.Tensor, torch.Tensor] | None = None,
                     scatter: tuple | None = None) -> torch.Tensor | None:
        """Grouped gate/up + SwiGLU and grouped down -> y [num_routes, H] (route order).

        ``routes_hint``: the expected number of routes when ``packed`` is
        bounded on the device (its host num_routes is then only a maximum);
        it picks the tcgen05 variant and the row-gather strategy, and the
        streaming engine (whose route bound is compiled in) is not used.
        ``weights``: (w13, w2) to use instead of the local experts' (the
        routed + shared storage).  ``scatter``: (src_rank, src_route, bufs)
        of the NVLink exchange: the down rows go straight to the sources'
        return buffers (tcgen05 wide / swap-AB down) and None is returned."""
        w13, w2 = (self.gate_up_proj, self.down_proj) if weights is None else weights
        routes = packed.num_routes if routes_hint is None else max(1, int(routes_hint))
        engine = self._engine(routes)
        if routes_hint is not None and engine in (_lib.ENGINE_STREAM, _lib.ENGINE_TCGEN05):
            engine = (_lib.ENGINE_TCGEN05_SWAP if routes <= 4096 else _lib.ENGINE_TCGEN05_WIDE)
        ops = self._ops
        timer = self.kernel_timer
        if engine == _lib.ENGINE_STREAM or (engine != _lib.ENGINE_TCGEN05_PAIR and
                                            routes <= FUSED_GATHER_MAX_ROUTES):
            # The streaming engine reads token rows directly; for small
            # buckets the one-SM tcgen05 engines gather them inside their TMA
            # loads (four rows per tile::gather4), saving the gather launch.
            x_packed = None
        else:
            # Larger calls: one 128-row (or 16-row) TMA box per stage from a
            # packed copy beats 32 four-row gathers per stage.
            x_packed = ops.gather_rows(x, packed, top_k, token_of_route)
        if timer is not None:
            timer.begin("gate_up")
        act = ops.expert_gate_up(engine, x, x_packed, w13, packed, top_k, token_of_route)
        if timer is not None:
            timer.end("gate_up")
            timer.begin("down")
        if scatter is not None:
            down_engine = (engine if engine in (_lib.ENGINE_TCGEN05_WIDE, _lib.ENGINE_TCGEN05_SWAP)
                           else _lib.ENGINE_TCGEN05_SWAP if routes <= 4096
                           else _lib.ENGINE_TCGEN05_WIDE)
            ops.expert_down_scatter(down_engine, act, w2, packed, flat_weights, *scatter)
            y = None
        else:
            y = ops.expert_down(engine, act, w2, packed, flat_weights, x.size(0))
        if timer is not None:
            timer.end("down")
        return y

    def _output_dtype(self, dtype: torch.dtype) -> torch.dtype:
        return torch.float64 if self.fp64_combine else torch.float32 if self.fp32_reduce else dtype

    def _combine_expert_routes(self, expert_output: torch.Tensor, route_rows: torch.Tensor,
                               num_tokens: int, top_k: int) -> torch.Tensor:
        """Route-order combine (moe.py:642-678) on the native kernel."""
        return self._ops.combine(expert_output, route_rows, num_tokens, top_k,
                                 self._output_dtype(expert_output.dtype), self.fp64_combine)

    def _check_inputs(self, hidden_states: torch.Tensor) -> None:
        if hidden_states.dtype != torch.bfloat16:
            raise NotImplementedError(
                f"the B200 MoE path computes in bf16; got {hidden_states.dtype}")
        if self.gate_up_proj.dtype != torch.bfloat16 or self.down_proj.dtype != torch.bfloat16:
            raise NotImplementedError("expert weights must be bf16")

    def _route(self, hidden_states: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Router + capacity (moe.py:870-920) -> (bf16 weights [T,k], int64 ids [T,k])."""
        logits = self.gate(hidden_states)
        weights, experts = self._ops.route_topk(logits, self.top_k, self.norm_topk_prob)
        capacity = self._capacity(hidden_states.size(0))
        if capacity is not None:
            packed = self._pack(experts.view(-1), weights.view(-1), capacity=capacity)
            if not _capturing():
                self.dropped_assignment_count += int(
                    packed.counters[_lib.CNT_DROPPED].item())
        return weights, experts

    def _execute_local(self, hidden_states: torch.Tensor, routing_weights: torch.Tensor,
                       selected_experts: torch.Tensor) -> tuple[torch.Tensor, int]:
        """Local experts for given routes -> (output [T,H], local assignments) (moe.py:922-940)."""
        if hidden_states.size(0) == 0:
            return torch.zeros_like(hidden_states), 0
        if not self._can_use_native_kernel(hidden_states) and self._ops is _native_ops:
            raise RuntimeError(
                "the B200 MoE path needs CUDA bf16 activations and weights (no CPU path)")
        if self.graph_safe_decode and hidden_states.size(0) <= self.graph_token_limit:
            return self._forward_static_decode(hidden_states, routing_weights, selected_experts)
        return self._forward_dynamic(hidden_states, routing_weights, selected_experts)

    def _forward_compact(self, hidden_states, routing_weights, selected_experts):
        num_tokens = hidden_states.size(0)
        top_k = selected_experts.size(1)
        ids = selected_experts.contiguous()
        weights = routing_weights.contiguous().view(-1)
        packed = self._pack(ids.view(-1), None)
        y = self._run_experts(hidden_states.contiguous(), weights, packed, top_k)
        output = self._combine_expert_routes(y, packed.combine_rows, num_tokens, top_k)
        local = 0 if _capturing() else int(packed.counters[_lib.CNT_LOCAL_KEPT].item())
        return output, local

    def _forward_static_decode(self, hidden_states, routing_weights, selected_experts):
        """Graph-safe path (moe.py:783-868): fixed-capacity buffers, device-side lengths."""
        return self._forward_compact(hidden_states, routing_weights, selected_experts)

    def _forward_dynamic(self, hidden_states, routing_weights, selected_experts):
        """Eager path (reference _forward_triton, moe.py:680-771).  The native
        path needs no host synchronisation, so it is the same computation as
        the graph-safe one."""
        return self._forward_compact(hidden_states, routing_weights, selected_experts)

    # The reference's seam name for the eager path.
    _forward_triton = _forward_dynamic

    # ------------------------------------------------------------------
    # Forward.
    # ------------------------------------------------------------------
    def _forward_local(self, x: torch.Tensor, shared: bool = False) -> torch.Tensor:
        """Route + capacity + local experts + combine, no host synchronisation.
        ``shared``: include the shared expert (one more grouped expert)."""
        if x.size(0) == 0:
            return torch.zeros_like(x)
        if (self.fuse_router_gate and not shared and self._ops is _native_ops and x.is_cuda
                and x.size(0) <= _native_ops.ROUTE_GATE_MAX_TOKENS
                and x.dtype == torch.bfloat16 and self.gate.weight.dtype == torch.bfloat16):
            return self._forward_fused_gate(x)
        return self._forward_from_logits(x, self.gate(x), shared=shared)

    def _forward_fused_gate(self, x: torch.Tensor) -> torch.Tensor:
        """The router projection inside the routing launch (fuse_router_gate)."""
        num_tokens = x.size(0)
        self._check_inputs(x)
        weights, ids, logits = self._ops.route_gate_topk(x, self.gate.weight, self.top_k,
                                                         self.norm_topk_prob)
        if self._use_tiny_path(num_tokens, logits):
            # The tiny kernels route from the logits themselves (same routine).
            return self._forward_from_logits(x, logits)
        stats = self._device_stats(x.device)
        flat_w = weights.view(-1)
        packed = self._pack(ids.view(-1), flat_w, capacity=self._capacity(num_tokens),
                            stats=stats)
        y = self._run_experts(x, flat_w, packed, self.top_k)
        self.total_assignment_count += ids.numel()
        return self._combine_expert_routes(y, packed.combine_rows, num_tokens, self.top_k)

    def _forward_from_logits(self, x: torch.Tensor, logits: torch.Tensor,
                             shared: bool = False) -> torch.Tensor:
        """The expert path from given router logits [T, E] (fp32, bf16 or fp16):
        softmax top-k, capacity, packing, grouped GEMMs and combine."""
        num_tokens = x.size(0)
        if num_tokens == 0:
            return torch.zeros_like(x)
        self._check_inputs(x)
        stats = self._device_stats(x.device)
        if shared:
            return self._forward_with_shared(x, logits, stats)
        if self._use_tiny_path(num_tokens, logits):
            local_index = (self.expert_local_index_tensor if self.expert_id_to_local is not None
                           else None)
            self.total_assignment_count += num_tokens * self.top_k
            return self._ops.decode_tiny(
                logits, x.contiguous(), self.gate_up_proj, self.down_proj, self.top_k,
                self.norm_topk_prob, self.num_experts, local_index=local_index,
                expert_start=max(self.expert_start, 0), stats=stats)
        if (self._ops is _native_ops and num_tokens <= ROUTE_PACK_MAX_TOKENS
                and num_tokens * self.top_k <= _native_ops.ROUTE_PACK_MAX_ROUTES
                and self.num_experts <= 1024 and self.top_k <= 32):
            # Small batches: router and packing in one launch (same results).
            local_index = (self.expert_local_index_tensor if self.expert_id_to_local is not None
                           else None)
            weights, ids, packed = self._ops.route_pack(
                logits, self.top_k, self.norm_topk_prob, self.num_experts,
                self.num_local_experts, local_index=local_index,
                expert_start=max(self.expert_start, 0), capacity=self._capacity(num_tokens),
                stats=stats)
        else:
            weights, ids = self._ops.route_topk(logits, self.top_k, self.norm_topk_prob)
            packed = self._pack(ids.view(-1), weights.view(-1),
                                capacity=self._capacity(num_tokens), stats=stats)
        flat_w = weights.view(-1)
        y = self._run_experts(x, flat_w, packed, self.top_k)
        self.total_assignment_count += ids.numel()
        return self._combine_expert_routes(y, packed.combine_rows, num_tokens, self.top_k)

    def _forward_with_shared(self, x: torch.Tensor, logits: torch.Tensor,
                             stats: torch.Tensor | None) -> torch.Tensor:
        """Routed experts and the shared expert in one grouped expert path.

        The reference adds the shared expert after the routed output
        (moe.py:1259-1262: output + sigmoid(shared_expert_gate(x)) *
        shared_expert(x), with the MLP of moe.py:212-234).  Here every token
        gets a (top_k + 1)-th route to expert E (the shared expert, stored
        after the local experts) weighted by the bf16 sigmoid of its gate
        logit; capacity applies to the routed slots only, so routing, packing
        of the routed experts and drops are unchanged; the down epilogue
        applies the gate weight in fp32 and the route-order combine adds the
        shared row after the routed ones."""
        num_tokens = x.size(0)
        slots = self.top_k + 1
        weights, ids = self._ops.route_topk(logits, self.top_k, self.norm_topk_prob,
                                            shared_logits=self.shared_expert_gate(x))
        flat_w = weights.view(-1)
        # One EP rank: every expert is local and in order.
        packed = self._ops.pack_routes(
            ids.view(-1), flat_w, self.num_experts + 1, self.num_local_experts + 1,
            expert_start=0, capacity=self._capacity(num_tokens), stats=stats,
            num_shared_experts=1)
        y = self._run_experts(x, flat_w, packed, slots, weights=self._shared_store())
        self.total_assignment_count += num_tokens * self.top_k
        return self._combine_expert_routes(y, packed.combine_rows, num_tokens, slots)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        original_shape = hidden_states.shape
        x = hidden_states.reshape(-1, self.hidden_size)
        fused_shared = self._fused_shared(x)
        if self.dispatch_backend in ("allgather_reduce", "allgather_reducescatter") \
                and self.ep_size > 1:
            output = self._forward_global_dp(
                x, self.dispatch_backend == "allgather_reducescatter")
        elif self.dispatch_backend == "all_to_all_nvlink" and self.ep_size > 1:
            from .ep import forward_all_to_all_nvlink
            output = forward_all_to_all_nvlink(self, x)
        elif self.dispatch_backend in ("all_to_all", "all_to_all_reduce") and self.ep_size > 1:
            from .ep import forward_rank0_all_to_all
            output = forward_rank0_all_to_all(self, x, self.dispatch_backend == "all_to_all_reduce")
        else:
            output = self._forward_local(x, shared=fused_shared)
            if self.ep_size > 1:
                group = dist_env.get_moe_group()
                if self.fp64_staged_reduce:
                    output = reduce_fp64_to_bf16(output.double(), group, x.dtype)
                    self.ep_reduce_scatter_count += 1
                    self.ep_all_gather_count += 1
                else:
                    dist.all_reduce(output, group=group)
                    if output.dtype != x.dtype:
                        output = output.to(x.dtype)
                    self.ep_all_reduce_count += 1
            elif output.dtype != x.dtype:
                output = output.to(x.dtype)
        if self.shared_expert is not None and not fused_shared:
            shared = self.shared_expert(x)
            output = output + torch.sigmoid(self.shared_expert_gate(x)) * shared
        return output.reshape(original_shape)

    def _forward_global_dp(self, hidden_states: torch.Tensor,
                           reduce_scatter_output: bool) -> torch.Tensor:
        """Cross-DP all-gather backends (moe.py:942-1018) on the native kernels."""
        from .ep import forward_global_dp
        return forward_global_dp(self, hidden_states, reduce_scatter_output)
