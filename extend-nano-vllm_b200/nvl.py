"""Exchange buffers of the expert-parallel NVLink exchange (csrc/nvl.cu).

Each EP rank owns one device buffer, laid out by b200moe_nvl_buffer_bytes
(flags, epoch, mailboxes, per-source route records and token rows, and the
return rows of its own routes), and maps every peer's buffer into its
address space with CUDA IPC.  The handles are exchanged once, with
torch.distributed object collectives on the MoE group, the first time a
layer of a given shape runs; that first call must not be under CUDA-graph
capture (the model runner's eager warm-up makes it).  Every MoE layer of the
same shape and group shares one buffer: layers run one after another on
every rank, and a rank writes into a peer's region again only after that
peer returned the previous exchange's rows, which it does after its last
read of the region.
"""

from __future__ import annotations

import atexit
import ctypes
import os

import torch
import torch.distributed as dist

from . import _lib
from ._lib import call

# Largest batch (tokens per rank) an exchange buffer is sized for unless the
# layer says otherwise (ExpertParallelMoE.nvl_max_tokens).
DEFAULT_MAX_TOKENS = int(os.environ.get("B200MOE_NVL_MAX_TOKENS", "8192"))

_LAYOUT_FIELDS = ("flags", "control", "mailbox", "hist", "meta", "records", "tokens",
                  "returned", "route_cap", "total")


class ExchangeBuffers:
    """One rank's exchange buffer and the device addresses of every rank's."""

    def __init__(self, *, ep_size: int, rank: int, max_tokens: int, top_k: int,
                 num_experts: int, num_local_experts: int, hidden: int,
                 device: torch.device) -> None:
        self.ep_size = ep_size
        self.rank = rank
        self.max_tokens = max_tokens
        self.top_k = top_k
        self.num_experts = num_experts
        self.num_local_experts = num_local_experts
        self.hidden = hidden
        self.device = torch.device(device)
        self._layout = (ctypes.c_int64 * _lib.NVL_LAYOUT_WORDS)()
        nbytes = int(_lib.LIB.b200moe_nvl_buffer_bytes(ep_size, max_tokens, top_k, num_experts,
                                                        num_local_experts, hidden,
                                                        self._layout))
        if nbytes < 0:
            raise ValueError(_lib.LIB.b200moe_last_error().decode(errors="replace"))
        self.layout = dict(zip(_LAYOUT_FIELDS, list(self._layout)))
        self.layout_ptr = ctypes.cast(self._layout, ctypes.c_void_p)
        self.route_cap = self.layout["route_cap"]
        self.max_routes = ep_size * self.route_cap
        # Zeroed: flags, epoch and retirement counters start at 0 on every rank.
        self.buffer = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self._bases = (ctypes.c_uint64 * ep_size)()
        self.peer_bases = ctypes.cast(self._bases, ctypes.c_void_p)
        self._opened: list[tuple[int, int]] = []

    # -- connecting ----------------------------------------------------------
    def connect_local(self, all_ranks: list["ExchangeBuffers"]) -> None:
        """Every rank's buffer lives in this process (one GPU driving all the
        ranks of an exchange, e.g. to test the exchange on a single device)."""
        for r, other in enumerate(all_ranks):
            self._bases[r] = other.buffer.data_ptr()

    def connect_group(self, group) -> None:
        """Exchange CUDA IPC handles with the other ranks of `group` and map
        their buffers (collective: every rank of the group calls it)."""
        handle = (ctypes.c_char * 64)()
        offset = ctypes.c_int64(0)
        call("b200moe_ipc_handle", ctypes.c_void_p(self.buffer.data_ptr()), handle,
             ctypes.byref(offset))
        mine = (self.rank, bytes(handle), int(offset.value), self.buffer.data_ptr())
        everyone = [None] * self.ep_size
        dist.all_gather_object(everyone, mine, group=group)
        for rank, raw, off, ptr in everyone:
            if rank == self.rank:
                self._bases[rank] = self.buffer.data_ptr()
                continue
            mapped = ctypes.c_void_p(0)
            call("b200moe_ipc_open", ctypes.create_string_buffer(raw, 64), off,
                 ctypes.byref(mapped))
            self._bases[rank] = mapped.value
            self._opened.append((mapped.value, off))

    def close(self) -> None:
        for ptr, off in self._opened:
            try:
                call("b200moe_ipc_close", ctypes.c_void_p(ptr), off)
            except Exception:  # noqa: BLE001 - best effort at shutdown
                pass
        self._opened.clear()

    # -- views -----------------------------------------------------------------
    def tokens_view(self) -> torch.Tensor:
        """Received token rows [ep_size * max_tokens, hidden] (bf16)."""
        start = self.layout["tokens"]
        n = self.ep_size * self.max_tokens * self.hidden * 2
        return self.buffer[start:start + n].view(torch.bfloat16).view(-1, self.hidden)

    def returned_view(self, rows: int) -> torch.Tensor:
        """This rank's returned route rows [rows, hidden] (bf16), route order."""
        start = self.layout["returned"]
        return self.buffer[start:start + rows * self.hidden * 2].view(torch.bfloat16).view(
            rows, self.hidden)

    def stream_ptr(self) -> ctypes.c_void_p:
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)


_CACHE: dict[tuple, ExchangeBuffers] = {}


def buffers_for(layer, device: torch.device, group) -> ExchangeBuffers:
    """The exchange buffer shared by layers of this shape on this group/device."""
    max_tokens = int(getattr(layer, "nvl_max_tokens", None) or DEFAULT_MAX_TOKENS)
    key = (id(group), layer.ep_size, layer.ep_rank, max_tokens, layer.top_k, layer.num_experts,
           layer.num_local_experts, layer.hidden_size, str(device))
    bufs = _CACHE.get(key)
    if bufs is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the NVLink exchange buffers are set up on the first eager call; "
                               "run one forward before capturing a CUDA graph")
        bufs = ExchangeBuffers(ep_size=layer.ep_size, rank=layer.ep_rank, max_tokens=max_tokens,
                               top_k=layer.top_k, num_experts=layer.num_experts,
                               num_local_experts=layer.num_local_experts,
                               hidden=layer.hidden_size, device=device)
        bufs.connect_group(group)
        _CACHE[key] = bufs
    return bufs


@atexit.register
def _close_all() -> None:
    for bufs in _CACHE.values():
        bufs.close()
