"""Process-group and forward-context accessors used by the MoE layer.

Inside nano-vLLM the layer reads its groups from
``nanovllm.distributed.parallel_state`` (EP group = DP x TP ranks,
parallel_state.py:92-110) and the cross-DP token counts from
``nanovllm.utils.context.get_context()`` (context.py:15-17).  When nano-vLLM
is importable those are used unchanged; otherwise (standalone use, the tests
and the benchmark) the MoE group is the default torch.distributed group, TP
size is 1 and the context is a module-level object.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch.distributed as dist

try:  # Running inside nano-vLLM: share its groups and forward context.
    from nanovllm.distributed import parallel_state as _ps  # type: ignore
    from nanovllm.utils.context import get_context as _nano_get_context  # type: ignore
except Exception:  # noqa: BLE001 - any import failure means standalone use
    _ps = None
    _nano_get_context = None


@dataclass
class MoEContext:
    """The two fields of nano-vLLM's Context that the MoE layer reads."""

    moe_token_counts: tuple[int, ...] | None = None
    is_dummy: bool = False


_LOCAL_CONTEXT = MoEContext()


def get_context():
    return _nano_get_context() if _nano_get_context is not None else _LOCAL_CONTEXT


def set_moe_token_counts(counts: tuple[int, ...] | None, is_dummy: bool = False) -> None:
    """Standalone use: record every DP replica's token count for this forward."""
    ctx = get_context()
    ctx.moe_token_counts = None if counts is None else tuple(int(c) for c in counts)
    ctx.is_dummy = is_dummy


def _world():
    return dist.group.WORLD if dist.is_initialized() else None


def get_moe_group():
    return _ps.get_moe_group() if _ps is not None else _world()


def get_ep_group():
    return _ps.get_ep_group() if _ps is not None else _world()


def get_ep_group_ranks() -> tuple[int, ...]:
    if _ps is not None:
        return _ps.get_ep_group_ranks()
    return tuple(range(dist.get_world_size())) if dist.is_initialized() else (0,)


def get_tp_group():
    return _ps.get_tp_group() if _ps is not None else None


def get_tp_world_size() -> int:
    return _ps.get_tp_world_size() if _ps is not None else 1
