"""The C-ABI library loads without a GPU, exports every declared symbol, and
rejects bad arguments before touching the device."""

import ctypes
import os
import re

import pytest

from extend_nano_vllm_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "b200moe.h")


def declared_symbols() -> list[str]:
    text = open(HEADER).read()
    return re.findall(r"B200MOE_API\s+[\w\s\*]+?\b(b200moe_\w+)\s*\(", text)


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_symbols()
    assert len(names) >= 15
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_abi_version():
    assert _lib.LIB.b200moe_abi_version() == 1


def test_layout_sizes_match_reference_formulas():
    # tests/test_moe_compact_layout.py:38: T=512, k=8, E=128 -> 6016 index rows.
    assert _lib.LIB.b200moe_pack_row_capacity(4096, 128) == 6016
    assert _lib.LIB.b200moe_pack_row_capacity(8, 128) == 128
    assert _lib.LIB.b200moe_pack_max_mtiles(4096, 128) == 32 + 128
    assert _lib.LIB.b200moe_pack_max_mtiles(8, 128) == 1 + 8
    assert _lib.LIB.b200moe_pack_scratch_bytes(1024, 128) == 129 * 4
    assert _lib.LIB.b200moe_pack_scratch_bytes(65536, 128) == 64 * 129 * 4


def test_argument_errors_without_device():
    null = ctypes.c_void_p(0)
    with pytest.raises(ValueError, match="top_k"):
        _lib.call("b200moe_route_topk", null, _lib.F32, 4, 8, 9, 1, null, null, null)
    with pytest.raises(NotImplementedError, match="top_k"):
        _lib.call("b200moe_route_topk", null, _lib.F32, 4, 64, 33, 1, null, null, null)
    with pytest.raises(ValueError, match="num_local_experts"):
        _lib.call("b200moe_pack_routes", null, null, 16, 8, null, 0, 9, null, -1, 32, null,
                  null, null, null, null, null, null, 10, null, null, null, null, 0, null)
    with pytest.raises(NotImplementedError, match="multiples of 16"):
        _lib.call("b200moe_expert_gate_up", 0, null, 1, null, 24, 64, null, 1, null, null, 1, 1,
                  16, null, 1, null, null, null, null)
    with pytest.raises(ValueError, match="ep_size"):
        _lib.call("b200moe_ep_plan", null, 1, 1, 8, null, 17, null, null, null, null)


def test_static_scratch_limit_is_the_scratch_rule_not_a_route_bound():
    """The no-scratch packing call accepts exactly the calls whose scratch need
    fits the library's array; the need is not monotone in the route count
    (route chunks widen once more than 512 blocks would be needed)."""
    cap = int(_lib.LIB.b200moe_pack_static_scratch_capacity())
    need = lambda r, e: int(_lib.LIB.b200moe_pack_scratch_bytes(r, e))  # noqa: E731
    assert need(520_192, 128) <= cap < need(520_193, 128)
    assert need(524_288, 128) > cap and need(600_000, 128) <= cap
    null = ctypes.c_void_p(0)
    for routes in (520_193, 524_288):
        with pytest.raises(ValueError, match="static scratch"):
            _lib.call("b200moe_pack_routes_static_scratch", null, null, routes, 128, null, 0,
                      128, null, -1, 0, null, null, null, null, null, null, null, 0, null, null,
                      null)


def test_argument_errors_of_the_fused_entry_points():
    """The shared-expert, route+pack, fused-projection and scattered-down
    entry points check their arguments before touching a device."""
    null = ctypes.c_void_p(0)
    fake = ctypes.c_void_p(256)  # checked for null only, never dereferenced here
    with pytest.raises(NotImplementedError, match="top_k 32 > 31"):
        _lib.call("b200moe_route_topk_shared", null, _lib.F32, 4, 64, 32, 1, fake, null, null,
                  null)
    with pytest.raises(ValueError, match="shared_logits is null"):
        _lib.call("b200moe_route_topk_shared", null, _lib.F32, 4, 64, 8, 1, null, null, null,
                  null)
    with pytest.raises(ValueError, match="num_shared_experts"):
        _lib.call("b200moe_pack_routes_shared", null, null, 16, 8, 8, null, 0, 8, -1, 32, null,
                  null, null, null, fake, fake, null, 10, null, fake, null, null, 0, null)
    with pytest.raises(ValueError, match="num_tokens \\* top_k"):
        _lib.call("b200moe_route_pack", null, _lib.F32, 200, 128, 8, 1, null, null, null, 0,
                  128, -1, 0, null, null, null, null, null, null, null, 0, null, null, null,
                  null, 0, null)
    with pytest.raises(NotImplementedError, match="at most 64 tokens"):
        _lib.call("b200moe_route_gate_topk", null, 2048, null, 65, 128, 8, 1, null, null, null,
                  null, null)
    with pytest.raises(ValueError, match="dst_ranks"):
        _lib.call("b200moe_expert_down_scatter", 0, null, 64, 64, null, 1, null, null, 1, 16,
                  null, 1, null, null, 17, 0, null, null, 1, null)
    with pytest.raises(ValueError, match="ep_size|rank"):
        _lib.call("b200moe_nvl_return_signal", 3, 2, null, null, null)
