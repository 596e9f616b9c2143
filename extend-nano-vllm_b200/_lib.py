"""ctypes binding of libb200moe.so, the C ABI declared in include/b200moe.h.

The library is loaded once per process from this package directory.  There
is no fallback: if the shared library is missing the import fails with a
message saying how to build it, and every call that returns a non-zero status
raises ``B200MoEError`` with the library's own message.
"""

from __future__ import annotations

import ctypes
import os

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libb200moe.so")

OK = 0
EINVAL = 1
ECUDA = 2
EUNSUPPORTED = 3

BF16, F16, F32, F64 = 0, 1, 2, 3
ENGINE_STREAM, ENGINE_TCGEN05, ENGINE_TCGEN05_WIDE, ENGINE_TCGEN05_SWAP = 0, 1, 2, 3
ENGINE_TCGEN05_PAIR = 4
ENGINE_TCGEN05_TALL = 5
MTILE_WORDS = 3
MTILE_ROWS = 128
CHUNK_ROWS = 256
BLOCK_ROWS = 16
CNT_PADDED_ROWS, CNT_MTILES, CNT_LOCAL_KEPT, CNT_DROPPED, CNT_CHUNKS = 0, 1, 2, 3, 4
NUM_COUNTERS = 5

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_S = ctypes.c_size_t

# name -> (restype, argtypes); must match include/b200moe.h.
SIGNATURES: dict[str, tuple] = {
    "b200moe_last_error": (ctypes.c_char_p, []),
    "b200moe_abi_version": (_I, []),
    "b200moe_device_status": (_I, [_P, _I]),
    "b200moe_route_topk": (_I, [_P, _I, _L, _I, _I, _I, _P, _P, _P]),
    "b200moe_route_topk_shared": (_I, [_P, _I, _L, _I, _I, _I, _P, _P, _P, _P]),
    "b200moe_route_gate_topk": (_I, [_P, _I, _P, _L, _I, _I, _I, _P, _P, _P, _P, _P]),
    "b200moe_pack_scratch_bytes": (_S, [_L, _I]),
    "b200moe_pack_row_capacity": (_L, [_L, _I]),
    "b200moe_pack_max_mtiles": (_L, [_L, _I]),
    "b200moe_pack_routes": (_I, [_P, _P, _L, _I, _P, _I, _I, _P, _L, _L, _P, _P, _P, _P, _P,
                                 _P, _P, _L, _P, _P, _P, _P, _S, _P]),
    "b200moe_pack_routes_shared": (_I, [_P, _P, _L, _I, _I, _P, _I, _I, _L, _L, _P, _P, _P, _P,
                                        _P, _P, _P, _L, _P, _P, _P, _P, _S, _P]),
    "b200moe_route_pack": (_I, [_P, _I, _L, _I, _I, _I, _P, _P, _P, _I, _I, _L, _L, _P, _P, _P,
                                _P, _P, _P, _P, _L, _P, _P, _P, _P, _S, _P]),
    "b200moe_pack_static_scratch_capacity": (_S, []),
    "b200moe_pack_routes_static_scratch": (_I, [_P, _P, _L, _I, _P, _I, _I, _P, _L, _L, _P, _P,
                                                _P, _P, _P, _P, _P, _L, _P, _P, _P]),
    "b200moe_expert_histogram": (_I, [_P, _L, _I, _P, _P]),
    "b200moe_gather_rows": (_I, [_P, _L, _I, _P, _P, _I, _L, _L, _P, _P, _P]),
    "b200moe_expert_gate_up": (_I, [_I, _P, _L, _P, _I, _I, _P, _I, _P, _P, _I, _L, _L, _P,
                                    _L, _P, _P, _P, _P]),
    "b200moe_expert_down": (_I, [_I, _P, _I, _I, _P, _I, _P, _P, _L, _L, _L, _P, _L, _P, _P,
                                 _P, _P]),
    "b200moe_expert_down_scatter": (_I, [_I, _P, _I, _I, _P, _I, _P, _P, _L, _L, _P, _L, _P,
                                         _P, _I, _L, _P, _P, _L, _P]),
    "b200moe_decode_tiny": (_I, [_P, _I, _P, _L, _I, _I, _I, _I, _I, _P, _P, _I, _P, _I, _P, _P,
                                 _P, _P]),
    "b200moe_combine": (_I, [_P, _L, _P, _L, _I, _I, _I, _P, _I, _P]),
    "b200moe_ep_plan": (_I, [_P, _L, _I, _I, _P, _I, _P, _P, _P, _P]),
    "b200moe_ep_pack": (_I, [_P, _I, _P, _P, _L, _I, _I, _P, _I, _P, _P, _P, _P, _P, _P, _P]),
    "b200moe_ep_unpack_routes": (_I, [_P, _L, _I, _P, _P, _P, _P, _P, _P, _P]),
    "b200moe_ep_return_rows": (_I, [_P, _P, _L, _I, _I, _P, _P, _L, _P, _P]),
    "b200moe_pack_routes_device_bounds": (_I, [_P, _P, _L, _P, _I, _P, _I, _I, _P, _L, _P, _L,
                                               _P, _P, _P, _P, _P, _P, _P, _L, _P, _P, _P, _P,
                                               _S, _P]),
    "b200moe_nvl_buffer_bytes": (_L, [_I, _L, _I, _I, _I, _I, _P]),
    "b200moe_ipc_handle": (_I, [_P, _P, _P]),
    "b200moe_ipc_open": (_I, [_P, _L, _P]),
    "b200moe_ipc_close": (_I, [_P, _L]),
    "b200moe_nvl_histogram_send": (_I, [_P, _L, _I, _I, _I, _I, _P, _P, _P]),
    "b200moe_nvl_histogram_wait": (_I, [_I, _I, _I, _I, _P, _P, ctypes.c_double, _P, _P, _P,
                                        _P]),
    "b200moe_nvl_dispatch": (_I, [_P, _I, _P, _P, _L, _I, _I, _P, _I, _I, _P, _P, _P, _P, _P, _L,
                                  _I, _P, _P]),
    "b200moe_nvl_receive": (_I, [_I, _I, _P, _P, _L, _P, _P, _P, _P, _P, _P, _P]),
    "b200moe_nvl_return": (_I, [_P, _I, _P, _P, _P, _L, _L, _I, _I, _P, _P, _P]),
    "b200moe_nvl_wait_return": (_I, [_I, _I, _P, _P, _P]),
    "b200moe_nvl_return_signal": (_I, [_I, _I, _P, _P, _P]),
}
NVL_LAYOUT_WORDS = 10
NVL_ROUTE_CAP = 8  # layout word: route records per source region


class B200MoEError(RuntimeError):
    """A b200moe C-ABI call returned a non-zero status."""

    def __init__(self, function: str, code: int, message: str) -> None:
        super().__init__(f"{function} failed (code {code}): {message}")
        self.function = function
        self.code = code


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library with "
            "`python extend-nano-vllm_b200/build.py` (nvcc, sm_100a)"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


LIB = _load()


# Largest route count the packing call handles with one kernel (one route
# block: the scatter kernel builds its own histogram); above it, two.
PACK_SINGLE_LAUNCH_ROUTES = 1024
# Calls made through call(), by entry-point name, and the kernels they
# launched (launch accounting; the streaming and tcgen05 engines launch one
# kernel per projection, the tiny decode path two).
CALL_COUNTS: dict[str, int] = {}
LAUNCH_COUNTS: dict[str, int] = {}
_NO_KERNEL = ("b200moe_device_status", "b200moe_ipc_handle", "b200moe_ipc_open",
              "b200moe_ipc_close")


def _kernels_launched(name: str, args: tuple) -> int:
    if name in _NO_KERNEL:
        return 0
    if name in ("b200moe_pack_routes", "b200moe_pack_routes_static_scratch",
                "b200moe_pack_routes_shared"):
        routes = int(args[2])
        return 0 if routes == 0 else 1 if routes <= PACK_SINGLE_LAUNCH_ROUTES else 2
    if name == "b200moe_decode_tiny":
        return 2 if int(args[3]) > 0 else 0
    if name == "b200moe_pack_routes_device_bounds":
        return 1 if int(args[2]) <= PACK_SINGLE_LAUNCH_ROUTES else 2
    if name == "b200moe_nvl_receive":
        return 2
    return 1


def launches_since(snapshot: dict[str, int]) -> int:
    """Kernels launched by library calls made after ``snapshot`` (a copy of
    LAUNCH_COUNTS) was taken."""
    return sum(count - snapshot.get(name, 0) for name, count in LAUNCH_COUNTS.items())


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise on a non-zero status."""
    CALL_COUNTS[name] = CALL_COUNTS.get(name, 0) + 1
    LAUNCH_COUNTS[name] = LAUNCH_COUNTS.get(name, 0) + _kernels_launched(name, args)
    rc = getattr(LIB, name)(*args)
    if rc != OK:
        message = LIB.b200moe_last_error().decode(errors="replace")
        if rc == EINVAL:
            raise ValueError(f"{name}: {message}")
        if rc == EUNSUPPORTED:
            raise NotImplementedError(f"{name}: {message}")
        raise B200MoEError(name, rc, message)


def device_status(clear: bool = False) -> int:
    """Sticky device status word of the current device (synchronises)."""
    value = ctypes.c_int(0)
    call("b200moe_device_status", ctypes.byref(value), int(clear))
    return value.value
