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
    "b200moe_pack_scratch_bytes": (_S, [_L, _I]),
    "b200moe_pack_row_capacity": (_L, [_L, _I]),
    "b200moe_pack_max_mtiles": (_L, [_L, _I]),
    "b200moe_pack_routes": (_I, [_P, _P, _L, _I, _P, _I, _I, _P, _L, _L, _P, _P, _P, _P, _P,
                                 _P, _P, _L, _P, _P, _P, _P, _S, _P]),
    "b200moe_pack_static_scratch_capacity": (_S, []),
    "b200moe_pack_routes_static_scratch": (_I, [_P, _P, _L, _I, _P, _I, _I, _P, _L, _L, _P, _P,
                                                _P, _P, _P, _P, _P, _L, _P, _P, _P]),
    "b200moe_expert_histogram": (_I, [_P, _L, _I, _P, _P]),
    "b200moe_gather_rows": (_I, [_P, _L, _I, _P, _P, _I, _L, _L, _P, _P, _P]),
    "b200moe_expert_gate_up": (_I, [_I, _P, _L, _P, _I, _I, _P, _I, _P, _P, _I, _L, _L, _P,
                                    _L, _P, _P, _P, _P]),
    "b200moe_expert_down": (_I, [_I, _P, _I, _I, _P, _I, _P, _P, _L, _L, _L, _P, _L, _P, _P,
                                 _P, _P]),
    "b200moe_decode_tiny": (_I, [_P, _I, _P, _L, _I, _I, _I, _I, _I, _P, _P, _I, _P, _I, _P, _P,
                                 _P, _P]),
    "b200moe_combine": (_I, [_P, _L, _P, _L, _I, _I, _I, _P, _I, _P]),
    "b200moe_ep_plan": (_I, [_P, _L, _I, _I, _P, _I, _P, _P, _P, _P]),
    "b200moe_ep_pack": (_I, [_P, _I, _P, _P, _L, _I, _I, _P, _I, _P, _P, _P, _P, _P, _P, _P]),
    "b200moe_ep_unpack_routes": (_I, [_P, _L, _I, _P, _P, _P, _P, _P, _P, _P]),
    "b200moe_ep_return_rows": (_I, [_P, _P, _L, _I, _I, _P, _P, _L, _P, _P]),
}


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


# Kernels each entry point launches (for launch accounting; the streaming
# and tcgen05 engines both launch one kernel per projection).
KERNELS_PER_CALL = {"b200moe_pack_routes": 2, "b200moe_pack_routes_static_scratch": 2,
                    "b200moe_decode_tiny": 2}
# Calls made through call(), by entry-point name (launch accounting).
CALL_COUNTS: dict[str, int] = {}


def launches_since(snapshot: dict[str, int]) -> int:
    """Kernels launched by library calls made after ``snapshot`` was taken."""
    total = 0
    for name, count in CALL_COUNTS.items():
        if name.startswith("b200moe_device_status"):
            continue
        total += (count - snapshot.get(name, 0)) * KERNELS_PER_CALL.get(name, 1)
    return total


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise on a non-zero status."""
    CALL_COUNTS[name] = CALL_COUNTS.get(name, 0) + 1
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
