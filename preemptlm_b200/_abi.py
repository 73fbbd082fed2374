"""ctypes binding of libsg_b200.so (the C-ABI declared in include/sg_abi.h).

Device buffers are passed as ``tensor.data_ptr()`` and the stream as
``torch.cuda.current_stream().cuda_stream``.  Every call checks the returned
status and raises ``SlottedGLUError`` on failure.  There is no fallback: if the
shared library is missing the import of the calling module fails loudly.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "lib" / "libsg_b200.so"

SG_OK = 0
SG_ERR_INVALID_ARG = -1
SG_ERR_SHAPE = -2
SG_ERR_FORMAT = -3
SG_ERR_CUDA = -4
SG_ERR_CAPACITY = -5
SG_ERR_TIMEOUT = -6

SG_IN_DISPATCH_ORDER = 1
SG_OUT_DISPATCH_ORDER = 2

# Every symbol include/sg_abi.h declares (checked by the CPU tests).
EXPORTED_SYMBOLS = (
    "sg_status_string", "sg_version", "sg_built_arch", "sg_router_logits", "sg_route_topk",
    "sg_dispatch", "sg_route_dispatch", "sg_host_device_ptr", "sg_glu_forward", "sg_glu_forward_noalloc", "sg_glu_forward_scratch_bytes", "sg_glu_use_permute",
    "sg_permute_rows", "sg_permute_pairs", "sg_glu_gate_up", "sg_glu_gate_up_work_bytes", "sg_glu_gate_up_work", "sg_quantize_pieces",
    "sg_glu_down", "sg_glu_down_work_bytes", "sg_glu_down_work",
    "sg_dense_glu", "sg_combine", "sg_refill_h2d",
    "sg_expert_bytes", "sg_set_glu_path", "sg_set_glu_tile", "sg_device_status",
    "sg_ep_region_bytes", "sg_ep_layout", "sg_ep_alloc", "sg_ep_free", "sg_ep_ipc_handle", "sg_ep_ipc_open",
    "sg_ep_ipc_close", "sg_ep_send", "sg_ep_wait_inbox", "sg_ep_send_back", "sg_ep_wait_back",
    "sg_ep_set_wait_limit",
)


class SlottedGLUError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {status_string(status)} (status {status})")


class sg_route_trace(ctypes.Structure):
    _fields_ = [("ids", ctypes.c_void_p), ("scores", ctypes.c_void_p), ("logits", ctypes.c_void_p)]


class sg_arena(ctypes.Structure):
    _fields_ = [
        ("num_slots", ctypes.c_int32), ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32),
        ("bits", ctypes.c_int32), ("group_size", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("gate_w", ctypes.c_void_p), ("gate_s", ctypes.c_void_p), ("gate_b", ctypes.c_void_p),
        ("up_w", ctypes.c_void_p), ("up_s", ctypes.c_void_p), ("up_b", ctypes.c_void_p),
        ("down_w", ctypes.c_void_p), ("down_s", ctypes.c_void_p), ("down_b", ctypes.c_void_p),
    ]


_lib = None


def lib_path() -> Path:
    return Path(os.environ.get("SG_B200_LIB", _LIB_PATH))


def load() -> ctypes.CDLL:
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build the CUDA extension first "
            "(python -m preemptlm_b200.build); there is no CPU fallback"
        )
    lib = ctypes.CDLL(str(path))
    P, I32, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    A = ctypes.POINTER(sg_arena)
    sigs = {
        "sg_status_string": (ctypes.c_char_p, [I32]),
        "sg_version": (I32, []),
        "sg_built_arch": (I32, []),
        "sg_router_logits": (I32, [P, P, P, I32, I32, I32, P]),
        "sg_route_topk": (I32, [P, I32, I32, I32, I32, P, P, P]),
        "sg_dispatch": (I32, [P, I32, I32, P, P, P, P, P, P, P, P, I32, P]),
        "sg_route_dispatch": (I32, [P, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P, P, I32, P, P, P]),
        "sg_host_device_ptr": (I32, [P, P]),
        "sg_glu_forward": (I32, [A, P, I32, I32, P, P, P, P, I32, P, P, P, P]),
        "sg_glu_forward_noalloc": (I32, [A, P, I32, I32, P, P, P, P, I32, P, P]),
        "sg_glu_forward_scratch_bytes": (ctypes.c_longlong, [A, I32, I32, I32]),
        "sg_glu_use_permute": (I32, [A, I32, I32]),
        "sg_glu_gate_up_work_bytes": (ctypes.c_longlong, [A, I32, I32, I32, I32]),
        "sg_glu_gate_up_work": (I32, [A, P, I32, I32, P, P, P, P, I32, P, I32, P, ctypes.c_longlong, P]),
        "sg_quantize_pieces": (I32, [P, I32, I32, I32, P, P, P]),
        "sg_glu_down_work_bytes": (ctypes.c_longlong, [A, I32, I32]),
        "sg_glu_down_work": (I32, [A, P, I32, P, P, P, P, I32, P, I32, P, ctypes.c_longlong, P]),
        "sg_permute_rows": (I32, [P, P, I32, I32, I32, P, P]),
        "sg_permute_pairs": (I32, [P, P, I32, P, P, I32, I32, P, P]),
        "sg_glu_gate_up": (I32, [A, P, I32, I32, P, P, P, P, I32, P, I32, P]),
        "sg_glu_down": (I32, [A, P, I32, P, P, P, P, I32, P, I32, P]),
        "sg_dense_glu": (I32, [A, I32, P, I32, P, P, P]),
        "sg_set_glu_path": (I32, [I32]),
        "sg_set_glu_tile": (I32, [I32]),
        "sg_device_status": (I32, [I32]),
        "sg_combine": (I32, [P, P, I32, I32, I32, P, P, P, P]),
        "sg_refill_h2d": (I32, [P, SZ, A, I32, P]),
        "sg_expert_bytes": (SZ, [A]),
        "sg_ep_region_bytes": (ctypes.c_longlong, [I32, I32, I32]),
        "sg_ep_layout": (I32, [I32, I32, I32, P]),
        "sg_ep_alloc": (I32, [ctypes.c_longlong, P]),
        "sg_ep_free": (I32, [P]),
        "sg_ep_ipc_handle": (I32, [P, P]),
        "sg_ep_ipc_open": (I32, [P, P]),
        "sg_ep_ipc_close": (I32, [P]),
        "sg_ep_send": (I32, [P, I32, I32, I32, I32, P, P, I32, I32, I32, P, P]),
        "sg_ep_wait_inbox": (I32, [P, I32, I32, I32, P]),
        "sg_ep_send_back": (I32, [P, I32, I32, I32, I32, P, P]),
        "sg_ep_wait_back": (I32, [P, I32, I32, I32, P, I32, I32, I32, P]),
        "sg_ep_set_wait_limit": (I32, [ctypes.c_longlong]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def status_string(status: int) -> str:
    try:
        return load().sg_status_string(status).decode()
    except ImportError:
        return "libsg_b200.so not loaded"


def check(status: int, where: str) -> None:
    if status != SG_OK:
        raise SlottedGLUError(status, where)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
