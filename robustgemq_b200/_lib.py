"""ctypes binding of ``libgemq_b200.so`` (the C ABI in ``include/gemq_b200.h``).

The product path has no fallback: when the library is missing or fails to load,
every call raises. ``load()`` builds it in-tree first if the sources are newer.
"""

from __future__ import annotations

import ctypes
import functools
import inspect
import threading
from pathlib import Path
from typing import Optional

import torch

LIB_PATH = Path(__file__).resolve().parent / "libgemq_b200.so"

GEMQ_OK = 0
GEMQ_ERR_INVALID_ARGUMENT = 1
GEMQ_ERR_UNSUPPORTED = 2
GEMQ_ERR_CUDA = 3
GEMQ_ERR_WORKSPACE = 4

GEMQ_ROUTER_FP16 = 0
GEMQ_ROUTER_FP32 = 1

FWD_ONE_TOKEN = 1
FWD_GIVEN_ROUTING = 2
FWD_GIVEN_LOGITS = 4
FWD_FP16_SOFTMAX = 8
FWD_FP32_COMBINE = 16
FWD_FORCE_SIMT = 32
FWD_RESIDUAL = 64
FWD_TIME_STAGES = 128
FWD_SMEM_DEQUANT = 256
FWD_PERMUTED_ROWS = 512
FWD_NO_CHAIN = 1024
FWD_TEST_WAIT_EXPIRY = 2048
ROUTE_WORKSPACE_BYTES = 1024
STAGES = ("route", "dispatch", "up", "down", "shared", "combine")

# every symbol include/gemq_b200.h declares
EXPORTED = [
    "gemq_last_error_string", "gemq_version", "gemq_get_device_error",
    "gemq_pack_weights_over_cols", "gemq_unpack_over_cols", "gemq_dequant_expert",
    "gemq_group_gemm_workspace_size", "gemq_dequant_group_gemm", "gemq_dequant_group_gemm_noalloc",
    "gemq_dequant_gemm",
    "gemq_gemv_workspace_size", "gemq_dequant_gemv", "gemq_fused_up_proj", "gemq_fused_down_proj",
    "gemq_layer_create", "gemq_layer_destroy", "gemq_moe_workspace_size", "gemq_moe_route",
    "gemq_moe_forward", "gemq_layer_stage_times", "gemq_route", "gemq_moe_combine",
    "gemq_dispatch_workspace_size", "gemq_moe_dispatch", "gemq_moe_experts_workspace_size", "gemq_moe_experts",
    "gemq_moe_experts_row_order", "gemq_layer_dequant_forms", "gemq_rms_norm",
    "gemq_qk_norm_rope", "gemq_decode_attention", "gemq_layer_set_routing", "gemq_route_ex",
]


class GemqError(RuntimeError):
    """A non-zero status from the C ABI (the reference raises AssertionError /
    ValueError for the argument errors; those map to ``GemqArgumentError``)."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"gemq status {status}: {msg}")
        self.status = status


class GemqArgumentError(GemqError, ValueError):
    pass


class ProjT(ctypes.Structure):
    _fields_ = [
        ("wq", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("zeros", ctypes.c_void_p),
        ("nbits", ctypes.c_void_p), ("wq_strides", ctypes.c_void_p), ("zs_strides", ctypes.c_void_p),
        ("wq_rows", ctypes.c_int64), ("num_experts", ctypes.c_int32), ("k", ctypes.c_int32),
        ("n", ctypes.c_int32), ("group_size", ctypes.c_int32),
    ]


class LayerDescT(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("num_experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32), ("group_size", ctypes.c_int32), ("norm_topk_prob", ctypes.c_int32),
        ("router", ctypes.c_int32), ("gate_weight", ctypes.c_void_p),
        ("w1", ProjT), ("w3", ProjT), ("w2", ProjT),
        ("has_shared", ctypes.c_int32),
        ("shared_w1", ProjT), ("shared_w3", ProjT), ("shared_w2", ProjT),
    ]


class RoutingT(ctypes.Structure):
    """gemq_routing_t: renormalisation, group-limited greedy and the routing scale."""

    _fields_ = [
        ("norm_topk_prob", ctypes.c_int32), ("n_group", ctypes.c_int32), ("topk_group", ctypes.c_int32),
        ("scale", ctypes.c_float),
    ]


_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


def _declare(lib: ctypes.CDLL) -> None:
    vp, i32, i64, sz, u32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_uint32
    P = ctypes.POINTER
    sig = {
        "gemq_last_error_string": (ctypes.c_char_p, []),
        "gemq_version": (ctypes.c_int, []),
        "gemq_get_device_error": (ctypes.c_int, [P(u32)]),
        "gemq_pack_weights_over_cols": (ctypes.c_int, [vp, i64, i64, i32, vp, vp]),
        "gemq_unpack_over_cols": (ctypes.c_int, [vp, i64, i64, i64, i32, vp, vp]),
        "gemq_dequant_expert": (ctypes.c_int, [P(ProjT), i32, vp, vp]),
        "gemq_group_gemm_workspace_size": (sz, [i32]),
        "gemq_dequant_group_gemm": (ctypes.c_int, [P(ProjT), vp, i64, vp, i32, vp, vp, sz, vp]),
        "gemq_dequant_group_gemm_noalloc": (ctypes.c_int, [P(ProjT), vp, i64, vp, i32, vp, vp]),
        "gemq_dequant_gemm": (ctypes.c_int, [P(ProjT), vp, i64, vp, vp, sz, vp]),
        "gemq_gemv_workspace_size": (sz, [P(ProjT), i32]),
        "gemq_dequant_gemv": (ctypes.c_int, [P(ProjT), vp, vp, vp, sz, vp]),
        "gemq_fused_up_proj": (ctypes.c_int, [P(ProjT), P(ProjT), vp, vp, i32, vp, vp, vp, sz, vp]),
        "gemq_fused_down_proj": (ctypes.c_int, [P(ProjT), vp, vp, vp, i32, vp, vp, sz, vp]),
        "gemq_layer_create": (ctypes.c_int, [P(LayerDescT), P(vp)]),
        "gemq_layer_destroy": (ctypes.c_int, [vp]),
        "gemq_moe_workspace_size": (sz, [vp, i64, u32]),
        "gemq_moe_route": (ctypes.c_int, [vp, vp, i64, vp, vp, vp, u32, vp, sz, vp]),
        "gemq_moe_forward": (ctypes.c_int, [vp, vp, i64, vp, vp, vp, vp, u32, vp, sz, vp]),
        "gemq_layer_stage_times": (ctypes.c_int, [vp, P(ctypes.c_float)]),
        "gemq_layer_dequant_forms": (ctypes.c_int, [vp, P(ctypes.c_int32)]),
        "gemq_rms_norm": (ctypes.c_int, [vp, vp, i64, i32, ctypes.c_float, vp, vp]),
        "gemq_qk_norm_rope": (ctypes.c_int, [vp, i64, i64, i32, i32, vp, vp, ctypes.c_float, vp, vp, vp, vp,
                                             vp, vp, i32, vp, vp]),
        "gemq_decode_attention": (ctypes.c_int, [vp, vp, vp, i32, i32, i32, vp, ctypes.c_float, vp, vp]),
        "gemq_route": (ctypes.c_int, [vp, i64, i32, vp, i32, i32, i32, i32, u32, vp, vp, vp, vp, sz, vp]),
        "gemq_route_ex": (ctypes.c_int, [vp, i64, i32, vp, i32, i32, i32, P(RoutingT), u32, vp, vp, vp, vp, sz,
                                         vp]),
        "gemq_layer_set_routing": (ctypes.c_int, [vp, P(RoutingT)]),
        "gemq_moe_combine": (ctypes.c_int, [vp, vp, vp, i64, i32, i32, u32, vp, vp, vp]),
        "gemq_dispatch_workspace_size": (sz, [i64, i32, i32]),
        "gemq_moe_dispatch": (ctypes.c_int, [vp, vp, vp, i64, i32, i32, i32, vp, vp, vp, vp, vp, vp, sz, vp]),
        "gemq_moe_experts_row_order": (ctypes.c_int, [vp]),
        "gemq_moe_experts_workspace_size": (sz, [vp, i64, i32]),
        "gemq_moe_experts": (ctypes.c_int, [vp, vp, i64, vp, i32, vp, vp, i32, u32, vp, sz, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def load(build_if_stale: bool = True) -> ctypes.CDLL:
    """Load (building first if needed) the in-tree library; raises if impossible."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if build_if_stale:
            from . import build as _build
            try:
                _build.build()
            except Exception as exc:  # no nvcc on this machine: fall through to a prebuilt .so
                if not LIB_PATH.exists():
                    raise RuntimeError(f"libgemq_b200.so is missing and could not be built: {exc}") from exc
        if not LIB_PATH.exists():
            raise RuntimeError(f"libgemq_b200.so not found at {LIB_PATH}")
        lib = ctypes.CDLL(str(LIB_PATH))
        _declare(lib)
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != GEMQ_OK:
        msg = load().gemq_last_error_string().decode(errors="replace")
        if status == GEMQ_ERR_INVALID_ARGUMENT:
            raise GemqArgumentError(status, msg)
        raise GemqError(status, msg)


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def off_current_device(t: torch.Tensor) -> bool:
    """True when ``t`` is a CUDA tensor on a device other than the current one.

    The library launches on the current CUDA device, with the stream of the
    tensors' device. A model spread over several GPUs in one process (layers placed
    with a device map) moves each layer's inputs to that layer's GPU but does not
    make it the current device, so callers switch devices when this is true."""
    return t.is_cuda and t.device.index != torch.cuda.current_device()


def on_input_device(fn):
    """Decorator: run ``fn`` with the device of its first parameter (a tensor) current."""
    first = next(iter(inspect.signature(fn).parameters))

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        t = args[0] if args else kwargs.get(first)
        if isinstance(t, torch.Tensor) and off_current_device(t):
            with torch.cuda.device(t.device):
                return fn(*args, **kwargs)
        return fn(*args, **kwargs)

    return wrapper


def device_error() -> int:
    """Synchronises and returns (and clears) the library's device error word."""
    code = ctypes.c_uint32(0)
    check(load().gemq_get_device_error(ctypes.byref(code)))
    return int(code.value)
