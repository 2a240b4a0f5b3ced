"""ctypes binding of include/rmoe.h (librmoe.so, built in-tree by rusty_engine_b200.build).

There is no fallback: if the shared library is missing or fails to load, every entry point
raises.  The library is the product; this module only marshals pointers and sizes.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librmoe.so")

RMOE_OK, RMOE_ERR_INVALID, RMOE_ERR_UNSUPPORTED, RMOE_ERR_CUDA, RMOE_ERR_NCCL, RMOE_ERR_DEVICE, RMOE_ERR_OOM = range(7)
STATUS_NAMES = {0: "OK", 1: "INVALID", 2: "UNSUPPORTED", 3: "CUDA", 4: "NCCL", 5: "DEVICE", 6: "OOM"}

FLAG_HOST_IO = 1 << 0
FLAG_DETERMINISTIC = 1 << 1
FLAG_FORCE_SMALL = 1 << 2
FLAG_FORCE_LARGE = 1 << 3
FLAG_ROUTING_OUT = 1 << 4
FLAG_STAGE_TIMING = 1 << 5
FLAG_EXACT_ROUTER = 1 << 6


class RmoeError(RuntimeError):
    """A non-OK rmoe_status; ``status`` holds the code, the message is rmoe_last_error()."""

    def __init__(self, status: int, message: str):
        super().__init__(f"rmoe {STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


class Tensor(C.Structure):
    _fields_ = [("ggml_type", C.c_uint32), ("data", C.c_void_p), ("nbytes", C.c_uint64), ("dims", C.c_uint64 * 3)]


class LayerDesc(C.Structure):
    _fields_ = [
        ("hidden", C.c_uint32), ("inter", C.c_uint32), ("n_experts", C.c_uint32), ("top_k", C.c_uint32),
        ("gate", C.c_uint32), ("router_w", C.c_void_p),
        ("gate_exps", Tensor), ("up_exps", Tensor), ("down_exps", Tensor),
        ("has_shared", C.c_uint32),
        ("gate_shexp", Tensor), ("up_shexp", Tensor), ("down_shexp", Tensor),
        ("device", C.c_int32),
    ]


# Every symbol include/rmoe.h declares (the tests check the library exports all of them).
EXPORTS = [
    "rmoe_layer_create", "rmoe_layer_forward", "rmoe_layer_routing", "rmoe_layer_logits", "rmoe_layer_destroy",
    "rmoe_last_error", "rmoe_dequant", "rmoe_qmat_matmul", "rmoe_route", "rmoe_ep_unique_id",
    "rmoe_ep_layer_create", "rmoe_ep_layer_create_placed", "rmoe_build_info", "rmoe_layer_stage_ms", "rmoe_layer_forward_noalloc",
    "rmoe_route_grouped", "rmoe_qmat_create", "rmoe_qmat_forward", "rmoe_qmat_status", "rmoe_qmat_destroy",
    "rmoe_gguf_open", "rmoe_gguf_close", "rmoe_gguf_tensor", "rmoe_gguf_meta_uint", "rmoe_gguf_moe_layer_desc",
    "rmoe_layer_router_refined", "rmoe_noalloc_status", "rmoe_selftest_bounded_wait",
]

NOALLOC_SCRATCH_BYTES = 8 << 20  # RMOE_NOALLOC_SCRATCH_BYTES

_lib = None
_lock = threading.Lock()


def load():
    """Load librmoe.so (raises if it is absent: the product has no CPU fallback)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m rusty_engine_b200.build`")
        L = C.CDLL(LIB_PATH)
        vp, u32, u64, i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32
        L.rmoe_layer_create.argtypes = [C.POINTER(LayerDesc), C.POINTER(vp)]
        L.rmoe_layer_forward.argtypes = [vp, vp, u32, vp, vp, u32]
        L.rmoe_layer_forward_noalloc.argtypes = [vp, vp, u32, vp, vp]
        L.rmoe_layer_routing.argtypes = [vp, u32, vp, vp]
        L.rmoe_layer_logits.argtypes = [vp, u32, vp]
        L.rmoe_layer_stage_ms.argtypes = [vp, vp]
        L.rmoe_layer_router_refined.argtypes = [vp, vp]
        L.rmoe_noalloc_status.argtypes = [i32]
        L.rmoe_selftest_bounded_wait.argtypes = [i32, u32]
        L.rmoe_layer_destroy.argtypes = [vp]
        L.rmoe_layer_destroy.restype = None
        L.rmoe_last_error.restype = C.c_char_p
        L.rmoe_dequant.argtypes = [u32, vp, u64, vp, vp]
        L.rmoe_qmat_matmul.argtypes = [u32, vp, u64, u32, u32, vp, u32, vp, vp]
        L.rmoe_route.argtypes = [vp, u32, u32, u32, u32, vp, vp, vp]
        L.rmoe_qmat_create.argtypes = [u32, vp, u64, u32, u32, i32, C.POINTER(vp)]
        L.rmoe_qmat_forward.argtypes = [vp, vp, u32, vp, vp]
        L.rmoe_qmat_status.argtypes = [vp]
        L.rmoe_qmat_destroy.argtypes = [vp]
        L.rmoe_qmat_destroy.restype = None
        L.rmoe_route_grouped.argtypes = [vp, vp, u32, u32, u32, u32, u32, i32, i32, vp, vp, vp]
        L.rmoe_ep_unique_id.argtypes = [vp]
        L.rmoe_ep_layer_create.argtypes = [C.POINTER(LayerDesc), i32, i32, vp, C.POINTER(vp)]
        L.rmoe_ep_layer_create_placed.argtypes = [C.POINTER(LayerDesc), i32, i32, vp, vp, C.POINTER(vp)]
        L.rmoe_build_info.restype = C.c_char_p
        L.rmoe_gguf_open.argtypes = [C.c_char_p, C.POINTER(vp)]
        L.rmoe_gguf_close.argtypes = [vp]
        L.rmoe_gguf_close.restype = None
        L.rmoe_gguf_tensor.argtypes = [vp, C.c_char_p, C.POINTER(Tensor)]
        L.rmoe_gguf_meta_uint.argtypes = [vp, C.c_char_p, C.POINTER(u64)]
        L.rmoe_gguf_moe_layer_desc.argtypes = [vp, u32, C.POINTER(LayerDesc)]
        for name in EXPORTS:
            fn = getattr(L, name)
            if fn.restype is C.c_int or name in ("rmoe_layer_create",):
                fn.restype = C.c_int
        _lib = L
        return L


def check(status: int):
    if status != RMOE_OK:
        raise RmoeError(status, load().rmoe_last_error().decode(errors="replace"))
