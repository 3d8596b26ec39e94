"""ctypes binding of ``libb200moe.so`` (the C ABI in ``include/b200moe.h``).

Importing this module loads the library; a missing library is an ImportError
(there is no CPU implementation to fall back to). ``check`` turns a non-zero
status into ValueError (bad argument), NotImplementedError (unsupported
shape) or RuntimeError (CUDA failure), the reference's fail-fast convention
(moe_serving/efficient_kernels.py:1-4).
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_longlong, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200moe.so"

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3
STATUS_WAIT_TIMEOUT, STATUS_BAD_TILE, STATUS_BAD_INDEX, STATUS_PEER_TIMEOUT = 1, 2, 4, 8

ROUTER_QWEN3, ROUTER_GPT_OSS, ROUTER_NATIVE = 0, 1, 2
W_BF16, W_FP8, W_MXFP4 = 0, 1, 2
EPI_SWIGLU, EPI_CLAMP_SWIGLU, EPI_DOWN, EPI_CLAMP_SWIGLU_F32, EPI_DOWN_F32 = 0, 1, 2, 3, 4
ORDER_EXPERT, ORDER_RANK_SLOT, ORDER_SLOT_SUM = 0, 1, 2
PERMUTE_SCRATCH_BYTES = 1 << 20

EXPORTED = (
    "b200moe_last_error",
    "b200moe_version",
    "b200moe_device_status",
    "b200moe_router",
    "b200moe_route_record",
    "b200moe_act_quant_fp8",
    "b200moe_permute_workspace",
    "b200moe_permute",
    "b200moe_permute_noalloc",
    "b200moe_expert_gemm",
    "b200moe_w8a8_gemm",
    "b200moe_combine",
    "b200moe_combine_f32",
    "b200moe_append_shared_slot",
    "b200moe_gather_rows",
    "b200moe_gather_rows_range",
    "b200moe_a2a_recv_plan",
    "b200moe_gemm_args_size",
    "b200moe_p2p_buffer_bytes",
    "b200moe_p2p_alloc",
    "b200moe_p2p_free",
    "b200moe_p2p_export",
    "b200moe_p2p_import",
    "b200moe_p2p_close",
    "b200moe_combine_allreduce",
    "b200moe_layer_workspace",
    "b200moe_expert_layer",
    "b200moe_layer_args_size",
    "b200moe_peer_rows_bytes",
    "b200moe_a2a_counts",
    "b200moe_a2a_dispatch",
    "b200moe_a2a_return",
    "b200moe_ep_gather",
)


class GemmArgs(ctypes.Structure):
    """Mirror of ``b200moe_gemm_args``."""

    _fields_ = [
        ("offsets", c_void_p),
        ("expert_begin", c_int),
        ("n_experts", c_int),
        ("max_rows", c_int),
        ("token_tile", c_int),
        ("split_k", c_int),
        ("wfmt", c_int),
        ("planes", c_int),
        ("feat_pad", c_int),
        ("n_feat", c_int),
        ("k_pad", c_int),
        ("weight", c_void_p),
        ("sc_br", c_int),
        ("sc_bc", c_int),
        ("b_src", c_void_p),
        ("ldb", c_longlong),
        ("b_rows", c_int),
        ("k_valid", c_int),
        ("b_map", c_void_p),
        ("b_div", c_int),
        ("epilogue", c_int),
        ("bias", c_void_p),
        ("alpha", c_float),
        ("limit", c_float),
        ("row_weight", c_void_p),
        ("row_weight_bf16", c_int),
        ("row_src", c_void_p),
        ("out", c_void_p),
        ("ldo", c_longlong),
    ]


class LayerArgs(ctypes.Structure):
    """Mirror of ``b200moe_layer_args``."""

    _fields_ = [
        ("indices", c_void_p),
        ("weights", c_void_p),
        ("weights_bf16", c_int),
        ("T", c_int),
        ("K", c_int),
        ("E", c_int),
        ("expert_begin", c_int),
        ("hidden", c_void_p),
        ("ldh", c_longlong),
        ("H", c_int),
        ("I", c_int),
        ("wfmt", c_int),
        ("n_experts", c_int),
        ("w1", c_void_p),
        ("w2", c_void_p),
        ("b1", c_void_p),
        ("b2", c_void_p),
        ("sc_br", c_int),
        ("sc_bc", c_int),
        ("gated_epilogue", c_int),
        ("alpha", c_float),
        ("limit", c_float),
        ("out", c_void_p),
        ("ldo", c_longlong),
    ]


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing; build it with `python -m moe_serving_profile_b200.build`"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.b200moe_last_error.restype = c_char_p
    lib.b200moe_last_error.argtypes = []
    lib.b200moe_version.restype = c_char_p
    lib.b200moe_version.argtypes = []
    lib.b200moe_device_status.restype = c_int
    lib.b200moe_device_status.argtypes = [c_int, c_int, POINTER(c_int)]
    lib.b200moe_router.restype = c_int
    lib.b200moe_router.argtypes = [
        c_int, c_void_p, c_int, c_void_p, c_longlong, c_void_p, c_void_p, c_int, c_int, c_int,
        c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
    ]
    lib.b200moe_route_record.restype = c_int
    lib.b200moe_route_record.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_int, c_longlong,
                                         c_void_p, c_void_p]
    lib.b200moe_act_quant_fp8.restype = c_int
    lib.b200moe_act_quant_fp8.argtypes = [c_int, c_void_p, c_void_p, c_longlong, c_void_p, c_int, c_int,
                                          c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int]
    lib.b200moe_permute_workspace.restype = c_int
    lib.b200moe_permute_workspace.argtypes = [c_int, c_int, c_int, POINTER(c_size_t)]
    lib.b200moe_permute.restype = c_int
    lib.b200moe_permute.argtypes = [
        c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
        c_void_p, c_size_t,
    ]
    lib.b200moe_permute_noalloc.restype = c_int
    lib.b200moe_permute_noalloc.argtypes = [
        c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
    ]
    lib.b200moe_expert_gemm.restype = c_int
    lib.b200moe_expert_gemm.argtypes = [c_int, c_void_p, POINTER(GemmArgs)]
    lib.b200moe_w8a8_gemm.restype = c_int
    lib.b200moe_w8a8_gemm.argtypes = [c_int, c_void_p, POINTER(GemmArgs), c_void_p, c_void_p]
    lib.b200moe_gemm_args_size.restype = c_size_t
    lib.b200moe_gemm_args_size.argtypes = []
    if lib.b200moe_gemm_args_size() != ctypes.sizeof(GemmArgs):
        raise ImportError("b200moe_gemm_args layout differs between the library and _lib.GemmArgs")
    lib.b200moe_combine.restype = c_int
    lib.b200moe_combine.argtypes = [
        c_int, c_void_p, c_void_p, c_longlong, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
        c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_longlong,
    ]
    lib.b200moe_combine_f32.restype = c_int
    lib.b200moe_combine_f32.argtypes = [
        c_int, c_void_p, c_void_p, c_longlong, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
        c_void_p, c_int, c_void_p, c_longlong,
    ]
    lib.b200moe_append_shared_slot.restype = c_int
    lib.b200moe_append_shared_slot.argtypes = [
        c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_longlong, c_int, c_int, c_longlong, c_void_p,
        c_void_p,
    ]
    lib.b200moe_gather_rows.restype = c_int
    lib.b200moe_gather_rows.argtypes = [
        c_int, c_void_p, c_void_p, c_longlong, c_void_p, c_int, c_int, c_int, c_void_p,
        c_longlong,
    ]
    lib.b200moe_p2p_buffer_bytes.restype = c_size_t
    lib.b200moe_p2p_buffer_bytes.argtypes = [c_int, c_int, c_int]
    lib.b200moe_p2p_alloc.restype = c_int
    lib.b200moe_p2p_alloc.argtypes = [c_int, c_size_t, POINTER(c_void_p)]
    lib.b200moe_p2p_free.restype = c_int
    lib.b200moe_p2p_free.argtypes = [c_int, c_void_p]
    lib.b200moe_p2p_export.restype = c_int
    lib.b200moe_p2p_export.argtypes = [c_int, c_void_p, c_char_p]
    lib.b200moe_p2p_import.restype = c_int
    lib.b200moe_p2p_import.argtypes = [c_int, c_char_p, POINTER(c_void_p)]
    lib.b200moe_p2p_close.restype = c_int
    lib.b200moe_p2p_close.argtypes = [c_int, c_void_p]
    lib.b200moe_combine_allreduce.restype = c_int
    lib.b200moe_combine_allreduce.argtypes = [
        c_int, c_void_p, c_void_p, c_longlong, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
        c_int, c_int, c_void_p, c_int, c_int, c_int, POINTER(c_void_p), c_int, c_void_p,
        c_longlong, ctypes.c_ulonglong,
    ]
    lib.b200moe_gather_rows_range.restype = c_int
    lib.b200moe_gather_rows_range.argtypes = [
        c_int, c_void_p, c_void_p, c_longlong, c_void_p, c_int, c_int, c_int, c_void_p,
        c_longlong, c_void_p, c_int, c_int,
    ]
    lib.b200moe_layer_args_size.restype = c_size_t
    lib.b200moe_layer_args_size.argtypes = []
    if lib.b200moe_layer_args_size() != ctypes.sizeof(LayerArgs):
        raise ImportError("b200moe_layer_args layout differs between the library and _lib.LayerArgs")
    lib.b200moe_layer_workspace.restype = c_size_t
    lib.b200moe_layer_workspace.argtypes = [POINTER(LayerArgs)]
    lib.b200moe_expert_layer.restype = c_int
    lib.b200moe_expert_layer.argtypes = [c_int, c_void_p, POINTER(LayerArgs), c_void_p, c_size_t]
    lib.b200moe_peer_rows_bytes.restype = c_size_t
    lib.b200moe_peer_rows_bytes.argtypes = [c_int, c_longlong, c_longlong]
    lib.b200moe_a2a_counts.restype = c_int
    lib.b200moe_a2a_counts.argtypes = [
        c_int, c_void_p, POINTER(c_void_p), c_int, c_int, c_int, c_void_p, c_void_p, c_longlong,
        c_longlong, ctypes.c_ulonglong,
    ]
    lib.b200moe_a2a_dispatch.restype = c_int
    lib.b200moe_a2a_dispatch.argtypes = [
        c_int, c_void_p, POINTER(c_void_p), c_int, c_int, c_int, c_void_p, c_longlong, c_int,
        c_void_p, c_void_p, c_void_p, c_int, c_int, c_longlong, ctypes.c_ulonglong,
    ]
    lib.b200moe_a2a_return.restype = c_int
    lib.b200moe_a2a_return.argtypes = [
        c_int, c_void_p, POINTER(c_void_p), c_int, c_int, c_int, c_void_p, c_longlong, c_int,
        c_longlong, c_longlong, ctypes.c_ulonglong,
    ]
    lib.b200moe_ep_gather.restype = c_int
    lib.b200moe_ep_gather.argtypes = [
        c_int, c_void_p, POINTER(c_void_p), c_int, c_int, c_int, c_void_p, c_int, c_int, c_int,
        c_longlong, ctypes.c_ulonglong,
    ]
    lib.b200moe_a2a_recv_plan.restype = c_int
    lib.b200moe_a2a_recv_plan.argtypes = [
        c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
    ]
    return lib


lib = _load()


def check(rc: int, what: str) -> None:
    if rc == OK:
        return
    msg = f"{what}: {lib.b200moe_last_error().decode(errors='replace')}"
    if rc == ERR_INVALID:
        raise ValueError(msg)
    if rc == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def version() -> str:
    return lib.b200moe_version().decode()


def device_status(device: int, clear: bool = True) -> int:
    """Synchronise ``device`` and return (and clear) its kernel status bits."""
    out = c_int(0)
    check(lib.b200moe_device_status(device, int(clear), ctypes.byref(out)), "device_status")
    return out.value
