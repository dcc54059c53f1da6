"""ctypes binding of libmegamoe.so (the C ABI declared in include/megamoe.h).

The shared library is built in-tree (megamoe/_build.py) next to this file. There
is no fallback: importing the binding without the library, or calling a kernel
without a CUDA device, raises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int32, c_int64, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmegamoe.so")

MM_OK = 0
MM_ERR_INVALID = 1
MM_ERR_UNSUPPORTED = 2
MM_ERR_CUDA = 3
MM_ERR_DEVICE_TIMEOUT = 4
MM_ERR_DEVICE = 5
MM_IPC_HANDLE_BYTES = 64

MM_SCORE_SIGMOID = 0
MM_SCORE_SOFTMAX = 1
MM_SCORE_SQRTSOFTPLUS = 2
MM_SCORE_SQRTSOFTPLUS_DSV41 = 3
SCORES = {"sigmoid": MM_SCORE_SIGMOID, "softmax": MM_SCORE_SOFTMAX, "sqrtsoftplus": MM_SCORE_SQRTSOFTPLUS,
          "sqrtsoftplus_dsv41": MM_SCORE_SQRTSOFTPLUS_DSV41}

MM_RENORM_NONE = 0
MM_RENORM_SUM = 1
MM_RENORM_SCALED_BF16 = 2
# renormalize= of the Python API: a bool (sum rule or none) or one of these names
RENORMS = {"none": MM_RENORM_NONE, "sum": MM_RENORM_SUM, "scaled_bf16": MM_RENORM_SCALED_BF16}

MM_WEIGHT_MXFP4 = 0
MM_WEIGHT_NVFP4 = 1

MM_SCRATCH_X_CODES = 0
MM_SCRATCH_X_SCALES = 1
MM_SCRATCH_H_CODES = 2
MM_SCRATCH_H_SCALES = 3


def renorm_code(renormalize) -> int:
    """The C routing weight rule of a Python ``renormalize`` argument."""
    if isinstance(renormalize, str):
        if renormalize not in RENORMS:
            raise ValueError(f"renormalize {renormalize!r}: True, False or one of {sorted(RENORMS)}")
        return RENORMS[renormalize]
    return MM_RENORM_SUM if renormalize else MM_RENORM_NONE


class MMExpertWeights(ctypes.Structure):
    _fields_ = [("w13", c_void_p), ("w13_scale", c_void_p), ("w2", c_void_p), ("w2_scale", c_void_p),
                ("w13_scale_2", c_void_p), ("w2_scale_2", c_void_p)]


class MMLayerDesc(ctypes.Structure):
    _fields_ = [
        ("hidden", c_int32),
        ("intermediate", c_int32),
        ("experts", c_int32),
        ("router_experts", c_int32),
        ("expert_offset", c_int32),
        ("top_k", c_int32),
        ("max_tokens", c_int32),
        ("weight_format", c_int32),
        ("act_terms", c_int32),
        ("device", c_int32),
        ("routed", MMExpertWeights),
        ("shared", MMExpertWeights),
        ("clamp", c_void_p),
        ("shared_clamp", c_void_p),
        ("input_scale", c_float * 2),
    ]


class MMGateArgs(ctypes.Structure):
    _fields_ = [
        ("logits", c_void_p),
        ("bias", c_void_p),
        ("num_valid", c_void_p),
        ("score_func", c_int32),
        ("renormalize", c_int32),
        ("routed_scaling", c_float),
        ("renorm_eps", c_float),
        ("weights", c_void_p),
        ("ids", c_void_p),
        ("bias_alt", c_void_p),
        ("input_ids", c_void_p),
        ("input_ids64", c_int32),
        ("alt_token_id", c_int64),
    ]


class MMLayerInfo(ctypes.Structure):
    _fields_ = [
        ("hidden", c_int32),
        ("intermediate", c_int32),
        ("experts", c_int32),
        ("router_experts", c_int32),
        ("expert_offset", c_int32),
        ("top_k", c_int32),
        ("max_tokens", c_int32),
        ("has_shared", c_int32),
        ("rows_capacity", c_int64),
        ("shared_row_base", c_int64),
        ("route_words", c_int64),
        ("weight_bytes", c_int64),
        ("act_terms", c_int32),
        ("h_row_bytes", c_int32),
        ("h_scale_row_bytes", c_int64),
    ]


class MMForwardArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p),
        ("router_w", c_void_p),
        ("logits", c_void_p),
        ("logits_out", c_void_p),
        ("bias", c_void_p),
        ("num_valid", c_void_p),
        ("score_func", c_int32),
        ("renormalize", c_int32),
        ("routed_scaling", c_float),
        ("renorm_eps", c_float),
        ("tokens", c_int32),
        ("weights", c_void_p),
        ("ids", c_void_p),
        ("permuted", c_void_p),
        ("record", c_void_p),
        ("rows", c_void_p),
        ("out", c_void_p),
        ("partial", c_void_p),
        ("comm", c_void_p),
        ("bias_alt", c_void_p),
        ("input_ids", c_void_p),
        ("input_ids64", c_int32),
        ("alt_token_id", c_int64),
        ("residual", c_void_p),
        ("gamma", c_void_p),
        ("norm_eps", c_float),
        ("residual_out", c_void_p),
    ]


class MMStackLayer(ctypes.Structure):
    _fields_ = [("layer", c_void_p), ("args", MMForwardArgs)]


# name -> (restype, argtypes); every extern "C" symbol of include/megamoe.h
SIGNATURES = {
    "mm_last_error": (ctypes.c_char_p, []),
    "mm_version": (c_int32, []),
    "mm_router_gemv": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "mm_gate_topk": (c_int32, [POINTER(MMGateArgs), c_int32, c_int32, c_int32, c_void_p]),
    "mm_route_words": (c_int64, [c_int32, c_int32, c_int32]),
    "mm_route": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p]),
    "mm_gate_route_noalloc": (
        c_int32,
        [POINTER(MMGateArgs), c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p],
    ),
    "mm_finalize": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p],
    ),
    "mm_finalize_partial": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p]),
    "mm_layer_create": (c_int32, [POINTER(MMLayerDesc), POINTER(c_void_p)]),
    "mm_layer_destroy": (c_int32, [c_void_p]),
    "mm_layer_get_info": (c_int32, [c_void_p, POINTER(MMLayerInfo)]),
    "mm_layer_experts": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "mm_layer_gate_experts": (
        c_int32,
        [c_void_p, c_void_p, POINTER(MMGateArgs), c_int32, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "mm_layer_experts_mxfp8": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "mm_layer_gate_experts_mxfp8": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, POINTER(MMGateArgs), c_int32, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "mm_layer_scratch_bytes": (c_int64, [c_void_p, c_int32]),
    "mm_layer_read_scratch": (c_int32, [c_void_p, c_int32, c_void_p, c_int64, c_void_p]),
    "mm_layer_rerun_experts": (c_int32, [c_void_p, c_int32, c_void_p, c_void_p, c_void_p]),
    "mm_layer_rearm_experts": (c_int32, [c_void_p, c_void_p]),
    "mm_layer_block_downs": (c_int32, [c_void_p, c_void_p]),
    "mm_layer_set_wait_budget": (c_int32, [c_void_p, c_int64]),
    "mm_layer_forward": (c_int32, [c_void_p, POINTER(MMForwardArgs), c_void_p]),
    "mm_layer_check": (c_int32, [c_void_p]),
    "mm_stack_forward": (c_int32, [POINTER(MMStackLayer), c_int32, c_void_p]),
    "mm_comm_create": (c_int32, [c_int32, c_int32, c_int32, c_int32, c_int32, POINTER(c_void_p)]),
    "mm_comm_handle": (c_int32, [c_void_p, c_void_p]),
    "mm_comm_open": (c_int32, [c_void_p, c_void_p]),
    "mm_comm_open_local": (c_int32, [c_void_p, POINTER(c_void_p)]),
    "mm_comm_destroy": (c_int32, [c_void_p]),
    "mm_comm_check": (c_int32, [c_void_p]),
    "mm_comm_set_wait_budget": (c_int32, [c_void_p, c_int64]),
    "mm_finalize_allreduce_norm": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
         c_int32, c_int32, c_int32, c_void_p],
    ),
    "mm_finalize_allreduce": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p],
    ),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python __graft_entry__.py build` "
                "(or megamoe._build.build())"
            )
        handle = ctypes.CDLL(LIB_PATH)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


class DeviceTimeoutError(RuntimeError):
    """A bounded device wait gave up (MM_ERR_DEVICE_TIMEOUT): a producer, a peer
    or a mailbox never arrived within the wait budget."""


def check(rc: int, what: str) -> None:
    """Map a status code to the reference's exception types (ValueError for
    shape/argument violations, RuntimeError for device/driver failures;
    DeviceTimeoutError, a RuntimeError, for a bounded wait that gave up)."""
    if rc == MM_OK:
        return
    msg = lib().mm_last_error().decode(errors="replace")
    if rc in (MM_ERR_INVALID, MM_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    if rc == MM_ERR_DEVICE_TIMEOUT:
        raise DeviceTimeoutError(f"{what}: {msg} (status {rc})")
    raise RuntimeError(f"{what}: {msg} (status {rc})")
