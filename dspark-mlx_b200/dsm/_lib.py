"""ctypes bindings of ``libdsm.so`` (the C ABI declared in ``include/dsm.h``).

The library is loaded from this directory; there is no fallback: if it is missing or was
not built for this GPU, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_int64, c_size_t, c_void_p

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libdsm.so")

# status / enums (mirror include/dsm.h)
DSM_OK = 0
DT_F32, DT_BF16, DT_F16, DT_I32, DT_I64 = 0, 1, 2, 3, 4
ATTN_KERNEL_DEFAULT = 0  # dsm_set_attn_kernel's default: the tensor-core attention kernels
SCORE = {"softmax": 0, "sigmoid": 1, "sqrtsoftplus": 2}
WFMT_F16, WFMT_FP8_B128, WFMT_FP4_G32, WFMT_AFFINE8, WFMT_AFFINE4 = 0, 1, 2, 3, 4
ACT_SWIGLU_CLAMP, ACT_SILU_MUL_BF16 = 0, 1
STAGE_PITCH = 160
DEVICE_ERRORS = {0x10: "expert id out of range", 0x11: "token id out of range",
                 0x12: "pipeline wait ran out of its time budget",
                 0x13: "an expert-parallel peer did not signal in time",
                 0x14: "more expert-parallel rows than the exchange buffer holds"}

EXPORTED = (
    "dsm_abi_version", "dsm_status_string", "dsm_last_error_message", "dsm_device_error",
    "dsm_router_workspace_bytes", "dsm_router", "dsm_router_noalloc", "dsm_permute_workspace_bytes", "dsm_permute", "dsm_stage_bytes",
    "dsm_stage_rows_cap", "dsm_stage_rows", "dsm_packed_bytes", "dsm_pack_weights",
    "dsm_affine_quantize", "dsm_expert_gate_up", "dsm_expert_down", "dsm_combine",
    "dsm_moe_workspace_bytes", "dsm_moe_forward", "dsm_gather_rows", "dsm_stage_rows_count",
    "dsm_ep_buffer_bytes", "dsm_ep_rows_offset", "dsm_ep_results_offset", "dsm_ep_dispatch", "dsm_ep_receive", "dsm_ep_return",
    "dsm_ep_wait_results", "dsm_enable_peer_access", "dsm_ipc_get_handle", "dsm_ipc_open", "dsm_ipc_close",
    "dsm_set_expert_regime", "dsm_hc_pre_norm", "dsm_hc_post", "dsm_dense_mlp_workspace_bytes",
    "dsm_dense_mlp", "dsm_linear", "dsm_hc_head_norm", "dsm_markov_head", "dsm_draft_head_workspace_bytes",
    "dsm_draft_head", "dsm_rows_norm_rope", "dsm_q_head_norm_rope", "dsm_kv_window_write",
    "dsm_sparse_attn_scratch_bytes", "dsm_sparse_attn", "dsm_round_rows", "dsm_stage_rows_hilo",
    "dsm_qkv_norm_rope", "dsm_gqa_attn_workspace_bytes", "dsm_gqa_attn", "dsm_set_attn_kernel",
    "dsm_linear_splitk_workspace_bytes", "dsm_linear_splitk", "dsm_add_rms_norm",
    "dsm_grouped_linear", "dsm_grouped_linear_splitk",
)


class MoEDesc(ctypes.Structure):
    """``dsm_moe_desc`` (field order and types follow the C struct)."""

    _fields_ = [
        ("n_tokens", c_int64),
        ("dim", c_int), ("inter", c_int), ("n_experts", c_int), ("topk", c_int),
        ("score_func", c_int),
        ("route_scale", c_float), ("swiglu_limit", c_float),
        ("gate_weight", c_void_p), ("gate_bias", c_void_p), ("tid2eid", c_void_p),
        ("vocab", c_int64),
        ("wfmt", c_int), ("group_size", c_int),
        ("w1", c_void_p), ("w3", c_void_p), ("w2", c_void_p),
        ("round_gu", c_int), ("round_o", c_int),
        ("shared_wfmt", c_int), ("shared_group_size", c_int),
        ("s1", c_void_p), ("s3", c_void_p), ("s2", c_void_p),
        ("shared_inter", c_int), ("shared_round_gu", c_int), ("shared_round_o", c_int),
        ("act", c_int),
    ]


class EpDesc(ctypes.Structure):
    """``dsm_ep_desc`` (field order and types follow the C struct)."""

    _fields_ = [("world", c_int), ("rank", c_int), ("e_local", c_int), ("dim", c_int), ("x_dtype", c_int),
                ("capacity", c_int64)]


class HeadDesc(ctypes.Structure):
    """``dsm_head_desc`` (field order and types follow the C struct)."""

    _fields_ = [
        ("batch", c_int64),
        ("block", c_int), ("hc_mult", c_int), ("dim", c_int), ("vocab", c_int), ("rank", c_int),
        ("norm_eps", c_float), ("hc_eps", c_float),
        ("hc_fn", c_void_p), ("hc_scale", c_void_p), ("hc_base", c_void_p), ("norm_weight", c_void_p),
        ("head_wfmt", c_int), ("head_group_size", c_int),
        ("head_w", c_void_p),
        ("markov_dtype", c_int),
        ("markov_w1", c_void_p), ("markov_w2", c_void_p),
        ("conf_w", c_void_p),
        ("conf_bias", c_float),
    ]


class DsmError(RuntimeError):
    pass


_lib = None


def _declare(lib):
    V, I, I64, F, S = c_void_p, c_int, c_int64, c_float, c_size_t
    sig = {
        "dsm_abi_version": (I, []),
        "dsm_status_string": (ctypes.c_char_p, [I]),
        "dsm_last_error_message": (ctypes.c_char_p, []),
        "dsm_device_error": (I, [POINTER(c_int), I, V]),
        "dsm_router_workspace_bytes": (S, [I64, I, I]),
        "dsm_router": (I, [V, I, I64, I, V, I, V, V, I64, V, I, I64, I, I, F, V, V, V, V]),
        "dsm_router_noalloc": (I, [V, I, I64, I, V, I, V, V, I64, V, I, I64, I, I, F, V, V, V]),
        "dsm_permute_workspace_bytes": (S, [I64, I]),
        "dsm_permute": (I, [V, I64, I, V, V, V, V, V, S, V]),
        "dsm_stage_bytes": (S, [I64, I]),
        "dsm_stage_rows_cap": (I64, [I64]),
        "dsm_stage_rows": (I, [V, I, I64, I, V, I64, I, V, I64, V, V]),
        "dsm_packed_bytes": (S, [I, I, I, I, I]),
        "dsm_pack_weights": (I, [I, I, I, I, I, I, V, V, V, V, V, V]),
        "dsm_affine_quantize": (I, [V, I, I64, I, I, I, V, V, V, V]),
        "dsm_expert_gate_up": (I, [V, V, I64, I, V, I, I, I, V, V, I, I, F, I, V, F, I64, V]),
        "dsm_expert_down": (I, [V, F, I64, I, V, I, I, I, V, I, I, V, I, V, I64, V]),
        "dsm_gather_rows": (I, [V, I, I64, I, V, I64, I, V, V]),
        "dsm_stage_rows_count": (I, [V, I, I64, I, V, I64, I, V, I64, V, V, V]),
        "dsm_ep_buffer_bytes": (S, [POINTER(EpDesc)]),
        "dsm_ep_rows_offset": (I64, [POINTER(EpDesc), ctypes.c_uint32]),
        "dsm_ep_results_offset": (I64, [POINTER(EpDesc), ctypes.c_uint32]),
        "dsm_ep_dispatch": (I, [POINTER(EpDesc), V, I64, V, V, V, V, I, V, V, V, ctypes.c_uint32, V]),
        "dsm_ep_receive": (I, [POINTER(EpDesc), V, ctypes.c_uint32, V, V, V, V]),
        "dsm_ep_return": (I, [POINTER(EpDesc), V, V, V, V, ctypes.c_uint32, V]),
        "dsm_ep_wait_results": (I, [POINTER(EpDesc), V, ctypes.c_uint32, V]),
        "dsm_enable_peer_access": (I, [I]),
        "dsm_ipc_get_handle": (I, [V, V, POINTER(c_int64)]),
        "dsm_ipc_open": (I, [V, POINTER(ctypes.c_uint64)]),
        "dsm_ipc_close": (I, [ctypes.c_uint64]),
        "dsm_set_expert_regime": (I, [I]),
        "dsm_combine": (I, [V, V, V, I64, I, I, V, V, I, V]),
        "dsm_hc_pre_norm": (I, [V, I, I64, I, I, V, V, V, I, F, F, V, V, V, V, V]),
        "dsm_hc_post": (I, [V, V, I, I64, I, I, V, V, V, V]),
        "dsm_dense_mlp_workspace_bytes": (S, [I64, I, I]),
        "dsm_dense_mlp": (I, [V, I, I64, I, I, I, I, V, V, V, I, F, I, I, V, I, V, S, V]),
        "dsm_linear": (I, [V, V, I64, I, I, I, V, I, V, I, I64, V]),
        "dsm_hc_head_norm": (I, [V, I, I64, I, I, V, V, V, F, F, V, V, V, V, V, V]),
        "dsm_markov_head": (I, [V, I, I64, I, I, V, V, I, V, V, V]),
        "dsm_draft_head_workspace_bytes": (S, [POINTER(HeadDesc), I]),
        "dsm_draft_head": (I, [POINTER(HeadDesc), V, I, V, I, F, V, V, V, V, V, V, S, V]),
        "dsm_rows_norm_rope": (I, [V, V, I64, I, V, F, I, V, V, I, I, V, I, V]),
        "dsm_q_head_norm_rope": (I, [V, V, I64, I, I, F, I, V, V, I, I, V, I, V]),
        "dsm_kv_window_write": (I, [V, I, I, I, I, I, I, V, V]),
        "dsm_sparse_attn_scratch_bytes": (S, [I, I, I, I]),
        "dsm_sparse_attn": (I, [V, V, V, I, V, I, I, I, I, I, I, F, I, V, V, I, I, V, V, V]),
        "dsm_round_rows": (I, [V, V, I64, V, I, V]),
        "dsm_qkv_norm_rope": (I, [V, V, I64, I, I, I, V, V, F, V, V, I, I, I, V, V, V, I, I, I, V]),
        "dsm_gqa_attn_workspace_bytes": (S, [I, I, I, I, I, I]),
        "dsm_gqa_attn": (I, [V, V, V, I64, I64, I, V, V, I, I, I, I, I, I, F, V, V, S, V]),
        "dsm_set_attn_kernel": (I, [I]),
        "dsm_linear_splitk_workspace_bytes": (S, [I64, I]),
        "dsm_linear_splitk": (I, [V, V, I64, I, I, I, V, I, V, I, I64, V, S, V]),
        "dsm_add_rms_norm": (I, [V, V, I, I64, I, V, F, V, V, V]),
        "dsm_grouped_linear": (I, [V, V, I64, I, I, I, V, I, V, I, V, I, V, I64, V]),
        "dsm_grouped_linear_splitk": (I, [V, V, I64, I, I, I, V, I, V, I, V, I, V, I64, V, S, V]),
        "dsm_stage_rows_hilo": (I, [V, I64, I, V, I64, V, V]),
        "dsm_moe_workspace_bytes": (S, [POINTER(MoEDesc)]),
        "dsm_moe_forward": (I, [POINTER(MoEDesc), V, I, V, I, I64, V, V, V, V, S, V]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib():
    """The loaded library (raises if ``libdsm.so`` is missing: there is no CPU fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise DsmError(f"{LIB_PATH} is missing; build it with `python -m dsm.build`")
        handle = ctypes.CDLL(LIB_PATH)
        _declare(handle)
        if handle.dsm_abi_version() != 1:
            raise DsmError("libdsm ABI version mismatch")
        _lib = handle
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != DSM_OK:
        L = lib()
        msg = L.dsm_last_error_message().decode() or L.dsm_status_string(rc).decode()
        raise DsmError(f"{what}: {msg}" if what else msg)


def device_error(clear: bool = True, stream=None) -> int:
    """Read the device-side error word (synchronises the stream)."""
    code = c_int(0)
    check(lib().dsm_device_error(ctypes.byref(code), int(clear), stream_ptr(stream)), "dsm_device_error")
    return code.value


def raise_device_error(stream=None) -> None:
    code = device_error(True, stream)
    if code:
        raise DsmError(f"device error 0x{code:x}: {DEVICE_ERRORS.get(code, 'unknown')}")


def stream_ptr(stream=None) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)


def ptr(t):
    return None if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    return {torch.float32: DT_F32, torch.bfloat16: DT_BF16, torch.float16: DT_F16,
            torch.int32: DT_I32, torch.int64: DT_I64}[dt]
