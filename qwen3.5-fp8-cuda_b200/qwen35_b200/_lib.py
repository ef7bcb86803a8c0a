"""ctypes binding of the two sm_100a shared libraries.

Mirrors the reference loader (main.py:89-240): the libraries are opened with
``ctypes.CDLL`` from ``QWEN_FUSED_DLL`` / ``QWEN_FP8_DLL`` when set (the same
environment variables the reference honours), otherwise from the in-tree build
directory ``qwen35_b200/lib``.  The reference-named symbols get the reference's
``argtypes``; the new symbols return an ``int`` status.

There is no fallback: if a library is missing, ``fused()`` / ``fp8()`` raise.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(_HERE, "lib")
FUSED_NAME = "libqwen_fused.so"
FP8_NAME = "libqwen_fp8.so"

P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float

# Reference-named exports: argtypes exactly as main.py:108-240.
REFERENCE_FUSED_ARGTYPES = {
    "launch_gemv_v4_extern": [P, P, P, P, I, I, I, P],
    "launch_gemv_v3_extern": [P, P, P, P, I, I, I, P],
    "launch_linear_in_proj4": [P, P, P, P, I, I, P, P, P, I, I, P, P, P, I, I, P, P, P, I, I, I, P],
    "launch_fused_qkv": [P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, P],
    "launch_fused_gate_up": [P, P, P, P, P, P, P, I, I, I, I, I, I, P],
    "launch_rmsnorm_ip": [P, P, I, I, F, P],
    "launch_rmsnorm_out": [P, P, P, I, I, F, P],
    "launch_fused_attn_v2": [P, P, P, P, I, I, I, I, I, P],
    "launch_fused_attn": [P, P, P, P, I, I, I, I, I, P],
    "layer_mid_attn": [P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, P],
    "layer_pre_attn": [P, P, P, P, I, I, P, P, I, I, P, P, I, I, P, P, P, P, I, I, P],
    "layer_post_attn": [P, P, P, P, I, I, P, P, P, I, I, P, P, I, I, P, P, I, I, P, P, P, P, P, I, I, I, I, I, P],
    "layer_post_o_fp8_mlp": [P, P, P, P, P, I, P, P, I, P, P, I, P, P, P, P, P, I, I, I, P],
    "launch_prepare_linear_gates": [P, P, P, P, P, P, I, P],
    "launch_rmsnorm_gated_decode": [P, P, P, P, I, I, F, P],
    "launch_delta_rule_decode": [P, P, P, P, P, P, P, I, I, P],
}
REFERENCE_FP8_ARGTYPES = {
    "fp8_gemm_batch": [P, P, P, P, I, I, I, I, P],
}

# New exports (include/qwen_fused.h): (restype, argtypes).
NEW_FUSED = {
    "qwen_last_error": (I, []),
    "qwen_get_device_error": (I, [P]),
    "qwen_set_wait_timeout_ns": (I, [ctypes.c_ulonglong]),
    "qwen_set_pdl": (None, [I]),
    "qwen_set_prefetch": (None, [P, ctypes.c_ulonglong, P, ctypes.c_ulonglong, P, ctypes.c_ulonglong, P,
                                 ctypes.c_ulonglong]),
    "qwen_abi_version": (I, []),
    "launch_gemv_f32s": (I, [P, P, P, P, I, I, I, P]),
    "qwen_gemv_generic": (I, [P, P, P, I, P, I, I, I, P]),
    "launch_lm_head_argmax": (I, [P, P, F, P, P, I, I, I, I, P, P, P, P, P, P]),
    "qwen_embed": (I, [P, P, P, I, P]),
    "qwen_attn_in_proj": (I, [P, P, F, P, P, I, P, P, I, P, P, I, I, I, P, P, P, P]),
    "qwen_gdn_in_proj": (I, [P, P, F, I, I, P, P, I, P, P, I, P, P, P, I, P, P, P, P, P, I, P, P, P, P, P]),
    "qwen_gdn_decode": (I, [P, P, P, P, P, P, F, P, I, I, I, P]),
    "qwen_linear_resid": (I, [P, P, P, I, I, I, P, P, P]),
    "qwen_linear_slices": (I, [P, P, P, I, I, I, P, P, I, P]),
    "qwen_set_slices_input": (I, [P, P, I, I, P]),
    "qwen_mlp_gate_up": (I, [P, P, F, P, P, P, P, I, I, I, P, P]),
    "qwen_attn_decode": (I, [P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, F, I, I, P, P, P, P]),
    "qwen_attn_decode_noalloc": (I, [P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, F, I, I, P, P]),
    "qwen_linear_partial": (I, [P, P, P, I, I, I, P, P]),
    "qwen_resid_add_f32": (I, [P, P, P, I, P]),
    "qwen_token_from_key": (I, [P, P, P]),
    "qwen_publish_token": (I, [P, P, P, P]),
    "qwen_p2p_create": (I, [I, I, P, P]),
    "qwen_p2p_open": (I, [P, P]),
    "qwen_p2p_close": (I, [P]),
    "qwen_p2p_destroy": (I, [P]),
    "qwen_p2p_table": (I, [P, I, I, I, P]),
    "qwen_p2p_table_free": (I, [P]),
    "qwen_linear_partial_p2p": (I, [P, P, P, I, I, I, P, P]),
    "qwen_resid_add_p2p": (I, [P, P, P, I, P]),
    "qwen_token_p2p": (I, [P, P, P, P]),
    "qwen_set_p2p_input": (I, [P, P, I]),
    "qwen_gdn_decode_core": (I, [P, P, P, P, P, I, I, I, P]),
    "qwen_set_gated_input": (I, [P, P, F]),
    # persistent decode step (include/qwen_step.h)
    "qwen_step_packed_bytes": (ctypes.c_size_t, [I, I]),
    "qwen_step_pack": (I, [P, P, I, I, I, I, P, P]),
    "qwen_step_create": (I, [P, I, P]),
    "qwen_step_launch": (I, [P, P]),
    "qwen_step_reset": (I, [P, P]),
    "qwen_step_packed_bytes_bf16": (ctypes.c_size_t, [I, I]),
    "qwen_step_create_tp": (I, [P, I, I, I, P, P, P, P]),
    "qwen_step_counter_bytes": (ctypes.c_size_t, [I]),
    "qwen_ipc_alloc": (I, [ctypes.c_size_t, P, P]),
    "qwen_step_pack_bf16": (I, [P, I, I, P, P]),
    "qwen_step_set_drop": (I, [P, I]),
    "qwen_step_destroy": (I, [P]),
    "qwen_step_set_timeline": (I, [P, P]),
    "qwen_step_grid": (I, [P]),
    "qwen_step_smem_bytes": (I, []),
}
NEW_FP8 = {
    "qwen_fp8_last_error": (I, []),
}

_fused = None
_fp8 = None


def fused_path() -> str:
    return os.environ.get("QWEN_FUSED_DLL") or os.path.join(LIB_DIR, FUSED_NAME)


def fp8_path() -> str:
    return os.environ.get("QWEN_FP8_DLL") or os.path.join(LIB_DIR, FP8_NAME)


def _open(path: str) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise RuntimeError(
            f"CUDA library {path} is missing: build it with `make -C qwen3.5-fp8-cuda_b200/csrc` "
            "(or __graft_entry__.build()); there is no CPU fallback")
    return ctypes.CDLL(path)


def _bind(lib, ref_types, new_types):
    for name, argtypes in ref_types.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = None
    for name, (restype, argtypes) in new_types.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype


def fused() -> ctypes.CDLL:
    global _fused
    if _fused is None:
        lib = _open(fused_path())
        _bind(lib, REFERENCE_FUSED_ARGTYPES, NEW_FUSED)
        _fused = lib
    return _fused


def fp8() -> ctypes.CDLL:
    global _fp8
    if _fp8 is None:
        lib = _open(fp8_path())
        _bind(lib, REFERENCE_FP8_ARGTYPES, NEW_FP8)
        _fp8 = lib
    return _fp8


def check(status: int, what: str = "") -> None:
    """Raise on a non-zero status from a new-style export."""
    if status:
        raise RuntimeError(f"{what or 'qwen kernel'} failed with CUDA error {status}")


def check_last(what: str = "") -> None:
    """Raise if a reference-style (void) export recorded an error."""
    e = fused().qwen_last_error()
    if e:
        raise RuntimeError(f"{what or 'qwen kernel'} failed with CUDA error {e}")


def device_error() -> int:
    """Read and clear the device-side error word (bounded-wait timeouts)."""
    v = ctypes.c_uint(0)
    check(fused().qwen_get_device_error(ctypes.byref(v)), "qwen_get_device_error")
    return int(v.value)
