"""ctypes binding of libscope_b200.so (the C ABI in include/scope_b200.h).

The library is loaded once, in-tree.  If it is missing the import fails
loudly: there is no CPU or library fallback for any op of this package.
The argument structs are mirrored field for field; ``check_abi()``
compares their size and last-field offset with what the compiled library
reports.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libscope_b200.so")

P = ctypes.c_void_p
I32 = ctypes.c_int32
I64 = ctypes.c_int64
F32 = ctypes.c_float


class ScopeMaskArgs(ctypes.Structure):
    _fields_ = [
        ("H", I32), ("QB", I32), ("M", I32), ("block_size", I32),
        ("sel_logits", P), ("sel_gumbel", P),
        ("sel_head_stride", I64), ("sel_row_stride", I64),
        ("sel_tau", F32),
        ("delta_rep", P),
        ("delta_head_stride", I64), ("delta_row_stride", I64), ("delta_m_stride", I64),
        ("budget_rep", P),
        ("budget_head_stride", I64), ("budget_row_stride", I64), ("budget_m_stride", I64),
        ("peak_gumbel", P),
        ("gumbel_k", I32),
        ("gumbel_tau", F32),
        ("block_info", P),
        ("local_blocks", I32), ("half_blocks", I32), ("half_active", I32), ("ptr_enabled", I32),
        ("global_max", I32), ("global_active", I32), ("radius_mode", I32), ("budget_rem", I32),
        ("budget_temp", F32),
        ("kv_num", P), ("kv_indices", P),
        ("kv_stride", I32), ("flex_padded", I32),
        ("q_bitmap", P), ("r_m_out", P), ("centres_out", P), ("stats", P), ("err_flag", P),
    ]


class ScopeAttnArgs(ctypes.Structure):
    _fields_ = [
        ("H", I32), ("T", I32), ("D", I32), ("block_size", I32),
        ("dtype", I32),
        ("q", P), ("k", P), ("v", P),
        ("q_sh", I64), ("q_st", I64), ("k_sh", I64), ("k_st", I64), ("v_sh", I64), ("v_st", I64),
        ("out", P),
        ("o_sh", I64), ("o_st", I64),
        ("lse", P),
        ("kv_num", P), ("kv_indices", P),
        ("kv_stride", I32),
        ("q_bitmap", P), ("block_info", P), ("docs", P),
        ("scale", F32),
        ("bias_mode", I32), ("K", I32),
        ("coeff_cos", P), ("coeff_sin", P),
        ("cos_tab", P), ("sin_tab", P),
        ("tab_len", I32),
        ("b0", P), ("slope", P), ("delta_main", P), ("width", P),
        ("gate", I32),
        ("beta", F32), ("gate_lambda", F32), ("gate_tau", F32),
        ("q_aug", P), ("k_aug", P),
        ("d_aug", I32),
        ("dout", P),
        ("do_sh", I64), ("do_st", I64),
        ("dq", P), ("dk", P), ("dv", P),
        ("dq_sh", I64), ("dq_st", I64), ("dk_sh", I64), ("dk_st", I64), ("dv_sh", I64), ("dv_st", I64),
        ("dcoeff_cos", P), ("dcoeff_sin", P),
        ("db0", P), ("dslope", P), ("ddelta_main", P), ("dwidth", P),
        ("workspace", P),
        ("workspace_bytes", ctypes.c_size_t),
        ("flags", I32),
        ("err_flag", P),
    ]


class ScopeCoeffMlpBwdArgs(ctypes.Structure):
    _fields_ = [
        ("H", I32), ("T", I32), ("n_out", I32),
        ("q", P),
        ("q_sh", I64), ("q_st", I64),
        ("w1", P), ("b1", P), ("w2", P),
        ("dy", P),
        ("dq", P),
        ("dw1", P), ("db1", P), ("dw2", P),
        ("err_flag", P),
    ]


# symbols declared in include/scope_b200.h, with ctypes signatures
class ScopeCoeffArgs(ctypes.Structure):
    _fields_ = [
        ("H", I32), ("T", I32), ("D", I32), ("hidden", I32), ("K", I32), ("M", I32),
        ("use_slope", I32), ("subtract_b0", I32),
        ("q", P),
        ("q_sh", I64), ("q_st", I64),
        ("w_heads", I32),
        ("w1", P), ("b1", P), ("w2", P), ("b2", P),
        ("omegas", P), ("log_omegas", P),
        ("delta_cap", F32),
        ("logw_min", F32), ("logw_max", F32), ("c_scale", F32), ("width_min", F32), ("width_max", F32),
        ("eps", F32),
        ("coeff_cos", P), ("coeff_sin", P),
        ("slope", P), ("b0", P),
        ("delta_star", P), ("pi", P), ("budget_logits", P),
        ("delta_main", P), ("width", P),
        ("mlp_out", P),
        ("omega_reg", P),
        ("err_flag", P),
    ]


class ScopeCoeffBwdArgs(ctypes.Structure):
    _fields_ = [
        ("H", I32), ("T", I32), ("K", I32), ("M", I32), ("use_slope", I32), ("subtract_b0", I32),
        ("mlp_out", P),
        ("dcoeff_cos", P), ("dcoeff_sin", P),
        ("db0", P), ("dslope", P), ("ddelta_main", P), ("dwidth", P),
        ("ddelta_star", P), ("dpi", P), ("dbudget_logits", P),
        ("domega_reg", P),
        ("omegas", P), ("log_omegas", P),
        ("delta_cap", F32), ("logw_min", F32), ("logw_max", F32), ("c_scale", F32), ("width_min", F32),
        ("width_max", F32), ("eps", F32),
        ("dy", P), ("dy_bf16", P), ("dy_ld", I32),
        ("err_flag", P),
    ]


SIGNATURES = {
    "scope_block_info": (I32, [P, I32, I32, I32, I32, I32, P, P]),
    "scope_mask_max_kv": (I32, [I32, I32, I32, I32]),
    "scope_mask_build": (I32, [ctypes.POINTER(ScopeMaskArgs), P]),
    "scope_mask_transpose": (I32, [P, I32, I32, P, P, P]),
    "scope_mask_refine": (I32, [P, P, I32, I32, I32, P, P, I32, P, P, P]),
    "scope_mask_bitmap_from_lists": (I32, [P, P, I32, I32, I32, P, P, P]),
    "scope_trig_tables": (I32, [P, I32, I32, P, P, P]),
    "scope_qk_aug_prepare": (I32, [P, P, P, P, P, I32, I32, I32, I32, I32, F32, F32, I32, P, P, P]),
    "scope_spectral_coeffs": (I32, [ctypes.POINTER(ScopeCoeffArgs), P]),
    "scope_spectral_coeffs_bwd": (I32, [ctypes.POINTER(ScopeCoeffBwdArgs), P]),
    "scope_spectral_mlp_bwd": (I32, [ctypes.POINTER(ScopeCoeffMlpBwdArgs), P]),
    "scope_selftest_wait_timeout": (I32, [P, ctypes.c_uint32, P]),
    "scope_selftest_exp2_fma": (I32, [P, P, I32, P]),
    "scope_attn_fwd": (I32, [ctypes.POINTER(ScopeAttnArgs), P]),
    "scope_attn_bwd": (I32, [ctypes.POINTER(ScopeAttnArgs), P]),
    "scope_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(ScopeAttnArgs)]),
    "scope_block_mass": (I32, [ctypes.POINTER(ScopeAttnArgs), P, P]),
    "scope_attn_bwd_static_scratch": (I32, [ctypes.POINTER(ScopeAttnArgs), P]),
    "scope_static_scratch_bytes": (ctypes.c_size_t, []),
    "scope_error_string": (ctypes.c_char_p, [I32]),
    "scope_abi_layout": (ctypes.c_size_t, [I32, I32]),
    "scope_device_supported": (I32, []),
    "scope_launch_count": (ctypes.c_uint64, []),
}

SCOPE_ERRORS = {
    -1: ValueError, -2: TypeError, -3: ValueError, -4: RuntimeError, -5: RuntimeError, -6: ValueError,
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (loaded on first use).  Raises if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"scope_b200: {LIB_PATH} is missing; build it with `python -m scope_b200.build` "
                "(there is no fallback implementation)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    """Raise the Python exception matching a scope_status, as flex would."""
    if status != 0:
        msg = lib().scope_error_string(status).decode()
        raise SCOPE_ERRORS.get(status, RuntimeError)(f"{what}: {msg} (status {status})")


def check_abi() -> None:
    L = lib()
    for which, S in ((0, ScopeMaskArgs), (1, ScopeAttnArgs), (2, ScopeCoeffArgs), (3, ScopeCoeffBwdArgs),
                     (4, ScopeCoeffMlpBwdArgs)):
        size, last = L.scope_abi_layout(which, 0), L.scope_abi_layout(which, 1)
        if size != ctypes.sizeof(S) or last != S.err_flag.offset:
            raise RuntimeError(f"scope_b200 ABI mismatch for {S.__name__}: C sizeof={size} last={last}, "
                               f"ctypes sizeof={ctypes.sizeof(S)} last={S.err_flag.offset}")


FLAG_CUDA_CORES = 0x1
DEVERR_INDEX, DEVERR_TIMEOUT, DEVERR_SHAPE = 0x1, 0x2, 0x4

_err_words = {}


def err_word_ptr(device) -> int:
    """Address of this device's error word (int32, zero-initialised), which
    every launch from this package passes as ``err_flag``."""
    import torch
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _err_words.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _err_words[idx] = t
    return t.data_ptr()


def device_errors(device=None, reset: bool = True) -> int:
    """Error bits the kernels have set on a device since the last reset
    (synchronises with the device)."""
    import torch
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _err_words.get(idx)
    if t is None:
        return 0
    v = int(t.item())
    if reset:
        t.zero_()
    return v


def ptr(t) -> int | None:
    """Device address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
