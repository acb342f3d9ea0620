"""ctypes binding of ``libtinker_b200.so``, the C-ABI kernel library.

The library is loaded on first use. There is no fallback: if it is missing, or
a call is made with tensors that are not on an sm_100 GPU, the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtinker_b200.so")

TK_F16, TK_BF16, TK_F32 = 0, 1, 2
TK_OK, TK_ERR_INVALID, TK_ERR_CUDA, TK_ERR_UNSUPPORTED = 0, 1, 2, 3

_DTYPE = {torch.float16: TK_F16, torch.bfloat16: TK_BF16, torch.float32: TK_F32}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float



class Epilogue(ctypes.Structure):
    """``tk_epilogue`` of tinker_b200.h: options of tk_linear_ex / tk_gate_up_swiglu_ex."""
    _fields_ = [("residual", _P), ("row_ssq_in", _P), ("row_ssq_parts", _I), ("row_ssq_eps", _F),
                ("row_ssq_out", _P), ("rope_seq", _I), ("rope_start", _I), ("rope_head_dim", _I),
                ("rope_cos", _P), ("rope_sin", _P), ("rope_table_rows", _I64),
                ("weights_prefetch", _I), ("l2_prefetch", _P * 8), ("l2_prefetch_bytes", _I64 * 8)]


_EPI = ctypes.POINTER(Epilogue)


class StepLayer(ctypes.Structure):
    """``tk_step_layer`` of tinker_b200.h: one layer of tk_decode_step_setup's table."""
    _fields_ = [("wq", _P), ("wk", _P), ("wv", _P), ("wo", _P), ("wg", _P), ("wu", _P), ("wd", _P),
                ("k_cache", _P), ("v_cache", _P), ("eps_attn", _F), ("eps_ffn", _F)]

class StackLayer(ctypes.Structure):
    """``tk_stack_layer`` of tinker_b200.h: one layer of tk_stack_setup's table."""
    _fields_ = [("wq", _P), ("wk", _P), ("wv", _P), ("wo", _P), ("wg", _P), ("wu", _P), ("wd", _P),
                ("eps_attn", _F), ("eps_ffn", _F)]


# name -> argtypes; every entry point returns int (status)
SIGNATURES = {
    "tk_version": [],
    "tk_check_device": [_I],
    "tk_device_error": [ctypes.POINTER(_I), _I],
    "tk_rmsnorm": [_P, _I64, _P, _I, _P, _I64, _I64, _I64, _F, _I, _P],
    "tk_add_rmsnorm": [_P, _P, _P, _I, _P, _P, _I64, _I64, _F, _I, _P],
    "tk_swiglu": [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I, _P],
    "tk_rope_attention": [_P, _I64, _P, _I64, _P, _I64, _P, _P, _I, _I64, _P, _I64, _I, _I, _I, _I, _I, _I, _I, _P],
    "tk_rope_qk": [_P, _I64, _P, _I64, _P, _P, _I, _I64, _P, _I64, _I, _I, _I, _I, _I, _I, _I, _P],
    "tk_causal_attention": [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _I, _I, _I, _P],
    "tk_linear": [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I, _P],
    "tk_linear_rope": [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I, _I, _I, _P, _P, _I64, _I,
                       _P],
    "tk_linear_ex": [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _EPI, _I, _P],
    "tk_gate_up_swiglu": [_P, _I64, _P, _P, _P, _I64, _I64, _I64, _I, _P],
    "tk_gate_up_swiglu_ex": [_P, _I64, _P, _P, _P, _I64, _I64, _I64, _EPI, _I, _P],
    "tk_row_sumsq": [_P, _I64, _I64, _I64, _P, _I, _P],
    "tk_embedding_rows": [_P, _P, _I64, _I64, _P, _P, _I64, _I, _P],
    "tk_swiglu_ffn": [_P, _I64, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _P],
    "tk_swiglu_ffn_noalloc": [_P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _P],
    "tk_kv_attention": [_P, _I64, _P, _I64, _P, _I64, _P, _P, _I, _P, _P, _I64, _P, _I64, _I, _I, _I, _I, _I, _I,
                        _P, _P, _I64, _I, _P],
    "tk_kv_attention_workspace": [_I, _I, _I, _I, _I, _I],
    "tk_kv_append": [_P, _I64, _P, _I64, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P],
    "tk_decode_step_scratch_bytes": [_I, _I, _I, _I, _I, _I, _I, _I],
    "tk_decode_step_setup": [ctypes.POINTER(StepLayer), _I, _I, _I, _I, _I, _I, _I, _P, _P, _I64, _I, _P, _P, _F, _I,
                             _P, _I64],
    "tk_decode_step": [_P, _P, _P, _P],
    "tk_decode_step_release": [_P],
    "tk_decode_step_withhold_arrival": [_P, _I],
    "tk_stack_scratch_bytes": [_I, _I, _I, _I, _I, _I, _I, _I],
    "tk_stack_setup": [ctypes.POINTER(StackLayer), _I, _I, _I, _I, _I, _I, _I, _I, _P, _I64, _P, _P, _I64, _I, _P,
                       _F, _I, _P, _I64],
    "tk_stack_forward": [_P, _P, _P, _P],
    "tk_stack_plan": [_P, ctypes.POINTER(_I), _I],
    "tk_stack_release": [_P],
    "tk_stack_trace": [_P, _P],
}

# entry points whose return value is not a status
RESTYPES = {"tk_kv_attention_workspace": _I64, "tk_decode_step_scratch_bytes": _I64, "tk_stack_scratch_bytes": _I64}

_lock = threading.Lock()
_lib = None
_checked_devices: set[int] = set()


class TinkerKernelError(RuntimeError):
    """A call into libtinker_b200 returned an error status."""


def lib() -> ctypes.CDLL:
    """Load the library (once) and declare every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is not built; run `python -m tinker_b200.build` (needs nvcc). "
                    "tinker_b200 has no fallback path.")
            L = ctypes.CDLL(LIB_PATH)
            for name, argtypes in SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = argtypes
                fn.restype = RESTYPES.get(name, _I)
            L.tk_last_error.argtypes = []
            L.tk_last_error.restype = ctypes.c_char_p
            _lib = L
    return _lib


def last_error() -> str:
    return (lib().tk_last_error() or b"").decode(errors="replace")


# Kernels this process has enqueued through the library (each successful
# compute entry point adds the number of kernels it launched).
launch_counter = [0]


def check(rc: int, what: str, kernels: int = 0) -> None:
    if rc != TK_OK:
        raise TinkerKernelError(f"{what}: {last_error()} (status {rc})")
    launch_counter[0] += kernels


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected float16, bfloat16 or float32") from None


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors on one CUDA device that is an sm_100 GPU; returns that device."""
    dev = tensors[0].device
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("tinker_b200 kernels need CUDA tensors on a B200 (sm_100a); "
                               "there is no CPU fallback")
        if t.device != dev:
            raise RuntimeError(f"tensors on different devices: {t.device} vs {dev}")
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _checked_devices:
        check(lib().tk_check_device(idx), "tk_check_device")
        _checked_devices.add(idx)
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_error(clear: bool = True) -> int:
    """Sticky device-side error word (0: none; 1: a bounded wait timed out; 2: a device-side
    position beyond a KV cache or RoPE table; 3: a token id outside the embedding table)."""
    code = _I(0)
    check(lib().tk_device_error(ctypes.byref(code), 1 if clear else 0), "tk_device_error")
    return code.value
