"""Loads libwpt_b200.so (built in-tree by wpt_b200/build.py) and declares
the C ABI of include/wpt_attn.h for ctypes. There is no fallback: when the
library is missing or was built for another GPU, every operation raises."""

import ctypes
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libwpt_b200.so")

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float

# name -> argument types, in include/wpt_attn.h's order
SIGNATURES = {
    "wpt_last_error": [],
    "wpt_status": [ctypes.POINTER(ctypes.c_uint), _I],
    "wpt_attn_prefill": [_P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I,
                         _I, _I, _I, _I, _I, _I, _F, _P],
    "wpt_attn_decode": [_P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I,
                        _I, _I, _I, _I, _I, _I, _F, _P],
    "wpt_attn_topk": [_P, _P, _I64, _I64, _P, _P, _P, _I64, _P, _I, _I, _I, _I, _I, _I, _I, _F, _P],
    "wpt_accept": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P],
    "wpt_head_scores": [_P, _I64, _P, _I64, _I, _I, _I, _I, _P, _P],
    "wpt_accept_scratch_bytes": [_I, _I, _I],
    "wpt_temperature_scale": [_P, _I64, _F, _P, _P],
    "wpt_attn_decode_noalloc": [_P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _I, _P, _P, _P, _I, _I, _I, _I,
                                _I, _I, _I, _I, _F, _P],
    "wpt_attn_merge": [_P, _P, _I, _I64, _I64, _I, _I, _P, _P, _P, _P],
    "wpt_tree_bits": [_P, _I64, _I, _I, _P, _P, _P, _P],
    "wpt_attn_backward_scratch_bytes": [_I, _I, _I, _I, _I],
    "wpt_attn_backward": [_P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P,
                          _P, _I, _I, _I, _I, _I, _I, _I, _F, _P],
    "wpt_f32_to_bf16": [_P, _I64, _P, _P],
    "wpt_debug_backward_fault": [_I, ctypes.c_ulonglong],
    "wpt_cache_append": [_P, _I64, _I64, _P, _I64, _I64, _P, _P, _I, _I, _I, _I64, _P],
    "wpt_attn_merge_groups": [_P, _I, _I, _I64, _I64, _I, _I, _P, _P, _P, _P],
    "wpt_attn_merge_partial": [_P, _P, _I, _I64, _I64, _I, _P, _P, _P],
    "wpt_peer_bytes": [_I, _I64, _I],
    "wpt_peer_alloc": [ctypes.c_size_t, ctypes.POINTER(_P), _P],
    "wpt_peer_open": [_P, ctypes.POINTER(_P)],
    "wpt_peer_close": [_P, _I],
    "wpt_attn_exchange": [_P, _P, _I, _I64, _I, _I, _P, ctypes.POINTER(_P), _I, _I, _P, _P, _P],
}

RESTYPES = {"wpt_last_error": ctypes.c_char_p, "wpt_accept_scratch_bytes": ctypes.c_size_t,
            "wpt_attn_backward_scratch_bytes": ctypes.c_size_t, "wpt_peer_bytes": ctypes.c_size_t}

_lib = None


class LibraryMissing(ImportError):
    """libwpt_b200.so is not built: run `python -m wpt_b200.build`."""


def lib():
    """The loaded library (declared once)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LibraryMissing(f"{LIB_PATH} is not built: run `python -m wpt_b200.build`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        _lib = handle
    return _lib


def check(rc):
    """Raises for a non-zero status of a C-ABI call: NotImplementedError for
    a shape the kernels do not compute (the reference's tests skip those),
    ValueError for a broken contract, RuntimeError for a CUDA failure."""
    if rc == OK:
        return
    message = lib().wpt_last_error().decode(errors="replace")
    if rc == ERR_UNSUPPORTED:
        raise NotImplementedError(message)
    if rc == ERR_INVALID:
        raise ValueError(message)
    raise RuntimeError(message)


def ptr(t):
    """A tensor's device address for the C ABI, or NULL for None (the
    declared argument types convert plain integers)."""
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream(device):
    """The current CUDA stream of `device` as a handle (the raw query skips
    building a torch Stream object on every call)."""
    if _raw_stream is not None:
        index = device.index if device.index is not None else torch.cuda.current_device()
        return _raw_stream(index)
    return torch.cuda.current_stream(device).cuda_stream


def device_status(reset=True):
    """The device-side status word (bit 0: a bounded wait ran out of time);
    synchronises the device."""
    value = ctypes.c_uint(0)
    check(lib().wpt_status(ctypes.byref(value), 1 if reset else 0))
    return value.value
