"""Bindings of libqfn.so, the C ABI declared in include/qfn.h: ctypes for every
entry point (lib()), and the thin torch extension over the same ABI for the
hot-path operators (ops(): torch.ops.qfn.moe_decode / moe_prefill / gemv /
linear).

Both libraries are loaded from this directory (built in-tree by build.py).
There is no fallback: if a library is missing or the device is not an sm_100
part, every call raises.
"""
import contextlib
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqfn.so")

DTYPE_F32 = 0
DTYPE_BF16 = 1

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int

# name -> (argtypes); every entry point returns int status.
SIGNATURES = {
    "qfn_deq": [_P, _P, ctypes.c_float, _P, _I64, _I64, _P],
    "qfn_block_deq": [_P, _P, _P, _P, _P, _P],
    "qfn_moe_decode": [_P, _I64, _P, _P, _P, _P, _I, _P, _P, _I, _P],
    "qfn_moe_decode_variant": [_P, _I64, _P, _P, _P, _P, _I, _P, _P, _I, _I, _P],
    "qfn_moe_decode_noalloc": [_P, _I64, _P, _P, _P, _P, _I, _P, _I, _P],
    "qfn_device_status": [_P, _I],
    "qfn_gemv_e4m3": [_P, _P, _P, _P, _I, _I64, _I64, _P],
    "qfn_e4m3_rows_to_bf16": [_P, _P, _P, _I64, _I64, _P],
    "qfn_linear_e4m3": [_P, _P, _P, _P, _I64, _I64, _I64, _P],
    "qfn_moe_prefill_workspace": [_I64, _I, _I],
    "qfn_moe_prefill": [_P, _I64, _P, _I, _P, _I, _I, _P, _I64, _I64, _P, _I, _P, _P, ctypes.c_size_t, _P],
    "qfn_prefill_status": [_P, _I],
    "qfn_set_prefill_sm_budget": [_I],
    "qfn_moe_route": [_P, _P, _I64, _I, _I, _I64, _P, _P, _P, _P, _P, _P, _P, _P],
    "qfn_shared_expert": [_P, _I64, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P],
    "qfn_moe_prefill_ep_workspace": [_I64, _I, _I, _I],
    "qfn_moe_prefill_ep": [_P, _I64, _P, _I, _P, _I, _I, _P, _I64, _I64, _P, _I, _P, _I, _P, _P, _P, ctypes.c_size_t, _P],
    "qfn_nccl_unique_id": [_P],
    "qfn_nccl_comm_init": [_P, _I, _I, _P],
    "qfn_nccl_comm_destroy": [_P],
    "qfn_shared_expert_gate_up": [_P, _I64, _P, _P, _P, _I, _P, _P, _P],
    "qfn_shared_expert_down": [_P, _I, _I64, _P, _P, _P, _P, _P],
    "qfn_deltanet_step": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
}
# entry points whose return value is not an int status
RESTYPES = {"qfn_moe_prefill_workspace": ctypes.c_size_t, "qfn_moe_prefill_ep_workspace": ctypes.c_size_t}


class QfnError(RuntimeError):
    """A libqfn entry point returned a non-zero status."""


_lib = None


def lib():
    """Load libqfn.so once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python {HERE}/build.py` "
                              "(or __graft_entry__.build()); there is no non-CUDA fallback")
        L = ctypes.CDLL(LIB_PATH)
        L.qfn_version.restype = _I
        L.qfn_strerror.argtypes = [_I]
        L.qfn_strerror.restype = ctypes.c_char_p
        L.qfn_last_error.restype = ctypes.c_char_p
        for name, argtypes in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = argtypes
            fn.restype = RESTYPES.get(name, _I)
        _lib = L
    return _lib


_ops = None
TORCH_EXT_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libqfn_torch.so")


def ops():
    """torch.ops.qfn: the thin torch extension over the C ABI (moe_decode,
    moe_prefill, gemv, linear).  Loads libqfn_torch.so (built next to libqfn.so by
    build.py); there is no fallback when it is missing."""
    global _ops
    if _ops is None:
        lib()   # libqfn.so first (the extension links it)
        if not os.path.exists(TORCH_EXT_PATH):
            raise RuntimeError(f"{TORCH_EXT_PATH} not built: run qwen-flash-next-8gb_b200/build.py "
                               "(or __graft_entry__.build()); there is no non-CUDA fallback")
        torch.ops.load_library(TORCH_EXT_PATH)
        _ops = torch.ops.qfn
    return _ops


def check(rc, what):
    if rc != 0:
        L = lib()
        raise QfnError(f"{what}: {L.qfn_strerror(rc).decode()} ({L.qfn_last_error().decode()})")


def device_status(clear=True):
    """Device status word of the current device (bit 0: a kernel wait timed out)."""
    v = ctypes.c_uint(0)
    check(lib().qfn_device_status(ctypes.byref(v), int(clear)), "qfn_device_status")
    return v.value


def prefill_status(clear=True):
    """Prefill status word of the current device (bit 0: a wait timed out; bit 2: bad expert id skipped)."""
    v = ctypes.c_uint(0)
    check(lib().qfn_prefill_status(ctypes.byref(v), int(clear)), "qfn_prefill_status")
    return v.value


def set_prefill_sm_budget(n_sms):
    """Persistent prefill GEMMs on at most n_sms SMs of the current device (0 = all)."""
    check(lib().qfn_set_prefill_sm_budget(int(n_sms)), "qfn_set_prefill_sm_budget")


def stream_of(t):
    """Raw cudaStream_t of torch's current stream on tensor t's device."""
    return torch._C._cuda_getCurrentRawStream(t.device.index)


_SAME_DEVICE = contextlib.nullcontext()


def on_device(dev):
    """Make `dev` the current CUDA device for a library call (the library
    launches on the current device); free when it already is."""
    if dev.index == torch._C._cuda_getDevice():
        return _SAME_DEVICE
    return torch.cuda.device(dev)


def require_cuda(name, t, dtype=None, contiguous=True):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (libqfn has no CPU path)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
