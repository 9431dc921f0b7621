"""ctypes binding of libnvm_attn.so (the C ABI declared in include/nvm_attn.h).

There is no CPU path: every operator raises if the library is missing or the
tensors are not on a CUDA device.  The library is built in-tree by
``nano-vllm-metal_b200/build.py`` (``__graft_entry__.build()`` calls it).
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnvm_attn.so")

NVM_F32, NVM_F16, NVM_BF16, NVM_I8, NVM_I32, NVM_I64 = 0, 1, 2, 3, 4, 5
NVM_OK = 0

_DTYPE_CODE = {
    torch.float32: NVM_F32,
    torch.float16: NVM_F16,
    torch.bfloat16: NVM_BF16,
    torch.int8: NVM_I8,
    torch.int32: NVM_I32,
    torch.int64: NVM_I64,
}

# Every exported symbol of include/nvm_attn.h with (restype, argtypes).
_P, _I, _I64, _F, _SZ, _CP = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                              ctypes.c_size_t, ctypes.c_char_p)
SIGNATURES = {
    "nvm_status_string": (_CP, [_I]),
    "nvm_last_error": (_CP, []),
    "nvm_version": (_CP, []),
    "nvm_device_error": (_I, [_P, _I]),
    "nvm_selftest_wait_expiry": (_I, [_I64, _P, _P]),
    "nvm_paged_attention": (_I, [_P, _I, _P, _P, _I, _P, _P, _I, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64,
                                 _I64, _I64, _I64, _F, _I, _P, _SZ, _P]),
    "nvm_paged_attention_workspace_size": (_SZ, [_I64, _I64, _I64, _I64, _I64, _I64, _I64, _I]),
    "nvm_paged_attention_noalloc": (_I, [_P, _I, _P, _P, _I, _P, _P, _I, _P, _P, _P, _I, _I64, _I64, _I64, _I64,
                                         _I64, _I64, _I64, _I64, _F, _I, _P]),
    "nvm_flash_attention": (_I, [_P, _P, _P, _I, _P, _I64, _I64, _I64, _P, _I, _I64, _I64, _I64, _I64, _I64,
                                 _I64, _F, _I, _P]),
    "nvm_reshape_and_cache": (_I, [_P, _P, _I, _I64, _I64, _P, _P, _I, _P, _P, _I, _P, _I64, _I64, _I64, _I64,
                                   _I64, _P]),
    "nvm_paged_append": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _P]),
    "nvm_paged_rewind": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "nvm_paged_attach": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "nvm_spec_verify_accept": (_I, [_P, _P, _I64, _I64, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "nvm_w4a16_matmul": (_I, [_P, _I, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "nvm_qk_norm_rope_write": (_I, [_P, _P, _P, _I, _I64, _I64, _P, _P, _F, _P, _P, _I64, _I, _P, _P, _I64, _P,
                                    _P, _I, _P, _P, _I, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load libnvm_attn.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"libnvm_attn.so not found at {LIB_PATH}; build it with "
                        "`python nano-vllm-metal_b200/build.py` (nvcc, sm_100a)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise RuntimeError(f"nvm: unsupported dtype {dtype}") from None


def check(status: int) -> None:
    """Raise RuntimeError carrying the library's message for a failed call."""
    if status != NVM_OK:
        L = lib()
        msg = L.nvm_last_error().decode() or L.nvm_status_string(status).decode()
        raise RuntimeError(f"{msg} [{L.nvm_status_string(status).decode()}]")


def require_cuda(op: str, *tensors: torch.Tensor) -> torch.device:
    """All tensors must live on one CUDA device; returns it."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{op}: tensors must be on a CUDA device (libnvm_attn has no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{op}: all tensors must be on the same CUDA device")
    if dev is None:
        raise RuntimeError(f"{op}: no tensor given")
    return dev


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# Split-K workspace: one zero-filled buffer per (device, stream), grown on demand.
# Successful calls leave its ticket region zero; calls on one stream never overlap on
# the GPU.  A call whose bounded wait expired may leave tickets non-zero, so
# device_error() re-zeroes every workspace of the device after a non-zero word.
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream_ptr(device))
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def device_error(device: torch.device, clear: bool = True) -> int:
    """Synchronise and read the device error word (0 = no bounded wait expired).

    After a non-zero word (a kernel gave up on a wait and returned early), the split-K
    workspaces cached for this device are zero-filled again once the device is idle,
    so the next call cannot merge a half-finished call's tickets or partials.
    """
    with torch.cuda.device(device):
        word = int(lib().nvm_device_error(stream_ptr(device), 1 if clear else 0))
        if word != 0:
            index = device.index if device.index is not None else torch.cuda.current_device()
            torch.cuda.synchronize(device)
            for (dev_index, _), ws in _workspaces.items():
                if dev_index == index:
                    ws.zero_()
            torch.cuda.synchronize(device)
        return word
