"""ctypes binding of `libveda_b200.so` (the C ABI declared in
include/veda_b200.h).

The library is loaded on first use. Every call checks the returned code and
raises the reference's exception types: ValueError for argument misuse,
NotImplementedError for an unsupported device (naming the architecture and
the operation), RuntimeError for CUDA errors and expired device waits. There
is no fallback path: without the library or a B200, the operations raise.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, 'libveda_b200.so')

VEDA_OK = 0
VEDA_ERR_INVALID = 1
VEDA_ERR_UNSUPPORTED = 2
VEDA_ERR_CUDA = 3
VEDA_ERR_TIMEOUT = 4

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_ptr = ctypes.c_void_p


class Span(ctypes.Structure):
    """veda_span_t."""
    _fields_ = [('start', c_i64), ('grid', c_i32 * 3), ('shape', c_i32 * 3)]


class ColumnBlockC(ctypes.Structure):
    """veda_column_block_t."""
    _fields_ = [('start', c_i32), ('stop', c_i32), ('k_lo', c_i32),
                ('k_hi', c_i32), ('frac', ctypes.c_double),
                ('keeps_all', c_i32), ('pad_', c_i32)]


# name -> (restype, argtypes), in the order of include/veda_b200.h
SIGNATURES = {
    'veda_last_error': (c_i32, [ctypes.c_char_p, ctypes.c_size_t]),
    'veda_device_status': (c_i32, [ctypes.POINTER(c_i32), c_i32]),
    'veda_set_sm_reserve': (c_i32, [c_i32]),
    'veda_set_fwd_groups': (c_i32, [c_i32]),
    'veda_ipc_handle': (c_i32, [c_ptr, c_ptr, c_ptr]),
    'veda_ipc_open': (c_i32, [c_ptr, c_ptr]),
    'veda_ipc_close': (c_i32, [c_ptr]),
    'veda_copy_2d': (c_i32, [c_ptr, c_i64, c_ptr, c_i64, c_i64, c_i64,
                             c_ptr]),
    'veda_supported_device': (c_i32, []),
    'veda_build_layout': (c_i32, [ctypes.POINTER(Span), c_i32, c_i64, c_i64,
                                  c_i64, c_ptr, c_ptr, c_ptr]),
    'veda_build_box_layout': (c_i32, [ctypes.POINTER(Span), c_i32, c_i64,
                                      c_i64, c_i64, c_ptr, c_ptr, c_ptr]),
    'veda_gather_pool': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_ptr, c_i64,
                                 c_ptr, c_i32, c_ptr, c_i64, c_i64, c_ptr,
                                 c_ptr, c_ptr, c_ptr]),
    'veda_gather_pool_images': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_ptr,
                                        c_i64, c_ptr, c_i32, c_ptr, c_ptr,
                                        c_ptr]),
    'veda_head_blocks': (c_i32, [c_ptr, c_ptr, c_i64, c_i32, c_i64, c_i64,
                                 c_i64, c_i64, c_i32, c_ptr]),
    'veda_scatter': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_i64, c_ptr, c_i32,
                             c_ptr, c_i64, c_i64, c_ptr]),
    'veda_gather_lse': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_i64, c_ptr,
                                c_i32, c_ptr, c_ptr]),
    'veda_predict_workspace': (c_i64, [c_i32, c_i64, c_i64]),
    'veda_predict_logits': (c_i32, [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32,
                                    c_i64, c_i64, c_ptr, c_ptr, c_i64,
                                    c_ptr]),
    'veda_predict_logits_noalloc': (c_i32, [c_ptr, c_ptr, c_ptr, c_ptr,
                                            c_ptr, c_i32, c_i64, c_i64,
                                            c_ptr, c_ptr]),
    'veda_block_select': (c_i32, [c_ptr, c_i64, c_i32, c_i64, c_ptr, c_ptr,
                                  c_i64, c_i64, ctypes.POINTER(ColumnBlockC),
                                  c_i32, c_i32, c_ptr, c_ptr, c_ptr, c_ptr,
                                  c_ptr, c_i32, c_ptr, c_ptr, c_ptr]),
    'veda_index_lists': (c_i32, [c_ptr, c_i32, c_i64, c_i64, c_ptr, c_i32,
                                 c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_ptr]),
    'veda_bsa_fwd': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_i64, c_i64, c_ptr,
                             c_i64, c_i64, c_i32, c_i64, c_i64, c_ptr, c_ptr,
                             c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_i64, c_i64,
                             c_ptr, c_f32, c_ptr]),
    'veda_bsa_fwd_packed': (c_i32, [c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_i64,
                                    c_i32, c_i32, c_i64, c_i64, c_ptr, c_ptr,
                                    c_ptr, c_i64, c_i64, ctypes.POINTER(Span),
                                    c_i32, c_i64, c_i64, c_ptr, c_i32, c_ptr,
                                    c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr,
                                    c_i64, c_ptr, c_i64, c_i64, c_f32,
                                    c_ptr, c_i32, c_i64, c_ptr]),
    'veda_dense_fwd': (c_i32, [c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_i64,
                               c_i64, c_i32, c_ptr, c_i64, c_i64, c_ptr,
                               c_i64, c_i64, c_f32, c_ptr]),
    'veda_bsa_bwd_workspace': (c_i64, [c_i32, c_i64]),
    'veda_bsa_bwd': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_i64, c_i64, c_ptr,
                             c_i64, c_i64, c_ptr, c_i64, c_i64, c_ptr, c_i64,
                             c_i64, c_ptr, c_i64, c_i64, c_i32, c_i64, c_i64,
                             c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_ptr,
                             c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_i64, c_i64,
                             c_ptr, c_i64, c_i64, c_ptr, c_i64, c_i64, c_f32,
                             c_ptr, ctypes.c_size_t, c_ptr]),
    'veda_teacher_heat': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_i64, c_i64,
                                  c_ptr, c_i64, c_i64, c_i32, c_i64, c_ptr,
                                  c_ptr, c_i64, c_i32, c_ptr, c_f32, c_ptr]),
    'veda_bsa_fwd_heat_workspace': (c_i64, [c_i64]),
    'veda_bsa_fwd_heat': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_i64, c_i64,
                                  c_ptr, c_i64, c_i64, c_i32, c_i64, c_ptr,
                                  c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_ptr,
                                  c_i64, c_i64, c_ptr, c_i32, c_ptr, c_f32,
                                  c_ptr, c_i64, c_ptr]),
    'veda_rel_mse_workspace': (c_i64, [c_i64, c_i32]),
    'veda_rel_mse': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_i64, c_i64, c_ptr,
                             c_ptr, c_i64, c_i32, c_ptr, c_ptr, c_i64, c_ptr]),
    'veda_compensate_workspace': (c_i64, [c_i32, c_i64]),
    'veda_compensate': (c_i32, [c_ptr, c_i64, c_i64, c_ptr, c_ptr, c_i64,
                                c_i64, c_ptr, c_i64, c_i64, c_ptr, c_i64,
                                c_i64, c_i32, c_i64, c_i64, c_ptr, c_ptr,
                                c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_i64,
                                c_i64, c_f32, c_ptr, c_i64, c_ptr]),
    'veda_probe_umma': (c_i32, [c_ptr, c_ptr, c_ptr, c_i32, c_ptr]),
    'veda_expire_wait': (c_i32, [c_i64, c_ptr, c_ptr]),
}

_LOCK = threading.Lock()
_LIB = None


def load() -> ctypes.CDLL:
    """The loaded library (raises if it was not built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f'{LIB_PATH} is missing: build it with '
                    '`python -m miowtion_b200.build` (there is no fallback)')
            lib = ctypes.CDLL(LIB_PATH)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _LIB = lib
    return _LIB


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().veda_last_error(buf, len(buf))
    return buf.value.decode(errors='replace')


def check(rc: int, op: str) -> None:
    if rc == VEDA_OK:
        return
    msg = f'{op}: {last_error()}'
    if rc == VEDA_ERR_INVALID:
        raise ValueError(msg)
    if rc == VEDA_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    """Calls an int-returning entry point and raises on failure."""
    check(getattr(load(), name)(*args), name)


def device_status(reset: bool = True) -> int:
    """The device status word (VEDA_ERR_TIMEOUT after an expired wait)."""
    status = c_i32(0)
    call('veda_device_status', ctypes.byref(status), 1 if reset else 0)
    return status.value


def raise_on_device_status() -> None:
    """Reads and clears the device status word; raises RuntimeError when a
    kernel's bounded wait expired since the last read (the kernel returned
    early, so its outputs are not to be trusted)."""
    status = device_status(reset=True)
    if status == VEDA_ERR_TIMEOUT:
        raise RuntimeError('a Veda kernel wait timed out on the device; its '
                           'outputs are incomplete')
    if status != 0:
        raise RuntimeError(f'device status word holds {status}')


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()
