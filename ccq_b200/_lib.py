"""ctypes binding of the C ABI in ``include/ccq_b200.h`` (library: ``ccq_b200/lib/libccq_b200.so``).

The library is built in-tree by ``ccq_b200.build``; there is no fallback implementation: if
the shared object cannot be loaded, every operator raises.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, 'lib', 'libccq_b200.so')

# enums of include/ccq_b200.h
CCQ_OK, CCQ_ERR_INVALID, CCQ_ERR_UNSUPPORTED, CCQ_ERR_CUDA, CCQ_ERR_WORKSPACE = 0, 1, 2, 3, 4
CCQ_F32, CCQ_BF16, CCQ_F16 = 0, 1, 2
CCQ_LAMBDA_TOKEN, CCQ_LAMBDA_GATE = 0, 1
CCQ_OP_FWD, CCQ_OP_BWD, CCQ_OP_DECODE = 0, 1, 2
PATHS = {0: 'none', 1: 'simt', 2: 'tcgen05', 3: 'decode'}

EXPORTS = ('ccq_last_error', 'ccq_last_path', 'ccq_version', 'ccq_last_launch_count',
           'ccq_workspace_size', 'ccq_workspace_size_for', 'ccq_device_status', 'ccq_clean_fwd', 'ccq_clean_bwd',
           'ccq_decode_step', 'ccq_clean_bwd_noalloc', 'ccq_noalloc_status', 'ccq_clean_l2norm_fwd',
           'ccq_clean_l2norm_bwd', 'ccq_decode_step_l2norm')
CCQ_WS_HAVE_FWD_OUTPUTS, CCQ_WS_L2NORM = 1, 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t

_SIGS = {
    'ccq_last_error': (ctypes.c_char_p, []),
    'ccq_last_path': (_I, []),
    'ccq_version': (_I, []),
    'ccq_last_launch_count': (_I, []),
    'ccq_workspace_size': (_SZ, [_I, _I, _I, _I, _I, _I, _I]),
    'ccq_workspace_size_for': (_SZ, [_I, _I, _I, _I, _I, _I, _I, _I]),
    'ccq_device_status': (_I, [_P, _P, ctypes.POINTER(_I)]),
    'ccq_noalloc_status': (_I, [_P, ctypes.POINTER(_I)]),
    'ccq_clean_fwd': (_I, [_I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P, _P,
                           _P, _SZ, _P]),
    'ccq_clean_bwd': (_I, [_I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P, _P, _P,
                           _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    'ccq_clean_bwd_noalloc': (_I, [_I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P, _P,
                                   _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    'ccq_decode_step': (_I, [_I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P, _P, _P]),
    'ccq_decode_step_l2norm': (_I, [_I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P,
                                    _P, _P, _P]),
    'ccq_clean_l2norm_fwd': (_I, [_I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P,
                                  _P, _P, _P, _P, _SZ, _P]),
    'ccq_clean_l2norm_bwd': (_I, [_I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P, _P,
                                  _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
}

_lib = None


class CCQError(RuntimeError):
    """A ccq_* entry point returned a non-zero status."""

    def __init__(self, status, message):
        super().__init__(f'ccq status {status}: {message}')
        self.status = status


def load():
    """Load (once) and return the ctypes library handle."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f'{LIB_PATH} is missing: build it with `python -m ccq_b200.build`')
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status):
    if status != CCQ_OK:
        msg = load().ccq_last_error().decode(errors='replace')
        raise CCQError(status, msg)


def last_path():
    return PATHS.get(load().ccq_last_path(), 'unknown')


def last_launch_count():
    return int(load().ccq_last_launch_count())
