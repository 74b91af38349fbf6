"""ctypes binding of ``libbdm_b200.so`` (the C ABI declared in include/bdm_b200.h).

The library is loaded from this package directory.  There is no fallback: if
it is missing or fails to load, every op raises.  Status codes map to the
exception types the reference raises for the same conditions
(ValueError for bad arguments, NotImplementedError for unsupported geometry,
RuntimeError for CUDA failures).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, 'libbdm_b200.so')

BDM_OK, BDM_ERR_INVALID, BDM_ERR_DTYPE, BDM_ERR_UNSUPPORTED, BDM_ERR_CUDA, BDM_ERR_WORKSPACE = range(6)
BDM_F32, BDM_BF16 = 0, 1

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_flt = ctypes.c_float

# name -> (restype, argtypes); mirrors include/bdm_b200.h
SIGNATURES = {
    'bdm_status_string': (ctypes.c_char_p, [_int]),
    'bdm_last_cuda_error': (_int, []),
    'bdm_abi_version': (_int, []),
    'bdm_kernel_launches': (ctypes.c_longlong, []),
    'bdm_route': (_int, [_vp, _i64, _i64, _int, _int, _int, _int, _vp, _vp, _vp]),
    'bdm_route_pair': (_int, [_vp, _i64, _i64, _i64, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _vp]),
    'bdm_dispatch_workspace_bytes': (_i64, [_i64, _i64, _int, _int, _i64]),
    'bdm_dispatch': (_int, [_vp, _vp, _i64, _i64, _int, _int, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp]),
    'bdm_dispatch_noalloc': (_int, [_vp, _vp, _i64, _i64, _int, _int, _i64, _vp, _vp, _vp, _vp, _vp, _vp]),
    'bdm_controllers': (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _int, _vp, _vp,
                               _int, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    'bdm_product_state': (_int, [_vp, _vp, _i64, _i64, _int, _i64, _i64, _int, _int, _int, _vp, _int, _vp]),
    'bdm_bank_scan_workspace_bytes': (_i64, [_i64, _i64]),
    'bdm_bank_scan': (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _int,
                             _int, _int, _int, _int, _int, _flt, _vp, _vp, _i64, _int, _vp, _i64, _int, _int, _vp,
                             _int, _int, _int, _vp, _vp, _i64, _vp, _int, _vp]),
    'bdm_scan_test_fault': (_int, [_int, ctypes.c_ulonglong]),
    'bdm_bank_scan_chunked': (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int,
                                     _int, _int, _int, _int, _int, _int, _flt, _vp, _vp, _i64, _int, _vp, _i64, _int,
                                     _int, _vp, _int, _int, _int, _vp, _vp, _i64, _vp, _int, _vp]),
    'bdm_decode_token_step': (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _int,
                                     _vp, _vp, _int, _int, _int, _int, _i64, _int, _int, _int, _int, _int, _flt, _vp,
                                     _int, _vp, _vp, _flt, _int, _vp, _vp]),
    'bdm_combine_norm_gate': (_int, [_vp, _vp, _i64, _int, _i64, _vp, _i64, _vp, _vp, _flt, _int, _int, _int, _vp,
                                     _vp]),
    'bdm_combine_norm_gate_save': (_int, [_vp, _vp, _i64, _int, _i64, _vp, _i64, _vp, _vp, _flt, _int, _int, _int,
                                          _vp, _vp, _vp]),
    'bdm_combine_project': (_int, [_vp, _vp, _i64, _int, _i64, _vp, _i64, _vp, _vp, _flt, _int, _int, _vp, _vp,
                                   _i64, _int, _vp, _i64, _vp, _vp]),
    'bdm_combine_project_supported': (_int, [_i64, _i64, _int, _int]),
    'bdm_status_or': (_int, [_vp, _vp, _vp]),
    'bdm_norm_gate_backward_partial_floats': (_i64, [_i64, _i64]),
    'bdm_norm_gate_backward': (_int, [_vp, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _flt, _int, _int, _vp, _vp, _i64,
                                      _vp, _vp, _vp, _vp]),
    'bdm_scan_backward_tiles': (_int, [_int, _int]),
    'bdm_scan_backward_block_events': (_int, [_int, _int]),
    'bdm_scan_backward_checkpoint_bytes': (_i64, [_i64, _i64, _int, _int, _i64, _int, _int, _int]),
    'bdm_scan_backward': (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _int,
                                 _int, _int, _int, _int, _flt, _vp, _vp, _i64, _int, _int, _vp, _vp, _vp, _vp, _vp,
                                 _i64, _int, _vp]),
    'bdm_event_vjp': (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _int, _int,
                             _int, _int, _flt, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    'bdm_product_state_backward': (_int, [_vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _vp]),
    'bdm_route_backward': (_int, [_vp, _i64, _i64, _i64, _i64, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _int, _vp,
                                  _i64, _vp]),
    'bdm_controllers_backward_partial_floats': (_i64, [_i64, _int, _int]),
    'bdm_controllers_backward': (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _vp,
                                        _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, _int, _int, _vp, _i64,
                                        _vp, _vp, _vp, _vp, _vp]),
    'bdm_bank_histogram': (_int, [_vp, _vp, _i64, _int, _int, _i64, _vp, _vp]),
    'bdm_bank_owners': (_int, [_vp, _i64, _int, _int, _vp, _vp, _vp, _vp]),
    'bdm_dispatch_owned_workspace_bytes': (_i64, [_i64, _i64, _int, _int, _i64]),
    'bdm_dispatch_owned': (_int, [_vp, _vp, _i64, _i64, _int, _int, _i64, _vp, _vp, _int, _i64, _vp, _vp, _vp, _vp,
                                  _vp, _vp, _i64, _vp]),
    'bdm_combine_partial': (_int, [_vp, _vp, _i64, _int, _i64, _vp, _i64, _int, _int, _vp, _vp]),
    'bdm_norm_gate_f32': (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _flt, _int, _int, _vp, _vp]),
    'bdm_decode_step': (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, _int, _int, _int,
                               _int, _int, _int, _flt, _vp, _int, _vp, _vp, _i64, _vp, _vp, _flt, _int, _vp, _vp]),
}

_lib = None


class BDMError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f'{LIB_PATH} is missing: build it with `python -m bdm_b200.build` '
                          '(bdm_b200 has no CPU fallback)')
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, name: str) -> None:
    if status == BDM_OK:
        return
    lib = load()
    text = lib.bdm_status_string(status).decode()
    msg = f'{name}: {text}'
    if status == BDM_ERR_CUDA:
        raise BDMError(f'{msg} (cudaError {lib.bdm_last_cuda_error()})')
    if status == BDM_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if status in (BDM_ERR_INVALID, BDM_ERR_DTYPE):
        raise ValueError(msg)
    raise BDMError(msg)
