"""ctypes binding of the C oracle (bdm_oracle.c) -- TEST INFRASTRUCTURE ONLY.

All arrays are NumPy, float32 for floating point (holding BF16-representable
values when ``bf16`` is set) and int64 for indices.  Each wrapper cites the
reference function it restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, '_build', 'libbdm_oracle.so')
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags='C_CONTIGUOUS')
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags='C_CONTIGUOUS')
_i64 = ctypes.c_int64
_int = ctypes.c_int
_flt = ctypes.c_float


def build() -> str:
    """Compile bdm_oracle.c with its Makefile (no-op when up to date)."""
    subprocess.run(['make', '-s', '-C', _HERE], check=True)
    return _LIB_PATH


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
            os.path.join(_HERE, 'bdm_oracle.c')):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    lib.oracle_route.argtypes = [_f32p, _i64, _int, _int, _int, _int, _i64p, _f32p]
    lib.oracle_dispatch.argtypes = [_i64p, _i64p, _i64, _i64, _int, _int, _i64, _i64p, _i64p, _i64p, _i64p]
    lib.oracle_recurrence.argtypes = [_f32p] * 6 + [_i64p, _f32p, _i64p, _f32p, _f32p, _i64, _i64, _i64, _i64,
                                                    _int, _int, _int, _int, _int, _int, _int, _int, _flt, _f32p,
                                                    ctypes.c_void_p]
    lib.oracle_combine.argtypes = [_f32p, _i64p, _i64, _int, _i64, _int, _int, _f32p]
    lib.oracle_decode_step.argtypes = [_f32p] * 6 + [_i64p, _f32p, _i64p, _f32p, _f32p, _i64, _i64, _int, _int,
                                                     _int, _int, _int, _int, _int, _int, _flt, _f32p]
    lib.oracle_bf16_round.argtypes = [_flt]
    lib.oracle_bf16_round.restype = _flt
    lib.oracle_set_threads.argtypes = [_int]
    lib.oracle_set_threads.restype = _int
    for name in ('oracle_route', 'oracle_dispatch', 'oracle_recurrence', 'oracle_combine', 'oracle_decode_step'):
        getattr(lib, name).restype = _int
    _lib = lib
    return lib


def set_threads(n: int = 0) -> int:
    """Thread count for the C oracle; 0 means every online core."""
    return load().oracle_set_threads(int(n))


def _check(rc: int, name: str):
    if rc != 0:
        raise ValueError(f'{name} failed with status {rc}')


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


def _i64a(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.int64)


def bf16_round(x) -> np.ndarray:
    """Round-to-nearest-even to BF16, returned as float32 (torch ``.to(bfloat16)``)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    special = (u & 0x7F800000) == 0x7F800000
    finite = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    nan_fix = (u & np.uint32(0xFFFF0000)) | np.where((u & 0x7FFFFF) != 0, np.uint32(0x400000), np.uint32(0))
    out = np.where(special, nan_fix, finite).astype(np.uint32)
    return out.view(np.float32).reshape(x.shape)


def oracle_route(logits, *, bank_count: int, selected_banks: int, bf16: bool, factors=None):
    """product_key_route (gdn2_banks.py:74-114) with lower-index tie breaking.

    logits [..., J1+J2] -> (weights [..., count] float32, indices [..., count] int64).
    """
    from .layer import near_square_factors
    j1, j2 = factors or near_square_factors(bank_count)
    z = _f32(logits)
    if z.shape[-1] != j1 + j2:
        raise ValueError('projected route width does not match the bank table')
    lead = z.shape[:-1]
    ntok = int(np.prod(lead)) if lead else 1
    sub = min(selected_banks, j1, j2)
    count = min(selected_banks, sub * sub)
    idx = np.empty((ntok, count), np.int64)
    w = np.empty((ntok, count), np.float32)
    _check(load().oracle_route(z.reshape(ntok, j1 + j2), ntok, j1, j2, selected_banks, int(bf16), idx, w),
           'oracle_route')
    return w.reshape(*lead, count), idx.reshape(*lead, count)


def oracle_dispatch(wi, ri, bank_count: int):
    """pack_bank_events ordering (gdn2_banks.py:174-185,237-246).

    wi [B,T,KW], ri [B,T,KR] -> dict(order, inverse, tokens, cu_seqlens), all int64.
    """
    wi, ri = _i64a(wi), _i64a(ri)
    batch, time, kw = wi.shape
    kr = ri.shape[-1]
    e = batch * time * (kw + kr)
    order, inverse, tokens = (np.empty(e, np.int64) for _ in range(3))
    cu = np.empty(batch * bank_count + 1, np.int64)
    _check(load().oracle_dispatch(wi, ri, batch, time, kw, kr, bank_count, order, inverse, tokens, cu),
           'oracle_dispatch')
    return dict(order=order, inverse=inverse, tokens=tokens, cu_seqlens=cu)


def oracle_recurrence(q, k, v, g, b, w, wi, ww, ri, rw, init, *, bank_count: int, bf16: bool,
                      routed_decay: bool, interval: int, scale: float, want_state: bool = True):
    """Route-weighted packing + reference_packed_gdn2 (gdn2_banks.py:22-43,196-224).

    q,k,g,b [B,T,H,S]; v,w [B,T,H,dv]; wi,ww [B,T,KW]; ri,rw [B,T,KR];
    init [1 or B, J, H, S, dv].  Returns (reads [B,T,KR,H*dv], final_state [B,J,H,S,dv] or None).
    """
    q, k, v, g, b, w = (_f32(x) for x in (q, k, v, g, b, w))
    batch, time, heads, s = q.shape
    dv = v.shape[-1]
    kw, kr = wi.shape[-1], ri.shape[-1]
    init = _f32(init)
    reads = np.zeros((batch, time, kr, heads * dv), np.float32)
    final = np.zeros((batch, bank_count, heads, s, dv), np.float32) if want_state else None
    _check(load().oracle_recurrence(q, k, v, g, b, w, _i64a(wi), _f32(ww), _i64a(ri), _f32(rw), init,
                                    init.shape[0], batch, time, bank_count, heads, s, dv, kw, kr, int(bf16),
                                    int(routed_decay), int(interval), float(scale), reads,
                                    final.ctypes.data if final is not None else None), 'oracle_recurrence')
    return reads, final


def oracle_combine(reads, ri, *, bf16: bool, round_each: bool = False):
    """Read combine in ascending bank order: reads [..., KR, V] -> [..., V].

    round_each=False: FP32 accumulation, one rounding (CPU scatter_bank_outputs,
    gdn2_banks.py:265-283).  round_each=True: rounding after every add (GPU
    readouts, role_bank_dispatch.py:201-216, inference.py:53-85).
    """
    reads = _f32(reads)
    ri = _i64a(ri)
    kr, width = reads.shape[-2], reads.shape[-1]
    lead = reads.shape[:-2]
    ntok = int(np.prod(lead)) if lead else 1
    raw = np.empty((ntok, width), np.float32)
    _check(load().oracle_combine(reads.reshape(ntok, kr, width), ri.reshape(ntok, kr), ntok, kr, width, int(bf16),
                                 int(round_each), raw), 'oracle_combine')
    return raw.reshape(*lead, width)


def oracle_decode_step(q, k, v, g, b, w, wi, ww, ri, rw, state, *, bf16: bool, cache_bf16: bool,
                       routed_decay: bool, scale: float):
    """inference.step bank part (inference.py:21-67,161-194); updates ``state`` in place.

    q,k,g,b [B,H,S]; v,w [B,H,dv]; routes [B,K]; state [B,J,H,S,dv] float32 (C-contiguous).
    Returns raw [B, H*dv].
    """
    if state.dtype != np.float32 or not state.flags['C_CONTIGUOUS']:
        raise ValueError('state must be a C-contiguous float32 array')
    q, k, v, g, b, w = (_f32(x) for x in (q, k, v, g, b, w))
    batch, heads, s = q.shape
    dv = v.shape[-1]
    bank_count = state.shape[1]
    kw, kr = wi.shape[-1], ri.shape[-1]
    raw = np.empty((batch, heads * dv), np.float32)
    _check(load().oracle_decode_step(q, k, v, g, b, w, _i64a(wi), _f32(ww), _i64a(ri), _f32(rw), state, batch,
                                     bank_count, heads, s, dv, kw, kr, int(bf16), int(cache_bf16),
                                     int(routed_decay), float(scale), raw), 'oracle_decode_step')
    return raw
