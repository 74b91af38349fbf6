"""The C-ABI library loads without a GPU and exports every entry point of include/bdm_b200.h.

Only host-side paths run here (status text, workspace sizing, argument
validation that returns before any CUDA call); nothing launches a kernel.
"""
import ctypes
import os
import re

import pytest

from bdm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, 'include', 'bdm_b200.h')


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r'^BDM_API\s+[\w\s\*]*?\b(bdm_\w+)\s*\(', text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), 'ctypes signatures must mirror the header'


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.bdm_abi_version() == 1
    assert lib.bdm_status_string(0) == b'ok'
    for code in range(1, 6):
        assert lib.bdm_status_string(code) != b'unknown status'


def test_dispatch_workspace_sizing():
    lib = _lib.load()
    small = lib.bdm_dispatch_workspace_bytes(2, 64, 8, 8, 256)
    big = lib.bdm_dispatch_workspace_bytes(16, 8192, 16, 16, 16384)
    assert 0 < small < big
    assert lib.bdm_dispatch_workspace_bytes(0, 64, 8, 8, 256) == -1


@pytest.mark.parametrize('call', [
    lambda lib: lib.bdm_route(None, -1, 32, 16, 16, 8, 1, None, None, None),
    lambda lib: lib.bdm_route(None, 4, 8, 16, 16, 8, 1, None, None, None),        # ld < j1 + j2
    lambda lib: lib.bdm_dispatch(None, None, 2, 4, 8, 8, 256, None, None, None, None, None, None, 0, None),
    lambda lib: lib.bdm_combine_norm_gate(None, None, 4, 8, 0, None, 0, None, None, 1e-5, 1, 0, 1, None, None),
    lambda lib: lib.bdm_status_or(None, None, None),                                  # null words
    lambda lib: lib.bdm_bank_owners(None, 256, 4, 1, None, None, None, None),          # balanced needs counts
    lambda lib: lib.bdm_bank_owners(None, 256, 0, 0, None, None, None, None),          # world 0
    lambda lib: lib.bdm_dispatch_owned(None, None, 2, 4, 8, 8, 256, None, None, 0, 64, None, None, None, None, None,
                                       None, 0, None),
    lambda lib: lib.bdm_combine_partial(None, None, 4, 8, 64, None, 256, 0, 1, None, None),
    lambda lib: lib.bdm_norm_gate_f32(None, 4, 64, None, 64, None, None, 1e-5, 1, 1, None, None),
    lambda lib: lib.bdm_combine_norm_gate_save(None, None, 4, 8, 64, None, 64, None, None, 1e-5, 1, 0, 1, None, None,
                                               None),
    lambda lib: lib.bdm_combine_project(None, None, 4, 8, 1024, None, 1000, None, None, 1e-5, 1, 0, None, None,
                                        1024, 1, None, 1024, None, None),                  # ld_gate < width
    lambda lib: lib.bdm_combine_project(None, None, 4, 8, 1024, None, 1024, None, None, 1e-5, 1, 0, None, None,
                                        1024, 1, None, 1024, None, None),                  # null inputs
    lambda lib: lib.bdm_norm_gate_backward(None, None, 4, 64, None, 32, None, None, 1e-5, 1, 1, None, None, 64, None,
                                           None, None, None),                          # ld_gate < width
    lambda lib: lib.bdm_scan_backward(*([None] * 10), 2, 4, 16, 1, 8, 32, 4, 4, 1, 1, 0.35, None, None, 0, 0, 0,
                                      *([None] * 5), 0, 0, None),                      # null inputs
    lambda lib: lib.bdm_event_vjp(*([None] * 10), 4, 1, 8, 32, 4, 4, 1, 1, 0.35, *([None] * 8), None),
    lambda lib: lib.bdm_product_state_backward(None, 2, 0, 4, 32, 1, None, None, None, None),
    lambda lib: lib.bdm_route_backward(None, 4, 32, 0, 4, 4, 4, 4, 1, None, None, None, None, 1, None, 32, None),
    lambda lib: lib.bdm_controllers_backward(None, 4, 64, 0, 8, 16, 48, 56, None, 8, *([None] * 11), 1, 8, 32, 0,
                                             1, None, 64, None, None, None, None, None),  # col_w + V > ld
])
def test_invalid_arguments_are_rejected_on_the_host(call):
    assert call(_lib.load()) == _lib.BDM_ERR_INVALID


def test_bank_partition_limits():
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    # every rank must get the same number of banks
    assert lib.bdm_bank_owners(dummy, 250, 4, 0, dummy, dummy, dummy, None) == _lib.BDM_ERR_UNSUPPORTED
    # the balanced partition sorts the table in one CTA: at most 16384 banks and 32 ranks
    assert lib.bdm_bank_owners(dummy, 32768, 8, 1, dummy, dummy, dummy, None) == _lib.BDM_ERR_UNSUPPORTED
    assert lib.bdm_bank_owners(dummy, 16384 * 2, 64, 1, dummy, dummy, dummy, None) == _lib.BDM_ERR_UNSUPPORTED
    assert lib.bdm_dispatch_owned_workspace_bytes(16, 8192, 16, 16, 2048) > 0
    assert lib.bdm_dispatch_owned_workspace_bytes(16, 8192, 16, 16, 0) == -1


def test_unsupported_geometry_is_reported():
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    rc = lib.bdm_bank_scan(*([dummy] * 12), 1, 4, 16, 1, 32, 64, 8, 8, 1, 1, 0.25, None, None, 0, 0, None, 0, 0, 0,
                           None, 0, 0, 0, dummy, dummy, 1 << 20, None, 0, None)
    assert rc == _lib.BDM_ERR_UNSUPPORTED  # bank_size 32 is not implemented
    with pytest.raises(NotImplementedError):
        _lib.check(rc, 'bdm_bank_scan')


def test_backward_sizing_and_limits():
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    small = lib.bdm_scan_backward_checkpoint_bytes(2, 64, 8, 8, 64, 1, 8, 32)
    assert 0 < small < lib.bdm_scan_backward_checkpoint_bytes(32, 2048, 8, 8, 512, 12, 8, 64)
    assert lib.bdm_scan_backward_checkpoint_bytes(2, 64, 8, 8, 64, 1, 6, 32) == -1   # bank_size 4, 8 or 16
    # one warp per 64 value columns for S <= 8 and dv >= 64, else per 32
    assert [lib.bdm_scan_backward_tiles(8, d) for d in (16, 32, 64, 128)] == [1, 1, 1, 2]
    assert [lib.bdm_scan_backward_tiles(16, d) for d in (32, 64, 128)] == [1, 2, 4]
    assert lib.bdm_scan_backward_tiles(6, 64) == -1
    assert lib.bdm_norm_gate_backward_partial_floats(33, 64) == 2 * 3 * 64
    assert lib.bdm_controllers_backward_partial_floats(65, 2, 8) == (2 * 2 + 1) * 16
    # head value width above 8 columns per lane, more selected banks than a route warp's lanes
    assert lib.bdm_event_vjp(*([dummy] * 10), 4, 2, 8, 512, 4, 4, 1, 1, 0.35, *([dummy] * 8), None) \
        == _lib.BDM_ERR_UNSUPPORTED
    assert lib.bdm_route_backward(dummy, 4, 200, 0, 100, 10, 10, 40, 1, dummy, dummy, dummy, dummy, 1, dummy, 200,
                                  None) == _lib.BDM_ERR_UNSUPPORTED
    # checkpoint scratch below the required size
    assert lib.bdm_scan_backward(*([dummy] * 10), 2, 4, 16, 1, 8, 32, 4, 4, 1, 1, 0.35, None, None, 0, 0, 0, dummy,
                                 dummy, dummy, dummy, dummy, 16, 0, None) == _lib.BDM_ERR_WORKSPACE
    # checkpoint blocks: 128 / (S * columns per lane) events
    assert [lib.bdm_scan_backward_block_events(8, d) for d in (32, 64)] == [16, 8]
    assert lib.bdm_scan_backward_block_events(16, 128) == 8 and lib.bdm_scan_backward_block_events(5, 64) == -1
    # a training forward's checkpoints need the whole-layer, factor-initialised form
    assert lib.bdm_bank_scan(*([dummy] * 12), 1, 4, 16, 1, 8, 64, 8, 8, 1, 1, 0.35, None, None, 0, 0, None, 0, 0, 0,
                             dummy, 1, 0, 0, dummy, dummy, 1 << 20, dummy, 8, None) == _lib.BDM_ERR_INVALID


def test_scan_test_fault_validates_its_flag():
    lib = _lib.load()
    assert lib.bdm_scan_test_fault(2, 0) == _lib.BDM_ERR_INVALID
    assert lib.bdm_scan_test_fault(0, 0) == _lib.BDM_OK


def test_combine_project_geometry_is_reported_without_a_launch():
    lib = _lib.load()
    bf, f32 = _lib.BDM_BF16, _lib.BDM_F32
    assert lib.bdm_combine_project_supported(1024, 1024, 8, bf) == 1   # c2
    assert lib.bdm_combine_project_supported(768, 768, 8, bf) == 1     # c5
    assert lib.bdm_combine_project_supported(512, 128, 16, bf) == 1
    for args in ((2048, 2048, 16, bf), (1024, 1024, 8, f32), (1024, 1088, 8, bf), (1024, 2048, 8, bf),
                 (256, 256, 8, bf), (640, 256, 8, bf), (1024, 1024, 0, bf), (1024, 1024, 17, bf)):
        assert lib.bdm_combine_project_supported(*args) == 0, args
    dummy = ctypes.c_void_p(16)
    # a geometry the kernel does not take is reported before any device work (c4: V = 2048)
    assert lib.bdm_combine_project(dummy, dummy, 4, 16, 2048, dummy, 2048, dummy, None, 1e-5, 1, 0, dummy, None, 2048,
                                   bf, dummy, 2048, None, None) == _lib.BDM_ERR_UNSUPPORTED
    assert lib.bdm_combine_project(None, None, 0, 8, 1024, None, 1024, None, None, 1e-5, 1, 0, None, None, 1024, bf,
                                   None, 1024, None, None) == _lib.BDM_OK  # no tokens: nothing to do
