"""bdm_dispatch_noalloc: the dispatch entry point for callers that cannot allocate.

Code under CUDA graph capture, runtimes that own every device allocation, and
request paths that must not allocate cannot hand the library a workspace.
bdm_dispatch_noalloc sorts with a fixed scratch array inside the library
instead.  This test calls it through the C ABI and checks that its results are
identical to bdm_dispatch (integer outputs: bit-exact) on two calls in a row
with different inputs, so a call cannot depend on what the previous one left in
the shared scratch.  It also checks the size limit is reported, not overrun.
This file is named to run last.
"""
import numpy as np
import pytest
import torch

from bdm_b200 import _lib, near_square_factors

pytestmark = pytest.mark.gpu

DEV = 'cuda'
LIMIT = 32 << 20


def _routes(seed, batch, time, bank_count, selected):
    gen = torch.Generator().manual_seed(seed)
    j1, j2 = near_square_factors(bank_count)
    out = []
    for _ in range(2):  # write banks, read banks: distinct per token, like the router's
        a = torch.randn(batch * time, j1, generator=gen).topk(selected, dim=-1).indices
        b = torch.randn(batch * time, j2, generator=gen).topk(1, dim=-1).indices
        out.append((a * j2 + b).reshape(batch, time, selected).to(DEV))
    return out


def _call(fn, wi, ri, bank_count, workspace=None):
    lib = _lib.load()
    batch, time, kw = wi.shape
    kr = ri.shape[-1]
    e = batch * time * (kw + kr)
    order = torch.full((e,), -1, dtype=torch.int64, device=DEV)
    cu = torch.full((batch * bank_count + 1,), -1, dtype=torch.int64, device=DEV)
    inverse = torch.full((e,), -1, dtype=torch.int64, device=DEV)
    tokens = torch.full((e,), -1, dtype=torch.int64, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    args = [wi.data_ptr(), ri.data_ptr(), batch, time, kw, kr, bank_count, order.data_ptr(), cu.data_ptr(),
            inverse.data_ptr(), tokens.data_ptr(), err.data_ptr()]
    if fn == 'bdm_dispatch':
        nbytes = lib.bdm_dispatch_workspace_bytes(batch, time, kw, kr, bank_count)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        rc = lib.bdm_dispatch(*args, ws.data_ptr(), nbytes, stream)
    else:
        rc = lib.bdm_dispatch_noalloc(*args, stream)
    torch.cuda.synchronize()
    return rc, dict(order=order, cu=cu, inverse=inverse, tokens=tokens, err=err)


@pytest.mark.parametrize('geometry', [(8, 512, 256, 8), (4, 256, 16384, 16)])
def test_noalloc_dispatch_matches_workspace_dispatch_twice(geometry):
    batch, time, bank_count, selected = geometry
    lib = _lib.load()
    assert lib.bdm_dispatch_workspace_bytes(batch, time, selected, selected, bank_count) <= LIMIT
    for call, seed in enumerate((1, 2)):  # second call reuses the scratch the first one left behind
        wi, ri = _routes(seed, batch, time, bank_count, selected)
        rc_ref, ref = _call('bdm_dispatch', wi, ri, bank_count)
        rc, got = _call('bdm_dispatch_noalloc', wi, ri, bank_count)
        assert rc_ref == 0 and rc == 0, (rc_ref, rc)
        for key in ('order', 'cu', 'inverse', 'tokens', 'err'):
            np.testing.assert_array_equal(got[key].cpu().numpy(), ref[key].cpu().numpy(),
                                          err_msg=f'call {call}: {key}')


def test_noalloc_dispatch_rejects_geometry_beyond_fixed_scratch():
    lib = _lib.load()
    batch, time, kw, kr, bank_count = 16, 8192, 16, 16, 16384  # needs ~50 MB of scratch
    assert lib.bdm_dispatch_workspace_bytes(batch, time, kw, kr, bank_count) > LIMIT
    dummy = torch.empty(1, dtype=torch.int64, device=DEV)
    p = dummy.data_ptr()
    rc = lib.bdm_dispatch_noalloc(p, p, batch, time, kw, kr, bank_count, p, p, None, None, None,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.BDM_ERR_WORKSPACE
