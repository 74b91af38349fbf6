"""CUDA path vs the CPU oracle (and the reference's golden vectors), through the C ABI.

Bit-exact: routing indices, dispatch order / cu_seqlens / inverse / tokens.
Floating point, max-relative error max|a-b| / max|b|:
  FP32 runs            1e-4   (north star: "within 1e-4 against an FP32 run")
  BF16 runs            2e-2   (north star: "2e-2 max-relative error in BF16")
"""
import os

import numpy as np
import pytest
import torch

import oracle
from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory, _lib, near_square_factors, ops, state_interval

pytestmark = pytest.mark.gpu

DEV = 'cuda'
FP32_TOL, BF16_TOL = 1e-4, 2e-2


def npf(t):
    return t.detach().float().cpu().numpy()


def max_rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _logits(gen, ntok, width, dtype, ties=False):
    if ties:
        return torch.randint(-3, 4, (ntok, width), generator=gen).to(dtype)
    return torch.randn(ntok, width, generator=gen).to(dtype)


# ------------------------------------------------------------------ router
@pytest.mark.parametrize('bank_count,selected', [(256, 8), (2048, 8), (16384, 16), (64, 4), (512, 8)])
@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
@pytest.mark.parametrize('ties', [False, True])
def test_router_bit_exact(bank_count, selected, dtype, ties):
    gen = torch.Generator().manual_seed(bank_count + selected + int(ties))
    j1, j2 = near_square_factors(bank_count)
    z = _logits(gen, 3000, j1 + j2, dtype, ties)
    w, i = ops.route(z.to(DEV), bank_count=bank_count, selected_banks=selected)
    ow, oi = oracle.oracle_route(npf(z), bank_count=bank_count, selected_banks=selected,
                                 bf16=dtype == torch.bfloat16)
    np.testing.assert_array_equal(i.cpu().numpy(), oi)
    if dtype == torch.bfloat16:
        # the softmax sum order differs (warp tree vs sequential): at most one BF16 ulp
        assert np.abs(npf(w) - ow).max() <= 2 ** -8
    else:
        np.testing.assert_allclose(npf(w), ow, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_route_pair_equals_two_routes(dtype):
    gen = torch.Generator().manual_seed(17)
    bank_count, selected = 2048, 8
    j1, j2 = near_square_factors(bank_count)
    proj = torch.randn(700, 40 + 2 * (j1 + j2) + 13, generator=gen).to(dtype).to(DEV)
    first, second = 40, 40 + j1 + j2
    (w1, i1), (w2, i2) = ops.route_pair(proj, first, second, bank_count=bank_count, selected_banks=selected)
    rw1, ri1 = ops.route(proj[:, first:first + j1 + j2], bank_count=bank_count, selected_banks=selected)
    rw2, ri2 = ops.route(proj[:, second:second + j1 + j2], bank_count=bank_count, selected_banks=selected)
    for a, b in ((w1, rw1), (i1, ri1), (w2, rw2), (i2, ri2)):
        assert torch.equal(a, b)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_controllers_in_kernel_f_proj(dtype):
    # f_proj.1 computed in the controllers kernel (few tokens) vs the GEMM path
    cfg = dict(dim=256, bank_count=256, bank_size=8, selected_banks=8, value_width=512, num_heads=4)
    m = BlockSparseDeltaMemory(BSDMConfig(**cfg), seed=9).to(dtype).to(DEV)
    x = torch.randn(64, 256, generator=torch.Generator().manual_seed(2)).to(dtype).to(DEV)
    with torch.no_grad():
        proj, cols = m._project(x)
        f = torch.mm(proj[:, cols['f']:cols['f'] + m.head_value_width], m.f_proj[1].weight.t())
        kw = dict(heads=m.num_heads, bank_size=m.bank_size, head_value_width=m.head_value_width,
                  qk_norm=m.config.qk_normalization)
        a = ops.controllers(proj, cols, f, m.A_log, m.dt_bias, **kw)
        b = ops.controllers(proj, cols, None, m.A_log, m.dt_bias, **kw, f_weight=m.f_proj[1].weight,
                            f1_width=m.head_value_width)
    for i in (0, 1, 2, 4, 5):  # q, k, v, b, w do not depend on f
        assert torch.equal(a[i], b[i])
    # f's FP32 accumulation order differs from the GEMM's: at most one ulp of f apart
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert max_rel(npf(b[3]), npf(a[3])) <= tol


def test_router_strided_logits_and_golden(golden_dir):
    data = torch.load(os.path.join(golden_dir, 'router.pt'), weights_only=False)
    for case in data['cases']:
        if case['kind'] != 'random' or case['logits'].dtype != torch.float32:
            continue
        z = case['logits'][0]
        wide = torch.zeros(z.shape[0], z.shape[1] + 40, dtype=z.dtype)
        wide[:, 24:24 + z.shape[1]] = z
        w, i = ops.route(wide.to(DEV)[:, 24:24 + z.shape[1]], bank_count=case['bank_count'],
                         selected_banks=case['selected'])
        ref_i = case['indices'][0]
        agree = (i.cpu() == ref_i).all(-1).float().mean().item()
        assert agree > 0.99, agree  # FP32 ties are vanishingly rare
        ow, oi = oracle.oracle_route(npf(z), bank_count=case['bank_count'], selected_banks=case['selected'],
                                     bf16=False)
        np.testing.assert_array_equal(i.cpu().numpy(), oi)


# ----------------------------------------------------------------- dispatch
def _random_routes(gen, batch, time, bank_count, selected):
    j1, j2 = near_square_factors(bank_count)
    wl = torch.randn(batch * time, j1 + j2, generator=gen)
    rl = torch.randn(batch * time, j1 + j2, generator=gen)
    ww, wi = oracle.oracle_route(wl.numpy(), bank_count=bank_count, selected_banks=selected, bf16=False)
    rw, ri = oracle.oracle_route(rl.numpy(), bank_count=bank_count, selected_banks=selected, bf16=False)
    shape = (batch, time, -1)
    return (torch.from_numpy(ww).reshape(shape), torch.from_numpy(wi).reshape(shape),
            torch.from_numpy(rw).reshape(shape), torch.from_numpy(ri).reshape(shape))


@pytest.mark.parametrize('batch,time,bank_count,selected', [
    (8, 4096, 256, 8),       # c2 geometry: one 11-bit pass
    (16, 512, 16384, 16),    # c4 bank table: two passes
    (2, 512, 256, 8),        # c1
    (64, 16, 131072, 2),     # 23-bit sequence ids: three passes
    (3, 5, 16, 2),           # ragged tiny
])
def test_dispatch_bit_exact(batch, time, bank_count, selected):
    gen = torch.Generator().manual_seed(batch * 7 + time)
    ww, wi, rw, ri = _random_routes(gen, batch, time, bank_count, selected)
    out = ops.dispatch(wi.to(DEV), ri.to(DEV), bank_count, want_inverse=True, want_tokens=True)
    ref = oracle.oracle_dispatch(wi.numpy(), ri.numpy(), bank_count)
    for key in ('order', 'cu_seqlens', 'inverse', 'tokens'):
        np.testing.assert_array_equal(out[key].cpu().numpy(), ref[key], err_msg=key)


def test_dispatch_edge_cases_and_golden(golden_dir):
    # every event in one bank: a single maximal sequence per batch row
    wi = torch.zeros(2, 300, 3, dtype=torch.long)
    ri = torch.zeros(2, 300, 3, dtype=torch.long)
    out = ops.dispatch(wi.to(DEV), ri.to(DEV), 64, want_inverse=True, want_tokens=True)
    ref = oracle.oracle_dispatch(wi.numpy(), ri.numpy(), 64)
    for key in ('order', 'cu_seqlens', 'inverse', 'tokens'):
        np.testing.assert_array_equal(out[key].cpu().numpy(), ref[key], err_msg=key)
    # out-of-range banks are counted, never written out of bounds
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    bad = torch.tensor([[[0, 70]]], dtype=torch.long)
    out = ops.dispatch(bad.to(DEV), torch.tensor([[[1, -3]]]).to(DEV), 64, error_word=err)
    torch.cuda.synchronize()
    assert err.item() == 2
    assert sorted(out['order'].cpu().tolist()) == [0, 1, 2, 3]
    for case in torch.load(os.path.join(golden_dir, 'dispatch.pt'), weights_only=False)['cases']:
        out = ops.dispatch(case['wi'].to(DEV), case['ri'].to(DEV), case['bank_count'], want_tokens=True)
        np.testing.assert_array_equal(out['order'].cpu().numpy(), case['order'].numpy())
        np.testing.assert_array_equal(out['cu_seqlens'].cpu().numpy(), case['cu_seqlens'].numpy())
        np.testing.assert_array_equal(out['tokens'].cpu().numpy(), case['tokens'].numpy())


# -------------------------------------------------------------- recurrence
def _controls(gen, nt, heads, s, dv, dtype, decay=0.3):
    q = torch.nn.functional.normalize(torch.randn(nt, heads, s, generator=gen), dim=-1).to(dtype)
    k = torch.nn.functional.normalize(torch.randn(nt, heads, s, generator=gen), dim=-1).to(dtype)
    v = torch.randn(nt, heads * dv, generator=gen).to(dtype)
    g = -torch.rand(nt, heads, s, generator=gen) * decay
    b = torch.rand(nt, heads, s, generator=gen).to(dtype)
    w = torch.rand(nt, heads * dv, generator=gen).to(dtype)
    return q.reshape(nt, -1), k.reshape(nt, -1), v, g.reshape(nt, -1), b.reshape(nt, -1), w


def _run_scan(batch, time, bank_count, selected, heads, s, dv, dtype, *, interval, routed, cache_dtype=None,
              seed=0, decay=0.3, chunked=False):
    gen = torch.Generator().manual_seed(seed)
    nt = batch * time
    ctl = _controls(gen, nt, heads, s, dv, dtype, decay)
    ww, wi, rw, ri = _random_routes(gen, batch, time, bank_count, selected)
    ww, rw = ww.to(dtype), rw.to(dtype)
    rows, cols = near_square_factors(bank_count * heads * s)
    u = (0.05 * torch.randn(rows, dv, generator=gen)).to(dtype)
    z = (0.05 * torch.randn(cols, dv, generator=gen)).to(dtype)
    meta = ops.dispatch(wi.to(DEV), ri.to(DEV), bank_count)
    args = [t.to(DEV) for t in ctl] + [wi.to(DEV), ww.to(DEV), ri.to(DEV), rw.to(DEV), meta['order'],
                                       meta['cu_seqlens']]
    init = npf(u)[:, None, :] + npf(z)[None, :, :]
    init = (oracle.bf16_round(init) if dtype == torch.bfloat16 else init).reshape(bank_count, heads, s, dv)
    kw = dict(batch=batch, time=time, bank_count=bank_count, heads=heads, bank_size=s, head_value_width=dv,
              routed_decay=routed, scale=s ** -0.5)
    if cache_dtype is None:
        reads = ops.bank_scan(*args, **kw, row_factor=u.to(DEV), col_factor=z.to(DEV), state_interval=interval,
                              check_status=True, chunked=chunked)
        final = None
        init_b = init[None]
    else:
        cache = torch.from_numpy(np.broadcast_to(init, (batch,) + init.shape).copy()).to(cache_dtype).to(DEV)
        init_b = npf(cache)
        reads = ops.bank_scan(*args, **kw, cache=cache, store_final=True, state_interval=interval,
                              check_status=True, chunked=chunked)
        final = cache
    q, k, v, g, b, w = (npf(t) for t in ctl)
    sh = lambda x, last: x.reshape(batch, time, heads, last)
    oreads, ofinal = oracle.oracle_recurrence(sh(q, s), sh(k, s), sh(v, dv), sh(g, s), sh(b, s), sh(w, dv),
                                              wi.numpy(), npf(ww), ri.numpy(), npf(rw), init_b,
                                              bank_count=bank_count, bf16=dtype == torch.bfloat16,
                                              routed_decay=routed, interval=interval, scale=s ** -0.5)
    return npf(reads).reshape(oreads.shape), oreads, (npf(final) if final is not None else None), ofinal


@pytest.mark.parametrize('s,dv,heads', [(8, 128, 1), (8, 64, 2), (4, 128, 1), (16, 128, 2), (8, 128, 3)])
@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_bank_scan_forward(s, dv, heads, dtype):
    interval = state_interval(s) if dtype == torch.bfloat16 else 0
    ours, ref, _, _ = _run_scan(2, 200, 64, 4, heads, s, dv, dtype, interval=interval, routed=True, seed=s + dv)
    tol = BF16_TOL if dtype == torch.bfloat16 else FP32_TOL
    assert max_rel(ours, ref) <= tol, max_rel(ours, ref)


@pytest.mark.parametrize('s,dv,heads', [(16, 128, 2), (8, 128, 1), (8, 192, 1), (16, 192, 1), (4, 64, 2)])
@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_bank_scan_long_sequences(s, dv, heads, dtype):
    # 4 banks, 2 per role: every (batch, bank) sequence has ~2600 events, so the
    # sequences run on the warp-specialised (producer / consumer warps) path
    interval = state_interval(s) if dtype == torch.bfloat16 else 0
    ours, ref, _, _ = _run_scan(2, 2600, 4, 2, heads, s, dv, dtype, interval=interval, routed=True, seed=11 + s)
    tol = BF16_TOL if dtype == torch.bfloat16 else FP32_TOL
    assert max_rel(ours, ref) <= tol, max_rel(ours, ref)


@pytest.mark.parametrize('cache_dtype', [torch.float32, torch.bfloat16])
def test_bank_scan_long_sequences_prefill_and_decay_cuts(cache_dtype):
    # strong decays: the cumulative log-decay crosses the -60 floor inside batches,
    # so batches are cut short and the staging restarts mid-batch
    for dtype in (torch.float32, torch.bfloat16):
        ours, ref, final, ofinal = _run_scan(1, 2400, 4, 2, 2, 16, 128, dtype, interval=0, routed=True,
                                             cache_dtype=cache_dtype, seed=5, decay=12.0)
        tol = BF16_TOL if dtype == torch.bfloat16 else FP32_TOL
        assert max_rel(ours, ref) <= tol, max_rel(ours, ref)
        ofinal_c = oracle.bf16_round(ofinal) if cache_dtype == torch.bfloat16 else ofinal
        assert max_rel(final.reshape(ofinal_c.shape), ofinal_c) <= (tol if cache_dtype == torch.float32 else BF16_TOL)


@pytest.mark.parametrize('cache_dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_bank_scan_prefill_final_state(cache_dtype, dtype):
    ours, ref, final, ofinal = _run_scan(3, 150, 256, 8, 1, 8, 128, dtype, interval=0, routed=True,
                                         cache_dtype=cache_dtype, seed=7)
    tol = BF16_TOL if dtype == torch.bfloat16 else FP32_TOL
    assert max_rel(ours, ref) <= tol
    ofinal_c = oracle.bf16_round(ofinal) if cache_dtype == torch.bfloat16 else ofinal
    assert max_rel(final.reshape(ofinal_c.shape), ofinal_c) <= (tol if cache_dtype == torch.float32 else BF16_TOL)


def test_bank_scan_plain_decay_and_fp32_against_golden(golden_dir):
    # routed_decay=False path
    ours, ref, _, _ = _run_scan(2, 100, 64, 4, 1, 8, 128, torch.float32, interval=0, routed=False, seed=3)
    assert max_rel(ours, ref) <= FP32_TOL
    # the reference's own serial equation oracle (FP32)
    case = torch.load(os.path.join(golden_dir, 'recurrence.pt'), weights_only=False)['cases'][0]
    batch, time, J, s, dv = case['batch'], case['time'], case['bank_count'], case['bank_size'], case['dv']
    nt = batch * time
    meta = ops.dispatch(case['wi'].to(DEV), case['ri'].to(DEV), J)
    ctl = [case[n].reshape(nt, -1).float().to(DEV) for n in 'qkvgbw']
    cache = case['init'].float().unsqueeze(0).expand(batch, -1, -1, -1).contiguous().to(DEV)
    reads = ops.bank_scan(*ctl, case['wi'].to(DEV), case['ww'].float().to(DEV), case['ri'].to(DEV),
                          case['rw'].float().to(DEV), meta['order'], meta['cu_seqlens'], batch=batch, time=time,
                          bank_count=J, heads=1, bank_size=s, head_value_width=dv, routed_decay=True,
                          scale=s ** -0.5, cache=cache, store_final=True)
    out = reads.reshape(batch, time, -1, dv).sum(2)  # FP32: summation order is within tolerance
    assert max_rel(npf(out), npf(case['serial_out'])) <= FP32_TOL
    assert max_rel(npf(cache), npf(case['serial_state'])) <= FP32_TOL


def test_bank_scan_c2_full_size_bf16():
    """c2 geometry (8 x 4096 tokens, H=8, S=8, dv=128, J=256, B=8) against the oracle."""
    ours, ref, _, _ = _run_scan(8, 4096, 256, 8, 8, 8, 128, torch.bfloat16, interval=16, routed=True, seed=11)
    assert max_rel(ours, ref) <= BF16_TOL, max_rel(ours, ref)
    assert np.mean(ours == ref) > 0.5


# ------------------------------------------------- tensor-core chunked recurrence
@pytest.mark.parametrize('s,heads', [(8, 1), (8, 2), (4, 1), (4, 2), (16, 1), (16, 2), (8, 3)])
def test_bank_scan_chunked_matches_oracle(s, heads):
    # training storage policy (BF16 state rounded every C = 16 / 8 events, the chunk length)
    ours, ref, _, _ = _run_scan(2, 200, 64, 4, heads, s, 128, torch.bfloat16, interval=state_interval(s),
                                routed=True, seed=40 + s + heads, chunked=True)
    assert max_rel(ours, ref) <= BF16_TOL, max_rel(ours, ref)


@pytest.mark.parametrize('cache_dtype', [torch.float32, torch.bfloat16])
def test_bank_scan_chunked_prefill_final_state_and_strong_decay(cache_dtype):
    # prefill policy (no rounding until the cache store), two column tiles (dv = 256), and decays
    # strong enough that chunks exceed the split pair factor's range (the direct exp path)
    for decay, seed in ((0.3, 7), (40.0, 8)):
        ours, ref, final, ofinal = _run_scan(3, 150, 64, 8, 2, 8, 256, torch.bfloat16, interval=0, routed=True,
                                             cache_dtype=cache_dtype, seed=seed, decay=decay, chunked=True)
        assert max_rel(ours, ref) <= BF16_TOL, (decay, max_rel(ours, ref))
        ofinal_c = oracle.bf16_round(ofinal) if cache_dtype == torch.bfloat16 else ofinal
        assert max_rel(final.reshape(ofinal_c.shape), ofinal_c) <= BF16_TOL


def test_bank_scan_chunked_c2_full_size():
    """c2 geometry (8 x 4096 tokens, H=8, S=8, dv=128, J=256, B=8) against the oracle."""
    ours, ref, _, _ = _run_scan(8, 4096, 256, 8, 8, 8, 128, torch.bfloat16, interval=16, routed=True, seed=11,
                                chunked=True)
    assert max_rel(ours, ref) <= BF16_TOL, max_rel(ours, ref)


def test_bank_scan_chunked_rejects_unsupported():
    gen = torch.Generator().manual_seed(0)
    for dtype, dv, interval in ((torch.float32, 128, 0), (torch.bfloat16, 64, 16), (torch.bfloat16, 128, 4)):
        ctl = [t.to(DEV) for t in _controls(gen, 32, 1, 8, dv, dtype)]
        ww, wi, rw, ri = _random_routes(gen, 1, 32, 16, 2)
        meta = ops.dispatch(wi.to(DEV), ri.to(DEV), 16)
        with pytest.raises(NotImplementedError):
            ops.bank_scan(*ctl, wi.to(DEV), ww.to(dtype).to(DEV), ri.to(DEV), rw.to(dtype).to(DEV), meta['order'],
                          meta['cu_seqlens'], batch=1, time=32, bank_count=16, heads=1, bank_size=8,
                          head_value_width=dv, routed_decay=True, scale=8 ** -0.5, state_interval=interval,
                          chunked=True)


def test_scan_status_is_sticky_and_polled_without_blocking():
    dev = torch.device(DEV, torch.cuda.current_device())
    ops._SCAN_STATUS.pop(dev.index, None)
    with torch.inference_mode():  # first use under inference_mode, later use outside it
        _run_scan(1, 32, 16, 2, 1, 8, 128, torch.bfloat16, interval=16, routed=True, seed=1)
    ops.reset_scan_status(dev)
    _run_scan(1, 64, 16, 2, 1, 8, 128, torch.bfloat16, interval=16, routed=True, seed=2)
    assert ops.scan_status(dev, wait=True) == 0
    ops.check_scan_status(dev)
    # a launch's error bits (set here by hand: a wait that gave up) stay until reset; the
    # non-blocking poll reports them once its snapshot has reached the host
    ops._scan_status_of(dev).word.fill_(1)
    torch.cuda.synchronize()
    ops.scan_status(dev)
    torch.cuda.synchronize()
    with pytest.raises(_lib.BDMError):
        ops.check_scan_status(dev)
    with pytest.raises(_lib.BDMError):
        ops.check_scan_status(dev, wait=True)
    ops.reset_scan_status(dev)
    assert ops.scan_status(dev, wait=True) == 0


def test_long_kernel_wait_runs_out_sets_status_and_returns():
    # The long-sequence kernel's producer withholds its first batch hand-off (a test flag that
    # nothing sets in normal use), with a 2 ms wait limit: the consumers' bounded wait runs out,
    # the launch records BDM_SCAN_ERR_TIMEOUT and every warp returns; the context stays usable.
    lib = _lib.load()
    dev = torch.device(DEV, torch.cuda.current_device())
    try:
        assert lib.bdm_scan_test_fault(1, 2_000_000) == 0
        with pytest.raises(_lib.BDMError, match='status 0x1'):
            _run_scan(2, 2600, 4, 2, 1, 8, 128, torch.bfloat16, interval=16, routed=True, seed=5)
        with pytest.raises(_lib.BDMError):  # the sticky word reports it to later callers too
            ops.check_scan_status(dev, wait=True)
    finally:
        lib.bdm_scan_test_fault(0, 0)
        ops.reset_scan_status(dev)
    ours, ref, _, _ = _run_scan(2, 2600, 4, 2, 1, 8, 128, torch.bfloat16, interval=16, routed=True, seed=5)
    assert max_rel(ours, ref) <= BF16_TOL
    assert ops.scan_status(dev, wait=True) == 0


# ------------------------------------------------------------------ layer
LAYER_GOLDEN = [('h1_fp32', 2e-2), ('h1_fp32_state32', FP32_TOL), ('h2_fp32_state32', FP32_TOL),
                ('c1_t64', 2e-2)]


def _module_from_golden(data):
    cfg = BSDMConfig(**data['config'])
    m = BlockSparseDeltaMemory(cfg, seed=data['seed'])
    if data['dtype'] == 'torch.bfloat16':
        m = m.to(torch.bfloat16)
    m.load_state_dict(data['state_dict'])
    return m.to(DEV)


@pytest.mark.parametrize('name,tol', LAYER_GOLDEN)
def test_layer_forward_matches_reference_golden(golden_dir, name, tol):
    data = torch.load(os.path.join(golden_dir, f'layer_{name}.pt'), weights_only=False)
    m = _module_from_golden(data)
    with torch.no_grad():
        y = m(data['x'].to(DEV))
    assert max_rel(npf(y), npf(data['out'])) <= tol, max_rel(npf(y), npf(data['out']))


@pytest.mark.parametrize('name', ['h1_bf16', 'h2_bf16'])
def test_layer_bf16_with_reference_routes(golden_dir, name):
    """BF16 logits tie often; drive our kernels with the reference's own routes."""
    data = torch.load(os.path.join(golden_dir, f'layer_{name}.pt'), weights_only=False)
    m = _module_from_golden(data)
    x = data['x'].to(DEV)
    batch, time, _ = x.shape
    with torch.no_grad():
        controls, _, gate = m._controls_and_routes(x)
        r = data['routes']
        routes = tuple(t.to(DEV) for t in (r['ww'], r['wi'], r['rw'], r['ri']))
        interval = state_interval(m.bank_size)
        reads = m._bank_pass(controls, routes, batch, time, row_factor=m.initial_row_factor,
                             col_factor=m.initial_column_factor, state_interval=interval)
        y = m._output(x, reads, routes[3].reshape(batch * time, -1), gate, round_each=False)
    assert max_rel(npf(y), npf(data['out'])) <= BF16_TOL, max_rel(npf(y), npf(data['out']))


def _oracle_layer(m):
    params = {k: npf(v) for k, v in m.state_dict().items()}
    cfg = {k: getattr(m.config, k) for k in m.config.__dataclass_fields__}
    return oracle.OracleLayer(cfg, params, bf16=m.q_proj.weight.dtype == torch.bfloat16)


def _our_controls_routes(m, x):
    batch, time, _ = x.shape
    controls, routes, _ = m._controls_and_routes(x)
    H, S, dv = m.num_heads, m.bank_size, m.head_value_width
    q, k, v, g, b, w = (npf(t) for t in controls)
    sh = lambda t, last: t.reshape(batch, time, H, last)
    ctl = (sh(q, S), sh(k, S), sh(v, dv), sh(g, S), sh(b, S), sh(w, dv))
    ww, wi, rw, ri = routes
    return ctl, ((npf(ww), wi.cpu().numpy()), (npf(rw), ri.cpu().numpy()))


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('heads', [1, 2])
def test_prefill_and_decode_steps_match_oracle(dtype, heads):
    cfg = BSDMConfig(dim=128, bank_count=256, bank_size=8, selected_banks=8, value_width=64 * heads,
                     num_heads=heads)
    torch.manual_seed(5)
    m = BlockSparseDeltaMemory(cfg, seed=1).to(dtype).to(DEV)
    ol = _oracle_layer(m)
    tol = BF16_TOL if dtype == torch.bfloat16 else FP32_TOL
    x = torch.randn(4, 48, 128).to(dtype).to(DEV)
    with torch.no_grad():
        ctl, routes = _our_controls_routes(m, x)
        # the router on our own logits equals the oracle's router on the same logits
        proj, cols = m._project(x.reshape(-1, 128))
        width = sum(m.factors)
        for role in ('write', 'read'):
            lg = npf(proj[:, cols[role]:cols[role] + width])
            _, oi = oracle.oracle_route(lg, bank_count=256, selected_banks=8, bf16=dtype == torch.bfloat16)
            got = routes[0][1] if role == 'write' else routes[1][1]
            np.testing.assert_array_equal(got.reshape(oi.shape), oi)
        y, state = m.prefill(x, state_dtype=torch.bfloat16)
        oy, ostate = ol.prefill(npf(x), controls=ctl, routes=routes, cache_bf16=True)
        assert max_rel(npf(y), oy) <= tol, max_rel(npf(y), oy)
        assert max_rel(npf(state).reshape(ostate.shape), ostate) <= BF16_TOL
        for i in range(4):
            xt = torch.randn(4, 1, 128).to(dtype).to(DEV)
            ctl, routes = _our_controls_routes(m, xt)
            # each step starts both sides from the same BF16 cache (a rounding that lands on the
            # other side of a tie in an earlier step would otherwise carry over)
            before = np.ascontiguousarray(npf(state).reshape(ostate.shape))
            y, state = m.step(xt, state)
            oy, ostate = ol.step(npf(xt), before, controls=ctl, routes=routes, cache_bf16=True)
            assert max_rel(npf(y), oy) <= tol, (i, max_rel(npf(y), oy))
            assert max_rel(npf(state).reshape(ostate.shape), ostate) <= BF16_TOL, i


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_layer_forward_matches_oracle_with_same_routes(dtype):
    cfg = BSDMConfig(dim=256, bank_count=256, bank_size=8, selected_banks=8, value_width=256, num_heads=2,
                     training_state_dtype='float32' if dtype == torch.float32 else 'bfloat16')
    torch.manual_seed(9)
    m = BlockSparseDeltaMemory(cfg, seed=2).to(dtype).to(DEV)
    ol = _oracle_layer(m)
    x = torch.randn(2, 96, 256).to(dtype).to(DEV)
    with torch.no_grad():
        y = m(x)
        ctl, routes = _our_controls_routes(m, x)
    oy = ol.forward(npf(x), controls=ctl, routes=routes)
    tol = BF16_TOL if dtype == torch.bfloat16 else FP32_TOL
    assert max_rel(npf(y), oy) <= tol, max_rel(npf(y), oy)


def test_controllers_match_oracle_directly():
    # the controller epilogue (fused projection + bdm_controllers) against the oracle's own
    # controllers computed from x (FP32: 1e-4; BF16: one BF16 rounding step of slack)
    for dtype, tol in ((torch.float32, FP32_TOL), (torch.bfloat16, BF16_TOL)):
        for qk in ('nvidia', 'original'):
            cfg = BSDMConfig(dim=256, bank_count=256, bank_size=8, selected_banks=8, value_width=256, num_heads=2,
                             qk_normalization=qk)
            torch.manual_seed(13)
            m = BlockSparseDeltaMemory(cfg, seed=6).to(dtype).to(DEV)
            ol = _oracle_layer(m)
            x = torch.randn(2, 80, 256).to(dtype).to(DEV)
            with torch.no_grad():
                ours, _ = _our_controls_routes(m, x)
            ref = ol.controllers(npf(x))
            for name, a, b in zip('qkvgbw', ours, ref):
                assert max_rel(a, b) <= tol, (dtype, qk, name, max_rel(a, b))


def test_decode_at_c3_geometry_matches_oracle():
    """c3: J = 2048 (32 x 64 product key), S = 8, B = 8, d_v = 128, H = 1, batch 64: a 2048-token
    prefill, then 8 steps, each against the oracle from the same BF16 cache."""
    cfg = BSDMConfig(dim=1024, bank_count=2048, bank_size=8, selected_banks=8, value_width=128, num_heads=1)
    assert near_square_factors(2048) == (32, 64)
    torch.manual_seed(2)
    m = BlockSparseDeltaMemory(cfg, seed=2).to(torch.bfloat16).to(DEV)
    ol = _oracle_layer(m)
    x = torch.randn(64, 2048, 1024).to(torch.bfloat16).to(DEV)
    with torch.no_grad():
        ctl, routes = _our_controls_routes(m, x)
        proj, cols = m._project(x.reshape(-1, 1024))
        for role, got in (('write', routes[0][1]), ('read', routes[1][1])):
            lg = npf(proj[:, cols[role]:cols[role] + sum(m.factors)])
            _, oi = oracle.oracle_route(lg, bank_count=2048, selected_banks=8, bf16=True)
            np.testing.assert_array_equal(got.reshape(oi.shape), oi)
        del proj
        y, state = m.prefill(x)
        oy, ostate = ol.prefill(npf(x), controls=ctl, routes=routes, cache_bf16=True)
        assert max_rel(npf(y), oy) <= BF16_TOL
        assert max_rel(npf(state).reshape(ostate.shape), ostate) <= BF16_TOL
        del x, y, oy, ctl
        for i in range(8):
            xt = torch.randn(64, 1, 1024).to(torch.bfloat16).to(DEV)
            ctl, routes = _our_controls_routes(m, xt)
            before = np.ascontiguousarray(npf(state).reshape(ostate.shape))
            y, state = m.step(xt, state)
            oy, ostate = ol.step(npf(xt), before, controls=ctl, routes=routes, cache_bf16=True)
            assert max_rel(npf(y), oy) <= BF16_TOL, (i, max_rel(npf(y), oy))
            assert max_rel(npf(state).reshape(ostate.shape), ostate) <= BF16_TOL, i


def test_layer_forward_at_c4_geometry_matches_oracle():
    """c4 slice: S = 16, H = 16, J = 16384 (128 x 128), B = 16, d_v = 128, the Zipf(1.1) router skew,
    the product-key initial state through the bank table; batch 1 x 1024 tokens, BF16."""
    from bench import zipf_router_bias
    cfg = BSDMConfig(dim=2048, bank_count=16384, bank_size=16, selected_banks=16, value_width=2048, num_heads=16)
    torch.manual_seed(3)
    m = BlockSparseDeltaMemory(cfg, seed=3)
    zipf_router_bias(m, 1.1, seed=3)
    m = m.to(torch.bfloat16).to(DEV)
    ol = _oracle_layer(m)
    x = torch.randn(1, 1024, 2048).to(torch.bfloat16).to(DEV)
    with torch.no_grad():
        y = m(x)
        ctl, routes = _our_controls_routes(m, x)
    oy = ol.forward(npf(x), controls=ctl, routes=routes)
    assert max_rel(npf(y), oy) <= BF16_TOL, max_rel(npf(y), oy)
    # the skew makes some (row, bank) sequences long: at least one bank takes > 1% of the events
    counts = np.bincount(np.concatenate([routes[0][1].ravel(), routes[1][1].ravel()]), minlength=16384)
    assert counts.max() > 0.01 * counts.sum()


def test_forward_is_deterministic():
    cfg = BSDMConfig(dim=256, bank_count=256, bank_size=8, selected_banks=8, value_width=256, num_heads=2)
    m = BlockSparseDeltaMemory(cfg, seed=4).to(torch.bfloat16).to(DEV)
    x = torch.randn(2, 300, 256).to(torch.bfloat16).to(DEV)
    with torch.no_grad():
        a, b = m(x), m(x)
    assert torch.equal(a, b)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
@pytest.mark.parametrize('layer_norm', [True, False])
def test_decode_step_fused_norm_gate(dtype, layer_norm):
    # the step kernel's fused output norm + gate equals the separate combine_norm_gate over its raw sum
    gen = torch.Generator().manual_seed(21)
    batch, heads, s, dv, J, k = 16, 2, 8, 64, 64, 4
    ctl = [t.to(DEV) for t in _controls(gen, batch, heads, s, dv, dtype)]
    wi = torch.stack([torch.randperm(J, generator=gen)[:k] for _ in range(batch)]).to(DEV)
    ri = torch.stack([torch.randperm(J, generator=gen)[:k] for _ in range(batch)]).to(DEV)
    ww = torch.softmax(torch.randn(batch, k, generator=gen), -1).to(dtype).to(DEV)
    rw = torch.softmax(torch.randn(batch, k, generator=gen), -1).to(dtype).to(DEV)
    state = (0.1 * torch.randn(batch, J, heads, s, dv, generator=gen)).to(dtype).to(DEV)
    gate = torch.randn(batch, heads * dv + 8, generator=gen).to(dtype).to(DEV)[:, :heads * dv]
    nw = (1 + 0.1 * torch.randn(heads * dv, generator=gen)).to(DEV)
    nb = 0.1 * torch.randn(heads * dv, generator=gen).to(DEV) if layer_norm else None
    kw = dict(bank_count=J, heads=heads, bank_size=s, head_value_width=dv, routed_decay=True, scale=s ** -0.5)
    st1, st2 = state.clone(), state.clone()
    raw = ops.decode_step(*ctl, wi, ww, ri, rw, st1, **kw)
    want = ops.combine_norm_gate(raw, None, gate, nw, nb, eps=1e-5, layer_norm=layer_norm, round_each=True)
    got = ops.decode_step(*ctl, wi, ww, ri, rw, st2, **kw, gate=gate, norm_weight=nw, norm_bias=nb, eps=1e-5,
                          layer_norm=layer_norm)
    assert torch.equal(st1, st2)
    # the norm's FP32 sums associate differently (one column per thread): BF16 outputs at most one
    # ulp apart, FP32 outputs within 1e-6 max-relative
    diff = (got.float() - want.float()).abs()
    if dtype == torch.bfloat16:
        assert (diff <= 2 ** -7 * want.float().abs().clamp_min(1e-3)).all()
    else:
        assert diff.max() <= 1e-6 * want.float().abs().max()


@pytest.mark.parametrize('dtype,cache_dtype', [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                               (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize('heads,bank_size,norm,qk', [(1, 8, 'layer', 'nvidia'), (2, 16, 'rms', 'original'),
                                                     (4, 4, 'layer', 'original')])
def test_fused_decode_step_equals_separate_kernels(dtype, cache_dtype, heads, bank_size, norm, qk):
    # bdm_decode_token_step (controllers + routers + bank step in one launch) against
    # bdm_controllers + bdm_route_pair + bdm_decode_step on the same cache: bit for bit
    cfg = BSDMConfig(dim=256, bank_count=512, bank_size=bank_size, selected_banks=8, value_width=64 * heads,
                     num_heads=heads, output_normalization=norm, qk_normalization=qk)
    torch.manual_seed(21)
    m = BlockSparseDeltaMemory(cfg, seed=3).to(dtype).to(DEV)
    with torch.no_grad():
        x0 = torch.randn(6, 40, 256).to(dtype).to(DEV)
        _, state = m.prefill(x0, state_dtype=cache_dtype)
        for i in range(3):
            xt = torch.randn(6, 1, 256).to(dtype).to(DEV)
            ref_state = state.clone()
            controls, routes, gate = m._controls_and_routes(xt)
            ww, wi, rw, ri = (r.reshape(6, -1) for r in routes)
            normed = ops.decode_step(*controls, wi, ww, ri, rw, ref_state, bank_count=m.bank_count, heads=heads,
                                     bank_size=bank_size, head_value_width=m.head_value_width,
                                     routed_decay=m.config.routed_decay, scale=bank_size ** -0.5, gate=gate,
                                     norm_weight=m.output_norm_weight,
                                     norm_bias=getattr(m, 'output_norm_bias', None), eps=m.norm_eps,
                                     layer_norm=norm == 'layer')
            ref = torch.nn.functional.linear(normed, m.o_proj.weight, m.o_proj.bias).reshape(6, 1, 256)
            y, state = m.step(xt, state)
            assert torch.equal(y, ref), i
            assert torch.equal(state, ref_state), i


def test_captured_decode_step_matches_eager_step():
    cfg = BSDMConfig(dim=256, bank_count=2048, bank_size=8, selected_banks=8, value_width=128, num_heads=1)
    m = BlockSparseDeltaMemory(cfg, seed=2).to(torch.bfloat16).to(DEV)
    prefix = torch.randn(16, 40, 256).to(torch.bfloat16).to(DEV)
    toks = torch.randn(5, 16, 1, 256).to(torch.bfloat16).to(DEV)
    with torch.inference_mode():
        _, state = m.prefill(prefix)
        eager_state = state.clone()
        run = m.capture_step(state)
        assert torch.equal(state, eager_state), 'capturing must not advance the cache'
        for i in range(5):
            y_graph = run(toks[i]).clone()
            y_eager, _ = m.step(toks[i], eager_state)
            assert torch.equal(y_graph, y_eager), i
            assert torch.equal(state, eager_state), i


# ------------------------------------------------------- fused combine + output projection
def _combine_project_case(ntok, kr, width, out_dim, norm_bias, o_bias, seed):
    gen = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    reads = torch.randn(ntok, kr, width, generator=gen).to(bf).to(DEV)
    banks = torch.randint(0, 64, (ntok, kr), generator=gen).to(DEV)  # repeats exercise the slot tie rule
    proj = torch.randn(ntok, width + 40, generator=gen).to(bf).to(DEV)  # gate as a strided column block
    gate = proj[:, 24:24 + width]
    nw = (1 + 0.1 * torch.randn(width, generator=gen)).to(bf).to(DEV)
    nb = (0.1 * torch.randn(width, generator=gen)).to(bf).to(DEV) if norm_bias else None
    w = (torch.randn(out_dim, width, generator=gen) * width ** -0.5).to(bf).to(DEV)
    b = (0.1 * torch.randn(out_dim, generator=gen)).to(bf).to(DEV) if o_bias else None
    return reads, banks, gate, nw, nb, w, b


@pytest.mark.parametrize('ntok,kr,width,out_dim,layer_norm,norm_bias,o_bias,round_each', [
    (4096, 8, 1024, 1024, True, True, True, False),   # c2 output interface
    (1000, 8, 1024, 1024, True, True, False, True),   # ragged last tile, no o_proj bias, round-each combine
    (777, 16, 512, 256, False, False, True, False),   # RMS norm, 16 read slots
    (130, 3, 768, 768, True, False, True, False),     # 3-warp token groups (V = 768), 6 accumulators
    (64, 8, 1024, 128, True, True, True, False),      # one tile, one accumulator
    (300, 8, 512, 1024, True, True, True, False),     # more features than columns: two staging chunks
    (1, 1, 512, 1024, True, True, True, True),        # one token
])
def test_combine_project_matches_combine_then_exact_gemm(ntok, kr, width, out_dim, layer_norm, norm_bias, o_bias,
                                                         round_each):
    """The fused kernel's output is one BF16 rounding of the exact product of the
    combine_norm_gate output with o_proj's weight (plus bias)."""
    assert ops.combine_project_supported(width, out_dim, kr, torch.bfloat16)
    reads, banks, gate, nw, nb, w, b = _combine_project_case(ntok, kr, width, out_dim, norm_bias, o_bias,
                                                             seed=ntok + kr)
    ops.reset_scan_status()
    out = ops.combine_project(reads, banks, gate, nw, nb, w, b, eps=1e-5, layer_norm=layer_norm,
                              round_each=round_each)
    normed = ops.combine_norm_gate(reads, banks, gate, nw, nb, eps=1e-5, layer_norm=layer_norm,
                                   round_each=round_each)
    ref = normed.double() @ w.double().t()
    if b is not None:
        ref = ref + b.double()
    got = out.double()
    # BF16 rounding (half an ulp, 2^-9 relative) plus the FP32 accumulation-order difference
    bound = 2.0 ** -8 * ref.abs() + 1e-5 * ref.abs().max()
    assert bool(((got - ref).abs() <= bound).all()), float(((got - ref).abs() / (ref.abs() + 1e-6)).max())
    assert ops.scan_status(wait=True) == 0


def test_combine_project_rejects_shapes_it_does_not_take():
    bf = torch.bfloat16
    for width, out_dim, kr, dt in ((2048, 1024, 8, bf), (1024, 1152, 8, bf), (1024, 1000, 8, bf), (320, 256, 8, bf),
                                   (1024, 1024, 17, bf), (1024, 1024, 8, torch.float32)):
        assert not ops.combine_project_supported(width, out_dim, kr, dt)
    reads = torch.zeros(4, 8, 2048, dtype=bf, device=DEV)
    with pytest.raises(NotImplementedError):
        ops.combine_project(reads, torch.zeros(4, 8, dtype=torch.int64, device=DEV), reads[:, 0],
                            torch.ones(2048, dtype=bf, device=DEV), None, torch.zeros(1024, 2048, dtype=bf, device=DEV),
                            None, eps=1e-5, layer_norm=True, round_each=False)


def test_layer_fused_output_matches_unfused_and_oracle():
    """A BF16 layer whose output interface fits the fused kernel: forward (FP32 combine) and
    prefill (round-each combine) against the combine_norm_gate + cuBLAS path and the oracle."""
    cfg = BSDMConfig(dim=512, bank_count=256, bank_size=8, selected_banks=8, value_width=512, num_heads=4)
    torch.manual_seed(21)
    m = BlockSparseDeltaMemory(cfg, seed=5)
    with torch.no_grad():
        m.output_norm_weight.add_(0.1 * torch.randn_like(m.output_norm_weight))
        m.output_norm_bias.add_(0.1 * torch.randn_like(m.output_norm_bias))
        if m.o_proj.bias is not None:
            m.o_proj.bias.add_(0.1 * torch.randn_like(m.o_proj.bias))
    m = m.to(torch.bfloat16).to(DEV)
    assert ops.combine_project_supported(512, 512, 8, torch.bfloat16)
    x = torch.randn(2, 300, 512).to(torch.bfloat16).to(DEV)
    with torch.no_grad():
        m.fused_output = True
        y_fused = m(x)
        yp_fused, st_fused = m.prefill(x)
        m.fused_output = False
        y_plain = m(x)
        yp_plain, st_plain = m.prefill(x)
        ctl, routes = _our_controls_routes(m, x)
    for a, b in ((y_fused, y_plain), (yp_fused, yp_plain)):
        d = (a.double() - b.double()).abs()
        # one BF16 ulp where the two GEMMs' FP32 sums round to neighbouring values
        assert bool((d <= 2.0 ** -7 * b.double().abs() + 1e-5).all()), float(d.max())
    assert torch.equal(st_fused, st_plain)
    oy = _oracle_layer(m).forward(npf(x), controls=ctl, routes=routes)
    assert max_rel(npf(y_fused), oy) <= BF16_TOL, max_rel(npf(y_fused), oy)


@pytest.mark.parametrize('dtype,chunks,graphs', [(torch.bfloat16, 4, False), (torch.float32, 3, False),
                                                 (torch.bfloat16, 1, False), (torch.bfloat16, 2, True),
                                                 (torch.float32, 4, True), (torch.bfloat16, 3, True)])
def test_forward_host_streams_row_groups_like_forward(dtype, chunks, graphs):
    """forward_host (host batch in, host result out, row groups with overlapped copies; with graphs,
    replays of captured row-group forwards) against forward on the device copy: the bank path is
    per row, so only the GEMMs' accumulation order at a smaller row count may differ.  After a
    parameter update the captured forwards are recaptured."""
    cfg = BSDMConfig(dim=256, bank_count=256, bank_size=8, selected_banks=8, value_width=256, num_heads=2)
    torch.manual_seed(31)
    m = BlockSparseDeltaMemory(cfg, seed=3).to(dtype).to(DEV)
    x = torch.randn(8, 96, 256).to(dtype).pin_memory()
    tol = FP32_TOL if dtype == torch.float32 else BF16_TOL
    with torch.no_grad():
        for update in (False, True):
            if update:
                m.o_proj.weight.mul_(1.5)  # in place: bumps the parameter's version
            ref = m(x.to(DEV))
            got = m.forward_host(x, chunks=chunks, graphs=graphs)
            torch.cuda.synchronize()
            again = m.forward_host(x, torch.empty_like(got).pin_memory(), chunks=chunks, graphs=graphs)
            torch.cuda.synchronize()
            assert not got.is_cuda and got.shape == ref.shape
            assert max_rel(npf(got), npf(ref)) <= tol, (update, max_rel(npf(got), npf(ref)))
            assert torch.equal(got, again)
