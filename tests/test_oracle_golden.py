"""Pin the CPU oracle against golden vectors produced by the reference itself.

Fixtures come from tests/golden/make_golden.py, which imports the reference
package and runs its own CPU functions.  Integer work (routing indices,
dispatch order) must agree exactly; floating point agrees to the tolerances
named in each test.
"""
import os

import numpy as np
import pytest
import torch

from oracle import (OracleLayer, bf16_round, near_square_factors, oracle_combine, oracle_dispatch,
                    oracle_recurrence, oracle_route)


def _load(golden_dir, name):
    return torch.load(os.path.join(golden_dir, name), weights_only=False)


def _np(t):
    return t.detach().float().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def max_rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def stable_route_py(z, bank_count, selected, bf16):
    """Pure-Python restatement of product_key_route with lower-index tie breaking."""
    j1, j2 = near_square_factors(bank_count)
    sub = min(selected, j1, j2)
    first, second = z[:j1], z[j1:j1 + j2]
    fi = sorted(range(j1), key=lambda i: (-first[i], i))[:sub]
    si = sorted(range(j2), key=lambda i: (-second[i], i))[:sub]
    pv = [first[fi[i]] + second[si[l]] for i in range(sub) for l in range(sub)]
    if bf16:
        pv = list(bf16_round(np.array(pv, np.float32)))
    count = min(selected, sub * sub)
    best = sorted(range(sub * sub), key=lambda p: (-pv[p], p))[:count]
    return [fi[p // sub] * j2 + si[p % sub] for p in best], [pv[p] for p in best]


def _ambiguous(z, bank_count, selected, bf16):
    """True when a tie could change the selected set or its order."""
    j1, j2 = near_square_factors(bank_count)
    sub = min(selected, j1, j2)
    for part in (z[:j1], z[j1:j1 + j2]):
        s = np.sort(part)[::-1]
        if len(np.unique(s[:sub + 1])) < min(sub + 1, len(s)):
            return True
    first = np.sort(z[:j1])[::-1][:sub]
    second = np.sort(z[j1:j1 + j2])[::-1][:sub]
    pv = (first[:, None] + second[None, :]).astype(np.float32).reshape(-1)
    if bf16:
        pv = bf16_round(pv)
    s = np.sort(pv)[::-1]
    count = min(selected, sub * sub)
    top = s[:count + 1]
    return len(np.unique(top)) < len(top)


@pytest.mark.parametrize('field', ['indices', 'indices_batch'])
def test_router_matches_reference(golden_dir, field):
    data = _load(golden_dir, 'router.pt')
    checked = 0
    for case in data['cases']:
        if case[field] is None:
            continue
        logits = case['logits']
        bf16 = logits.dtype == torch.bfloat16
        z = _np(logits)[0]
        w, i = oracle_route(z, bank_count=case['bank_count'], selected_banks=case['selected'], bf16=bf16)
        ref_i = case[field].numpy()[0]
        ref_w = _np(case['weights' if field == 'indices' else 'weights_batch'])[0]
        j1, j2 = near_square_factors(case['bank_count'])
        unamb = 0
        for t in range(z.shape[0]):
            # the selected pair values agree on every token (tie-invariant)
            zt = z[t]

            def vals(idx):
                pv = (zt[:j1][idx // j2] + zt[j1:][idx % j2]).astype(np.float32)
                return np.sort(bf16_round(pv) if bf16 else pv)

            assert np.array_equal(vals(i[t]), vals(ref_i[t])), (case['bank_count'], t)
            if case['kind'] == 'random' and not _ambiguous(z[t], case['bank_count'], case['selected'], bf16):
                unamb += 1
                assert np.array_equal(i[t], ref_i[t]), (case['bank_count'], t, i[t], ref_i[t])
                if bf16:
                    assert np.abs(w[t] - ref_w[t]).max() <= 2 ** -8 * np.abs(ref_w[t]).max()
                else:
                    np.testing.assert_allclose(w[t], ref_w[t], rtol=2e-6, atol=1e-7)
            exp_i, _ = stable_route_py(z[t], case['bank_count'], case['selected'], bf16)
            assert list(i[t]) == exp_i
        if case['kind'] == 'random' and not bf16:
            # BF16 pair sums tie often on wide tables; FP32 logits must pin most tokens
            assert unamb >= z.shape[0] // 4, 'too few tie-free tokens to pin the router'
        checked += unamb
    assert checked > 0


def test_router_lower_index_wins_ties():
    z = np.zeros(32, np.float32)
    w, i = oracle_route(z, bank_count=256, selected_banks=8, bf16=True)
    assert list(i) == [0, 1, 2, 3, 4, 5, 6, 7]
    np.testing.assert_array_equal(w, np.full(8, 0.125, np.float32))
    z = np.array([1, 2, 2, 0.5] + [0] * 4, np.float32)  # J=16: 4x4, B=2
    w, i = oracle_route(z, bank_count=16, selected_banks=2, bf16=False)
    assert list(i) == [1 * 4 + 0, 1 * 4 + 1]


def test_dispatch_matches_reference(golden_dir):
    for case in _load(golden_dir, 'dispatch.pt')['cases']:
        out = oracle_dispatch(case['wi'].numpy(), case['ri'].numpy(), case['bank_count'])
        np.testing.assert_array_equal(out['order'], case['order'].numpy())
        np.testing.assert_array_equal(out['cu_seqlens'], case['cu_seqlens'].numpy())
        np.testing.assert_array_equal(out['tokens'], case['tokens'].numpy())
        ne = case['wi'].numel()
        np.testing.assert_array_equal(out['order'] >= ne, case['read_events'].numpy())
        inv = np.empty_like(out['order'])
        inv[out['order']] = np.arange(len(inv))
        np.testing.assert_array_equal(out['inverse'], inv)


def _rec_inputs(case):
    add_head = lambda t: _np(t)[:, :, None]
    q, k, v, g, b, w = (add_head(case[n]) for n in 'qkvgbw')
    init = _np(case['init'])[None, :, None]
    return q, k, v, g, b, w, init


@pytest.mark.parametrize('which', [0, 1])
def test_recurrence_matches_reference_packed(golden_dir, which):
    case = _load(golden_dir, 'recurrence.pt')['cases'][which]
    bf16 = case['dtype'] == 'torch.bfloat16'
    q, k, v, g, b, w, init = _rec_inputs(case)
    for (state_dtype, interval), ref in case['packed'].items():
        use = interval if state_dtype == 'torch.bfloat16' else 0
        reads, _ = oracle_recurrence(q, k, v, g, b, w, case['wi'].numpy(), _np(case['ww']), case['ri'].numpy(),
                                     _np(case['rw']), init, bank_count=case['bank_count'], bf16=bf16,
                                     routed_decay=True, interval=use, scale=case['bank_size'] ** -0.5)
        raw = oracle_combine(reads, case['ri'].numpy(), bf16=bf16)
        ref = _np(ref)
        if bf16:
            assert max_rel(raw, ref) <= 1e-2, (state_dtype, interval)
            assert np.mean(raw == ref) >= 0.95
        else:
            assert max_rel(raw, ref) <= 1e-5, (state_dtype, interval)


@pytest.mark.parametrize('which', [0, 1])
def test_recurrence_matches_serial_equation_oracle(golden_dir, which):
    case = _load(golden_dir, 'recurrence.pt')['cases'][which]
    q, k, v, g, b, w, init = _rec_inputs(case)
    reads, state = oracle_recurrence(q, k, v, g, b, w, case['wi'].numpy(), _np(case['ww']), case['ri'].numpy(),
                                     _np(case['rw']), init, bank_count=case['bank_count'], bf16=False,
                                     routed_decay=True, interval=0, scale=case['bank_size'] ** -0.5)
    raw = oracle_combine(reads, case['ri'].numpy(), bf16=False)
    ref_out = _np(case['serial_out'])
    ref_state = _np(case['serial_state'])
    assert max_rel(raw, ref_out) <= 1e-5
    assert max_rel(state[:, :, 0], ref_state) <= 1e-5


LAYERS = [('h1_fp32', 2e-2), ('h1_fp32_state32', 1e-4), ('h1_bf16', 2e-2), ('h2_bf16', 2e-2),
          ('h2_fp32_state32', 1e-4), ('c1_t64', 2e-2)]


@pytest.mark.parametrize('name,tol', LAYERS)
def test_layer_forward_matches_reference(golden_dir, name, tol):
    data = _load(golden_dir, f'layer_{name}.pt')
    bf16 = data['dtype'] == 'torch.bfloat16'
    params = {k: _np(v) for k, v in data['state_dict'].items()}
    layer = OracleLayer(data['config'], params, bf16=bf16)
    x = _np(data['x'])
    # controllers agree to dtype precision
    ours = layer.controllers(x)
    heads = data['config']['num_heads']
    for got, ref in zip(ours, data['controls']):
        ref = _np(ref).reshape(got.shape) if heads > 1 else _np(ref)[..., None, :]
        assert max_rel(got, ref) <= (1e-2 if bf16 else 1e-5)
    # the reference's own routes (torch.topk tie order) drive recurrence, combine and projection
    r = data['routes']
    routes = ((_np(r['ww']), r['wi'].numpy()), (_np(r['rw']), r['ri'].numpy()))
    controls = tuple(_np(c).reshape(o.shape) for c, o in zip(data['controls'], ours))
    out = layer.forward(x, controls=controls, routes=routes)
    assert max_rel(out, _np(data['out'])) <= tol, max_rel(out, _np(data['out']))
    # routing from the reference's logits: identical wherever no tie decides the selection
    rl, wl = _np(data['read_logits']), _np(data['write_logits'])
    for logits, (ref_w, ref_i) in ((wl, routes[0]), (rl, routes[1])):
        w_, i_ = layer.route(logits)
        flat = logits.reshape(-1, logits.shape[-1])
        for t in range(flat.shape[0]):
            if not _ambiguous(flat[t], layer.J, layer.B, bf16):
                assert np.array_equal(i_.reshape(-1, layer.B)[t], ref_i.reshape(-1, layer.B)[t])
    if not bf16:
        # FP32 logits rarely tie: the oracle's own end-to-end forward agrees as well
        assert max_rel(layer.forward(x), _np(data['out'])) <= tol


GRADS = ['h1_fp32_state32', 'h2_fp32_state32', 'bdm_h1_fp32_state32', 'h2_bf16', 'bdm_h2_bf16']


@pytest.mark.parametrize('name', GRADS)
def test_gradient_oracle_matches_reference(golden_dir, name):
    """oracle/grad.py autograd against the reference's own autograd (tests/golden/grad_*.pt).

    FP32: 1e-5 max-relative per tensor.  BF16: 2e-2 (both sides round intermediate
    gradients to BF16 at slightly different points); the reference's bank selections
    are used, since torch.topk orders exact BF16 score ties its own way.
    """
    from oracle.grad import layer_grads
    data = _load(golden_dir, f'grad_{name}.pt')
    bf16 = data['dtype'] == 'torch.bfloat16'
    grads, xg, y = layer_grads(data['state_dict'], data['x'], data['dy'], data['config'], data['write_idx'],
                               data['read_idx'])
    tol = 2e-2 if bf16 else 1e-5
    assert max_rel(y.float().numpy(), _np(data['out'])) <= (0.0 if bf16 else 1e-6)
    assert set(grads) == set(data['grads'])
    for n, ref in data['grads'].items():
        assert max_rel(grads[n].float().numpy(), _np(ref)) <= tol, n
    assert max_rel(xg.float().numpy(), _np(data['x_grad'])) <= tol
