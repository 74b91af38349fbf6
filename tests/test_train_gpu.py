"""Training backward on the GPU against the reference's gradients and the autograd oracle.

* golden: gradients produced by the reference itself (tests/golden/grad_*.pt, torch
  autograd through BlockSparseDeltaMemory / BankedDeltaMemory with backend='reference').
* oracle: oracle/grad.py (torch autograd over a CPU restatement of the training
  forward, pinned to the golden files by test_oracle_golden.py) on seeded cases the
  golden files do not cover: bank sizes 4 / 16, two column tiles, sequences longer
  than one checkpoint block, plain decay, RMS output norm.
* a size-independent property at a larger size: the directional derivative of
  <dy, layer(x)> along parameters that do not move the routing equals the gradient's
  projection (central difference, FP32).

Tolerances: FP32 runs 1e-4 max-relative per tensor (FP32 storage) or 2e-3 (BF16
storage policy: a replayed state can round to the neighbouring BF16 value where the
oracle's does not); BF16 runs 3e-2 max-relative (the reference's own BF16 gradients
differ from the oracle's by ~1e-2, BF16 rounding of intermediate gradients).
"""
import glob
import os

import pytest
import torch

from oracle.grad import layer_grads

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _cls(name):
    from bdm_b200 import BDMConfig, BSDMConfig
    return BSDMConfig if name == 'BSDM' else BDMConfig


def _module(cfg_cls, cfg: dict, seed: int, dtype, state_dict=None):
    from bdm_b200 import BankedDeltaMemory
    m = BankedDeltaMemory(cfg_cls(**cfg), seed=seed).to(dtype).cuda()
    if state_dict is not None:
        m.load_state_dict({k: v.cuda() for k, v in state_dict.items()})
    return m


def _cuda_grads(m, x, dy):
    xx = x.cuda().clone().requires_grad_(True)
    for p in m.parameters():
        p.grad = None
    y = m(xx)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    return {n: p.grad.detach().cpu() for n, p in m.named_parameters() if p.grad is not None}, xx.grad.cpu(), y.cpu()


def _max_rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def _report(got, got_x, ref, ref_x, tol):
    errs = {n: _max_rel(got[n], ref[n]) for n in ref}
    errs['x'] = _max_rel(got_x, ref_x)
    missing = sorted(set(ref) - set(got))
    bad = {n: e for n, e in errs.items() if not e <= tol}
    return missing, bad, errs


@pytest.mark.parametrize('path', sorted(glob.glob(os.path.join(HERE, 'golden', 'grad_*.pt'))),
                         ids=lambda p: os.path.basename(p)[5:-3])
def test_backward_matches_reference_golden(path):
    d = torch.load(path)
    dtype = torch.bfloat16 if 'bfloat16' in d['dtype'] else torch.float32
    m = _module(_cls(d['config_class']), d['config'], d['seed'], dtype, d['state_dict'])
    grads, xg, y = _cuda_grads(m, d['x'], d['dy'])
    if dtype == torch.float32:
        ref, ref_x = d['grads'], d['x_grad']
        tol = 1e-4
        assert _max_rel(y, d['out']) < 1e-4
    else:
        # BF16: the reference's torch.topk orders exact score ties its own way; the kernels
        # (and the oracle by default) take the lower index.  Compare with the oracle on the
        # kernels' own selections; the oracle matches the golden file on the reference's.
        ref, ref_x, _ = layer_grads(d['state_dict'], d['x'], d['dy'], d['config'])
        tol = 3e-2
    missing, bad, errs = _report(grads, xg, ref, ref_x, tol)
    assert not missing, f'no gradient for {missing}'
    assert not bad, f'gradients outside {tol}: {bad} (all: {errs})'


def _case(cfg_cls, cfg, *, batch, time, seed, dtype):
    torch.manual_seed(seed)
    m = _module(cfg_cls, cfg, seed, dtype)
    gen = torch.Generator().manual_seed(seed + 77)
    with torch.no_grad():  # a nonzero initial memory so the factor gradients are exercised
        m.initial_row_factor.copy_((0.05 * torch.randn(m.initial_row_factor.shape, generator=gen)).to(dtype))
        m.initial_column_factor.copy_((0.05 * torch.randn(m.initial_column_factor.shape, generator=gen)).to(dtype))
    x = torch.randn(batch, time, cfg['dim'], generator=gen).to(dtype)
    dy = torch.randn(batch, time, cfg['dim'], generator=gen).to(dtype)
    sd = {k: v.detach().cpu() for k, v in m.state_dict().items()}
    return m, x, dy, sd


ORACLE_CASES = {
    # name: (config class, config, batch, time, dtype, state dtype)
    's8_two_tiles_long': ('BSDM', dict(dim=48, bank_count=16, bank_size=8, selected_banks=4, value_width=64,
                                       num_heads=1), 1, 160, torch.float32, 'float32'),
    's16_h2_long': ('BSDM', dict(dim=48, bank_count=16, bank_size=16, selected_banks=4, value_width=64,
                                 num_heads=2), 2, 96, torch.float32, 'float32'),
    's4_long_plain_rms': ('BDM', dict(dim=32, bank_count=16, bank_size=4, selected_banks=4, value_width=32,
                                      num_heads=1), 1, 300, torch.float32, 'float32'),
    's8_h4_bf16_storage': ('BSDM', dict(dim=64, bank_count=64, bank_size=8, selected_banks=8, value_width=128,
                                        num_heads=4), 2, 64, torch.float32, 'bfloat16'),
    's8_h2_bf16': ('BDM', dict(dim=64, bank_count=36, bank_size=8, selected_banks=4, value_width=64,
                               num_heads=2), 2, 48, torch.bfloat16, 'bfloat16'),
}


@pytest.mark.parametrize('name', sorted(ORACLE_CASES))
def test_backward_matches_oracle(name):
    cls_name, cfg, batch, time, dtype, state = ORACLE_CASES[name]
    cfg = dict(cfg, training_state_dtype=state)
    m, x, dy, sd = _case(_cls(cls_name), cfg, batch=batch, time=time, seed=11 + sorted(ORACLE_CASES).index(name),
                         dtype=dtype)
    grads, xg, y = _cuda_grads(m, x, dy)
    full_cfg = {k: getattr(m.config, k) for k in m.config.__dataclass_fields__}
    ref, ref_x, ref_y = layer_grads(sd, x, dy, full_cfg)
    if dtype == torch.float32:
        tol = 1e-4 if state == 'float32' else 2e-3
    else:
        tol = 3e-2
    assert _max_rel(y, ref_y) < max(tol, 1e-4)
    missing, bad, errs = _report(grads, xg, ref, ref_x, tol)
    assert not missing, f'no gradient for {missing}'
    assert not bad, f'gradients outside {tol}: {bad} (all: {errs})'


def test_backward_deterministic():
    cls_name, cfg, batch, time, dtype, state = ORACLE_CASES['s8_h4_bf16_storage']
    m, x, dy, _ = _case(_cls(cls_name), dict(cfg, training_state_dtype=state), batch=batch, time=time, seed=5,
                        dtype=dtype)
    g1, x1, _ = _cuda_grads(m, x, dy)
    g2, x2, _ = _cuda_grads(m, x, dy)
    assert torch.equal(x1, x2)
    for n in g1:
        assert torch.equal(g1[n], g2[n]), n


def test_directional_derivative_c5_layer():
    """<grad, delta> against a central difference at the c5 layer geometry (FP32, 2 x 1024 tokens)."""
    from bdm_b200 import BSDMConfig
    cfg = dict(dim=768, bank_count=512, bank_size=8, selected_banks=8, value_width=768, num_heads=12,
               training_state_dtype='float32')
    m, x, dy, _ = _case(BSDMConfig, cfg, batch=2, time=1024, seed=4, dtype=torch.float32)
    grads, _, _ = _cuda_grads(m, x, dy)
    # parameters that leave the routing unchanged
    names = ['q_proj.weight', 'k_proj.weight', 'v_proj.weight', 'f_proj.0.weight', 'f_proj.1.weight', 'b_proj.weight',
             'w_proj.weight', 'A_log', 'dt_bias', 'initial_row_factor', 'initial_column_factor', 'output_norm_weight',
             'output_norm_bias', 'output_gate.weight', 'output_gate.bias', 'o_proj.weight']
    params = dict(m.named_parameters())
    gen = torch.Generator().manual_seed(9)
    delta = {n: torch.randn(params[n].shape, generator=gen) * params[n].detach().float().pow(2).mean().sqrt().cpu()
             for n in names}
    proj = sum(float((grads[n].double() * delta[n].double()).sum()) for n in names)
    eps = 3e-3
    xc, dyc = x.cuda(), dy.cuda().double()
    vals = []
    with torch.no_grad():
        base = {n: params[n].detach().clone() for n in names}
        for sgn in (1.0, -1.0):
            for n in names:
                params[n].copy_(base[n] + sgn * eps * delta[n].cuda())
            m._fused_cache = None
            vals.append(float((m(xc).double() * dyc).sum()))
        for n in names:
            params[n].copy_(base[n])
    fd = (vals[0] - vals[1]) / (2 * eps)
    assert abs(fd - proj) <= 5e-3 * abs(proj), (fd, proj)
