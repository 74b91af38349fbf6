"""Differentiable CPU restatement of the BDM training forward -- TEST INFRASTRUCTURE ONLY.

The gradients of the reference's training path are the autograd derivatives of
its forward (model.py:88-140, heads.py:25-66) with one rule of its own: a BF16
state-storage point rounds the forward state but passes the adjoint through
unrounded (gdn2_banks.py:11-19 _StoredState; role_bank_kernel.py:58-66 keeps the
same FP32 adjoint).  ``layer_forward`` restates that forward with torch ops on
the CPU, so ``torch.autograd`` over it yields the oracle gradients:

* controllers             _parameters.py:189-220, heads.py:11-22
* shared-residual router  routing.py:23-35
* product-key routing     gdn2_banks.py:74-114 (indices from the C oracle,
                          weights = softmax of the selected pair scores)
* initial bank memory     _parameters.py:40-67 (U[row // Q] + Z[row % Q])
* packing + recurrence    gdn2_banks.py:22-43,196-224 (route-weighted packing
                          rounded to the activation dtype; FP32 recurrence)
* read combine            gdn2_banks.py:265-283
* output interface        _parameters.py:222-232

The recurrence advances every (batch*bank, head) sequence one event per step
(events in the dispatch order of the C oracle), so a step is a few batched
tensor ops and autograd records one node group per step.  Meant for small
cases (a few thousand events).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from .core import oracle_dispatch, oracle_route
from .layer import near_square_factors, state_interval


class _StoredState(torch.autograd.Function):
    """BF16 storage rounding of the forward state; the adjoint passes unchanged."""

    @staticmethod
    def forward(ctx, value):
        return value.to(torch.bfloat16).float()

    @staticmethod
    def backward(ctx, grad):
        return grad


def _linear(x, p, name, bias=None):
    return F.linear(x, p[name], None if bias is None else p[bias])


def _normalize(x, mode):
    """_parameters.py:214-220 (CPU forms): FP32 math, result in the input dtype."""
    xf = x.float()
    if mode == 'nvidia':
        return (xf * torch.rsqrt(xf.square().sum(-1, keepdim=True) + 1e-6)).to(x.dtype)
    return F.normalize(xf, dim=-1).to(x.dtype)


def controllers(p, x, cfg):
    """q, k, b, g [NT, H, S]; v, w [NT, H, dv] (g float32)."""
    H, S = cfg['num_heads'], cfg['bank_size']
    dv = cfg['value_width'] // H
    lead = x.shape[:-1]
    q = _normalize(F.silu(_linear(x, p, 'q_proj.weight')).reshape(*lead, H, S), cfg['qk_normalization'])
    k = _normalize(F.silu(_linear(x, p, 'k_proj.weight')).reshape(*lead, H, S), cfg['qk_normalization'])
    v = F.silu(_linear(x, p, 'v_proj.weight')).reshape(*lead, H, dv)
    f = F.linear(F.linear(x, p['f_proj.0.weight']), p['f_proj.1.weight'])
    g = (-p['A_log'].float().exp()[:, None]
         * F.softplus((f.float() + p['dt_bias'].float()).reshape(*lead, H, S)))
    b = torch.sigmoid(_linear(x, p, 'b_proj.weight')).reshape(*lead, H, S)
    w = torch.sigmoid(_linear(x, p, 'w_proj.weight')).reshape(*lead, H, dv)
    return q, k, v, g, b, w


def route_logits(p, x):
    """SharedResidualRouter.read / .write: base + residual, in the parameter dtype."""
    read = F.linear(x, p['shared_router.base.weight'] + p['shared_router.read_residual.weight'],
                    p['shared_router.base.bias'] + p['shared_router.read_residual.bias'])
    write = F.linear(x, p['shared_router.base.weight'] + p['shared_router.write_residual.weight'],
                     p['shared_router.base.bias'] + p['shared_router.write_residual.bias'])
    return read, write


def route(logits, cfg, idx=None):
    """Product-key selection and differentiable weights.

    ``idx``: the selected banks in score order; by default the C oracle's (ties to
    the lower index).  A caller may pass another implementation's selections (for
    example the reference's own, whose torch.topk orders exact BF16 ties its own way).
    """
    J, sel = cfg['bank_count'], cfg['selected_banks']
    j1, j2 = near_square_factors(J)
    if idx is None:
        bf16 = logits.dtype == torch.bfloat16
        _, idx = oracle_route(logits.detach().float().numpy(), bank_count=J, selected_banks=sel, bf16=bf16)
        idx = torch.from_numpy(idx)
    first = torch.gather(logits[..., :j1], -1, idx // j2)
    second = torch.gather(logits[..., j1:], -1, idx % j2)
    weights = torch.softmax((first + second).float(), dim=-1).to(logits.dtype)
    return weights, idx


def initial_state(p, cfg):
    """[J, H, S, dv] = U[row // Q] + Z[row % Q] in the parameter dtype."""
    H, S, J = cfg['num_heads'], cfg['bank_size'], cfg['bank_count']
    dv = cfg['value_width'] // H
    u, z = p['initial_row_factor'], p['initial_column_factor']
    return (u[:, None, :] + z[None, :, :]).reshape(J, H, S, dv)


def bank_reads(controls, routes, init, cfg, *, interval):
    """Packed recurrence; returns reads [NT, KR, H, dv] in the activation dtype."""
    q, k, v, g, b, w = controls
    ww, wi, rw, ri = routes
    batch, time, kw = wi.shape
    kr = ri.shape[-1]
    H, S = q.shape[-2], q.shape[-1]
    dv = v.shape[-1]
    J = cfg['bank_count']
    nt, nw = batch * time, batch * time * kw
    dt = v.dtype
    scale = S ** -0.5
    disp = oracle_dispatch(wi.numpy(), ri.numpy(), J)
    order, cu = disp['order'], disp['cu_seqlens']
    nseq = batch * J
    lens = cu[1:] - cu[:-1]
    lmax = int(lens.max()) if nseq else 0
    table = np.full((nseq, max(lmax, 1)), -1, np.int64)
    for s in range(nseq):
        table[s, :lens[s]] = order[cu[s]:cu[s + 1]]
    qf, kf, vf, gf, bf, wf = (t.reshape(nt, *t.shape[2:]) for t in (q, k, v, g, b, w))
    wwf, rwf = ww.reshape(-1), rw.reshape(-1)
    state = init.float().unsqueeze(0).expand(batch, -1, -1, -1, -1).reshape(nseq, H, S, dv)
    if interval:
        state = _StoredState.apply(state)
    read_ids, read_vals = [], []
    for i in range(lmax):
        if interval and i % interval == 0 and i > 0:
            state = _StoredState.apply(state)
        ids = table[:, i]
        wsel = np.nonzero((ids >= 0) & (ids < nw))[0]
        rsel = np.nonzero(ids >= nw)[0]
        if len(rsel):
            rid = torch.from_numpy(ids[rsel] - nw)
            tok = rid // kr
            qe = (qf[tok] * rwf[rid][:, None, None]).float()
            out = scale * (qe.unsqueeze(-1) * state[torch.from_numpy(rsel)]).sum(-2)
            read_ids.append(rid)
            read_vals.append(out.to(dt))
        if len(wsel):
            sel = torch.from_numpy(wsel)
            wid = torch.from_numpy(ids[wsel])
            tok = wid // kw
            pw = wwf[wid]
            key = kf[tok].float()
            be = (bf[tok] * pw[:, None, None]).float()
            ge = gf[tok].float() * pw.float()[:, None, None] if cfg['routed_decay'] else gf[tok].float()
            we = (wf[tok] * pw[:, None, None]).float()
            cur = state[sel] * ge.exp().unsqueeze(-1)
            erase = ((be * key).unsqueeze(-1) * cur).sum(-2)
            cur = cur + key.unsqueeze(-1) * (we * vf[tok].float() - erase).unsqueeze(-2)
            state = state.index_put((sel,), cur)
    reads = torch.zeros(nt * kr, H, dv, dtype=dt)
    if read_ids:
        reads = reads.index_put((torch.cat(read_ids),), torch.cat(read_vals))
    return reads.reshape(nt, kr, H * dv)


def project(p, x, raw, cfg):
    """_parameters.py:222-232: LayerNorm or RMS, sigmoid gate, o_proj."""
    V = cfg['value_width']
    gate = torch.sigmoid(_linear(x, p, 'output_gate.weight', 'output_gate.bias')).to(raw.dtype)
    if cfg['output_normalization'] == 'layer':
        n = F.layer_norm(raw, (V,), p['output_norm_weight'], p['output_norm_bias'], cfg['norm_eps'])
    else:
        var = raw.float().square().mean(-1, keepdim=True)
        n = raw * torch.rsqrt(var + cfg['norm_eps']).to(raw.dtype)
        n = n * p['output_norm_weight'].to(raw.dtype)
    return F.linear(n * gate, p['o_proj.weight'], p.get('o_proj.bias'))


def layer_forward(p: dict, x: torch.Tensor, cfg: dict, write_idx=None, read_idx=None) -> torch.Tensor:
    """Training forward of one layer: ``p`` maps state_dict names to (leaf) tensors;
    ``write_idx`` / ``read_idx`` optionally fix the bank selections (see ``route``)."""
    batch, time, _ = x.shape
    q, k, v, g, b, w = controllers(p, x, cfg)
    rl, wl = route_logits(p, x)
    ww, wi = route(wl, cfg, write_idx)
    rw, ri = route(rl, cfg, read_idx)
    interval = state_interval(cfg['bank_size']) if cfg['training_state_dtype'] == 'bfloat16' else 0
    reads = bank_reads((q, k, v, g, b, w), (ww, wi, rw, ri), initial_state(p, cfg), cfg, interval=interval)
    raw = reads.float().sum(1).to(x.dtype).reshape(batch, time, -1)
    return project(p, x, raw, cfg)


def layer_grads(state_dict: dict, x: torch.Tensor, dy: torch.Tensor, cfg: dict, write_idx=None, read_idx=None):
    """Gradients of <dy, layer_forward(x)>: (dict name -> grad, x grad, output)."""
    p = {n: t.detach().clone().requires_grad_(t.is_floating_point()) for n, t in state_dict.items()}
    xx = x.detach().clone().requires_grad_(True)
    y = layer_forward(p, xx, cfg, write_idx, read_idx)
    y.backward(dy)
    grads = {n: t.grad for n, t in p.items() if t.grad is not None}
    return grads, xx.grad, y.detach()
