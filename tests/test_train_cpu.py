"""Host logic of the training path (bdm_b200.layer._BankTraining) on the CPU.

The CUDA ops are replaced by shape-checking stand-ins, so only the autograd plumbing runs:
* every parameter of the layer receives a gradient, and the backward writes each column of
  the fused projection's gradient exactly once (q, k, v, b, w by the controllers backward,
  f1 by the f_proj.1 GEMM, the router blocks by the router backward, the gate block by the
  norm/gate backward);
* data parallelism: the LM shell under DistributedDataParallel (gloo, world size 2)
  all-reduces to the mean of the ranks' local gradients.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bdm_b200 import BDMConfig, BSDMConfig, BankedDeltaMemory
from bdm_b200 import layer as layer_mod
from bdm_b200 import ops


class _Recorder:
    def __init__(self):
        self.writes = []  # (first column, width) blocks written into d_proj

    def block(self, d_proj, first, width):
        d_proj[:, first:first + width] = 1.0
        self.writes.append((first, width))


def _install(set_attr, rec):
    """Replace the CUDA ops with CPU stand-ins; ``set_attr(obj, name, value)``."""
    def controllers(proj, cols, f, a_log, dt_bias, *, heads, bank_size, head_value_width, qk_norm, f_weight=None,
                    f1_width=0):
        nt, hs, v = proj.shape[0], heads * bank_size, heads * head_value_width
        assert f.shape == (nt, hs)
        return (proj[:, cols['q']:cols['q'] + hs].contiguous(), proj[:, cols['k']:cols['k'] + hs].contiguous(),
                proj[:, cols['v']:cols['v'] + v].contiguous(), proj[:, cols['q']:cols['q'] + hs].float().contiguous(),
                proj[:, cols['b']:cols['b'] + hs].contiguous(), proj[:, cols['w']:cols['w'] + v].contiguous())

    def route_pair(proj, first, second, *, bank_count, selected_banks, factors):
        nt = proj.shape[0]
        idx = (torch.arange(nt)[:, None] * 7 + torch.arange(selected_banks)[None, :]) % bank_count
        w = torch.softmax(proj[:, first:first + selected_banks].float(), -1).to(proj.dtype)
        return (w, idx), (w.clone(), idx.clone())

    def dispatch(wi, ri, bank_count):
        b, t, kw = wi.shape
        return dict(order=torch.arange(b * t * (kw + ri.shape[-1])),
                    cu_seqlens=torch.zeros(b * bank_count + 1, dtype=torch.long))

    def bank_scan(q, k, v, g, b, w, wi, ww, ri, rw, order, cu, *, batch, time, heads, head_value_width,
                  checkpoints=None, checkpoint_block=0, **kw):
        assert checkpoints is not None and checkpoint_block > 0
        return torch.zeros(batch * time, ri.shape[-1], heads * head_value_width, dtype=q.dtype)

    def combine_norm_gate(reads, ri, gate, nw, nb, *, eps, layer_norm, round_each, save_raw=False):
        assert save_raw and not round_each
        raw = reads.sum(1)
        return (raw * gate).to(reads.dtype), raw

    def norm_gate_backward(d_out, raw, gate, nw, nb, *, eps, layer_norm, d_gate):
        d_gate.fill_(1.0)
        rec.writes.append(('gate', d_gate.shape[1]))
        return d_out.clone(), torch.zeros(raw.shape[1]), torch.zeros(raw.shape[1]) if nb is not None else None

    def scan_backward(q, k, v, g, b, w, ww, rw, order, cu, d_raw, *, batch, time, bank_count, heads, bank_size,
                      head_value_width, kw, kr, routed_decay, scale, row_factor, col_factor, state_interval,
                      checkpoints=None):
        assert checkpoints is not None  # the forward's checkpoints reach the backward
        nt = batch * time
        return (torch.zeros(1, nt * (kw + kr), heads, 3 * bank_size), torch.zeros(nt * kw, heads * head_value_width),
                torch.zeros(batch * bank_count, heads, bank_size, head_value_width))

    def event_vjp(q, k, v, g, b, w, ww, rw, evg, du, *, heads, bank_size, head_value_width, routed_decay, scale):
        nt = q.shape[0]
        return (torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v), torch.zeros_like(g),
                torch.zeros_like(b), torch.zeros_like(w), torch.zeros(nt, heads, ww.shape[-1], dtype=ww.dtype),
                torch.zeros(nt, heads, rw.shape[-1], dtype=rw.dtype))

    def route_backward(proj, first, second, i1, w1, i2, w2, d_proj, *, bank_count, factors):
        assert w1.ndim == 3 and w2.ndim == 3  # per-head route-weight gradients
        width = sum(factors)
        rec.block(d_proj, first, width)
        rec.block(d_proj, second, width)

    def controllers_backward(proj, cols, f, a_log, dt_bias, g, b, w, dq, dk, dv, dg, db, dw, d_proj, *, heads,
                             bank_size, head_value_width, qk_norm):
        hs, v = heads * bank_size, heads * head_value_width
        for c, n in (('q', hs), ('k', hs), ('v', v), ('b', hs), ('w', v)):
            rec.block(d_proj, cols[c], n)
        return torch.zeros(proj.shape[0], hs, dtype=proj.dtype), torch.zeros(heads), torch.zeros(hs)

    def product_state_backward(dinit, *, batch, rows_p, cols_q, factor_dtype):
        return torch.zeros(rows_p, dinit.shape[-1]), torch.zeros(cols_q, dinit.shape[-1])

    for name, fn in dict(controllers=controllers, route_pair=route_pair, dispatch=dispatch, bank_scan=bank_scan,
                         combine_norm_gate=combine_norm_gate, norm_gate_backward=norm_gate_backward,
                         scan_backward=scan_backward, event_vjp=event_vjp, route_backward=route_backward,
                         controllers_backward=controllers_backward,
                         product_state_backward=product_state_backward).items():
        set_attr(ops, name, fn)


@pytest.mark.parametrize('cfg_cls,heads,dtype', [(BSDMConfig, 2, torch.float32), (BSDMConfig, 1, torch.bfloat16),
                                                  (BDMConfig, 1, torch.float32)])
def test_training_plumbing_covers_every_gradient(monkeypatch, cfg_cls, heads, dtype):
    rec = _Recorder()
    _install(monkeypatch.setattr, rec)
    cfg = cfg_cls(dim=64, bank_count=64, bank_size=8, selected_banks=4, value_width=32, num_heads=heads)
    m = BankedDeltaMemory(cfg, seed=1).to(dtype)
    x = torch.randn(2, 5, 64).to(dtype).requires_grad_(True)
    weight, bias, cols = m._fused_projection_autograd()
    proj = torch.addmm(bias, x.reshape(10, 64), weight.t())
    normed = layer_mod._BankTraining.apply(proj, m.f_proj[1].weight, m.A_log, m.dt_bias, m.initial_row_factor,
                                           m.initial_column_factor, m.output_norm_weight,
                                           getattr(m, 'output_norm_bias', None), m, cols, 2, 5)
    torch.nn.functional.linear(normed, m.o_proj.weight, m.o_proj.bias).sum().backward()
    assert [n for n, p in m.named_parameters() if p.grad is None] == []
    assert x.grad is not None
    # every column block of d proj written exactly once: kernels' blocks + f1 (GEMM) + gate
    covered = torch.zeros(proj.shape[1], dtype=torch.int32)
    for first, width in rec.writes:
        if first == 'gate':
            covered[cols['gate']:cols['gate'] + width] += 1
        else:
            covered[first:first + width] += 1
    covered[cols['f']:cols['f'] + m.head_value_width] += 1  # torch.mm(df, f_proj.1 weight)
    assert torch.equal(covered, torch.ones_like(covered))


def test_training_rejects_wide_heads_before_any_work():
    # H = 1 with value_width 512: the backward's event VJP supports head_value_width <= 256, so the
    # training forward refuses up front instead of failing in backward after the forward ran
    cfg = BSDMConfig(dim=64, bank_count=64, bank_size=8, selected_banks=4, value_width=512, num_heads=1)
    m = BankedDeltaMemory(cfg, seed=1)
    with pytest.raises(NotImplementedError, match='head_value_width'):
        m._forward_train(torch.randn(1, 4, 64, requires_grad=True))


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _lm():
    from bdm_b200 import LanguageModelConfig
    from bdm_b200.lm import BDMLanguageModel
    mem = BSDMConfig(dim=32, bank_count=16, bank_size=8, selected_banks=4, value_width=32, num_heads=2,
                     training_state_dtype='float32')
    return BDMLanguageModel(LanguageModelConfig(memory=mem, vocab_size=40, layers=2, seed=3, ffn_multiple_of=32))


def _tokens(rank):
    gen = torch.Generator().manual_seed(100 + rank)
    return torch.randint(0, 40, (2, 6), generator=gen), torch.randint(0, 40, (2, 6), generator=gen)


def _allow_cpu(set_attr):
    """The layer refuses CPU tensors (it has no CPU path); with the ops stubbed, let them through."""
    set_attr(BankedDeltaMemory, '_check_hidden', lambda self, hidden: None)


def _ddp_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        _install(setattr, _Recorder())
        _allow_cpu(setattr)
        model = torch.nn.parallel.DistributedDataParallel(_lm())
        tokens, target = _tokens(rank)
        model(tokens, target).backward()
        torch.save({n: p.grad for n, p in model.module.named_parameters()}, os.path.join(out_dir, f'g{rank}.pt'))
    finally:
        dist.destroy_process_group()


def test_lm_data_parallel_gloo_world2(monkeypatch, tmp_path):
    world = 2
    mp.spawn(_ddp_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    _install(monkeypatch.setattr, _Recorder())
    _allow_cpu(monkeypatch.setattr)
    local = []
    for rank in range(world):  # each rank's local gradients, without DDP
        m = _lm()
        tokens, target = _tokens(rank)
        m(tokens, target).backward()
        local.append({n: p.grad for n, p in m.named_parameters()})
    got = [torch.load(tmp_path / f'g{r}.pt') for r in range(world)]
    for n in local[0]:
        want = (local[0][n] + local[1][n]) / world
        assert torch.equal(got[0][n], got[1][n]), n  # every rank holds the same all-reduced gradient
        assert torch.allclose(got[0][n], want, rtol=1e-5, atol=1e-7), n
