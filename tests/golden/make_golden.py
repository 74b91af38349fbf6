"""Generate golden vectors from the reference implementation itself.

Run where the reference checkout is present.  Its ``implementation`` directory is
imported from ``$BDM_REFERENCE``, by default ``reference/implementation`` beside this
repository's root directory:

    python tests/golden/make_golden.py

Writes small ``.pt`` fixtures next to this script.  The tests only read the
fixtures, so they run where the reference is absent (for example on the GPU
box).  Every fixture records which reference function produced it.

Fixtures:
  router.pt     product_key_route (gdn2_banks.py:74-114) on BF16/FP32 logits
                for the c1/c2 (16x16), c3 (32x64) and c4 (128x128) tables,
                including batch_factors=True (decode) and tie-heavy inputs.
  dispatch.pt   pack_bank_events (gdn2_banks.py:117-262): order, cu_seqlens, tokens.
  recurrence.pt reference_packed_gdn2 + scatter_bank_outputs (BF16 storage
                policy) and serial_banked_gdn2 (FP32 equation oracle).
  layer_*.pt    BlockSparseDeltaMemory(backend='reference').forward on small
                configs (FP32 and BF16, H=1 and H=2) with their state_dicts,
                controller tensors and router logits; plus c1 at T=64.
  lm_small.pt   BDMLanguageModel(backend='reference') at a small geometry: its seeded
                initial state_dict, and the loss and gradients of one training step.
  grad_*.pt     torch autograd through the same reference forward (backend='reference'):
                the gradients of every parameter and of the input for a seeded
                output cotangent, on BSDMConfig (routed decay, 'nvidia' q/k norm,
                LayerNorm) and BDMConfig (plain decay, 'original' norm, RMS) layers.
"""
from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get('BDM_REFERENCE',
                     os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))), 'reference',
                                  'implementation'))
sys.path.insert(0, REF)

from bdm.gdn2_banks import (pack_bank_events, product_key_route, reference_packed_gdn2,  # noqa: E402
                            scatter_bank_outputs, serial_banked_gdn2)
from bdm import BankedDeltaMemory, BDMConfig, BDMLanguageModel, LanguageModelConfig  # noqa: E402
from bsdm import BlockSparseDeltaMemory, BSDMConfig  # noqa: E402


def _route_cases():
    cases = []
    gen = torch.Generator().manual_seed(11)
    for (bank_count, selected, ntok) in ((256, 8, 512), (2048, 8, 256), (16384, 16, 64), (64, 4, 256)):
        j1 = int(bank_count ** 0.5)
        while bank_count % j1:
            j1 -= 1
        width = j1 + bank_count // j1
        for dtype in (torch.float32, torch.bfloat16):
            logits = torch.randn(1, ntok, width, generator=gen).to(dtype)
            w, i = product_key_route(logits, bank_count=bank_count, selected_banks=selected)
            wb, ib = product_key_route(logits, bank_count=bank_count, selected_banks=selected, batch_factors=True)
            cases.append(dict(kind='random', bank_count=bank_count, selected=selected, logits=logits,
                              weights=w, indices=i, weights_batch=wb, indices_batch=ib))
        # tie-heavy: small integers make exact ties common at both stages
        logits = torch.randint(-3, 4, (1, ntok, width), generator=gen).to(torch.bfloat16)
        w, i = product_key_route(logits, bank_count=bank_count, selected_banks=selected)
        cases.append(dict(kind='ties', bank_count=bank_count, selected=selected, logits=logits, weights=w,
                          indices=i, weights_batch=None, indices_batch=None))
    return cases


def _controls(gen, batch, time, heads, s, dv, dtype):
    q = torch.nn.functional.normalize(torch.randn(batch, time, heads, s, generator=gen), dim=-1).to(dtype)
    k = torch.nn.functional.normalize(torch.randn(batch, time, heads, s, generator=gen), dim=-1).to(dtype)
    v = torch.randn(batch, time, heads, dv, generator=gen).to(dtype)
    g = -torch.rand(batch, time, heads, s, generator=gen) * 0.5
    b = torch.rand(batch, time, heads, s, generator=gen).to(dtype)
    w = torch.rand(batch, time, heads, dv, generator=gen).to(dtype)
    return q, k, v, g, b, w


def _routes(gen, batch, time, bank_count, selected, dtype):
    j1 = int(bank_count ** 0.5)
    while bank_count % j1:
        j1 -= 1
    width = j1 + bank_count // j1
    wl = torch.randn(batch, time, width, generator=gen).to(dtype)
    rl = torch.randn(batch, time, width, generator=gen).to(dtype)
    ww, wi = product_key_route(wl, bank_count=bank_count, selected_banks=selected)
    rw, ri = product_key_route(rl, bank_count=bank_count, selected_banks=selected)
    return wl, rl, ww, wi, rw, ri


def make_dispatch():
    gen = torch.Generator().manual_seed(12)
    out = []
    for (batch, time, bank_count, selected) in ((2, 64, 256, 8), (3, 40, 64, 4), (1, 7, 16, 2)):
        _, _, ww, wi, rw, ri = _routes(gen, batch, time, bank_count, selected, torch.float32)
        s = 8
        q, k, v, g, b, w = (x[:, :, 0] for x in _controls(gen, batch, time, 1, s, 4, torch.float32))
        ev = pack_bank_events(q, k, v, g, b, w, wi, ww, ri, rw, bank_count=bank_count, kernel_key_width=s,
                              routed_decay=True)
        # recover the argsort order from the packed token/role columns
        write_tokens = torch.arange(batch * time).repeat_interleave(selected)
        keys_w = ((wi.reshape(-1) + torch.arange(batch).repeat_interleave(time * selected) * bank_count) * time
                  + (write_tokens % time)) * 2
        keys_r = ((ri.reshape(-1) + torch.arange(batch).repeat_interleave(time * selected) * bank_count) * time
                  + (write_tokens % time)) * 2 + 1
        order = torch.argsort(torch.cat((keys_w, keys_r)))
        out.append(dict(batch=batch, time=time, bank_count=bank_count, selected=selected, wi=wi, ri=ri,
                        order=order, cu_seqlens=ev.cu_seqlens, tokens=ev.token_indices,
                        read_events=ev.read_events))
    return out


def make_recurrence():
    gen = torch.Generator().manual_seed(13)
    out = []
    for dtype in (torch.float32, torch.bfloat16):
        batch, time, bank_count, selected, s, dv = 2, 48, 16, 4, 8, 16
        q, k, v, g, b, w = (x[:, :, 0] for x in _controls(gen, batch, time, 1, s, dv, dtype))
        _, _, ww, wi, rw, ri = _routes(gen, batch, time, bank_count, selected, dtype)
        init = (0.1 * torch.randn(bank_count, s, dv, generator=gen)).to(dtype)
        ev = pack_bank_events(q, k, v, g, b, w, wi, ww, ri, rw, bank_count=bank_count, kernel_key_width=s,
                              routed_decay=True)
        initial = init.unsqueeze(0).expand(batch, -1, -1, -1).reshape(batch * bank_count, 1, s, dv).float()
        packed = {}
        for state_dtype, interval in ((torch.float32, 16), (torch.bfloat16, 16), (torch.bfloat16, 4)):
            vals = reference_packed_gdn2(q=ev.q, k=ev.k, v=ev.v, g=ev.g, b=ev.b, w=ev.w, scale=s ** -0.5,
                                         initial_state=initial, cu_seqlens=ev.cu_seqlens, state_dtype=state_dtype,
                                         state_interval=interval)
            raw = scatter_bank_outputs(vals, ev.token_indices, batch=batch, time=time)
            packed[(str(state_dtype), interval)] = raw
        serial_out, serial_state = serial_banked_gdn2(q.float(), k.float(), v.float(), g, b.float(), w.float(),
                                                      init.float().unsqueeze(0).expand(batch, -1, -1, -1),
                                                      wi, ww.float(), ri, rw.float(), scale=s ** -0.5,
                                                      routed_decay=True)
        out.append(dict(dtype=str(dtype), batch=batch, time=time, bank_count=bank_count, selected=selected,
                        bank_size=s, dv=dv, q=q, k=k, v=v, g=g, b=b, w=w, ww=ww, wi=wi, rw=rw, ri=ri, init=init,
                        packed=packed, serial_out=serial_out, serial_state=serial_state))
    return out


def make_layer(name, cfg, batch, time, dtype, seed=0, x_seed=0, factor_std=None):
    m = BlockSparseDeltaMemory(cfg, seed=seed, backend='reference')
    if factor_std is not None:
        g = torch.Generator().manual_seed(x_seed)
        with torch.no_grad():
            m.initial_row_factor.copy_(torch.randn(m.initial_row_factor.shape, generator=g) * factor_std)
            m.initial_column_factor.copy_(torch.randn(m.initial_column_factor.shape, generator=g) * factor_std)
    m = m.to(dtype)
    torch.manual_seed(x_seed)
    x = torch.randn(batch, time, cfg.dim).to(dtype)
    with torch.no_grad():
        y = m(x)
        controls = m._controllers(x)
        rl, wl = m._route_projections(x)
        ww, wi = m._route(wl, m.num_writes)
        rw, ri = m._route(rl, m.num_reads)
    cfg_dict = {k: getattr(cfg, k) for k in cfg.__dataclass_fields__}
    torch.save(dict(config=cfg_dict, dtype=str(dtype), seed=seed, state_dict=m.state_dict(), x=x, out=y,
                    controls=controls, read_logits=rl, write_logits=wl,
                    routes=dict(ww=ww, wi=wi, rw=rw, ri=ri),
                    source='bsdm.BlockSparseDeltaMemory(backend="reference").forward'),
               os.path.join(HERE, f'layer_{name}.pt'))


def make_grad(name, cls, cfg, batch, time, dtype, seed=0, x_seed=0):
    """Gradients of <dy, layer(x)> for every parameter and for x (reference autograd)."""
    m = cls(cfg, seed=seed, backend='reference').to(dtype)
    gen = torch.Generator().manual_seed(1000 + x_seed)
    x = torch.randn(batch, time, cfg.dim, generator=gen).to(dtype).requires_grad_(True)
    y = m(x)
    dy = torch.randn(y.shape, generator=gen).to(dtype)
    y.backward(dy)
    grads = {n: p.grad.detach().clone() for n, p in m.named_parameters() if p.grad is not None}
    with torch.no_grad():  # the reference's own selections: torch.topk orders BF16 ties its own way
        rl, wl = m._route_projections(x)
        wi = m._route(wl, m.num_writes)[1]
        ri = m._route(rl, m.num_reads)[1]
    cfg_dict = {k: getattr(cfg, k) for k in cfg.__dataclass_fields__}
    torch.save(dict(config=cfg_dict, config_class='BSDM' if isinstance(cfg, BSDMConfig) else 'BDM',
                    dtype=str(dtype), seed=seed, state_dict={k: v.detach() for k, v in m.state_dict().items()},
                    x=x.detach(), out=y.detach(), dy=dy, x_grad=x.grad.detach(), grads=grads, write_idx=wi, read_idx=ri,
                    source=f'{cls.__module__}.{cls.__name__}(backend="reference"): torch autograd of <dy, forward(x)>'),
               os.path.join(HERE, f'grad_{name}.pt'))


def make_lm():
    """Small LM: seeded initial parameters, loss and gradients of one step (FP32, FP32 state storage)."""
    mem = BSDMConfig(dim=64, bank_count=64, bank_size=8, selected_banks=4, value_width=32, num_heads=2,
                     training_state_dtype='float32')
    cfg = LanguageModelConfig(memory=mem, vocab_size=96, layers=2, seed=1)
    m = BDMLanguageModel(cfg, backend='reference')
    init = {k: v.detach().clone() for k, v in m.state_dict().items()}
    gen = torch.Generator().manual_seed(44)
    tokens = torch.randint(0, cfg.vocab_size, (2, 24), generator=gen)
    target = torch.randint(0, cfg.vocab_size, (2, 24), generator=gen)
    loss = m(tokens, target)
    loss.backward()
    grads = {n: p.grad.detach().clone() for n, p in m.named_parameters() if p.grad is not None}
    mem_dict = {k: getattr(mem, k) for k in mem.__dataclass_fields__}
    torch.save(dict(memory=mem_dict, vocab_size=cfg.vocab_size, layers=cfg.layers, seed=cfg.seed,
                    ffn_multiple_of=cfg.ffn_multiple_of, state_dict=init, tokens=tokens, target=target,
                    loss=loss.detach(), grads=grads,
                    source='bdm.BDMLanguageModel(backend="reference"): init, cross-entropy loss and its gradients'),
               os.path.join(HERE, 'lm_small.pt'))


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    torch.save(dict(cases=_route_cases(), source='bdm.gdn2_banks.product_key_route'), os.path.join(HERE, 'router.pt'))
    torch.save(dict(cases=make_dispatch(), source='bdm.gdn2_banks.pack_bank_events'),
               os.path.join(HERE, 'dispatch.pt'))
    torch.save(dict(cases=make_recurrence(),
                    source='bdm.gdn2_banks.reference_packed_gdn2 + scatter_bank_outputs; serial_banked_gdn2'),
               os.path.join(HERE, 'recurrence.pt'))
    small = dict(dim=64, bank_count=64, bank_size=8, selected_banks=4, value_width=32)
    make_layer('h1_fp32', BSDMConfig(**small, num_heads=1), 2, 40, torch.float32)
    make_layer('h1_fp32_state32', BSDMConfig(**small, num_heads=1, training_state_dtype='float32'), 2, 40,
               torch.float32)
    make_layer('h1_bf16', BSDMConfig(**small, num_heads=1), 2, 40, torch.bfloat16)
    make_layer('h2_bf16', BSDMConfig(**small, num_heads=2), 2, 40, torch.bfloat16, seed=3)
    make_layer('h2_fp32_state32', BSDMConfig(**small, num_heads=2, training_state_dtype='float32'), 2, 40,
               torch.float32, seed=3)
    c1 = BSDMConfig(dim=256, bank_count=256, bank_size=8, selected_banks=8, value_width=64, num_heads=1)
    make_layer('c1_t64', c1, 2, 64, torch.float32, seed=0, x_seed=0, factor_std=0.02 / 2 ** 0.5)
    make_lm()
    make_grad('h1_fp32_state32', BlockSparseDeltaMemory,
              BSDMConfig(**small, num_heads=1, training_state_dtype='float32'), 2, 40, torch.float32, seed=1)
    make_grad('h2_fp32_state32', BlockSparseDeltaMemory,
              BSDMConfig(**small, num_heads=2, training_state_dtype='float32'), 2, 40, torch.float32, seed=2)
    make_grad('h2_bf16', BlockSparseDeltaMemory, BSDMConfig(**small, num_heads=2), 2, 40, torch.bfloat16, seed=3)
    make_grad('bdm_h1_fp32_state32', BankedDeltaMemory,
              BDMConfig(**small, num_heads=1, training_state_dtype='float32'), 2, 40, torch.float32, seed=4)
    make_grad('bdm_h2_bf16', BankedDeltaMemory, BDMConfig(**small, num_heads=2), 2, 40, torch.bfloat16, seed=5)
    print('golden fixtures written to', HERE)


if __name__ == '__main__':
    main()
