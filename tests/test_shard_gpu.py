"""Bank-sharded forward on the GPU, through the C ABI.

Bit-exact against the oracle restatement (oracle/shard.py): per-bank histogram,
bank partition (contiguous and balanced), owned dispatch, partial combine.
Bit-exact against the single-device path: the recurrence of one rank's banks
(local sequences, product-key initial state through the local->global bank
map) reproduces the single-device reads of those banks' events, and the FP32
norm-gate over a one-rank partial equals the round-once combine.
End to end: two ranks (gloo, sharing cuda:0, or NCCL over two GPUs when the
box has them) against the single-device forward of the whole batch, to the
FP32 summation order of the read combine.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory, near_square_factors, ops, state_interval
from bdm_b200.sharded import BankShardedMemory

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def _routes(gen, batch, time, bank_count, k, skew=0.0):
    """Distinct banks per token; with skew > 0 low bank ids are favoured (hot banks)."""
    scores = torch.rand(batch * time, bank_count, generator=gen)
    if skew:
        scores = scores + skew * torch.linspace(1.0, 0.0, bank_count)
    return scores.topk(k, dim=-1).indices.reshape(batch, time, k)


@pytest.mark.parametrize('bank_count', [256, 16384, 65536])
def test_histogram_bit_exact(bank_count):
    gen = torch.Generator().manual_seed(bank_count)
    wi = torch.randint(0, bank_count, (3, 257, 8), generator=gen)
    ri = torch.randint(0, bank_count, (3, 257, 6), generator=gen)
    wi[0, 0, 0] = 0  # a hot bank
    wi[:, :, 1] = 0
    got = ops.bank_histogram(wi.to(DEV), ri.to(DEV), bank_count).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.oracle_bank_histogram(wi.numpy(), ri.numpy(), bank_count))


@pytest.mark.parametrize('bank_count,world', [(256, 1), (256, 2), (256, 8), (1024, 4), (16384, 8), (16384, 2),
                                              (96, 32), (3072, 3)])
def test_owners_bit_exact(bank_count, world):
    rng = np.random.default_rng(bank_count + world)
    counts = np.minimum(rng.zipf(1.2, bank_count), 1 << 20).astype(np.int32)
    counts[rng.integers(0, bank_count, bank_count // 4)] = 7  # many equal counts: index ties
    counts[:3] = 0
    ct = torch.from_numpy(counts).to(DEV)
    for mode in ('contiguous', 'balanced'):
        got = ops.bank_owners(ct, bank_count, world, mode=mode)
        want = oracle.oracle_bank_owners(counts, bank_count, world, mode)
        for g, w in zip(got, want):
            np.testing.assert_array_equal(g.cpu().numpy(), w)


@pytest.mark.parametrize('world', [2, 4])
def test_dispatch_owned_bit_exact(world):
    gen = torch.Generator().manual_seed(world)
    batch, time, J = 2, 96, 256
    wi = _routes(gen, batch, time, J, 8, skew=2.0)
    ri = _routes(gen, batch, time, J, 8, skew=2.0)
    counts = oracle.oracle_bank_histogram(wi.numpy(), ri.numpy(), J)
    owner, slot, _ = ops.bank_owners(torch.from_numpy(counts).to(DEV), J, world, mode='balanced')
    total = 0
    for rank in range(world):
        meta = ops.dispatch_owned(wi.to(DEV), ri.to(DEV), J, owner, slot, rank, J // world)
        order, cu = oracle.oracle_dispatch_owned(wi.numpy(), ri.numpy(), J, owner.cpu().numpy(), slot.cpu().numpy(),
                                                 rank, J // world)
        np.testing.assert_array_equal(meta['cu_seqlens'].cpu().numpy(), cu)
        np.testing.assert_array_equal(meta['order'].cpu().numpy(), order)
        total += int(cu[-1])
    assert total == batch * time * 16  # every event owned exactly once


def _layer(cfg, seed, dtype):
    m = BlockSparseDeltaMemory(BSDMConfig(**cfg), seed=seed).to(dtype).to(DEV)
    with torch.no_grad():
        m.shared_router.base.bias.add_(torch.linspace(2.0, -2.0, m.shared_router.base.bias.numel(), device=DEV)
                                       .to(dtype))
    m._fused_cache = None
    return m


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
@pytest.mark.parametrize('world', [2, 4])
def test_owned_recurrence_reproduces_single_device_reads(dtype, world):
    cfg = dict(dim=128, bank_count=256, bank_size=8, selected_banks=8, value_width=256, num_heads=2)
    m = _layer(cfg, 11, dtype)
    batch, time = 2, 200
    x = torch.randn(batch, time, cfg['dim'], generator=torch.Generator().manual_seed(3)).to(dtype).to(DEV)
    J, H, S, dv = m.bank_count, m.num_heads, m.bank_size, m.head_value_width
    interval = state_interval(S)
    common = dict(batch=batch, time=time, heads=H, bank_size=S, head_value_width=dv, routed_decay=True,
                  scale=S ** -0.5, row_factor=m.initial_row_factor, col_factor=m.initial_column_factor,
                  state_interval=interval)
    with torch.no_grad():
        controls, routes, _ = m._controls_and_routes(x)
        ww, wi, rw, ri = routes
        meta = ops.dispatch(wi, ri, J)
        full = ops.bank_scan(*controls, wi, ww, ri, rw, meta['order'], meta['cu_seqlens'], bank_count=J, **common)
        counts = ops.bank_histogram(wi, ri, J)
        owner, slot, members = ops.bank_owners(counts, J, world, mode='balanced')
        summed = torch.zeros(batch * time, m.value_width, dtype=torch.float32, device=DEV)
        for rank in range(world):
            mo = ops.dispatch_owned(wi, ri, J, owner, slot, rank, J // world)
            local = ops.bank_scan(*controls, wi, ww, ri, rw, mo['order'], mo['cu_seqlens'], bank_count=J // world,
                                  bank_ids=members[rank], total_banks=J, **common)
            mine = (owner[ri.reshape(-1)] == rank).reshape(batch * time, -1)
            assert torch.equal(local[mine], full[mine])
            part = ops.combine_partial(local, ri.reshape(batch * time, -1), owner, rank)
            want = oracle.oracle_combine_partial(local.float().cpu().numpy(), ri.reshape(batch * time, -1).cpu(),
                                                 owner.cpu().numpy(), rank)
            np.testing.assert_array_equal(part.cpu().numpy(), want)
            summed += part
        # the sum of partials is the full FP32 read sum up to association
        one = ops.combine_partial(full, ri.reshape(batch * time, -1), torch.zeros_like(owner), 0)
        torch.testing.assert_close(summed, one, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_head_group_recurrence_reproduces_all_head_reads(dtype):
    cfg = dict(dim=128, bank_count=256, bank_size=4, selected_banks=8, value_width=512, num_heads=4)
    m = _layer(cfg, 12, dtype)
    batch, time = 2, 150
    x = torch.randn(batch, time, cfg['dim'], generator=torch.Generator().manual_seed(5)).to(dtype).to(DEV)
    J, H, S, dv = m.bank_count, m.num_heads, m.bank_size, m.head_value_width
    common = dict(batch=batch, time=time, bank_size=S, head_value_width=dv, routed_decay=True, scale=S ** -0.5,
                  row_factor=m.initial_row_factor, col_factor=m.initial_column_factor, state_interval=state_interval(S))
    with torch.no_grad():
        controls, routes, _ = m._controls_and_routes(x)
        ww, wi, rw, ri = routes
        counts = ops.bank_histogram(wi, ri, J)
        owner, slot, members = ops.bank_owners(counts, J, 2, mode='balanced')
        mo = ops.dispatch_owned(wi, ri, J, owner, slot, 1, J // 2)
        full = ops.bank_scan(*controls, wi, ww, ri, rw, mo['order'], mo['cu_seqlens'], bank_count=J // 2, heads=H,
                             bank_ids=members[1], total_banks=J, **common)
        mine = (owner[ri.reshape(-1)] == 1).reshape(batch * time, -1)
        for h0, h1 in ((0, 2), (2, 3), (3, 4)):
            part = [c.reshape(batch * time, H, -1)[:, h0:h1].reshape(batch * time, -1).contiguous() for c in controls]
            got = ops.bank_scan(*part, wi, ww, ri, rw, mo['order'], mo['cu_seqlens'], bank_count=J // 2,
                                heads=h1 - h0, bank_ids=members[1], total_banks=J, head_offset=h0, total_heads=H,
                                **common)
            assert torch.equal(got[mine], full[mine][:, h0 * dv:h1 * dv])


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
@pytest.mark.parametrize('layer_norm', [True, False])
def test_norm_gate_f32_equals_round_once_combine(dtype, layer_norm):
    gen = torch.Generator().manual_seed(4)
    nt, kr, width, J = 300, 8, 512, 64
    reads = torch.randn(nt, kr, width, generator=gen).to(dtype).to(DEV)
    ri = torch.stack([torch.randperm(J, generator=gen)[:kr] for _ in range(nt)]).to(DEV)
    gate = torch.randn(nt, width + 16, generator=gen).to(dtype).to(DEV)[:, :width]
    nw = (1 + 0.1 * torch.randn(width, generator=gen)).to(DEV)
    nb = 0.1 * torch.randn(width, generator=gen).to(DEV) if layer_norm else None
    want = ops.combine_norm_gate(reads, ri, gate, nw, nb, eps=1e-5, layer_norm=layer_norm, round_each=False)
    owner = torch.zeros(J, dtype=torch.int32, device=DEV)
    combined = ops.combine_partial(reads, ri, owner, 0)
    got = ops.norm_gate_f32(combined, gate, nw, nb, eps=1e-5, layer_norm=layer_norm, dtype=dtype)
    assert torch.equal(got, want)


# ------------------------------------------------------------ end to end
SHARD_CFG = dict(dim=256, bank_count=1024, bank_size=16, selected_banks=16, value_width=512, num_heads=4)
SHARD_BATCH, SHARD_TIME = 4, 256


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _shard_inputs():
    return torch.randn(SHARD_BATCH, SHARD_TIME, SHARD_CFG['dim'],
                       generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)


def _shard_worker(rank, world, port, backend, mode, groups, out_dir):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dev = torch.device('cuda', rank if backend == 'nccl' else 0)
    torch.cuda.set_device(dev)
    kw = dict(device_id=dev) if backend == 'nccl' else {}
    dist.init_process_group(backend, rank=rank, world_size=world, **kw)
    try:
        m = BlockSparseDeltaMemory(BSDMConfig(**SHARD_CFG), seed=3).to(torch.bfloat16).to(dev)
        with torch.no_grad():
            m.shared_router.base.bias.add_(torch.linspace(3.0, -3.0, m.shared_router.base.bias.numel())
                                           .to(torch.bfloat16).to(dev))
        m._fused_cache = None
        rows = SHARD_BATCH // world
        x = _shard_inputs()[rank * rows:(rank + 1) * rows].to(dev)
        y = BankShardedMemory(m, ownership=mode, row_chunks=groups)(x)
        torch.cuda.synchronize()
        torch.save(y.cpu(), os.path.join(out_dir, f'rank{rank}.pt'))
    finally:
        dist.destroy_process_group()


def _single_device_reference():
    m = BlockSparseDeltaMemory(BSDMConfig(**SHARD_CFG), seed=3).to(torch.bfloat16).to(DEV)
    with torch.no_grad():
        m.shared_router.base.bias.add_(torch.linspace(3.0, -3.0, m.shared_router.base.bias.numel())
                                       .to(torch.bfloat16).to(DEV))
        m._fused_cache = None
        return m(_shard_inputs().to(DEV)).float().cpu()


@pytest.mark.parametrize('mode,groups', [('balanced', 2), ('contiguous', 1)])
def test_sharded_forward_two_ranks_one_gpu(tmp_path, mode, groups):
    world = 2
    mp.spawn(_shard_worker, args=(world, _free_port(), 'gloo', mode, groups, str(tmp_path)), nprocs=world,
             join=True)
    got = torch.cat([torch.load(tmp_path / f'rank{r}.pt') for r in range(world)]).float()
    want = _single_device_reference()
    err = ((got - want).abs().max() / want.abs().max()).item()
    assert err <= 1e-2, err
    assert (got == want).float().mean().item() > 0.9


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs two GPUs')
def test_sharded_forward_nccl():
    world = 4 if torch.cuda.device_count() >= 4 else 2
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_shard_worker, args=(world, _free_port(), 'nccl', 'balanced', 2, d), nprocs=world, join=True)
        got = torch.cat([torch.load(os.path.join(d, f'rank{r}.pt')) for r in range(world)]).float()
    want = _single_device_reference()
    err = ((got - want).abs().max() / want.abs().max()).item()
    assert err <= 1e-2, err
