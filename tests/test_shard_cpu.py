"""Bank-sharded forward host logic on CPU: partition rules and the collective choreography.

Two gloo ranks run ``BankShardedMemory.forward`` -- histogram all-reduce,
partition, all-gather of controller records and routes, per-rank bank stage,
reduce-scatter of FP32 read partials, output stage -- with every compute stage
replaced by the CPU oracle.  The ranks' outputs must equal the single-process
oracle forward of the whole batch up to the FP32 summation order of the read
combine.  The CUDA stages themselves are checked against the same oracle in
test_shard_gpu.py.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory
from bdm_b200.sharded import BankShardedMemory

CFG = dict(dim=64, bank_count=64, bank_size=8, selected_banks=4, value_width=64, num_heads=2)
BATCH, TIME = 4, 12


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _loads(counts, owner, world):
    return np.bincount(owner, weights=counts, minlength=world)


@pytest.mark.parametrize('world', [1, 2, 4, 8])
def test_partition_rules(world):
    rng = np.random.default_rng(world)
    J = 256
    counts = np.minimum(rng.zipf(1.3, J), 5000).astype(np.int32)
    for mode in ('contiguous', 'balanced'):
        owner, slot, members = oracle.oracle_bank_owners(counts, J, world, mode)
        assert members.shape == (world, J // world)
        assert sorted(members.ravel().tolist()) == list(range(J))   # a partition of the table
        for r in range(world):
            assert (np.diff(members[r]) > 0).all()                  # slots in ascending bank order
            assert (owner[members[r]] == r).all()
            assert (slot[members[r]] == np.arange(J // world)).all()
    c_owner = oracle.oracle_bank_owners(counts, J, world, 'contiguous')[0]
    assert (c_owner == np.arange(J) // (J // world)).all()
    b_owner = oracle.oracle_bank_owners(counts, J, world, 'balanced')[0]
    lb, lc = _loads(counts, b_owner, world), _loads(counts, c_owner, world)
    assert lb.max() <= lc.max()
    # dealing in groups keeps every rank within one heaviest bank of the mean
    assert lb.max() - lb.mean() <= counts.max()


class _FakeComm:
    def __init__(self, rank, world):
        self.rank, self.world = rank, world


@pytest.mark.parametrize('bank_count,world', [(32768, 2), (16384 * 4, 8), (16384, 64)])
def test_balanced_partition_beyond_its_limits_uses_contiguous_ranges(bank_count, world):
    cfg = BSDMConfig(dim=64, bank_count=bank_count, bank_size=8, selected_banks=4, value_width=32, num_heads=1)
    m = BlockSparseDeltaMemory(cfg, seed=0)
    with pytest.warns(UserWarning, match='contiguous'):
        sharded = BankShardedMemory(m, comm=_FakeComm(0, world), ownership='balanced')
    assert sharded.ownership == 'contiguous' and sharded.local_banks == bank_count // world
    # within the limits the requested partition stays
    small = BlockSparseDeltaMemory(BSDMConfig(dim=64, bank_count=256, bank_size=8, selected_banks=4, value_width=32,
                                              num_heads=1), seed=0)
    assert BankShardedMemory(small, comm=_FakeComm(0, 2), ownership='balanced').ownership == 'balanced'


class OracleStages(BankShardedMemory):
    """The sharded forward with every compute stage done by the CPU oracle."""

    def __init__(self, layer, olayer, **kw):
        super().__init__(layer, **kw)
        self.o = olayer

    def local_stage(self, hidden):
        x = self.o.r(hidden.float().numpy())
        lb, t, _ = x.shape
        q, k, v, g, b, w = self.o.controllers(x)
        rl, wl = self.o.route_logits(x)
        (ww, wi), (rw, ri) = self.o.route(wl), self.o.route(rl)
        controls = [torch.from_numpy(np.ascontiguousarray(c.reshape(lb * t, -1))) for c in (q, k, v, g, b, w)]
        routes = [torch.from_numpy(np.ascontiguousarray(a)) for a in (ww, wi, rw, ri)]
        return controls, routes, None

    def histogram(self, wi, ri):
        return torch.from_numpy(oracle.oracle_bank_histogram(wi.numpy(), ri.numpy(), self.layer.bank_count))

    def owners(self, counts):
        return tuple(torch.from_numpy(a) for a in oracle.oracle_bank_owners(
            counts.numpy(), self.layer.bank_count, self.world, self.ownership))

    def dispatch_stage(self, routes, owner, slot):
        return None  # the oracle recurrence orders events itself

    def bank_stage(self, controls, routes, meta, owner, members, *, batch, time):
        o = self.o
        q, k, v, g, b, w = (c.numpy().reshape(batch, time, o.H, -1) for c in controls)
        ww, wi, rw, ri = (r.numpy() for r in routes)
        interval = oracle.state_interval(o.S) if o.c['training_state_dtype'] == 'bfloat16' else 0
        init = o.initial_state()[None]
        reads, _ = oracle.oracle_recurrence(q, k, v, g, b, w, wi, ww, ri, rw, init,
                                            bank_count=o.J, bf16=o.bf16, routed_decay=o.c['routed_decay'],
                                            interval=interval, scale=o.S ** -0.5, want_state=False)
        kr = ri.shape[-1]
        part = oracle.oracle_combine_partial(reads.reshape(batch * time, kr, -1), ri.reshape(batch * time, kr),
                                             owner.numpy(), self.rank)
        return torch.from_numpy(part)

    def output_stage(self, hidden, combined, gate):
        raw = self.o.r(combined.numpy())   # the forward's round-once combine
        x = self.o.r(hidden.float().numpy()).reshape(-1, self.layer.hidden_size)
        return torch.from_numpy(self.o.project(x, raw))


def _model():
    m = BlockSparseDeltaMemory(BSDMConfig(**CFG), seed=5).to(torch.bfloat16)
    with torch.no_grad():  # a skewed router, so the balanced partition differs from the contiguous one
        m.shared_router.base.bias.copy_(torch.linspace(3.0, -3.0, m.shared_router.base.bias.numel()))
    params = {k: v.detach().float().numpy() for k, v in m.state_dict().items()}
    cfg = {k: getattr(m.config, k) for k in m.config.__dataclass_fields__}
    return m, oracle.OracleLayer(cfg, params, bf16=True)


def _hidden():
    return torch.randn(BATCH, TIME, CFG['dim'], generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)


def _worker(rank, world, port, mode, groups, out_dir):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        m, olayer = _model()
        x = _hidden()
        rows = BATCH // world
        sharded = OracleStages(m, olayer, ownership=mode, row_chunks=groups)
        y = sharded(x[rank * rows:(rank + 1) * rows])
        owner = sharded.last_partition[0]
        # the gather carries any element type bit for bit (bf16 controllers, int64 routes)
        comm = sharded.comm
        probe = [torch.full((3, 5), rank + 0.5, dtype=torch.bfloat16), torch.full((2, 4, 3), 7 * rank + 1)]
        gathered = [comm.all_gather(t).wait() for t in probe]
        torch.save({'y': y, 'owner': owner, 'gathered': gathered}, os.path.join(out_dir, f'rank{rank}.pt'))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('mode,groups', [('balanced', 2), ('contiguous', 1), ('balanced', 3)])
def test_sharded_forward_gloo_world2(tmp_path, mode, groups):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), mode, groups, str(tmp_path)), nprocs=world, join=True)
    m, olayer = _model()
    want = olayer.forward(olayer.r(_hidden().float().numpy()))
    parts = [torch.load(tmp_path / f'rank{r}.pt') for r in range(world)]
    got = np.concatenate([p['y'].float().numpy() for p in parts], 0)
    assert got.shape == want.shape
    # identical partitions on both ranks, and every rank owns half the table
    assert torch.equal(parts[0]['owner'], parts[1]['owner'])
    assert (np.bincount(parts[0]['owner'].numpy(), minlength=world) == CFG['bank_count'] // world).all()
    for p in parts:
        g16, g64 = p['gathered']
        assert g16.dtype == torch.bfloat16 and torch.equal(g16[:3], torch.full((3, 5), 0.5, dtype=torch.bfloat16))
        assert torch.equal(g16[3:], torch.full((3, 5), 1.5, dtype=torch.bfloat16))
        assert torch.equal(g64, torch.cat([torch.full((2, 4, 3), 1), torch.full((2, 4, 3), 8)]))
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= 1e-2, err   # FP32 read-sum order only: a few BF16 ulps at most
    assert np.mean(got == want) > 0.9
