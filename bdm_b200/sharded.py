"""Bank-sharded BDM forward: one bank table partitioned over the GPUs of a node.

The reference runs the whole layer on one device (implementation/bdm/model.py:88-140).
For large memories -- J >= 16K banks, e.g. 16 x 8192 tokens over J = 16384
banks of 16 x 128 per head, 16 GiB of bank state -- this module splits the
bank table over R ranks (one process per GPU, ``torch.distributed``):

* tokens are sharded by batch row: rank r holds global rows [r*B/R, (r+1)*B/R)
  and runs the fused projection, controllers and router on them;
* the per-bank event counts are all-reduced and every rank derives the same
  bank partition (``ops.bank_owners``): balanced by load by default, so a
  Zipf-skewed router does not pile the hot banks onto one rank; contiguous
  index ranges on request.  Every rank owns J/R banks;
* the controller records and routes of all tokens are all-gathered.  Under a
  balanced partition a token's 2*B routed banks land on nearly every rank, so
  shipping one record per (token, rank) pair would move the same bytes as the
  all-gather; the all-gather is the MoE-style exchange in its dense form;
* each rank sorts the events of its own banks (``ops.dispatch_owned``), runs
  the recurrence over its banks' sequences (``ops.bank_scan`` with local bank
  ids mapped into the full table for the product-key initial state), and sums,
  per token, the reads of its banks in ascending bank order (FP32);
* a reduce-scatter sums the FP32 partials and returns each token's read sum to
  the rank that holds the token, which rounds it once to the activation dtype
  (the forward's round-once combine) and applies norm, gate and o_proj.

The exchange runs in row chunks: chunk c holds local batch row(s) c of every
rank, whose bank sequences are independent of the other chunks'.  Each chunk
runs on its own CUDA stream: its recurrence starts as soon as its all-gather
lands, so the gather of chunk c+1 overlaps the recurrence of chunk c, its
reduce-scatter starts as soon as its partial combine ends, and the chunks'
longest bank sequences (the critical path of a skewed router) run side by side.

Results match the single-device forward up to the FP32 summation order of the
read combine (the partials are added across ranks, not bank by bank).
Every rank must call ``forward`` with the same [B/R, T, D] shape.

The stages (``local_stage``, ``histogram``, ``owners``, ``dispatch_stage``,
``bank_stage``, ``output_stage``) are methods so that the collective
choreography in ``forward`` can be exercised with other stage implementations
(the CPU tests run it over gloo with the CPU oracle's stages).
"""
from __future__ import annotations

import warnings

import torch
import torch.distributed as dist
from torch.nn import functional as F

from . import ops
from .config import state_interval


class _Ready:
    """A collective result that is already complete."""

    def __init__(self, value):
        self.value = value

    def wait(self):
        return self.value


class _InFlight:
    """An asynchronous NCCL collective; ``wait`` orders the current stream after it."""

    def __init__(self, value, work):
        self.value, self.work = value, work

    def wait(self):
        self.work.wait()
        return self.value


class _NoStream:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


class ShardComm:
    """The collectives of the sharded forward over a ``torch.distributed`` group.

    NCCL moves device tensors directly and asynchronously (on its own stream).
    With gloo (CPU tests, or several ranks sharing one GPU) device tensors are
    staged through host memory, every call completes before it returns, and the
    gather moves raw bytes (gloo has no 16-bit integer or bfloat16 type).
    ``all_gather`` and ``reduce_scatter_sum`` return a handle whose ``wait()``
    gives the result.
    """

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.host_staged = dist.get_backend(group) == 'gloo'

    def _host(self, t):
        return t.cpu() if (self.host_staged and t.is_cuda) else t

    def all_reduce_sum_(self, t: torch.Tensor) -> torch.Tensor:
        h = self._host(t)
        dist.all_reduce(h, op=dist.ReduceOp.SUM, group=self.group)
        if h is not t:
            t.copy_(h)
        return t

    def all_gather(self, t: torch.Tensor):
        """[n, ...] on every rank -> handle of [world*n, ...], rank-major."""
        t = t.contiguous()
        out = torch.empty((self.world * t.shape[0], *t.shape[1:]), dtype=t.dtype, device=t.device)
        if not self.host_staged:
            return _InFlight(out, dist.all_gather_into_tensor(out, t, group=self.group, async_op=True))
        src, dst = self._host(t), (out.cpu() if out.is_cuda else out)
        if t.numel() > 0:
            dist.all_gather_into_tensor(dst.reshape(self.world, -1).view(torch.uint8),
                                        src.reshape(1, -1).view(torch.uint8), group=self.group)
        if dst is not out:
            out.copy_(dst)
        return _Ready(out)

    def reduce_scatter_sum(self, t: torch.Tensor):
        """[world*n, ...] on every rank -> handle of the sum over ranks of rows [rank*n, (rank+1)*n)."""
        if t.shape[0] % self.world:
            raise ValueError('reduce-scatter rows must divide evenly over the ranks')
        t = t.contiguous()
        out = torch.empty((t.shape[0] // self.world, *t.shape[1:]), dtype=t.dtype, device=t.device)
        if not self.host_staged:
            return _InFlight(out, dist.reduce_scatter_tensor(out, t, op=dist.ReduceOp.SUM, group=self.group,
                                                             async_op=True))
        src, dst = self._host(t), (out.cpu() if out.is_cuda else out)
        dist.reduce_scatter_tensor(dst, src, op=dist.ReduceOp.SUM, group=self.group)
        if dst is not out:
            out.copy_(dst)
        return _Ready(out)


class BankShardedMemory:
    """Runs ``layer.forward`` with the bank table partitioned over the ranks of ``group``.

    ``layer`` is a ``BankedDeltaMemory`` with identical parameters on every rank
    (e.g. the same seed).  ``forward(hidden)`` takes this rank's batch rows and
    returns this rank's output rows.
    """

    def __init__(self, layer, group=None, *, ownership: str = 'balanced', row_chunks: int = 1,
                 comm: ShardComm | None = None):
        if ownership not in ops.OWNERSHIP_MODES:
            raise ValueError(f'ownership must be one of {sorted(ops.OWNERSHIP_MODES)}')
        if row_chunks <= 0:
            raise ValueError('row_chunks must be positive')
        self.layer = layer
        self.comm = comm or ShardComm(group)
        self.ownership = ownership
        self.row_chunks = row_chunks
        self.rank, self.world = self.comm.rank, self.comm.world
        if layer.bank_count % self.world:
            raise NotImplementedError(f'{layer.bank_count} banks do not divide over {self.world} ranks')
        if ownership == 'balanced' and (layer.bank_count > ops.MAX_BALANCED_BANKS
                                        or self.world > ops.MAX_BALANCED_WORLD):
            warnings.warn(f'the balanced bank partition supports at most {ops.MAX_BALANCED_BANKS} banks and '
                          f'{ops.MAX_BALANCED_WORLD} ranks; {layer.bank_count} banks over {self.world} ranks use '
                          'contiguous ranges', stacklevel=2)
            self.ownership = 'contiguous'
        self.local_banks = layer.bank_count // self.world
        self.last_partition = None  # (owner, slot, members, counts) of the latest call
        self._chunk_streams = None
        # Optional list; when set (device tensors, one row chunk), forward appends
        # (phase name, CUDA event) pairs recorded on the current stream at each phase end.
        self.phase_events = None

    # ------------------------------------------------------------ the exchange
    @torch.no_grad()
    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        lay = self.layer
        comm = self.comm
        lb, time, _ = hidden.shape
        self._mark('start', hidden)
        controls, routes, gate = self.local_stage(hidden)
        ww, wi, rw, ri = routes
        self._mark('local', hidden)
        counts = self.histogram(wi, ri)
        comm.all_reduce_sum_(counts)
        owner, slot, members = self.owners(counts)
        self.last_partition = (owner, slot, members, counts)
        self._mark('partition', hidden)
        chunks = self.chunks(lb)
        # every gather is queued now, chunk by chunk; NCCL runs them in order while the streams compute
        gathers = []
        for r0, r1 in chunks:
            t0, t1 = r0 * time, r1 * time
            gathers.append(([comm.all_gather(r[r0:r1]) for r in routes],
                            [comm.all_gather(c[t0:t1]) for c in controls]))
        streams = self._streams(hidden, len(chunks))
        main = torch.cuda.current_stream(hidden.device) if streams else None
        partial_h = []
        for ci, ((r0, r1), (route_h, control_h)) in enumerate(zip(chunks, gathers)):
            if streams:
                streams[ci].wait_stream(main)
                ctx = torch.cuda.stream(streams[ci])
            else:
                ctx = _NoStream()
            with ctx:
                all_routes = [h.wait() for h in route_h]
                all_controls = [h.wait() for h in control_h]
                self._mark('gather', hidden)
                meta = self.dispatch_stage(all_routes, owner, slot)
                self._mark('dispatch', hidden)
                partial = self.bank_stage(all_controls, all_routes, meta, owner, members,
                                          batch=(r1 - r0) * self.world, time=time)
                partial_h.append(comm.reduce_scatter_sum(partial))
        for st in streams:
            main.wait_stream(st)  # before any tensor used on a chunk stream is released
        if len(chunks) == 1:
            combined = partial_h[0].wait()
            self._mark('reduce_scatter', hidden)
        else:
            combined = torch.empty((lb * time, lay.value_width), dtype=torch.float32, device=hidden.device)
            for (r0, r1), h in zip(chunks, partial_h):
                combined[r0 * time:r1 * time] = h.wait()
        out = self.output_stage(hidden, combined, gate)
        self._mark('output', hidden)
        return out.reshape(lb, time, lay.hidden_size)

    def _mark(self, name, hidden):
        if self.phase_events is not None and hidden.is_cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.phase_events.append((name, ev))

    def phase_times(self):
        """Milliseconds of each recorded phase (after a synchronize), from ``phase_events``."""
        ev = self.phase_events or []
        return {name: ev[i - 1][1].elapsed_time(e) for i, (name, e) in enumerate(ev) if i > 0}

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.forward(hidden)

    def chunks(self, rows):
        """Local row ranges of the exchange's chunks (at most ``row_chunks``, near-equal)."""
        n = max(1, min(self.row_chunks, rows))
        bounds = [rows * i // n for i in range(n + 1)]
        return [(bounds[i], bounds[i + 1]) for i in range(n) if bounds[i + 1] > bounds[i]]

    def _streams(self, hidden, n):
        """One side stream per chunk (device tensors, more than one chunk), created once."""
        if not hidden.is_cuda or n == 1:
            return []
        cached = self._chunk_streams
        if cached is None or len(cached) < n or cached[0].device != hidden.device:
            self._chunk_streams = cached = [torch.cuda.Stream(device=hidden.device) for _ in range(n)]
        return cached[:n]

    # --------------------------------------------------------------- stages
    def local_stage(self, hidden):
        """Projection, controllers and routes of this rank's tokens."""
        self.layer._check_hidden(hidden)
        return self.layer._controls_and_routes(hidden)

    def histogram(self, write_idx, read_idx):
        return ops.bank_histogram(write_idx, read_idx, self.layer.bank_count)

    def owners(self, counts):
        mode = self.ownership
        return ops.bank_owners(counts if mode == 'balanced' else None, self.layer.bank_count, self.world, mode=mode,
                               device=counts.device)

    def dispatch_stage(self, routes, owner, slot):
        ww, wi, rw, ri = routes
        return ops.dispatch_owned(wi, ri, self.layer.bank_count, owner, slot, self.rank, self.local_banks)

    def bank_stage(self, controls, routes, meta, owner, members, *, batch, time):
        """Recurrence and partial combine of this rank's banks -> FP32 [batch*time, V]."""
        lay = self.layer
        ww, wi, rw, ri = routes
        interval = state_interval(lay.bank_size) if lay.config.training_state_dtype == 'bfloat16' else 0
        reads = ops.bank_scan(*controls, wi, ww, ri, rw, meta['order'], meta['cu_seqlens'], batch=batch, time=time,
                              bank_count=self.local_banks, heads=lay.num_heads, bank_size=lay.bank_size,
                              head_value_width=lay.head_value_width, routed_decay=lay.config.routed_decay,
                              scale=lay.bank_size ** -0.5, row_factor=lay.initial_row_factor,
                              col_factor=lay.initial_column_factor, state_interval=interval,
                              bank_ids=members[self.rank], total_banks=lay.bank_count)
        self._mark('recurrence', reads)
        ops.check_scan_status(reads.device)  # non-blocking: raises once an earlier timeout is seen
        part = ops.combine_partial(reads, ri.reshape(batch * time, -1), owner, self.rank)
        self._mark('partial_combine', part)
        return part

    def output_stage(self, hidden, combined, gate):
        lay = self.layer
        normed = ops.norm_gate_f32(combined, gate, lay.output_norm_weight, getattr(lay, 'output_norm_bias', None),
                                   eps=lay.norm_eps, layer_norm=lay.config.output_normalization == 'layer',
                                   dtype=hidden.dtype)
        return F.linear(normed, lay.o_proj.weight, lay.o_proj.bias)
