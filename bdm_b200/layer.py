"""Drop-in BDM layer whose bank path runs on hand-written sm_100a kernels.

``BankedDeltaMemory`` (alias ``BlockSparseDeltaMemory``) keeps the reference
module's constructor, parameter names, shapes and seeded initialisation
(implementation/bdm/model.py:15-78, _parameters.py:69-177, routing.py:12-68),
so ``state_dict``s move between the two unchanged, and its entry points:

* ``forward(hidden)``                      model.py:88-140   (prefill / training forward)
* ``prefill(hidden, state=None, *, state_dtype=None)``  inference.py:110-131
* ``step(hidden, state)``                  inference.py:161-194
* ``create_state(batch, dtype=...)``       inference.py:100-107

Per forward: ONE projection GEMM (all controllers, both routers and the output
gate, biases in its epilogue) and the small f_proj.1 GEMM, then the CUDA kernels
of ``ops`` -- controller epilogue, router, dispatch, bank recurrence, combine +
norm + gate -- and the o_proj GEMM.  There is no backend switch and no CPU path; CPU inputs raise.

Training: when autograd needs gradients, ``forward`` runs the same kernels inside
``_BankTraining`` (a torch.autograd.Function from the fused projection's output to
the o_proj input) whose backward runs the CUDA backward kernels of ``ops``
(role_bank_kernel.py:76-150, routed_update.py:31-49, role_bank_dispatch.py:76-132,
product_routed_update.py:51-76); the GEMMs around it (fused projection, f_proj.1,
o_proj) differentiate through cuBLAS via autograd.
"""
from __future__ import annotations

import hashlib
import math
import weakref

import torch
from torch import nn
from torch.nn import functional as F

from . import ops
from .config import BDMConfig, near_square_factors, state_interval


FUSED_F_MAX_TOKENS = 4096  # at most this many tokens: the controllers kernel computes f_proj.1 itself
_COPY_STREAMS: dict = {}  # per device: (upload, download, (extra compute streams)) of forward_host
HOST_COMPUTE_STREAMS = 2  # compute streams forward_host's row groups rotate over (current + extras)
_MAX_HOST_COMPUTE_STREAMS = 4
# per layer: {(rows, time): (parameter key, [captured forwards])} for forward_host's row groups
_HOST_GRAPHS: 'weakref.WeakKeyDictionary' = weakref.WeakKeyDictionary()


def _copy_streams(device):
    st = _COPY_STREAMS.get(device.index)
    if st is None:
        st = _COPY_STREAMS[device.index] = (torch.cuda.Stream(device), torch.cuda.Stream(device),
                                            tuple(torch.cuda.Stream(device)
                                                  for _ in range(_MAX_HOST_COMPUTE_STREAMS - 1)))
    return st


class SharedResidualRouter(nn.Module):
    """Routing base plus learned read / write residuals (routing.py:12-35).

    ``read``/``write`` are kept for API parity; the layer folds both into its
    fused projection instead of calling them.
    """

    def __init__(self, input_width: int, output_width: int) -> None:
        super().__init__()
        if input_width <= 0 or output_width <= 0:
            raise ValueError('router widths must be positive')
        self.base = nn.Linear(input_width, output_width)
        self.read_residual = nn.Linear(input_width, output_width)
        self.write_residual = nn.Linear(input_width, output_width)

    def read_params(self):
        return self.base.weight + self.read_residual.weight, self.base.bias + self.read_residual.bias

    def write_params(self):
        return self.base.weight + self.write_residual.weight, self.base.bias + self.write_residual.bias

    def read(self, hidden):
        return F.linear(hidden, *self.read_params())

    def write(self, hidden):
        return F.linear(hidden, *self.write_params())

    @torch.no_grad()
    def initialize_from_independent(self, *, std: float, read_generator=None, write_generator=None) -> None:
        """Base = mean of two matched truncated-normal draws; residuals and biases zero (routing.py:37-68)."""
        if std <= 0:
            raise ValueError('router initialization scale must be positive')
        draws = []
        for generator in (read_generator, write_generator):
            weight = torch.empty_like(self.base.weight)
            nn.init.trunc_normal_(weight, mean=0.0, std=std, a=-3.0 * std, b=3.0 * std, generator=generator)
            draws.append(weight)
        self.base.weight.copy_(0.5 * (draws[0] + draws[1]))
        for t in (self.base.bias, self.read_residual.weight, self.read_residual.bias, self.write_residual.weight,
                  self.write_residual.bias):
            t.zero_()


class BankedDeltaMemory(nn.Module):
    """Shared-residual product routing around GDN2 memory banks, on B200 kernels."""

    def __init__(self, config: BDMConfig, *, layer_id=0, seed=0, backend='role', compact_replay=None):
        super().__init__()
        if backend != 'role':
            raise ValueError("bdm_b200 runs only its CUDA path (backend='role'); there is no CPU or FLA backend")
        if seed < 0 or layer_id < 0:
            raise ValueError('seed and layer_id must be nonnegative')
        if compact_replay is not None and type(compact_replay) is not bool:
            raise ValueError('compact_replay must be None, True, or False')
        self.compact_replay = compact_replay
        self.config, self.backend = config, backend
        self.hidden_size, self.bank_count, self.bank_size = config.dim, config.bank_count, config.bank_size
        self.value_width, self.kernel_key_width = config.value_width, config.bank_size
        self.num_heads = config.num_heads
        self.head_value_width = config.head_value_width
        key_width = config.num_heads * config.bank_size
        self.num_reads = self.num_writes = config.selected_banks
        self.layer_id, self.initialization_seed = layer_id, seed * 100_000 + 6000 + layer_id
        self.norm_eps = config.norm_eps
        self.shared_residual_router = True
        self.initial_state_mode = 'product_key'
        self.routing_mode = 'product_topk'
        self.factors = near_square_factors(config.bank_count)
        route_width = sum(self.factors)
        self.factor_route_width = self.route_projection_width = route_width
        # Module creation order matches the reference, so the global RNG
        # draws of nn.Linear's default init (overwritten below) line up too.
        self.q_proj = nn.Linear(config.dim, key_width, bias=False)
        self.k_proj = nn.Linear(config.dim, key_width, bias=False)
        self.v_proj = nn.Linear(config.dim, config.value_width, bias=False)
        self.shared_router = SharedResidualRouter(config.dim, route_width)
        self.read_route_proj = self.write_route_proj = None
        self.f_proj = nn.Sequential(nn.Linear(config.dim, config.head_value_width, bias=False),
                                    nn.Linear(config.head_value_width, key_width, bias=False))
        self.b_proj = nn.Linear(config.dim, key_width, bias=False)
        self.w_proj = nn.Linear(config.dim, config.value_width, bias=False)
        self.A_log = nn.Parameter(torch.empty(config.num_heads, dtype=torch.float32))
        self.dt_bias = nn.Parameter(torch.empty(key_width, dtype=torch.float32))
        self.A_log._no_weight_decay = self.dt_bias._no_weight_decay = True
        rows, columns = near_square_factors(config.logical_rows)
        self.register_parameter('initial_state', None)
        self.initial_row_factor = nn.Parameter(torch.zeros(rows, config.head_value_width))
        self.initial_column_factor = nn.Parameter(torch.zeros(columns, config.head_value_width))
        self.initial_row_factor._sdm_memory_bank = self.initial_column_factor._sdm_memory_bank = True
        self.output_gate = nn.Linear(config.dim, config.value_width, bias=True)
        self.output_norm_weight = nn.Parameter(torch.ones(config.value_width))
        if config.output_normalization == 'layer':
            self.output_norm_bias = nn.Parameter(torch.zeros(config.value_width))
        self.o_proj = nn.Linear(config.value_width, config.dim, bias=config.output_bias)
        self._fused_cache = None
        # Optional lists; when set, (start, end) CUDA events bracket every bank-recurrence launch
        # (forward) and every recurrence-backward launch.
        self.scan_events = None
        self.backward_events = None
        # True: inference forwards / prefills of BF16 layers whose shapes fit run the read combine,
        # norm, gate and o_proj as one tensor-core kernel (ops.combine_project); False (default):
        # the combine_norm_gate kernel followed by a cuBLAS o_proj.
        self.fused_output = False
        self.init_weights(initialization_seed=self.initialization_seed)

    # ---------------------------------------------------------- initialisation
    def _role_generator(self, role, parameter, initialization_seed):
        """Per-role generator seeded by blake2b of the role name (_parameters.py:69-84)."""
        if initialization_seed is None:
            return None
        digest = hashlib.blake2b(f'bank_sparse_gdn2.{self.layer_id}.{role}'.encode(), digest_size=8).digest()
        generator = torch.Generator(device=parameter.device)
        generator.manual_seed((initialization_seed ^ int.from_bytes(digest, byteorder='little')) % (1 << 63))
        return generator

    def init_weights(self, init_std=None, factor=1.0, width_scaling=None, *, initialization_seed=None):
        """Seeded initialisation identical to the reference (_parameters.py:86-177)."""
        del width_scaling
        if initialization_seed is None:
            initialization_seed = self.initialization_seed
        if initialization_seed is not None and initialization_seed < 0:
            raise ValueError('initialization_seed must be non-negative')
        for name, module in self.named_modules():
            if isinstance(module, nn.Linear) and not name.startswith('shared_router.'):
                nn.init.xavier_uniform_(module.weight, gain=2 ** -2.5,
                                        generator=self._role_generator(f'{name}.weight', module.weight,
                                                                       initialization_seed))
                if module.bias is not None:
                    nn.init.zeros_(module.bias)
        base_std = (init_std or self.hidden_size ** -0.5) / factor
        self.shared_router.initialize_from_independent(
            std=base_std,
            read_generator=self._role_generator('read_router.weight', self.shared_router.base.weight,
                                                initialization_seed),
            write_generator=self._role_generator('write_router.weight', self.shared_router.base.weight,
                                                 initialization_seed))
        with torch.no_grad():
            self.A_log.uniform_(1.0, 16.0, generator=self._role_generator('decay_rate', self.A_log,
                                                                          initialization_seed)).log_()
            log_dt = torch.empty_like(self.dt_bias).uniform_(
                math.log(0.001), math.log(0.1),
                generator=self._role_generator('time_step', self.dt_bias, initialization_seed))
            dt = log_dt.exp().clamp_min(1e-4)
            self.dt_bias.copy_(dt + torch.log(-torch.expm1(-dt)))  # inverse softplus
            for role, parameter in (('initial_state.row', self.initial_row_factor),
                                    ('initial_state.column', self.initial_column_factor)):
                nn.init.trunc_normal_(parameter, mean=0.0, std=base_std, a=-3 * base_std, b=3 * base_std,
                                      generator=self._role_generator(role, parameter, initialization_seed))
                # two additive factors share one row's variance budget
                parameter.mul_(1 / math.sqrt(2))
            self.output_norm_weight.fill_(1.0)
            if hasattr(self, 'output_norm_bias'):
                self.output_norm_bias.zero_()
        self._fused_cache = None

    def reset_parameters(self) -> None:
        self.init_weights(initialization_seed=self.initialization_seed)

    # ------------------------------------------------------------- properties
    @property
    def total_rows(self) -> int:
        return self.bank_count * self.num_heads * self.bank_size

    @property
    def touched_rows(self) -> int:
        return self.num_writes * self.num_heads * self.bank_size

    @property
    def logical_reads(self) -> int:
        return self.num_reads * self.num_heads * self.bank_size

    @property
    def logical_writes(self) -> int:
        return self.num_writes * self.num_heads * self.bank_size

    @property
    def initial_state_parameter_count(self) -> int:
        return self.initial_row_factor.numel() + self.initial_column_factor.numel()

    # ------------------------------------------------------- fused projection
    def _fused_projection(self):
        """Concatenated [W; bias] of every projection that reads ``hidden``.

        Column blocks: q | k | v | f1 | b | w | read router | write router | gate.
        Router weights are base + residual in the parameter dtype, as
        SharedResidualRouter.read/write form them.  Rebuilt when a parameter changes.
        """
        params = [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.f_proj[0].weight,
                  self.b_proj.weight, self.w_proj.weight, *self.shared_router.parameters(), self.output_gate.weight,
                  self.output_gate.bias]
        key = tuple((p.data_ptr(), p._version, p.dtype, p.device) for p in params)
        if self._fused_cache is not None and self._fused_cache[0] == key:
            return self._fused_cache[1]
        with torch.no_grad():
            rw, rb = self.shared_router.read_params()
            ww, wb = self.shared_router.write_params()
            blocks = [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.f_proj[0].weight,
                      self.b_proj.weight, self.w_proj.weight, rw, ww, self.output_gate.weight]
            weight = torch.cat([b.detach() for b in blocks], 0).contiguous()
            widths = [b.shape[0] for b in blocks]
            offsets = [0]
            for wdt in widths:
                offsets.append(offsets[-1] + wdt)
            bias = torch.zeros(weight.shape[0], dtype=weight.dtype, device=weight.device)
            bias[offsets[6]:offsets[7]] = rb.detach()
            bias[offsets[7]:offsets[8]] = wb.detach()
            bias[offsets[8]:offsets[9]] = self.output_gate.bias.detach()
            names = ['q', 'k', 'v', 'f', 'b', 'w', 'read', 'write', 'gate']
            cols = dict(zip(names, offsets[:-1]))
        fused = (weight, bias, cols)
        self._fused_cache = (key, fused)
        return fused

    def _project(self, hidden2d):
        weight, bias, cols = self._fused_projection()
        return torch.addmm(bias, hidden2d, weight.t()), cols

    def _fused_projection_autograd(self):
        """``_fused_projection`` built from the live parameters (autograd records the concatenation)."""
        _, _, cols = self._fused_projection()
        router = self.shared_router
        rw = router.base.weight + router.read_residual.weight
        rb = router.base.bias + router.read_residual.bias
        ww = router.base.weight + router.write_residual.weight
        wb = router.base.bias + router.write_residual.bias
        weight = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.f_proj[0].weight,
                            self.b_proj.weight, self.w_proj.weight, rw, ww, self.output_gate.weight], 0)
        zeros = torch.zeros(cols['read'], dtype=weight.dtype, device=weight.device)
        bias = torch.cat([zeros, rb, wb, self.output_gate.bias], 0)
        return weight, bias, cols

    # ------------------------------------------------------------------ steps
    def _check_hidden(self, hidden):
        if hidden.ndim != 3 or hidden.shape[-1] != self.hidden_size or hidden.shape[1] == 0:
            raise ValueError('hidden must be [batch, positive time, dim]')
        if not hidden.is_cuda:
            raise ValueError('bdm_b200 requires CUDA tensors; there is no CPU path')
        if hidden.dtype != self.q_proj.weight.dtype:
            raise ValueError(f'hidden dtype {hidden.dtype} does not match the parameters ({self.q_proj.weight.dtype})')
        ops.dtype_code(hidden.dtype)

    def _controls_and_routes(self, hidden):
        batch, time, _ = hidden.shape
        proj, cols = self._project(hidden.reshape(batch * time, self.hidden_size))
        f = None
        if batch * time > FUSED_F_MAX_TOKENS:  # many tokens: f_proj.1 as a GEMM; few (decode): in the kernel
            f1 = proj[:, cols['f']:cols['f'] + self.head_value_width]
            f = torch.mm(f1, self.f_proj[1].weight.t())  # f_proj.1, rounded to the activation dtype
        q, k, v, g, b, w = ops.controllers(proj, cols, f, self.A_log, self.dt_bias,
                                           heads=self.num_heads, bank_size=self.bank_size,
                                           head_value_width=self.head_value_width,
                                           qk_norm=self.config.qk_normalization,
                                           f_weight=self.f_proj[1].weight, f1_width=self.head_value_width)
        # both routers (read block, then write block of the fused projection) in one launch
        (rw, ri), (ww, wi) = ops.route_pair(proj, cols['read'], cols['write'], bank_count=self.bank_count,
                                            selected_banks=self.num_reads, factors=self.factors)
        shape = (batch, time, -1)
        routes = (ww.reshape(shape), wi.reshape(shape), rw.reshape(shape), ri.reshape(shape))
        gate = proj[:, cols['gate']:cols['gate'] + self.value_width]
        return (q, k, v, g, b, w), routes, gate

    def _output(self, hidden, reads, read_idx, gate, *, round_each):
        batch, time, _ = hidden.shape
        if self.fused_output and ops.combine_project_supported(self.value_width, self.hidden_size,
                                                              read_idx.shape[-1], reads.dtype):
            # combine, norm, gate and o_proj in one tensor-core kernel; the o_proj input stays on chip
            out = ops.combine_project(reads, read_idx, gate, self.output_norm_weight,
                                      getattr(self, 'output_norm_bias', None), self.o_proj.weight, self.o_proj.bias,
                                      eps=self.norm_eps, layer_norm=self.config.output_normalization == 'layer',
                                      round_each=round_each)
            return out.reshape(batch, time, self.hidden_size)
        normed = ops.combine_norm_gate(reads, read_idx, gate, self.output_norm_weight,
                                       getattr(self, 'output_norm_bias', None), eps=self.norm_eps,
                                       layer_norm=self.config.output_normalization == 'layer', round_each=round_each)
        return F.linear(normed, self.o_proj.weight, self.o_proj.bias).reshape(batch, time, self.hidden_size)

    def _bank_pass(self, controls, routes, batch, time, **state_args):
        ww, wi, rw, ri = routes
        meta = ops.dispatch(wi, ri, self.bank_count)
        timing = self.scan_events is not None
        if timing:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
        reads = ops.bank_scan(*controls, wi, ww, ri, rw, meta['order'], meta['cu_seqlens'], batch=batch, time=time,
                              bank_count=self.bank_count, heads=self.num_heads, bank_size=self.bank_size,
                              head_value_width=self.head_value_width, routed_decay=self.config.routed_decay,
                              scale=self.bank_size ** -0.5, **state_args)
        if timing:
            end.record()
            self.scan_events.append((start, end))
        return reads

    def forward(self, hidden):
        """Full-sequence forward (model.py:88-140): training-state BF16 storage policy, FP32 combine.

        Differentiable when autograd is on and the input or a parameter requires a gradient.
        """
        self._check_hidden(hidden)
        if torch.is_grad_enabled() and (hidden.requires_grad or any(p.requires_grad for p in self.parameters())):
            return self._forward_train(hidden)
        batch, time, _ = hidden.shape
        controls, routes, gate = self._controls_and_routes(hidden)
        interval = state_interval(self.bank_size) if self.config.training_state_dtype == 'bfloat16' else 0
        reads = self._bank_pass(controls, routes, batch, time, row_factor=self.initial_row_factor,
                                col_factor=self.initial_column_factor, state_interval=interval)
        ri = routes[3].reshape(batch * time, -1)
        out = self._output(hidden, reads, ri, gate, round_each=False)
        ops.check_scan_status(hidden.device)  # non-blocking: raises once an earlier timeout is seen
        return out

    def capture_forward(self, batch: int, time: int, *, warmup: int = 2):
        """CUDA-graph ``forward`` for inputs [batch, time, dim].

        Returns ``run(hidden=None) -> out``: copies ``hidden`` (if given) into the graph's input
        buffer ``run.input``, replays the forward and returns its output buffer ``run.output``,
        which the next replay overwrites.  Parameters must not change afterwards (the graph holds
        their fused copy); ``forward_host`` recaptures when they do.
        """
        if torch.is_grad_enabled():
            raise RuntimeError('capture_forward requires no_grad or inference_mode')
        dev, dt = self.q_proj.weight.device, self.q_proj.weight.dtype
        x = torch.zeros(batch, time, self.hidden_size, dtype=dt, device=dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.forward(x)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y = self.forward(x)

        def run(hidden=None):
            if hidden is not None:
                x.copy_(hidden)
            graph.replay()
            return y

        run.graph, run.input, run.output = graph, x, y  # keep the graph and its buffers alive
        return run

    def _host_graphs(self, rows: int, time: int, slots: int):
        """(captured forwards, their download events, fresh): up to ``slots`` captured forwards of
        [rows, time] inputs, recaptured when a parameter changes; ``freed[i]`` is the event after
        slot i's last output download (None before its first use), kept across calls."""
        key = tuple((p.data_ptr(), p._version) for p in self.parameters())
        per_layer = _HOST_GRAPHS.setdefault(self, {})
        entry = per_layer.get((rows, time))
        fresh = entry is None or entry[0] != key or len(entry[1]) < slots
        if fresh:
            per_layer.pop((rows, time), None)  # free stale graphs before capturing new ones
            entry = (key, [self.capture_forward(rows, time) for _ in range(slots)], [None] * slots)
            per_layer[(rows, time)] = entry
        return entry[1][:slots], entry[2], fresh

    @torch.no_grad()
    def forward_host(self, hidden, out=None, *, chunks: int = 4, graphs: bool = True):
        """``forward`` of a batch held in host memory, returned in host memory.

        The batch streams through the GPU in ``chunks`` groups of rows: each group is uploaded on
        one copy stream, its forward runs on the current stream once its rows have landed, and
        its output goes back on a second copy stream, so the uploads, the downloads (the two
        directions of the host link) and the compute of different groups overlap.  With
        ``graphs`` and equal groups, each group's forward is a replay of one of up to four
        captured forwards (``capture_forward``, cached per layer and group shape, recaptured when
        a parameter changes) used in rotation, which removes the per-group host launch cost; a
        slot is refilled only once its previous output has been downloaded (tracked across calls,
        so back-to-back calls overlap too), and consecutive groups replay on two compute streams
        so that their kernels overlap.  Batch rows are
        independent (each bank sequence belongs to one row), so the result is ``forward``'s up to
        the GEMMs' accumulation order at the smaller row count.  ``hidden`` should be pinned
        (pageable memory makes the copies synchronous); ``out`` (pinned, [B, T, D]) receives the
        result and is returned, else a new pinned tensor is.  The current stream waits for the
        downloads before this returns; the host must synchronise before reading ``out``.
        """
        if hidden.is_cuda or hidden.ndim != 3 or hidden.shape[-1] != self.hidden_size or hidden.shape[1] == 0:
            raise ValueError('forward_host takes a host tensor [batch, positive time, dim]')
        dev = self.q_proj.weight.device
        if dev.type != 'cuda':
            raise ValueError('bdm_b200 requires the layer on a CUDA device; there is no CPU path')
        if hidden.dtype != self.q_proj.weight.dtype:
            raise ValueError(f'hidden dtype {hidden.dtype} does not match the parameters ({self.q_proj.weight.dtype})')
        batch, time = hidden.shape[0], hidden.shape[1]
        if out is None:
            out = torch.empty(hidden.shape[:2] + (self.hidden_size,), dtype=hidden.dtype, pin_memory=True)
        elif out.shape != hidden.shape[:2] + (self.hidden_size,) or out.is_cuda:
            raise ValueError('out must be a host tensor [batch, time, dim]')
        groups = max(1, min(int(chunks), batch))
        bounds = [(batch * i // groups, batch * (i + 1) // groups) for i in range(groups)]
        cur = torch.cuda.current_stream(dev)
        up, down, extra = _copy_streams(dev)
        down.wait_stream(cur)
        if graphs and batch % groups == 0:
            runs, freed, fresh = self._host_graphs(batch // groups, time, min(groups, 4))
            # A slot's input is rewritten only after its previous output went down (``freed``, kept
            # across calls), so this call's first uploads may overlap the previous call's last
            # groups; right after a capture the uploads wait for everything before.
            if fresh:
                up.wait_stream(cur)
            # groups rotate over the compute streams, so the recurrences of neighbouring groups
            # (each latency-bound on its own: a group keeps the full sequence length) overlap
            n_comp = max(1, min(HOST_COMPUTE_STREAMS, _MAX_HOST_COMPUTE_STREAMS))
            computes = (cur,) + extra[:n_comp - 1]
            for cs in computes[1:]:
                cs.wait_stream(cur)
            for i, (a, b) in enumerate(bounds):
                slot = i % len(runs)
                run = runs[slot]
                cs = computes[i % len(computes)]
                with torch.cuda.stream(up):
                    if freed[slot] is not None:
                        up.wait_event(freed[slot])
                    run.input.copy_(hidden[a:b], non_blocking=True)
                    landed = torch.cuda.Event()
                    landed.record(up)
                cs.wait_event(landed)
                with torch.cuda.stream(cs):
                    run.graph.replay()
                    done = torch.cuda.Event()
                    done.record(cs)
                with torch.cuda.stream(down):
                    down.wait_event(done)
                    out[a:b].copy_(run.output, non_blocking=True)
                    freed[slot] = torch.cuda.Event()
                    freed[slot].record(down)
            for cs in computes[1:]:
                cur.wait_stream(cs)
            cur.wait_stream(down)
            ops.check_scan_status(dev)  # non-blocking: the replays skip the forward's own poll
            return out
        up.wait_stream(cur)
        inputs, landed = [], []
        for a, b in bounds:
            with torch.cuda.stream(up):
                x = hidden[a:b].to(dev, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(up)
            x.record_stream(cur)
            inputs.append(x)
            landed.append(ev)
        for (a, b), x, ev in zip(bounds, inputs, landed):
            cur.wait_event(ev)
            y = self.forward(x)
            done = torch.cuda.Event()
            done.record(cur)
            down.wait_event(done)
            with torch.cuda.stream(down):
                out[a:b].copy_(y, non_blocking=True)
            y.record_stream(down)
        cur.wait_stream(down)
        return out

    def _forward_train(self, hidden):
        batch, time, _ = hidden.shape
        if self.bank_size not in (4, 8, 16):
            raise NotImplementedError('the training backward supports bank_size 4, 8 or 16')
        if self.head_value_width > 256:  # the event VJP keeps a head's value row in one warp
            raise NotImplementedError('the training backward supports head_value_width <= 256')
        weight, bias, cols = self._fused_projection_autograd()
        proj = torch.addmm(bias, hidden.reshape(batch * time, self.hidden_size), weight.t())
        normed = _BankTraining.apply(proj, self.f_proj[1].weight, self.A_log, self.dt_bias, self.initial_row_factor,
                                     self.initial_column_factor, self.output_norm_weight,
                                     getattr(self, 'output_norm_bias', None), self, cols, batch, time)
        ops.check_scan_status(hidden.device)
        return F.linear(normed, self.o_proj.weight, self.o_proj.bias).reshape(batch, time, self.hidden_size)

    # ---------------------------------------------------- stateful inference
    def _state_shape(self, batch):
        if self.num_heads == 1:
            return (batch, self.bank_count, self.bank_size, self.value_width)
        return (batch, self.bank_count, self.num_heads, self.bank_size, self.head_value_width)

    def create_state(self, batch, *, dtype=torch.bfloat16):
        """Product-key initial cache [batch, J, S, V] (H = 1) or [batch, J, H, S, dv] (inference.py:100-107)."""
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError('cache dtype must be FP32 or BF16')
        state = ops.product_state(self.initial_row_factor, self.initial_column_factor, batch=batch,
                                  bank_count=self.bank_count, heads=self.num_heads, bank_size=self.bank_size,
                                  dtype=dtype)
        return state.reshape(self._state_shape(batch))

    def _validate_state(self, hidden, state):
        if state is not None and (tuple(state.shape) != self._state_shape(hidden.shape[0])
                                  or state.dtype not in (torch.float32, torch.bfloat16)
                                  or state.device != hidden.device or not state.is_contiguous()):
            raise ValueError(f'state must be contiguous FP32 or BF16 {self._state_shape(hidden.shape[0])} '
                             'on the input device')

    @torch.no_grad()
    def _prefill(self, hidden, state, state_dtype):
        batch, time, _ = hidden.shape
        cache_dtype = state_dtype or (state.dtype if state is not None else torch.bfloat16)
        if cache_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError('cache dtype must be FP32 or BF16')
        if state is None:
            # Wider factors are not rounded early to a narrower cache (inference.py:117-121).
            work = torch.float32 if self.initial_row_factor.dtype != cache_dtype else cache_dtype
            state = self.create_state(batch, dtype=work)
        elif state_dtype is not None and state_dtype != state.dtype:
            raise ValueError('state_dtype must match the supplied cache')
        controls, routes, gate = self._controls_and_routes(hidden)
        reads = self._bank_pass(controls, routes, batch, time, cache=state, store_final=True, state_interval=0)
        if state.dtype != cache_dtype:
            state = state.to(cache_dtype)
        ri = routes[3].reshape(batch * time, -1)
        out = self._output(hidden, reads, ri, gate, round_each=True)
        ops.check_scan_status(hidden.device)
        return out, state

    def prefill(self, hidden, state=None, *, state_dtype=None):
        """Process a prefix (inference.py:110-131); BF16 cache storage rounds once, at handoff."""
        self._check_hidden(hidden)
        self._validate_state(hidden, state)
        if torch.is_grad_enabled():
            raise RuntimeError('Stateful inference requires no_grad or inference_mode')
        return self._prefill(hidden, state, state_dtype)

    def step(self, hidden, state):
        """Advance the cache by one token per row (inference.py:161-194); mutates and returns ``state``."""
        self._check_hidden(hidden)
        self._validate_state(hidden, state)
        if torch.is_grad_enabled() or hidden.shape[1] != 1:
            raise ValueError('step requires one token under no_grad/inference_mode')
        batch = hidden.shape[0]
        if self.num_reads == self.num_writes:
            # controllers, both routers and the bank step in one kernel after the projection GEMM
            proj, cols = self._project(hidden.reshape(batch, self.hidden_size))
            normed = ops.decode_token_step(
                proj, cols, self.f_proj[1].weight, self.A_log, self.dt_bias, state, bank_count=self.bank_count,
                selected_banks=self.num_reads, factors=self.factors, heads=self.num_heads, bank_size=self.bank_size,
                head_value_width=self.head_value_width, qk_norm=self.config.qk_normalization,
                routed_decay=self.config.routed_decay, scale=self.bank_size ** -0.5,
                norm_weight=self.output_norm_weight, norm_bias=getattr(self, 'output_norm_bias', None),
                eps=self.norm_eps, layer_norm=self.config.output_normalization == 'layer')
            out = F.linear(normed, self.o_proj.weight, self.o_proj.bias)
            return out.reshape(batch, 1, self.hidden_size), state
        controls, routes, gate = self._controls_and_routes(hidden)
        ww, wi, rw, ri = (r.reshape(batch, -1) for r in routes)
        # the step kernel also applies the output norm and gate (one launch instead of two)
        normed = ops.decode_step(*controls, wi, ww, ri, rw, state, bank_count=self.bank_count, heads=self.num_heads,
                                 bank_size=self.bank_size, head_value_width=self.head_value_width,
                                 routed_decay=self.config.routed_decay, scale=self.bank_size ** -0.5, gate=gate,
                                 norm_weight=self.output_norm_weight,
                                 norm_bias=getattr(self, 'output_norm_bias', None), eps=self.norm_eps,
                                 layer_norm=self.config.output_normalization == 'layer')
        out = F.linear(normed, self.o_proj.weight, self.o_proj.bias)
        return out.reshape(batch, 1, self.hidden_size), state

    def capture_step(self, state, *, warmup=2):
        """CUDA-graph one decode step bound to ``state`` (a cache from ``prefill``/``create_state``).

        Returns ``run(hidden[B,1,D]) -> out[B,1,D]``; each call copies ``hidden`` into the graph's
        input buffer, replays the step (``state`` is advanced in place exactly as ``step`` does)
        and returns the graph's output buffer, which the next call overwrites.  Warm-up runs on a
        clone of ``state``, so capturing does not advance the cache.  Parameters must not change
        afterwards (the graph holds their fused copy).
        """
        if torch.is_grad_enabled():
            raise RuntimeError('capture_step requires no_grad or inference_mode')
        batch = state.shape[0]
        dev, dt = state.device, self.q_proj.weight.dtype
        hidden_in = torch.zeros(batch, 1, self.hidden_size, dtype=dt, device=dev)
        self._validate_state(hidden_in, state)
        scratch = state.clone()
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(hidden_in, scratch)
        torch.cuda.current_stream(dev).wait_stream(side)
        del scratch
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out, _ = self.step(hidden_in, state)

        def run(hidden):
            hidden_in.copy_(hidden)
            graph.replay()
            return out

        run.graph = graph  # keep the graph (and its memory pool) alive with the callable
        return run


class _BankTraining(torch.autograd.Function):
    """Differentiable bank path: fused projection output ``proj`` [NT, ld] -> o_proj input [NT, V].

    Forward: f_proj.1 (cuBLAS), controller epilogue, both routers, dispatch, the
    factor-initialised recurrence under the training storage policy, and the combine
    with norm and gate (which also keeps the combined read sum for the backward).
    Backward (the reference's RoutedUpdate / ProductRoutedUpdate backward plus the
    autograd of the ops around it): norm and gate, recurrence, event VJP, router,
    controllers, f_proj.1 and the product-key factors; every column block of
    d proj is written by exactly one of them.
    """

    @staticmethod
    def forward(ctx, proj, wf2, a_log, dt_bias, row_factor, col_factor, norm_w, norm_b, layer, cols, batch, time):
        m = layer
        H, S, dv, V, J = m.num_heads, m.bank_size, m.head_value_width, m.value_width, m.bank_count
        f1 = proj[:, cols['f']:cols['f'] + dv]
        f = torch.mm(f1, wf2.t())
        q, k, v, g, b, w = ops.controllers(proj, cols, f, a_log, dt_bias, heads=H, bank_size=S, head_value_width=dv,
                                           qk_norm=m.config.qk_normalization)
        (rw, ri), (ww, wi) = ops.route_pair(proj, cols['read'], cols['write'], bank_count=J,
                                            selected_banks=m.num_reads, factors=m.factors)
        shape = (batch, time, -1)
        meta = ops.dispatch(wi.reshape(shape), ri.reshape(shape), J)
        interval = state_interval(S) if m.config.training_state_dtype == 'bfloat16' else 0
        # the recurrence also writes the backward's state checkpoints (no replay sweep in the backward)
        ckpt, block = ops.checkpoint_buffer(batch=batch, time=time, kw=wi.shape[-1], kr=ri.shape[-1], bank_count=J,
                                            heads=H, bank_size=S, head_value_width=dv, device=proj.device)
        reads = ops.bank_scan(q, k, v, g, b, w, wi.reshape(shape), ww.reshape(shape), ri.reshape(shape),
                              rw.reshape(shape), meta['order'], meta['cu_seqlens'], batch=batch, time=time,
                              bank_count=J, heads=H, bank_size=S, head_value_width=dv,
                              routed_decay=m.config.routed_decay, scale=S ** -0.5, row_factor=row_factor,
                              col_factor=col_factor, state_interval=interval, checkpoints=ckpt,
                              checkpoint_block=block)
        gate = proj[:, cols['gate']:cols['gate'] + V]
        layer_norm = m.config.output_normalization == 'layer'
        normed, raw = ops.combine_norm_gate(reads, ri, gate, norm_w, norm_b if layer_norm else None, eps=m.norm_eps,
                                            layer_norm=layer_norm, round_each=False, save_raw=True)
        del reads
        ctx.save_for_backward(proj, f, wf2, a_log, dt_bias, row_factor, col_factor, norm_w, norm_b, q, k, v, g, b, w,
                              ww, wi, rw, ri, meta['order'], meta['cu_seqlens'], raw, ckpt)
        ctx.layer, ctx.cols, ctx.batch, ctx.time, ctx.interval = m, cols, batch, time, interval
        return normed

    @staticmethod
    def backward(ctx, d_normed):
        (proj, f, wf2, a_log, dt_bias, row_factor, col_factor, norm_w, norm_b, q, k, v, g, b, w, ww, wi, rw, ri,
         order, cu, raw, ckpt) = ctx.saved_tensors
        m, cols, batch, time = ctx.layer, ctx.cols, ctx.batch, ctx.time
        ops.check_scan_status(proj.device)  # the forward's reads and checkpoints feed everything below
        H, S, dv, V, J = m.num_heads, m.bank_size, m.head_value_width, m.value_width, m.bank_count
        layer_norm = m.config.output_normalization == 'layer'
        d_proj = torch.empty_like(proj)
        d_raw, d_nw, d_nb = ops.norm_gate_backward(d_normed, raw, proj[:, cols['gate']:cols['gate'] + V], norm_w,
                                                   norm_b if layer_norm else None, eps=m.norm_eps,
                                                   layer_norm=layer_norm,
                                                   d_gate=d_proj[:, cols['gate']:cols['gate'] + V])
        kw, kr = ww.shape[-1], rw.shape[-1]
        timing = m.backward_events is not None
        if timing:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
        evg, du, dinit = ops.scan_backward(q, k, v, g, b, w, ww, rw, order, cu, d_raw, batch=batch, time=time,
                                           bank_count=J, heads=H, bank_size=S, head_value_width=dv, kw=kw, kr=kr,
                                           routed_decay=m.config.routed_decay, scale=S ** -0.5,
                                           row_factor=row_factor, col_factor=col_factor,
                                           state_interval=ctx.interval, checkpoints=ckpt)
        if timing:
            end.record()
            m.backward_events.append((start, end))
        dq, dk, dvv, dg, db, dw, dww, drw = ops.event_vjp(q, k, v, g, b, w, ww, rw, evg, du, heads=H, bank_size=S,
                                                          head_value_width=dv, routed_decay=m.config.routed_decay,
                                                          scale=S ** -0.5)
        del evg, du
        ops.route_backward(proj, cols['read'], cols['write'], ri, drw, wi, dww, d_proj, bank_count=J,
                           factors=m.factors)
        df, d_a, d_dt = ops.controllers_backward(proj, cols, f, a_log, dt_bias, g, b, w, dq, dk, dvv, dg, db, dw,
                                                 d_proj, heads=H, bank_size=S, head_value_width=dv,
                                                 qk_norm=m.config.qk_normalization)
        f1 = proj[:, cols['f']:cols['f'] + dv]
        d_proj[:, cols['f']:cols['f'] + dv] = torch.mm(df, wf2)
        d_wf2 = torch.mm(df.t(), f1)
        d_u, d_z = ops.product_state_backward(dinit, batch=batch, rows_p=row_factor.shape[0],
                                              cols_q=col_factor.shape[0], factor_dtype=row_factor.dtype)
        d_nb_out = d_nb.to(norm_b.dtype) if (norm_b is not None and d_nb is not None) else (
            torch.zeros_like(norm_b) if norm_b is not None else None)
        return (d_proj, d_wf2, d_a.to(a_log.dtype), d_dt.to(dt_bias.dtype), d_u.to(row_factor.dtype),
                d_z.to(col_factor.dtype), d_nw.to(norm_w.dtype), d_nb_out, None, None, None, None)


BlockSparseDeltaMemory = BankedDeltaMemory
