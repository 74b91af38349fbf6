"""Benchmark: BDM layer prefill tokens/s on B200 (config c2), plus c3 decode, c4 and training.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one process per GPU; every rank runs its own
replica of the c2 workload (batch shards trivially: weak scaling, no
data-path collective).  Rank 0 prints ONE JSON line.

The line also carries ``c4``: the large-memory prefill (batch 16 x 8192,
J = 16384 banks, Zipf(1.1) router skew) on all N GPUs at once -- the plain
layer at N = 1, the bank-sharded forward (bdm_b200.sharded, NCCL all-gather /
reduce-scatter) at N > 1.  Its total work is fixed, so it scales strongly.
``train``: one layer's forward + backward at the c5 layer geometry (batch 32 x
2048 split over the ranks, gradients all-reduced over NCCL at N > 1).
``c5``: a full training step (forward, backward, AdamW) of the 12-layer BDM
language model, batch 32 x 2048 split over the ranks, DDP over NCCL at N > 1.

Timed region (value): K forward steps of the public module call
``layer(hidden)`` with the input already in HBM; an L2 flush (256 MiB write)
runs between steps, outside the per-step CUDA events.  Time is the sum of
per-step event times, maximised over ranks.  ``e2e`` times the same call with
the input copied from pinned host memory and the output copied back inside
each step.  ``roofline`` is for the dominant kernel, the bank recurrence
(bdm_bank_scan), timed with CUDA events on its launch stream in the same steps.
``cpu_baseline`` times the CPU restatement of the reference (oracle/) on the
host cores on a bounded sample.  ``--impl reference`` runs only that CPU
restatement (rank 0; other ranks exit 0).
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# ----------------------------------------------------------------- workloads
C1 = dict(dim=256, bank_count=256, bank_size=8, selected_banks=8, value_width=64, num_heads=1)
C1_BATCH, C1_TIME = 2, 512
C2 = dict(dim=1024, bank_count=256, bank_size=8, selected_banks=8, value_width=1024, num_heads=8)
C2_BATCH, C2_TIME, C2_CHUNK = 8, 4096, 64
E2E_CHUNKS = 4  # row groups of BlockSparseDeltaMemory.forward_host (captured forwards) in the e2e measurement: measured best of 2, 4, 8
C3 = dict(dim=1024, bank_count=2048, bank_size=8, selected_banks=8, value_width=128, num_heads=1)
C3_BATCH, C3_PREFIX, C3_STEPS = 64, 2048, 1024
C4 = dict(dim=2048, bank_count=16384, bank_size=16, selected_banks=16, value_width=2048, num_heads=16)
C4_BATCH, C4_TIME, C4_ZIPF = 16, 8192, 1.1
C5 = dict(dim=768, bank_count=512, bank_size=8, selected_banks=8, value_width=768, num_heads=12)
C5_BATCH, C5_TIME = 32, 2048
C4_WARMUP = C5_WARMUP = 3  # untimed steps before the c4 / c5 timed steps
C5_METRIC = ('BDM layer training step (forward + backward) tokens/sec, c5 layer geometry (batch 32 x seq 2048, '
             'd_model 768, H=12, J=512, S=8, B=8, d_v=64)')
C5_LM = dict(vocab_size=32000, layers=12)
C5_LM_METRIC = ('BDM language-model training tokens/sec (c5: 12 layers, d_model 768, 12 heads, vocab 32000, '
                'J=512, S=8, B=8, d_v=64, SwiGLU; batch 32 x seq 2048, data parallel)')
C4_METRIC = ('BDM layer prefill tokens/sec, bank-sharded large memory (c4: batch 16 x seq 8192, d_model 2048, '
             'H=16, J=16384, S=16, B=16, d_v=128, Zipf(1.1) bank popularity)')
METRIC = 'BDM layer prefill tokens/sec (c2: batch 8 x seq 4096, d_model 1024, H=8, J=256, S=8, B=8, d_v=128)'


def c2_bytes_per_token(cfg=C2, batch=C2_BATCH, time_=C2_TIME):
    """Algorithmic bytes per token of the bank recurrence (fixed per-token definition).

    write events B*(3*H*S*2 + 2*V*2) + read events B*(H*S*2 + V*4) + bank state in/out
    2*(batch*J*H*S*dv*2)/(batch*T).  The layer-level figure adds hidden in/out 2*D*2.
    """
    B, H, S, V, J = cfg['selected_banks'], cfg['num_heads'], cfg['bank_size'], cfg['value_width'], cfg['bank_count']
    dv = V // H
    kernel = B * (3 * H * S * 2 + 2 * V * 2) + B * (H * S * 2 + V * 4) + 2 * (batch * J * H * S * dv * 2) / (batch * time_)
    return kernel, kernel + 2 * cfg['dim'] * 2


def c2_flops_per_token(cfg=C2, chunk=C2_CHUNK):
    """Chunked-form FLOPs per token: 2*B*H*[2(3CS + 2C dv + 3S dv) + (2/3)C^2]."""
    B, H, S, V = cfg['selected_banks'], cfg['num_heads'], cfg['bank_size'], cfg['value_width']
    dv = V // H
    return 2 * B * H * (2 * (3 * chunk * S + 2 * chunk * dv + 3 * S * dv) + (2 / 3) * chunk * chunk)


def c3_bytes_per_token(cfg=C3, batch=C3_BATCH, weight_bytes=0):
    """Decode bytes per token: 3*B*H*S*dv*2 (write tiles in+out, read tiles) + 2*D*2 + weights/batch."""
    B, H, S, V = cfg['selected_banks'], cfg['num_heads'], cfg['bank_size'], cfg['value_width']
    return 3 * B * H * S * (V // H) * 2 + 2 * cfg['dim'] * 2 + weight_bytes / batch


def zipf_router_bias(layer, exponent=C4_ZIPF, seed=3):
    """Add log Zipf(exponent) popularity to each product-key factor's routing bias.

    Each factor's entries get Zipf ranks through a seeded permutation, so bank
    popularity is p1(row) * p2(col); the bias goes on the shared router base,
    i.e. on both the read and the write router.
    """
    j1, j2 = layer.factors
    gen = torch.Generator().manual_seed(seed)
    bias = []
    for width in (j1, j2):
        ranks = torch.randperm(width, generator=gen).double() + 1.0
        pmf = ranks.pow(-exponent)
        bias.append((pmf / pmf.sum()).log())
    with torch.no_grad():
        b = layer.shared_router.base.bias
        b.add_(torch.cat(bias).to(b.dtype).to(b.device))
    layer._fused_cache = None


def c4_bytes_per_token(cfg=C4, batch=C4_BATCH, time_=C4_TIME):
    return c2_bytes_per_token(cfg, batch, time_)


def load_peaks():
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p['hbm_gbs'], p['bf16_tflops'], 'measured'
    return 6650.0, 1590.0, 'fallback'


def load_traffic():
    """DRAM bytes per bank-recurrence launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, 'profiles', 'bank_scan_c2.json')
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get('dram_bytes_per_launch')
    return None


# -------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons while the GPU is under load.

    Sampling starts before the warm-up steps (nvidia-smi needs a few hundred ms
    to produce its first line) and stops after the timed steps; every sample
    taken in between is under load.
    """

    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, device_index, interval_ms=50):
        self.index = device_index
        self.interval_ms = interval_ms
        self.proc = None
        self.out = ''

    def start(self):
        import tempfile
        self.file = tempfile.TemporaryFile(mode='w+')
        try:
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(self.index), f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', str(self.interval_ms)],
                                         stdout=self.file, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return self
        deadline = time.time() + 5.0
        while time.time() < deadline:  # wait for the first sample
            self.file.flush()
            if os.fstat(self.file.fileno()).st_size > 0:
                break
            time.sleep(0.05)
        return self

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            self.file.seek(0)
            self.out = self.file.read()
            self.file.close()

    def summary(self):
        if self.proc is None or not self.out:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable']}
        rows = [r for r in csv.reader(io.StringIO(self.out)) if len(r) >= 9]
        sm, mx, reasons = [], None, set()
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == 'active':
                    reasons.add(name)
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': mx, 'samples': len(sm),
                'reasons': sorted(reasons)}


# ------------------------------------------------------------- distributed
def dist_setup(gpus):
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device('cuda', local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device='cuda')
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


# ------------------------------------------------------------ CPU baseline
def cpu_forward_sample(batch, time_, seed=1):
    """Time the CPU restatement (oracle/) of the c2 layer forward on batch x time_ tokens."""
    import numpy as np

    import oracle
    from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory
    threads = oracle.set_threads(0)
    cfg = BSDMConfig(**C2)
    m = BlockSparseDeltaMemory(cfg, seed=1).to(torch.bfloat16)
    params = {k: v.float().numpy() for k, v in m.state_dict().items()}
    params['initial_row_factor'][:] = 0
    params['initial_column_factor'][:] = 0
    layer = oracle.OracleLayer({k: getattr(cfg, k) for k in cfg.__dataclass_fields__}, params, bf16=True)
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, time_, cfg.dim, generator=gen).to(torch.bfloat16).float().numpy()
    t0 = time.perf_counter()
    y = layer.forward(x)
    dt = time.perf_counter() - t0
    assert np.isfinite(y).all()
    return batch * time_ / dt, dt, threads


def cpu_decode_sample(steps=8, seed=2):
    """Time ``steps`` decode steps of the CPU restatement (oracle/) at c3 (batch 64, J = 2048) on a c3-shaped
    BF16 cache (the product-key initial state: a step's cost does not depend on the cache values)."""
    import numpy as np

    import oracle
    from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory
    threads = oracle.set_threads(0)
    cfg = BSDMConfig(**C3)
    m = BlockSparseDeltaMemory(cfg, seed=2).to(torch.bfloat16)
    params = {k: v.float().numpy() for k, v in m.state_dict().items()}
    layer = oracle.OracleLayer({k: getattr(cfg, k) for k in cfg.__dataclass_fields__}, params, bf16=True)
    state = np.ascontiguousarray(np.broadcast_to(layer.initial_state()[None], (C3_BATCH,) +
                                                 layer.initial_state().shape))
    gen = torch.Generator().manual_seed(seed)
    xs = [torch.randn(C3_BATCH, 1, cfg.dim, generator=gen).to(torch.bfloat16).float().numpy() for _ in range(steps)]
    layer.step(xs[0], state)  # warm-up
    t0 = time.perf_counter()
    for x in xs:
        y, state = layer.step(x, state)
    dt = time.perf_counter() - t0
    assert np.isfinite(y).all()
    return C3_BATCH * steps / dt, dt, threads


def cpu_c4_sample(time_=256, seed=3):
    """Time the CPU restatement of the c4 layer forward (Zipf-skewed router) on one row of time_ tokens."""
    import numpy as np

    import oracle
    from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory
    threads = oracle.set_threads(0)
    cfg = BSDMConfig(**C4)
    m = BlockSparseDeltaMemory(cfg, seed=3)
    zipf_router_bias(m)
    m = m.to(torch.bfloat16)
    params = {k: v.float().numpy() for k, v in m.state_dict().items()}
    layer = oracle.OracleLayer({k: getattr(cfg, k) for k in cfg.__dataclass_fields__}, params, bf16=True)
    gen = torch.Generator().manual_seed(3000 + seed)
    x = torch.randn(1, time_, cfg.dim, generator=gen).to(torch.bfloat16).float().numpy()
    t0 = time.perf_counter()
    y = layer.forward(x)
    dt = time.perf_counter() - t0
    assert np.isfinite(y).all()
    return time_ / dt, dt, threads


def c1_layer(dtype=torch.float32):
    """c1: BSDMConfig(256, 256, 8, 8, 64, 1), seed 0, initial memory N(0, 0.02) (factors N(0, 0.02 / sqrt 2))."""
    from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory
    m = BlockSparseDeltaMemory(BSDMConfig(**C1), seed=0)
    gen = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for f in (m.initial_row_factor, m.initial_column_factor):
            f.copy_(torch.randn(f.shape, generator=gen) * (0.02 / 2 ** 0.5))
    return m.to(dtype)


def cpu_c1_sample():
    """The CPU restatement of the c1 layer forward in full (batch 2 x 512, FP32)."""
    import numpy as np

    import oracle
    threads = oracle.set_threads(0)
    m = c1_layer()
    params = {k: v.float().numpy() for k, v in m.state_dict().items()}
    layer = oracle.OracleLayer({k: getattr(m.config, k) for k in m.config.__dataclass_fields__}, params, bf16=False)
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(C1_BATCH, C1_TIME, C1['dim'], generator=gen).numpy()
    t0 = time.perf_counter()
    y = layer.forward(x)
    dt = time.perf_counter() - t0
    assert np.isfinite(y).all()
    return C1_BATCH * C1_TIME / dt, dt, threads


def run_c1(dev, rank, world, args):
    """c1 (the reference's CPU-runnable case) on one GPU: forward of batch 2 x 512, FP32, CUDA events."""
    m = c1_layer().to(dev)
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(C1_BATCH, C1_TIME, C1['dim'], generator=gen).to(dev)
    steps = 20
    with torch.inference_mode():
        for _ in range(3):
            m(x)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            m(x)
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    out = {'metric': 'BDM layer forward tokens/sec (c1: batch 2 x seq 512, d_model 256, J=256, S=8, B=8, d_v=64, '
                     'FP32 activations, BF16 state storage policy)',
           'value': C1_BATCH * C1_TIME / (ms / 1000), 'unit': 'tokens/s', 'steps': steps, 'warmup': 3,
           'ms_per_step': ms, 'path': 'BlockSparseDeltaMemory.forward (one GPU; launch-bound at 1024 tokens)'}
    if rank == 0 and world == 1 and not args.skip_cpu:
        tps, dt, threads = cpu_c1_sample()
        out['cpu_baseline'] = {'value': tps, 'unit': 'tokens/s', 'cores': threads, 'kind': 'port',
                               'sample': f'full c1 forward, batch {C1_BATCH} x seq {C1_TIME} ({dt:.2f} s), '
                                         'CPU restatement oracle/'}
    return out


def cpu_train_sample(batch, time_, seed=4):
    """Time one forward + backward of the c5 layer (BF16) with the gradient oracle (torch autograd
    over the CPU restatement, oracle/grad.py) on batch x time_ tokens, on the host cores."""
    from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory
    from oracle.grad import layer_grads
    cfg = BSDMConfig(**C5)
    m = BlockSparseDeltaMemory(cfg, seed=seed).to(torch.bfloat16)
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, time_, cfg.dim, generator=gen).to(torch.bfloat16)
    dy = torch.randn(batch, time_, cfg.dim, generator=gen).to(torch.bfloat16)
    t0 = time.perf_counter()
    grads, _, _ = layer_grads(sd, x, dy, {k: getattr(cfg, k) for k in cfg.__dataclass_fields__})
    dt = time.perf_counter() - t0
    assert all(torch.isfinite(g.float()).all() for g in grads.values())
    return batch * time_ / dt, dt, torch.get_num_threads()


def run_reference(args, world, rank):
    if rank != 0:
        return
    batch, time_ = C2_BATCH, 512
    for _ in range(args.warmup):
        cpu_forward_sample(batch, time_)
    total_tok, total_s, threads = 0, 0.0, 1
    for i in range(args.steps):
        tps, dt, threads = cpu_forward_sample(batch, time_, seed=1 + i)
        total_tok += batch * time_
        total_s += dt
    value = total_tok / total_s
    sample = f'c2 geometry truncated to batch {batch} x seq {time_} per step (CPU restatement oracle/, BF16 emulated)'
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': 'tokens/s', 'n_gpus': args.gpus,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': 1000 * total_s / args.steps,
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic',
        'config': {'workload': 'c2 prefill (truncated sample)', 'global_batch': batch, 'seq_len': time_,
                   'parallelism': 'cpu'},
        'cpu_baseline': {'value': value, 'unit': 'tokens/s', 'cores': threads, 'kind': 'port', 'sample': sample},
        'e2e': {'value': value, 'unit': 'tokens/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- ours
def run_ours(args, world, rank, local):
    from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory, _lib
    dev = torch.device('cuda', local)
    lib = _lib.load()
    hbm_peak, bf16_peak, peak_kind = load_peaks()

    cfg = BSDMConfig(**C2)
    layer = BlockSparseDeltaMemory(cfg, seed=1).to(torch.bfloat16).to(dev)
    with torch.no_grad():  # c2: bank states start at zero
        layer.initial_row_factor.zero_()
        layer.initial_column_factor.zero_()
    gen = torch.Generator().manual_seed(1 + rank)
    x_host = torch.randn(args.batch, C2_TIME, cfg.dim, generator=gen).to(torch.bfloat16).pin_memory()
    x = x_host.to(dev)
    y_host = torch.empty_like(x_host).pin_memory()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    tokens = args.batch * C2_TIME

    clocks = ClockSampler(dev.index).start()
    with torch.inference_mode():
        for _ in range(args.warmup):
            layer(x)
        torch.cuda.synchronize()
        # ------------------------------------------------------- value
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        layer.scan_events = []
        barrier(world)
        torch.cuda.synchronize()
        launches0 = lib.bdm_kernel_launches()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            layer(x)
            ends[i].record()
        torch.cuda.synchronize()
        clocks.stop()
        barrier(world)
        launches = lib.bdm_kernel_launches() - launches0
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        scan_ms = [s.elapsed_time(e) for s, e in layer.scan_events]
        layer.scan_events = None
        total_ms = max_over_ranks(sum(step_ms), world)
        scan_mean = max_over_ranks(statistics.mean(scan_ms), world)
        # --------------------------------------------------------- e2e
        for _ in range(args.warmup):  # the row groups run the forward at their own shapes: warm those too
            layer.forward_host(x_host, y_host, chunks=E2E_CHUNKS)
        barrier(world)
        torch.cuda.synchronize()
        # K back-to-back calls timed as one interval (a call's first uploads overlap the previous
        # call's last groups, as in a serving loop); no L2 flush: the forward's working set (read
        # outputs alone 0.5 GB) is far larger than L2, and every call's data comes from the host
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record()
        for i in range(args.steps):
            # host in, host out: the layer streams the batch through in row groups, copies overlapped
            layer.forward_host(x_host, y_host, chunks=E2E_CHUNKS)
        e_end.record()
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)

    value = world * tokens * args.steps / (total_ms / 1000)
    kernel_bytes, layer_bytes = c2_bytes_per_token(batch=args.batch)
    achieved = kernel_bytes * tokens / (scan_mean / 1000) / 1e9
    flops = c2_flops_per_token() * tokens
    roof_ms = max(flops / (bf16_peak * 1e12), layer_bytes * tokens / (hbm_peak * 1e9)) * 1000
    line = {
        'metric': METRIC, 'value': value, 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': total_ms / args.steps, 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (x ~ N(0,1), seed 1 + rank; random-init weights, seed 1)',
        'config': {'workload': 'c2 BDM layer prefill forward: BSDMConfig(dim=1024, bank_count=256, bank_size=8, '
                               'selected_banks=8, value_width=1024, num_heads=8), zero initial banks',
                   'global_batch': args.batch * world, 'seq_len': C2_TIME, 'parallelism': f'dp{world} replicas',
                   'l2': 'flushed between timed steps (256 MiB write, outside the step events)'},
        'gpu_launches': int(launches),
        'e2e': {'value': world * tokens * args.steps / (e2e_ms / 1000), 'unit': 'tokens/s',
                'h2d_bytes_per_step': x_host.numel() * x_host.element_size(),
                'd2h_bytes_per_step': y_host.numel() * y_host.element_size(),
                'path': f'BlockSparseDeltaMemory.forward_host (pinned host in and out, {E2E_CHUNKS} row groups as '
                        'replays of captured forwards, uploads / downloads overlapped with compute)',
                'timing': f'{args.steps} back-to-back calls as one CUDA-event interval, no L2 flush between calls'},
        'roofline': {'kernel': 'bdm_bank_scan (bank_scan_kernel<bf16, S=8, 8 columns/lane, 2 heads/warp>)',
                     'bound': 'hbm',
                     'achieved': achieved, 'peak': hbm_peak, 'unit': 'GB/s', 'frac': achieved / hbm_peak,
                     'peak_source': peak_kind, 'kernel_ms': scan_mean, 'bytes_per_token': kernel_bytes,
                     'traffic': load_traffic(),
                     'layer_frac': roof_ms / (total_ms / args.steps), 'layer_roofline_ms': roof_ms},
        'clocks': clocks.summary(),
    }
    if not args.skip_scan_variants:
        try:
            line['scan_variants'] = run_scan_variants(layer, x, dev, args)
        except Exception as e:  # keep the headline line even if the extra workload fails
            line['scan_variants'] = {'error': repr(e)[:300]}
    if not args.skip_output_variants:
        try:
            line['output_variants'] = run_output_variants(layer, x, dev, args)
        except Exception as e:  # keep the headline line even if the extra workload fails
            line['output_variants'] = {'error': repr(e)[:300]}
    if args.reference_gpu and rank == 0 and world == 1:
        line['reference_gpu'] = run_reference_gpu(dev, args)
    if not args.skip_c1 and world == 1:
        try:
            line['c1'] = run_c1(dev, rank, world, args)
        except Exception as e:  # keep the headline line even if the extra workload fails
            line['c1'] = {'error': repr(e)[:300]}
    if not args.skip_decode:
        try:
            line['decode'] = run_decode(dev, rank, world, args)
        except Exception as e:  # keep the headline line even if the extra workload fails
            line['decode'] = {'error': repr(e)[:300]}
    if not args.skip_c4:
        try:
            line['c4'] = run_c4(dev, rank, world, args)
        except Exception as e:  # keep the headline line even if the extra workload fails
            line['c4'] = {'error': repr(e)[:300]}
    if not args.skip_train:
        try:
            line['train'] = run_train(dev, rank, world, args)
        except Exception as e:  # keep the headline line even if the extra workload fails
            line['train'] = {'error': repr(e)[:300]}
    if not args.skip_c5:
        try:
            line['c5'] = run_c5(dev, rank, world, args)
        except Exception as e:  # keep the headline line even if the extra workload fails
            line['c5'] = {'error': repr(e)[:300]}
    if rank == 0 and world == 1 and not args.skip_cpu and isinstance(line.get('train'), dict) \
            and 'value' in line['train']:
        tps, dt, threads = cpu_train_sample(args.cpu_train_batch, C5_TIME)
        line['train']['cpu_baseline'] = {
            'value': tps, 'unit': 'tokens/s', 'cores': threads, 'kind': 'port',
            'sample': f'c5 layer forward + backward, batch {args.cpu_train_batch} x seq {C5_TIME} ({dt:.1f} s), '
                      f'torch autograd over the CPU restatement oracle/grad.py'}
    if rank == 0 and world == 1 and not args.skip_cpu:
        tps, dt, threads = cpu_forward_sample(C2_BATCH, args.cpu_time)
        line['cpu_baseline'] = {'value': tps, 'unit': 'tokens/s', 'cores': threads, 'kind': 'port',
                                'sample': f'full c2 layer forward, batch {C2_BATCH} x seq {args.cpu_time} '
                                          f'({dt:.1f} s) with the CPU restatement oracle/'}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_scan_variants(layer, x, dev, args):
    """The c2 recurrence alone on the layer's own controls and routes: the default per-event kernel
    (bdm_bank_scan) and the tensor-core chunked kernel (bdm_bank_scan_chunked), CUDA events around
    each call, the 256 MiB L2 flush between calls."""
    from bdm_b200 import ops, state_interval
    batch, time_ = x.shape[0], x.shape[1]
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    with torch.inference_mode():
        controls, routes, _ = layer._controls_and_routes(x)
        ww, wi, rw, ri = routes
        meta = ops.dispatch(wi, ri, layer.bank_count)
        args_ = (*controls, wi, ww, ri, rw, meta['order'], meta['cu_seqlens'])
        kw = dict(batch=batch, time=time_, bank_count=layer.bank_count, heads=layer.num_heads,
                  bank_size=layer.bank_size, head_value_width=layer.head_value_width,
                  routed_decay=layer.config.routed_decay, scale=layer.bank_size ** -0.5,
                  row_factor=layer.initial_row_factor, col_factor=layer.initial_column_factor,
                  state_interval=state_interval(layer.bank_size))
        out = {}
        for name, chunked in (('per_event', False), ('chunked_tensor_core', True)):
            for _ in range(3):
                ops.bank_scan(*args_, **kw, chunked=chunked)
            times = []
            for _ in range(max(args.steps, 3)):
                flush.zero_()
                s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s_.record()
                ops.bank_scan(*args_, **kw, chunked=chunked)
                e_.record()
                torch.cuda.synchronize()
                times.append(s_.elapsed_time(e_))
            out[name] = {'kernel_ms': statistics.mean(times), 'min_ms': min(times)}
    hbm_peak, _, _ = load_peaks()
    kernel_bytes, _ = c2_bytes_per_token(batch=batch)
    for v in out.values():
        v['achieved_gbs'] = kernel_bytes * batch * time_ / (v['kernel_ms'] / 1000) / 1e9
        v['frac'] = v['achieved_gbs'] / hbm_peak
    return {'what': 'c2 recurrence alone (bdm_bank_scan vs bdm_bank_scan_chunked), same inputs, BF16 storage policy',
            **out}


def run_output_variants(layer, x, dev, args):
    """The c2 output interface alone on the layer's own read rows: bdm_combine_norm_gate followed by
    the cuBLAS o_proj (the forward's default), and the fused tensor-core bdm_combine_project (the
    o_proj input never written to memory); CUDA events around each, the 256 MiB L2 flush between."""
    from bdm_b200 import ops, state_interval
    from torch.nn import functional as F
    batch, time_ = x.shape[0], x.shape[1]
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    with torch.inference_mode():
        controls, routes, gate = layer._controls_and_routes(x)
        reads = layer._bank_pass(controls, routes, batch, time_, row_factor=layer.initial_row_factor,
                                 col_factor=layer.initial_column_factor,
                                 state_interval=state_interval(layer.bank_size))
        ri = routes[3].reshape(batch * time_, -1)
        rd = reads.reshape(batch * time_, ri.shape[-1], -1)
        nb = getattr(layer, 'output_norm_bias', None)
        ln = layer.config.output_normalization == 'layer'
        w, b = layer.o_proj.weight, layer.o_proj.bias

        def unfused():
            n = ops.combine_norm_gate(rd, ri, gate, layer.output_norm_weight, nb, eps=layer.norm_eps, layer_norm=ln,
                                      round_each=False)
            return F.linear(n, w, b)

        def fused():
            return ops.combine_project(rd, ri, gate, layer.output_norm_weight, nb, w, b, eps=layer.norm_eps,
                                       layer_norm=ln, round_each=False)
        out = {}
        for name, fn in (('combine_then_cublas', unfused), ('fused_combine_project', fused)):
            for _ in range(3):
                fn()
            times = []
            for _ in range(max(args.steps, 3)):
                flush.zero_()
                s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s_.record()
                fn()
                e_.record()
                torch.cuda.synchronize()
                times.append(s_.elapsed_time(e_))
            out[name] = {'ms': statistics.mean(times), 'min_ms': min(times)}
        diff = (unfused().float() - fused().float()).abs().max().item()
    return {'what': 'c2 read combine + norm + gate + o_proj, same inputs: two launches vs one fused kernel',
            'max_abs_diff': diff, **out}


def run_reference_gpu(dev, args):
    """The reference's own GPU path on this GPU (its Triton 'role' backend, unmodified, from the copy
    installed in baseline/_ref): the c2 forward and the c3 prefill + eager steps, CUDA events."""
    ref_dir = os.path.join(ROOT, 'baseline', '_ref')
    if not os.path.isdir(os.path.join(ref_dir, 'bsdm')):
        return {'unavailable': 'reference not installed in baseline/_ref'}
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    try:
        import bsdm
    except Exception as e:  # noqa: BLE001
        return {'unavailable': f'import failed: {e!r}'[:300]}
    out = {'path': "bsdm.BlockSparseDeltaMemory(backend='role') (reference Triton kernels), unmodified"}
    try:
        cfg = bsdm.BSDMConfig(**C2)
        layer = bsdm.BlockSparseDeltaMemory(cfg, seed=1, backend='role').to(torch.bfloat16).to(dev)
        with torch.no_grad():
            layer.initial_row_factor.zero_()
            layer.initial_column_factor.zero_()
        gen = torch.Generator().manual_seed(1)
        x = torch.randn(C2_BATCH, C2_TIME, cfg.dim, generator=gen).to(torch.bfloat16).to(dev)
        with torch.no_grad():
            for _ in range(3):  # warm-up (Triton compilation and autotuning happen on the first call)
                layer(x)
            torch.cuda.synchronize()
            n = 3
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            for _ in range(n):
                layer(x)
            e_.record()
            torch.cuda.synchronize()
        ms = s_.elapsed_time(e_) / n
        out['c2_forward'] = {'ms_per_step': ms, 'value': C2_BATCH * C2_TIME / (ms / 1000), 'unit': 'tokens/s',
                             'steps': n, 'warmup': 3}
        del layer, x
    except Exception as e:  # noqa: BLE001
        out['c2_forward'] = {'error': repr(e)[:300]}
    try:
        cfg = bsdm.BSDMConfig(**C3)
        layer = bsdm.BlockSparseDeltaMemory(cfg, seed=2, backend='role').to(torch.bfloat16).to(dev)
        gen = torch.Generator().manual_seed(2)
        prefix = torch.randn(C3_BATCH, C3_PREFIX, cfg.dim, generator=gen).to(torch.bfloat16).to(dev)
        toks = torch.randn(72, C3_BATCH, 1, cfg.dim, generator=gen).to(torch.bfloat16).to(dev)
        with torch.no_grad():
            layer.prefill(prefix[:1, :64])  # compiles its kernels
            torch.cuda.synchronize()
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            _, state = layer.prefill(prefix)
            e_.record()
            torch.cuda.synchronize()
            prefill_ms = s_.elapsed_time(e_)
            for i in range(8):
                _, state = layer.step(toks[64 + i], state)
            torch.cuda.synchronize()
            s_.record()
            for i in range(64):
                _, state = layer.step(toks[i], state)
            e_.record()
            torch.cuda.synchronize()
        step_ms = s_.elapsed_time(e_) / 64
        out['c3'] = {'prefill_ms': prefill_ms, 'step_ms': step_ms,
                     'decode_value': C3_BATCH / (step_ms / 1000), 'unit': 'tokens/s', 'steps': 64, 'warmup': 8,
                     'note': 'eager steps (the reference records cuda_graph=False for its sustained decode)'}
    except Exception as e:  # noqa: BLE001
        out['c3'] = {'error': repr(e)[:300]}
    return out


def run_decode(dev, rank, world, args):
    """c3: 1024 single-token steps at batch 64 on a state pre-filled by a 2048-token prefill.

    The timed loop replays the CUDA-graphed step (``capture_step``); the per-call ``step``
    path is timed on a short loop beside it.
    """
    from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory
    cfg = BSDMConfig(**C3)
    layer = BlockSparseDeltaMemory(cfg, seed=2).to(torch.bfloat16).to(dev)
    gen = torch.Generator().manual_seed(2 + rank)
    prefix = torch.randn(C3_BATCH, C3_PREFIX, cfg.dim, generator=gen).to(torch.bfloat16).to(dev)
    steps = args.decode_steps
    toks = torch.randn(steps + 8, C3_BATCH, 1, cfg.dim, generator=gen).to(torch.bfloat16).to(dev)
    with torch.inference_mode():
        _, state = layer.prefill(prefix)
        run = layer.capture_step(state)
        for i in range(8):
            run(toks[steps + i])
        torch.cuda.synchronize()
        barrier(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(steps):
            run(toks[i])
        end.record()
        torch.cuda.synchronize()
        eager_n = min(64, steps + 8)
        es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        es.record()
        for i in range(eager_n):
            layer.step(toks[i], state)
        ee.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world)
    eager_ms = es.elapsed_time(ee) / eager_n
    del state, run
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        tps_cpu, dt, threads = cpu_decode_sample()
        cpu = {'value': tps_cpu, 'unit': 'tokens/s', 'cores': threads, 'kind': 'port',
               'sample': f'8 decode steps at batch {C3_BATCH} ({dt:.2f} s) on a c3-shaped BF16 cache, '
                         'CPU restatement oracle/ (controllers, routers, the per-bank step and the output)'}
    weight_bytes = sum(p.numel() * p.element_size() for p in layer.parameters())
    hbm_peak, _, _ = load_peaks()
    bpt = c3_bytes_per_token(weight_bytes=weight_bytes)
    tps = world * C3_BATCH * steps / (ms / 1000)
    return {'metric': 'BDM decode tokens/sec (c3: batch 64, J=2048, S=8, B=8, d_v=128, 2048-token prefill)',
            'value': tps, 'unit': 'tokens/s', 'steps': steps, 'ms_per_step': ms / steps,
            'path': 'CUDA-graphed step (BlockSparseDeltaMemory.capture_step)',
            'eager_step_ms': eager_ms, 'state_bytes': C3_BATCH * C3['bank_count'] * C3['bank_size'] * C3['value_width'] * 2,
            **({'cpu_baseline': cpu} if cpu else {}),
            'roofline': {'bound': 'hbm', 'bytes_per_token': bpt, 'achieved': bpt * tps / world / 1e9,
                         'peak': hbm_peak, 'unit': 'GB/s', 'frac': bpt * tps / world / 1e9 / hbm_peak}}


def c5_gemm_flops(tokens, cfg=C5):
    """Dense GEMM FLOPs of one layer training step: fused input projection, f_proj.1 and o_proj,
    forward (1x) plus backward (2x: input and weight gradients)."""
    H, S, V, D = cfg['num_heads'], cfg['bank_size'], cfg['value_width'], cfg['dim']
    dv = V // H
    j = cfg['bank_count']
    first = 1
    while first * first <= j:
        first += 1
    first -= 1
    while j % first:
        first -= 1
    route = first + j // first
    width = 3 * H * S + 2 * V + dv + 2 * route + V  # q k b | v w | f1 | read write | gate
    per_token = 2 * D * width + 2 * dv * H * S + 2 * V * D
    return 3 * per_token * tokens


def run_train(dev, rank, world, args):
    """c5 layer geometry: forward + backward of one BDM layer (BF16), the global batch split over the
    ranks; at N > 1 the layer's parameter gradients are all-reduced over NCCL (data parallel)."""
    from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory, _lib
    batch = args.train_batch
    if batch % world:
        return {'skipped': f'batch {batch} does not split over {world} ranks'}
    lib = _lib.load()
    cfg = BSDMConfig(**C5)
    layer = BlockSparseDeltaMemory(cfg, seed=4).to(torch.bfloat16).to(dev)
    rows = batch // world
    gen = torch.Generator(device=dev).manual_seed(4000 + rank)
    x = torch.randn(rows, C5_TIME, cfg.dim, generator=gen, device=dev).to(torch.bfloat16)
    dy = torch.randn(rows, C5_TIME, cfg.dim, generator=gen, device=dev).to(torch.bfloat16)
    params = [p for p in layer.parameters()]
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    steps = args.train_steps

    def step():
        for p in params:
            p.grad = None
        y = layer(x)
        y.backward(dy)
        if world > 1:
            flat = torch.cat([p.grad.reshape(-1).float() for p in params])
            torch.distributed.all_reduce(flat)

    clocks = ClockSampler(dev.index).start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    layer.backward_events = []
    barrier(world)
    torch.cuda.synchronize()
    launches0 = lib.bdm_kernel_launches()
    for i in range(steps):
        flush.zero_()
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    clocks.stop()
    launches = lib.bdm_kernel_launches() - launches0
    barrier(world)
    scan_bwd_ms = max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in layer.backward_events), world)
    layer.backward_events = None
    ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)), world) / steps
    tokens = batch * C5_TIME
    _, bf16_peak, peak_kind = load_peaks()
    gemm_ms = c5_gemm_flops(tokens // world) / (bf16_peak * 1e12) * 1000
    return {'metric': C5_METRIC, 'value': tokens / (ms / 1000), 'unit': 'tokens/s', 'n_gpus': world,
            'steps': steps, 'warmup': args.warmup, 'ms_per_step': ms, 'scaling': 'strong',
            'dtype': 'bf16', 'path': 'BlockSparseDeltaMemory.forward + autograd backward (bdm_b200 CUDA kernels)'
                                     + (', NCCL all-reduce of the parameter gradients' if world > 1 else ''),
            'config': {'workload': 'c5 layer: BSDMConfig(dim=768, bank_count=512, bank_size=8, selected_banks=8, '
                                   'value_width=768, num_heads=12), seed 4, random-init; one layer, no LM shell',
                       'global_batch': batch, 'seq_len': C5_TIME, 'rows_per_rank': rows,
                       'l2': 'inputs larger than L2; 256 MiB flush between steps'},
            'gpu_launches': int(launches),
            'scan_backward_ms': scan_bwd_ms,
            'roofline': {'bound': 'tensor', 'what': 'the step\'s dense GEMMs (projection, f_proj.1, o_proj; fwd+bwd) '
                                                   'at the measured bf16 peak: a lower bound on the step',
                         'gemm_floor_ms': gemm_ms, 'peak': bf16_peak, 'unit': 'TFLOP/s', 'peak_source': peak_kind,
                         'frac': gemm_ms / ms},
            'clocks': clocks.summary()}


def run_c5(dev, rank, world, args):
    """c5: one training step (forward, backward, fused AdamW) of the 12-layer BDM language model in BF16,
    the global batch of uniform-random token ids split over the ranks; DDP (NCCL) at N > 1."""
    from bdm_b200 import BSDMConfig, _lib
    from bdm_b200.lm import BDMLanguageModel, LanguageModelConfig
    batch = args.c5_batch
    if batch % world:
        return {'skipped': f'batch {batch} does not split over {world} ranks'}
    lib = _lib.load()
    rows = batch // world
    cfg = LanguageModelConfig(memory=BSDMConfig(**C5), vocab_size=C5_LM['vocab_size'], layers=C5_LM['layers'],
                              seed=4)
    model = BDMLanguageModel(cfg).to(torch.bfloat16).to(dev)
    params = sum(p.numel() for p in model.parameters())
    gemm_params = sum(m.weight.numel() for m in model.modules() if isinstance(m, torch.nn.Linear))
    net = model
    if world > 1:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[dev.index])
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    gen = torch.Generator(device=dev).manual_seed(4000 + rank)
    tokens = torch.randint(0, cfg.vocab_size, (rows, C5_TIME + 1), generator=gen, device=dev)
    inp, tgt = tokens[:, :-1].contiguous(), tokens[:, 1:].contiguous()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    steps = args.c5_steps

    def step():
        opt.zero_grad(set_to_none=True)
        loss = net(inp, tgt)
        loss.backward()
        opt.step()
        return loss

    clocks = ClockSampler(dev.index).start()
    for _ in range(C5_WARMUP):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier(world)
    torch.cuda.synchronize()
    launches0 = lib.bdm_kernel_launches()
    for i in range(steps):
        flush.zero_()
        starts[i].record()
        loss = step()
        ends[i].record()
    torch.cuda.synchronize()
    clocks.stop()
    launches = lib.bdm_kernel_launches() - launches0
    barrier(world)
    ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)), world) / steps
    tokens_step = batch * C5_TIME
    _, bf16_peak, peak_kind = load_peaks()
    dense_flops = 6 * gemm_params * tokens_step  # every GEMM weight: forward + two backward products
    floor_ms = dense_flops / world / (bf16_peak * 1e12) * 1000
    out = {'metric': C5_LM_METRIC, 'value': tokens_step / (ms / 1000), 'unit': 'tokens/s', 'n_gpus': world,
           'steps': steps, 'warmup': C5_WARMUP, 'ms_per_step': ms, 'scaling': 'strong', 'dtype': 'bf16',
           'loss': float(loss.item()),
           'path': 'bdm_b200.lm.BDMLanguageModel (B200 BDM layers, cuBLAS SwiGLU/head), fused AdamW'
                   + (', DistributedDataParallel over NCCL' if world > 1 else ''),
           'config': {'workload': 'c5: 12 x BSDMConfig(dim=768, bank_count=512, bank_size=8, selected_banks=8, '
                                  'value_width=768, num_heads=12) + SwiGLU FFN, vocab 32000, seed 4, random init',
                      'parameters': params, 'global_batch': batch, 'seq_len': C5_TIME, 'rows_per_rank': rows,
                      'data': 'uniform-random token ids (seed 4000 + rank), next-token targets',
                      'l2': 'working set larger than L2; 256 MiB flush between steps'},
           'gpu_launches': int(launches),
           'roofline': {'bound': 'tensor', 'what': '6 x GEMM parameters x tokens at the measured bf16 peak',
                        'dense_floor_ms': floor_ms, 'peak': bf16_peak, 'unit': 'TFLOP/s', 'peak_source': peak_kind,
                        'achieved': dense_flops / world / (ms / 1000) / 1e12, 'frac': floor_ms / ms},
           'clocks': clocks.summary()}
    del net, model, opt
    return out


def c4_hidden(rows, dev):
    """c4 input rows: row b of the global batch is N(0,1) from seed 3000 + b, for any rank count."""
    out = torch.empty(len(rows), C4_TIME, C4['dim'], dtype=torch.bfloat16, device=dev)
    for i, b in enumerate(rows):
        gen = torch.Generator(device=dev).manual_seed(3000 + b)
        out[i] = torch.randn(C4_TIME, C4['dim'], generator=gen, device=dev).to(torch.bfloat16)
    return out


def run_c4(dev, rank, world, args):
    """c4 bank-sharded large-memory prefill forward on all ranks together (strong scaling)."""
    from bdm_b200 import BSDMConfig, BlockSparseDeltaMemory, _lib
    from bdm_b200.sharded import BankShardedMemory
    if C4_BATCH % world:
        return {'skipped': f'batch {C4_BATCH} does not split over {world} ranks'}
    lib = _lib.load()
    cfg = BSDMConfig(**C4)
    layer = BlockSparseDeltaMemory(cfg, seed=3).to(torch.bfloat16).to(dev)
    zipf_router_bias(layer)
    rows = C4_BATCH // world
    x = c4_hidden(range(rank * rows, (rank + 1) * rows), dev)
    fwd = layer if world == 1 else BankShardedMemory(layer, ownership=args.c4_ownership)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    steps = args.c4_steps
    clocks = ClockSampler(dev.index).start()
    with torch.inference_mode():
        for _ in range(C4_WARMUP):
            fwd(x)
        torch.cuda.synchronize()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        barrier(world)
        torch.cuda.synchronize()
        launches0 = lib.bdm_kernel_launches()
        for i in range(steps):
            flush.zero_()
            starts[i].record()
            fwd(x)
            ends[i].record()
        torch.cuda.synchronize()
        clocks.stop()
        launches = lib.bdm_kernel_launches() - launches0
        barrier(world)
    ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)), world) / steps
    tokens = C4_BATCH * C4_TIME
    hbm_peak, _, peak_kind = load_peaks()
    _, layer_bytes = c4_bytes_per_token()
    roof_ms = layer_bytes * tokens / (hbm_peak * 1e9 * world) * 1000
    out = {'metric': C4_METRIC, 'value': tokens / (ms / 1000), 'unit': 'tokens/s', 'n_gpus': world,
           'steps': steps, 'warmup': C4_WARMUP, 'ms_per_step': ms, 'scaling': 'strong',
           'path': 'BlockSparseDeltaMemory.forward' if world == 1 else
                   f'BankShardedMemory (bank-sharded, {args.c4_ownership} partition, NCCL all-gather/reduce-scatter)',
           'config': {'workload': 'c4: BSDMConfig(dim=2048, bank_count=16384, bank_size=16, selected_banks=16, '
                                  'value_width=2048, num_heads=16), seed 3, Zipf(1.1) bias on both router factors',
                      'global_batch': C4_BATCH, 'seq_len': C4_TIME, 'rows_per_rank': rows,
                      'l2': 'inputs larger than L2; 256 MiB flush between steps'},
           'gpu_launches': int(launches),
           'roofline': {'bound': 'hbm', 'bytes_per_token': layer_bytes, 'peak': hbm_peak, 'peak_source': peak_kind,
                        'unit': 'GB/s', 'achieved': layer_bytes * tokens / (ms / 1000) / 1e9 / world,
                        'frac': roof_ms / ms, 'roofline_ms': roof_ms},
           'clocks': clocks.summary()}
    if rank == 0 and world == 1 and not args.skip_cpu:
        tps_cpu, dt, threads = cpu_c4_sample()
        out['cpu_baseline'] = {'value': tps_cpu, 'unit': 'tokens/s', 'cores': threads, 'kind': 'port',
                               'sample': f'c4 layer forward truncated to batch 1 x seq 256 ({dt:.1f} s; truncated T), '
                                         'CPU restatement oracle/'}
    if world > 1 and args.c4_ownership == 'balanced':
        # the bank table as contiguous index ranges (rank r owns [r J/R, (r+1) J/R)), timed the same way
        ranges = BankShardedMemory(layer, ownership='contiguous')
        with torch.inference_mode():
            ranges(x)
            torch.cuda.synchronize()
            barrier(world)
            cs, ce = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            cs.record()
            for _ in range(steps):
                ranges(x)
            ce.record()
            torch.cuda.synchronize()
            barrier(world)
        c_ms = max_over_ranks(cs.elapsed_time(ce), world) / steps
        owner, _, _, counts = ranges.last_partition
        load = torch.zeros(world, dtype=torch.float64, device=dev).index_add_(0, owner.long(), counts.double())
        out['contiguous_partition'] = {'ms_per_step': c_ms, 'value': tokens / (c_ms / 1000),
                                       'partition_load_max_over_mean': (load.max() / load.mean()).item()}
    if world > 1 and fwd.last_partition is not None:
        owner, _, _, counts = fwd.last_partition
        load = torch.zeros(world, dtype=torch.float64, device=dev).index_add_(0, owner.long(), counts.double())
        out['partition_load_max_over_mean'] = (load.max() / load.mean()).item()
        # one more (untimed) step with per-phase CUDA events; every rank reports, rank 0 prints the max
        with torch.inference_mode():
            fwd.phase_events = []
            barrier(world)
            fwd(x)
            torch.cuda.synchronize()
            phases = fwd.phase_times()
            fwd.phase_events = None
        out['phases_ms_max_over_ranks'] = {k: max_over_ranks(v, world) for k, v in phases.items()}
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=10)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', choices=('ours', 'reference'), default='ours')
    ap.add_argument('--batch', type=int, default=C2_BATCH, help='c2 batch (8 is the benchmark; smaller for profiling)')
    ap.add_argument('--decode-steps', type=int, default=C3_STEPS)
    ap.add_argument('--cpu-time', type=int, default=C2_TIME, help='sequence length of the CPU baseline sample')
    ap.add_argument('--skip-decode', action='store_true')
    ap.add_argument('--skip-c1', action='store_true')
    ap.add_argument('--reference-gpu', action='store_true',
                    help="also time the reference's own Triton GPU path (installed in baseline/_ref)")
    ap.add_argument('--skip-scan-variants', action='store_true')
    ap.add_argument('--skip-output-variants', action='store_true')
    ap.add_argument('--skip-cpu', action='store_true')
    ap.add_argument('--skip-c4', action='store_true')
    ap.add_argument('--c4-steps', type=int, default=5)
    ap.add_argument('--c4-ownership', choices=('balanced', 'contiguous'), default='balanced')
    ap.add_argument('--skip-train', action='store_true')
    ap.add_argument('--cpu-train-batch', type=int, default=2, help='rows (x 2048 tokens) of the training CPU sample')
    ap.add_argument('--skip-c5', action='store_true')
    ap.add_argument('--c5-steps', type=int, default=3)
    ap.add_argument('--c5-batch', type=int, default=32, help='c5 global batch (32 is the benchmark)')
    ap.add_argument('--train-steps', type=int, default=3)
    ap.add_argument('--train-batch', type=int, default=C5_BATCH, help='c5 batch (32 is the benchmark)')
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == 'ours':
        args.warmup = 3
    if args.impl == 'reference':
        world = int(os.environ.get('WORLD_SIZE', '1'))
        rank = int(os.environ.get('RANK', '0'))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == '__main__':
    main()
