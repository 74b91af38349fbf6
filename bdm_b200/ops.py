"""Torch-facing wrappers of the sm_100a kernels.

Each function validates shapes, allocates outputs with the PyTorch caching
allocator, and calls one C-ABI entry point on the current CUDA stream.
Nothing here computes on the host; a CPU tensor is an error.

Reference interfaces each op replaces (p0rc314in/bdm, implementation/bdm/):
  route            gdn2_banks.py:74-114          product_key_route
  dispatch         role_bank_dispatch.py:143-153 metadata (keys, sort, bounds)
  controllers      _parameters.py:189-220        _controllers (after the GEMM)
  product_state    _parameters.py:40-67          materialize_initial_state
  bank_scan        routed_update.py:16-32, role_bank_kernel.py:177-202, inference.py:134-158
  combine_norm_gate role_bank_dispatch.py:219-231, _parameters.py:222-232
  combine_project  role_bank_dispatch.py:201-216 + _parameters.py:222-232 (with o_proj)
  decode_step      inference.py:161-194
Bank-sharded forward (no reference counterpart; the reference runs on one device):
  bank_histogram, bank_owners, dispatch_owned, combine_partial, norm_gate_f32
Training backward:
  norm_gate_backward     autograd of _project_bank_output (_parameters.py:222-232)
  scan_backward          role_bank_kernel.py:76-150 (checkpoint replay + reverse chain)
  event_vjp              role_bank_dispatch.py:76-132 + routed_update.py:43-47
  product_state_backward product_routed_update.py:72-75
  route_backward         autograd of product_key_route (gdn2_banks.py:74-114)
  controllers_backward   autograd of _controllers (_parameters.py:189-220, heads.py:11-22)
"""
from __future__ import annotations

import torch

from . import _lib
from .config import near_square_factors

_DT = {torch.float32: _lib.BDM_F32, torch.bfloat16: _lib.BDM_BF16}
SCAN_STATUS_OFFSET = 128  # int32 error bits in the bank-scan workspace header


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DT[dtype]
    except KeyError:
        raise ValueError(f'unsupported dtype {dtype}; bdm_b200 computes in float32 or bfloat16') from None


def _cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError('bdm_b200 ops require CUDA tensors (there is no CPU path)')


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# --------------------------------------------------------------- recurrence status
class _ScanStatus:
    """Sticky error bits of the bank kernels on one device.

    Every bank_scan ORs its launch's status word into ``word`` on the launch stream (no host
    sync), and combine_project ORs into it directly.  Bit 0x1: a bounded wait inside the
    recurrence gave up (a producer / consumer staging wait or a tensor-core completion wait);
    the reads and final states of that launch are then unspecified.  Bit 0x2: a bounded wait
    inside the fused combine + output projection gave up; its outputs are unspecified.  The
    bits stay set until reset_scan_status.
    """

    def __init__(self, device):
        # normal tensors even when the first call runs under inference_mode, so later calls
        # outside it may update them in place
        with torch.inference_mode(False):
            self.word = torch.zeros(1, dtype=torch.int32, device=device)
            self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.event = None
        self.last = 0


_SCAN_STATUS: dict = {}


def _scan_status_of(device) -> _ScanStatus:
    device = torch.device('cuda', torch.cuda.current_device()) if device is None else torch.device(device)
    if device.index is None:
        device = torch.device('cuda', torch.cuda.current_device())
    st = _SCAN_STATUS.get(device.index)
    if st is None:
        st = _SCAN_STATUS[device.index] = _ScanStatus(device)
    return st


def scan_status(device=None, *, wait: bool = False) -> int:
    """Error bits the bank recurrence has recorded on ``device`` (0 = none).

    Without ``wait`` this never blocks: it returns the latest snapshot that has reached the
    host and starts the next asynchronous snapshot, so an error shows up at most one poll
    late.  With ``wait`` it synchronises the current stream and returns the current bits.
    """
    st = _scan_status_of(device)
    if torch.cuda.is_current_stream_capturing():
        return st.last
    stream = torch.cuda.current_stream(st.word.device)
    if wait:
        stream.synchronize()
        st.last = int(st.word.item())
        return st.last
    if st.event is not None and st.event.query():
        st.last = int(st.host.item())
        st.event = None
    if st.event is None:
        st.host.copy_(st.word, non_blocking=True)
        st.event = torch.cuda.Event()
        st.event.record(stream)
    return st.last


def check_scan_status(device=None, *, wait: bool = False) -> None:
    """Raises BDMError if the recurrence recorded an error (see scan_status).  No-op off CUDA."""
    if device is not None and torch.device(device).type != 'cuda':
        return
    bits = scan_status(device, wait=wait)
    if bits:
        raise _lib.BDMError(f'bank kernels: device status {bits:#x} (a bounded wait inside a kernel gave up: 0x1 '
                            f'recurrence, 0x2 combine + output projection; outputs since then are unspecified; '
                            f'reset with ops.reset_scan_status)')


def reset_scan_status(device=None) -> None:
    st = _scan_status_of(device)
    st.word.zero_()
    if st.event is not None:
        st.event.synchronize()
        st.event = None
    st.last = 0


def route(logits: torch.Tensor, *, bank_count: int, selected_banks: int, factors=None):
    """Product-key top-B routing of ``logits[..., J1+J2]`` (last dim may be a strided view).

    Returns (weights [..., count] in the logits dtype, indices [..., count] int64),
    ordered by descending pair score, ties to the lower index.
    """
    _cuda(logits)
    j1, j2 = factors or near_square_factors(bank_count)
    if logits.shape[-1] != j1 + j2:
        raise ValueError('projected route width does not match the bank table')
    if not 1 <= selected_banks <= bank_count:
        raise ValueError('selected bank count is outside the bank table')
    lead = logits.shape[:-1]
    z = logits.reshape(-1, logits.shape[-1])
    if z.stride(-1) != 1:
        z = z.contiguous()
    ntok = z.shape[0]
    sub = min(selected_banks, j1, j2)
    count = min(selected_banks, sub * sub)
    idx = torch.empty((ntok, count), dtype=torch.int64, device=z.device)
    w = torch.empty((ntok, count), dtype=z.dtype, device=z.device)
    ld = z.stride(0) if ntok > 1 else j1 + j2
    _lib.check(_lib.load().bdm_route(_ptr(z), ntok, ld, j1, j2, selected_banks, dtype_code(z.dtype), _ptr(idx),
                                     _ptr(w), _stream(z.device)), 'bdm_route')
    return w.reshape(*lead, count), idx.reshape(*lead, count)


def route_pair(proj: torch.Tensor, first: int, second: int, *, bank_count: int, selected_banks: int, factors=None):
    """Two product-key routers over the rows of ``proj`` [NT, ld] in one launch: the logits at
    columns [first, first+J1+J2) and [second, second+J1+J2).  Returns ((weights, indices) of the
    first block, (weights, indices) of the second), each [NT, count], as two ``route`` calls.
    """
    _cuda(proj)
    j1, j2 = factors or near_square_factors(bank_count)
    if proj.ndim != 2 or proj.stride(1) != 1:
        raise ValueError('proj must be a row-major [tokens, width] matrix')
    if not 1 <= selected_banks <= bank_count:
        raise ValueError('selected bank count is outside the bank table')
    if second < first:
        raise ValueError('the second block must follow the first')
    ntok = proj.shape[0]
    sub = min(selected_banks, j1, j2)
    count = min(selected_banks, sub * sub)
    dev, dt = proj.device, proj.dtype
    idx1 = torch.empty((ntok, count), dtype=torch.int64, device=dev)
    w1 = torch.empty((ntok, count), dtype=dt, device=dev)
    idx2, w2 = torch.empty_like(idx1), torch.empty_like(w1)
    ld = proj.stride(0) if ntok > 1 else proj.shape[1]
    base = proj[:, first:] if ntok else proj
    _lib.check(_lib.load().bdm_route_pair(_ptr(base), ntok, ld, second - first, j1, j2, selected_banks,
                                          dtype_code(dt), _ptr(idx1), _ptr(w1), _ptr(idx2), _ptr(w2),
                                          _stream(dev)), 'bdm_route_pair')
    return (w1, idx1), (w2, idx2)


def dispatch(write_idx: torch.Tensor, read_idx: torch.Tensor, bank_count: int, *, want_inverse=False,
             want_tokens=False, error_word: torch.Tensor | None = None):
    """Stable (batch, bank) counting sort of all routed events.

    write_idx [B,T,KW], read_idx [B,T,KR] int64 -> dict(order [E], cu_seqlens [B*J+1], inverse?, tokens?).
    """
    _cuda(write_idx, read_idx)
    if write_idx.dtype != torch.long or read_idx.dtype != torch.long:
        raise ValueError('bank indices must be int64')
    if write_idx.ndim != 3 or read_idx.ndim != 3 or write_idx.shape[:2] != read_idx.shape[:2]:
        raise ValueError('routes must be [batch, time, banks] with matching batch and time')
    batch, time, kw = write_idx.shape
    kr = read_idx.shape[-1]
    dev = write_idx.device
    wi, ri = write_idx.contiguous(), read_idx.contiguous()
    e = batch * time * (kw + kr)
    order = torch.empty(e, dtype=torch.int64, device=dev)
    cu = torch.empty(batch * bank_count + 1, dtype=torch.int64, device=dev)
    inverse = torch.empty(e, dtype=torch.int64, device=dev) if want_inverse else None
    tokens = torch.empty(e, dtype=torch.int64, device=dev) if want_tokens else None
    lib = _lib.load()
    nbytes = lib.bdm_dispatch_workspace_bytes(batch, time, kw, kr, bank_count)
    if nbytes < 0:
        raise ValueError('invalid dispatch geometry')
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    _lib.check(lib.bdm_dispatch(_ptr(wi), _ptr(ri), batch, time, kw, kr, bank_count, _ptr(order), _ptr(cu),
                                _ptr(inverse), _ptr(tokens), _ptr(error_word), _ptr(ws), nbytes, _stream(dev)),
               'bdm_dispatch')
    out = dict(order=order, cu_seqlens=cu)
    if want_inverse:
        out['inverse'] = inverse
    if want_tokens:
        out['tokens'] = tokens
    return out


def controllers(proj: torch.Tensor, cols: dict, f: torch.Tensor | None, a_log: torch.Tensor, dt_bias: torch.Tensor,
                *, heads: int, bank_size: int, head_value_width: int, qk_norm: str, f_weight=None,
                f1_width: int = 0):
    """Controller epilogue over the fused projection ``proj [NT, ld]`` (column offsets in ``cols``)
    and the f_proj output ``f [NT, H*S]``, or, with ``f=None``, ``f_weight`` (f_proj.1's
    [H*S, f1_width]) applied in the kernel to the f1 columns of ``proj``.

    Returns q, k, v, g, b, w as [NT, H*S] / [NT, V] tensors (g float32).
    """
    _cuda(proj, f, f_weight)
    if proj.ndim != 2 or proj.stride(1) != 1 or (f is not None and (f.ndim != 2 or f.stride(1) != 1)):
        raise ValueError('proj and f must be row-major [tokens, width] matrices')
    nt = proj.shape[0]
    hs, v_width = heads * bank_size, heads * head_value_width
    dev, dt = proj.device, proj.dtype
    wf2 = None
    if f is not None:
        if f.dtype != dt or f.shape != (nt, hs):
            raise ValueError(f'f must be [{nt}, {hs}] in {dt}')
    else:
        if f_weight is None or tuple(f_weight.shape) != (hs, f1_width) or f_weight.dtype != dt:
            raise ValueError(f'f_weight must be [{hs}, {f1_width}] in {dt}')
        wf2 = f_weight.detach().contiguous()
    q = torch.empty((nt, hs), dtype=dt, device=dev)
    k = torch.empty_like(q)
    b = torch.empty_like(q)
    g = torch.empty((nt, hs), dtype=torch.float32, device=dev)
    v = torch.empty((nt, v_width), dtype=dt, device=dev)
    w = torch.empty_like(v)
    al = a_log.detach().float().contiguous()
    dtb = dt_bias.detach().float().contiguous()
    _lib.check(_lib.load().bdm_controllers(
        _ptr(proj), nt, proj.stride(0) if nt > 1 else proj.shape[1], cols['q'], cols['k'], cols['v'], cols['b'],
        cols['w'], _ptr(f), (f.stride(0) if nt > 1 else f.shape[1]) if f is not None else 0, _ptr(wf2),
        cols['f'], int(f1_width), _ptr(al), _ptr(dtb), heads, bank_size,
        head_value_width, 1 if qk_norm == 'nvidia' else 0, dtype_code(dt), _ptr(q), _ptr(k), _ptr(v), _ptr(g),
        _ptr(b), _ptr(w), _stream(dev)), 'bdm_controllers')
    return q, k, v, g, b, w


def product_state(row_factor, col_factor, *, batch: int, bank_count: int, heads: int, bank_size: int,
                  dtype: torch.dtype):
    """Product-key initial memory [batch, J, H, S, dv] in ``dtype``."""
    _cuda(row_factor, col_factor)
    u, z = row_factor.detach().contiguous(), col_factor.detach().contiguous()
    dv = u.shape[-1]
    out = torch.empty((batch, bank_count, heads, bank_size, dv), dtype=dtype, device=u.device)
    _lib.check(_lib.load().bdm_product_state(_ptr(u), _ptr(z), u.shape[0], z.shape[0], dtype_code(u.dtype), batch,
                                             bank_count, heads, bank_size, dv, _ptr(out), dtype_code(dtype),
                                             _stream(u.device)), 'bdm_product_state')
    return out


def bank_scan(q, k, v, g, b, w, write_idx, write_w, read_idx, read_w, order, cu_seqlens, *, batch: int, time: int,
              bank_count: int, heads: int, bank_size: int, head_value_width: int, routed_decay: bool, scale: float,
              row_factor=None, col_factor=None, cache=None, store_final=False, state_interval=0,
              bank_ids=None, total_banks=0, head_offset=0, total_heads=0, check_status=False,
              checkpoints=None, checkpoint_block=0, chunked=False):
    """Per-bank recurrence over dispatched events; returns reads [NT, KR, V] in the activation dtype.

    With ``cache`` ([batch, J, H, S, dv]) the state starts from it and, with
    ``store_final``, ends in it; otherwise it starts from the product-key factors
    (or zero when they are None).  On a bank-sharded rank ``bank_count`` is the
    local bank count and ``bank_ids`` (int32 [bank_count]) maps local banks into
    the full table of ``total_banks`` banks.  ``heads`` may be a head group
    [head_offset, head_offset + heads) of a layer with ``total_heads`` heads.
    ``checkpoints`` (float32, training): receives the states the recurrence backward
    replays from, every ``checkpoint_block`` events (see ``scan_backward``).
    ``chunked``: run the sequences on the tensor-core chunked kernel (``bdm_bank_scan_chunked``;
    BF16, head_value_width a multiple of 128, no checkpoints).
    """
    _cuda(q, k, v, g, b, w, write_idx, read_idx, order, cu_seqlens, cache, bank_ids)
    if bank_ids is not None and (bank_ids.dtype != torch.int32 or bank_ids.numel() != bank_count
                                 or total_banks < bank_count):
        raise ValueError('bank_ids must be int32 [bank_count] into a table of total_banks >= bank_count banks')
    dt = q.dtype
    nt = batch * time
    kw, kr = write_idx.shape[-1], read_idx.shape[-1]
    v_width = heads * head_value_width
    for name, t, shape in (('q', q, (nt, heads * bank_size)), ('k', k, (nt, heads * bank_size)),
                           ('b', b, (nt, heads * bank_size)), ('g', g, (nt, heads * bank_size)),
                           ('v', v, (nt, v_width)), ('w', w, (nt, v_width))):
        if tuple(t.shape) != shape or not t.is_contiguous():
            raise ValueError(f'{name} must be contiguous {shape}, got {tuple(t.shape)}')
    if g.dtype != torch.float32 or any(t.dtype != dt for t in (k, v, b, w, write_w, read_w)):
        raise ValueError('controllers and route weights must share the activation dtype (g is float32)')
    reads = torch.empty((nt, kr, v_width), dtype=dt, device=q.device)
    if cache is not None and not cache.is_contiguous():
        raise ValueError('cache must be contiguous')
    u = z = None
    if cache is None and row_factor is not None:
        u, z = row_factor.detach().contiguous(), col_factor.detach().contiguous()
    # keep contiguous copies alive across the asynchronous call
    wi, ww, ri, rw = (t.contiguous() for t in (write_idx, write_w, read_idx, read_w))
    lib = _lib.load()
    nbytes = lib.bdm_bank_scan_workspace_bytes(batch, bank_count)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    entry = lib.bdm_bank_scan_chunked if chunked else lib.bdm_bank_scan
    _lib.check(entry(
        _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(b), _ptr(w), _ptr(wi), _ptr(ww), _ptr(ri), _ptr(rw), _ptr(order),
        _ptr(cu_seqlens), batch, time, bank_count, heads, bank_size, head_value_width, kw, kr, dtype_code(dt),
        int(routed_decay), float(scale), _ptr(u), _ptr(z), z.shape[0] if z is not None else 0,
        dtype_code(u.dtype) if u is not None else 0, _ptr(bank_ids), int(total_banks) if bank_ids is not None else 0,
        int(head_offset), int(total_heads),
        _ptr(cache), dtype_code(cache.dtype) if cache is not None else 0,
        int(store_final), int(state_interval), _ptr(reads), _ptr(ws), nbytes, _ptr(checkpoints),
        int(checkpoint_block) if checkpoints is not None else 0, _stream(q.device)),
        'bdm_bank_scan_chunked' if chunked else 'bdm_bank_scan')
    # atomic: recurrences on several streams (forward_host's row groups) share the sticky word
    sticky = _scan_status_of(q.device).word
    _lib.check(_lib.load().bdm_status_or(_ptr(sticky), ws.data_ptr() + SCAN_STATUS_OFFSET, _stream(q.device)),
               'bdm_status_or')
    if check_status:  # synchronises: the kernel's error bits (a bounded producer/consumer wait that gave up)
        status = int(ws[SCAN_STATUS_OFFSET:SCAN_STATUS_OFFSET + 4].view(torch.int32).item())
        if status:
            raise _lib.BDMError(f'bdm_bank_scan: device status {status:#x} (a staging wait timed out)')
    return reads


def combine_norm_gate(reads, read_idx, gate, norm_weight, norm_bias, *, eps: float, layer_norm: bool,
                      round_each: bool, save_raw: bool = False):
    """Ascending-bank read combine, LayerNorm/RMS and sigmoid gate -> [NT, V].

    ``reads`` [NT, KR, V] with ``read_idx`` [NT, KR], or an already combined
    [NT, V] with ``read_idx=None``; ``gate`` [NT, >=V] (row stride honoured).
    With ``save_raw`` returns (out, raw): raw is the combined read sum [NT, V]
    in the activation dtype (what the output backward consumes).
    """
    _cuda(reads, gate, norm_weight)
    dt = reads.dtype
    nt, width = reads.shape[0], reads.shape[-1]
    kr = read_idx.shape[-1] if read_idx is not None else 1
    if gate.stride(-1) != 1:
        raise ValueError('gate rows must be contiguous')
    out = torch.empty((nt, width), dtype=dt, device=reads.device)
    nw = norm_weight.detach().to(dt).contiguous()
    nb = norm_bias.detach().to(dt).contiguous() if norm_bias is not None else None
    rd = reads.contiguous()
    ri = read_idx.contiguous() if read_idx is not None else None
    ld_gate = gate.stride(0) if nt > 1 else gate.shape[-1]
    if save_raw:
        raw = torch.empty((nt, width), dtype=dt, device=reads.device)
        _lib.check(_lib.load().bdm_combine_norm_gate_save(
            _ptr(rd), _ptr(ri), nt, kr, width, _ptr(gate), ld_gate, _ptr(nw), _ptr(nb), float(eps),
            1 if layer_norm else 0, int(round_each), dtype_code(dt), _ptr(out), _ptr(raw), _stream(reads.device)),
            'bdm_combine_norm_gate_save')
        return out, raw
    _lib.check(_lib.load().bdm_combine_norm_gate(
        _ptr(rd), _ptr(ri), nt, kr, width,
        _ptr(gate), ld_gate, _ptr(nw), _ptr(nb), float(eps),
        1 if layer_norm else 0, int(round_each), dtype_code(dt), _ptr(out), _stream(reads.device)),
        'bdm_combine_norm_gate')
    return out


def combine_project_supported(width: int, out_dim: int, kr: int, dtype) -> bool:
    """Whether ``combine_project`` takes this geometry (BF16, 512 <= V <= 1024, V % 256 == 0,
    D % 128 == 0 and <= 1024, 1 <= KR <= 16)."""
    if dtype != torch.bfloat16:
        return False
    return bool(_lib.load().bdm_combine_project_supported(int(width), int(out_dim), int(kr), dtype_code(dtype)))


def combine_project(reads, read_idx, gate, norm_weight, norm_bias, o_weight, o_bias, *, eps: float,
                    layer_norm: bool, round_each: bool):
    """Read combine, norm, gate and the output projection in one kernel -> [NT, D].

    ``reads`` [NT, KR, V] with ``read_idx`` [NT, KR]; ``gate`` [NT, >=V] (row stride honoured);
    ``o_weight`` [D, V] and ``o_bias`` [D] (or None) of o_proj.  The o_proj input equals
    ``combine_norm_gate``'s output bit for bit; the product accumulates in FP32 on the tensor
    cores.  Only shapes ``combine_project_supported`` accepts.
    """
    _cuda(reads, gate, norm_weight, o_weight)
    dt = reads.dtype
    nt, width = reads.shape[0], reads.shape[-1]
    kr = read_idx.shape[-1]
    out_dim = o_weight.shape[0]
    if o_weight.shape != (out_dim, width):
        raise ValueError(f'o_weight must be [out_dim, {width}], got {tuple(o_weight.shape)}')
    if gate.stride(-1) != 1:
        raise ValueError('gate rows must be contiguous')
    out = torch.empty((nt, out_dim), dtype=dt, device=reads.device)
    nw = norm_weight.detach().to(dt).contiguous()
    nb = norm_bias.detach().to(dt).contiguous() if norm_bias is not None else None
    w = o_weight.detach().to(dt).contiguous()
    bo = o_bias.detach().to(dt).contiguous() if o_bias is not None else None
    rd = reads.contiguous()
    ri = read_idx.contiguous()
    ld_gate = gate.stride(0) if nt > 1 else gate.shape[-1]
    status = _scan_status_of(reads.device).word
    _lib.check(_lib.load().bdm_combine_project(
        _ptr(rd), _ptr(ri), nt, kr, width, _ptr(gate), ld_gate, _ptr(nw), _ptr(nb), float(eps),
        1 if layer_norm else 0, int(round_each), _ptr(w), _ptr(bo), out_dim, dtype_code(dt), _ptr(out), out_dim,
        _ptr(status), _stream(reads.device)), 'bdm_combine_project')
    return out


def decode_step(q, k, v, g, b, w, write_idx, write_w, read_idx, read_w, state, *, bank_count: int, heads: int,
                bank_size: int, head_value_width: int, routed_decay: bool, scale: float, gate=None,
                norm_weight=None, norm_bias=None, eps: float = 1e-5, layer_norm: bool = True):
    """One decode token per batch row; ``state`` [B, J, H, S, dv] updated in place.

    Returns raw [B, V] (the ascending-bank read sum), or, with ``gate`` ([B, >=V], row stride
    honoured), the normalised and gated [B, V] of the output interface, computed in the same kernel.
    """
    _cuda(q, state, gate)
    if not state.is_contiguous():
        raise ValueError('state must be contiguous')
    batch = q.shape[0]
    kw, kr = write_idx.shape[-1], read_idx.shape[-1]
    v_width = heads * head_value_width
    raw = out = nw = nb = None
    if gate is None:
        raw = torch.empty((batch, v_width), dtype=q.dtype, device=q.device)
    else:
        if gate.stride(-1) != 1:
            raise ValueError('gate rows must be contiguous')
        out = torch.empty((batch, v_width), dtype=q.dtype, device=q.device)
        nw = norm_weight.detach().to(q.dtype).contiguous()
        nb = norm_bias.detach().to(q.dtype).contiguous() if norm_bias is not None else None
    wi, ww, ri, rw = (t.contiguous() for t in (write_idx, write_w, read_idx, read_w))
    q, k, v, g, b, w = (t.contiguous() for t in (q, k, v, g, b, w))
    ld_gate = (gate.stride(0) if batch > 1 else gate.shape[-1]) if gate is not None else 0
    _lib.check(_lib.load().bdm_decode_step(
        _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(b), _ptr(w), _ptr(wi), _ptr(ww), _ptr(ri), _ptr(rw), batch,
        bank_count, heads, bank_size, head_value_width, kw, kr, dtype_code(q.dtype), int(routed_decay), float(scale),
        _ptr(state), dtype_code(state.dtype), _ptr(raw), _ptr(gate), ld_gate, _ptr(nw), _ptr(nb), float(eps),
        1 if layer_norm else 0, _ptr(out), _stream(q.device)), 'bdm_decode_step')
    return raw if gate is None else out


def decode_token_step(proj, cols, f_weight, a_log, dt_bias, state, *, bank_count: int, selected_banks: int,
                      factors, heads: int, bank_size: int, head_value_width: int, qk_norm: str, routed_decay: bool,
                      scale: float, norm_weight, norm_bias=None, eps: float = 1e-5, layer_norm: bool = True):
    """A whole decode step from the fused projection ``proj`` [B, ld] (one token per row): controllers,
    both routers and the bank step with combine, norm and gate in one launch; ``state`` updated in place.
    Returns the normalised, gated [B, H*dv] (o_proj's input)."""
    _cuda(proj, state)
    if proj.stride(-1) != 1 or not state.is_contiguous():
        raise ValueError('proj rows and the state must be contiguous')
    batch = proj.shape[0]
    ld = proj.stride(0) if batch > 1 else proj.shape[-1]
    j1, j2 = factors
    out = torch.empty((batch, heads * head_value_width), dtype=proj.dtype, device=proj.device)
    wf2 = f_weight.detach().to(proj.dtype).contiguous()
    nw = norm_weight.detach().to(proj.dtype).contiguous()
    nb = norm_bias.detach().to(proj.dtype).contiguous() if norm_bias is not None else None
    al = a_log.detach().float().contiguous()
    dt = dt_bias.detach().float().contiguous()
    _lib.check(_lib.load().bdm_decode_token_step(
        _ptr(proj), batch, ld, cols['q'], cols['k'], cols['v'], cols['f'], cols['b'], cols['w'], cols['read'],
        cols['write'], cols['gate'], _ptr(wf2), head_value_width, _ptr(al), _ptr(dt),
        1 if qk_norm == 'nvidia' else 0, j1, j2, selected_banks, bank_count, heads, bank_size, head_value_width,
        dtype_code(proj.dtype), int(routed_decay), float(scale), _ptr(state), dtype_code(state.dtype), _ptr(nw),
        _ptr(nb), float(eps), 1 if layer_norm else 0, _ptr(out), _stream(proj.device)), 'bdm_decode_token_step')
    return out


# ------------------------------------------------------------ bank sharding

def bank_histogram(write_idx: torch.Tensor, read_idx: torch.Tensor, bank_count: int,
                   counts: torch.Tensor | None = None) -> torch.Tensor:
    """Events per bank (int32 [bank_count]) of routes [..., KW] / [..., KR]; adds into ``counts`` if given."""
    _cuda(write_idx, read_idx)
    wi = write_idx.reshape(-1, write_idx.shape[-1]).contiguous()
    ri = read_idx.reshape(-1, read_idx.shape[-1]).contiguous()
    if wi.dtype != torch.long or ri.dtype != torch.long or wi.shape[0] != ri.shape[0]:
        raise ValueError('routes must be int64 with matching token counts')
    if counts is None:
        counts = torch.zeros(bank_count, dtype=torch.int32, device=wi.device)
    elif counts.dtype != torch.int32 or counts.numel() != bank_count or not counts.is_contiguous():
        raise ValueError('counts must be contiguous int32 [bank_count]')
    _lib.check(_lib.load().bdm_bank_histogram(_ptr(wi), _ptr(ri), wi.shape[0], wi.shape[1], ri.shape[1], bank_count,
                                              _ptr(counts), _stream(wi.device)), 'bdm_bank_histogram')
    return counts


OWNERSHIP_MODES = {'contiguous': 0, 'balanced': 1}
# Limits of the balanced partition (one CTA sorts the whole bank table in shared memory, one
# lane per rank); larger tables or worlds use contiguous ranges.
MAX_BALANCED_BANKS, MAX_BALANCED_WORLD = 16384, 32


def bank_owners(counts: torch.Tensor | None, bank_count: int, world: int, *, mode: str = 'balanced',
                device=None):
    """Partition of the bank table over ``world`` ranks -> (owner [J], slot [J], members [world, J/world]) int32."""
    if mode not in OWNERSHIP_MODES:
        raise ValueError(f'ownership mode must be one of {sorted(OWNERSHIP_MODES)}')
    if counts is not None:
        _cuda(counts)
        if counts.dtype != torch.int32 or counts.numel() != bank_count or not counts.is_contiguous():
            raise ValueError('counts must be contiguous int32 [bank_count]')
        device = counts.device
    elif mode == 'balanced':
        raise ValueError('the balanced partition needs the per-bank event counts')
    if world <= 0 or bank_count % world:
        raise NotImplementedError('the bank count must divide evenly over the ranks')
    owner = torch.empty(bank_count, dtype=torch.int32, device=device)
    slot = torch.empty_like(owner)
    members = torch.empty((world, bank_count // world), dtype=torch.int32, device=device)
    _lib.check(_lib.load().bdm_bank_owners(_ptr(counts), bank_count, world, OWNERSHIP_MODES[mode], _ptr(owner),
                                           _ptr(slot), _ptr(members), _stream(owner.device)), 'bdm_bank_owners')
    return owner, slot, members


def dispatch_owned(write_idx: torch.Tensor, read_idx: torch.Tensor, bank_count: int, owner: torch.Tensor,
                   slot: torch.Tensor, rank: int, local_banks: int):
    """``dispatch`` of the events whose bank ``rank`` owns, as (batch, local bank) sequences.

    Returns dict(order [E] (owned events first), cu_seqlens [B*local_banks + 1]).
    """
    _cuda(write_idx, read_idx, owner, slot)
    if write_idx.dtype != torch.long or read_idx.dtype != torch.long:
        raise ValueError('bank indices must be int64')
    if write_idx.ndim != 3 or read_idx.ndim != 3 or write_idx.shape[:2] != read_idx.shape[:2]:
        raise ValueError('routes must be [batch, time, banks] with matching batch and time')
    for name, t in (('owner', owner), ('slot', slot)):
        if t.dtype != torch.int32 or t.numel() != bank_count or not t.is_contiguous():
            raise ValueError(f'{name} must be contiguous int32 [bank_count]')
    batch, time, kw = write_idx.shape
    kr = read_idx.shape[-1]
    dev = write_idx.device
    wi, ri = write_idx.contiguous(), read_idx.contiguous()
    order = torch.empty(batch * time * (kw + kr), dtype=torch.int64, device=dev)
    cu = torch.empty(batch * local_banks + 1, dtype=torch.int64, device=dev)
    lib = _lib.load()
    nbytes = lib.bdm_dispatch_owned_workspace_bytes(batch, time, kw, kr, local_banks)
    if nbytes < 0:
        raise ValueError('invalid dispatch geometry')
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    _lib.check(lib.bdm_dispatch_owned(_ptr(wi), _ptr(ri), batch, time, kw, kr, bank_count, _ptr(owner), _ptr(slot),
                                      int(rank), local_banks, _ptr(order), _ptr(cu), None, None, None, _ptr(ws),
                                      nbytes, _stream(dev)), 'bdm_dispatch_owned')
    return dict(order=order, cu_seqlens=cu)


def combine_partial(reads: torch.Tensor, read_idx: torch.Tensor, owner: torch.Tensor, rank: int,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """FP32 [NT, V]: per token, the ascending-bank sum of the read rows of banks ``rank`` owns."""
    _cuda(reads, read_idx, owner)
    nt, kr, width = reads.shape
    ri = read_idx.reshape(nt, kr).contiguous()
    if owner.dtype != torch.int32 or not owner.is_contiguous():
        raise ValueError('owner must be contiguous int32 [bank_count]')
    if out is None:
        out = torch.empty((nt, width), dtype=torch.float32, device=reads.device)
    elif out.dtype != torch.float32 or tuple(out.shape) != (nt, width) or not out.is_contiguous():
        raise ValueError(f'out must be contiguous float32 [{nt}, {width}]')
    rd = reads.contiguous()
    _lib.check(_lib.load().bdm_combine_partial(_ptr(rd), _ptr(ri), nt, kr, width, _ptr(owner), owner.numel(),
                                               int(rank), dtype_code(reads.dtype), _ptr(out), _stream(reads.device)),
               'bdm_combine_partial')
    return out


def norm_gate_f32(combined: torch.Tensor, gate, norm_weight, norm_bias, *, eps: float, layer_norm: bool,
                  dtype: torch.dtype) -> torch.Tensor:
    """``combine_norm_gate`` over an FP32 combined read sum [NT, V], rounded once to ``dtype`` first."""
    _cuda(combined, gate, norm_weight)
    if combined.dtype != torch.float32 or combined.ndim != 2 or not combined.is_contiguous():
        raise ValueError('combined must be contiguous float32 [tokens, width]')
    if gate.stride(-1) != 1:
        raise ValueError('gate rows must be contiguous')
    nt, width = combined.shape
    out = torch.empty((nt, width), dtype=dtype, device=combined.device)
    nw = norm_weight.detach().to(dtype).contiguous()
    nb = norm_bias.detach().to(dtype).contiguous() if norm_bias is not None else None
    _lib.check(_lib.load().bdm_norm_gate_f32(
        _ptr(combined), nt, width, _ptr(gate), gate.stride(0) if nt > 1 else gate.shape[-1], _ptr(nw), _ptr(nb),
        float(eps), 1 if layer_norm else 0, dtype_code(dtype), _ptr(out), _stream(combined.device)),
        'bdm_norm_gate_f32')
    return out


# -------------------------------------------------------- training backward

def norm_gate_backward(d_out, raw, gate, norm_weight, norm_bias, *, eps: float, layer_norm: bool,
                       d_gate: torch.Tensor):
    """Backward of ``combine_norm_gate``'s norm and gate over the saved combined sum ``raw`` [NT, V].

    Writes the gate pre-activation gradient into ``d_gate`` ([NT, >=V] view, row stride
    honoured) and returns (d_raw [NT, V] in the activation dtype, d_norm_weight,
    d_norm_bias or None) with the parameter gradients in FP32.
    """
    _cuda(d_out, raw, gate, norm_weight, d_gate)
    nt, width = raw.shape
    dt = raw.dtype
    if gate.stride(-1) != 1 or d_gate.stride(-1) != 1:
        raise ValueError('gate rows must be contiguous')
    dout = d_out.reshape(nt, width).to(dt).contiguous()
    nw = norm_weight.detach().to(dt).contiguous()
    nb = norm_bias.detach().to(dt).contiguous() if (norm_bias is not None and layer_norm) else None
    dev = raw.device
    d_raw = torch.empty((nt, width), dtype=dt, device=dev)
    lib = _lib.load()
    part = torch.empty(max(lib.bdm_norm_gate_backward_partial_floats(nt, width), 1), dtype=torch.float32, device=dev)
    dw = torch.empty(width, dtype=torch.float32, device=dev)
    db = torch.empty(width, dtype=torch.float32, device=dev) if nb is not None else None
    ld_gate = gate.stride(0) if nt > 1 else gate.shape[-1]
    ldd = d_gate.stride(0) if nt > 1 else d_gate.shape[-1]
    lib_check = _lib.check
    lib_check(lib.bdm_norm_gate_backward(_ptr(dout), _ptr(raw), nt, width, _ptr(gate), ld_gate, _ptr(nw), _ptr(nb),
                                         float(eps), 1 if layer_norm else 0, dtype_code(dt), _ptr(d_raw),
                                         _ptr(d_gate), ldd, _ptr(part), _ptr(dw), _ptr(db), _stream(dev)),
              'bdm_norm_gate_backward')
    return d_raw, dw, db


def scan_backward(q, k, v, g, b, w, write_w, read_w, order, cu_seqlens, d_read, *, batch: int, time: int,
                  bank_count: int, heads: int, bank_size: int, head_value_width: int, kw: int, kr: int,
                  routed_decay: bool, scale: float, row_factor=None, col_factor=None, state_interval=0,
                  checkpoints=None):
    """Recurrence backward over the dispatched events of a factor-initialised training forward.

    ``d_read`` [NT, H*dv] is the gradient of the combined read sum.  ``checkpoints``: the buffer
    the forward filled (``checkpoint_buffer``), or None to replay them here.  Returns
    (event_grads [tiles, E, H, 3S], d_write_value [NT*KW, H*dv], d_initial [B*J, H, S, dv]), FP32.
    """
    _cuda(q, k, v, g, b, w, write_w, read_w, order, cu_seqlens, d_read)
    dt, dev = q.dtype, q.device
    nt = batch * time
    e = nt * (kw + kr)
    v_width = heads * head_value_width
    lib = _lib.load()
    tiles = lib.bdm_scan_backward_tiles(bank_size, head_value_width)
    ck_bytes = lib.bdm_scan_backward_checkpoint_bytes(batch, time, kw, kr, bank_count, heads, bank_size,
                                                      head_value_width)
    if ck_bytes < 0:
        raise NotImplementedError('scan backward supports bank_size 4, 8 or 16')
    ready = checkpoints is not None
    if ready:
        if checkpoints.dtype != torch.float32 or checkpoints.numel() * 4 < ck_bytes:
            raise ValueError('checkpoints must be the float32 buffer of checkpoint_buffer()')
        ck = checkpoints
    else:
        ck = torch.empty(max(ck_bytes // 4, 1), dtype=torch.float32, device=dev)
    evg = torch.empty((tiles, e, heads, 3 * bank_size), dtype=torch.float32, device=dev)
    du = torch.empty((nt * kw, v_width), dtype=torch.float32, device=dev)
    dinit = torch.empty((batch * bank_count, heads, bank_size, head_value_width), dtype=torch.float32, device=dev)
    u = z = None
    if row_factor is not None:
        u, z = row_factor.detach().contiguous(), col_factor.detach().contiguous()
    dr = d_read.reshape(nt, v_width).to(dt).contiguous()
    ww, rw = write_w.contiguous(), read_w.contiguous()
    _lib.check(lib.bdm_scan_backward(
        _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(b), _ptr(w), _ptr(ww), _ptr(rw), _ptr(order), _ptr(cu_seqlens),
        batch, time, bank_count, heads, bank_size, head_value_width, kw, kr, dtype_code(dt), int(routed_decay),
        float(scale), _ptr(u), _ptr(z), z.shape[0] if z is not None else 0,
        dtype_code(u.dtype) if u is not None else 0, int(state_interval), _ptr(dr), _ptr(evg), _ptr(du),
        _ptr(dinit), _ptr(ck), ck_bytes, int(ready), _stream(dev)), 'bdm_scan_backward')
    return evg, du, dinit


def checkpoint_buffer(*, batch: int, time: int, kw: int, kr: int, bank_count: int, heads: int, bank_size: int,
                      head_value_width: int, device):
    """(float32 buffer, block) for a training forward's ``bank_scan(checkpoints=, checkpoint_block=)``."""
    lib = _lib.load()
    nbytes = lib.bdm_scan_backward_checkpoint_bytes(batch, time, kw, kr, bank_count, heads, bank_size,
                                                    head_value_width)
    block = lib.bdm_scan_backward_block_events(bank_size, head_value_width)
    if nbytes < 0 or block <= 0:
        raise NotImplementedError('the training backward supports bank_size 4, 8 or 16')
    return torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=device), block


def event_vjp(q, k, v, g, b, w, write_w, read_w, event_grads, d_write_value, *, heads: int, bank_size: int,
              head_value_width: int, routed_decay: bool, scale: float):
    """Token gradients from the event gradients: (dq, dk, dv, dg, db, dw, d_write_w, d_read_w), the route
    weight gradients per head ([NT, H, KW] / [NT, H, KR]; ``route_backward`` sums them)."""
    _cuda(q, event_grads, d_write_value)
    dt, dev = q.dtype, q.device
    nt = q.shape[0]
    kw, kr = write_w.shape[-1], read_w.shape[-1]
    ww, rw = write_w.reshape(nt, kw).contiguous(), read_w.reshape(nt, kr).contiguous()
    dq, dk, db = (torch.empty_like(q) for _ in range(3))
    dg = torch.empty_like(g)
    dv, dw = torch.empty_like(v), torch.empty_like(w)
    dww = torch.empty((nt, heads, kw), dtype=dt, device=dev)
    drw = torch.empty((nt, heads, kr), dtype=dt, device=dev)
    _lib.check(_lib.load().bdm_event_vjp(
        _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(b), _ptr(w), _ptr(ww), _ptr(rw), _ptr(event_grads),
        _ptr(d_write_value), nt, heads, bank_size, head_value_width, kw, kr, dtype_code(dt), int(routed_decay),
        float(scale), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dg), _ptr(db), _ptr(dw), _ptr(dww), _ptr(drw),
        _stream(dev)), 'bdm_event_vjp')
    return dq, dk, dv, dg, db, dw, dww, drw


def product_state_backward(d_initial, *, batch: int, rows_p: int, cols_q: int, factor_dtype: torch.dtype):
    """Factor gradients (FP32 holding factor-dtype values) from d_initial [B*J, H, S, dv]."""
    _cuda(d_initial)
    dv = d_initial.shape[-1]
    dev = d_initial.device
    rows = torch.empty((rows_p * cols_q, dv), dtype=torch.float32, device=dev)
    du = torch.empty((rows_p, dv), dtype=torch.float32, device=dev)
    dz = torch.empty((cols_q, dv), dtype=torch.float32, device=dev)
    _lib.check(_lib.load().bdm_product_state_backward(_ptr(d_initial.contiguous()), batch, rows_p, cols_q, dv,
                                                      dtype_code(factor_dtype), _ptr(rows), _ptr(du), _ptr(dz),
                                                      _stream(dev)), 'bdm_product_state_backward')
    return du, dz


def route_backward(proj, first: int, second: int, idx_first, dw_first, idx_second, dw_second, d_proj, *,
                   bank_count: int, factors=None):
    """Both routers' logit gradients into ``d_proj`` (blocks at columns ``first`` and ``second``).

    ``dw_*``: weight gradients [NT, count] or per head [NT, H, count] (summed over heads here).
    """
    _cuda(proj, idx_first, dw_first, idx_second, dw_second, d_proj)
    j1, j2 = factors or near_square_factors(bank_count)
    nt = proj.shape[0]
    count = idx_first.shape[-1]
    heads = dw_first.shape[1] if dw_first.ndim == 3 else 1
    i1, i2 = idx_first.reshape(nt, count).contiguous(), idx_second.reshape(nt, count).contiguous()
    w1, w2 = (t.reshape(nt, heads, count).to(proj.dtype).contiguous() for t in (dw_first, dw_second))
    ld = proj.stride(0) if nt > 1 else proj.shape[1]
    ldd = d_proj.stride(0) if nt > 1 else d_proj.shape[1]
    _lib.check(_lib.load().bdm_route_backward(_ptr(proj), nt, ld, first, second, j1, j2, count, heads, _ptr(i1),
                                              _ptr(w1),
                                              _ptr(i2), _ptr(w2), dtype_code(proj.dtype), _ptr(d_proj), ldd,
                                              _stream(proj.device)), 'bdm_route_backward')


def controllers_backward(proj, cols: dict, f, a_log, dt_bias, g, b, w, dq, dk, dv, dg, db, dw, d_proj, *,
                         heads: int, bank_size: int, head_value_width: int, qk_norm: str):
    """Controller-epilogue backward: writes the q, k, v, b, w blocks of ``d_proj``; returns
    (df [NT, H*S] in the activation dtype, d_a_log [H] FP32, d_dt_bias [H*S] FP32)."""
    _cuda(proj, f, d_proj)
    nt = proj.shape[0]
    dt, dev = proj.dtype, proj.device
    hs = heads * bank_size
    df = torch.empty((nt, hs), dtype=dt, device=dev)
    lib = _lib.load()
    part = torch.empty(max(lib.bdm_controllers_backward_partial_floats(nt, heads, bank_size), 1),
                       dtype=torch.float32, device=dev)
    d_dt = torch.empty(hs, dtype=torch.float32, device=dev)
    d_a = torch.empty(heads, dtype=torch.float32, device=dev)
    al = a_log.detach().float().contiguous()
    dtb = dt_bias.detach().float().contiguous()
    ld = proj.stride(0) if nt > 1 else proj.shape[1]
    ldd = d_proj.stride(0) if nt > 1 else d_proj.shape[1]
    ldf = f.stride(0) if nt > 1 else f.shape[1]
    _lib.check(lib.bdm_controllers_backward(
        _ptr(proj), nt, ld, cols['q'], cols['k'], cols['v'], cols['b'], cols['w'], _ptr(f), ldf, _ptr(al), _ptr(dtb),
        _ptr(g), _ptr(b), _ptr(w), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dg), _ptr(db), _ptr(dw), heads, bank_size,
        head_value_width, 1 if qk_norm == 'nvidia' else 0, dtype_code(dt), _ptr(d_proj), ldd, _ptr(df), _ptr(part),
        _ptr(d_dt), _ptr(d_a), _stream(dev)), 'bdm_controllers_backward')
    return df, d_a, d_dt
