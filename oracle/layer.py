"""NumPy restatement of the reference BDM layer around the C oracle -- TEST INFRASTRUCTURE ONLY.

``OracleLayer(config, params, bf16)`` mirrors ``bdm.model.BankedDeltaMemory``
(implementation/bdm/model.py:15-140) with ``backend='reference'``:

* controllers            _parameters.py:189-220, heads.py:11-22
* shared-residual router routing.py:23-35
* product-key routing    gdn2_banks.py:74-114          (oracle_route)
* initial bank memory    _parameters.py:40-67           (U[row//Q] + Z[row%Q])
* packing + recurrence   gdn2_banks.py:22-43,117-262    (oracle_recurrence)
* read combine           gdn2_banks.py:265-283          (oracle_combine)
* output interface       _parameters.py:222-232
* stateful prefill/step  inference.py:110-194           (oracle_decode_step)

BF16 runs keep every tensor the reference stores in BF16 rounded to BF16
(``bf16_round``) at the same op boundaries; matrix products accumulate in
FP32 and round once, as torch's CPU BF16 matmul does.  Accumulation order
inside a product can differ from torch's, so layer outputs agree to a few BF16
ulps, not bit-for-bit; the integer work (routing, dispatch) is exact given the
same router logits.
"""
from __future__ import annotations

import math

import numpy as np

from .core import bf16_round, oracle_combine, oracle_decode_step, oracle_recurrence, oracle_route


def near_square_factors(value: int) -> tuple[int, int]:
    """config.py:7-13: the largest divisor <= sqrt(value) and its cofactor."""
    if value <= 0:
        raise ValueError('value must be positive')
    for first in range(math.isqrt(value), 0, -1):
        if value % first == 0:
            return first, value // first
    raise AssertionError('unreachable')


def state_interval(bank_size: int) -> int:
    """model.py:131: BF16 state storage cadence min(16, max(4, 128 // next_pow2(S)))."""
    return min(16, max(4, 128 // (1 << (bank_size - 1).bit_length())))


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _softplus(x):
    # torch.nn.functional.softplus(beta=1, threshold=20)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


class OracleLayer:
    """CPU restatement of one BDM layer.

    ``config``: dict with dim, bank_count, bank_size, selected_banks, value_width,
    num_heads, norm_eps, routed_decay, qk_normalization, output_normalization,
    output_bias, training_state_dtype.  ``params``: state_dict names -> arrays
    (parameter dtype values held in float32).  ``bf16``: parameters and
    activations are BF16.
    """

    def __init__(self, config: dict, params: dict, bf16: bool):
        self.c = dict(config)
        self.p = {k: np.asarray(v, dtype=np.float32) for k, v in params.items()}
        self.bf16 = bool(bf16)
        self.J = self.c['bank_count']
        self.S = self.c['bank_size']
        self.H = self.c['num_heads']
        self.V = self.c['value_width']
        self.dv = self.V // self.H
        self.B = self.c['selected_banks']
        self.j1, self.j2 = near_square_factors(self.J)

    # ------------------------------------------------------------------ utils
    def r(self, x):
        """Round to the activation / parameter dtype."""
        return bf16_round(x) if self.bf16 else np.asarray(x, np.float32)

    def linear(self, x, weight, bias=None):
        y = np.matmul(x.astype(np.float32), weight.T.astype(np.float32))
        if bias is not None:
            y = y + bias
        return self.r(y)

    def _normalize(self, x):
        x = x.astype(np.float32)
        if self.c['qk_normalization'] == 'nvidia':
            y = x * (1.0 / np.sqrt(np.square(x).sum(-1, keepdims=True) + np.float32(1e-6)))
        else:
            n = np.sqrt(np.square(x).sum(-1, keepdims=True))
            y = x / np.maximum(n, np.float32(1e-12))
        return self.r(y)

    # ------------------------------------------------------------ controllers
    def controllers(self, x):
        """q,k,b,g [B,T,H,S] and v,w [B,T,H,dv] (_parameters.py:189-212, heads.py:11-22)."""
        p, H, S, dv = self.p, self.H, self.S, self.dv
        lead = x.shape[:-1]
        q = self._normalize(self.r(_silu(self.linear(x, p['q_proj.weight']))).reshape(*lead, H, S))
        k = self._normalize(self.r(_silu(self.linear(x, p['k_proj.weight']))).reshape(*lead, H, S))
        v = self.r(_silu(self.linear(x, p['v_proj.weight']))).reshape(*lead, H, dv)
        f = self.linear(self.linear(x, p['f_proj.0.weight']), p['f_proj.1.weight'])
        a = np.exp(p['A_log'].astype(np.float32))
        g = (-np.repeat(a, S) * _softplus(f + p['dt_bias'])).astype(np.float32).reshape(*lead, H, S)
        b = self.r(_sigmoid(self.linear(x, p['b_proj.weight']))).reshape(*lead, H, S)
        w = self.r(_sigmoid(self.linear(x, p['w_proj.weight']))).reshape(*lead, H, dv)
        return q, k, v, g, b, w

    def route_logits(self, x):
        """SharedResidualRouter.read / .write (routing.py:23-35)."""
        p = self.p
        base_w, base_b = p['shared_router.base.weight'], p['shared_router.base.bias']
        rw_ = self.r(base_w + p['shared_router.read_residual.weight'])
        rb_ = self.r(base_b + p['shared_router.read_residual.bias'])
        ww_ = self.r(base_w + p['shared_router.write_residual.weight'])
        wb_ = self.r(base_b + p['shared_router.write_residual.bias'])
        return self.linear(x, rw_, rb_), self.linear(x, ww_, wb_)

    def route(self, logits):
        return oracle_route(logits, bank_count=self.J, selected_banks=self.B, bf16=self.bf16)

    def initial_state(self):
        """_parameters.py:40-61: [J, H, S, dv] = U[row // Q] + Z[row % Q] in parameter dtype."""
        u = self.p['initial_row_factor']
        z = self.p['initial_column_factor']
        m = self.r(u[:, None, :] + z[None, :, :])
        return m.reshape(self.J, self.H, self.S, self.dv)

    # ----------------------------------------------------------------- output
    def project(self, x, raw):
        """_parameters.py:222-232: LayerNorm or RMS, sigmoid gate, o_proj."""
        p = self.p
        raw = raw.astype(np.float32)
        if self.c['output_normalization'] == 'layer':
            mean = raw.astype(np.float64).mean(-1, keepdims=True)
            var = raw.astype(np.float64).var(-1, keepdims=True)
            n = (raw - mean) / np.sqrt(var + self.c['norm_eps'])
            n = self.r(n * p['output_norm_weight'] + p['output_norm_bias'])
        else:
            var = np.square(raw.astype(np.float32)).mean(-1, keepdims=True)
            scale = self.r(1.0 / np.sqrt(var + np.float32(self.c['norm_eps'])))
            n = self.r(raw * scale)
            n = self.r(n * p['output_norm_weight'])
        gate = self.r(_sigmoid(self.linear(x, p['output_gate.weight'], p['output_gate.bias'])))
        return self.linear(self.r(n * gate), p['o_proj.weight'], p.get('o_proj.bias'))

    # ---------------------------------------------------------------- forward
    def bank_reads(self, controls, routes, init, *, interval, want_state=False):
        q, k, v, g, b, w = controls
        (ww, wi), (rw, ri) = routes
        return oracle_recurrence(q, k, v, g, b, w, wi, ww, ri, rw, init, bank_count=self.J, bf16=self.bf16,
                                 routed_decay=self.c['routed_decay'], interval=interval, scale=self.S ** -0.5,
                                 want_state=want_state)

    def forward(self, x, *, controls=None, routes=None):
        """model.py:88-140 with backend='reference' (training forward)."""
        x = self.r(x)
        controls = controls or self.controllers(x)
        if routes is None:
            rl, wl = self.route_logits(x)
            routes = (self.route(wl), self.route(rl))
        interval = state_interval(self.S) if self.c['training_state_dtype'] == 'bfloat16' else 0
        init = self.initial_state()[None]
        reads, _ = self.bank_reads(controls, routes, init, interval=interval)
        raw = oracle_combine(reads, routes[1][1], bf16=self.bf16)
        return self.project(x, raw)

    def prefill(self, x, state=None, *, cache_bf16=True, controls=None, routes=None):
        """inference.py:110-158 semantics: no state rounding until handoff to the cache dtype.

        state: [B, J, H, S, dv] cache values or None (product-key initial memory).
        Returns (out, state [B,J,H,S,dv] float32 holding cache-dtype values).
        """
        x = self.r(x)
        controls = controls or self.controllers(x)
        if routes is None:
            rl, wl = self.route_logits(x)
            routes = (self.route(wl), self.route(rl))
        init = self.initial_state()[None] if state is None else np.asarray(state, np.float32)
        reads, final = self.bank_reads(controls, routes, init, interval=0, want_state=True)
        final = bf16_round(final) if cache_bf16 else final
        raw = oracle_combine(reads, routes[1][1], bf16=self.bf16, round_each=True)
        return self.project(x, raw), final

    def step(self, x, state, *, cache_bf16=True, controls=None, routes=None):
        """inference.py:161-194: one token per batch row; ``state`` [B,J,H,S,dv] updated in place."""
        x = self.r(x)
        if x.shape[1] != 1:
            raise ValueError('step requires one token')
        controls = controls or self.controllers(x)
        if routes is None:
            rl, wl = self.route_logits(x)
            routes = (self.route(wl), self.route(rl))
        q, k, v, g, b, w = (c[:, 0] for c in controls)
        (ww, wi), (rw, ri) = routes
        raw = oracle_decode_step(q, k, v, g, b, w, wi[:, 0], ww[:, 0], ri[:, 0], rw[:, 0], state, bf16=self.bf16,
                                 cache_bf16=cache_bf16, routed_decay=self.c['routed_decay'], scale=self.S ** -0.5)
        return self.project(x, raw[:, None, :]), state
