"""CPU oracle for the BDM layer hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm import this package, and only as the checker or as the timed CPU
baseline.  The product (``bdm_b200``) never imports it and has no CPU fallback.

``oracle.core`` binds the C restatement (``bdm_oracle.c``); ``oracle.layer``
restates the reference module's controllers, routing, recurrence and output
interface around it with NumPy, emulating BF16 storage where the reference
stores BF16; ``oracle.shard`` restates the bank-sharded forward's partition,
owned dispatch and partial combine.
"""
from .core import (bf16_round, load, oracle_combine, oracle_decode_step, oracle_dispatch, oracle_recurrence,
                   oracle_route, set_threads)
from .layer import OracleLayer, near_square_factors, state_interval
from .shard import oracle_bank_histogram, oracle_bank_owners, oracle_combine_partial, oracle_dispatch_owned

__all__ = ['bf16_round', 'load', 'oracle_combine', 'oracle_decode_step', 'oracle_dispatch', 'oracle_recurrence',
           'oracle_route', 'set_threads', 'OracleLayer', 'near_square_factors', 'state_interval',
           'oracle_bank_histogram', 'oracle_bank_owners', 'oracle_combine_partial', 'oracle_dispatch_owned']
