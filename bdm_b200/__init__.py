"""B200-native Block Delta Memory (BDM) layer hot path.

Drop-in for the reference module's layer API (``BSDMConfig``,
``BlockSparseDeltaMemory(config, layer_id=, seed=)``, ``forward`` /
``prefill`` / ``step``; training backward; the ``BDMLanguageModel`` shell).  The bank path -- controllers epilogue, product-key
router, causal dispatch, per-bank recurrence, read combine, decode step -- runs
in hand-written sm_100a kernels behind the C ABI in ``include/bdm_b200.h``
(``libbdm_b200.so`` in this directory, built by ``python -m bdm_b200.build``).
"""
from .config import BDMConfig, BSDMConfig, near_square_factors, state_interval
from .layer import BankedDeltaMemory, BlockSparseDeltaMemory, SharedResidualRouter
from .lm import BDMLanguageModel, LanguageModelConfig

__all__ = ['BDMConfig', 'BSDMConfig', 'BankedDeltaMemory', 'BlockSparseDeltaMemory', 'SharedResidualRouter',
           'BDMLanguageModel', 'LanguageModelConfig', 'near_square_factors', 'state_interval']
