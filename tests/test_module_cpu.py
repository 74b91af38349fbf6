"""Host-side parity of the drop-in module: config validation, parameters and seeded init.

The golden layer fixtures hold state_dicts produced by the reference's own
constructor and init_weights; the B200 module must reproduce them bit for bit
(same names, shapes, dtypes, values), so checkpoints move between the two.
"""
import os

import pytest
import torch

from bdm_b200 import BDMConfig, BlockSparseDeltaMemory, BSDMConfig, near_square_factors, state_interval


def _golden(golden_dir, name):
    return torch.load(os.path.join(golden_dir, f'layer_{name}.pt'), weights_only=False)


@pytest.mark.parametrize('name', ['h1_fp32', 'h1_fp32_state32', 'h1_bf16', 'h2_bf16', 'h2_fp32_state32'])
def test_init_matches_reference_state_dict(golden_dir, name):
    data = _golden(golden_dir, name)
    cfg = BSDMConfig(**data['config'])
    m = BlockSparseDeltaMemory(cfg, seed=data['seed'])
    if data['dtype'] == 'torch.bfloat16':
        m = m.to(torch.bfloat16)
    ours, ref = m.state_dict(), data['state_dict']
    assert list(ours) == list(ref)
    for key in ref:
        assert ours[key].dtype == ref[key].dtype, key
        assert torch.equal(ours[key], ref[key]), key


def test_global_rng_consumption_matches_reference_order(golden_dir):
    """Constructing the layer draws the same global RNG as the reference (nn.Linear defaults)."""
    data = _golden(golden_dir, 'h1_fp32')
    cfg = BSDMConfig(**data['config'])
    torch.manual_seed(123)
    BlockSparseDeltaMemory(cfg)
    after = torch.rand(4)
    torch.manual_seed(123)
    for shape, bias in (((8, 64), False), ((8, 64), False), ((32, 64), False), ((16, 64), True), ((16, 64), True),
                        ((16, 64), True), ((32, 64), False), ((8, 32), False), ((8, 64), False), ((32, 64), False),
                        ((32, 64), True), ((64, 32), True)):
        torch.nn.Linear(shape[1], shape[0], bias=bias)
    assert torch.equal(torch.rand(4), after)


def test_config_validation_and_record_round_trip():
    cfg = BSDMConfig(dim=1024, bank_count=256, bank_size=8, selected_banks=8, value_width=1024, num_heads=8)
    assert cfg.logical_rows == 256 * 8 * 8 and cfg.head_value_width == 128
    assert BSDMConfig.from_record(cfg.record()) == cfg
    assert near_square_factors(2048) == (32, 64) and near_square_factors(16384) == (128, 128)
    assert state_interval(8) == 16 and state_interval(16) == 8 and state_interval(4) == 16
    with pytest.raises(ValueError):
        BDMConfig(bank_count=256, selected_banks=17)
    with pytest.raises(ValueError):
        BDMConfig(value_width=100, num_heads=3)
    with pytest.raises(ValueError):
        BDMConfig(bank_size=300)


def test_cpu_inputs_fail_loudly():
    cfg = BSDMConfig(dim=64, bank_count=64, bank_size=8, selected_banks=4, value_width=32)
    m = BlockSparseDeltaMemory(cfg)
    with torch.no_grad(), pytest.raises(ValueError, match='CUDA'):
        m(torch.randn(1, 4, 64))
    with pytest.raises(ValueError):
        BlockSparseDeltaMemory(cfg, backend='reference')
