"""LM shell (bdm_b200.lm) against the reference's BDMLanguageModel (tests/golden/lm_small.pt).

CPU: the seeded initial parameters equal the reference's bit for bit (same names, shapes,
values), and the config validates like the reference's.  GPU: the cross-entropy loss of one
training step and the gradients of every parameter match the reference's autograd (FP32,
FP32 state storage: 1e-4 max-relative per tensor).
"""
import os

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _golden():
    return torch.load(os.path.join(HERE, 'golden', 'lm_small.pt'))


def _model(d):
    from bdm_b200 import BSDMConfig
    from bdm_b200.lm import BDMLanguageModel, LanguageModelConfig
    cfg = LanguageModelConfig(memory=BSDMConfig(**d['memory']), vocab_size=d['vocab_size'], layers=d['layers'],
                              seed=d['seed'], ffn_multiple_of=d['ffn_multiple_of'])
    return BDMLanguageModel(cfg)


def test_lm_initialisation_matches_reference():
    d = _golden()
    sd = _model(d).state_dict()
    assert set(sd) == set(d['state_dict'])
    for k, ref in d['state_dict'].items():
        assert sd[k].shape == ref.shape and torch.equal(sd[k], ref), k


def test_lm_config_validation():
    from bdm_b200.lm import LanguageModelConfig
    with pytest.raises(ValueError):
        LanguageModelConfig(layers=0)
    with pytest.raises(ValueError):
        LanguageModelConfig(compact_replay=1)
    rec = LanguageModelConfig().record()
    assert rec['layers'] == 8 and rec['memory']['router'] == 'shared_residual_product_key'


@pytest.mark.gpu
def test_lm_training_step_matches_reference():
    d = _golden()
    m = _model(d).cuda()
    loss = m(d['tokens'].cuda(), d['target'].cuda())
    loss.backward()
    assert abs(loss.item() - d['loss'].item()) <= 1e-5 * abs(d['loss'].item())
    grads = {n: p.grad.cpu() for n, p in m.named_parameters() if p.grad is not None}
    assert set(grads) == set(d['grads'])
    bad = {}
    for n, ref in d['grads'].items():
        err = ((grads[n] - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()
        if not err <= 1e-4:
            bad[n] = err
    assert not bad, bad


@pytest.mark.gpu
def test_lm_prefill_step_and_graphed_step_match_forward():
    """FP32 model and caches: prefill over T tokens then one step reproduce the full forward's
    logits (same recurrence, no storage rounding); the CUDA-graphed step equals the eager one."""
    d = _golden()
    m = _model(d).cuda()
    gen = torch.Generator().manual_seed(8)
    tokens = torch.randint(0, d['vocab_size'], (2, 25), generator=gen).cuda()
    with torch.inference_mode():
        full = m(tokens)
        logits_p, caches = m.prefill(tokens[:, :24], state_dtype=torch.float32)
        eager_caches = [c.clone() for c in caches]
        logits_s = m.step(tokens[:, 24:], eager_caches)
        run = m.capture_step(caches)
        logits_g = run(tokens[:, 24:]).clone()
    scale = full.abs().max()
    assert ((logits_p - full[:, :24]).abs().max() / scale).item() <= 1e-4
    assert ((logits_s[:, 0] - full[:, 24]).abs().max() / scale).item() <= 1e-4
    assert torch.equal(logits_g, logits_s)
    for a, b in zip(caches, eager_caches):
        assert torch.equal(a, b)
