"""Language-model shell around the B200 BDM layer (the c5 training host).

Mirrors the reference's ``BDMLanguageModel`` / ``LanguageModelConfig`` / ``BDMBlock``
(implementation/bdm/model.py:143-216) and the RMSNorm and SwiGLU feed-forward it uses
(_shell.py:10-112): the same module tree, parameter names, shapes and seeded
initialisation, so checkpoints move between the two.  Per block:
``h + mixer(norm(h))`` then ``h + ffn(norm(h))``, where the mixer is
``bdm_b200.BankedDeltaMemory`` (the hand-written sm_100a kernels, forward and
backward) and the feed-forward is three cuBLAS GEMMs around SiLU-gating.

Data parallelism is plain ``torch.nn.parallel.DistributedDataParallel`` over NCCL:
every parameter, the BDM layers' included, gets an ordinary ``.grad`` from the
layer's autograd Function, so DDP's bucketed all-reduce overlaps the backward.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field

import torch
from torch import nn
from torch.nn import functional as F
from torch.utils.checkpoint import checkpoint

from .config import BDMConfig
from .layer import BankedDeltaMemory


@dataclass(frozen=True)
class LanguageModelConfig:
    """model.py:143-160: memory geometry, vocabulary, depth, FFN rounding, seed."""
    memory: BDMConfig = field(default_factory=BDMConfig)
    vocab_size: int = 192
    layers: int = 8
    ffn_multiple_of: int = 256
    seed: int = 0
    recompute_ffn: bool = True
    compact_replay: bool | None = None

    def __post_init__(self):
        if min(self.vocab_size, self.layers, self.ffn_multiple_of) <= 0 or self.seed < 0:
            raise ValueError('invalid language-model geometry or seed')
        if self.compact_replay is not None and type(self.compact_replay) is not bool:
            raise ValueError('compact_replay must be None, True, or False')

    def record(self):
        return dict(asdict(self), memory=self.memory.record())


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight, computed in FP32 and returned in x's dtype."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).type_as(x)

    def reset_parameters(self):
        nn.init.ones_(self.weight)


class FeedForward(nn.Module):
    """SwiGLU feed-forward w2(silu(w1 x) * w3 x); hidden width int(2h/3) rounded up to multiple_of.

    Like the reference, large BF16 training calls recompute the hidden activations in the
    backward instead of keeping them.
    """

    def __init__(self, dim: int, hidden_dim: int, multiple_of: int, ffn_dim_multiplier=None,
                 recompute_activations: bool = False):
        super().__init__()
        hidden = int(2 * hidden_dim / 3)
        if ffn_dim_multiplier is not None:
            hidden = int(ffn_dim_multiplier * hidden)
        hidden = multiple_of * ((hidden + multiple_of - 1) // multiple_of)
        self.dim, self.hidden_dim = dim, hidden
        self.recompute_activations = recompute_activations
        self.w1 = nn.Linear(dim, hidden, bias=False)
        self.w3 = nn.Linear(dim, hidden, bias=False)
        self.w2 = nn.Linear(hidden, dim, bias=False)

    def _body(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))

    def forward(self, x):
        if (self.recompute_activations and torch.is_grad_enabled() and x.is_cuda and x.dtype == torch.bfloat16
                and x.numel() // self.dim >= 1024):
            return checkpoint(self._body, x, use_reentrant=False, preserve_rng_state=False)
        return self._body(x)

    def reset_parameters(self, init_std=None, factor=1.0):
        """Truncated normals: std dim^-1/2 for w1 / w3, hidden^-1/2 / factor for w2 (3 std cut)."""
        std_in = init_std or self.dim ** -0.5
        std_out = (init_std or self.hidden_dim ** -0.5) / factor
        for w, std in ((self.w1, std_in), (self.w3, std_in), (self.w2, std_out)):
            nn.init.trunc_normal_(w.weight, mean=0.0, std=std, a=-3 * std, b=3 * std)


class BDMBlock(nn.Module):
    def __init__(self, config: LanguageModelConfig, index: int, backend: str = 'role'):
        super().__init__()
        dim = config.memory.dim
        self.attention = BankedDeltaMemory(config.memory, layer_id=index, seed=config.seed, backend=backend,
                                           compact_replay=config.compact_replay)
        self.feed_forward = FeedForward(dim, 4 * dim, config.ffn_multiple_of, None,
                                        recompute_activations=config.recompute_ffn)
        self.attention_norm = RMSNorm(dim, eps=config.memory.norm_eps)
        self.ffn_norm = RMSNorm(dim, eps=config.memory.norm_eps)

    def forward(self, hidden):
        hidden = hidden + self.attention(self.attention_norm(hidden))
        return hidden + self.feed_forward(self.ffn_norm(hidden))


class BDMLanguageModel(nn.Module):
    """Embedding, ``layers`` BDM blocks, final RMSNorm and an untied output head."""

    def __init__(self, config: LanguageModelConfig, *, backend: str = 'role'):
        super().__init__()
        self.config = config
        self.dim = config.memory.dim
        self.layers = nn.ModuleList([BDMBlock(config, i, backend) for i in range(config.layers)])
        self.tok_embeddings = nn.Embedding(config.vocab_size, self.dim)
        self.norm = RMSNorm(self.dim, eps=config.memory.norm_eps)
        self.output = nn.Linear(self.dim, config.vocab_size, bias=False)
        # seeded initialisation (model.py:186-195): embeddings and head from seed*1e5 + 100,
        # each block's memory from seed*1e5 + 6000 + i, each feed-forward from seed*1e5 + 1000 + i
        base, std = config.seed * 100_000, self.dim ** -0.5
        with torch.random.fork_rng(devices=[]):
            torch.manual_seed(base + 100)
            for parameter in (self.tok_embeddings.weight, self.output.weight):
                nn.init.trunc_normal_(parameter, mean=0.0, std=std, a=-3 * std, b=3 * std)
        for i, block in enumerate(self.layers):
            block.attention.init_weights(initialization_seed=base + 6000 + i)
            with torch.random.fork_rng(devices=[]):
                torch.manual_seed(base + 1000 + i)
                block.feed_forward.reset_parameters()

    def hidden_states(self, tokens):
        hidden = self.tok_embeddings(tokens)
        for block in self.layers:
            hidden = block(hidden)
        return hidden

    def forward(self, tokens, target=None):
        """Logits [B, T, vocab], or with ``target`` the mean token cross-entropy (FP32)."""
        logits = self.output(self.norm(self.hidden_states(tokens)))
        if target is not None:
            return F.cross_entropy(logits.float().flatten(0, -2), target.flatten())
        return logits

    # ---------------------------------------------------- stateful inference
    def prefill(self, tokens, caches=None, *, state_dtype=None):
        """Process a prefix [B, T] -> (logits [B, T, vocab], per-layer bank caches).

        Every block's mixer runs ``BankedDeltaMemory.prefill`` (inference.py:110-131): FP32
        recurrence, the cache rounded once to its storage dtype (BF16 unless ``state_dtype`` or the
        given caches say otherwise).  Requires no_grad / inference_mode.
        """
        hidden = self.tok_embeddings(tokens)
        out = []
        for i, block in enumerate(self.layers):
            mix, cache = block.attention.prefill(block.attention_norm(hidden), None if caches is None else caches[i],
                                                 state_dtype=state_dtype)
            hidden = hidden + mix
            hidden = hidden + block.feed_forward(block.ffn_norm(hidden))
            out.append(cache)
        return self.output(self.norm(hidden)), out

    def step(self, tokens, caches):
        """One token per row [B, 1] -> logits [B, 1, vocab]; advances ``caches`` in place."""
        hidden = self.tok_embeddings(tokens)
        for block, cache in zip(self.layers, caches):
            mix, _ = block.attention.step(block.attention_norm(hidden), cache)
            hidden = hidden + mix
            hidden = hidden + block.feed_forward(block.ffn_norm(hidden))
        return self.output(self.norm(hidden))

    def capture_step(self, caches, *, warmup=2):
        """CUDA-graph one decode step of the whole model bound to ``caches`` (from ``prefill``).

        Returns ``run(tokens[B, 1]) -> logits[B, 1, vocab]``: copies the tokens into the graph's
        input, replays the step (advancing ``caches`` in place, as ``step`` does) and returns the
        graph's logits buffer, which the next call overwrites.  Warm-up runs on clones of the
        caches.  Parameters must not change afterwards.
        """
        if torch.is_grad_enabled():
            raise RuntimeError('capture_step requires no_grad or inference_mode')
        batch = caches[0].shape[0]
        dev = caches[0].device
        tokens_in = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        scratch = [c.clone() for c in caches]
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(tokens_in, scratch)
        torch.cuda.current_stream(dev).wait_stream(side)
        del scratch
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            logits = self.step(tokens_in, caches)

        def run(tokens):
            tokens_in.copy_(tokens)
            graph.replay()
            return logits

        run.graph = graph
        return run
