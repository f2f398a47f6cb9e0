"""Host logic of the SSM gateway (no GPU): the conv context captured at a cut
node is the last K-1 pre-conv inputs on its root-to-node path, the same tokens
the reference's per-chunk recursion keeps (tree_grad_hybrid_ssm.py:164-199:
conv_states[c] = last K-1 of (parent context ++ chunk), zero padded at
roots), including through an injected gateway context."""
import numpy as np
import pytest
import torch

from tree_training_b200.ssm import _path_tail


def _reference_contexts(bounds, parents, K, init=None):
    """The reference's recursion on token labels (-1 = zero padding)."""
    ctx = {}
    if init is not None:
        ctx[-1] = list(init)
    for c, (s, e) in enumerate(bounds):
        chunk = list(range(s, e))
        par = ctx.get(parents[c])
        ext = (par + chunk) if par is not None else ([-1] * max(0, K - 1 - len(chunk)) + chunk)
        ctx[c] = ext[-(K - 1):]
    return ctx


def _random_tree(seed, n):
    g = np.random.default_rng(seed)
    lens = g.integers(1, 6, n)
    parents = [-1] + [int(g.integers(-1, i)) for i in range(1, n)]
    # pre-order: each node's parent must come earlier, which holds by construction
    bounds, s0 = [], 0
    for L in lens:
        bounds.append((s0, s0 + int(L)))
        s0 += int(L)
    return bounds, parents


@pytest.mark.parametrize("seed", [0, 1, 2])
@pytest.mark.parametrize("K", [2, 4, 6])
def test_path_tail_equals_reference_conv_context(seed, K):
    bounds, parents = _random_tree(seed, 12)
    ref = _reference_contexts(bounds, parents, K)
    for c in range(len(bounds)):
        assert _path_tail(bounds, parents, c, K - 1) == ref[c], c


def test_path_tail_continues_into_injected_context():
    """With a gateway context the root chunks hang below a (K-1)-token prefix
    node, as conv_varlen_capture builds it."""
    K = 4
    bounds, parents = _random_tree(7, 10)
    off = K - 1
    ext_bounds = [(0, off)] + [(s + off, e + off) for s, e in bounds]
    ext_parents = [-1] + [p + 1 if p >= 0 else 0 for p in parents]
    init = [100, 101, 102]                      # labels of the injected context
    ref = _reference_contexts(bounds, parents, K, init=init)
    for c in range(len(bounds)):
        got = _path_tail(ext_bounds, ext_parents, c + 1, K - 1)
        got = [init[t] if t < off else t - off for t in got]
        assert got == ref[c], c


def test_fused_gated_norm_selection():
    """The hybrid layers run the fused gated-RMSNorm kernels only for
    transformers' torch gated norms of a supported width; anything else keeps
    its own forward, and the fused op itself refuses CPU tensors."""
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeRMSNormGated

    from tree_training_b200.gated_norm import fusable, gated_rmsnorm
    for d in (32, 64, 128, 256):
        assert fusable(Qwen3_5MoeRMSNormGated(d))
    assert not fusable(Qwen3_5MoeRMSNormGated(48))
    assert not fusable(torch.nn.LayerNorm(64))
    assert not fusable(torch.nn.RMSNorm(64))
    x = torch.randn(4, 64)
    with pytest.raises(RuntimeError):
        gated_rmsnorm(x, x, torch.ones(64), 1e-6)
