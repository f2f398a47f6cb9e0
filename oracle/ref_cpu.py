"""The reference's attention path on host cores (CPU baseline of bench.py).

TEST AND CPU-BASELINE INFRASTRUCTURE ONLY: used by ``bench.py``'s cpu_baseline leg
and ``--impl reference`` arm, never by the product package.

This is the call the reference makes for every attention layer, run on CPU:
the dense additive mask built as dfs_tree_forward.py:548-550 builds it (0 on
the visible pairs of dfs_tree_forward.py:157-172, -inf elsewhere) handed to
transformers' ``sdpa_attention_forward`` (TF/integrations/sdpa_attention.py:
40-104, which repeats K/V over the GQA group when a mask is given), forward
and torch-autograd backward.
"""
from __future__ import annotations

import time

import numpy as np
import torch


def dense_additive_mask(allowed: np.ndarray, dtype) -> torch.Tensor:
    n_q, n_kv = allowed.shape
    m = torch.full((1, 1, n_q, n_kv), float("-inf"), dtype=dtype)
    m[0, 0][torch.from_numpy(allowed)] = 0.0
    return m


class _Module(torch.nn.Module):
    def __init__(self, groups):
        super().__init__()
        self.num_key_value_groups = groups
        self.is_causal = True


def sdpa_tree_fwd_bwd(q, k, v, dout, mask, scale):
    """q [1,hq,n,D], k/v [1,hkv,n_kv,D], dout [1,n,hq,D] CPU tensors.
    Returns (out, dq, dk, dv)."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    q = q.detach().requires_grad_(True)
    k = k.detach().requires_grad_(True)
    v = v.detach().requires_grad_(True)
    out, _ = sdpa_attention_forward(_Module(q.shape[1] // k.shape[1]), q, k, v, mask,
                                    dropout=0.0, scaling=scale)
    out.backward(dout)
    return out.detach(), q.grad, k.grad, v.grad


def sample_rows(n_q: int, stride: int) -> np.ndarray:
    """Every ``stride``-th query row (spread over the whole tree, so the
    sample sees root, interior and leaf rows in proportion)."""
    return np.arange(0, n_q, max(1, int(stride)))


def visible_pairs(meta, rows=None) -> int:
    """Visible (query, key) pairs of the given query rows (all rows if None)."""
    allowed = meta.dense_mask()
    return int(allowed.sum() if rows is None else allowed[rows].sum())


def time_sample(meta, hq: int, hkv: int, D: int, dtype=torch.bfloat16, seed: int = 0,
                repeats: int = 1, rows=None):
    """Time fwd+bwd of the reference CPU path for ``hq`` query heads sharing
    ``hkv`` kv heads, on all n_q query rows or on the subset ``rows`` (each
    query row's attention is independent, so a row subset is an exact slice of
    the same computation, with every key).  Returns seconds per repeat (best)."""
    g = torch.Generator().manual_seed(seed)
    nr = meta.n_q if rows is None else len(rows)
    q = (torch.randn(1, hq, nr, D, generator=g) * 0.5).to(dtype)
    k = (torch.randn(1, hkv, meta.n_kv, D, generator=g) * 0.5).to(dtype)
    v = (torch.randn(1, hkv, meta.n_kv, D, generator=g) * 0.5).to(dtype)
    do = (torch.randn(1, nr, hq, D, generator=g) * 0.5).to(dtype)
    allowed = meta.dense_mask()
    mask = dense_additive_mask(allowed if rows is None else allowed[rows], dtype)
    best = float("inf")
    for _ in range(repeats):
        t0 = time.perf_counter()
        sdpa_tree_fwd_bwd(q, k, v, do, mask, D ** -0.5)
        best = min(best, time.perf_counter() - t0)
    return best
