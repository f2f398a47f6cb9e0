"""Pins the torch GDN / conv ports (oracle/gdn_torch.py) to the numpy oracle.

Both restate torch_chunk_gated_delta_rule_tree_varlen (tree_dfs_ssm.py:38-156);
the oracle is itself pinned to the reference's outputs by
``tests/test_oracle_golden.py``.  float64 on CPU: forward, last state and the
autograd gradients against the oracle's analytic ones, to 1e-10.
"""
import numpy as np
import torch

from oracle import tree_oracle as O
from oracle.gdn_torch import gdn_tree_torch, tree_conv_torch

import tree_training_b200 as tt
from tree_training_b200.synthetic import random_branching_tree


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


def test_torch_checker_matches_numpy_oracle():
    S, Hk, H, Dk = 700, 2, 4, 16
    info = tt.build_dfs_tree_info(random_branching_tree(17, S, 8, 120))
    bounds, parents = info.chunk_boundaries, info.chunk_parent_map
    g_ = np.random.default_rng(17)
    q = g_.standard_normal((1, S, Hk, Dk))
    k = g_.standard_normal((1, S, Hk, Dk))
    v = g_.standard_normal((1, S, H, Dk)) * 0.5
    gg = -np.log1p(np.exp(-g_.standard_normal((1, S, H))))
    bt = 1.0 / (1.0 + np.exp(-g_.standard_normal((1, S, H))))
    s0 = g_.standard_normal((1, H, Dk, Dk)) * 0.05
    do = g_.standard_normal((1, S, H, Dk))
    dl = g_.standard_normal((1, H, Dk, Dk))
    ref_out, ref_states = O.gdn_tree_fwd(q, k, v, gg, bt, bounds, parents, s0, True)
    ref_grads = O.gdn_tree_bwd(q, k, v, gg, bt, bounds, parents, do, s0, True, dl)
    ts = [torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (q, k, v, gg, bt, s0)]
    out, last = gdn_tree_torch(*ts[:5], bounds, parents, ts[5], True)
    ((out * torch.from_numpy(do)).sum() + (last * torch.from_numpy(dl)).sum()).backward()
    assert _rel(out.detach(), ref_out) < 1e-10
    assert _rel(last.detach(), ref_states[-1]) < 1e-10
    for t, ref in zip(ts, ref_grads):
        assert _rel(t.grad, ref) < 1e-10


def test_torch_row_loop_equals_closed_form():
    S, H, Dk = 300, 2, 8
    info = tt.build_dfs_tree_info(random_branching_tree(5, S, 4, 60))
    g_ = np.random.default_rng(5)
    ts = [torch.tensor(x, dtype=torch.float64) for x in (
        g_.standard_normal((1, S, H, Dk)), g_.standard_normal((1, S, H, Dk)),
        g_.standard_normal((1, S, H, Dk)), -np.log1p(np.exp(-g_.standard_normal((1, S, H)))),
        1.0 / (1.0 + np.exp(-g_.standard_normal((1, S, H)))))]
    a, _ = gdn_tree_torch(*ts, info.chunk_boundaries, info.chunk_parent_map, None, True)
    b, _ = gdn_tree_torch(*ts, info.chunk_boundaries, info.chunk_parent_map, None, True,
                          row_loop=True)
    assert _rel(a, b) < 1e-12


def test_torch_conv_matches_numpy_oracle():
    info = tt.build_dfs_tree_info(random_branching_tree(6, 500, 1, 12))
    g_ = np.random.default_rng(6)
    x = g_.standard_normal((2, 5, info.N))
    w = g_.standard_normal((5, 4)) * 0.5
    dy = g_.standard_normal((2, 5, info.N))
    xt = torch.tensor(x, requires_grad=True)
    wt = torch.tensor(w, requires_grad=True)
    y = tree_conv_torch(xt, wt, info.chunk_boundaries, info.chunk_parent_map)
    y.backward(torch.from_numpy(dy))
    ref_y, _ = O.tree_conv_fwd(x, w, info.chunk_boundaries, info.chunk_parent_map)
    dx, dw, _ = O.tree_conv_bwd(x, w, info.chunk_boundaries, info.chunk_parent_map, dy)
    assert _rel(y.detach(), ref_y) < 1e-12
    assert _rel(xt.grad, dx) < 1e-12
    assert _rel(wt.grad, dw) < 1e-12
