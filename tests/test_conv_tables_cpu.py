"""Host-side conv tables (tt_conv_predecessors / tt_conv_successors) vs the
oracle's restatement of the reference's parent-context rule
(tree_dfs_ssm.py:316-318, 338-346)."""
import numpy as np
import pytest

from oracle import tree_oracle as O

import tree_training_b200 as tt
from tree_training_b200 import _lib
from tree_training_b200.synthetic import random_branching_tree


@pytest.mark.parametrize("seed,lo,hi,K", [(0, 1, 3, 4), (1, 1, 1, 4), (2, 2, 9, 3), (3, 1, 5, 6)])
def test_predecessors_and_successors(seed, lo, hi, K):
    info = tt.build_dfs_tree_info(random_branching_tree(seed, 300, lo, hi))
    ref = O.conv_predecessors(info.chunk_boundaries, info.chunk_parent_map, K)
    b = np.ascontiguousarray(info.chunk_bounds_np, np.int32)
    p = np.ascontiguousarray(info.parents_np, np.int32)
    pred = np.zeros((info.N, K - 1), np.int32)
    _lib.call("tt_conv_predecessors", info.n_chunks, b.ctypes.data, p.ctypes.data, K,
              pred.ctypes.data)
    assert np.array_equal(pred, ref)
    cap = info.N * (K - 1)
    sp = np.zeros(info.N + 1, np.int32)
    st = np.zeros(cap, np.int32)
    sl = np.zeros(cap, np.int32)
    _lib.call("tt_conv_successors", info.N, K, pred.ctypes.data, sp.ctypes.data, st.ctypes.data,
              sl.ctypes.data, cap)
    for t in range(info.N):
        got = sorted(zip(st[sp[t]:sp[t + 1]].tolist(), sl[sp[t]:sp[t + 1]].tolist()))
        want = sorted((u, m + 1) for u in range(info.N) for m in range(K - 1) if ref[u, m] == t)
        assert got == want


@pytest.mark.parametrize("seed,lo,hi,K", [(4, 1, 3, 4), (5, 1, 1, 4), (6, 2, 9, 8), (7, 1, 40, 4)])
def test_successor_lists_start_with_the_near_chain(seed, lo, hi, K):
    """The order the fused token-major conv backward relies on: in every
    token's CSR list the entries (t + l, l) -- the tokens that follow t inside
    its path -- form a prefix l = 1 .. n, and every later entry (u, l) has
    u > t + l (a later child of t's node, further on in DFS order)."""
    info = tt.build_dfs_tree_info(random_branching_tree(seed, 400, lo, hi))
    b = np.ascontiguousarray(info.chunk_bounds_np, np.int32)
    p = np.ascontiguousarray(info.parents_np, np.int32)
    pred = np.zeros((info.N, K - 1), np.int32)
    _lib.call("tt_conv_predecessors", info.n_chunks, b.ctypes.data, p.ctypes.data, K,
              pred.ctypes.data)
    cap = info.N * (K - 1)
    sp = np.zeros(info.N + 1, np.int32)
    st = np.zeros(cap, np.int32)
    sl = np.zeros(cap, np.int32)
    _lib.call("tt_conv_successors", info.N, K, pred.ctypes.data, sp.ctypes.data, st.ctypes.data,
              sl.ctypes.data, cap)
    far_lists = 0
    for t in range(info.N):
        ent = list(zip(st[sp[t]:sp[t + 1]].tolist(), sl[sp[t]:sp[t + 1]].tolist()))
        near = 0
        while near < len(ent) and ent[near] == (t + near + 1, near + 1):
            near += 1
        assert all(u > t + l for u, l in ent[near:]), (t, ent)
        far_lists += near < len(ent)
    if hi > 1:
        assert far_lists > 0          # the case the far walk covers does occur


def test_gdn_workspace_size_is_positive_and_rejects_bad_bounds():
    b = np.array([[0, 5], [5, 9]], np.int32)
    assert _lib.lib().tt_gdn_tree_workspace_size(9, 4, 64, 64, 2, b.ctypes.data, 0) > 0
    assert (_lib.lib().tt_gdn_tree_workspace_size(9, 4, 64, 64, 2, b.ctypes.data, 1)
            > _lib.lib().tt_gdn_tree_workspace_size(9, 4, 64, 64, 2, b.ctypes.data, 0))
    bad = np.array([[0, 5], [6, 9]], np.int32)      # gap between nodes
    assert _lib.lib().tt_gdn_tree_workspace_size(9, 4, 64, 64, 2, bad.ctypes.data, 0) < 0
