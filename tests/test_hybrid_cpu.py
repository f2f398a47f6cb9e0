"""Partitioner and gateway of the B200 drivers vs the reference's own outputs
(golden fixtures from tree_grad_hybrid.py:60-250)."""
import glob
import os

import numpy as np
import pytest

from tests.golden_util import forest47_roots, rand_a_roots, twolevel_roots

from tree_training_b200 import build_dfs_tree_info
from tree_training_b200.hybrid import _partition_forest, gateway_visibility, partition_tree


def _roots(name):
    if "forest47" in name:
        return forest47_roots()
    if "rand_a" in name:
        return rand_a_roots()
    return twolevel_roots()


def _walk(parts, mode):
    """Yield (partition index, info, gateway visibility, pos_offset) in order."""
    gw = {}
    for i, p in enumerate(parts):
        g = gw.get(i)
        p.pos_offset = g[2] if g else 0
        info = build_dfs_tree_info(_partition_forest(p), pos_offset=p.pos_offset)
        yield i, p, info, g
        node_idx = {id(n.orig): k for k, n in enumerate(info.nodes)}
        for j, c in enumerate(parts):
            if c.parent is p:
                gw[j] = gateway_visibility(info, node_idx[id(c.parent_cut_node)], p.pos_offset,
                                           g[1] if g else None, mode)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(
    os.path.dirname(__file__), "golden", "partition_*.npz"))), ids=os.path.basename)
def test_partitions_and_reference_gateways_match(path):
    d = np.load(path)
    parts = partition_tree(_roots(os.path.basename(path)), int(d["max_tokens"]))
    assert len(parts) == int(d["n_parts"])
    order = {id(p): i for i, p in enumerate(parts)}
    for i, p, info, g in _walk(parts, "reference"):
        assert p.token_count == int(d[f"p{i}_token_count"])
        assert (order[id(p.parent)] if p.parent else -1) == int(d[f"p{i}_parent"])
        assert p.pos_offset == int(d[f"p{i}_pos_offset"])
        assert info.dfs_token_ids == d[f"p{i}_dfs_token_ids"].tolist()
        assert (info.dfs_pos_ids_np - p.pos_offset).tolist() == d[f"p{i}_dfs_pos_ids"].tolist()
        assert info.chunk_parent_map == d[f"p{i}_chunk_parent_map"].tolist()
        past = int(d[f"p{i}_past_len"])
        assert (g[0] if g else 0) == past
        if g:
            assert np.array_equal(g[1], d[f"p{i}_gateway_bias"] == 0)
        loss_leaf = [int(x) for x, f in zip(d[f"p{i}_leaf_chunk_ids"], d[f"p{i}_leaf_is_loss"]) if f]
        ours = [c for c in info.leaf_chunk_ids if id(info.nodes[c].orig) in p.leaf_node_set]
        assert ours == loss_leaf


def f2_roots(cls=None):
    """R[2] -> A[2], B[2]; B -> C[2] -> D[2] -> E[4].  With max_tokens=7 the
    partitions are {R,A,B}, {C,D}, {E}: the middle partition's gateway holds A
    masked (a DFS sibling of B), and E's gateway contains that gateway."""
    from tests.golden_util import Node
    cls = cls or Node
    r = cls([1, 2])
    r.add_child([3, 4])
    b = r.add_child([5, 6])
    b.add_child([7, 8]).add_child([9, 10]).add_child([11, 12, 13, 14])
    return [r]


def test_tree_mode_keeps_parent_gateway_masking():
    """With two cut levels the reference re-exposes keys its parent had
    masked (tree_grad_hybrid.py:207); the default mode keeps them masked."""
    parts = partition_tree(f2_roots(), 7)
    assert [p.token_count for p in parts] == [6, 4, 4]
    ref = {i: g for i, _, _, g in _walk(parts, "reference") if g}
    tree = {i: g for i, _, _, g in _walk(parts, "tree") if g}
    assert ref.keys() == tree.keys()
    diff = [i for i in ref if not np.array_equal(ref[i][1], tree[i][1])]
    assert diff, "the two-level case must exercise a parent-masked gateway key"
    for i in diff:
        # tree mode only ever hides keys the reference shows
        assert np.all(tree[i][1] <= ref[i][1])
        assert ref[i][0] == tree[i][0] and ref[i][2] == tree[i][2]
