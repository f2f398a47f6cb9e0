"""The reference arm's inputs (oracle/workloads.py) are the product arm's inputs.

``bench.py --impl reference`` builds its tree and mask without importing the
product package; these checks show that it times the same work: the oracle's
generator gives the package generator's tree token for token, its intervals
equal the native packer's, and the port of the reference packer's mask loop
sets exactly the dense mask.
"""
import numpy as np

from oracle import tree_oracle as O
from oracle.workloads import OracleAttnMeta, bfs_tree, time_reference_mask_loop

import tree_training_b200 as tt
from tree_training_b200 import synthetic


def _flat(roots):
    out = []
    stack = list(reversed(roots))
    while stack:
        n = stack.pop()
        out.append((tuple(n.token_ids), len(n.children)))
        stack.extend(reversed(n.children))
    return out


def test_generator_and_intervals_match_the_package():
    for seed, tokens in ((1000, 16384), (1001, 16384), (7, 3000)):
        a = bfs_tree(seed, tokens, 64, 512, min(2048, tokens // 8))
        b = synthetic.bfs_tree(seed, tokens, 64, 512, min(2048, tokens // 8))
        assert _flat(a) == _flat(b)
        om = OracleAttnMeta(a)
        pm = tt.build_dfs_tree_info(b).attn_meta()
        assert om.n_q == pm.n_q and om.visible_pairs == pm.visible_pairs
        assert np.array_equal(om.kv_lo, pm.kv_lo) and np.array_equal(om.kv_hi, pm.kv_hi)


def test_reference_mask_loop_port_sets_the_dense_mask():
    roots = bfs_tree(3, 900, 16, 80, 100)
    info = O.build_dfs_tree_info(roots)
    secs, pairs = time_reference_mask_loop(info, max_pairs=10 ** 9)
    assert secs > 0
    assert pairs == int(info.attn_mask_bool().sum())
