"""Pin the numpy oracle against golden vectors made by the reference itself.

The fixtures were produced by ``tests/golden/make_golden.py`` running the
reference's own Python code; these tests read only the committed ``.npz``.
"""
import glob
import os

import numpy as np
import pytest

from oracle import tree_oracle as O

from tests.golden_util import forest_from_arrays, load


def _packer_files():
    return sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "packer_*.npz")))


@pytest.mark.parametrize("path", _packer_files(), ids=lambda p: os.path.basename(p))
def test_oracle_packer_matches_reference(path):
    d = np.load(path)
    roots = forest_from_arrays(d["node_len"], d["node_parent"], d["node_tokens"])
    info = O.build_dfs_tree_info(roots)
    assert info.dfs_token_ids == d["dfs_token_ids"].tolist()
    assert info.dfs_pos_ids == d["dfs_pos_ids"].tolist()
    assert [list(b) for b in info.chunk_boundaries] == d["chunk_boundaries"].tolist()
    assert info.chunk_parent_map == d["chunk_parent_map"].tolist()
    assert info.leaf_chunk_ids == d["leaf_chunk_ids"].tolist()
    N = int(d["N"])
    mask = np.unpackbits(d["attn_mask_bool"])[: N * N].reshape(N, N).astype(bool)
    assert np.array_equal(info.attn_mask_bool(), mask)
    # the interval form reproduces the reference mask exactly
    lo, hi = O.key_intervals(info.chunk_boundaries, info.chunk_parent_map, N)
    assert np.array_equal(O.mask_from_intervals(lo, hi, N), mask)
    lo2, hi2 = O.intervals_from_mask(mask)
    nz = hi2 > lo2
    assert np.array_equal(lo2[nz], lo[nz]) and np.array_equal(hi2[nz], hi[nz])


def test_forest47_known_answers():
    """Topology facts of verify_hybrid.py:38-60 (47 tokens, 13 chunks)."""
    d = load("packer_forest47")
    assert int(d["N"]) == 47
    assert d["chunk_parent_map"].tolist() == [-1, 0, 1, 2, 3, 3, 2, 6, -1, 8, 9, 8, 11]
    assert d["leaf_chunk_ids"].tolist() == [4, 5, 7, 10, 12]


def _partition_files():
    return sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "partition_*.npz")))


@pytest.mark.parametrize("path", _partition_files(), ids=lambda p: os.path.basename(p))
def test_oracle_partition_and_gateway_match_reference(path):
    d = np.load(path)
    name = os.path.basename(path)
    src = "packer_forest47" if "forest47" in name else None
    roots = _roots_for_partition(name)
    parts = O.partition_tree(roots, int(d["max_tokens"]))
    assert len(parts) == int(d["n_parts"])
    gw = {}
    for i, p in enumerate(parts):
        assert p.token_count == int(d[f"p{i}_token_count"])
        assert (p.parent if p.parent is not None else -1) == int(d[f"p{i}_parent"])
        g = gw.get(i)
        p.pos_offset = g[2] if g else 0
        assert p.pos_offset == int(d[f"p{i}_pos_offset"])
        shims = O.partition_local_forest(p)
        info = O.build_dfs_tree_info(shims)
        assert info.dfs_token_ids == d[f"p{i}_dfs_token_ids"].tolist()
        assert info.dfs_pos_ids == d[f"p{i}_dfs_pos_ids"].tolist()
        assert info.chunk_parent_map == d[f"p{i}_chunk_parent_map"].tolist()
        past = int(d[f"p{i}_past_len"])
        assert (g[0] if g else 0) == past
        if g:
            assert np.array_equal(g[1], d[f"p{i}_gateway_bias"])
        # gateways for this partition's children
        seen = {}
        for j, c in enumerate(parts):
            if c.parent == i:
                cn = c.parent_cut_node
                if id(cn) not in seen:
                    seen[id(cn)] = O.gateway_for_cut(info, shims, cn, p.pos_offset, past)
                gw[j] = seen[id(cn)]
    del src


def _roots_for_partition(name):
    from tests.golden_util import forest47_roots, rand_a_roots, twolevel_roots
    if "forest47" in name:
        return forest47_roots()
    if "rand_a" in name:
        return rand_a_roots()
    return twolevel_roots()


@pytest.mark.parametrize("name", ["attn_forest47_f64", "attn_forest47_f32", "attn_rand_f64",
                                  "attn_gateway_f64"])
def test_oracle_attention_matches_reference(name):
    d = load(name)
    n_rows, n_cols = int(d["n_rows"]), int(d["n_cols"])
    allowed = np.unpackbits(d["allowed_bits"])[: n_rows * n_cols].reshape(n_rows, n_cols).astype(bool)
    q, k, v = d["q"][0], d["k"][0], d["v"][0]
    do = d["dout"][0].transpose(1, 0, 2)
    out, _ = O.attention_fwd(q, k, v, allowed, float(d["scale"]))
    dq, dk, dv = O.attention_bwd(q, k, v, allowed, float(d["scale"]), do)
    tol = 1e-10 if "f64" in name else 2e-5
    ref_out = d["out"][0].transpose(1, 0, 2)

    def rel(a, b):
        return np.abs(a - b).max() / (np.abs(b).max() + 1e-30)
    assert rel(out, ref_out) < tol
    assert rel(dq, d["dq"][0]) < tol
    assert rel(dk, d["dk"][0]) < tol
    assert rel(dv, d["dv"][0]) < tol
    # the mask is an interval per key column: what the kernels consume
    lo, hi = O.intervals_from_mask(allowed)
    assert np.array_equal(O.mask_from_intervals(lo, hi, n_rows), allowed)


@pytest.mark.parametrize("name", ["gdn_tree_l2", "gdn_tree_init_final", "gdn_forest47"])
def test_oracle_gdn_matches_reference(name):
    d = load(name)
    bounds = [tuple(b) for b in d["chunk_boundaries"].tolist()]
    parents = d["chunk_parent_map"].tolist()
    init = d["init"] if d["init"].size else None
    dlast = d["dlast"] if d["dlast"].size else None
    l2 = bool(int(d["l2norm"]))
    out, states = O.gdn_tree_fwd(d["q"], d["k"], d["v"], d["g"], d["beta"], bounds, parents,
                                 init, l2)

    def rel(a, b):
        return np.abs(a - b).max() / (np.abs(b).max() + 1e-30)
    # the reference computes in float32 internally (tree_dfs_ssm.py:72-76)
    tol = 2e-5
    assert rel(out, d["out"]) < tol
    if d["last"].size:
        assert rel(states[-1], d["last"]) < tol
    grads = O.gdn_tree_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], bounds, parents,
                           d["dout"], init, l2, dlast)
    for got, key in zip(grads, ["dq", "dk", "dv", "dg", "dbeta", "dinit"]):
        if key == "dinit" and init is None:
            continue
        assert rel(got, d[key]) < tol, key


@pytest.mark.parametrize("name", ["conv_tree", "conv_short_nodes"])
def test_oracle_conv_matches_reference(name):
    d = load(name)
    bounds = [tuple(b) for b in d["chunk_boundaries"].tolist()]
    parents = d["chunk_parent_map"].tolist()
    y, _ = O.tree_conv_fwd(d["x"], d["weight"], bounds, parents)
    dx, dw, _ = O.tree_conv_bwd(d["x"], d["weight"], bounds, parents, d["dout"])

    def rel(a, b):
        return np.abs(a - b).max() / (np.abs(b).max() + 1e-30)
    assert rel(y, d["out"]) < 1e-12
    assert rel(dx, d["dx"]) < 1e-12
    assert rel(dw, d["dweight"]) < 1e-12
