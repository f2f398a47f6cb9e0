"""Native packer, gateway intervals and tile lists vs the oracle (CPU only).

These call the host-side C-ABI functions (no CUDA work), so they run here and
on the GPU box alike."""
import glob
import os
import random
import re

import numpy as np
import pytest

from oracle import tree_oracle as O
from tests.golden_util import Node, forest_from_arrays, load

import tree_training_b200 as tt
from tree_training_b200 import _lib


def _packer_files():
    return sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "packer_*.npz")))


@pytest.mark.parametrize("path", _packer_files(), ids=lambda p: os.path.basename(p))
def test_native_packer_bit_exact_vs_reference(path):
    d = np.load(path)
    roots = forest_from_arrays(d["node_len"], d["node_parent"], d["node_tokens"])
    info = tt.build_dfs_tree_info(roots)
    assert info.dfs_token_ids == d["dfs_token_ids"].tolist()
    assert info.dfs_pos_ids == d["dfs_pos_ids"].tolist()
    assert [list(b) for b in info.chunk_boundaries] == d["chunk_boundaries"].tolist()
    assert info.chunk_parent_map == d["chunk_parent_map"].tolist()
    assert info.leaf_chunk_ids == d["leaf_chunk_ids"].tolist()
    assert info.N == int(d["N"]) and info.n_chunks == int(d["n_chunks"])
    N = int(d["N"])
    mask = np.unpackbits(d["attn_mask_bool"])[: N * N].reshape(N, N).astype(bool)
    assert np.array_equal(info.attn_mask_bool.numpy(), mask)
    assert np.array_equal(info.attn_meta().dense_mask(), mask)


def _random_forest(rng, n_roots, depth, branch, lo, hi):
    def make(d):
        n = Node([rng.randrange(32000) for _ in range(rng.randint(lo, hi))])
        if d < depth:
            for _ in range(rng.randint(*branch)):
                n.children.append(make(d + 1))
        return n
    return [make(0) for _ in range(n_roots)]


@pytest.mark.parametrize("seed", range(12))
def test_native_packer_random_forests_vs_oracle(seed):
    rng = random.Random(seed)
    roots = _random_forest(rng, rng.randint(1, 3), rng.randint(0, 5), (0, 4), 0, 9)
    ref = O.build_dfs_tree_info(roots)
    info = tt.build_dfs_tree_info(roots, pos_offset=seed * 7)
    assert info.dfs_token_ids == ref.dfs_token_ids
    assert info.dfs_pos_ids == [p + seed * 7 for p in ref.dfs_pos_ids]
    assert info.chunk_boundaries == ref.chunk_boundaries
    assert info.chunk_parent_map == ref.chunk_parent_map
    assert info.leaf_chunk_ids == ref.leaf_chunk_ids
    lo, hi = O.key_intervals(ref.chunk_boundaries, ref.chunk_parent_map, ref.N)
    assert np.array_equal(info.kv_lo, lo) and np.array_equal(info.kv_hi, hi)
    assert np.array_equal(info.attn_mask_bool.numpy(), ref.attn_mask_bool())


def test_packer_rejects_non_preorder():
    # node 2's parent (0) is not on the path to node 1's subtree end when node
    # 1 is a child of 0 and node 2 claims parent 1 after a sibling: valid; but
    # parent index >= own index is invalid
    with pytest.raises(_lib.TTError):
        tt.pack_arrays(np.array([1, 1], np.int32), np.array([1, -1], np.int32))
    # pre-order violation: 0 -> 1 -> 2, then node 3 claims parent 1 after
    # node 2's subtree closed under a different root
    with pytest.raises(_lib.TTError):
        tt.pack_arrays(np.array([1, 1, 1, 1], np.int32), np.array([-1, 0, -1, 1], np.int32))


def test_empty_forest():
    info = tt.build_dfs_tree_info([])
    assert info.N == 0 and info.n_chunks == 0 and info.dfs_token_ids == []


def test_gateway_intervals_from_reference_bias():
    d = load("attn_gateway_f64")
    bias = d["past"]
    lo, hi = tt.gateway_intervals_from_bias(bias, 17)
    assert np.array_equal(lo, np.zeros(len(bias), np.int32))
    assert np.array_equal(hi, np.where(bias == 0, 17, 0))
    with pytest.raises(_lib.TTError):
        tt.gateway_intervals_from_bias(np.array([0.0, -1.5]), 4)


def _tile_lists_reference(lo, hi, n_q, tq, tk):
    """Brute force (row, key) classification of every tile pair."""
    vis = O.mask_from_intervals(lo, hi, n_q)
    n_kv = len(lo)
    nqt, nkt = -(-n_q // tq), -(-n_kv // tk)
    out = {}
    for a in range(nqt):
        for b in range(nkt):
            blk = vis[a * tq:(a + 1) * tq, b * tk:(b + 1) * tk]
            if blk.any():
                full = blk.all() and blk.shape[1] == tk
                out[(a, b)] = full
    return out, int(vis.sum())


@pytest.mark.parametrize("seed,tq,tk", [(0, 4, 4), (1, 8, 16), (2, 16, 8), (3, 64, 64),
                                        (4, 5, 7)])
def test_tile_lists_match_brute_force(seed, tq, tk):
    rng = random.Random(100 + seed)
    roots = _random_forest(rng, 2, 4, (1, 3), 1, 30)
    info = tt.build_dfs_tree_info(roots)
    P = rng.randint(0, 20)
    glo = np.zeros(P, np.int32)
    ghi = np.where(np.array([rng.random() < 0.6 for _ in range(P)]), info.N, 0).astype(np.int32)
    meta = info.attn_meta(glo, ghi)
    t = meta.tiles(tq, tk)
    ref, pairs = _tile_lists_reference(meta.kv_lo, meta.kv_hi, meta.n_q, tq, tk)
    assert t["visible_pairs"] == pairs
    got_f = {}
    for a in range(len(t["fwd_ptr"]) - 1):
        for e in t["fwd_list"][t["fwd_ptr"][a]:t["fwd_ptr"][a + 1]]:
            got_f[(a, int(e) >> 1)] = (int(e) & 1) == 0
    got_b = {}
    for b in range(len(t["bwd_ptr"]) - 1):
        for e in t["bwd_list"][t["bwd_ptr"][b]:t["bwd_ptr"][b + 1]]:
            got_b[(int(e) >> 1, b)] = (int(e) & 1) == 0
    assert got_f == ref
    assert got_b == ref
    # each kv tile's q tiles ascend: the stored-dS backward finds a (q tile,
    # kv tile) pair's bwd entry from its fwd entry by binary search
    for b in range(len(t["bwd_ptr"]) - 1):
        qts = [int(e) >> 1 for e in t["bwd_list"][t["bwd_ptr"][b]:t["bwd_ptr"][b + 1]]]
        assert qts == sorted(set(qts))
    assert int(t["fwd_ptr"][-1]) == int(t["bwd_ptr"][-1])
    # full tiles must be really full: the kernels skip the mask test on them
    for (a, b), full in ref.items():
        assert got_f[(a, b)] == full


def _header_functions():
    hdr = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "include", "tree_training_b200.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(tt_[a-z0-9_]+)\s*\(", hdr)))


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    names = _header_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert L.tt_abi_version() == 3
    assert _lib.status_string(_lib.TT_ERR_NOT_INTERVAL).startswith("mask is not")


def test_attention_refuses_cpu_tensors():
    import torch
    info = tt.build_dfs_tree_info([Node([1, 2, 3])])
    q = torch.zeros(3, 2, 64)
    with pytest.raises(RuntimeError):
        tt.tree_attention(q, q[:, :1], q[:, :1], info.attn_meta())
