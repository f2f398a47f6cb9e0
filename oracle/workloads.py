"""Benchmark trees and attention metadata built without the product package.

TEST AND CPU-BASELINE INFRASTRUCTURE ONLY: ``bench.py --impl reference`` runs
the reference's CPU path on these, so that arm never loads this repository's
compiled library; ``tests/test_oracle_workloads_cpu.py`` checks that the
generators here yield exactly the trees of ``tree_training_b200.synthetic``.

* :func:`bfs_tree` restates the config-2 generator (root prompt, BFS
  expansion with U{2..4} children of U[lo, hi] tokens, depth <= 6, children
  past the token budget skipped), drawing from ``random.Random`` in the same
  order so the same seed gives the same tree.
* :class:`OracleAttnMeta` is the dense mask of the reference's
  ``attn_mask_bool`` (dfs_tree_forward.py:157-172) in the column-interval form
  of :func:`oracle.tree_oracle.key_intervals`.
* :func:`time_reference_mask_loop` times the reference packer's element-by-
  element mask construction (dfs_tree_forward.py:157-172), the part of
  ``build_dfs_tree_info`` whose cost grows with the visible pairs, on a bounded
  sample of chunks.
"""
from __future__ import annotations

import random
import time
from typing import List

import numpy as np

from . import tree_oracle as O


class Node:
    """Forest node with the reference TreeNode's attributes (token_ids, children)."""
    __slots__ = ("token_ids", "children")

    def __init__(self, token_ids):
        self.token_ids = list(token_ids)
        self.children: List["Node"] = []

    def add_child(self, token_ids):
        c = Node(token_ids)
        self.children.append(c)
        return c

    @property
    def is_leaf(self):
        return not self.children


def bfs_tree(seed: int, n_tokens: int, len_lo: int, len_hi: int, root_len: int,
             branch=(2, 4), max_depth: int = 6, vocab: int = 32000) -> List[Node]:
    rng = random.Random(seed)
    tok = lambda n: [rng.randrange(vocab) for _ in range(n)]
    root = Node(tok(root_len))
    total = root_len
    frontier = [(root, 0)]
    while frontier and total < n_tokens:
        nxt = []
        for node, depth in frontier:
            if depth >= max_depth:
                continue
            for _ in range(rng.randint(*branch)):
                L = rng.randint(len_lo, len_hi)
                if total + L > n_tokens:
                    continue
                nxt.append((node.add_child(tok(L)), depth + 1))
                total += L
        frontier = nxt
    return [root]


class OracleAttnMeta:
    """n_q / n_kv / dense_mask() of a packed forest (no gateway keys)."""

    def __init__(self, roots):
        self.info = O.build_dfs_tree_info(roots)
        self.n_q = self.n_kv = self.info.N
        lo, hi = O.key_intervals(self.info.chunk_boundaries, self.info.chunk_parent_map,
                                 self.info.N)
        self.kv_lo, self.kv_hi = lo, hi
        self.visible_pairs = int((hi - lo).sum())

    def dense_mask(self) -> np.ndarray:
        return O.mask_from_intervals(self.kv_lo, self.kv_hi, self.n_q)

    def visible_pairs_of_rows(self, rows) -> int:
        rows = np.asarray(rows)
        return int(((rows[:, None] >= self.kv_lo[None, :]) &
                    (rows[:, None] < self.kv_hi[None, :])).sum())


def time_reference_mask_loop(info: O.OracleDFSInfo, max_pairs: int = 2_000_000):
    """The reference's mask loop (dfs_tree_forward.py:157-172: one Python
    ``attn_mask_bool[i, j] = True`` per visible pair, into a torch bool
    tensor) over the first chunks of the DFS order until about ``max_pairs``
    pairs are set.  Returns (seconds, pairs set); the whole packer costs about
    seconds * V / pairs for a tree with V visible pairs (the rest of
    build_dfs_tree_info is linear in the token count)."""
    import torch
    N = info.N
    anc: List[List[int]] = []
    for c, p in enumerate(info.chunk_parent_map):
        anc.append([c] if p == -1 else anc[p] + [c])
    mask = torch.zeros(N, N, dtype=torch.bool)
    pairs = 0
    t0 = time.perf_counter()
    for c in range(info.n_chunks):
        c_start, c_end = info.chunk_boundaries[c]
        for a in anc[c]:
            a_start, a_end = info.chunk_boundaries[a]
            for i in range(c_start, c_end):
                if a == c:
                    for j in range(c_start, i + 1):
                        mask[i, j] = True
                    pairs += i + 1 - c_start
                else:
                    for j in range(a_start, a_end):
                        mask[i, j] = True
                    pairs += a_end - a_start
                if pairs >= max_pairs:
                    return time.perf_counter() - t0, pairs
    return time.perf_counter() - t0, pairs
