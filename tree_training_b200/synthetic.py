"""Seeded synthetic trees with the shapes of the benchmark configurations.

No dataset ships with the reference; these generators reproduce the tree
statistics the benchmark configurations specify (token ids are irrelevant to
attention timing and are drawn uniformly).
"""
from __future__ import annotations

import math
import random
from typing import List

from .packer import TreeNode


def bfs_tree(seed: int, n_tokens: int, len_lo: int, len_hi: int, root_len: int,
             branch=(2, 4), max_depth: int = 6, vocab: int = 32000) -> List[TreeNode]:
    """Config-2 style: a root prompt, then BFS expansion where every internal
    node gets U{branch} children of U[len_lo, len_hi] tokens, depth <= max_depth,
    children that would pass the token budget are skipped."""
    rng = random.Random(seed)
    tok = lambda n: [rng.randrange(vocab) for _ in range(n)]
    root = TreeNode(tok(root_len))
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
                c = node.add_child(tok(L))
                total += L
                nxt.append((c, depth + 1))
        frontier = nxt
    return [root]


def config2_tree(seed: int = 0) -> List[TreeNode]:
    """16,384-token tree: root prompt 2048, 2-4 children, lengths U[64,512], depth <= 6."""
    return bfs_tree(seed, 16384, 64, 512, 2048)


def agentic_tree(seed: int, n_tokens: int = 65536, root_len: int = 8192, n_leaves: int = 32,
                 len_lo: int = 32, len_hi: int = 4096, max_depth: int = 10,
                 vocab: int = 32000) -> List[TreeNode]:
    """Config-3 style long trajectory tree: shared root prefix, ``n_leaves``
    leaves from repeated binary splits of random leaves (depth <= max_depth),
    node lengths log-uniform in [len_lo, len_hi], rescaled so the tree holds
    exactly ``n_tokens`` tokens."""
    rng = random.Random(seed)
    root = TreeNode([])
    nodes = [(root, 0)]
    leaves = [(root, 0)]
    while len(leaves) < n_leaves:
        cand = [i for i, (_, d) in enumerate(leaves) if d < max_depth]
        i = rng.choice(cand)
        node, d = leaves.pop(i)
        for _ in range(2):
            c = node.add_child([])
            nodes.append((c, d + 1))
            leaves.append((c, d + 1))
    rest = [n for n, _ in nodes[1:]]
    lens = [math.exp(rng.uniform(math.log(len_lo), math.log(len_hi))) for _ in rest]
    budget = n_tokens - root_len
    scale = budget / sum(lens)
    ints = [max(len_lo, min(len_hi, int(L * scale))) for L in lens]
    ints[-1] += budget - sum(ints)
    root.token_ids = [rng.randrange(vocab) for _ in range(root_len)]
    for n, L in zip(rest, ints):
        n.token_ids = [rng.randrange(vocab) for _ in range(max(L, 1))]
    return [root]


def random_branching_tree(seed: int, n_tokens: int, len_lo: int, len_hi: int,
                          branch=(2, 4), vocab: int = 32000) -> List[TreeNode]:
    """Config-4/5 style: random 2-4 branching, node lengths U[len_lo, len_hi],
    filled breadth-first up to exactly ``n_tokens`` tokens (the last node is
    truncated to land on the budget)."""
    rng = random.Random(seed)
    L0 = rng.randint(len_lo, len_hi)
    root = TreeNode([rng.randrange(vocab) for _ in range(L0)])
    total = L0
    frontier = [root]
    while total < n_tokens:
        nxt = []
        for node in frontier:
            for _ in range(rng.randint(*branch)):
                if total >= n_tokens:
                    break
                L = min(rng.randint(len_lo, len_hi), n_tokens - total)
                nxt.append(node.add_child([rng.randrange(vocab) for _ in range(L)]))
                total += L
        frontier = nxt
    return [root]
