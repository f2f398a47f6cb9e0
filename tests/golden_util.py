"""Helpers shared by the tests: load fixtures and rebuild their forests."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


class Node:
    """Minimal forest node with the reference TreeNode's two attributes."""
    __slots__ = ("token_ids", "children")

    def __init__(self, token_ids, children=None):
        self.token_ids = list(token_ids)
        self.children = list(children) if children else []

    def add_child(self, token_ids):
        c = Node(token_ids)
        self.children.append(c)
        return c

    @property
    def is_leaf(self):
        return not self.children


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def forest_from_arrays(node_len, node_parent, node_tokens, cls=Node):
    """Rebuild a forest from pre-order (len, parent, tokens) arrays."""
    nodes, roots, off = [], [], 0
    for L, p in zip(node_len.tolist(), node_parent.tolist()):
        n = cls(node_tokens[off:off + L].tolist())
        off += L
        nodes.append(n)
        if p < 0:
            roots.append(n)
        else:
            nodes[p].children.append(n)
    return roots


def forest47_roots(cls=Node):
    d = load("packer_forest47")
    return forest_from_arrays(d["node_len"], d["node_parent"], d["node_tokens"], cls)


def rand_a_roots(cls=Node):
    d = load("packer_rand_a")
    return forest_from_arrays(d["node_len"], d["node_parent"], d["node_tokens"], cls)


def twolevel_roots(cls=Node):
    """Same literal tree as make_golden.py's 'twolevel' partition case."""
    root = cls([1, 2, 3])
    a1 = root.add_child([4, 5, 6])
    root.add_child([7, 8])
    b1 = a1.add_child([9, 10, 11])
    a1.add_child([12, 13])
    b1.add_child([14, 15, 16]).add_child([17])
    return [root]
