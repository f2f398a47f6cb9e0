"""Helpers shared by the tests: load fixtures and rebuild their forests."""
import os

import numpy as np
import torch

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


def config1_model(seed=0):
    """The benchmark's config-1 model: random-init 2-layer Qwen3 (hidden 256,
    4/2 heads, head_dim 64, rope theta 1e6, intermediate 688), fp32, on CPU."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(seed)
    cfg = Qwen3Config(vocab_size=32000, hidden_size=256, intermediate_size=688,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=64, rope_theta=1e6, max_position_embeddings=4096,
                      tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    m = Qwen3ForCausalLM(cfg).to(torch.float32)
    m.train()
    return m


def config1_forest(TreeNode):
    """The 47-token forest (packer_forest47 topology) with token ids uniform in
    [0, 32000) from torch.Generator seed 0, and the leaf labels (seed 99)."""
    d = load("packer_forest47")
    g = torch.Generator().manual_seed(0)
    nodes, roots = [], []
    for L, p in zip(d["node_len"].tolist(), d["node_parent"].tolist()):
        n = TreeNode(torch.randint(0, 32000, (L,), generator=g).tolist())
        nodes.append(n)
        (roots if p < 0 else nodes[p].children).append(n)
    leaves = []

    def walk(n):
        if not n.children:
            leaves.append(n)
        for c in n.children:
            walk(c)
    for r in roots:
        walk(r)
    gl = torch.Generator().manual_seed(99)
    labels = [torch.randint(0, 32000, (len(n.token_ids),), generator=gl) for n in leaves]
    return roots, leaves, labels


def grad_projections(model, n_proj=32):
    """Per parameter: n_proj seeded Gaussian projections of the gradient, its
    norm and its max |entry| (size-independent fingerprints; the generator of
    parameter i is seeded 1000 + i)."""
    out = {}
    for i, (name, p) in enumerate(model.named_parameters()):
        if p.grad is None:
            continue
        g = p.grad.detach().double().reshape(-1)
        gen = torch.Generator().manual_seed(1000 + i)
        P = torch.randn(n_proj, g.numel(), generator=gen, dtype=torch.float64) / g.numel() ** 0.5
        out[name] = np.concatenate([(P @ g).numpy(), [g.norm().item(), g.abs().max().item()]])
    return out
