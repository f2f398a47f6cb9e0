"""Benchmark config 1 (the 47-token forest, 2-layer Qwen3) on a B200: the drivers with the tree_sm100 attention vs a
flat per-path forward, gradients of a random-init 2-layer Qwen3 in fp32.

The flat per-path forward runs each root-to-leaf path on its own with stock
SDPA causal attention: the ground truth that the reference's tree training is
equivalent to (verify_hybrid.py:120-151 metric: per-parameter
max|dg| / max|g_ref|, max over parameters; bar 1e-4).
"""
import copy

import pytest
import torch
import torch.nn.functional as F

from tests.golden_util import Node, load
from tests.test_hybrid_cpu import f2_roots

import tree_training_b200 as tt
from tree_training_b200.hybrid import (make_tree_loss_fn, tree_grad_ckpt_sequential,
                                       tree_grad_hybrid)

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _model():
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=32000, hidden_size=256, intermediate_size=688,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=64, rope_theta=1e6, max_position_embeddings=4096,
                      tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    m = Qwen3ForCausalLM(cfg).to(DEV, torch.float32)
    m.train()
    return m


def _forest47():
    """verify_hybrid.py:38-60 topology with token ids uniform in [0, 32000)."""
    d = load("packer_forest47")
    g = torch.Generator().manual_seed(0)
    nodes, roots = [], []
    for L, p in zip(d["node_len"].tolist(), d["node_parent"].tolist()):
        n = Node(torch.randint(0, 32000, (L,), generator=g).tolist())
        nodes.append(n)
        (roots if p < 0 else nodes[p].children).append(n)
    return roots


def _paths(roots):
    out = []

    def walk(n, prefix):
        toks = prefix + list(n.token_ids)
        if not n.children:
            out.append((n, toks))
        for c in n.children:
            walk(c, toks)
    for r in roots:
        walk(r, [])
    return out


def _labels(leaves):
    g = torch.Generator().manual_seed(99)
    return [torch.randint(0, 32000, (len(n.token_ids),), generator=g) for n in leaves]


def _grads(model):
    return {n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None}


def flat_per_path_grads(model, roots):
    model.config._attn_implementation = "sdpa"
    model.zero_grad(set_to_none=True)
    paths = _paths(roots)
    leaves = [n for n, _ in paths]
    labels = _labels(leaves)
    for (leaf, toks), lab in zip(paths, labels):
        ids = torch.tensor([toks], device=DEV)
        logits = model(input_ids=ids, use_cache=False).logits
        L = len(leaf.token_ids)
        loss = F.cross_entropy(logits[0, -L:], lab.to(DEV)) / len(leaves)
        loss.backward()
    return _grads(model), leaves, labels


def max_rel(ref, new):
    worst = 0.0
    for n, g in ref.items():
        d = (g - new[n]).abs().max().item() / (g.abs().max().item() + 1e-12)
        worst = max(worst, d)
    return worst


@pytest.fixture(scope="module")
def setup():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    model = _model()
    roots = _forest47()
    ref, leaves, labels = flat_per_path_grads(model, roots)
    return model, roots, ref, leaves, labels


@pytest.mark.parametrize("backward,leaf_logits_only", [("fused", True), ("fused", False),
                                                       ("per_leaf", True)])
@pytest.mark.parametrize("max_tokens", [1000, 20, 10])
def test_tree_grad_hybrid_matches_flat_per_path(setup, max_tokens, backward, leaf_logits_only):
    model, roots, ref, leaves, labels = setup
    model.zero_grad(set_to_none=True)
    tree_grad_hybrid(model, roots, make_tree_loss_fn(labels, leaves, len(leaves)), max_tokens,
                     backward=backward, leaf_logits_only=leaf_logits_only)
    torch.cuda.synchronize()
    tt.check_device_status(DEV)
    assert max_rel(ref, _grads(model)) < 1e-4


@pytest.mark.parametrize("max_tokens", [1000, 10])
def test_tree_grad_hybrid_fused_ce_matches_flat_per_path(setup, max_tokens):
    """Leaf losses from the final hidden states through the chunked fused
    LM-head cross-entropy (no logits)."""
    model, roots, ref, leaves, labels = setup
    model.zero_grad(set_to_none=True)
    tree_grad_hybrid(model, roots, make_tree_loss_fn(labels, leaves, len(leaves)), max_tokens,
                     fused_ce=True)
    torch.cuda.synchronize()
    tt.check_device_status(DEV)
    assert max_rel(ref, _grads(model)) < 1e-4


def test_tree_grad_ckpt_sequential_matches_flat_per_path(setup):
    model, roots, ref, leaves, labels = setup
    model.zero_grad(set_to_none=True)
    tree_grad_ckpt_sequential(model, roots, make_tree_loss_fn(labels, leaves, len(leaves)))
    assert max_rel(ref, _grads(model)) < 1e-4


def test_reference_drivers_dense_mask_path(setup):
    """The attention also accepts the reference's dense additive mask (what its
    unmodified drivers pass): one packed forward through HF with that mask."""
    model, roots, ref, leaves, labels = setup
    model.zero_grad(set_to_none=True)
    tt.register_hf_attention()
    model.config._attn_implementation = tt.ATTN_IMPL_NAME
    info = tt.build_dfs_tree_info(roots)
    m = torch.full((1, 1, info.N, info.N), float("-inf"), device=DEV)
    m[0, 0][info.attn_mask_bool.to(DEV)] = 0.0
    logits = model(input_ids=torch.as_tensor(info.dfs_token_ids_np, device=DEV)[None],
                   attention_mask=m,
                   position_ids=torch.as_tensor(info.dfs_pos_ids_np, device=DEV).long()[None],
                   use_cache=False).logits
    fn = make_tree_loss_fn(labels, leaves, len(leaves))
    total = 0
    for c in info.leaf_chunk_ids:
        s, e = info.chunk_boundaries[c]
        total = total + fn(logits[:, s:e], info.nodes[c])
    total.backward()
    assert max_rel(ref, _grads(model)) < 1e-4


def test_two_level_gateway_tree_mode_is_exact_reference_mode_is_not():
    """Two cut levels (partitions {R,A,B}, {C,D}, {E}): the default gateway
    masking equals the per-path result; the reference's bias rule lets the
    DFS sibling A leak into E's attention."""
    torch.backends.cuda.matmul.allow_tf32 = False
    model = _model()
    roots = f2_roots()
    ref, leaves, labels = flat_per_path_grads(model, roots)
    fn = make_tree_loss_fn(labels, leaves, len(leaves))
    model.zero_grad(set_to_none=True)
    tree_grad_hybrid(model, roots, fn, 7, gateway_mask="tree")
    assert max_rel(ref, _grads(model)) < 1e-4
    model.zero_grad(set_to_none=True)
    tree_grad_hybrid(model, roots, fn, 7, gateway_mask="reference")
    assert max_rel(ref, _grads(model)) > 1e-3
