#!/usr/bin/env python3
"""Generate golden vectors by running the reference implementation itself.

Run once, in a container that has the reference checkout (path given by
``--ref``); the outputs (small ``.npz`` files next to this script) are
committed and the tests only read those files.  Nothing here is needed at
test time.

    python tests/golden/make_golden.py --ref <path-to-tree-training-checkout>

What is captured (all seeded, all small):
  * packer_*.npz     build_dfs_tree_info (dfs_tree_forward.py:91-184)
  * partition_*.npz  partition_tree + _dfs_info_for_partition +
                     _make_child_gateways (tree_grad_hybrid.py:60-250)
  * attn_*.npz       HF sdpa_attention_forward with the reference's dense
                     additive mask, forward + autograd backward
  * gdn_*.npz        torch_chunk_gated_delta_rule_tree_varlen fwd + autograd
                     (tree_dfs_ssm.py:38-156)
  * conv_*.npz       _tree_correct_conv_varlen fwd + autograd
                     (tree_dfs_ssm.py:285-348)
  * ref_driver_calls.npz  every attention call tree_grad_hybrid
                     (tree_grad_hybrid.py:434-539) and dfs_tree_forward
                     (dfs_tree_forward.py:513-576) make on the config-1 model,
                     and tree_grad_hybrid's gradient fingerprints
"""
import argparse
import os
import random
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def forest47(TreeNode, seed=42, vocab=32000):
    """verify_hybrid.py:38-60 topology, token ids drawn the same way."""
    torch.manual_seed(seed)
    V = min(vocab - 1, 1000)

    def rnd(n):
        return torch.randint(1, V, (n,)).tolist()

    root_a = TreeNode(rnd(3))
    b_left = root_a.add_child(rnd(4))
    c_left = b_left.add_child(rnd(3))
    d_left = c_left.add_child(rnd(4))
    d_left.add_child(rnd(5))
    d_left.add_child(rnd(3))
    f_node = c_left.add_child(rnd(3))
    f_node.add_child(rnd(4))
    root_b2 = TreeNode(rnd(4))
    c2 = root_b2.add_child(rnd(3))
    c2.add_child(rnd(4))
    x = root_b2.add_child(rnd(3))
    x.add_child(rnd(4))
    return [root_a, root_b2]


def random_forest(TreeNode, rng, n_roots, max_depth, branch, len_lo, len_hi, vocab=1000):
    def make(depth):
        n = TreeNode([rng.randrange(vocab) for _ in range(rng.randint(len_lo, len_hi))])
        if depth < max_depth:
            for _ in range(rng.randint(*branch)):
                n.children.append(make(depth + 1))
        return n
    return [make(0) for _ in range(n_roots)]


def chain_forest(TreeNode, lens):
    root = TreeNode(list(range(lens[0])))
    cur = root
    for i, L in enumerate(lens[1:]):
        cur = cur.add_child(list(range(100 * (i + 1), 100 * (i + 1) + L)))
    return [root]


def flatten_forest(roots):
    """Pre-order (len, parent, tokens) arrays describing a forest."""
    lens, par, toks = [], [], []
    stack = [(r, -1) for r in reversed(roots)]
    while stack:
        n, p = stack.pop()
        me = len(lens)
        lens.append(len(n.token_ids))
        par.append(p)
        toks.extend(n.token_ids)
        for ch in reversed(n.children):
            stack.append((ch, me))
    return np.array(lens, np.int64), np.array(par, np.int64), np.array(toks, np.int64)


def save_packer(name, roots, dft):
    info = dft.build_dfs_tree_info(roots)
    lens, par, toks = flatten_forest(roots)
    np.savez_compressed(
        os.path.join(HERE, f"packer_{name}.npz"),
        node_len=lens, node_parent=par, node_tokens=toks,
        dfs_token_ids=np.array(info.dfs_token_ids, np.int64),
        dfs_pos_ids=np.array(info.dfs_pos_ids, np.int64),
        chunk_boundaries=np.array(info.chunk_boundaries, np.int64).reshape(-1, 2),
        chunk_parent_map=np.array(info.chunk_parent_map, np.int64),
        leaf_chunk_ids=np.array(info.leaf_chunk_ids, np.int64),
        attn_mask_bool=np.packbits(info.attn_mask_bool.numpy(), axis=None),
        N=info.N, n_chunks=info.n_chunks)


def save_partition(name, roots, tgh, max_tokens):
    """Capture, per partition in the reference's order: its DFS info,
    pos_offset, and the gateway (past_len, bias) that feeds it."""
    parts = tgh.partition_tree(roots, max_tokens)
    children_of = {id(p): [] for p in parts}
    for p in parts:
        if p.parent is not None:
            children_of[id(p.parent)].append((p.parent_cut_node, p))
    gws = {}
    out = {"n_parts": len(parts), "max_tokens": max_tokens}
    order = {id(p): i for i, p in enumerate(parts)}
    for i, p in enumerate(parts):
        gw = gws.get(id(p))
        p.pos_offset = gw.pos_offset if gw is not None else 0
        (info, s_map, e_map, par_map, ci_map, cto) = tgh._dfs_info_for_partition(p)
        out[f"p{i}_token_count"] = p.token_count
        out[f"p{i}_parent"] = -1 if p.parent is None else order[id(p.parent)]
        out[f"p{i}_pos_offset"] = p.pos_offset
        out[f"p{i}_dfs_token_ids"] = np.array(info.dfs_token_ids, np.int64)
        out[f"p{i}_dfs_pos_ids"] = np.array(info.dfs_pos_ids, np.int64)
        out[f"p{i}_chunk_boundaries"] = np.array(info.chunk_boundaries, np.int64).reshape(-1, 2)
        out[f"p{i}_chunk_parent_map"] = np.array(info.chunk_parent_map, np.int64)
        leaf_mask = []
        for j, lc in enumerate(info.leaf_chunk_ids):
            orig = cto[id(info.leaf_nodes[j])]
            leaf_mask.append(1 if id(orig) in p.leaf_node_set else 0)
        out[f"p{i}_leaf_chunk_ids"] = np.array(info.leaf_chunk_ids, np.int64)
        out[f"p{i}_leaf_is_loss"] = np.array(leaf_mask, np.int64)
        out[f"p{i}_past_len"] = gw.past_len if gw is not None else 0
        out[f"p{i}_gateway_bias"] = (gw.attn_bias.numpy().astype(np.float64)
                                     if gw is not None else np.zeros(0))
        cuts = []
        for cn, _ in children_of[id(p)]:
            if id(cn) not in [id(c) for c in cuts]:
                cuts.append(cn)
        if cuts:
            fake_kv = [(torch.zeros(1, 1, (gw.past_len if gw else 0) + info.N, 1),
                        torch.zeros(1, 1, (gw.past_len if gw else 0) + info.N, 1))]
            child_gws = tgh._make_child_gateways(
                full_kv=fake_kv, dfs_info=info, orig_id_to_start=s_map,
                orig_id_to_end=e_map, orig_id_to_par=par_map,
                orig_id_to_chunk_idx=ci_map, cut_nodes=cuts,
                parent_pos_offset=p.pos_offset,
                parent_past_len=gw.past_len if gw is not None else 0,
                ssm_rec_captured={}, ssm_conv_captured={})
            for cn, child_p in children_of[id(p)]:
                gws[id(child_p)] = child_gws[id(cn)]
    np.savez_compressed(os.path.join(HERE, f"partition_{name}_{max_tokens}.npz"), **out)


def save_attention(name, roots, dft, hq, hkv, d, dtype, seed, past=None):
    """Reference attention: dense additive mask (dfs_tree_forward.py:548-550 /
    tree_grad_hybrid.py:313-317) fed to transformers' sdpa_attention_forward."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    info = dft.build_dfs_tree_info(roots)
    N = info.N
    P = 0 if past is None else len(past)
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(1, hq, N, d, generator=g) * 0.5).to(dtype).requires_grad_(True)
    k = (torch.randn(1, hkv, P + N, d, generator=g) * 0.5).to(dtype).requires_grad_(True)
    v = (torch.randn(1, hkv, P + N, d, generator=g) * 0.5).to(dtype).requires_grad_(True)
    do = (torch.randn(1, N, hq, d, generator=g) * 0.5).to(dtype)
    attn = torch.full((1, 1, N, P + N), float("-inf"), dtype=dtype)
    if P:
        attn[0, 0, :, :P] = torch.tensor(past, dtype=dtype)
    rows, cols = info.attn_mask_bool.nonzero(as_tuple=True)
    attn[0, 0, rows, cols + P] = 0.0

    class M(torch.nn.Module):
        num_key_value_groups = hq // hkv
        is_causal = True
    out, _ = sdpa_attention_forward(M(), q, k, v, attn, dropout=0.0, scaling=d ** -0.5)
    out.backward(do)
    np.savez_compressed(
        os.path.join(HERE, f"attn_{name}.npz"),
        q=q.detach().double().numpy(), k=k.detach().double().numpy(),
        v=v.detach().double().numpy(), dout=do.double().numpy(),
        allowed_bits=np.packbits((attn[0, 0] == 0).numpy(), axis=None),
        n_rows=N, n_cols=P + N,
        chunk_boundaries=np.array(info.chunk_boundaries, np.int64).reshape(-1, 2),
        chunk_parent_map=np.array(info.chunk_parent_map, np.int64),
        past=np.zeros(0) if past is None else np.array(past, np.float64),
        out=out.detach().double().numpy(), dq=q.grad.double().numpy(),
        dk=k.grad.double().numpy(), dv=v.grad.double().numpy(),
        scale=d ** -0.5, dtype=str(dtype))


def save_gdn(name, tds, bounds, parents, B, Hk, H, dk, dv, seed, l2norm, init,
             final_state=False):
    g_ = torch.Generator().manual_seed(seed)
    S = bounds[-1][1]
    q = torch.randn(B, S, Hk, dk, generator=g_, dtype=torch.float64)
    k = torch.randn(B, S, Hk, dk, generator=g_, dtype=torch.float64)
    if not l2norm:
        q = q / q.norm(dim=-1, keepdim=True)
        k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(B, S, H, dv, generator=g_, dtype=torch.float64)
    gg = torch.nn.functional.logsigmoid(torch.randn(B, S, H, generator=g_, dtype=torch.float64))
    bt = torch.sigmoid(torch.randn(B, S, H, generator=g_, dtype=torch.float64))
    s0 = (torch.randn(B, H, dk, dv, generator=g_, dtype=torch.float64) * 0.1) if init else None
    do = torch.randn(B, S, H, dv, generator=g_, dtype=torch.float64)
    ds = torch.randn(B, H, dk, dv, generator=g_, dtype=torch.float64) if final_state else None
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, gg, bt)]
    s0l = s0.clone().requires_grad_(True) if s0 is not None else None
    qq, kk = leaves[0], leaves[1]
    if H != Hk:
        qq = qq.repeat_interleave(H // Hk, dim=2)
        kk = kk.repeat_interleave(H // Hk, dim=2)
    out, last = tds.torch_chunk_gated_delta_rule_tree_varlen(
        qq, kk, leaves[2], leaves[3], leaves[4], bounds, parents,
        initial_state=s0l, output_final_state=final_state,
        use_qk_l2norm_in_kernel=l2norm)
    loss = (out.double() * do).sum()
    if final_state:
        loss = loss + (last.double() * ds).sum()
    loss.backward()
    np.savez_compressed(
        os.path.join(HERE, f"gdn_{name}.npz"),
        q=q.numpy(), k=k.numpy(), v=v.numpy(), g=gg.numpy(), beta=bt.numpy(),
        init=np.zeros(0) if s0 is None else s0.numpy(),
        dout=do.numpy(), dlast=np.zeros(0) if ds is None else ds.numpy(),
        chunk_boundaries=np.array(bounds, np.int64).reshape(-1, 2),
        chunk_parent_map=np.array(parents, np.int64), l2norm=int(l2norm),
        out=out.detach().double().numpy(),
        last=np.zeros(0) if last is None else last.detach().double().numpy(),
        dq=leaves[0].grad.numpy(), dk=leaves[1].grad.numpy(), dv=leaves[2].grad.numpy(),
        dg=leaves[3].grad.numpy(), dbeta=leaves[4].grad.numpy(),
        dinit=np.zeros(0) if s0l is None else s0l.grad.numpy())


def save_conv(name, tds, bounds, parents, B, C, K, seed):
    g_ = torch.Generator().manual_seed(seed)
    S = bounds[-1][1]

    class Shim:
        pass
    ssm = Shim()
    ssm.conv_kernel_size = K
    ssm.conv1d = torch.nn.Conv1d(C, C, K, groups=C, padding=K - 1, bias=False).double()
    with torch.no_grad():
        ssm.conv1d.weight.copy_(torch.randn(C, 1, K, generator=g_, dtype=torch.float64) * 0.5)
    ssm.causal_conv1d_fn = None
    ssm.activation = "silu"
    x = torch.randn(B, C, S, generator=g_, dtype=torch.float64).requires_grad_(True)
    do = torch.randn(B, C, S, generator=g_, dtype=torch.float64)
    y = tds._tree_correct_conv_varlen(ssm, x, bounds, parents)
    y.backward(do)
    np.savez_compressed(
        os.path.join(HERE, f"conv_{name}.npz"),
        x=x.detach().numpy(), weight=ssm.conv1d.weight.detach()[:, 0].numpy(),
        dout=do.numpy(), out=y.detach().numpy(), dx=x.grad.numpy(),
        dweight=ssm.conv1d.weight.grad[:, 0].numpy(),
        chunk_boundaries=np.array(bounds, np.int64).reshape(-1, 2),
        chunk_parent_map=np.array(parents, np.int64))


def save_driver_calls(dft, tgh):
    """The reference's unmodified drivers on the config-1 model with a
    recording attention function registered through transformers'
    AttentionInterface (the same hook tree_sm100 uses): every attention call's
    inputs exactly as the drivers pass them (dense additive mask, gateway K/V
    prefix from GatewayCache, scaling), and the parameter-gradient fingerprints
    of tree_grad_hybrid at max_tokens 1000 / 20 / 10.  SDPA computes each call."""
    from transformers import AttentionInterface
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    sys.path.insert(0, os.path.dirname(HERE))
    from golden_util import config1_forest, config1_model, grad_projections
    calls = []

    def recorder(module, query, key, value, attention_mask, dropout=0.0, scaling=None,
                 sliding_window=None, **kwargs):
        calls.append(dict(q=query.detach().numpy().copy(), k=key.detach().numpy().copy(),
                          v=value.detach().numpy().copy(),
                          mask=attention_mask.detach().numpy().copy(),
                          scaling=float(scaling), groups=int(module.num_key_value_groups),
                          layer=int(module.layer_idx)))
        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                      scaling=scaling, sliding_window=sliding_window, **kwargs)

    AttentionInterface.register("tt_recorder", recorder)
    model = config1_model()
    model.config._attn_implementation = "tt_recorder"
    roots, leaves, labels = config1_forest(dft.TreeNode)
    out = {}
    runs = [("hybrid_%d" % mt, mt) for mt in (1000, 20, 10)] + [("dfs_forward", None)]
    for tag, mt in runs:
        calls.clear()
        model.zero_grad(set_to_none=True)
        if mt is not None:
            tgh.tree_grad_hybrid(model, roots=roots, max_tokens=mt,
                                 leaf_loss_fn=tgh.make_tree_loss_fn(labels, leaves, len(leaves)))
            for name, v in grad_projections(model).items():
                out[f"{tag}/grad/{name}"] = v
        else:
            with torch.no_grad():
                dft.dfs_tree_forward(model, roots)
        out[f"{tag}/n_calls"] = np.array(len(calls))
        for i, c in enumerate(calls):
            for key in ("q", "k", "v", "mask"):
                out[f"{tag}/{i}/{key}"] = c[key]
            out[f"{tag}/{i}/meta"] = np.array([c["scaling"], c["groups"], c["layer"]])
    np.savez_compressed(os.path.join(HERE, "ref_driver_calls.npz"), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    import dfs_tree_forward as dft
    import tree_dfs_ssm as tds
    import tree_grad_hybrid as tgh
    TreeNode = dft.TreeNode
    torch.set_num_threads(8)

    # ---- packer ----
    save_packer("forest47", forest47(TreeNode), dft)
    rng = random.Random(1234)
    save_packer("rand_a", random_forest(TreeNode, rng, 3, 4, (0, 3), 1, 9), dft)
    save_packer("rand_b", random_forest(TreeNode, rng, 1, 6, (1, 3), 1, 5), dft)
    save_packer("single", [TreeNode([5, 6, 7])], dft)
    save_packer("one_token_nodes", random_forest(TreeNode, rng, 2, 5, (1, 2), 1, 1), dft)
    save_packer("chain", chain_forest(TreeNode, [7, 1, 130, 3, 64, 9]), dft)
    r = TreeNode([1, 2])
    r.add_child([])                      # empty node: reference keeps a (s, s) chunk
    r.add_child([3]).add_child([4, 5])
    save_packer("empty_node", [r], dft)

    # ---- partitions ----
    for mt in (1000, 20, 10):
        save_partition("forest47", forest47(TreeNode), tgh, mt)
    for mt in (12, 6):
        save_partition("rand_a", random_forest(TreeNode, random.Random(1234), 3, 4, (0, 3), 1, 9),
                       tgh, mt)
    # two cut levels with a DFS sibling in the middle partition: the input of
    # the reference's multi-level gateway bias (tree_grad_hybrid.py:207)
    root = TreeNode([1, 2, 3])
    a1 = root.add_child([4, 5, 6])
    root.add_child([7, 8])
    b1 = a1.add_child([9, 10, 11])
    a1.add_child([12, 13])
    b1.add_child([14, 15, 16]).add_child([17])
    save_partition("twolevel", [root], tgh, 7)

    # ---- attention ----
    save_attention("forest47_f64", forest47(TreeNode), dft, 4, 2, 64, torch.float64, 7)
    save_attention("forest47_f32", forest47(TreeNode), dft, 4, 2, 64, torch.float32, 7)
    big = random_forest(TreeNode, random.Random(99), 1, 3, (2, 3), 8, 40)
    save_attention("rand_f64", big, dft, 8, 2, 32, torch.float64, 11)
    past = [0.0] * 5 + [float("-inf")] * 4 + [0.0] * 3
    save_attention("gateway_f64", forest47(TreeNode)[1:], dft, 4, 2, 64, torch.float64, 13,
                   past=past)

    # ---- GDN ----
    info = dft.build_dfs_tree_info(random_forest(TreeNode, random.Random(5), 1, 3, (1, 3), 3, 24))
    save_gdn("tree_l2", tds, info.chunk_boundaries, info.chunk_parent_map,
             1, 2, 4, 16, 16, 21, True, False)
    save_gdn("tree_init_final", tds, info.chunk_boundaries, info.chunk_parent_map,
             2, 2, 2, 8, 16, 22, False, True, final_state=True)
    info47 = dft.build_dfs_tree_info(forest47(TreeNode))
    save_gdn("forest47", tds, info47.chunk_boundaries, info47.chunk_parent_map,
             1, 1, 2, 32, 32, 23, True, False)

    # ---- conv ----
    save_conv("tree", tds, info.chunk_boundaries, info.chunk_parent_map, 1, 6, 4, 31)
    ch = dft.build_dfs_tree_info(random_forest(TreeNode, random.Random(8), 2, 4, (1, 3), 1, 3))
    save_conv("short_nodes", tds, ch.chunk_boundaries, ch.chunk_parent_map, 2, 3, 4, 32)
    # ---- the reference's drivers with a recording attention function ----
    save_driver_calls(dft, tgh)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
