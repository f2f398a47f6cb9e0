"""Tree-training drivers on the B200 attention path (pure-attention models, and
hybrid models whose linear-attention layers run the tree GDN of ``ssm``).

Drop-ins for the reference drivers that call the hot path:

* ``partition_tree`` / ``SubtreePartition``   (tree_grad_hybrid.py:48-95)
* ``GatewayCache``                            (tree_grad_ckpt_opath.py:66-133)
* ``tree_grad_hybrid``                        (tree_grad_hybrid.py:434-539)
* ``tree_grad_ckpt_sequential``               (tree_grad_ckpt.py:39-107)
* ``make_tree_loss_fn``                       (tree_grad_hybrid.py:546-558)

Differences from the reference, all on the plumbing side of the op:

* no dense mask: each partition's keys carry row intervals (``TreeAttnMeta``)
  that reach the ``tree_sm100`` attention through ``model(..., tree_meta=)``;
* gateway keys inherit their parent partition's visibility
  (``gateway_mask="tree"``, the default).  ``gateway_mask="reference"``
  reproduces tree_grad_hybrid.py:207 exactly, where every key of the parent's
  own gateway is made visible again — with two cut levels that lets a DFS
  sibling of the parent partition leak into the child partition;
* gateway gradients are accumulated in fp32 on the device (the reference
  copies each one to host memory in fp32, tree_grad_hybrid.py:220-225);
* with linear-attention layers, each gateway also carries the recurrent state
  and conv context after the cut node (tree_grad_hybrid.py:232-250), and a
  partition that received them both injects them and captures its own
  (``ssm`` module docstring).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn.functional as F

from .attention import ATTN_IMPL_NAME, register_hf_attention, tree_mask_placeholder
from .packer import TreeNode, build_dfs_tree_info  # noqa: F401  (TreeNode re-export)
from .ce import fused_linear_cross_entropy
from .ssm import SSMPartitionState, has_ssm_layers, patch_ssm_layers


# ---------------------------------------------------------------------------
# partitioning
# ---------------------------------------------------------------------------

@dataclass
class SubtreePartition:
    entry_nodes: list
    dfs_nodes: list = field(default_factory=list)
    cut_node_set: set = field(default_factory=set)
    leaf_node_set: set = field(default_factory=set)
    parent: Optional["SubtreePartition"] = None
    parent_cut_node: object = None
    pos_offset: int = 0
    token_count: int = 0


def partition_tree(roots, max_tokens: int) -> List[SubtreePartition]:
    """Greedy DFS budget split with the reference's rules: a child that would
    push a non-empty partition past ``max_tokens`` is deferred, its parent
    becomes a cut node, every deferred child starts a new partition once the
    current one is complete, and every forest root starts its own partition."""
    parts: List[SubtreePartition] = []

    def build(entry, parent, cut_node):
        p = SubtreePartition(entry_nodes=list(entry), parent=parent, parent_cut_node=cut_node)
        parts.append(p)
        deferred = []

        def visit(node, is_entry):
            L = len(node.token_ids)
            if not is_entry and p.token_count > 0 and p.token_count + L > max_tokens:
                return False
            p.dfs_nodes.append(node)
            p.token_count += L
            for ch in node.children:
                if not visit(ch, False):
                    p.cut_node_set.add(id(node))
                    deferred.append((node, ch))
            if not node.children and id(node) not in p.cut_node_set:
                p.leaf_node_set.add(id(node))
            return True

        for r in entry:
            visit(r, True)
        for cn, ch in deferred:
            build([ch], p, cn)

    for r in roots:
        build([r], None, None)
    return parts


# ---------------------------------------------------------------------------
# gateway KV cache (HF Cache duck type)
# ---------------------------------------------------------------------------

class GatewayCache:
    """Concatenates a partition's gateway K/V (leaf tensors) in front of its
    own K/V in every attention layer and records the result for gradient
    chaining (tree_grad_ckpt_opath.py:66-133)."""

    def __init__(self, gate_kv: Dict[int, Tuple[torch.Tensor, torch.Tensor]]):
        self._gate_kv = gate_kv            # attention layer index -> gateway (K, V)
        self._full_kv: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        if layer_idx in self._gate_kv:
            gk, gv = self._gate_kv[layer_idx]
            full_k = torch.cat([gk, key_states], dim=-2)
            full_v = torch.cat([gv, value_states], dim=-2)
        else:
            full_k, full_v = key_states, value_states
        self._full_kv[layer_idx] = (full_k, full_v)
        return full_k, full_v

    def get_seq_length(self, layer_idx: Optional[int] = None) -> int:
        if layer_idx is None:               # any attention layer: all carry the same keys
            layer_idx = min(self._gate_kv) if self._gate_kv else 0
        if layer_idx in self._gate_kv:
            return self._gate_kv[layer_idx][0].shape[-2]
        return 0

    def get_mask_sizes(self, cache_position, layer_idx: Optional[int] = None):
        return self.get_seq_length(layer_idx) + cache_position.shape[0], 0

    def has_previous_state(self, layer_idx: Optional[int] = None) -> bool:
        """No decode-step recurrent state: hybrid models' mask code asks."""
        return False


@dataclass
class SubtreeGateway:
    key_gates: List[torch.Tensor]
    val_gates: List[torch.Tensor]
    raw_keys: List[torch.Tensor]
    raw_vals: List[torch.Tensor]
    acc_k: List[list]
    acc_v: List[list]
    past_len: int
    gw_lo: np.ndarray           # key intervals of the gateway keys (rows of the child)
    gw_visible: np.ndarray      # bool per gateway key
    pos_offset: int
    kv_layers: List[int] = field(default_factory=list)   # attention layer of each K/V entry
    # linear-attention layers: layer index -> (recurrent state, conv context)
    # leaves injected into the child, the tensors they were cut from, and the
    # fp32 accumulators of their gradients
    ssm_inject: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = field(default_factory=dict)
    ssm_raw: List[torch.Tensor] = field(default_factory=list)
    ssm_acc: List[list] = field(default_factory=list)


def _fp32_accumulator_hook(acc: list):
    """Sum the gradient reaching a gateway leaf in fp32 on its device and stop
    the 16-bit .grad accumulation (the reference does the sum on the host)."""
    def hook(g):
        g32 = g.detach().float()
        acc[0] = g32 if acc[0] is None else acc[0] + g32
        return torch.zeros_like(g)
    return hook


# ---------------------------------------------------------------------------
# one partition forward
# ---------------------------------------------------------------------------

def _partition_forest(p: SubtreePartition):
    """The partition's members as a forest of light nodes (reference copy order,
    tree_grad_hybrid.py:110-130) plus original-node bookkeeping."""
    members = {id(n) for n in p.dfs_nodes}

    class _N:
        __slots__ = ("token_ids", "children", "orig")

        def __init__(self, orig):
            self.orig = orig
            self.token_ids = orig.token_ids
            self.children = [_N(c) for c in orig.children if id(c) in members]

    return [_N(n) for n in p.entry_nodes if id(n) in members]


def _loss_leaf_spans(info, p: SubtreePartition):
    """(chunk, start, end) of the partition's loss leaves in DFS order."""
    out = []
    for c in info.leaf_chunk_ids_np.tolist():
        if id(info.nodes[c].orig) in p.leaf_node_set:
            s, e = info.chunk_bounds_np[c]
            out.append((c, int(s), int(e)))
    return out


def _subtree_forward(model, p: SubtreePartition, gw: Optional[SubtreeGateway], dev, gateway_mask,
                     leaf_logits_only: bool = False, cut_nodes=(), ssm_exact: bool = False,
                     fused_loss: Optional[TreeLeafLoss] = None):
    """Forward of one partition.  Returns (logits, info, full_kv, spans, ssm):
    with ``leaf_logits_only`` the LM head runs only on the loss leaves' tokens
    (HF ``logits_to_keep`` with an index tensor) and spans maps each loss leaf
    to its rows of the compact logits; otherwise logits cover every token and
    the spans are the leaves' own token ranges.  ``ssm`` holds the captured
    linear-attention states at ``cut_nodes`` (None without such layers).
    With ``fused_loss`` the first element is instead the partition's summed
    leaf loss, computed from the final hidden states by the fused LM-head
    cross-entropy (no logits), and spans is empty."""
    forest = _partition_forest(p)
    info = build_dfs_tree_info(forest, pos_offset=p.pos_offset)
    N = info.N
    past = gw.past_len if gw is not None else 0
    if gw is not None:
        vis = gw.gw_visible
        meta = info.attn_meta(np.zeros(past, np.int32), np.where(vis, N, 0).astype(np.int32))
    else:
        meta = info.attn_meta()
    ids = torch.as_tensor(info.dfs_token_ids_np, device=dev).unsqueeze(0)
    pos = torch.as_tensor(info.dfs_pos_ids_np.astype(np.int64), device=dev).unsqueeze(0)
    cache = GatewayCache({l: kv for l, kv in zip(gw.kv_layers, zip(gw.key_gates, gw.val_gates))}
                         if gw is not None else {})
    dtype = next(model.parameters()).dtype
    mask = tree_mask_placeholder(meta, dtype=dtype, device=dev)
    leaves = _loss_leaf_spans(info, p)
    kw = {}
    if fused_loss is not None:
        spans = []
    elif leaf_logits_only:
        idx = np.concatenate([np.arange(s, e) for _, s, e in leaves]) if leaves else \
            np.zeros(0, np.int64)
        kw["logits_to_keep"] = torch.as_tensor(idx, dtype=torch.long, device=dev)
        spans, off = [], 0
        for c, s, e in leaves:
            spans.append((c, off, off + (e - s)))
            off += e - s
    else:
        spans = leaves
    ssm = None
    net = _base_model(model) if fused_loss is not None else model
    args = dict(input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=cache,
                use_cache=True, tree_meta=meta, **kw)
    if has_ssm_layers(model):
        node_idx = {id(n.orig): i for i, n in enumerate(info.nodes)}
        ssm = SSMPartitionState(info.chunk_boundaries, info.chunk_parent_map,
                                inject=gw.ssm_inject if gw is not None else None,
                                capture_at=[node_idx[id(cn)] for cn in cut_nodes],
                                exact_inverse=ssm_exact)
        with patch_ssm_layers(model, ssm):
            out = net(**args)
    else:
        out = net(**args)
    full_kv = {l: cache._full_kv[l] for l in sorted(cache._full_kv)}
    if fused_loss is None:
        return out.logits, info, full_kv, spans, ssm
    return _fused_leaf_loss(model, out.last_hidden_state[0], info, leaves, fused_loss), info, \
        full_kv, spans, ssm


def _base_model(model):
    """The decoder stack under an HF causal-LM head (``model.model``)."""
    base = getattr(model, "model", None)
    if base is None or not hasattr(model, "lm_head"):
        raise ValueError("fused_ce needs an HF causal LM with .model and .lm_head")
    return base


def _fused_leaf_loss(model, hidden, info, leaves, loss: TreeLeafLoss) -> torch.Tensor:
    """sum over the partition's loss leaves of CE(leaf logits) / n_leaves from
    the final hidden states [N, H], without materialising the logits."""
    if not leaves:
        return hidden.sum() * 0.0
    idx = np.concatenate([np.arange(s, e) for _, s, e in leaves])
    labs, wts = [], []
    for c, s, e in leaves:
        lab = loss.labels(info.nodes[c]).to(hidden.device)
        labs.append(lab)
        wts.append(loss.token_weights(lab))
    h = hidden.index_select(0, torch.as_tensor(idx, dtype=torch.long, device=hidden.device))
    return fused_linear_cross_entropy(h, model.lm_head.weight, torch.cat(labs), torch.cat(wts),
                                      ignore_index=loss.ignore_index)


def _make_child_gateways(full_kv, info, p: SubtreePartition, gw: Optional[SubtreeGateway],
                         cut_nodes, gateway_mask: str, ssm=None) -> Dict[int, SubtreeGateway]:
    """Gateway of each cut node (tree_grad_hybrid.py:174-250): the parent's
    keys up to the end of the cut node, visible where they are the cut node's
    ancestors (or, for the parent's own gateway keys, where the parent saw
    them), and the depth-based position offset of the cut node's children."""
    node_idx = {id(n.orig): i for i, n in enumerate(info.nodes)}
    out = {}
    for cn in cut_nodes:
        total, vis, pos_off = gateway_visibility(
            info, node_idx[id(cn)], p.pos_offset, gw.gw_visible if gw is not None else None,
            gateway_mask)
        kg, vg, rk, rv, ak, av = [], [], [], [], [], []
        for fk, fv in full_kv.values():
            k_raw = fk[:, :, :total, :]
            v_raw = fv[:, :, :total, :]
            gk = k_raw.detach().requires_grad_(True)
            gv_ = v_raw.detach().requires_grad_(True)
            acc_k, acc_v = [None], [None]
            gk.register_hook(_fp32_accumulator_hook(acc_k))
            gv_.register_hook(_fp32_accumulator_hook(acc_v))
            kg.append(gk)
            vg.append(gv_)
            rk.append(k_raw)
            rv.append(v_raw)
            ak.append(acc_k)
            av.append(acc_v)
        g = SubtreeGateway(kg, vg, rk, rv, ak, av, total, np.zeros(total, np.int32), vis, pos_off,
                           kv_layers=list(full_kv))
        if ssm is not None:
            c = node_idx[id(cn)]
            for layer in sorted(ssm.rec):
                pair = []
                for raw in (ssm.rec[layer][c], ssm.conv[layer][c]):
                    leaf = raw.detach().requires_grad_(True)
                    acc = [None]
                    leaf.register_hook(_fp32_accumulator_hook(acc))
                    g.ssm_raw.append(raw)
                    g.ssm_acc.append(acc)
                    pair.append(leaf)
                g.ssm_inject[layer] = (pair[0], pair[1])
        out[id(cn)] = g
    return out


def gateway_visibility(info, c: int, pos_offset: int, parent_visible: Optional[np.ndarray],
                       gateway_mask: str = "tree"):
    """Gateway of cut node ``c`` of a partition (tree_grad_hybrid.py:198-209).

    Returns (total keys, bool visibility per key, pos_offset of the children).
    Keys are the partition's own gateway keys followed by its tokens up to the
    end of ``c``; a token key is visible iff it lies in an ancestor (or ``c``
    itself).  The partition's own gateway keys keep the visibility they had in
    the partition (``"tree"``) or are all made visible (``"reference"``, the
    reference's ``bias[:parent_past_len] = 0``)."""
    parent_past = 0 if parent_visible is None else len(parent_visible)
    bounds = info.chunk_bounds_np
    total = parent_past + int(bounds[c, 1])
    vis = np.zeros(total, bool)
    if parent_past:
        vis[:parent_past] = True if gateway_mask == "reference" else parent_visible
    a = c
    while a >= 0:
        s, e = bounds[a]
        vis[parent_past + s: parent_past + e] = True
        a = int(info.parents_np[a])
    # depth-based offset of the cut node's children (tree_grad_hybrid.py:202-204)
    pos_off = pos_offset + _depth_of(info, c) + int(bounds[c, 1] - bounds[c, 0])
    return total, vis, pos_off


def _depth_of(info, c) -> int:
    """Token count of c's ancestors (its depth offset), also for a 0-token node."""
    d = 0
    a = int(info.parents_np[c])
    while a >= 0:
        d += int(info.chunk_bounds_np[a, 1] - info.chunk_bounds_np[a, 0])
        a = int(info.parents_np[a])
    return d


def _gateway_roots(gw: SubtreeGateway):
    """(tensors, gradients) that chain the fp32 gateway gradients a partition
    received from its children into its own graph."""
    raws, grads = [], []
    for rk, rv, ak, av in zip(gw.raw_keys, gw.raw_vals, gw.acc_k, gw.acc_v):
        if ak[0] is not None:
            raws.append(rk)
            grads.append(ak[0].to(rk.dtype))
        if av[0] is not None:
            raws.append(rv)
            grads.append(av[0].to(rv.dtype))
    for raw, acc in zip(gw.ssm_raw, gw.ssm_acc):
        if acc[0] is not None and raw.requires_grad:
            raws.append(raw)
            grads.append(acc[0].to(raw.dtype))
    return raws, grads


def _chain_gateway_grads(gw: SubtreeGateway, retain_graph: bool) -> None:
    raws, grads = _gateway_roots(gw)
    if raws:
        torch.autograd.backward(raws, grads, retain_graph=retain_graph)


# ---------------------------------------------------------------------------
# drivers
# ---------------------------------------------------------------------------

def _ensure_tree_attention(model):
    register_hf_attention()
    cfg = model.config
    if getattr(cfg, "_attn_implementation", None) != ATTN_IMPL_NAME:
        cfg._attn_implementation = ATTN_IMPL_NAME


def tree_grad_hybrid(model, roots, leaf_loss_fn: Callable, max_tokens: int,
                     gateway_mask: str = "tree", backward: str = "fused",
                     leaf_logits_only: bool = True, ssm_exact_inverse: bool = False,
                     fused_ce: bool = False,
                     before_last_backward: Optional[Callable[[], None]] = None) -> torch.Tensor:
    """Partitioned tree forward/backward (tree_grad_hybrid.py:434-539):
    partitions run top-down, each with the gateway K/V of its cut node; then
    bottom-up, each partition backpropagates its leaf losses and chains the
    fp32 gateway gradients it received into its own graph, exactly once per
    gateway.  Accumulates parameter gradients into ``.grad``.

    ``backward="fused"`` takes each partition's leaf losses and gateway
    gradients through ONE autograd traversal of the partition graph;
    with ``fused_ce`` (a ``make_tree_loss_fn`` loss, ``backward="fused"``) the
    leaf losses come from the final hidden states through the chunked LM-head
    cross-entropy of ``ce`` and no logits are formed;
    ``"per_leaf"`` calls backward once per leaf loss and once per gateway with
    retain_graph, as the reference does (tree_grad_hybrid.py:521-539).  Both
    accumulate the same sum of gradients; every per-leaf call traverses the
    whole partition graph (each leaf's logits depend on every layer of the
    partition), so the fused form does 1/(leaves + gateways) of the backward
    work.

    ``leaf_logits_only`` runs the LM head only on loss-leaf tokens (the loss
    reads nothing else); ``leaf_loss_fn`` receives the same [1, len, vocab]
    slices either way.

    Models with linear-attention layers run them as tree GDN layers with SSM
    gateways; ``ssm_exact_inverse`` selects the exact delta-rule correction
    (T = (I - A)^-1) instead of the reference's truncated one.

    ``before_last_backward`` (``backward="fused"`` only) is called right before
    the last partition's backward traversal, the one that gives every
    parameter its final gradient of the step: ``dist.GradAverager.arm`` there
    lets the gradient all-reduce run during that traversal.

    Returns the summed leaf loss (a detached fp32 scalar on the device)."""
    if before_last_backward is not None and backward != "fused":
        raise ValueError("before_last_backward needs backward='fused' (one traversal per "
                         "partition)")
    if gateway_mask not in ("tree", "reference"):
        raise ValueError("gateway_mask must be 'tree' or 'reference'")
    if backward not in ("fused", "per_leaf"):
        raise ValueError("backward must be 'fused' or 'per_leaf'")
    if fused_ce and (backward != "fused" or not isinstance(leaf_loss_fn, TreeLeafLoss)):
        raise ValueError("fused_ce needs backward='fused' and a make_tree_loss_fn loss")
    _ensure_tree_attention(model)
    dev = next(model.parameters()).device
    parts = partition_tree(roots, max_tokens)
    children_of: Dict[int, List[Tuple[object, SubtreePartition]]] = {id(p): [] for p in parts}
    for p in parts:
        if p.parent is not None:
            children_of[id(p.parent)].append((p.parent_cut_node, p))
    gateways: Dict[int, SubtreeGateway] = {}
    fwd: Dict[int, tuple] = {}
    total = torch.zeros((), dtype=torch.float32, device=dev)
    for p in parts:
        gw = gateways.get(id(p))
        p.pos_offset = gw.pos_offset if gw is not None else 0
        seen, cuts = set(), []
        for cn, _ in children_of[id(p)]:
            if id(cn) not in seen:
                seen.add(id(cn))
                cuts.append(cn)
        logits, info, full_kv, spans, ssm = _subtree_forward(
            model, p, gw, dev, gateway_mask, leaf_logits_only, cuts, ssm_exact_inverse,
            leaf_loss_fn if fused_ce else None)
        fwd[id(p)] = (logits, info, spans)
        if cuts:
            child = _make_child_gateways(full_kv, info, p, gw, cuts, gateway_mask, ssm)
            for cn, cp in children_of[id(p)]:
                gateways[id(cp)] = child[id(cn)]
    for p in reversed(parts):
        logits, info, spans = fwd[id(p)]
        leaf_chunks = [(s, e, info.nodes[c].orig) for c, s, e in spans]
        uniq, seen = [], set()
        for cn, cp in children_of[id(p)]:
            g = gateways.get(id(cp))
            if g is not None and id(g) not in seen:
                seen.add(id(g))
                uniq.append(g)
        if backward == "fused":
            outs, grads = [], []
            if fused_ce:
                outs.append(logits)          # the partition's summed leaf loss
                grads.append(None)
            for s, e, orig in leaf_chunks:
                outs.append(leaf_loss_fn(logits[:, s:e, :], orig))
                grads.append(None)
            for o in outs:
                total += o.detach().float()
            for g in uniq:
                r, gr = _gateway_roots(g)
                outs.extend(r)
                grads.extend(gr)
            if before_last_backward is not None and p is parts[0]:
                before_last_backward()
            if outs:
                torch.autograd.backward(outs, [torch.ones_like(o) if g is None else g
                                               for o, g in zip(outs, grads)])
            del logits
            fwd.pop(id(p))
            continue
        remaining = len(leaf_chunks) + len(uniq)
        for s, e, orig in leaf_chunks:
            remaining -= 1
            l = leaf_loss_fn(logits[:, s:e, :], orig)
            total += l.detach().float()
            l.backward(retain_graph=remaining > 0)
        for g in uniq:
            remaining -= 1
            _chain_gateway_grads(g, retain_graph=remaining > 0)
    return total


def tree_grad_ckpt_sequential(model, roots, leaf_loss_fn: Callable,
                              ssm_exact_inverse: bool = False) -> None:
    """One packed forward over the whole forest, then per-leaf backward with
    retain_graph on all but the last leaf (tree_grad_ckpt.py:39-107).
    Linear-attention layers run as tree GDN layers (dfs_tree_forward.py:253-353)."""
    _ensure_tree_attention(model)
    dev = next(model.parameters()).device
    info = build_dfs_tree_info(roots)
    meta = info.attn_meta()
    ids = torch.as_tensor(info.dfs_token_ids_np, device=dev).unsqueeze(0)
    pos = torch.as_tensor(info.dfs_pos_ids_np.astype(np.int64), device=dev).unsqueeze(0)
    dtype = next(model.parameters()).dtype
    mask = tree_mask_placeholder(meta, dtype=dtype, device=dev)
    if has_ssm_layers(model):
        with patch_ssm_layers(model, SSMPartitionState(info.chunk_boundaries,
                                                        info.chunk_parent_map,
                                                        exact_inverse=ssm_exact_inverse)):
            logits = model(input_ids=ids, attention_mask=mask, position_ids=pos,
                           use_cache=False, tree_meta=meta).logits
    else:
        logits = model(input_ids=ids, attention_mask=mask, position_ids=pos, use_cache=False,
                       tree_meta=meta).logits
    leaves = info.leaf_chunk_ids_np.tolist()
    for i, c in enumerate(leaves):
        s, e = info.chunk_bounds_np[c]
        leaf_loss_fn(logits[:, int(s):int(e), :], info.nodes[c]).backward(
            retain_graph=i < len(leaves) - 1)


def checkpoint_mlps(model) -> int:
    """Recompute every decoder layer's MLP in the backward pass instead of
    saving its intermediates (torch.utils.checkpoint, non-reentrant).

    tree_grad_hybrid keeps the forward graph of every partition until the
    bottom-up backward (as the reference does, tree_grad_hybrid.py:466-539), so
    activation memory grows with the whole tree.  The MLP is the largest saved
    block of a Qwen3 layer (gate, up, activation and product, each
    tokens x intermediate) and touches no cache, so recomputing it changes no
    result.  Returns the number of MLPs wrapped."""
    import torch.utils.checkpoint as cp
    n = 0
    for layer in model.model.layers:
        mlp = getattr(layer, "mlp", None)
        if mlp is None or getattr(mlp, "_tt_checkpointed", False):
            continue
        fwd = mlp.forward

        def run(x, _f=fwd):
            if torch.is_grad_enabled():
                return cp.checkpoint(_f, x, use_reentrant=False)
            return _f(x)
        mlp.forward = run
        mlp._tt_checkpointed = True
        n += 1
    return n


class TreeLeafLoss:
    """Per-leaf CE / n_leaves (tree_grad_hybrid.py:546-558): called as
    ``loss_fn(logits [1, len, vocab], node)``.  The drivers' ``fused_ce``
    option recognises it and computes the same sum from the final hidden
    states with ``ce.fused_linear_cross_entropy`` instead of the logits."""

    def __init__(self, leaf_labels, leaf_nodes, n_leaves: int, ignore_index: int = -100):
        self.label_map = {id(n): lab for n, lab in zip(leaf_nodes, leaf_labels)}
        self.n_leaves = n_leaves
        self.ignore_index = ignore_index

    def labels(self, node) -> torch.Tensor:
        return self.label_map[id(getattr(node, "orig", node))]

    def __call__(self, logits, node):
        labels = self.labels(node).to(logits.device)
        return F.cross_entropy(logits[0], labels, ignore_index=self.ignore_index) / self.n_leaves

    def token_weights(self, labels: torch.Tensor) -> torch.Tensor:
        """w_t of the fused form: 1 / (valid tokens of the leaf * n_leaves), 0
        for ignored tokens (F.cross_entropy's mean over non-ignored targets)."""
        valid = labels != self.ignore_index
        n = int(valid.sum())
        return valid.float() / (max(n, 1) * self.n_leaves)


def make_tree_loss_fn(leaf_labels, leaf_nodes, n_leaves: int, ignore_index: int = -100):
    """Per-leaf CE / n_leaves (tree_grad_hybrid.py:546-558)."""
    return TreeLeafLoss(leaf_labels, leaf_nodes, n_leaves, ignore_index)
