"""numpy restatement of the Tree Training hot path (CPU oracle).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py``; never by the product package.

Pinned against golden vectors that ``tests/golden/make_golden.py`` produced by
running the reference's own Python code (``tests/test_oracle_golden.py``).

Reference citations are ``file:line`` inside Jinghui-Wang/tree-training.
Float work runs in float64 so that the oracle is tighter than every tolerance
the GPU tests apply.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


# ---------------------------------------------------------------------------
# Forest packing  (dfs_tree_forward.py:91-184)
# ---------------------------------------------------------------------------

@dataclass
class OracleDFSInfo:
    dfs_token_ids: List[int]
    dfs_pos_ids: List[int]
    chunk_boundaries: List[Tuple[int, int]]
    chunk_parent_map: List[int]
    leaf_chunk_ids: List[int]
    leaf_nodes: list
    N: int
    n_chunks: int

    def attn_mask_bool(self) -> np.ndarray:
        """Dense [N, N] mask: token i sees token j iff j lies in an ancestor
        chunk of i, or in i's own chunk with j <= i (dfs_tree_forward.py:157-172)."""
        N = self.N
        m = np.zeros((N, N), dtype=bool)
        anc: List[List[int]] = []
        for c, p in enumerate(self.chunk_parent_map):           # :144-155
            anc.append([c] if p == -1 else anc[p] + [c])
        for c, (cs, ce) in enumerate(self.chunk_boundaries):
            for a in anc[c]:
                a_s, a_e = self.chunk_boundaries[a]
                if a == c:
                    for i in range(cs, ce):
                        m[i, cs:i + 1] = True
                else:
                    m[cs:ce, a_s:a_e] = True
        return m


def build_dfs_tree_info(roots: Sequence) -> OracleDFSInfo:
    """Pre-order DFS of a forest (dfs_tree_forward.py:91-139).

    Position ids are depth based: token j of chunk c gets the total token count
    of c's ancestor chunks plus j (:125-126).  Works on any node object with
    ``token_ids`` and ``children`` attributes.
    """
    ids: List[int] = []
    pos: List[int] = []
    bounds: List[Tuple[int, int]] = []
    parents: List[int] = []
    leaves: List[int] = []
    leaf_nodes: list = []
    # explicit stack instead of recursion: (node, parent_chunk, depth_offset)
    stack = [(r, -1, 0) for r in reversed(list(roots))]
    while stack:
        node, par, off = stack.pop()
        c = len(parents)
        s = len(ids)
        L = len(node.token_ids)
        ids.extend(int(t) for t in node.token_ids)
        pos.extend(range(off, off + L))
        parents.append(par)
        bounds.append((s, s + L))
        if len(node.children) == 0:
            leaves.append(c)
            leaf_nodes.append(node)
        else:
            for ch in reversed(node.children):
                stack.append((ch, c, off + L))
    return OracleDFSInfo(ids, pos, bounds, parents, leaves, leaf_nodes,
                         len(ids), len(parents))


def subtree_token_end(bounds: Sequence[Tuple[int, int]],
                      parents: Sequence[int]) -> np.ndarray:
    """One past the last token of each chunk's subtree.  In pre-order a
    subtree is a contiguous token range starting at the chunk itself."""
    n = len(bounds)
    end = np.array([e for (_, e) in bounds], dtype=np.int64)
    for c in range(n - 1, -1, -1):
        p = parents[c]
        if p >= 0:
            end[p] = max(end[p], end[c])
    return end


def key_intervals(bounds, parents, N: int) -> Tuple[np.ndarray, np.ndarray]:
    """Column form of the dense mask of dfs_tree_forward.py:157-172: key j is
    visible to query rows [lo[j], hi[j]) with lo = j and hi = the end of the
    subtree of j's chunk."""
    sub_end = subtree_token_end(bounds, parents)
    lo = np.arange(N, dtype=np.int64)
    hi = np.zeros(N, dtype=np.int64)
    for c, (s, e) in enumerate(bounds):
        hi[s:e] = sub_end[c]
    return lo, hi


def mask_from_intervals(lo: np.ndarray, hi: np.ndarray, n_rows: int) -> np.ndarray:
    rows = np.arange(n_rows)[:, None]
    return (rows >= lo[None, :]) & (rows < hi[None, :])


def intervals_from_mask(allowed: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Inverse of :func:`mask_from_intervals`; raises if a column is not one
    contiguous run of rows."""
    nq, nk = allowed.shape
    lo = np.zeros(nk, dtype=np.int64)
    hi = np.zeros(nk, dtype=np.int64)
    for j in range(nk):
        r = np.nonzero(allowed[:, j])[0]
        if r.size == 0:
            continue
        if r[-1] - r[0] + 1 != r.size:
            raise ValueError(f"column {j} is not an interval")
        lo[j], hi[j] = r[0], r[-1] + 1
    return lo, hi


# ---------------------------------------------------------------------------
# Partitioning and gateways  (tree_grad_hybrid.py:60-95, 102-153, 198-209)
# ---------------------------------------------------------------------------

@dataclass
class OraclePartition:
    entry_nodes: list
    parent: Optional[int]
    parent_cut_node: object
    dfs_nodes: list = field(default_factory=list)
    cut_node_ids: set = field(default_factory=set)
    leaf_node_ids: set = field(default_factory=set)
    token_count: int = 0
    pos_offset: int = 0


def partition_tree(roots: Sequence, max_tokens: int) -> List[OraclePartition]:
    """Greedy DFS budget split (tree_grad_hybrid.py:60-95).

    A child is deferred when the partition already holds tokens and adding it
    would pass ``max_tokens`` (:76-77); its parent becomes a cut node (:81-83)
    and each deferred child starts a new partition after the current one is
    finished (:90-91).  Every forest root starts its own partition (:93-94).
    """
    parts: List[OraclePartition] = []

    def build(entry, parent_idx, cut_node):
        p = OraclePartition(entry_nodes=list(entry), parent=parent_idx,
                            parent_cut_node=cut_node)
        my = len(parts)
        parts.append(p)
        deferred = []

        def dfs(node, is_entry):
            L = len(node.token_ids)
            if not is_entry and p.token_count > 0 and p.token_count + L > max_tokens:
                return False
            p.dfs_nodes.append(node)
            p.token_count += L
            for ch in node.children:
                if not dfs(ch, False):
                    p.cut_node_ids.add(id(node))
                    deferred.append((node, ch))
            if not node.children and id(node) not in p.cut_node_ids:
                p.leaf_node_ids.add(id(node))
            return True

        for r in entry:
            dfs(r, True)
        for cn, ch in deferred:
            build([ch], my, cn)

    for r in roots:
        build([r], None, None)
    return parts


def partition_local_forest(part: OraclePartition):
    """The partition's nodes as a forest restricted to its own members, in the
    reference's copy order (tree_grad_hybrid.py:110-130).  Returns a list of
    (node, [children...]) structures via light-weight shims."""
    members = {id(n) for n in part.dfs_nodes}

    class _Shim:
        __slots__ = ("token_ids", "children", "orig")

        def __init__(self, orig):
            self.orig = orig
            self.token_ids = list(orig.token_ids)
            self.children = [_Shim(c) for c in orig.children if id(c) in members]

    return [_Shim(n) for n in part.entry_nodes if id(n) in members]


def gateway_for_cut(info: OracleDFSInfo, shim_roots, cut_node, parent_pos_offset: int,
                    parent_past_len: int):
    """Gateway length, ancestor bias and depth-based position offset of one
    cut node (tree_grad_hybrid.py:190-209).  ``bias[:parent_past_len] = 0``
    is kept exactly as the reference writes it (:207)."""
    start, end, par = {}, {}, {}
    ci = [0]

    def walk(s, par_id):                                       # :138-150
        idx = ci[0]
        ci[0] += 1
        b = info.chunk_boundaries[idx]
        start[id(s.orig)], end[id(s.orig)] = b
        par[id(s.orig)] = par_id
        for ch in s.children:
            walk(ch, id(s.orig))

    for r in shim_roots:
        walk(r, -1)
    cut_end = end[id(cut_node)]
    total = parent_past_len + cut_end                           # :199-200
    cn_start = start[id(cut_node)]
    pos_off = parent_pos_offset + info.dfs_pos_ids[cn_start] + len(cut_node.token_ids)
    bias = np.full(total, -np.inf)
    bias[:parent_past_len] = 0.0                                # :207
    nid = id(cut_node)
    while nid != -1 and nid in start:                           # :190-196
        bias[parent_past_len + start[nid]: parent_past_len + end[nid]] = 0.0
        nid = par.get(nid, -1)
    return total, bias, pos_off


# ---------------------------------------------------------------------------
# Attention with the additive tree mask
#   (dfs_tree_forward.py:548-560; tree_grad_hybrid.py:312-317 build the mask,
#    transformers integrations/sdpa_attention.py:40-104 evaluates
#    softmax(Q K^T * scale + M) V with GQA by head repetition)
# ---------------------------------------------------------------------------

def attention_fwd(q, k, v, allowed, scale):
    """q [Hq, Nq, D], k/v [Hkv, Nk, D], allowed bool [Nq, Nk].
    Returns out [Hq, Nq, D] and natural-log LSE [Hq, Nq] (float64)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    hq, hkv = q.shape[0], k.shape[0]
    rep = hq // hkv
    kk = np.repeat(k, rep, axis=0)
    vv = np.repeat(v, rep, axis=0)
    s = np.einsum("hid,hjd->hij", q, kk) * scale
    s = np.where(allowed[None], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    out = np.einsum("hij,hjd->hid", p / l, vv)
    lse = (m + np.log(l))[..., 0]
    return out, lse


def attention_bwd(q, k, v, allowed, scale, dout):
    """Analytic gradients of :func:`attention_fwd` (float64)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    do = np.asarray(dout, np.float64)
    hq, hkv = q.shape[0], k.shape[0]
    rep = hq // hkv
    kk = np.repeat(k, rep, axis=0)
    vv = np.repeat(v, rep, axis=0)
    s = np.einsum("hid,hjd->hij", q, kk) * scale
    s = np.where(allowed[None], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    p /= p.sum(axis=-1, keepdims=True)
    dvv = np.einsum("hij,hid->hjd", p, do)
    dp = np.einsum("hid,hjd->hij", do, vv)
    ds = p * (dp - (dp * p).sum(axis=-1, keepdims=True))
    dq = np.einsum("hij,hjd->hid", ds, kk) * scale
    dkk = np.einsum("hij,hid->hjd", ds, q) * scale
    dk = dkk.reshape(hkv, rep, *dkk.shape[1:]).sum(axis=1)
    dv = dvv.reshape(hkv, rep, *dvv.shape[1:]).sum(axis=1)
    return dq, dk, dv


# ---------------------------------------------------------------------------
# Tree gated delta rule  (tree_dfs_ssm.py:38-156)
# ---------------------------------------------------------------------------

def _l2norm(x, eps=1e-6):
    """transformers qwen3_5_moe l2norm: x * rsqrt(sum(x^2) + eps)."""
    return x / np.sqrt((x * x).sum(-1, keepdims=True) + eps)


def _l2norm_bwd(x, dy, eps=1e-6):
    r = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True) + eps)
    return r * dy - (r ** 3) * (x * dy).sum(-1, keepdims=True) * x


def _gqa_expand(q, hv):
    hq = q.shape[2]
    if hq == hv:
        return q
    return np.repeat(q, hv // hq, axis=2)


def _correction(A, exact_inverse):
    """The intra-node operator T applied to beta*v and beta*k*e^gam.  The
    reference's row loop (tree_dfs_ssm.py:119-126) uses uncorrected earlier
    rows, which is exactly T = I + A + A^2; ``exact_inverse`` gives the delta
    rule's exact T = (I - A)^-1 (what the in-place row loop of
    transformers' torch_chunk_gated_delta_rule computes)."""
    L = A.shape[-1]
    if exact_inverse:
        return np.linalg.inv(np.eye(L) - A)
    return np.eye(L) + A + A @ A


def gdn_tree_fwd(query, key, value, g, beta, bounds, parents, initial_state=None,
                 use_qk_l2norm=False, exact_inverse=False):
    """Tree-routed chunk gated delta rule, one chunk per tree node.

    query/key [B,S,Hk,Dk] (Hk == H, or H // Hk v-heads per k-head), value
    [B,S,H,Dv], g/beta [B,S,H].  Each node reads the state after its PARENT
    node (tree_dfs_ssm.py:131-132).  The intra-node correction is the
    reference's row loop (:119-126), which equals T = I + A + A^2 exactly.
    Returns (out [B,S,H,Dv], states [n_nodes+1, B,H,Dk,Dv]) in float64;
    ``states[0]`` is the initial state and ``states[i+1]`` the state after
    node i (:84-89, :149).
    """
    H = value.shape[2]
    q = np.asarray(query, np.float64)
    k = np.asarray(key, np.float64)
    if use_qk_l2norm:                                                   # :67-69
        q = _l2norm(q)
        k = _l2norm(k)
    q = _gqa_expand(q, H).transpose(0, 2, 1, 3)          # [B,H,S,Dk]   :72
    k = _gqa_expand(k, H).transpose(0, 2, 1, 3)
    v = np.asarray(value, np.float64).transpose(0, 2, 1, 3)
    bt = np.asarray(beta, np.float64).transpose(0, 2, 1)
    gg = np.asarray(g, np.float64).transpose(0, 2, 1)
    B, _, S, Dk = k.shape
    Dv = v.shape[-1]
    q = q * (Dk ** -0.5)                                                 # :82
    init = (np.zeros((B, H, Dk, Dv)) if initial_state is None
            else np.asarray(initial_state, np.float64))
    states = [init]
    out = np.zeros((B, H, S, Dv))
    for i, (cs, ce) in enumerate(bounds):
        L = ce - cs
        qi, ki, vi = q[:, :, cs:ce], k[:, :, cs:ce], v[:, :, cs:ce]
        bi, gi = bt[:, :, cs:ce], gg[:, :, cs:ce]
        gam = np.cumsum(gi, axis=-1)                                     # :106
        diff = gam[..., :, None] - gam[..., None, :]
        low_incl = np.tril(np.ones((L, L), dtype=bool))
        low_excl = np.tril(np.ones((L, L), dtype=bool), -1)
        decay = np.where(low_incl, np.exp(np.where(low_incl, diff, 0.0)), 0.0)  # :109
        kb = ki * bi[..., None]
        vb = vi * bi[..., None]
        A = np.where(low_excl, -(kb @ np.swapaxes(ki, -1, -2)) * decay, 0.0)     # :116
        T = _correction(A, exact_inverse)                                 # :119-126
        U = T @ vb                                                        # :127
        W = T @ (kb * np.exp(gam)[..., None])                             # :128
        Sin = states[parents[i] + 1]                                      # :131-132
        Vn = U - W @ Sin                                                  # :134-135
        Aqk = np.where(low_incl, (qi @ np.swapaxes(ki, -1, -2)) * decay, 0.0)  # :137
        out[:, :, cs:ce] = (qi * np.exp(gam)[..., None]) @ Sin + Aqk @ Vn      # :138-140
        gL = gam[..., -1]
        Kd = ki * np.exp(gL[..., None] - gam)[..., None]
        states.append(Sin * np.exp(gL)[..., None, None]
                      + np.swapaxes(Kd, -1, -2) @ Vn)                     # :144-148
    return out.transpose(0, 2, 1, 3), np.stack(states)


def gdn_tree_bwd(query, key, value, g, beta, bounds, parents, dout,
                 initial_state=None, use_qk_l2norm=False, dlast_state=None,
                 exact_inverse=False):
    """Analytic gradients of :func:`gdn_tree_fwd` (the reference relies on
    torch autograd through tree_dfs_ssm.py:92-156; this restates that
    gradient).  ``dlast_state`` is the gradient of ``last_state`` = the state
    after the last DFS node (:155).  Returns dq, dk, dv, dg, dbeta, dinit with
    the input shapes (dq/dk summed back over the GQA group)."""
    Hk = query.shape[2]
    H = value.shape[2]
    q0 = np.asarray(query, np.float64)
    k0 = np.asarray(key, np.float64)
    qn = _l2norm(q0) if use_qk_l2norm else q0
    kn = _l2norm(k0) if use_qk_l2norm else k0
    q = _gqa_expand(qn, H).transpose(0, 2, 1, 3)
    k = _gqa_expand(kn, H).transpose(0, 2, 1, 3)
    v = np.asarray(value, np.float64).transpose(0, 2, 1, 3)
    bt = np.asarray(beta, np.float64).transpose(0, 2, 1)
    gg = np.asarray(g, np.float64).transpose(0, 2, 1)
    do = np.asarray(dout, np.float64).transpose(0, 2, 1, 3)
    B, _, S, Dk = k.shape
    Dv = v.shape[-1]
    sc = Dk ** -0.5
    qs = q * sc
    _, states = gdn_tree_fwd(query, key, value, g, beta, bounds, parents,
                             initial_state, use_qk_l2norm, exact_inverse)
    n = len(bounds)
    dstate = [np.zeros((B, H, Dk, Dv)) for _ in range(n + 1)]
    if dlast_state is not None:
        dstate[n] = dstate[n] + np.asarray(dlast_state, np.float64)
    dq = np.zeros_like(qs)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    dgam_all = np.zeros_like(gg)
    dbt = np.zeros_like(bt)
    for i in range(n - 1, -1, -1):
        cs, ce = bounds[i]
        L = ce - cs
        qi, ki, vi = qs[:, :, cs:ce], k[:, :, cs:ce], v[:, :, cs:ce]
        bi, gi = bt[:, :, cs:ce], gg[:, :, cs:ce]
        gam = np.cumsum(gi, axis=-1)
        diff = gam[..., :, None] - gam[..., None, :]
        li = np.tril(np.ones((L, L), dtype=bool))
        le = np.tril(np.ones((L, L), dtype=bool), -1)
        D = np.where(li, np.exp(np.where(li, diff, 0.0)), 0.0)
        eg = np.exp(gam)
        gL = gam[..., -1]
        kb = ki * bi[..., None]
        vb = vi * bi[..., None]
        KK = kb @ np.swapaxes(ki, -1, -2)
        A = np.where(le, -KK * D, 0.0)
        T = _correction(A, exact_inverse)
        Kbg = kb * eg[..., None]
        U = T @ vb
        W = T @ Kbg
        Sin = states[parents[i] + 1]
        Vn = U - W @ Sin
        QK = qi @ np.swapaxes(ki, -1, -2)
        Aqk = np.where(li, QK * D, 0.0)
        Qg = qi * eg[..., None]
        Kd = ki * np.exp(gL[..., None] - gam)[..., None]
        dO = do[:, :, cs:ce]
        dSo = dstate[i + 1]
        tr = lambda x: np.swapaxes(x, -1, -2)
        dVn = tr(Aqk) @ dO + Kd @ dSo
        dAqk = np.where(li, dO @ tr(Vn), 0.0)
        dQg = dO @ tr(Sin)
        dSin = tr(Qg) @ dO + np.exp(gL)[..., None, None] * dSo - tr(W) @ dVn
        dKd = Vn @ tr(dSo)
        dW = -dVn @ tr(Sin)
        dT = dVn @ tr(vb) + dW @ tr(Kbg)
        dvb = tr(T) @ dVn
        dKbg = tr(T) @ dW
        if exact_inverse:       # T = (I - A)^-1: dL/dA = T^T dT T^T
            dA = np.where(le, tr(T) @ dT @ tr(T), 0.0)
        else:                   # T = I + A + A^2
            dA = np.where(le, dT + dT @ tr(A) + tr(A) @ dT, 0.0)
        dgam = np.zeros_like(gam)
        # A = -(kb k^T) * D on the strict lower triangle
        Gm = -dA * D
        dkb = Gm @ ki
        dki = tr(Gm) @ kb
        dD = -dA * KK
        # Aqk = (q k^T) * D on the lower triangle incl. diagonal
        F = dAqk * D
        dqi = F @ ki
        dki = dki + tr(F) @ qi
        dD = dD + np.where(li, dAqk * QK, 0.0)
        # D[j,m] = exp(gam_j - gam_m)
        dDD = dD * D
        dgam += dDD.sum(-1) - dDD.sum(-2)
        # Qg = q * e^gam
        dqi = dqi + dQg * eg[..., None]
        dgam += (Qg * dQg).sum(-1)
        # Kd = k * e^(gL - gam)
        dki = dki + dKd * np.exp(gL[..., None] - gam)[..., None]
        t = (Kd * dKd).sum(-1)
        dgam -= t
        dgam[..., -1] += t.sum(-1)
        # Kbg = kb * e^gam
        dkb = dkb + dKbg * eg[..., None]
        dgam += (Kbg * dKbg).sum(-1)
        # state decay e^gL * Sin
        dgam[..., -1] += np.exp(gL) * (Sin * dSo).sum((-1, -2))
        # kb = k * beta, vb = v * beta
        dki = dki + dkb * bi[..., None]
        dbi = (ki * dkb).sum(-1) + (vi * dvb).sum(-1)
        dvi = dvb * bi[..., None]
        dq[:, :, cs:ce] = dqi
        dk[:, :, cs:ce] = dki
        dv[:, :, cs:ce] = dvi
        dbt[:, :, cs:ce] = dbi
        dgam_all[:, :, cs:ce] = dgam
        dstate[parents[i] + 1] = dstate[parents[i] + 1] + dSin
    # gam = cumsum(g): reverse cumulative sum inside each node
    dg = np.zeros_like(gg)
    for (cs, ce) in bounds:
        dg[:, :, cs:ce] = np.flip(np.cumsum(np.flip(dgam_all[:, :, cs:ce], -1), -1), -1)
    dq = dq * sc
    dq = dq.transpose(0, 2, 1, 3)
    dk = dk.transpose(0, 2, 1, 3)
    if Hk != H:
        r = H // Hk
        dq = dq.reshape(B, S, Hk, r, Dk).sum(3)
        dk = dk.reshape(B, S, Hk, r, Dk).sum(3)
    if use_qk_l2norm:
        dq = _l2norm_bwd(q0, dq)
        dk = _l2norm_bwd(k0, dk)
    return (dq, dk, dv.transpose(0, 2, 1, 3), dg.transpose(0, 2, 1),
            dbt.transpose(0, 2, 1), dstate[0])


def gdn_tree_recurrent(query, key, value, g, beta, bounds, parents, initial_state=None,
                       use_qk_l2norm=False):
    """The gated delta rule token by token along each root-to-node path, in
    float64: the per-token recurrence of transformers'
    torch_recurrent_gated_delta_rule (models/qwen3_5_moe/modeling_qwen3_5_moe.py,
    lines 315-354: S <- S e^g; delta = beta (v - S^T k); S <- S + k delta^T;
    o = S^T q with q scaled by Dk^-1/2), each node starting from the state
    after its parent node.  Independent of how tokens are grouped into nodes,
    so it is the exact operator the chunked forms approximate (reference,
    T = I + A + A^2) or reproduce (exact inverse).  Same shapes and return
    value as :func:`gdn_tree_fwd`."""
    H = value.shape[2]
    q = np.asarray(query, np.float64)
    k = np.asarray(key, np.float64)
    if use_qk_l2norm:
        q = _l2norm(q)
        k = _l2norm(k)
    q = _gqa_expand(q, H).transpose(0, 2, 1, 3)
    k = _gqa_expand(k, H).transpose(0, 2, 1, 3)
    v = np.asarray(value, np.float64).transpose(0, 2, 1, 3)
    bt = np.asarray(beta, np.float64).transpose(0, 2, 1)
    gg = np.asarray(g, np.float64).transpose(0, 2, 1)
    B, _, S, Dk = k.shape
    Dv = v.shape[-1]
    q = q * (Dk ** -0.5)
    init = (np.zeros((B, H, Dk, Dv)) if initial_state is None
            else np.asarray(initial_state, np.float64))
    states = [init]
    out = np.zeros((B, H, S, Dv))
    for i, (cs, ce) in enumerate(bounds):
        St = states[parents[i] + 1].copy()
        for t in range(cs, ce):
            St = St * np.exp(gg[:, :, t])[..., None, None]
            kv = np.einsum("bhkv,bhk->bhv", St, k[:, :, t])
            delta = (v[:, :, t] - kv) * bt[:, :, t][..., None]
            St = St + k[:, :, t][..., :, None] * delta[..., None, :]
            out[:, :, t] = np.einsum("bhkv,bhk->bhv", St, q[:, :, t])
        states.append(St)
    return out.transpose(0, 2, 1, 3), np.stack(states)


# ---------------------------------------------------------------------------
# Tree-correct depthwise causal conv + SiLU  (tree_dfs_ssm.py:285-348;
# same semantics in dfs_tree_forward.py:191-246)
# ---------------------------------------------------------------------------

def conv_predecessors(bounds, parents, K: int) -> np.ndarray:
    """pred[t, m-1] = the token m steps before t on t's root-to-node path, or
    -1 (zero padding).  This is the effective history that the reference
    builds by prepending the parent's saved last K-1 inputs (:316-318,
    :338-346)."""
    N = bounds[-1][1] if len(bounds) else 0
    prev = np.full(N, -1, dtype=np.int64)
    last_tok = {}
    for c, (s, e) in enumerate(bounds):
        p = parents[c]
        before = last_tok.get(p, -1) if p >= 0 else -1
        for t in range(s, e):
            prev[t] = before
            before = t
        last_tok[c] = before          # a 0-token node passes its parent's context on
    pred = np.full((N, max(K - 1, 0)), -1, dtype=np.int64)
    for t in range(N):
        cur = t
        for m in range(K - 1):
            cur = prev[cur] if cur >= 0 else -1
            pred[t, m] = cur
    return pred


def tree_conv_fwd(x, weight, bounds, parents, bias=None):
    """x [B, C, S], weight [C, K] -> silu(causal depthwise conv over each
    token's tree path) [B, C, S] (float64)."""
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64)
    K = w.shape[1]
    pred = conv_predecessors(bounds, parents, K)
    pre = x * w[None, :, K - 1, None]
    for m in range(1, K):
        idx = pred[:, m - 1]
        xm = np.where(idx[None, None, :] >= 0, x[:, :, np.maximum(idx, 0)], 0.0)
        pre = pre + xm * w[None, :, K - 1 - m, None]
    if bias is not None:
        pre = pre + np.asarray(bias, np.float64)[None, :, None]
    return pre / (1.0 + np.exp(-pre)), pre


def tree_conv_bwd(x, weight, bounds, parents, dout, bias=None):
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64)
    K = w.shape[1]
    pred = conv_predecessors(bounds, parents, K)
    _, pre = tree_conv_fwd(x, w, bounds, parents, bias)
    sig = 1.0 / (1.0 + np.exp(-pre))
    dpre = np.asarray(dout, np.float64) * (sig * (1.0 + pre * (1.0 - sig)))
    dx = dpre * w[None, :, K - 1, None]
    dw = np.zeros_like(w)
    dw[:, K - 1] = (dpre * x).sum((0, 2))
    for m in range(1, K):
        idx = pred[:, m - 1]
        ok = idx >= 0
        xm = np.where(ok[None, None, :], x[:, :, np.maximum(idx, 0)], 0.0)
        dw[:, K - 1 - m] = (dpre * xm).sum((0, 2))
        contrib = dpre[:, :, ok] * w[None, :, K - 1 - m, None]
        np.add.at(dx, (slice(None), slice(None), idx[ok]), contrib)
    db = dpre.sum((0, 2)) if bias is not None else None
    return dx, dw, db
