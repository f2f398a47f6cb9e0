"""Tree GDN and tree conv in plain torch (checker and CPU baseline).

TEST AND CPU-BASELINE INFRASTRUCTURE ONLY: used by ``tests/`` (as a
batched-over-heads float64 checker on the GPU) and by ``bench.py``'s GDN
``cpu_baseline`` leg (timed on host cores); never by the product package.

* :func:`gdn_tree_torch` restates torch_chunk_gated_delta_rule_tree_varlen
  (tree_dfs_ssm.py:38-156) like ``oracle.tree_oracle.gdn_tree_fwd``, with
  torch ops, gradients by torch autograd (the reference itself relies on
  autograd through the same expressions).  ``row_loop=True`` builds the
  correction with the reference's own row loop (:119-126) instead of the
  equal closed form I + A + A^2, so that its CPU time is the reference's.
* :func:`tree_conv_torch` restates _tree_correct_conv_varlen
  (tree_dfs_ssm.py:285-348) with the layer's causal depthwise conv1d + SiLU.

Both are pinned to the numpy oracle by ``tests/test_gdn_torch_ref_cpu.py``.
"""
from __future__ import annotations

import time

import torch
import torch.nn.functional as F


def _l2norm(x, eps=1e-6):
    """transformers qwen3_5_moe l2norm: x * rsqrt(sum(x^2) + eps)."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gdn_tree_torch(query, key, value, g, beta, bounds, parents, initial_state=None,
                   use_qk_l2norm=False, row_loop=False):
    """query/key [B,S,Hk,Dk] (H // Hk v-heads per k-head, as the reference's
    repeat_interleave glue at dfs_tree_forward.py:403-410 expands them), value
    [B,S,H,Dv], g/beta [B,S,H]; computes in the inputs' dtype.  Returns
    (out [B,S,H,Dv], last_state [B,H,Dk,Dv])."""
    H = value.shape[2]
    q, k = query, key
    if use_qk_l2norm:                                                   # :67-69
        q, k = _l2norm(q), _l2norm(k)
    rep = H // q.shape[2]
    if rep > 1:
        q = q.repeat_interleave(rep, dim=2)
        k = k.repeat_interleave(rep, dim=2)
    q = q.transpose(1, 2)                                               # [B,H,S,Dk] :72
    k = k.transpose(1, 2)
    v = value.transpose(1, 2)
    bt = beta.transpose(1, 2)
    gg = g.transpose(1, 2)
    B, _, S, Dk = k.shape
    Dv = v.shape[-1]
    q = q * (Dk ** -0.5)                                                 # :82
    init = (torch.zeros(B, H, Dk, Dv, dtype=v.dtype, device=v.device)
            if initial_state is None else initial_state)
    states = [init]
    outs = []
    for i, (cs, ce) in enumerate(bounds):
        L = ce - cs
        qi, ki, vi = q[:, :, cs:ce], k[:, :, cs:ce], v[:, :, cs:ce]
        bi, gi = bt[:, :, cs:ce], gg[:, :, cs:ce]
        gam = gi.cumsum(-1)                                              # :106
        low_incl = torch.ones(L, L, dtype=torch.bool, device=v.device).tril()
        low_excl = torch.ones(L, L, dtype=torch.bool, device=v.device).tril(-1)
        diff = (gam[..., :, None] - gam[..., None, :]).masked_fill(~low_incl, 0.0)
        decay = diff.exp().masked_fill(~low_incl, 0.0)                   # :109
        kb = ki * bi[..., None]
        vb = vi * bi[..., None]
        A = (-(kb @ ki.transpose(-1, -2)) * decay).masked_fill(~low_excl, 0.0)   # :116
        KG = kb * gam.exp()[..., None]
        if row_loop:                                                     # :119-128
            rows = [A[..., 0:1, :]]
            for j in range(1, L):
                rows.append(A[..., j:j + 1, :] + A[..., j:j + 1, :j] @ A[..., :j, :])
            T = torch.cat(rows, dim=-2) + torch.eye(L, dtype=A.dtype, device=A.device)
            U, W = T @ vb, T @ KG
        else:                                                            # T = I + A + A^2
            AV = A @ vb
            AK = A @ KG
            U = vb + AV + A @ AV                                         # :127
            W = KG + AK + A @ AK                                         # :128
        Sin = states[parents[i] + 1]                                     # :131-132
        Vn = U - W @ Sin                                                 # :134-135
        Aqk = ((qi @ ki.transpose(-1, -2)) * decay).masked_fill(~low_incl, 0.0)  # :137
        outs.append((qi * gam.exp()[..., None]) @ Sin + Aqk @ Vn)        # :138-140
        gL = gam[..., -1:]
        Kd = ki * (gL - gam).exp()[..., None]
        states.append(Sin * gL.exp()[..., None] + Kd.transpose(-1, -2) @ Vn)   # :144-148
    out = torch.cat(outs, dim=2).transpose(1, 2)
    return out, states[-1]


def tree_conv_torch(x, weight, bounds, parents, bias=None):
    """x [B, C, S], weight [C, K] (the layer's conv1d weight without its
    singleton dim): each chunk is convolved after the last K-1 effective
    tokens of its parent chunk (zeros for a root), causal depthwise conv +
    SiLU, the prepended context dropped (tree_dfs_ssm.py:305-346)."""
    C, K = weight.shape
    w = weight[:, None, :]
    conv = lambda t: F.silu(F.conv1d(t, w, bias, padding=K - 1, groups=C)[..., :t.shape[-1]])
    outs, ctx = [], {}
    for c, (cs, ce) in enumerate(bounds):
        chunk = x[..., cs:ce]
        par = ctx.get(parents[c])
        if par is not None:
            ext = torch.cat([par, chunk], dim=-1)
            outs.append(conv(ext)[..., K - 1:])
            ctx[c] = ext[..., -(K - 1):]
        else:
            outs.append(conv(chunk))
            ctx[c] = F.pad(chunk, (max(0, K - 1 - (ce - cs)), 0))[..., -(K - 1):]
    return torch.cat(outs, dim=-1)


def time_gdn_step_sample(bounds, parents, S, Hk, H, D, K=4, seed=0):
    """One fwd+bwd step of the reference's hybrid-layer core on host cores:
    tree conv over the q/k/v channels of ``Hk`` k-heads and ``H`` v-heads,
    then the tree GDN (q/k L2-normalised, the reference's row loop), bf16
    inputs computed in fp32 as the reference does, torch autograd backward.
    Returns seconds."""
    g = torch.Generator().manual_seed(seed)
    C = 2 * Hk * D + H * D
    x = torch.randn(1, C, S, generator=g).to(torch.bfloat16).float().requires_grad_(True)
    w = (torch.randn(C, K, generator=g) * 0.5).requires_grad_(True)
    gg = F.logsigmoid(torch.randn(1, S, H, generator=g)).requires_grad_(True)
    bt = torch.sigmoid(torch.randn(1, S, H, generator=g)).requires_grad_(True)
    do = torch.randn(1, S, H, D, generator=g)
    t0 = time.perf_counter()
    y = tree_conv_torch(x, w, bounds, parents).transpose(1, 2)
    q = y[..., :Hk * D].reshape(1, S, Hk, D)
    k = y[..., Hk * D:2 * Hk * D].reshape(1, S, Hk, D)
    v = y[..., 2 * Hk * D:].reshape(1, S, H, D)
    out, _ = gdn_tree_torch(q, k, v, gg, bt, bounds, parents, None, True, row_loop=True)
    (out * do).sum().backward()
    return time.perf_counter() - t0
