"""Exact-inverse tree GDN: the oracle pinned against the token-by-token gated
delta rule (no GPU).

* forward: the chunked oracle with T = (I - A)^-1 per node equals
  ``gdn_tree_recurrent`` (the per-token recurrence of transformers'
  torch_recurrent_gated_delta_rule along each root-to-node path) to 1e-12;
* backward: the oracle's analytic exact-mode gradients equal torch autograd
  through an independent float64 torch version of that recurrence to 1e-9;
* the reference mode (T = I + A + A^2) does not equal the recurrence, which is
  the reason the exact mode exists.
"""
import numpy as np
import torch

from oracle import tree_oracle as O


def _inputs(seed=0, S=90, Hk=1, H=2, Dk=16, Dv=8):
    g_ = np.random.default_rng(seed)
    q = g_.standard_normal((1, S, Hk, Dk))
    k = g_.standard_normal((1, S, Hk, Dk))
    v = g_.standard_normal((1, S, H, Dv))
    gg = -g_.uniform(0.01, 0.3, (1, S, H))
    bt = g_.uniform(0.1, 0.9, (1, S, H))
    s0 = g_.standard_normal((1, H, Dk, Dv)) * 0.1
    do = g_.standard_normal((1, S, H, Dv))
    dl = g_.standard_normal((1, H, Dk, Dv))
    bounds = [(0, 25), (25, 40), (40, 41), (41, 70), (70, 90)]
    parents = [-1, 0, 1, 0, 3]
    return q, k, v, gg, bt, s0, do, dl, bounds, parents


def _torch_recurrent(q, k, v, g, beta, bounds, parents, s0):
    """float64 torch autograd version of the per-path recurrence
    (S <- S e^g; delta = beta (v - S^T k); S <- S + k delta^T; o = S^T q)."""
    H = v.shape[2]
    qn = q / torch.sqrt((q * q).sum(-1, keepdim=True) + 1e-6)
    kn = k / torch.sqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    rep = H // q.shape[2]
    qn = qn.repeat_interleave(rep, dim=2) * (q.shape[-1] ** -0.5)
    kn = kn.repeat_interleave(rep, dim=2)
    states = [s0[0]]
    outs = []
    for i, (cs, ce) in enumerate(bounds):
        st = states[parents[i] + 1]
        for t in range(cs, ce):
            st = st * torch.exp(g[0, t])[:, None, None]
            kv = torch.einsum("hkv,hk->hv", st, kn[0, t])
            delta = (v[0, t] - kv) * beta[0, t][:, None]
            st = st + kn[0, t][:, :, None] * delta[:, None, :]
            outs.append(torch.einsum("hkv,hk->hv", st, qn[0, t]))
        states.append(st)
    return torch.stack(outs, 0)[None], states[-1][None]


def test_exact_forward_equals_recurrence():
    q, k, v, gg, bt, s0, _, _, bounds, parents = _inputs()
    out, states = O.gdn_tree_fwd(q, k, v, gg, bt, bounds, parents, s0, True, True)
    rout, rstates = O.gdn_tree_recurrent(q, k, v, gg, bt, bounds, parents, s0, True)
    assert np.abs(out - rout).max() < 1e-12 * np.abs(rout).max()
    assert np.abs(states - rstates).max() < 1e-12 * np.abs(rstates).max()


def test_reference_mode_is_not_the_recurrence():
    q, k, v, gg, bt, s0, _, _, bounds, parents = _inputs()
    out, _ = O.gdn_tree_fwd(q, k, v, gg, bt, bounds, parents, s0, True, False)
    rout, _ = O.gdn_tree_recurrent(q, k, v, gg, bt, bounds, parents, s0, True)
    assert np.abs(out - rout).max() > 1e-6 * np.abs(rout).max()


def test_exact_backward_equals_autograd_of_recurrence():
    q, k, v, gg, bt, s0, do, dl, bounds, parents = _inputs(seed=1, Hk=1, H=2)
    ts = [torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (q, k, v, gg, bt, s0)]
    out, last = _torch_recurrent(*ts[:5], bounds, parents, ts[5])
    loss = (out * torch.tensor(do)).sum() + (last * torch.tensor(dl)).sum()
    loss.backward()
    want = [t.grad.numpy() for t in ts]
    got = O.gdn_tree_bwd(q, k, v, gg, bt, bounds, parents, do, s0, True, dl, True)
    for name, a, b in zip(("dq", "dk", "dv", "dg", "dbeta", "dinit"), got, want):
        assert np.abs(a - b).max() < 1e-9 * (np.abs(b).max() + 1e-30), name
