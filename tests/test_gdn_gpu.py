"""Tree GDN and tree conv on a B200 vs the reference's outputs and the oracle.

* golden fixtures produced by torch_chunk_gated_delta_rule_tree_varlen and
  _tree_correct_conv_varlen themselves: fp32 path, max_rel < 2e-5 (the GDN bar)
* random trees vs the float64 oracle: fp32 < 2e-5 (D = 64 and 128), bf16 < 2e-2
* config-4 size (16,384-token tree, 16 k-heads / 32 v-heads, D=128, bf16):
  every head of every output and gradient against a float64 torch
  restatement of the reference run on the GPU (oracle/gdn_torch.py,
  pinned to the oracle on CPU)
"""
import random

import numpy as np
import pytest
import torch

from oracle import tree_oracle as O
from tests.golden_util import load

import tree_training_b200 as tt
from tree_training_b200.gdn import _tree_correct_conv_varlen, torch_chunk_gated_delta_rule_tree_varlen
from tree_training_b200.synthetic import random_branching_tree

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


def run_gdn(q, k, v, g, beta, bounds, parents, init, l2, dout, dlast, dtype, exact=False):
    T = lambda x: torch.tensor(x, dtype=dtype, device=DEV, requires_grad=True)
    F32 = lambda x: torch.tensor(x, dtype=torch.float32, device=DEV, requires_grad=True)
    qt, kt, vt = T(q), T(k), T(v)
    gt, bt = F32(g), F32(beta)
    it = F32(init) if init is not None else None
    out, last = torch_chunk_gated_delta_rule_tree_varlen(
        qt, kt, vt, gt, bt, bounds, parents, initial_state=it,
        output_final_state=dlast is not None, use_qk_l2norm_in_kernel=l2, exact_inverse=exact)
    loss = (out.float() * torch.tensor(dout, dtype=torch.float32, device=DEV)).sum()
    if dlast is not None:
        loss = loss + (last * torch.tensor(dlast, dtype=torch.float32, device=DEV)).sum()
    loss.backward()
    torch.cuda.synchronize()
    f = lambda t: None if t is None else t.detach().double().cpu().numpy()
    return dict(out=f(out), last=f(last), dq=f(qt.grad), dk=f(kt.grad), dv=f(vt.grad),
                dg=f(gt.grad), dbeta=f(bt.grad), dinit=f(it.grad) if it is not None else None)


@pytest.mark.parametrize("name", ["gdn_tree_l2", "gdn_tree_init_final", "gdn_forest47"])
def test_gdn_matches_reference_fixture(name):
    d = load(name)
    bounds = [tuple(b) for b in d["chunk_boundaries"].tolist()]
    parents = d["chunk_parent_map"].tolist()
    init = d["init"] if d["init"].size else None
    dlast = d["dlast"] if d["dlast"].size else None
    got = run_gdn(d["q"], d["k"], d["v"], d["g"], d["beta"], bounds, parents, init,
                  bool(int(d["l2norm"])), d["dout"], dlast, torch.float32)
    for key in ("out", "dq", "dk", "dv", "dg", "dbeta"):
        assert rel(got[key], d[key]) < 2e-5, key
    if dlast is not None:
        assert rel(got["last"], d["last"]) < 2e-5
    if init is not None:
        assert rel(got["dinit"], d["dinit"]) < 2e-5


def _case(seed, S, Hk, H, D, lo, hi, init=False):
    roots = random_branching_tree(seed, S, lo, hi)
    info = tt.build_dfs_tree_info(roots)
    g_ = np.random.default_rng(seed)
    q = g_.standard_normal((1, S, Hk, D))
    k = g_.standard_normal((1, S, Hk, D))
    v = g_.standard_normal((1, S, H, D)) * 0.5
    gg = -np.log1p(np.exp(-g_.standard_normal((1, S, H))))         # logsigmoid(N(0,1))
    bt = 1.0 / (1.0 + np.exp(-g_.standard_normal((1, S, H))))      # sigmoid(N(0,1))
    s0 = g_.standard_normal((1, H, D, D)) * 0.05 if init else None
    do = g_.standard_normal((1, S, H, D))
    dl = g_.standard_normal((1, H, D, D)) if init else None
    return info, q, k, v, gg, bt, s0, do, dl


def _oracle(info, q, k, v, gg, bt, s0, do, dl, exact=False):
    out, states = O.gdn_tree_fwd(q, k, v, gg, bt, info.chunk_boundaries, info.chunk_parent_map,
                                 s0, True, exact)
    grads = O.gdn_tree_bwd(q, k, v, gg, bt, info.chunk_boundaries, info.chunk_parent_map, do,
                           s0, True, dl, exact)
    return dict(out=out, last=states[-1], dq=grads[0], dk=grads[1], dv=grads[2], dg=grads[3],
                dbeta=grads[4], dinit=grads[5])


@pytest.mark.parametrize("dtype,tol,init,D", [(torch.float32, 2e-5, True, 64),
                                               (torch.float32, 2e-5, True, 128),
                                               (torch.bfloat16, 2e-2, False, 64),
                                               (torch.bfloat16, 2e-2, False, 128)])
def test_gdn_random_tree_vs_oracle(dtype, tol, init, D):
    info, q, k, v, gg, bt, s0, do, dl = _case(3, 1200, 2, 4, D, 16, 300, init)
    if dtype == torch.bfloat16:
        rnd = lambda x: torch.tensor(x, dtype=torch.bfloat16).double().numpy()
        q, k, v = rnd(q), rnd(k), rnd(v)
    ref = _oracle(info, q, k, v, gg, bt, s0, do, dl)
    got = run_gdn(q, k, v, gg, bt, info.chunk_boundaries, info.chunk_parent_map, s0, True, do,
                  dl, dtype)
    keys = ["out", "dq", "dk", "dv", "dg", "dbeta"] + (["last", "dinit"] if init else [])
    for key in keys:
        assert rel(got[key], ref[key]) < tol, key


@pytest.mark.parametrize("lo,hi", [(16, 300), (500, 800)])
def test_gdn_exact_inverse_vs_oracle_and_recurrence(lo, hi):
    """Exact-inverse mode (T = (I - A)^-1 per node, computed as 64 x 64
    diagonal-block inverses plus block-row GEMMs): fp32 vs the float64 oracle
    of the same mode, and its output vs the token-by-token recurrence.  Node
    lengths up to 300 (5 blocks) and 500-800 (8-13 blocks)."""
    info, q, k, v, gg, bt, s0, do, dl = _case(5, 1800, 2, 4, 64, lo, hi, True)
    ref = _oracle(info, q, k, v, gg, bt, s0, do, dl, exact=True)
    got = run_gdn(q, k, v, gg, bt, info.chunk_boundaries, info.chunk_parent_map, s0, True, do,
                  dl, torch.float32, exact=True)
    for key in ["out", "last", "dq", "dk", "dv", "dg", "dbeta", "dinit"]:
        assert rel(got[key], ref[key]) < 5e-5, key
    rec, rec_states = O.gdn_tree_recurrent(q, k, v, gg, bt, info.chunk_boundaries,
                                           info.chunk_parent_map, s0, True)
    assert rel(got["out"], rec) < 5e-5
    assert rel(got["last"], rec_states[-1]) < 5e-5


def test_gdn_exact_inverse_block_edges():
    """Node lengths at the 64-token block edges of the inverse (1, 63, 64, 65,
    128, 129, 192) against the float64 recurrence."""
    lens = [64, 1, 63, 65, 128, 129, 192, 2]
    parents = [-1, 0, 0, 2, 3, 1, 4, 6]
    bounds, s0 = [], 0
    for L in lens:
        bounds.append((s0, s0 + L))
        s0 += L
    S, H, D = s0, 2, 32
    g_ = np.random.default_rng(21)
    q = g_.standard_normal((1, S, 1, D))
    k = g_.standard_normal((1, S, 1, D))
    v = g_.standard_normal((1, S, H, D)) * 0.5
    gg = -np.log1p(np.exp(-g_.standard_normal((1, S, H))))
    bt = 1.0 / (1.0 + np.exp(-g_.standard_normal((1, S, H))))
    do = g_.standard_normal((1, S, H, D))
    got = run_gdn(q, k, v, gg, bt, bounds, parents, None, True, do, None, torch.float32,
                  exact=True)
    rec, _ = O.gdn_tree_recurrent(q, k, v, gg, bt, bounds, parents, None, True)
    assert rel(got["out"], rec) < 5e-5
    grads = O.gdn_tree_bwd(q, k, v, gg, bt, bounds, parents, do, None, True, None, True)
    for key, ref in zip(("dq", "dk", "dv", "dg", "dbeta"), grads[:5]):
        assert rel(got[key], ref) < 5e-5, key


def test_gdn_exact_inverse_is_segmentation_invariant():
    """One 600-token path as a single node, and as a chain of 4 nodes: the
    exact mode gives the same output (the reference's truncated correction
    does not, which the second half of the test shows)."""
    S, H, D = 600, 2, 64
    g_ = np.random.default_rng(11)
    q = g_.standard_normal((1, S, H, D))
    k = g_.standard_normal((1, S, H, D))
    v = g_.standard_normal((1, S, H, D)) * 0.5
    gg = -np.log1p(np.exp(-g_.standard_normal((1, S, H))))
    bt = 1.0 / (1.0 + np.exp(-g_.standard_normal((1, S, H))))
    do = g_.standard_normal((1, S, H, D))
    one = ([(0, S)], [-1])
    chain = ([(0, 130), (130, 300), (300, 301), (301, S)], [-1, 0, 1, 2])
    run = lambda seg, ex: run_gdn(q, k, v, gg, bt, seg[0], seg[1], None, True, do, None,
                                  torch.float32, exact=ex)
    rec, _ = O.gdn_tree_recurrent(q, k, v, gg, bt, [(0, S)], [-1], None, True)
    a, b = run(one, True), run(chain, True)
    assert rel(a["out"], rec) < 3e-5
    assert rel(b["out"], rec) < 3e-5
    for key in ("dq", "dk", "dv", "dg", "dbeta"):
        assert rel(b[key], a[key]) < 1e-4, key
    # float64 oracle on these inputs: the truncated correction over the single
    # 600-token node is 1.9e-4 away from the recurrence (exact mode: 1e-14)
    ra = run(one, False)
    assert rel(ra["out"], rec) > 1e-4


@pytest.mark.parametrize("exact", [False, True])
def test_gdn_keep_forward_gives_identical_gradients(exact):
    """keep_forward=True: the backward reads the forward's workspace instead of
    recomputing it; the kernels are deterministic, so every output and
    gradient is bitwise equal to the recomputing path, also for a second
    backward through the same graph."""
    info, q, k, v, gg, bt, s0, do, dl = _case(8, 900, 2, 4, 64, 16, 300, True)
    res = []
    for keep in (False, True):
        T = lambda x: torch.tensor(x, dtype=torch.float32, device=DEV, requires_grad=True)
        ts = [T(x) for x in (q, k, v, gg, bt, s0)]
        out, last = torch_chunk_gated_delta_rule_tree_varlen(
            *ts[:5], info.chunk_boundaries, info.chunk_parent_map, initial_state=ts[5],
            output_final_state=True, use_qk_l2norm_in_kernel=True, exact_inverse=exact,
            keep_forward=keep)
        loss = (out * torch.tensor(do, dtype=torch.float32, device=DEV)).sum() + \
            (last * torch.tensor(dl, dtype=torch.float32, device=DEV)).sum()
        g1 = torch.autograd.grad(loss, ts, retain_graph=True)
        g2 = torch.autograd.grad(loss, ts)
        res.append((out.detach(), g1, g2))
    (o0, a0, b0), (o1, a1, b1) = res
    assert torch.equal(o0, o1)
    for x, y, z in zip(a0, a1, b1):
        assert torch.equal(x, y) and torch.equal(y, z)


def test_gdn_config4_size_all_heads_vs_fp64_torch():
    """Config-4 shape (16k tokens, 16 k / 32 v heads, D=128, bf16 inputs): every
    head of out, dq, dk, dv, dg and dbeta against the float64 torch checker on
    the same (bf16-rounded) inputs, at the bf16 bar of 2e-2."""
    from oracle.gdn_torch import gdn_tree_torch
    S, Hk, H, D = 16384, 16, 32, 128
    info, q, k, v, gg, bt, _, do, _ = _case(4, S, Hk, H, D, 16, 300)
    rnd = lambda x: torch.tensor(x, dtype=torch.bfloat16).double().numpy()
    q, k, v = rnd(q), rnd(k), rnd(v)
    got = run_gdn(q, k, v, gg, bt, info.chunk_boundaries, info.chunk_parent_map, None, True, do,
                  None, torch.bfloat16)
    ts = [torch.tensor(x, dtype=torch.float64, device=DEV, requires_grad=True)
          for x in (q, k, v, gg, bt)]
    out, _ = gdn_tree_torch(*ts, info.chunk_boundaries, info.chunk_parent_map, None, True)
    (out * torch.tensor(do, dtype=torch.float64, device=DEV)).sum().backward()
    ref = {"out": out.detach(), "dq": ts[0].grad, "dk": ts[1].grad, "dv": ts[2].grad,
           "dg": ts[3].grad, "dbeta": ts[4].grad}
    ref = {key: t.cpu().numpy() for key, t in ref.items()}
    for key, r in ref.items():
        assert np.isfinite(got[key]).all(), key
        assert rel(got[key], r) < 2e-2, (key, rel(got[key], r))
    # per head: a wrong head mapping cannot hide behind another head's magnitudes
    for h in range(H):
        for key in ("out", "dv", "dg", "dbeta"):
            assert rel(got[key][:, :, h], ref[key][:, :, h]) < 2e-2, (key, h)
    for h in range(Hk):
        for key in ("dq", "dk"):
            assert rel(got[key][:, :, h], ref[key][:, :, h]) < 2e-2, (key, h)


class _Conv:
    """The attributes of a GatedDeltaNet layer that the conv drop-in reads."""

    def __init__(self, w, b=None):
        self.conv1d = torch.nn.Conv1d(w.shape[0], w.shape[0], w.shape[1], groups=w.shape[0],
                                      padding=w.shape[1] - 1, bias=b is not None).to(DEV)
        with torch.no_grad():
            self.conv1d.weight.copy_(torch.tensor(w[:, None, :], dtype=torch.float32))
            if b is not None:
                self.conv1d.bias.copy_(torch.tensor(b, dtype=torch.float32))
        self.conv_kernel_size = w.shape[1]
        self.activation = "silu"
        self.causal_conv1d_fn = None


@pytest.mark.parametrize("name", ["conv_tree", "conv_short_nodes"])
def test_tree_conv_matches_reference_fixture(name):
    d = load(name)
    ssm = _Conv(d["weight"])
    x = torch.tensor(d["x"], dtype=torch.float32, device=DEV, requires_grad=True)
    bounds = [tuple(b) for b in d["chunk_boundaries"].tolist()]
    y = _tree_correct_conv_varlen(ssm, x, bounds, d["chunk_parent_map"].tolist())
    y.backward(torch.tensor(d["dout"], dtype=torch.float32, device=DEV))
    f = lambda t: t.detach().double().cpu().numpy()
    assert rel(f(y), d["out"]) < 1e-5
    assert rel(f(x.grad), d["dx"]) < 1e-5
    assert rel(f(ssm.conv1d.weight.grad)[:, 0], d["dweight"]) < 1e-5


@pytest.mark.parametrize("C,K,dtype,tol", [(64, 4, torch.float32, 1e-5),
                                            (13, 2, torch.float32, 1e-5),
                                            (21, 3, torch.float32, 1e-5),
                                            (9, 8, torch.float32, 1e-5),
                                            (40, 4, torch.bfloat16, 2e-2)])
def test_tree_conv_random_tree_with_bias_vs_oracle(C, K, dtype, tol):
    """Channel counts off the kernels' 8-channel blocks, every window length
    class, and bf16 (inputs rounded to bf16 for the float64 oracle too)."""
    info = tt.build_dfs_tree_info(random_branching_tree(9, 3000, 1, 40))
    g_ = np.random.default_rng(9 + C + K)
    x = g_.standard_normal((2, C, info.N))
    w = g_.standard_normal((C, K)) * 0.5
    b = g_.standard_normal(C) * 0.1
    dy = g_.standard_normal((2, C, info.N))
    if dtype == torch.bfloat16:
        x, dy = (torch.tensor(a).to(dtype).double().numpy() for a in (x, dy))
    ssm = _Conv(w, b)
    xt = torch.tensor(x, dtype=dtype, device=DEV, requires_grad=True)
    y = _tree_correct_conv_varlen(ssm, xt, info.chunk_boundaries, info.chunk_parent_map)
    y.backward(torch.tensor(dy, dtype=dtype, device=DEV))
    ref_y, _ = O.tree_conv_fwd(x, w, info.chunk_boundaries, info.chunk_parent_map, b)
    dx, dw, db = O.tree_conv_bwd(x, w, info.chunk_boundaries, info.chunk_parent_map, dy, b)
    f = lambda t: t.detach().double().cpu().numpy()
    assert rel(f(y), ref_y) < tol
    assert rel(f(xt.grad), dx) < tol
    assert rel(f(ssm.conv1d.weight.grad)[:, 0], dw) < tol
    assert rel(f(ssm.conv1d.bias.grad), db) < tol


def _gemm_mode(mode):
    from tree_training_b200 import _lib
    return _lib.lib().tt_gdn_set_gemm_mode(mode)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-5), (torch.bfloat16, 1e-2)])
def test_gdn_tensor_core_gemm_matches_cuda_core_gemm(dtype, tol):
    """The same forward and backward with the segmented GEMMs on the tensor
    cores (default: 3xTF32 products for fp32 inputs, TF32 for bf16, operands
    staged by TMA, decay masks applied in the K K^T / Q K^T epilogues), on the
    tensor cores with cp.async staging (masks applied by their own kernel) and
    on the CUDA cores (fp32 FMA).  The tree has an empty node, one-token nodes,
    and nodes past one 128-row tile (up to 300 tokens), D = 128 and GQA 2:4."""
    lens = [300, 0, 1, 129, 7, 128, 64, 1, 250, 33]
    parents = [-1, 0, 0, 2, 3, 3, 1, 6, 0, 8]
    bounds, s0 = [], 0
    for L in lens:
        bounds.append((s0, s0 + L))
        s0 += L
    S, Hk, H, D = s0, 2, 4, 128
    g_ = np.random.default_rng(31)
    q = g_.standard_normal((1, S, Hk, D))
    k = g_.standard_normal((1, S, Hk, D))
    v = g_.standard_normal((1, S, H, D)) * 0.5
    gg = -np.log1p(np.exp(-g_.standard_normal((1, S, H))))
    bt = 1.0 / (1.0 + np.exp(-g_.standard_normal((1, S, H))))
    s0_ = g_.standard_normal((1, H, D, D)) * 0.05
    do = g_.standard_normal((1, S, H, D))
    dl = g_.standard_normal((1, H, D, D))
    res = []
    for mode in (0, 2, 4):
        prev = _gemm_mode(mode)
        try:
            res.append(run_gdn(q, k, v, gg, bt, bounds, parents, s0_, True, do, dl, dtype))
        finally:
            _gemm_mode(prev)
    tt.check_device_status(DEV)
    for key in ("out", "last", "dq", "dk", "dv", "dg", "dbeta", "dinit"):
        assert np.isfinite(res[0][key]).all(), key
        for other in res[1:]:
            assert rel(res[0][key], other[key]) < tol, (key, rel(res[0][key], other[key]))
    # and the tensor-core result against the float64 oracle at the GDN bar, on
    # the same tree without its empty node (which the reference's algorithm,
    # like the oracle, cannot take: it reads the node's last cumulative gate)
    if dtype == torch.float32:
        keep = [i for i, L in enumerate(lens) if L > 0]
        remap = {old: new for new, old in enumerate(keep)}
        b2 = [bounds[i] for i in keep]
        p2 = []
        for i in keep:
            par = parents[i]
            while par >= 0 and lens[par] == 0:      # an empty node passes its parent's state on
                par = parents[par]
            p2.append(remap[par] if par >= 0 else -1)
        got = run_gdn(q, k, v, gg, bt, b2, p2, s0_, True, do, dl, dtype)
        ref = _oracle(_Info(b2, p2), q, k, v, gg, bt, s0_, do, dl)
        for key in ("out", "last", "dq", "dk", "dv", "dg", "dbeta", "dinit"):
            assert rel(got[key], ref[key]) < 2e-5, (key, rel(got[key], ref[key]))


class _Info:
    def __init__(self, bounds, parents):
        self.chunk_boundaries, self.chunk_parent_map = bounds, parents


@pytest.mark.parametrize("K,dtype", [(4, torch.bfloat16), (4, torch.float32), (2, torch.float32),
                                     (5, torch.bfloat16), (7, torch.float32)])
def test_tree_conv_four_token_kernels_match_one_token_kernels(K, dtype):
    """The conv kernels that take 4 tokens per thread (S % 4 == 0, 16-byte
    aligned rows) against the 1-token kernels on the same data placed one
    element off alignment: the same arithmetic per output, so out, dx and the
    input gradient of the SiLU agree bit for bit; dw and db are summed in
    another order."""
    from tree_training_b200 import _lib
    from tree_training_b200.gdn import TreeConvPlan, _tree_arrays
    info = tt.build_dfs_tree_info(random_branching_tree(17, 4000, 1, 60))
    S, C = info.N, 24
    assert S % 4 == 0
    bounds, parents = _tree_arrays(info.chunk_boundaries, info.chunk_parent_map)
    plan = TreeConvPlan(bounds, parents, K, DEV)
    g = torch.Generator(device=DEV).manual_seed(K)
    x = torch.randn(C * S, generator=g, device=DEV).to(dtype)
    dy = torch.randn(C * S, generator=g, device=DEV).to(dtype)
    w = torch.randn(C, K, generator=g, device=DEV) * 0.5
    b = torch.randn(C, generator=g, device=DEV) * 0.1
    dt = {torch.float32: _lib.TT_F32, torch.bfloat16: _lib.TT_BF16}[dtype]
    stream = torch.cuda.current_stream(DEV).cuda_stream

    def run(off):
        xb = torch.zeros(C * S + off, dtype=dtype, device=DEV)
        dyb = torch.zeros_like(xb)
        xb[off:] = x
        dyb[off:] = dy
        out = torch.zeros_like(xb)
        dx = torch.zeros_like(xb)
        dw = torch.zeros(C, K, device=DEV)
        db = torch.zeros(C, device=DEV)
        ws_bytes = int(_lib.lib().tt_tree_conv_bwd_workspace_size(C, S, K))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        es = xb.element_size()
        _lib.call("tt_tree_conv_fwd", dt, C, S, K, xb.data_ptr() + off * es, w.data_ptr(),
                  b.data_ptr(), plan.pred.data_ptr(), out.data_ptr() + off * es, stream)
        _lib.call("tt_tree_conv_bwd", dt, C, S, K, xb.data_ptr() + off * es, w.data_ptr(),
                  b.data_ptr(), plan.pred.data_ptr(), plan.succ_ptr.data_ptr(),
                  plan.succ_tok.data_ptr(), plan.succ_lag.data_ptr(),
                  dyb.data_ptr() + off * es, dx.data_ptr() + off * es, dw.data_ptr(),
                  db.data_ptr(), ws.data_ptr(), ws_bytes, stream)
        torch.cuda.synchronize()
        return out[off:], dx[off:], dw, db

    quad, single = run(0), run(1)
    assert torch.equal(quad[0], single[0])
    assert torch.equal(quad[1], single[1])
    for a, r in zip(quad[2:], single[2:]):
        assert rel(a.cpu().numpy(), r.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_token_major_conv_and_in_place_gdn_rows_match_packed(dtype):
    """The layer's path with the conv output in token-major memory (q / k / v
    split off it as views, read in place by the GDN, the conv gradient read
    token-major) against the same path with every tensor packed: the conv
    output, the GDN output and dq/dk/dv/dg/dbeta and dx agree bit for bit (the
    same arithmetic per element); dw is summed over other token blocks."""
    from tree_training_b200.gdn import _conv_plan, _conv_fwd_op, _tree_arrays
    Hk, H, D, K = 2, 4, 64, 4
    C = 2 * Hk * D + H * D
    info = tt.build_dfs_tree_info(random_branching_tree(23, 1200, 16, 120))
    S = info.N
    assert S % 8 == 0 and S % 128      # whole 16-byte token chunks; a partial last tile
    bounds, parents = _tree_arrays(info.chunk_boundaries, info.chunk_parent_map)
    plan = _conv_plan(bounds, parents, K, DEV)
    gen = torch.Generator(device=DEV).manual_seed(5)
    x0 = torch.randn(C, S, generator=gen, device=DEV).to(dtype)
    w0 = torch.randn(C, K, generator=gen, device=DEV) * 0.5
    g0 = torch.nn.functional.logsigmoid(torch.randn(S, H, generator=gen, device=DEV))
    b0 = torch.sigmoid(torch.randn(S, H, generator=gen, device=DEV))
    do = torch.randn(1, S, H, D, generator=gen, device=DEV).to(dtype)

    def run(token_major):
        x = x0.clone().requires_grad_(True)
        w = w0.clone().requires_grad_(True)
        gg = g0.clone().unsqueeze(0).requires_grad_(True)
        bt = b0.clone().unsqueeze(0).requires_grad_(True)
        y = _conv_fwd_op(x, w, w.new_empty(0), False, plan.pred, plan.succ_ptr, plan.succ_tok,
                         plan.succ_lag, token_major)
        assert (y.stride() == (1, C)) == token_major
        q, k, v = torch.split(y.t().unsqueeze(0), [Hk * D, Hk * D, H * D], dim=-1)
        q, k, v = q.reshape(1, S, Hk, D), k.reshape(1, S, Hk, D), v.reshape(1, S, H, D)
        if not token_major:
            q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        else:
            assert q.stride(1) == C and not q.is_contiguous()
        out, _ = torch_chunk_gated_delta_rule_tree_varlen(
            q, k, v, gg, bt, bounds, parents, use_qk_l2norm_in_kernel=True)
        out.backward(do)
        torch.cuda.synchronize()
        return y.detach().contiguous(), out.detach(), x.grad, w.grad, gg.grad, bt.grad

    tm, pk = run(True), run(False)
    for a, b in zip(tm[:3], pk[:3]):        # conv out, GDN out, conv dx
        assert torch.equal(a, b)
    assert torch.equal(tm[4], pk[4]) and torch.equal(tm[5], pk[5])   # dg, dbeta
    assert rel(tm[3].cpu().numpy(), pk[3].cpu().numpy()) < 1e-5       # dw


@pytest.mark.parametrize("K,dtype", [(1, torch.bfloat16), (2, torch.bfloat16), (4, torch.float32),
                                     (4, torch.bfloat16), (7, torch.bfloat16), (7, torch.float32),
                                     (8, torch.bfloat16)])
def test_tree_conv_token_major_kernels_match_channel_major(K, dtype):
    """The shared-memory-tiled token-major conv kernels (output / output
    gradient as [S, C] rows) against the channel-major ones on a tree of
    many short nodes (windows that leave a 128-token tile at node starts) with
    a partial last tile and a partial last 64-channel tile: out and dx bit for
    bit, dw and db (summed over other token blocks) to 1e-5."""
    from tree_training_b200 import _lib
    from tree_training_b200.gdn import TreeConvPlan, _tree_arrays
    info = tt.build_dfs_tree_info(random_branching_tree(41, 3000, 2, 40))
    S, C = info.N, 200
    assert S % 8 == 0 and S % 128 and C % 64
    bounds, parents = _tree_arrays(info.chunk_boundaries, info.chunk_parent_map)
    plan = TreeConvPlan(bounds, parents, K, DEV)
    g = torch.Generator(device=DEV).manual_seed(K + 100)
    x = torch.randn(C, S, generator=g, device=DEV).to(dtype)
    dy = torch.randn(C, S, generator=g, device=DEV).to(dtype)
    w = torch.randn(C, K, generator=g, device=DEV) * 0.5
    b = torch.randn(C, generator=g, device=DEV) * 0.1
    dt = {torch.float32: _lib.TT_F32, torch.bfloat16: _lib.TT_BF16}[dtype]
    stream = torch.cuda.current_stream(DEV).cuda_stream
    ws_bytes = int(_lib.lib().tt_tree_conv_bwd_workspace_size(C, S, K))

    def run(tm):
        out = torch.empty((S, C) if tm else (C, S), dtype=dtype, device=DEV)
        _lib.call("tt_tree_conv_fwd_ex", dt, C, S, K, x.data_ptr(), w.data_ptr(), b.data_ptr(),
                  plan.pred.data_ptr(), out.data_ptr(), int(tm), stream)
        dyl = dy.t().contiguous() if tm else dy
        dx = torch.empty_like(x)
        dw = torch.zeros(C, K, device=DEV)
        db = torch.zeros(C, device=DEV)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        _lib.call("tt_tree_conv_bwd_ex", dt, C, S, K, x.data_ptr(), w.data_ptr(), b.data_ptr(),
                  plan.pred.data_ptr(), plan.succ_ptr.data_ptr(), plan.succ_tok.data_ptr(),
                  plan.succ_lag.data_ptr(), dyl.data_ptr(), int(tm), dx.data_ptr(),
                  dw.data_ptr(), db.data_ptr(), ws.data_ptr(), ws_bytes, stream)
        torch.cuda.synchronize()
        return (out.t() if tm else out), dx, dw, db

    tm, cm = run(True), run(False)
    assert torch.equal(tm[0], cm[0])
    assert torch.equal(tm[1], cm[1])
    for a, r in zip(tm[2:], cm[2:]):
        assert rel(a.cpu().numpy(), r.cpu().numpy()) < 1e-5
