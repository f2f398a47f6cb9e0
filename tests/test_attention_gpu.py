"""Tree attention parity on a B200: CUDA kernels vs the oracle / reference.

* golden fixtures made by the reference (HF SDPA + dense mask), fp32 path,
  max_rel < 1e-4 (the reference's fp32 bar);
* bf16 tcgen05 path vs the float64 oracle on random trees, max_rel < 2e-2;
* tensor-core path vs the exact CUDA-core path on the same inputs;
* full config-2 size: sampled rows vs the CPU oracle, plus the exact path.
"""
import random

import numpy as np
import pytest
import torch

from oracle import tree_oracle as O
from tests.golden_util import Node, load

import tree_training_b200 as tt
from tree_training_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


def run(q, k, v, meta, dout, dtype, scale=None):
    """q [n_q,hq,D], k/v [n_kv,hkv,D], dout [n_q,hq,D] (numpy) -> float64 numpy
    out, dq, dk, dv through the custom op and autograd."""
    qt = torch.tensor(q, dtype=dtype, device=DEV, requires_grad=True)
    kt = torch.tensor(k, dtype=dtype, device=DEV, requires_grad=True)
    vt = torch.tensor(v, dtype=dtype, device=DEV, requires_grad=True)
    out = tt.tree_attention(qt, kt, vt, meta, scale)
    out.backward(torch.tensor(dout, dtype=dtype, device=DEV))
    torch.cuda.synchronize()
    tt.check_device_status(DEV)
    f = lambda t: t.detach().double().cpu().numpy()
    return f(out), f(qt.grad), f(kt.grad), f(vt.grad)


def _allowed(d):
    n_rows, n_cols = int(d["n_rows"]), int(d["n_cols"])
    return np.unpackbits(d["allowed_bits"])[: n_rows * n_cols].reshape(n_rows, n_cols).astype(bool)


@pytest.mark.parametrize("name", ["attn_forest47_f64", "attn_rand_f64", "attn_gateway_f64"])
def test_fp32_path_matches_reference_fixture(name):
    d = load(name)
    allowed = _allowed(d)
    lo, hi = O.intervals_from_mask(allowed)
    meta = tt.TreeAttnMeta(allowed.shape[0], lo, hi)
    q = d["q"][0].transpose(1, 0, 2)
    k = d["k"][0].transpose(1, 0, 2)
    v = d["v"][0].transpose(1, 0, 2)
    do = d["dout"][0]
    out, dq, dk, dv = run(q, k, v, meta, do, torch.float32, float(d["scale"]))
    assert rel(out, d["out"][0]) < 1e-4
    assert rel(dq, d["dq"][0].transpose(1, 0, 2)) < 1e-4
    assert rel(dk, d["dk"][0].transpose(1, 0, 2)) < 1e-4
    assert rel(dv, d["dv"][0].transpose(1, 0, 2)) < 1e-4


def random_tree(rng, n_target, len_lo, len_hi, branch=(2, 4), root_len=None, max_depth=6):
    """Config-2 style generator: BFS expansion, stops at the token budget."""
    root = Node([0] * (root_len or rng.randint(len_lo, len_hi)))
    total = len(root.token_ids)
    frontier = [(root, 0)]
    while frontier and total < n_target:
        nxt = []
        for node, depth in frontier:
            if depth >= max_depth:
                continue
            for _ in range(rng.randint(*branch)):
                L = rng.randint(len_lo, len_hi)
                if total + L > n_target:
                    continue
                c = node.add_child([0] * L)
                total += L
                nxt.append((c, depth + 1))
        frontier = nxt
    return [root]


def make_case(seed, n_target, hq, hkv, D, len_lo, len_hi, past=0, root_len=None):
    rng = random.Random(seed)
    roots = random_tree(rng, n_target, len_lo, len_hi, root_len=root_len)
    info = tt.build_dfs_tree_info(roots)
    if past:
        glo = np.zeros(past, np.int32)
        ghi = np.where(np.array([rng.random() < 0.5 for _ in range(past)]), info.N, 0)
        meta = info.attn_meta(glo, ghi.astype(np.int32))
    else:
        meta = info.attn_meta()
    g = np.random.default_rng(seed)
    q = g.standard_normal((meta.n_q, hq, D)) * 0.5
    k = g.standard_normal((meta.n_kv, hkv, D)) * 0.5
    v = g.standard_normal((meta.n_kv, hkv, D)) * 0.5
    do = g.standard_normal((meta.n_q, hq, D)) * 0.5
    return meta, q, k, v, do


def oracle_all(meta, q, k, v, do):
    allowed = meta.dense_mask()
    tr = lambda x: x.transpose(1, 0, 2)
    out, _ = O.attention_fwd(tr(q), tr(k), tr(v), allowed, q.shape[-1] ** -0.5)
    dq, dk, dv = O.attention_bwd(tr(q), tr(k), tr(v), allowed, q.shape[-1] ** -0.5, tr(do))
    return tr(out), tr(dq), tr(dk), tr(dv)


def bf16_round(x):
    return torch.tensor(x, dtype=torch.bfloat16).double().numpy()


@pytest.mark.parametrize("seed,n,hq,hkv,past", [(1, 700, 4, 1, 0), (2, 1000, 8, 2, 0),
                                                (3, 1500, 5, 1, 37), (4, 333, 4, 4, 130)])
def test_bf16_tensor_core_path_vs_oracle(seed, n, hq, hkv, past):
    meta, q, k, v, do = make_case(seed, n, hq, hkv, 128, 16, 200, past)
    q, k, v, do = map(bf16_round, (q, k, v, do))
    ref = oracle_all(meta, q, k, v, do)
    got = run(q, k, v, meta, do, torch.bfloat16)
    for name, a, b in zip(("out", "dq", "dk", "dv"), got, ref):
        assert rel(a, b) < 2e-2, name


@pytest.mark.parametrize("seed,n,D", [(5, 600, 64), (6, 400, 32), (7, 900, 128)])
def test_fp32_path_vs_oracle_random_trees(seed, n, D):
    meta, q, k, v, do = make_case(seed, n, 4, 2, D, 1, 90, past=11)
    ref = oracle_all(meta, q, k, v, do)
    got = run(q, k, v, meta, do, torch.float32)
    for name, a, b in zip(("out", "dq", "dk", "dv"), got, ref):
        assert rel(a, b) < 1e-4, name


def test_fp16_path_vs_oracle():
    meta, q, k, v, do = make_case(8, 800, 4, 2, 128, 16, 300)
    f16 = lambda x: torch.tensor(x, dtype=torch.float16).double().numpy()
    q, k, v, do = map(f16, (q, k, v, do))
    ref = oracle_all(meta, q, k, v, do)
    got = run(q, k, v, meta, do, torch.float16)
    for name, a, b in zip(("out", "dq", "dk", "dv"), got, ref):
        assert rel(a, b) < 1e-2, name


def test_tensor_core_forward_matches_exact_path():
    meta, q, k, v, do = make_case(9, 3000, 8, 2, 128, 64, 512, root_len=700)
    qt, kt, vt = (torch.tensor(x, dtype=torch.bfloat16, device=DEV) for x in (q, k, v))
    a = tt.tree_attention(qt, kt, vt, meta).float()
    prev = _lib.set_kernel_path(1)
    try:
        meta2 = tt.TreeAttnMeta(meta.n_q, meta.kv_lo, meta.kv_hi)
        b = tt.tree_attention(qt, kt, vt, meta2).float()
    finally:
        _lib.set_kernel_path(prev)
    torch.cuda.synchronize()
    assert float((a - b).abs().max() / b.abs().max()) < 1e-2


@pytest.mark.parametrize("seed,n,hq,hkv,past", [(11, 2500, 8, 2, 50), (12, 4000, 10, 2, 0),
                                                (13, 129, 4, 1, 1)])
def test_tensor_core_backward_matches_exact_path(seed, n, hq, hkv, past):
    """Full fwd+bwd through both kernel paths on the same bf16 inputs."""
    meta, q, k, v, do = make_case(seed, n, hq, hkv, 128, 32, 400, past)
    res = []
    for path in (0, 1):
        prev = _lib.set_kernel_path(path)
        try:
            m = tt.TreeAttnMeta(meta.n_q, meta.kv_lo, meta.kv_hi)
            res.append(run(q, k, v, m, do, torch.bfloat16))
        finally:
            _lib.set_kernel_path(prev)
    for name, a, b in zip(("out", "dq", "dk", "dv"), res[0], res[1]):
        assert rel(a, b) < 1.5e-2, name


def test_dense_mask_conversion_matches_packer():
    meta, *_ = make_case(10, 900, 1, 1, 32, 8, 100, past=21)
    m = torch.full((1, 1, meta.n_q, meta.n_kv), float("-inf"), device=DEV)
    m[0, 0][torch.from_numpy(meta.dense_mask()).to(DEV)] = 0.0
    got = tt.meta_from_dense_mask(m)
    nz = meta.kv_hi > meta.kv_lo
    assert np.array_equal(got.kv_lo[nz], meta.kv_lo[nz])
    assert np.array_equal(got.kv_hi[nz], meta.kv_hi[nz])
    assert np.all(got.kv_hi[~nz] <= got.kv_lo[~nz])
    bad = m.clone()
    bad[0, 0, 5, 0] = 0.0
    bad[0, 0, 3, 0] = float("-inf")
    bad[0, 0, 7, 0] = 0.0
    with pytest.raises(_lib.TTError):
        tt.meta_from_dense_mask(bad)


def _sampled_rows_oracle(meta, q, k, v, do, rows):
    """Exact float64 out / dq for a few query rows (each row is independent)."""
    hq, hkv, D = q.shape[1], k.shape[1], q.shape[2]
    rep = hq // hkv
    scale = D ** -0.5
    outs, dqs = [], []
    for i in rows:
        vis = np.nonzero((meta.kv_lo <= i) & (i < meta.kv_hi))[0]
        kk = np.repeat(k[vis], rep, axis=1)     # [n, hq, D]
        vv = np.repeat(v[vis], rep, axis=1)
        s = np.einsum("hd,nhd->hn", q[i], kk) * scale
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        o = np.einsum("hn,nhd->hd", p, vv)
        dp = np.einsum("hd,nhd->hn", do[i], vv)
        ds = p * (dp - (dp * p).sum(1, keepdims=True))
        outs.append(o)
        dqs.append(np.einsum("hn,nhd->hd", ds, kk) * scale)
    return np.stack(outs), np.stack(dqs)


def test_config2_full_size_sampled_rows_and_exact_cross_check():
    """16k-token tree, 32/8 heads, D=128, bf16 (the benchmark's config 2)."""
    rng = random.Random(2024)
    roots = random_tree(rng, 16384, 64, 512, root_len=2048)
    info = tt.build_dfs_tree_info(roots)
    meta = info.attn_meta()
    g = torch.Generator(device=DEV).manual_seed(0)
    mk = lambda *s: (torch.randn(*s, generator=g, device=DEV) * 0.5).to(torch.bfloat16)
    q, k, v, do = mk(meta.n_q, 32, 128), mk(meta.n_kv, 8, 128), mk(meta.n_kv, 8, 128), mk(meta.n_q, 32, 128)
    qg, kg, vg = (x.clone().requires_grad_(True) for x in (q, k, v))
    out = tt.tree_attention(qg, kg, vg, meta)
    out.backward(do)
    torch.cuda.synchronize()
    tt.check_device_status(DEV)
    rows = sorted(set([0, 1, 2047, 2048, meta.n_q - 1] + rng.sample(range(meta.n_q), 11)))
    f = lambda t: t.detach().double().cpu().numpy()
    qn, kn, vn, don = f(q), f(k), f(v), f(do)
    o_ref, dq_ref = _sampled_rows_oracle(meta, qn, kn, vn, don, rows)
    assert rel(f(out)[rows], o_ref) < 2e-2
    assert rel(f(qg.grad)[rows], dq_ref) < 2e-2
    assert torch.isfinite(kg.grad).all() and torch.isfinite(vg.grad).all()
    _check_grad_identities(do, kg.grad, vg.grad, 32 // 8)


class _Rows:
    """A few rows of a [n, heads, D] array, indexed by their row numbers."""

    def __init__(self, rows, data):
        self._d = {r: data[i] for i, r in enumerate(rows)}
        self.shape = (None,) + data.shape[1:]

    def __getitem__(self, i):
        return self._d[i]


def _check_grad_identities(do, dk, dv, rep):
    """Size-independent checks of every dK/dV entry: each row of P sums to 1, so
    sum_j dV_j = sum over the group's query rows and heads of dO; each row of dS
    sums to 0, so sum_j dK_j = 0."""
    n_q, hq, D = do.shape
    hkv = dv.shape[1]
    do_sum = do.float().sum(0).view(hkv, rep, D).sum(1)          # [hkv, D]
    dv_sum = dv.float().sum(0)
    assert float((dv_sum - do_sum).abs().max() / do_sum.abs().max()) < 1e-2
    dk_sum = dk.float().sum(0)
    dk_abs = dk.float().abs().sum(0)
    assert float((dk_sum.abs() / dk_abs.clamp_min(1e-30)).max()) < 1e-2


def test_config3_size_tree_sampled_rows_and_identities():
    """65,536-token agentic tree (the benchmark's config 3 shape), 40 q / 8 kv heads
    (an odd group of 5: the forward pairs heads and runs one single-head CTA
    per group), D=128, bf16."""
    from tree_training_b200.synthetic import agentic_tree
    info = tt.build_dfs_tree_info(agentic_tree(3000))
    meta = info.attn_meta()
    hq, hkv = 40, 8
    g = torch.Generator(device=DEV).manual_seed(3)
    mk = lambda *s: (torch.randn(*s, generator=g, device=DEV) * 0.5).to(torch.bfloat16)
    q, k, v, do = mk(meta.n_q, hq, 128), mk(meta.n_kv, hkv, 128), mk(meta.n_kv, hkv, 128), mk(meta.n_q, hq, 128)
    qg, kg, vg = (x.clone().requires_grad_(True) for x in (q, k, v))
    out = tt.tree_attention(qg, kg, vg, meta)
    out.backward(do)
    torch.cuda.synchronize()
    tt.check_device_status(DEV)
    rng = random.Random(3)
    rows = sorted(set([0, 8191, 8192, meta.n_q - 1] + rng.sample(range(meta.n_q), 8)))
    f = lambda t: t.detach().double().cpu().numpy()
    sel = lambda t: f(t[rows])
    kn, vn = f(k), f(v)
    o_ref, dq_ref = _sampled_rows_oracle(meta, _Rows(rows, sel(q)), kn, vn, _Rows(rows, sel(do)),
                                         rows)
    assert rel(f(out[rows]), o_ref) < 2e-2
    assert rel(f(qg.grad[rows]), dq_ref) < 2e-2
    assert torch.isfinite(kg.grad).all() and torch.isfinite(vg.grad).all()
    _check_grad_identities(do, kg.grad, vg.grad, hq // hkv)


def test_metadata_prefetched_on_upload_stream_matches_lazy_upload():
    """prefetch_tree_meta uploads the kernel metadata on a side stream (a
    training loop's prefetch stage); after the compute stream waits for that
    stream, the op's outputs and gradients are bit-identical to those of a
    call that uploads the metadata itself."""
    meta, q, k, v, do = make_case(21, 2000, 8, 2, 128, 32, 300, root_len=400)
    q, k, v, do = map(bf16_round, (q, k, v, do))
    ref = run(q, k, v, meta, do, torch.bfloat16)
    meta2 = tt.TreeAttnMeta(meta.n_q, meta.kv_lo, meta.kv_hi)
    up = torch.cuda.Stream(DEV)
    main = torch.cuda.current_stream(DEV)
    with torch.cuda.stream(up):
        assert tt.prefetch_tree_meta(meta2, DEV, torch.bfloat16, 128) is meta2
        # the large input copies of the same stage, then the inputs
        qt, kt, vt, dot = (torch.tensor(x, dtype=torch.bfloat16).pin_memory()
                           .to(DEV, non_blocking=True) for x in (q, k, v, do))
    main.wait_stream(up)
    for t in (qt, kt, vt, dot):
        t.record_stream(main)
    assert meta2.prefetched
    qt, kt, vt = (t.requires_grad_(True) for t in (qt, kt, vt))
    out = tt.tree_attention(qt, kt, vt, meta2)
    out.backward(dot)
    del meta2                      # the memory stays reserved for the compute stream's kernels
    torch.cuda.synchronize()
    tt.check_device_status(DEV)
    f = lambda t: t.detach().double().cpu().numpy()
    for name, a, b in zip(("out", "dq", "dk", "dv"), (f(out), f(qt.grad), f(kt.grad),
                                                      f(vt.grad)), ref):
        assert np.array_equal(a, b), name
