"""Tree attention at the benchmark sizes, every element against an fp32 torch reference.

The reference here is computed on the GPU with plain torch in fp32 (TF32 off),
independently of this package's kernels and packer: the key intervals come
from the CPU oracle's ``build_dfs_tree_info`` (pinned bit-exactly to the
reference's own packer by ``tests/test_oracle_golden.py``), the visibility
mask is the dense form of the reference's ``attn_mask_bool``
(dfs_tree_forward.py:157-172), and the attention is softmax(Q K^T s + M) V
with its gradients written out (the math of SDPA's backward).  The inputs are
the same bf16 values for both sides; the bar is the bf16 bar, max_rel < 2e-2
with max_rel = max|a - b| / max|b| over the whole tensor.

* config 2: the bench's own tree (seed 1000: 16,378 tokens, 32 q / 8 kv
  heads, D=128): out, dQ, dK and dV, every element of every head.
* config 3: the bench's first 65,536-token agentic tree (40 q / 8 kv heads):
  every element of out and dQ of the q heads of kv heads 0 and 7, and of dK
  and dV of those two kv heads, in row chunks (the dense mask of a 64k tree
  does not fit one buffer).
"""
import contextlib

import numpy as np
import pytest
import torch

from oracle import tree_oracle as O

import tree_training_b200 as tt
from tree_training_b200.synthetic import agentic_tree, bfs_tree

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
D = 128


@contextlib.contextmanager
def _fp32_matmul():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _oracle_intervals(roots):
    info = O.build_dfs_tree_info(roots)
    lo, hi = O.key_intervals(info.chunk_boundaries, info.chunk_parent_map, info.N)
    return (torch.from_numpy(lo.astype(np.int64)).to(DEV),
            torch.from_numpy(hi.astype(np.int64)).to(DEV), info.N)


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _kernel(q, k, v, do, roots):
    meta = tt.build_dfs_tree_info(roots).attn_meta()
    qg, kg, vg = (x.clone().requires_grad_(True) for x in (q, k, v))
    out = tt.tree_attention(qg, kg, vg, meta)
    out.backward(do)
    torch.cuda.synchronize()
    tt.check_device_status(DEV)
    return out.detach(), qg.grad, kg.grad, vg.grad


def _reference_heads(q, k, v, do, lo, hi, heads, kv_head, chunk):
    """fp32 out / dQ for the q heads ``heads`` (all sharing ``kv_head``) and
    that kv head's dK / dV restricted to those heads' contributions.  Rows are
    processed in chunks of ``chunk``; a chunk [r0, r1) only meets keys j < r1
    (every visible key has j <= row).  Two passes: LSE and O first, then the
    gradients (they need delta = rowsum(dO * O))."""
    n = q.shape[0]
    s = D ** -0.5
    kf, vf = k[:, kv_head].float(), v[:, kv_head].float()
    dk = torch.zeros(n, D, device=DEV)
    dv = torch.zeros(n, D, device=DEV)
    outs, dqs = {}, {}
    for h in heads:
        qf, dof = q[:, h].float(), do[:, h].float()
        lse = torch.empty(n, device=DEV)
        o = torch.empty(n, D, device=DEV)
        dq = torch.empty(n, D, device=DEV)
        for r0 in range(0, n, chunk):
            r1 = min(n, r0 + chunk)
            rows = torch.arange(r0, r1, device=DEV)[:, None]
            vis = (rows >= lo[None, :r1]) & (rows < hi[None, :r1])
            sc = (qf[r0:r1] @ kf[:r1].T) * s
            sc.masked_fill_(~vis, float("-inf"))
            lse[r0:r1] = torch.logsumexp(sc, dim=1)
            p = torch.exp(sc - lse[r0:r1, None])
            o[r0:r1] = p @ vf[:r1]
        delta = (dof * o).sum(1)
        for r0 in range(0, n, chunk):
            r1 = min(n, r0 + chunk)
            rows = torch.arange(r0, r1, device=DEV)[:, None]
            vis = (rows >= lo[None, :r1]) & (rows < hi[None, :r1])
            sc = (qf[r0:r1] @ kf[:r1].T) * s
            sc.masked_fill_(~vis, float("-inf"))
            p = torch.exp(sc - lse[r0:r1, None])
            dp = dof[r0:r1] @ vf[:r1].T
            ds = p * (dp - delta[r0:r1, None])
            dq[r0:r1] = (ds @ kf[:r1]) * s
            dk[:r1] += (ds.T @ qf[r0:r1]) * s
            dv[:r1] += p.T @ dof[r0:r1]
        outs[h], dqs[h] = o, dq
    return outs, dqs, dk, dv


def _inputs(n, hq, hkv, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=DEV) * 0.5).to(torch.bfloat16)
    return mk(n, hq, D), mk(n, hkv, D), mk(n, hkv, D), mk(n, hq, D)


def test_config2_every_element_vs_fp32_torch():
    roots = bfs_tree(1000, 16384, 64, 512, 2048)          # bench.py's rank-0 tree
    lo, hi, n = _oracle_intervals(roots)
    hq, hkv = 32, 8
    q, k, v, do = _inputs(n, hq, hkv, 0)
    out, dq, dk, dv = _kernel(q, k, v, do, roots)
    rep = hq // hkv
    ref_o = torch.empty(n, hq, D, device=DEV)
    ref_dq = torch.empty(n, hq, D, device=DEV)
    ref_dk = torch.empty(n, hkv, D, device=DEV)
    ref_dv = torch.empty(n, hkv, D, device=DEV)
    with _fp32_matmul():
        for kh in range(hkv):
            heads = list(range(kh * rep, (kh + 1) * rep))
            o_, dq_, dk_, dv_ = _reference_heads(q, k, v, do, lo, hi, heads, kh, n)
            for h in heads:
                ref_o[:, h], ref_dq[:, h] = o_[h], dq_[h]
            ref_dk[:, kh], ref_dv[:, kh] = dk_, dv_
    torch.cuda.synchronize()
    for name, a, b in (("out", out, ref_o), ("dq", dq, ref_dq), ("dk", dk, ref_dk),
                       ("dv", dv, ref_dv)):
        assert torch.isfinite(a.float()).all(), name
        assert _rel(a, b) < 2e-2, (name, _rel(a, b))
    # per head as well: a wrong tile schedule in one head cannot hide behind
    # another head's larger magnitudes
    for h in range(hq):
        assert _rel(out[:, h], ref_o[:, h]) < 2e-2, ("out", h)
        assert _rel(dq[:, h], ref_dq[:, h]) < 2e-2, ("dq", h)
    for kh in range(hkv):
        assert _rel(dk[:, kh], ref_dk[:, kh]) < 2e-2, ("dk", kh)
        assert _rel(dv[:, kh], ref_dv[:, kh]) < 2e-2, ("dv", kh)


def test_config3_two_kv_groups_every_element_vs_fp32_torch():
    roots = agentic_tree(1000)                            # bench.py --workload attn3, tree 0
    lo, hi, n = _oracle_intervals(roots)
    assert n == 65536
    hq, hkv = 40, 8
    rep = hq // hkv
    q, k, v, do = _inputs(n, hq, hkv, 3)
    out, dq, dk, dv = _kernel(q, k, v, do, roots)
    with _fp32_matmul():
        for kh in (0, hkv - 1):
            heads = list(range(kh * rep, (kh + 1) * rep))
            o_, dq_, dk_, dv_ = _reference_heads(q, k, v, do, lo, hi, heads, kh, 4096)
            for h in heads:
                assert _rel(out[:, h], o_[h]) < 2e-2, ("out", h, _rel(out[:, h], o_[h]))
                assert _rel(dq[:, h], dq_[h]) < 2e-2, ("dq", h, _rel(dq[:, h], dq_[h]))
            assert _rel(dk[:, kh], dk_) < 2e-2, ("dk", kh, _rel(dk[:, kh], dk_))
            assert _rel(dv[:, kh], dv_) < 2e-2, ("dv", kh, _rel(dv[:, kh], dv_))
