"""The tree GDN's segmented GEMM engines against a float64 reference.

``tt_gdn_segmented_gemm`` runs one list of segments (C = alpha A B + beta C per
segment and head) on the CUDA cores (engine 0), or on the tensor cores with
TF32 (1) or 3xTF32 (3) products, operands staged by TMA through per-segment
tensor maps (5 and 7: the same staged by cp.async copies): the engine behind
every product of tt_gdn_tree_fwd/_bwd.  The segments cover both storage orders of A and B
(contiguous along K or along M/N), ragged sizes around the 128-row tile and
the 32-wide K slice, empty K, and the triangular K ranges (kmode 1-4) with
operands that are triangular.
"""
import itertools

import numpy as np
import pytest
import torch

from tree_training_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _r4(x):
    return (x + 3) // 4 * 4


class _Buf:
    """A flat per-head float buffer that hands out 4-float-aligned regions."""

    def __init__(self):
        self.parts = []
        self.size = 0

    def put(self, arr):                       # arr [H, rows, cols] stored row-major
        off = self.size
        self.parts.append((off, arr))
        self.size = _r4(off + arr.shape[1] * arr.shape[2])
        return off

    def build(self, H):
        out = np.zeros((H, max(self.size, 4)), np.float32)
        for off, arr in self.parts:
            out[:, off:off + arr.shape[1] * arr.shape[2]] = arr.reshape(H, -1)
        return out


def _segments(rng, H):
    """Random segments; returns (rows of 13 int64, A, B, C buffers, expected)."""
    A, B, C = _Buf(), _Buf(), _Buf()
    rows, checks = [], []
    sizes = [(128, 128, 128), (1, 1, 1), (5, 129, 33), (300, 64, 257), (129, 300, 16),
             (64, 5, 128), (33, 128, 0), (200, 200, 200), (16, 16, 300), (127, 255, 31)]
    combos = list(itertools.product([True, False], [True, False]))
    for idx, ((M, N, K), (a_kc, b_kc)) in enumerate(itertools.product(sizes, combos)):
        kmode = 0
        a = rng.standard_normal((H, M, K)).astype(np.float32)
        b = rng.standard_normal((H, K, N)).astype(np.float32)
        tri = idx % 5
        if tri and M == K == N:
            # triangular operands for the kmodes: 1 A lower, 2 A upper, 3 B upper, 4 B lower
            if tri == 1:
                a = np.tril(a)
            elif tri == 2:
                a = np.triu(a)
            elif tri == 3:
                b = np.triu(b)
            else:
                b = np.tril(b)
            kmode = tri
        # storage: A K-contiguous -> rows of length K padded to 4; else transposed
        if a_kc:
            lda = _r4(max(K, 1))
            st = np.zeros((H, M, lda), np.float32)
            st[:, :, :K] = a
            a_off = A.put(st)
            a_rs, a_cs = lda, 1
        else:
            lda = _r4(max(M, 1))
            st = np.zeros((H, K, lda), np.float32)
            st[:, :, :M] = a.transpose(0, 2, 1)
            a_off = A.put(st)
            a_rs, a_cs = 1, lda
        if b_kc:                                # B[k][n] at n * ldb + k
            ldb = _r4(max(K, 1))
            st = np.zeros((H, N, ldb), np.float32)
            st[:, :, :K] = b.transpose(0, 2, 1)
            b_off = B.put(st)
            b_rs, b_cs = 1, ldb
        else:
            ldb = _r4(max(N, 1))
            st = np.zeros((H, K, ldb), np.float32)
            st[:, :, :N] = b
            b_off = B.put(st)
            b_rs, b_cs = ldb, 1
        ldc = _r4(max(N, 1))
        c0 = rng.standard_normal((H, M, ldc)).astype(np.float32)
        c_off = C.put(c0)
        rows.append([M, N, K, kmode, a_off, a_rs, a_cs, b_off, b_rs, b_cs, c_off, ldc, 1])
        checks.append((c_off, M, N, ldc, a.astype(np.float64) @ b.astype(np.float64),
                       c0[:, :, :N].astype(np.float64)))
    return np.asarray(rows, np.int64), A.build(H), B.build(H), C.build(H), checks


@pytest.mark.parametrize("engine,tol", [(0, 1e-5), (3, 1e-5), (1, 5e-3), (7, 1e-5), (5, 5e-3)])
def test_segmented_gemm_engines_vs_float64(engine, tol):
    H = 2
    rng = np.random.default_rng(engine + 7)
    segs, a, b, c, checks = _segments(rng, H)
    alpha, beta = 0.75, -0.5
    ta, tb = (torch.from_numpy(x).to(DEV) for x in (a, b))
    tc = torch.from_numpy(c).to(DEV)
    ws_bytes = int(_lib.lib().tt_gdn_segmented_gemm_workspace_size(len(segs), segs.ctypes.data))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    _lib.call("tt_gdn_segmented_gemm", engine, len(segs), segs.ctypes.data, H, ta.data_ptr(),
              ta.shape[1], tb.data_ptr(), tb.shape[1], tc.data_ptr(), tc.shape[1], alpha, beta,
              ws.data_ptr(), ws_bytes, torch.cuda.current_stream(DEV).cuda_stream)
    st = np.zeros(1, np.int32)
    _lib.call("tt_gdn_take_device_status", st.ctypes.data)
    assert int(st[0]) == 0
    got = tc.cpu().numpy().astype(np.float64)
    for i, (off, M, N, ldc, ab, c0) in enumerate(checks):
        if M == 0 or N == 0:
            continue
        out = got[:, off:off + M * ldc].reshape(H, M, ldc)[:, :, :N]
        ref = alpha * ab + beta * c0
        err = np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)
        assert err < tol, (i, segs[i].tolist(), err)
