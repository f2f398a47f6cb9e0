"""The allocation-free backward entry point against the regular one.

``tt_tree_attn_bwd_noalloc`` exists for callers that cannot give the library a
scratch buffer and must not let it call cudaMalloc (a binding that mirrors the
reference's inputs-and-outputs attention call, or a runtime whose device
memory belongs to its own pooling allocator).  It keeps its scratch in a fixed
array inside the library, so these checks call it twice in a row (the array
keeps the previous call's contents) and compare both results with
``tt_tree_attn_bwd`` given a torch-allocated workspace.  The two entry points
run the same deterministic kernels in the same tile order on the same inputs,
so the results must be bit-identical.  This file is named to be collected
last; it also passes when run alone in a fresh process.
"""
import random

import numpy as np
import pytest
import torch

import tree_training_b200 as tt
from tree_training_b200 import _lib
from tree_training_b200.attention import attn_fwd_raw, tile_shape
from tree_training_b200.synthetic import bfs_tree

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _case(seed, n_tokens, hq, hkv, D, dtype, past):
    rng = random.Random(seed)
    info = tt.build_dfs_tree_info(bfs_tree(seed, n_tokens, 16, 200, 150))
    glo = np.zeros(past, np.int32)
    ghi = np.where(np.array([rng.random() < 0.5 for _ in range(past)]), info.N, 0)
    meta = info.attn_meta(glo, ghi.astype(np.int32))
    g = torch.Generator(device=DEV).manual_seed(seed)
    mk = lambda n, h: (torch.randn(n, h, D, generator=g, device=DEV) * 0.5).to(dtype)
    q, k, v, do = mk(meta.n_q, hq), mk(meta.n_kv, hkv), mk(meta.n_kv, hkv), mk(meta.n_q, hq)
    return meta, q, k, v, do


def _common_args(meta, q, k, v, do, out, lse, mb, scale, dq, dk, dv):
    n_q, hq, D = q.shape
    n_kv, hkv, _ = k.shape
    dt = {torch.float32: _lib.TT_F32, torch.bfloat16: _lib.TT_BF16}[q.dtype]
    return [dt, n_q, n_kv, hq, hkv, D,
            q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
            v.data_ptr(), v.stride(0), v.stride(1), out.data_ptr(), do.data_ptr(),
            do.stride(0), do.stride(1), lse.data_ptr(), mb["kv_lo"].data_ptr(),
            mb["kv_hi"].data_ptr(), mb["fwd_ptr"].data_ptr(), mb["fwd_list"].data_ptr(),
            mb["bwd_ptr"].data_ptr(), mb["bwd_list"].data_ptr(), float(scale),
            dq.data_ptr(), dq.stride(0), dq.stride(1), dk.data_ptr(), dk.stride(0),
            dk.stride(1), dv.data_ptr(), dv.stride(0), dv.stride(1)]


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64)])
def test_noalloc_backward_matches_workspace_backward(dtype, D):
    prev = _lib.set_kernel_path(0)
    try:
        meta, q, k, v, do = _case(31, 1500, 8, 2, D, dtype, past=37)
        scale = D ** -0.5
        mf = meta.device(DEV, *tile_shape(dtype, D, 0))
        mb = meta.device(DEV, *tile_shape(dtype, D, 1))
        out, lse = attn_fwd_raw(q, k, v, mf, scale)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        stream = torch.cuda.current_stream(DEV).cuda_stream
        new = lambda: (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v))

        ref = new()
        ws_bytes = int(_lib.lib().tt_tree_attn_bwd_workspace_size(
            _common_args(meta, q, k, v, do, out, lse, mb, scale, *ref)[0],
            q.shape[0], k.shape[0], q.shape[1], k.shape[1], D))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        _lib.call("tt_tree_attn_bwd", *_common_args(meta, q, k, v, do, out, lse, mb, scale, *ref),
                  ws.data_ptr(), ws_bytes, _lib.TT_BWD_ALL, status.data_ptr(), stream)

        for _ in range(2):                      # the shared array keeps the last call's data
            got = new()
            _lib.call("tt_tree_attn_bwd_noalloc",
                      *_common_args(meta, q, k, v, do, out, lse, mb, scale, *got),
                      status.data_ptr(), stream)
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            for a, b in zip(got, ref):
                assert torch.isfinite(a.float()).all()
                assert torch.equal(a, b)
    finally:
        _lib.set_kernel_path(prev)


def test_noalloc_rejects_problems_beyond_its_fixed_scratch():
    limit = int(_lib.lib().tt_tree_attn_bwd_noalloc_max_row_terms())
    hq = 64
    n_q = limit // hq + 1                       # hq * round_up(n_q, 128) > limit
    rc = _lib.lib().tt_tree_attn_bwd_noalloc(
        _lib.TT_BF16, n_q, n_q, hq, 8, 128, *([None, 0, 0] * 3), None, None, 0, 0, None,
        None, None, None, None, None, None, 1.0, *([None, 0, 0] * 3), None, None)
    assert rc == _lib.TT_ERR_WORKSPACE


def test_noalloc_rejects_more_keys_than_its_tile_order_holds():
    n_kv = 16384 * 128 + 1                      # one 128-key tile past the fixed array
    rc = _lib.lib().tt_tree_attn_bwd_noalloc(
        _lib.TT_BF16, 128, n_kv, 8, 8, 128, *([None, 0, 0] * 3), None, None, 0, 0, None,
        None, None, None, None, None, None, 1.0, *([None, 0, 0] * 3), None, None)
    assert rc == _lib.TT_ERR_WORKSPACE
