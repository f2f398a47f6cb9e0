"""The stored-dS backward schedule (tt_tree_attn_bwd_stored) on a B200.

The dK/dV kernel stores every 16-bit dS tile it forms and a second kernel sums
dQ = scale * dS K from those tiles.  Checked here:

* against the float64 oracle at the bf16 / fp16 bar (max_rel < 2e-2), with
  gateway keys, GQA groups and ragged token counts;
* against the recompute schedule on the same inputs: dK and dV bit-identical
  (the same dK/dV kernel and tile order), dQ within 1e-2 (the recompute
  schedule rounds its own recomputed dS);
* several passes over the kv heads (a small workspace cap) give bit-identical
  results to one pass;
* two calls in a row give bit-identical results (deterministic sums);
* a workspace below the size function's answer is rejected before any launch.
The full config-2 / config-3 comparisons against an fp32 torch reference
(tests/test_attention_fullsize_gpu.py) run with this schedule, the default.
"""
import numpy as np
import pytest
import torch

import tree_training_b200 as tt
from tree_training_b200 import _lib
from tree_training_b200 import attention as A
from tests.test_attention_gpu import DEV, make_case, oracle_all, rel, run

pytestmark = pytest.mark.gpu


def _round(x, dtype):
    return torch.tensor(x, dtype=dtype).double().numpy()


def _with_schedule(schedule, fn):
    prev = A.set_backward_schedule(schedule)
    try:
        return fn()
    finally:
        A.set_backward_schedule(prev)


@pytest.mark.parametrize("seed,n,hq,hkv,past,dtype", [
    (41, 700, 4, 1, 0, torch.bfloat16),
    (42, 1500, 8, 2, 37, torch.bfloat16),
    (43, 1000, 12, 3, 130, torch.float16),
    (44, 333, 4, 4, 0, torch.bfloat16),
])
def test_stored_schedule_vs_oracle_and_recompute(seed, n, hq, hkv, past, dtype):
    meta, q, k, v, do = make_case(seed, n, hq, hkv, 128, 16, 200, past)
    q, k, v, do = (_round(x, dtype) for x in (q, k, v, do))
    stored = _with_schedule("stored", lambda: run(q, k, v, meta, do, dtype))
    recomp = _with_schedule("recompute", lambda: run(q, k, v, meta, do, dtype))
    ref = oracle_all(meta, q, k, v, do)
    for name, a, b in zip(("out", "dq", "dk", "dv"), stored, ref):
        assert rel(a, b) < 2e-2, name
    assert np.array_equal(stored[2], recomp[2]), "dk"
    assert np.array_equal(stored[3], recomp[3]), "dv"
    assert rel(stored[1], recomp[1]) < 1e-2


def test_stored_schedule_passes_and_repeat_are_bit_identical(monkeypatch):
    meta, q, k, v, do = make_case(45, 2500, 8, 4, 128, 16, 300, 50)
    q, k, v, do = (_round(x, torch.bfloat16) for x in (q, k, v, do))
    one = run(q, k, v, meta, do, torch.bfloat16)
    again = run(q, k, v, meta, do, torch.bfloat16)
    # a cap below two kv heads' slots: four passes of one kv head each
    n_pairs = int(meta.device(DEV, 128, 128)["fwd_list"].numel())
    per_head = 2 * n_pairs * 32768
    monkeypatch.setattr(A, "_DS_WORKSPACE_CAP", 2 * per_head - 1)
    plan = A._stored_plan(_lib.TT_BF16, meta.n_q, meta.n_kv, 8, 4, 128, n_pairs)
    assert plan is not None and plan[0] == 1
    passes = run(q, k, v, meta, do, torch.bfloat16)
    for name, a, b, c in zip(("out", "dq", "dk", "dv"), one, again, passes):
        assert np.array_equal(a, b), name
        assert np.array_equal(a, c), name


def test_stored_schedule_rejects_a_short_workspace():
    meta, q, k, v, do = make_case(46, 600, 4, 1, 128, 16, 200)
    md = meta.device(DEV, 128, 128)
    qt, kt, vt, dot = (torch.tensor(x, dtype=torch.bfloat16, device=DEV) for x in (q, k, v, do))
    out, lse = A.attn_fwd_raw(qt, kt, vt, md, 128 ** -0.5)
    n_pairs = int(md["fwd_list"].numel())
    need = int(_lib.lib().tt_tree_attn_bwd_stored_workspace_size(
        _lib.TT_BF16, meta.n_q, meta.n_kv, 4, 1, 128, n_pairs, 1))
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    dq, dk, dv = torch.empty_like(qt), torch.empty_like(kt), torch.empty_like(vt)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = _lib.lib().tt_tree_attn_bwd_stored(
        _lib.TT_BF16, meta.n_q, meta.n_kv, 4, 1, 128, qt.data_ptr(), qt.stride(0), qt.stride(1),
        kt.data_ptr(), kt.stride(0), kt.stride(1), vt.data_ptr(), vt.stride(0), vt.stride(1),
        out.data_ptr(), dot.data_ptr(), dot.stride(0), dot.stride(1), lse.data_ptr(),
        md["kv_lo"].data_ptr(), md["kv_hi"].data_ptr(), md["fwd_ptr"].data_ptr(),
        md["fwd_list"].data_ptr(), md["bwd_ptr"].data_ptr(), md["bwd_list"].data_ptr(),
        128 ** -0.5, dq.data_ptr(), dq.stride(0), dq.stride(1), dk.data_ptr(), dk.stride(0),
        dk.stride(1), dv.data_ptr(), dv.stride(0), dv.stride(1), n_pairs, 1, ws.data_ptr(),
        need - 1, _lib.TT_BWD_ALL, status.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == _lib.TT_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert int(status.item()) == 0
