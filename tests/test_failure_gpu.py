"""The bounded-wait failure path on a B200, without a GPU fault: a kernel
waits for an mbarrier phase nothing completes, gives up after the limit,
records TT_ERR_DEVICE_TIMEOUT in the device status word, and the context
stays usable for the next op."""
import pytest
import torch

import tree_training_b200 as tt
from tree_training_b200 import _lib
from tree_training_b200.attention import _status_word
from tree_training_b200.synthetic import bfs_tree

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def test_bounded_wait_reports_timeout_and_context_stays_usable():
    tt.check_device_status(DEV)                        # start clean
    st = _status_word(DEV)
    _lib.call("tt_diag_bounded_wait", st.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)
    torch.cuda.synchronize(DEV)
    with pytest.raises(_lib.TTError) as e:
        tt.check_device_status(DEV)
    assert "timed out" in str(e.value).lower() or "timeout" in str(e.value).lower()
    tt.check_device_status(DEV)                        # the word was cleared
    # the next op runs normally on the same context
    info = tt.build_dfs_tree_info(bfs_tree(5, 1024, 32, 128, 256))
    meta = info.attn_meta()
    g = torch.Generator(device=DEV).manual_seed(0)
    q = torch.randn(meta.n_q, 4, 128, generator=g, device=DEV).to(torch.bfloat16).requires_grad_(True)
    k = torch.randn(meta.n_kv, 1, 128, generator=g, device=DEV).to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(meta.n_kv, 1, 128, generator=g, device=DEV).to(torch.bfloat16).requires_grad_(True)
    out = tt.tree_attention(q, k, v, meta)
    out.float().sum().backward()
    torch.cuda.synchronize(DEV)
    tt.check_device_status(DEV)
    assert torch.isfinite(out.float()).all() and torch.isfinite(q.grad.float()).all()
