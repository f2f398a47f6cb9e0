"""The reference's unmodified drivers against this package's attention, by replay.

``tests/golden/make_golden.py`` ran the reference's own ``tree_grad_hybrid``
(tree_grad_hybrid.py:434-539, at max_tokens 1000 / 20 / 10) and
``dfs_tree_forward`` (dfs_tree_forward.py:513-576) on the config-1 model with a
recording function registered through transformers' AttentionInterface, the
hook through which ``tree_sm100`` is selected.  The fixture holds every
attention call exactly as those drivers make it: the dense additive mask with
the gateway bias columns, K/V with the GatewayCache prefix, the scaling.  (The
reference checkout is not on the GPU machine, so its drivers cannot run here;
replaying their calls is what shows the interface holds.)

* every recorded call through the registered ``tree_sm100`` function on the GPU
  (fp32) against transformers' SDPA call in float64 on the host: output and
  gradients, max_rel < 1e-4 (the reference's fp32 bar);
* this package's ``tree_grad_hybrid`` on the same seeded model, forest and
  labels against the reference driver's parameter gradients (32 seeded
  projections, norm and max |entry| of every parameter's gradient), 1e-4.
"""
import numpy as np
import pytest
import torch

from tests.golden_util import Node, config1_forest, config1_model, grad_projections, load

import tree_training_b200 as tt
from tree_training_b200.hybrid import make_tree_loss_fn, tree_grad_hybrid

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
RUNS = ("hybrid_1000", "hybrid_20", "hybrid_10", "dfs_forward")


class _Module(torch.nn.Module):
    def __init__(self, groups, layer):
        super().__init__()
        self.num_key_value_groups = groups
        self.layer_idx = layer
        self.is_causal = True


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


@pytest.fixture(scope="module")
def calls():
    return load("ref_driver_calls")


def test_every_recorded_driver_call_through_tree_sm100(calls):
    from transformers import AttentionInterface
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    tt.register_hf_attention()
    fn = AttentionInterface()[tt.ATTN_IMPL_NAME]
    n_gateway = 0
    for run in RUNS:
        n = int(calls[f"{run}/n_calls"])
        assert n > 0
        for i in range(n):
            q, k, v, mask = (calls[f"{run}/{i}/{x}"] for x in ("q", "k", "v", "mask"))
            scaling, groups, layer = calls[f"{run}/{i}/meta"].tolist()
            n_gateway += int(k.shape[2] > q.shape[2])
            mod = _Module(int(groups), int(layer))
            g = np.random.default_rng(i + 7 * len(run))
            dout = g.standard_normal((1, q.shape[2], q.shape[1], q.shape[3]))
            res = []
            for dev, dt, f in ((DEV, torch.float32, fn), ("cpu", torch.float64,
                                                         sdpa_attention_forward)):
                qt, kt, vt = (torch.tensor(x, dtype=dt, device=dev, requires_grad=True)
                              for x in (q, k, v))
                mt = torch.tensor(mask, dtype=dt, device=dev)
                out, _ = f(mod, qt, kt, vt, mt, dropout=0.0, scaling=scaling)
                out.backward(torch.tensor(dout, dtype=dt, device=dev))
                res.append([t.detach().double().cpu().numpy()
                            for t in (out, qt.grad, kt.grad, vt.grad)])
            for name, a, b in zip(("out", "dq", "dk", "dv"), *res):
                assert _rel(a, b) < 1e-4, (run, i, name, _rel(a, b))
    tt.check_device_status(DEV)
    assert n_gateway > 0      # the partitioned runs exercise the gateway prefix


@pytest.mark.parametrize("max_tokens", [1000, 20, 10])
def test_package_driver_matches_reference_driver_gradients(calls, max_tokens):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    model = config1_model().to(DEV)
    roots, leaves, labels = config1_forest(Node)
    model.zero_grad(set_to_none=True)
    tree_grad_hybrid(model, roots, make_tree_loss_fn(labels, leaves, len(leaves)), max_tokens)
    torch.cuda.synchronize()
    tt.check_device_status(DEV)
    got = grad_projections(model.cpu())
    prefix = f"hybrid_{max_tokens}/grad/"
    names = [k[len(prefix):] for k in calls.files if k.startswith(prefix)]
    assert names and set(names) == set(got)
    for name in names:
        ref = calls[prefix + name]
        assert _rel(got[name][:-2], ref[:-2]) < 1e-4, (name, "projections")
        assert _rel(got[name][-2:], ref[-2:]) < 1e-4, (name, "norm / max")
