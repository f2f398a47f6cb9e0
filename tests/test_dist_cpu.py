"""Multi-process data-parallel logic on CPU (gloo, world size 2): rank -> tree
assignment, gradient averaging equal to the single-process gradient of the
same trees, and host-side detection of a rank that left."""
import pytest
import torch

from tests import dist_workers as W
from tree_training_b200.dist import assign_trees


def test_assign_trees_round_robin_covers_each_tree_once():
    for n in (0, 1, 7, 8, 13):
        for world in (1, 2, 4, 8):
            got = [assign_trees(n, world, r) for r in range(world)]
            flat = sorted(i for g in got for i in g)
            assert flat == list(range(n))
            assert all(g == list(range(r, n, world)) for r, g in enumerate(got))
    with pytest.raises(ValueError):
        assign_trees(4, 2, 2)


@pytest.mark.parametrize("bucket_bytes", [64, 1 << 20])
def test_dp_step_matches_single_process(bucket_bytes):
    n_trees = 5
    out = W.run_ranks("dp_tree_step", 2, (n_trees, bucket_bytes))
    assert set(out) == {0, 1}, out
    for r in (0, 1):
        assert out[r][0] == "ok", out[r][1]
    assert out[0][1]["assigned"] == [0, 2, 4] and out[1][1]["assigned"] == [1, 3]
    ref = W.single_process_grads(n_trees)
    for r in (0, 1):
        for g, e in zip(out[r][1]["grads"], ref):
            torch.testing.assert_close(g, e, rtol=1e-12, atol=1e-14)


@pytest.mark.parametrize("bucket_bytes", [64, 1 << 20])
def test_overlapped_average_matches_single_process(bucket_bytes):
    """Buckets all-reduced from the gradient hooks during each rank's last
    backward (the ranks run different numbers of trees) give the same averaged
    gradients as the single-process run."""
    n_trees = 5
    out = W.run_ranks("dp_overlap_step", 2, (n_trees, bucket_bytes))
    ref = W.single_process_grads(n_trees)
    for r in (0, 1):
        assert out[r][0] == "ok", out[r][1]
        res = out[r][1]
        assert res["issued"] == res["buckets"]      # all issued before average()
        for g, e in zip(res["grads"], ref):
            torch.testing.assert_close(g, e, rtol=1e-12, atol=1e-14)


def test_average_counts_missing_grad_as_zero():
    out = W.run_ranks("average_with_missing_grad", 2)
    for r in (0, 1):
        assert out[r][0] == "ok", out[r][1]
        a, b = out[r][1]
        assert a == [1.5] * 5
        assert b == [2.0] * 3


def test_heartbeats_pass_when_all_ranks_alive():
    out = W.run_ranks("heartbeat_all_alive", 2)
    assert out == {0: ("ok", "ok"), 1: ("ok", "ok")}


def test_rank_failure_is_reported_not_hung():
    out = W.run_ranks("fail_rank1", 2, pg_timeout=5.0, limit_s=90.0, expect={0})
    assert 0 in out, out
    status, res = out[0]
    assert status == "ok", res
    assert res["heartbeat"] == "RankFailure [1]"
    assert res["heartbeat_s"] < 10
    assert res["collective"] != "no error"
    assert res["collective_s"] < 30
