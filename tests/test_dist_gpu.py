"""Data parallelism over NCCL on two B200s (skipped with fewer GPUs): two
ranks, one tree each, through the tcgen05 tree attention; gradient averaging
equals the single-GPU result, and a rank that leaves between steps is
reported by the next heartbeat instead of hanging the survivor.  Ranks are
spawned child processes with NVLS off; no rank leaves with a kernel or a
collective in flight."""
import pytest
import torch

from tests import dist_workers as W

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def test_nccl_dp_attention_step_matches_single_gpu():
    out = W.run_ranks("nccl_dp_attention_step", 2, backend="nccl", pg_timeout=60.0,
                      limit_s=240.0)
    assert set(out) == {0, 1}, out
    for r in (0, 1):
        assert out[r][0] == "ok", out[r][1]
        assert out[r][1] < 1e-5


def test_nccl_rank_leaving_between_steps_is_reported():
    out = W.run_ranks("nccl_fail_rank1", 2, backend="nccl", pg_timeout=30.0, limit_s=240.0,
                      expect={0})
    assert 0 in out, out
    status, res = out[0]
    assert status == "ok", res
    assert res["heartbeat"] == "RankFailure [1]"
    assert res["heartbeat_s"] < 10
