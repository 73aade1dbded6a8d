"""Two devices (skipped with fewer): the sharded stage through the C ABI, each rank holding half of the training
rows' chunks, equals the CPU path's stage over the whole cache within the stage bar; the f64 all-reduce used for
ensemble members' class-logit sums adds every rank's sums; a rank that leaves between steps is seen by the other on
the host before its next launch, and both abort their communicators with nothing waiting (NVLS off, as for every
test here)."""
import os

import pytest

from test_multi_rank import run_ranks

pytestmark = pytest.mark.gpu

STAGE = 5e-5


@pytest.mark.parametrize("exchange", ["peer stores", "collectives"])
def test_sharded_stage_on_two_gpus(exchange):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TCU_SHARD_P2P="1" if exchange == "peer stores" else "0")
    outs = run_ranks("stage-gpu", 2, timeout=900, env=env)
    for o in outs:
        for k, err in o["stage"].items():
            assert err < STAGE, (o["rank"], k, err)
        assert o["allreduce_f64"] == 3.0


def test_rank_leaving_between_steps_is_seen_before_the_next_launch():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    outs = run_ranks("leave-gpu", 2, timeout=300, env=env)
    by = {o["rank"]: o for o in outs}
    assert by[1]["left_after_step"] == 0 and by[1]["steps"] == 1
    assert by[0]["saw_leave_before_step"] == 1 and by[0]["steps"] == 1
