"""The size/world table behind ``NVLinkGroup.allreduce(method="auto")`` (host logic,
no GPU): the crossovers measured by benchmarks/collectives_bench.py on B200."""
import pytest

from dtrain_b200.parallel.nvlink import auto_allreduce_plan

KIB, MIB = 1 << 10, 1 << 20


@pytest.mark.parametrize("world,nbytes,plan", [
    (2, 4 * KIB, ("oneshot", 0)),
    (2, 16 * MIB, ("oneshot", 0)),          # same bytes as two-shot at W=2, one barrier fewer
    (2, 16 * MIB + 4, ("twoshot", 128)),
    (2, 1 << 30, ("twoshot", 128)),
    (4, 512 * KIB, ("oneshot", 0)),
    (4, 2 * MIB, ("oneshot", 128)),
    (4, 4 * MIB, ("oneshot", 128)),
    (4, 8 * MIB, ("twoshot", 0)),
    (4, 256 * MIB, ("twoshot", 128)),
    (3, 1 * MIB, ("oneshot", 128)),
    (8, 256 * KIB, ("oneshot", 0)),
    (8, 1 * MIB, ("twoshot", 0)),           # one-shot traffic grows with W
    (8, 64 * MIB, ("twoshot", 128)),
])
def test_auto_plan_follows_the_measured_crossovers(world, nbytes, plan):
    assert auto_allreduce_plan(world, nbytes) == plan


def test_plan_is_monotone_in_size():
    """Once a size gets two-shot, every larger size does too (no ping-pong)."""
    for world in (2, 3, 4, 8):
        seen_twoshot = False
        for k in range(12, 31):
            m, _ = auto_allreduce_plan(world, 1 << k)
            seen_twoshot = seen_twoshot or m == "twoshot"
            assert not (seen_twoshot and m == "oneshot"), (world, k)


def test_ddp_refuses_nvls_without_a_multicast_group_before_any_backward():
    """An NVLS request on a group without multicast fails when the DDP wrapper is made,
    not at the first bucket launch in the middle of a backward pass."""
    import torch

    from dtrain_b200.parallel.ddp import DDP

    class HostGroup:
        backend, world, rank, nvls = "tcp", 2, 0, False

    with pytest.raises(ValueError, match="nvls=True"):
        DDP(torch.nn.Linear(2, 2), HostGroup(), method="nvls")
    with pytest.raises(ValueError, match="unknown DDP all-reduce method"):
        DDP(torch.nn.Linear(2, 2), HostGroup(), method="ringz")
