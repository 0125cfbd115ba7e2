"""The GDN schedule planner ("auto") on the workloads whose schedules were timed on a B200 (148 SMs):
it must pick the one measured fastest.  Event-timed medians (ms, L2 flushed; fused / split /
overlap / segmented): B1 T2048 0.279 / 0.142 / 0.118 / 0.132; B1 T16384 2.08 / 0.93 / 0.66 /
0.71; B1 T65536 8.27 / 3.58 / 2.53 / 2.63; the varlen workload's slice for one of 2 GPUs (16
value heads) 2.92 / 1.91 / 8.31 / 1.93, of 4 GPUs (8) 2.86 / 1.38 / 1.19 / 1.16, of 8 GPUs (4)
2.78 / 1.11 / 0.88 / 0.650; the whole varlen workload 4.07 / 3.60 / - / 3.35; B16 T4096 fused
2.26, segmented 2.14.  Host-only: no GPU is touched (the SM count is given)."""

import pytest
import torch

import bench
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn


class _Props:
    multi_processor_count = 148


@pytest.fixture
def b200(monkeypatch):
    monkeypatch.setattr(gdn.torch.cuda, "get_device_properties", lambda dev: _Props())
    return torch.device("cpu")


VARLEN = tuple(bench.varlen_lengths())


@pytest.mark.parametrize("lengths, hv, best", [
    ((2048,), 32, "overlap"),
    ((16384,), 32, "overlap"),
    ((65536,), 32, "overlap"),
    (VARLEN, 16, "split"),
    (VARLEN, 8, "segmented"),
    (VARLEN, 4, "segmented"),
    (VARLEN, 32, "segmented"),
    ((4096,) * 16, 32, "segmented"),
])
def test_auto_picks_the_measured_fastest(b200, lengths, hv, best):
    sched, seg = gdn._plan_uncached("auto", lengths, hv, b200)
    assert sched == best
    assert (seg > 0) == (sched == "segmented")


def test_record_workspace_cap_falls_back_to_fused(b200):
    """B16 T65536 at 32 value heads needs 39 GB of records, above the 24 GiB cap."""
    assert gdn._plan_uncached("auto", (65536,) * 16, 32, b200) == ("fused", 0)


def test_checkpoints_take_a_record_fed_schedule(b200):
    for lengths, hv in (((2048,), 32), (VARLEN, 4), (VARLEN, 32)):
        assert gdn._plan_uncached("auto", lengths, hv, b200, checkpoints=True)[0] in ("split", "overlap")
    with pytest.raises(ValueError):
        gdn._plan_uncached("segmented", (2048,), 32, b200, checkpoints=True)


def test_explicit_modes_pass_through(b200):
    for mode in ("fused", "split", "overlap"):
        assert gdn._plan_uncached(mode, (2048,), 32, b200) == (mode, 0)
    sched, seg = gdn._plan_uncached("segmented", (8192,), 32, b200)
    assert sched == "segmented" and 1 <= seg <= 128
