"""Host-side multi-GPU logic on CPU: the work partition and the verification gather, with gloo
ranks (world size 2) standing in for GPUs and the oracle standing in for the kernels."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from kernel_opt_agent_b200 import sharding
from kernel_opt_agent_b200.kernel_configs import qwen35moe_gdn_prefill as gcfg


def test_even_ranges_cover_everything():
    for n in (1, 7, 8, 16, 33):
        for w in (1, 2, 3, 4, 8):
            r = sharding.even_ranges(n, w)
            assert r[0][0] == 0 and r[-1][1] == n and len(r) == w
            assert all(a <= b for a, b in r) and all(r[i][1] == r[i + 1][0] for i in range(w - 1))
            sizes = [b - a for a, b in r]
            assert max(sizes) - min(sizes) <= 1


def test_gdn_value_heads_keep_the_kernel_mapping():
    hk, hv = 16, 32
    for a, b in sharding.even_ranges(hk, 4):
        vh = sharding.gdn_value_heads(a, b, hk, hv)
        assert len(vh) == 2 * (b - a)
        for i, h in enumerate(vh):
            assert h % hk - a == i % (b - a)  # local value head i reads local key head i % (b - a)


def test_gdn_slice_equals_heads_of_full_run():
    inp = gcfg.random_inputs(1, 70, torch.float32, "cpu", seed=3, state_std=0.02, hk=4, hv=8)
    args = lambda d: [d[x].numpy() for x in ("q", "k", "v", "g", "beta", "state")]  # noqa: E731
    o_full, s_full = oracle.gdn_recurrent(*args(inp))
    parts_o, parts_s = [], []
    ranges = sharding.even_ranges(4, 2)
    for a, b in ranges:
        o, s = oracle.gdn_recurrent(*args(sharding.slice_gdn_inputs(inp, a, b)))
        parts_o.append(torch.from_numpy(o))
        parts_s.append(torch.from_numpy(s))
    o = sharding.unscatter_gdn_heads(parts_o, ranges, 4, 8, dim=2)
    s = sharding.unscatter_gdn_heads(parts_s, ranges, 4, 8, dim=1)
    np.testing.assert_array_equal(o.numpy(), o_full)
    np.testing.assert_array_equal(s.numpy(), s_full)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        # FA2: key/value heads split across ranks, outputs gathered along the head dimension
        gen = torch.Generator().manual_seed(1)
        qf = torch.randn(2, 8, 40, 64, generator=gen)
        kf = torch.randn(2, 4, 40, 64, generator=gen)
        vf = torch.randn(2, 4, 40, 64, generator=gen)
        a, b = sharding.even_ranges(4, world)[rank]
        loc = sharding.slice_fa2_inputs({"q": qf, "k": kf, "v": vf}, a, b)
        o = torch.from_numpy(oracle.fa2_attention(loc["q"].numpy(), loc["k"].numpy(), loc["v"].numpy()))
        full = sharding.gather_to_rank0(o, dim=1)
        # GDN: key-head groups, outputs and states gathered and put back in head order
        inp = gcfg.random_inputs(1, 50, torch.float32, "cpu", seed=5, state_std=0.02, hk=4, hv=8)
        ranges = sharding.even_ranges(4, world)
        sl = sharding.slice_gdn_inputs(inp, *ranges[rank])
        go, gs = oracle.gdn_recurrent(*(sl[x].numpy() for x in ("q", "k", "v", "g", "beta", "state")))
        go_all = sharding.gather_to_rank0(torch.from_numpy(go), dim=2)
        gs_all = sharding.gather_to_rank0(torch.from_numpy(gs), dim=1)
        if rank == 0:
            ref = oracle.fa2_attention(qf.numpy(), kf.numpy(), vf.numpy())
            np.testing.assert_allclose(full.numpy(), ref, rtol=1e-6, atol=1e-6)
            o_ref, s_ref = oracle.gdn_recurrent(*(inp[x].numpy() for x in ("q", "k", "v", "g", "beta", "state")))
            # gather_to_rank0 already concatenated the rank slices in rank order
            per = [go_all.narrow(2, 2 * a, 2 * (b - a)) for a, b in ranges]
            np.testing.assert_array_equal(sharding.unscatter_gdn_heads(per, ranges, 4, 8, 2).numpy(), o_ref)
            per = [gs_all.narrow(1, 2 * a, 2 * (b - a)) for a, b in ranges]
            np.testing.assert_array_equal(sharding.unscatter_gdn_heads(per, ranges, 4, 8, 1).numpy(), s_ref)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


@pytest.mark.timeout(240)
def test_two_gloo_ranks_shard_and_gather():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=200) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
