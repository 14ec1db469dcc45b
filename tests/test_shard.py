"""Segment sharding (batch_topk_b200.shard) on the CPU: partition arithmetic, the
thread-per-device driver with a checker-backed runner standing in for the devices, host-side
failure injection, and the one-process-per-rank gather over `gloo` at world_size 2.

The per-shard compute here is the oracle, so these tests pin only the host logic (split,
rebase, placement, failure reporting); the device path is covered by the gpu-marked test at
the end and by the parity suite.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from batch_topk_b200 import shard
from batch_topk_b200 import workloads as wl


@pytest.mark.parametrize("seg_num,world", [(10, 3), (3, 8), (0, 2), (1024, 8), (7, 1)])
def test_row_ranges_cover_and_balance(seg_num, world):
    r = shard.row_ranges(seg_num, world)
    assert len(r) == world and r[0][0] == 0 and r[-1][1] == seg_num
    assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
    sizes = [b - a for a, b in r]
    assert max(sizes) - min(sizes) <= 1


def test_csr_ranges_balance_elements():
    off = wl.c4_offsets()
    for world in (1, 2, 4, 8):
        r = shard.csr_ranges(off, world)
        assert r[0][0] == 0 and r[-1][1] == 4096
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        elems = [int(off[b] - off[a]) for a, b in r]
        share = off[-1] / world
        # each boundary is within one segment (<= 262144 values) of the ideal cut
        assert max(abs(e - share) for e in elems) <= 2 * wl.C4_MAX_LEN


def test_csr_ranges_degenerate():
    off = np.array([0, 0, 0, 5])
    r = shard.csr_ranges(off, 4)
    assert r[0][0] == 0 and r[-1][1] == 3 and sum(b - a for a, b in r) == 3
    loc, e0, e1 = shard.csr_local(np.array([0, 4, 9, 9, 20]), 1, 4)
    assert loc.tolist() == [0, 5, 5, 16] and (e0, e1) == (4, 20) and loc.dtype == np.int32


def oracle_runner(orc, fail_rank=None):
    def run(rank, device, x, offsets, k):
        if rank == fail_rank:
            raise RuntimeError("injected failure")
        if offsets is None:
            return orc.topk(x, k)
        return orc.topk_csr(x, offsets, k)
    return run


def test_multi_device_fixed_equals_single(orc):
    x = wl.gen_c1()
    ev, ei = orc.topk(x, 50)
    v, i = shard.topk_multi_gpu(x, 50, devices=[0, 1, 2], runner=oracle_runner(orc))
    assert np.array_equal(v, ev) and np.array_equal(i, ei)
    # more devices than rows: the extra shards are empty
    v, i = shard.topk_multi_gpu(x, 50, devices=list(range(6)), runner=oracle_runner(orc))
    assert np.array_equal(v, ev) and np.array_equal(i, ei)


def test_multi_device_csr_equals_single(orc):
    off = wl.c4_offsets()[:129]
    x = wl.gen_c4_range(0, 128)
    for k in (1, 50, 256):
        ev, ei = orc.topk_csr(x, off, k)
        v, i = shard.topk_multi_gpu(x, k, devices=[0, 1, 2, 3], offsets=off,
                                    runner=oracle_runner(orc))
        assert np.array_equal(v, ev) and np.array_equal(i, ei), k


def test_multi_device_failure_names_the_rank(orc):
    x = wl.gen_c1()
    with pytest.raises(shard.ShardFailure) as e:
        shard.topk_multi_gpu(x, 50, devices=[0, 1, 2, 3], runner=oracle_runner(orc, fail_rank=2))
    assert e.value.rank == 2 and "injected" in str(e.value)


# ---- one process per rank over gloo ----------------------------------------------------

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, mode, result_q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        _gloo_body(rank, world, mode, result_q)
    except Exception as e:  # report instead of leaving the parent waiting
        result_q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def _gloo_body(rank, world, mode, result_q):
    import torch

    import oracle

    orc = oracle.load()
    if mode == "csr":
        off = wl.c4_offsets()[:65]
        x = wl.gen_c4_range(0, 64)
        ranges = shard.csr_ranges(off, world)
        s0, s1 = ranges[rank]
        loc, e0, e1 = shard.csr_local(off, s0, s1)
        v, i = orc.topk_csr(x[e0:e1], loc, 8)
    else:
        x = wl.gen_c1(rows=slice(0, 4), seg_len=5000)
        ranges = shard.row_ranges(x.shape[0], world)
        s0, s1 = ranges[rank]
        v, i = orc.topk(x[s0:s1], 8)
    ok = not (mode == "fail" and rank == 1)
    try:
        shard.agree_ok(ok)
    except shard.ShardFailure as e:
        result_q.put((rank, "failure", e.rank))
        return
    gv, gi = shard.gather_rows(torch.from_numpy(v.view(np.int16)), torch.from_numpy(i), ranges)
    result_q.put((rank, "ok", (gv.numpy().view(np.uint16), gi.numpy())))


def _run_gloo(mode, world=2):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict()
    for _ in range(world):
        rank, status, payload = q.get(timeout=120)
        out[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("mode", ["fixed", "csr"])
def test_gloo_gather_equals_single(orc, mode):
    out = _run_gloo(mode)
    if mode == "csr":
        ev, ei = orc.topk_csr(wl.gen_c4_range(0, 64), wl.c4_offsets()[:65], 8)
    else:
        ev, ei = orc.topk(wl.gen_c1(rows=slice(0, 4), seg_len=5000), 8)
    for rank in range(2):
        status, payload = out[rank]
        assert status == "ok", payload
        v, i = payload
        assert np.array_equal(v, ev) and np.array_equal(i, ei)


def test_gloo_failure_reaches_every_rank():
    out = _run_gloo("fail")
    assert out[0] == ("failure", 1) and out[1] == ("failure", 1)


# ---- the device path -----------------------------------------------------------------

@pytest.mark.gpu
def test_device_shards_on_one_gpu_equal_single(orc):
    """Two shards on cuda:0 (own stream and workspace each), checked against the oracle."""
    x = wl.gen_c2(rows=slice(0, 6))
    ev, ei = orc.topk(x, 50)
    v, i = shard.topk_multi_gpu(x, 50, devices=[0, 0])
    assert np.array_equal(v, ev) and np.array_equal(i, ei)
    off = wl.c4_offsets()[:33]
    xc = wl.gen_c4_range(0, 32)
    ev, ei = orc.topk_csr(xc, off, 256)
    v, i = shard.topk_multi_gpu(xc, 256, devices=[0, 0, 0], offsets=off)
    assert np.array_equal(v, ev) and np.array_equal(i, ei)


@pytest.mark.gpu
def test_device_shards_bf16(orc):
    """bf16 rows and a CSR batch with an empty segment, sharded on cuda:0."""
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((6, 30000)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    ev, ei = orc.topk(x, 50, bf16=True)
    v, i = shard.topk_multi_gpu(x, 50, devices=[0, 0], bf16=True)
    assert np.array_equal(v, ev) and np.array_equal(i, ei)
    off = np.array([0, 0, 1000, 1000, 40000, 90000], np.int64)
    xc = (rng.standard_normal(90000).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    ev, ei = orc.topk_csr(xc, off, 64, bf16=True)
    v, i = shard.topk_multi_gpu(xc, 64, devices=[0, 0, 0], offsets=off, bf16=True)
    assert np.array_equal(v, ev) and np.array_equal(i, ei)
