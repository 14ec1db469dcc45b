"""Segment sharding across the GPUs of one node.  Segments are independent, so each device
owns a contiguous range of whole segments and nothing crosses between GPUs on the data path;
results meet on the host.

Two process models:

* one process, one host thread per device (``topk_multi_gpu``): each thread copies its
  shard in on its own stream, runs the top-k there and copies its rows of the result into
  the shared host output at its row offset;
* one process per device under torchrun (``gather_rows``): each rank computes its shard and
  the ranks gather the rows with one ``torch.distributed`` all-gather at the end, after an
  agreement step (``agree_ok``) that turns a failure on any rank into an error on every rank
  instead of a collective that waits forever.

Fixed-length batches split by rows (sizes differ by at most one); CSR batches split at the
segment boundary nearest each equal share of ELEMENTS, since segment lengths vary from 1 to
262144 within one batch.
"""
from __future__ import annotations

import threading
from typing import Callable, Sequence

import numpy as np


class ShardFailure(RuntimeError):
    """A shard failed; ``rank`` is its position in the device list (or the process rank)."""

    def __init__(self, rank: int, cause: BaseException | str):
        self.rank = rank
        self.cause = cause
        super().__init__(f"shard {rank} failed: {cause}")


def row_ranges(seg_num: int, world: int) -> list[tuple[int, int]]:
    """Contiguous [start, stop) row ranges, one per rank, sizes differing by at most one."""
    if world <= 0 or seg_num < 0:
        raise ValueError("world must be positive and seg_num non-negative")
    base, extra = divmod(seg_num, world)
    out, s = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((s, s + n))
        s += n
    return out


def csr_ranges(offsets: np.ndarray, world: int) -> list[tuple[int, int]]:
    """Contiguous segment ranges whose element counts are as close to equal as segment
    boundaries allow: rank r ends at the boundary nearest r+1 equal shares of the total."""
    off = np.asarray(offsets, dtype=np.int64)
    seg_num = off.size - 1
    if world <= 0 or seg_num < 0:
        raise ValueError("world must be positive and offsets non-empty")
    total = int(off[-1] - off[0])
    cuts = [0]
    for r in range(1, world):
        target = off[0] + total * r / world
        j = int(np.searchsorted(off, target))
        if j > 0 and (j > seg_num or abs(off[j - 1] - target) <= abs(off[j] - target)):
            j -= 1
        cuts.append(min(max(j, cuts[-1]), seg_num))
    cuts.append(seg_num)
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def csr_local(offsets: np.ndarray, s0: int, s1: int) -> tuple[np.ndarray, int, int]:
    """Offsets of segments [s0, s1) rebased to start at 0 (int32), and the element range
    [e0, e1) of the shard in the global value array."""
    off = np.asarray(offsets, dtype=np.int64)
    e0, e1 = int(off[s0]), int(off[s1])
    return (off[s0:s1 + 1] - e0).astype(np.int32), e0, e1


# Runner: (rank, device, values [rows, len] or 1-D, local offsets or None, k) -> (values u16,
# indices i32), both [rows, k].
Runner = Callable[[int, int, np.ndarray, "np.ndarray | None", int], tuple]


def device_runner(rank: int, device: int, x: np.ndarray, offsets, k: int, bf16: bool = False):
    """Top-k of one shard on `device` through the library, from and back to host memory
    (fp16 bits, or bf16 bits with bf16)."""
    import torch

    from . import torch_api

    dev = torch.device("cuda", device)
    with torch.cuda.device(dev):
        stream = torch.cuda.Stream(dev)
        if x.size == 0:
            rows = 0 if offsets is None else len(offsets) - 1
            pad = 0xFF80 if bf16 else 0xFC00  # -inf
            return (np.full((rows, k), pad, np.uint16), np.full((rows, k), -1, np.int32))
        xh = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).pin_memory()
        ws = torch_api.Workspace(dev)
        with torch.cuda.stream(stream):
            xd = xh.to(dev, non_blocking=True).view(torch.bfloat16 if bf16 else torch.float16)
            if offsets is None:
                v, i = torch_api.topk(xd, k, workspace=ws, stream=stream)
            else:
                od = torch.from_numpy(np.ascontiguousarray(offsets, np.int32)).to(dev)
                v, i = torch_api.topk_segmented(xd, od, k, workspace=ws, stream=stream)
            hv = v.view(torch.int16).to("cpu", non_blocking=True)
            hi = i.to("cpu", non_blocking=True)
        stream.synchronize()
        return hv.numpy().view(np.uint16), hi.numpy()


def topk_multi_gpu(x: np.ndarray, k: int, devices: Sequence[int], offsets=None,
                   runner: Runner | None = None, bf16: bool = False):
    """Top-k of a host batch sharded by segment over `devices` (one host thread each).

    x is [seg_num, seg_len] uint16 fp16 bits (bf16 bits with bf16), or 1-D with CSR
    `offsets` [seg_num+1].  Returns (values uint16 [seg_num, k], indices int32 [seg_num, k]).
    If any shard fails, every thread is joined first and then ShardFailure names the lowest
    failing rank.  A custom runner gets (rank, device, shard, offsets, k)."""
    run = runner or (lambda r, d, xs, o, kk: device_runner(r, d, xs, o, kk, bf16=bf16))
    world = len(devices)
    if world == 0:
        raise ValueError("no devices")
    if offsets is None:
        seg_num = x.shape[0]
        ranges = row_ranges(seg_num, world)
    else:
        seg_num = len(offsets) - 1
        ranges = csr_ranges(offsets, world)
    out_v = np.empty((seg_num, k), np.uint16)
    out_i = np.empty((seg_num, k), np.int32)
    errors: dict[int, BaseException] = {}

    def work(rank: int):
        s0, s1 = ranges[rank]
        if s1 == s0:
            return  # more devices than segments: nothing to run on this one
        try:
            if offsets is None:
                v, i = run(rank, devices[rank], x[s0:s1], None, k)
            else:
                loc, e0, e1 = csr_local(offsets, s0, s1)
                v, i = run(rank, devices[rank], x[e0:e1], loc, k)
            if v.shape != (s1 - s0, k) or i.shape != (s1 - s0, k):
                raise RuntimeError(f"shard result shape {v.shape}, expected {(s1 - s0, k)}")
            out_v[s0:s1] = v
            out_i[s0:s1] = i
        except BaseException as e:  # noqa: BLE001 -- reported to the caller below
            errors[rank] = e

    threads = [threading.Thread(target=work, args=(r,), name=f"bt-shard-{r}") for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        r = min(errors)
        raise ShardFailure(r, errors[r]) from errors[r]
    return out_v, out_i


def agree_ok(ok: bool, group=None, device=None) -> None:
    """Every rank states whether its shard succeeded; if any did not, every rank raises
    ShardFailure naming the lowest failing rank.  All ranks must call it, in the same order
    relative to their other collectives."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    flags = torch.zeros(world, dtype=torch.int32, device=device)
    flags[rank] = 0 if ok else 1
    dist.all_reduce(flags, group=group)
    bad = torch.nonzero(flags).flatten().tolist()
    if bad:
        raise ShardFailure(bad[0], "reported by that rank")


def gather_rows(values, indices, ranges: Sequence[tuple[int, int]], group=None):
    """All-gather every rank's [rows_r, k] result (tensors on the group's device) into full
    [seg_num, k] tensors on every rank.  `ranges` is the rank-ordered segment split that the
    shards were computed on (row_ranges or csr_ranges)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if len(ranges) != world:
        raise ValueError(f"{len(ranges)} ranges for {world} ranks")
    max_rows = max(max(s1 - s0 for s0, s1 in ranges), 1)
    k = values.shape[1]

    def padded(t):
        p = torch.zeros((max_rows, k), dtype=t.dtype, device=t.device)
        p[: t.shape[0]] = t
        return p

    out = []
    for t in (values, indices):
        dtype = t.dtype
        if t.element_size() == 2:  # fp16 bits travel as int32 (not every backend has 16-bit)
            t = t.view(torch.int16).to(torch.int32)
        parts = [torch.empty((max_rows, k), dtype=t.dtype, device=t.device) for _ in range(world)]
        dist.all_gather(parts, padded(t), group=group)
        full = torch.cat([p[: s1 - s0] for p, (s0, s1) in zip(parts, ranges)])
        if dtype != full.dtype:
            full = full.to(torch.int16).view(dtype)
        out.append(full)
    return out[0], out[1]
