"""bt_topk_half_noalloc: the entry point that runs on the library's fixed scratch array.

It has no counterpart in the reference (whose batch_topk_half always takes a caller
workspace, include/batch_topk.cuh:10-19), so its oracle is bt_topk_half itself: on the same
inputs both must give bit-identical values and indices, call after call.  The file name
makes pytest collect it last, so the GPU tests run both after every other test (in a full
run) and alone in a fresh process (`pytest tests/test_zz_no_alloc.py`).
"""
from __future__ import annotations

import numpy as np
import pytest

import batch_topk_b200 as bt

from util import _dev_copy


def _gen(seg_num: int, seg_len: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((seg_num, seg_len), dtype=np.float32).astype(np.float16)
    # A band of repeated values, so ties (resolved by index) reach the selected set.
    x[:, : seg_len // 4] = np.round(x[:, : seg_len // 4] * 4) / 4
    return x.view(np.uint16)


def _run(torch, x, seg_num, seg_len, k, noalloc: bool, stream):
    ov = torch.full((seg_num, k), 0x1234, dtype=torch.int16, device=x.device)
    oi = torch.full((seg_num, k), -7, dtype=torch.int32, device=x.device)
    if noalloc:
        rc = bt.batch_topk_half_noalloc(x.data_ptr(), seg_num, seg_len, k, ov.data_ptr(),
                                        oi.data_ptr(), stream.cuda_stream)
    else:
        nbytes = bt.batch_topk_half_workspace_size(seg_num, seg_len, k)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device).fill_(0xA5)
        rc = bt.batch_topk_half(x.data_ptr(), seg_num, seg_len, k, ov.data_ptr(), oi.data_ptr(),
                                ws.data_ptr(), nbytes, stream.cuda_stream)
    assert rc == 0, f"{'noalloc' if noalloc else 'workspace'} entry returned {rc}"
    stream.synchronize()
    return ov.cpu().numpy().view(np.uint16), oi.cpu().numpy()


# (seg_num, seg_len, k, input misalignment in elements); the first is the vocabulary-sized
# batch (about 10.5 MB of scratch), the others take the k > 128 path, short rows, and an
# input pointer that is not 16-byte aligned.
SHAPES = [
    (1024, 151936, 50, 0),
    (64, 50000, 256, 0),
    (300, 1000, 128, 3),
    (7, 70001, 1, 5),
    (2, 4096, 1024, 0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("seg_num,seg_len,k,mis", SHAPES)
def test_noalloc_matches_workspace_entry(seg_num, seg_len, k, mis):
    import torch

    assert bt.batch_topk_half_workspace_size(seg_num, seg_len, k) <= bt.NOALLOC_SCRATCH_BYTES
    dev = torch.device("cuda:0")
    s = torch.cuda.current_stream(dev)
    bits = _gen(seg_num, seg_len, seed=seg_num * 7919 + k)
    _buf, x = _dev_copy(torch, bits, mis, dev)
    ref_v, ref_i = _run(torch, x, seg_num, seg_len, k, noalloc=False, stream=s)
    for call in range(2):
        v, i = _run(torch, x, seg_num, seg_len, k, noalloc=True, stream=s)
        assert np.array_equal(i, ref_i), f"indices differ on no-alloc call {call}"
        assert np.array_equal(v, ref_v), f"values differ on no-alloc call {call}"


@pytest.mark.gpu
def test_noalloc_back_to_back_shapes_and_no_device_allocation():
    """Two different shapes queued back to back on one stream (the second call reuses the
    scratch the first left behind), and device free memory unchanged across warm calls."""
    import torch

    dev = torch.device("cuda:0")
    s = torch.cuda.current_stream(dev)
    a = _gen(512, 151936, seed=11)
    b = _gen(40, 20000, seed=12)
    _ba, xa = _dev_copy(torch, a, 0, dev)
    _bb, xb = _dev_copy(torch, b, 1, dev)
    ref_a = _run(torch, xa, 512, 151936, 64, noalloc=False, stream=s)
    ref_b = _run(torch, xb, 40, 20000, 300, noalloc=False, stream=s)

    outs = []
    for x, n, L, k in ((xa, 512, 151936, 64), (xb, 40, 20000, 300)):
        ov = torch.empty((n, k), dtype=torch.int16, device=dev)
        oi = torch.empty((n, k), dtype=torch.int32, device=dev)
        outs.append((x, n, L, k, ov, oi))

    def launch_both():
        for x, n, L, k, ov, oi in outs:
            rc = bt.batch_topk_half_noalloc(x.data_ptr(), n, L, k, ov.data_ptr(), oi.data_ptr(),
                                            s.cuda_stream)
            assert rc == 0

    launch_both()  # first calls on this device: set-up happens here
    s.synchronize()
    free_before = torch.cuda.mem_get_info(dev)[0]
    launch_both()
    s.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free_before
    for (x, n, L, k, ov, oi), (rv, ri) in zip(outs, (ref_a, ref_b)):
        assert np.array_equal(oi.cpu().numpy(), ri)
        assert np.array_equal(ov.cpu().numpy().view(np.uint16), rv)


def test_noalloc_rejects_oversized_and_invalid_shapes():
    """Refused before any device work, so this runs without a GPU: a shape whose workspace
    exceeds the fixed scratch, and the shapes bt_topk_half itself rejects."""
    big = (4096, 151936, 50)
    assert bt.batch_topk_half_workspace_size(*big) > bt.NOALLOC_SCRATCH_BYTES
    fake = 1 << 20  # never dereferenced: the call returns before launching
    assert bt.batch_topk_half_noalloc(fake, *big, fake, fake, 0) == bt.CUDA_ERROR_INVALID_VALUE
    for shape in ((0, 100, 1), (4, 100, 0), (4, 100, 101), (4, 5000, bt.MAX_K + 1)):
        assert bt.batch_topk_half_noalloc(fake, *shape, fake, fake, 0) == \
            bt.CUDA_ERROR_INVALID_VALUE


@pytest.mark.gpu
def test_noalloc_status_readback():
    """bt_noalloc_status reads the status word of the last no-alloc call from the fixed
    scratch array, so a failed device-side check is visible to callers of the no-alloc entry
    point too: clean after an ordinary call, BT_STATUS_WAIT_TIMEOUT after a call whose
    hand-off waits were made to give up at once, and clean (and exact) again after that."""
    import torch

    dev = torch.device("cuda:0")
    s = torch.cuda.current_stream(dev)
    seg_num, seg_len, k = 8, 151936, 50
    bits = _gen(seg_num, seg_len, seed=77)
    _buf, x = _dev_copy(torch, bits, 0, dev)
    ref_v, ref_i = _run(torch, x, seg_num, seg_len, k, noalloc=False, stream=s)
    _run(torch, x, seg_num, seg_len, k, noalloc=True, stream=s)
    assert bt.noalloc_status(s.cuda_stream)[0] == 0
    bt.set_handoff_wait_tries(0)
    try:
        _run(torch, x, seg_num, seg_len, k, noalloc=True, stream=s)
    finally:
        bt.set_handoff_wait_tries(None)
    assert bt.noalloc_status(s.cuda_stream)[0] & bt.STATUS_WAIT_TIMEOUT
    v, i = _run(torch, x, seg_num, seg_len, k, noalloc=True, stream=s)
    assert bt.noalloc_status(s.cuda_stream)[0] == 0
    assert np.array_equal(i, ref_i) and np.array_equal(v, ref_v)
