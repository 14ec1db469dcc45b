"""Device-side failure detection, made to fire without faulting or hanging the GPU.

The reference reports problems only through its return code and cudaGetLastError
(src/batch_topk.cu:51-60, :85-193 of fire-emblem/batch_topk).  This library also checks on the
device and records what it finds in the workspace status word (bt_workspace_status):
  * every wait is bounded; a wait that runs out sets BT_STATUS_WAIT_TIMEOUT and the kernel
    finishes without waiting further;
  * CSR offsets that decrease, or that span more than max_total_len values, set
    BT_STATUS_BAD_OFFSETS.
Here the bounded waits run out on purpose through the library's failure-path hook
(bt_set_handoff_wait_tries(0): the consumer <-> merger hand-off waits give up at once), and the
offsets cases use offsets that stay inside the input buffer, so no access leaves its
allocation.  After each failure the next ordinary call on the same workspace must be exact.
"""
from __future__ import annotations

import numpy as np
import pytest

import batch_topk_b200 as bt

from util import _dev_copy, assert_exact, gpu_topk


@pytest.fixture
def handoff_fails():
    bt.set_handoff_wait_tries(0)
    try:
        yield
    finally:
        bt.set_handoff_wait_tries(None)


def _call(torch, x, seg_num, seg_len, k, ws):
    dev = x.device
    ov = torch.empty((seg_num, k), dtype=torch.int16, device=dev)
    oi = torch.empty((seg_num, k), dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev)
    rc = bt.batch_topk_half(x.data_ptr(), seg_num, seg_len, k, ov.data_ptr(), oi.data_ptr(),
                            ws.data_ptr(), ws.numel(), s.cuda_stream)
    assert rc == 0
    s.synchronize()
    flags, _ = bt.workspace_status(ws.data_ptr(), seg_num, s.cuda_stream)
    return flags, ov.cpu().numpy().view(np.uint16), oi.cpu().numpy()


# (seg_num, seg_len): segments split across blocks (each block sends one batch: the merger's
# wait gives up), and many short segments per block (the consumers' wait for a free batch
# buffer gives up too, and they stop early; the producer then stops at its next stage).
TIMEOUT_SHAPES = [(8, 151936), (2048, 10000)]


@pytest.mark.gpu
@pytest.mark.parametrize("seg_num,seg_len", TIMEOUT_SHAPES)
def test_handoff_wait_timeout_is_reported_then_next_call_exact(orc, seg_num, seg_len):
    import torch

    dev = torch.device("cuda:0")
    k = 50
    rng = np.random.default_rng(seg_num)
    bits = rng.standard_normal((seg_num, seg_len)).astype(np.float16).view(np.uint16)
    _buf, x = _dev_copy(torch, bits, 0, dev)
    ws = torch.empty(bt.batch_topk_half_workspace_size(seg_num, seg_len, k), dtype=torch.uint8,
                     device=dev)
    bt.set_handoff_wait_tries(0)
    try:
        flags, _, _ = _call(torch, x, seg_num, seg_len, k, ws)
    finally:
        bt.set_handoff_wait_tries(None)
    assert flags & bt.STATUS_WAIT_TIMEOUT, f"status {flags:#x}: the timeout was not reported"
    # the next call on the same workspace starts from a clean status and is exact
    flags, v, i = _call(torch, x, seg_num, seg_len, k, ws)
    assert flags == 0
    exp_v, exp_i = orc.topk(bits, k)
    assert_exact(v, i, exp_v, exp_i, "after a timed-out call")


@pytest.mark.gpu
def test_torch_api_check_raises_on_device_status(handoff_fails):
    import torch

    from batch_topk_b200.torch_api import topk

    x = torch.randn(8, 151936, device="cuda").half()
    with pytest.raises(bt.DeviceStatusError) as e:
        topk(x, 50, check=True)
    assert e.value.flags & bt.STATUS_WAIT_TIMEOUT


@pytest.mark.gpu
def test_large_k_unaffected_by_handoff_hook(orc, handoff_fails):
    """k > 128 has no merger warp and no hand-off waits: the hook changes nothing there."""
    rng = np.random.default_rng(5)
    bits = rng.standard_normal((16, 70000)).astype(np.float16).view(np.uint16)
    v, i = gpu_topk(bits, 300)  # asserts status 0
    exp_v, exp_i = orc.topk(bits, 300)
    assert_exact(v, i, exp_v, exp_i, "k=300 under the hook")


def _csr_call(torch, vals, offsets, k, max_total_len):
    dev = torch.device("cuda:0")
    _buf, x = _dev_copy(torch, vals, 0, dev)
    d_off = torch.from_numpy(np.asarray(offsets, np.int32)).to(dev)
    seg_num = len(offsets) - 1
    nbytes = bt.batch_topk_half_segmented_workspace_size(seg_num, max_total_len, k)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev).fill_(0xA5)
    ov = torch.full((seg_num, k), 0x1234, dtype=torch.int16, device=dev)
    oi = torch.full((seg_num, k), -7, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev)
    rc = bt.batch_topk_half_segmented(x.data_ptr(), d_off.data_ptr(), seg_num, max_total_len, k,
                                      ov.data_ptr(), oi.data_ptr(), ws.data_ptr(), nbytes,
                                      s.cuda_stream)
    assert rc == 0
    s.synchronize()
    flags, _ = bt.workspace_status(ws.data_ptr(), seg_num, s.cuda_stream)
    return flags, ov.cpu().numpy().view(np.uint16), oi.cpu().numpy()


@pytest.mark.gpu
def test_bad_offsets_decreasing(orc):
    """A segment whose end lies before its start is flagged and treated as empty; the valid
    segments around it are still exact."""
    import torch

    rng = np.random.default_rng(8)
    vals = rng.standard_normal(9000).astype(np.float16).view(np.uint16)
    off = [0, 5000, 3000, 9000]
    flags, v, i = _csr_call(torch, vals, off, 50, 9000)
    assert flags & bt.STATUS_BAD_OFFSETS
    for s, (a, b) in ((0, (0, 5000)), (2, (3000, 9000))):
        exp_v, exp_i = orc.topk(vals[a:b].reshape(1, -1), 50)
        assert_exact(v[s:s + 1], i[s:s + 1], exp_v, exp_i, f"segment {s}")
    assert (i[1] == -1).all() and (v[1] == 0xFC00).all()


@pytest.mark.gpu
def test_bad_offsets_beyond_max_total_len():
    """Offsets spanning more values than max_total_len (the buffer really holds them all, so
    nothing is read out of bounds): flagged, and no segment is processed."""
    import torch

    rng = np.random.default_rng(9)
    vals = rng.standard_normal(8000).astype(np.float16).view(np.uint16)
    flags, v, i = _csr_call(torch, vals, [0, 4000, 8000], 50, 6000)
    assert flags & bt.STATUS_BAD_OFFSETS
    assert (i == -7).all() and (v == 0x1234).all(), "a flagged call must not write rows"


@pytest.mark.gpu
def test_bad_offsets_many_segments_flag_only():
    """More segments than resident blocks (whole segments, helping on) with offsets spanning
    more than max_total_len: only BT_STATUS_BAD_OFFSETS is reported (the streaming kernel
    still ends at once, with no wait running out), and no row is written."""
    import torch

    rng = np.random.default_rng(10)
    vals = rng.standard_normal(8000).astype(np.float16).view(np.uint16)
    off = list(range(0, 8001, 20))  # 400 segments of 20 values
    flags, v, i = _csr_call(torch, vals, off, 8, 6000)
    assert flags == bt.STATUS_BAD_OFFSETS, f"status {flags:#x}"
    assert (i == -7).all() and (v == 0x1234).all(), "a flagged call must not write rows"


@pytest.mark.gpu
def test_all_empty_many_segments():
    """400 empty CSR segments: every row is padding (-inf, index -1) and the status is clean."""
    import torch

    vals = np.zeros(16, np.uint16)
    flags, v, i = _csr_call(torch, vals, [0] * 401, 8, 16)
    assert flags == 0, f"status {flags:#x}"
    assert (i == -1).all() and (v == 0xFC00).all()
