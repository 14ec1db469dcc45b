"""Shared test helpers: GPU calls through the C ABI and bit-exact comparisons."""
from __future__ import annotations

import hashlib
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def sha(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


def load_npz(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN, name))
    return {k: z[k] for k in z.files}


def _dev_copy(torch, bits: np.ndarray, misalign: int, device):
    flat = np.ascontiguousarray(bits, dtype=np.uint16).reshape(-1)
    buf = torch.empty(flat.size + 16, dtype=torch.int16, device=device)
    buf.fill_(0x5A5A)  # junk around the payload must never leak into results
    view = buf[misalign : misalign + flat.size]
    view.copy_(torch.from_numpy(flat.view(np.int16)))
    return buf, view


def gpu_topk(bits: np.ndarray, k: int, misalign: int = 0, poison: bool = True,
             stream=None, ws_extra: int = 0, bf16: bool = False):
    """Fixed-length top-k on cuda:0 through bt_topk_half (bt_topk_bf16 with bf16); returns
    (value bits, indices)."""
    import torch

    import batch_topk_b200 as bt

    dev = torch.device("cuda:0")
    seg_num, seg_len = bits.shape
    _buf, x = _dev_copy(torch, bits, misalign, dev)
    nbytes = (bt.batch_topk_bf16_workspace_size if bf16 else bt.batch_topk_half_workspace_size)(
        seg_num, seg_len, k)
    assert nbytes > 0
    ws = torch.empty(nbytes + ws_extra, dtype=torch.uint8, device=dev)
    if poison:
        ws.fill_(0xA5)
    ov = torch.full((seg_num, k), 0x1234, dtype=torch.int16, device=dev)
    oi = torch.full((seg_num, k), -7, dtype=torch.int32, device=dev)
    s = stream or torch.cuda.current_stream(dev)
    fn = bt.batch_topk_bf16 if bf16 else bt.batch_topk_half
    rc = fn(x.data_ptr(), seg_num, seg_len, k, ov.data_ptr(), oi.data_ptr(), ws.data_ptr(),
            ws.numel(), s.cuda_stream)
    assert rc == 0, f"top-k returned {rc}"
    s.synchronize()
    flags, _ = bt.workspace_status(ws.data_ptr(), seg_num, s.cuda_stream)
    assert flags == 0, f"device status flags {flags}"
    return ov.cpu().numpy().view(np.uint16), oi.cpu().numpy()


def gpu_topk_csr(vals: np.ndarray, offsets: np.ndarray, k: int, misalign: int = 0,
                 max_total_len: int | None = None, check_status: bool = True,
                 bf16: bool = False):
    import torch

    import batch_topk_b200 as bt

    dev = torch.device("cuda:0")
    off = np.asarray(offsets, np.int64)
    seg_num = off.size - 1
    _buf, x = _dev_copy(torch, vals, misalign, dev)
    d_off = torch.from_numpy(off.astype(np.int32)).to(dev)
    total = int(off[-1] - off[0]) if max_total_len is None else max_total_len
    nbytes = (bt.batch_topk_bf16_segmented_workspace_size if bf16
              else bt.batch_topk_half_segmented_workspace_size)(seg_num, total, k)
    assert nbytes > 0
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    ws.fill_(0xA5)
    ov = torch.full((seg_num, k), 0x1234, dtype=torch.int16, device=dev)
    oi = torch.full((seg_num, k), -7, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev)
    fn = bt.batch_topk_bf16_segmented if bf16 else bt.batch_topk_half_segmented
    rc = fn(x.data_ptr(), d_off.data_ptr(), seg_num, total, k, ov.data_ptr(), oi.data_ptr(),
            ws.data_ptr(), ws.numel(), s.cuda_stream)
    assert rc == 0, f"segmented top-k returned {rc}"
    s.synchronize()
    flags, _ = bt.workspace_status(ws.data_ptr(), seg_num, s.cuda_stream)
    if check_status:
        assert flags == 0, f"device status flags {flags}"
    return ov.cpu().numpy().view(np.uint16), oi.cpu().numpy()


def assert_exact(got_v, got_i, exp_v, exp_i, what=""):
    """Bit-exact compare of fp16 value bits and int32 indices; reports the first mismatch."""
    got_v = np.asarray(got_v, np.uint16)
    exp_v = np.asarray(exp_v, np.uint16)
    bad = (got_i != exp_i) | (got_v != exp_v)
    if bad.any():
        r, c = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {int(bad.sum())} mismatches; first at row {r} rank {c}: got "
            f"(idx {got_i[r, c]}, 0x{int(got_v[r, c]):04x}) expected (idx {exp_i[r, c]}, "
            f"0x{int(exp_v[r, c]):04x})")


def expected_from_indices(bits_rows, idx):
    """Value bits = input bits at the reference's indices (-1 -> 0xFC00 padding)."""
    out = np.full(idx.shape, 0xFC00, np.uint16)
    for r in range(idx.shape[0]):
        row = bits_rows[r]
        m = idx[r] >= 0
        out[r, m] = row[idx[r, m]]
    return out


def _dev_copy32(torch, bits: np.ndarray, misalign: int, device):
    """32-bit patterns on the device, starting `misalign` floats past a 16-byte boundary."""
    flat = np.ascontiguousarray(bits, dtype=np.uint32).reshape(-1)
    buf = torch.empty(flat.size + 8, dtype=torch.int32, device=device)
    buf.fill_(0x5A5A5A5A)  # junk around the payload must never leak into results
    view = buf[misalign : misalign + flat.size]
    view.copy_(torch.from_numpy(flat.view(np.int32)))
    return buf, view


def assert_exact32(got_v, got_i, exp_v, exp_i, what=""):
    """Bit-exact compare of 32-bit value patterns and int32 indices."""
    got_v = np.asarray(got_v, np.uint32)
    exp_v = np.asarray(exp_v, np.uint32)
    bad = (got_i != exp_i) | (got_v != exp_v)
    if bad.any():
        r, c = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {int(bad.sum())} mismatches; first at row {r} rank {c}: got "
            f"(idx {got_i[r, c]}, 0x{int(got_v[r, c]):08x}) expected (idx {exp_i[r, c]}, "
            f"0x{int(exp_v[r, c]):08x})")
