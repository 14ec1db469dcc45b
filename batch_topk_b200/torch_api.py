"""Tensor-level helpers over the C ABI (PyTorch provides device memory and streams only).

    values, indices = topk(x, k)                      # x: [seg_num, seg_len] fp16/bf16/fp32 on CUDA
    values, indices = topk_segmented(x, offsets, k)   # x: 1-D fp16/bf16/fp32, offsets: int32 [seg_num+1]

Values come back in x's dtype (the input's own bit patterns), indices as int32, both
[seg_num, k]; descending by value, lower index first among equal values, NaN last.
"""
from __future__ import annotations

import torch

from . import (
    BatchTopkError,
    DeviceStatusError,
    batch_topk_bf16,
    batch_topk_bf16_segmented,
    batch_topk_bf16_segmented_workspace_size,
    batch_topk_bf16_workspace_size,
    batch_topk_f32,
    batch_topk_f32_segmented,
    batch_topk_f32_segmented_workspace_size,
    batch_topk_f32_workspace_size,
    batch_topk_half,
    batch_topk_half_segmented,
    batch_topk_half_segmented_workspace_size,
    batch_topk_half_workspace_size,
    workspace_status,
)

# entry points per element type: (fixed, fixed workspace size, CSR, CSR workspace size)
_ENTRY = {
    torch.float16: (batch_topk_half, batch_topk_half_workspace_size, batch_topk_half_segmented,
                    batch_topk_half_segmented_workspace_size),
    torch.bfloat16: (batch_topk_bf16, batch_topk_bf16_workspace_size, batch_topk_bf16_segmented,
                     batch_topk_bf16_segmented_workspace_size),
    torch.float32: (batch_topk_f32, batch_topk_f32_workspace_size, batch_topk_f32_segmented,
                    batch_topk_f32_segmented_workspace_size),
}


class Workspace:
    """Grow-only device workspace.  One Workspace must not serve calls that can overlap on the
    GPU (different streams without ordering between them): they would race on it."""

    def __init__(self, device=None):
        self.device = torch.device(device or "cuda")
        self.buf = None

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)
        return self.buf


_default_ws: dict = {}


def _ws(device, stream, ws):
    """The caller's workspace, or the default one of (device, launch stream): calls on one
    stream run in order, so they may share it; calls on different streams never do."""
    if ws is not None:
        return ws
    key = (device.index, stream.cuda_stream)
    if key not in _default_ws:
        _default_ws[key] = Workspace(device)
    return _default_ws[key]


def _launch_stream(device, stream):
    s = stream if stream is not None else torch.cuda.current_stream(device)
    if s.device != device:
        raise ValueError(f"stream is on {s.device}, the input on {device}")
    return s


def _check(ws: torch.Tensor, s, what: str):
    """Synchronous read of the device status word of the call just queued on s."""
    flags, _ = workspace_status(ws.data_ptr(), 0, s.cuda_stream)
    if flags:
        raise DeviceStatusError(flags, what)


def topk(x: torch.Tensor, k: int, *, workspace: Workspace | None = None, stream=None,
         out: tuple | None = None, check: bool = False):
    """Top-k of each row of x on x's device, queued on `stream` (default: the current stream
    of x's device).  The workspace and the outputs are allocated on that stream.  With
    check=True the call waits for the result and raises if a device-side check failed."""
    if x.dtype not in _ENTRY or x.dim() != 2 or not x.is_cuda:
        raise ValueError("x must be a 2-D float16, bfloat16 or float32 CUDA tensor")
    run, size, _, _ = _ENTRY[x.dtype]
    seg_num, seg_len = x.shape
    nbytes = size(seg_num, seg_len, k)
    if nbytes == 0:
        raise BatchTopkError(1, f"unsupported shape ({seg_num}, {seg_len}, k={k})")
    with torch.cuda.device(x.device):  # the library launches on the current device
        s = _launch_stream(x.device, stream)
        if s != torch.cuda.current_stream(x.device):
            x.record_stream(s)  # read on s: keep its memory from reuse until s has run
        with torch.cuda.stream(s):
            x = x.contiguous()
            ws = _ws(x.device, s, workspace).get(nbytes)
            if out is None:
                vals = torch.empty((seg_num, k), dtype=x.dtype, device=x.device)
                idx = torch.empty((seg_num, k), dtype=torch.int32, device=x.device)
            else:
                vals, idx = out
            rc = run(x.data_ptr(), seg_num, seg_len, k, vals.data_ptr(), idx.data_ptr(),
                     ws.data_ptr(), ws.numel(), s.cuda_stream)
        if rc != 0:
            raise BatchTopkError(rc, "top-k")
        if check:
            _check(ws, s, "top-k")
    return vals, idx


def topk_segmented(x: torch.Tensor, offsets: torch.Tensor, k: int, *,
                   max_total_len: int | None = None, workspace: Workspace | None = None,
                   stream=None, out: tuple | None = None, check: bool = False):
    """CSR top-k (segment s = x[offsets[s]:offsets[s+1]]), with topk's device, stream and
    check semantics."""
    if x.dtype not in _ENTRY or x.dim() != 1 or not x.is_cuda:
        raise ValueError("x must be a 1-D float16, bfloat16 or float32 CUDA tensor")
    _, _, run, size = _ENTRY[x.dtype]
    if offsets.dtype != torch.int32 or offsets.dim() != 1 or offsets.device != x.device:
        raise ValueError("offsets must be a 1-D int32 tensor on x's device")
    seg_num = offsets.numel() - 1
    total = x.numel() if max_total_len is None else max_total_len
    nbytes = size(seg_num, total, k)
    if nbytes == 0:
        raise BatchTopkError(1, f"unsupported CSR batch (seg_num={seg_num}, k={k})")
    with torch.cuda.device(x.device):
        s = _launch_stream(x.device, stream)
        if s != torch.cuda.current_stream(x.device):
            x.record_stream(s)
            offsets.record_stream(s)
        with torch.cuda.stream(s):
            ws = _ws(x.device, s, workspace).get(nbytes)
            if out is None:
                vals = torch.empty((seg_num, k), dtype=x.dtype, device=x.device)
                idx = torch.empty((seg_num, k), dtype=torch.int32, device=x.device)
            else:
                vals, idx = out
            rc = run(x.data_ptr(), offsets.data_ptr(), seg_num, total, k, vals.data_ptr(),
                     idx.data_ptr(), ws.data_ptr(), ws.numel(), s.cuda_stream)
        if rc != 0:
            raise BatchTopkError(rc, "segmented top-k")
        if check:
            _check(ws, s, "segmented top-k")
    return vals, idx


_staging: dict = {}


def topk_from_host(x_host: torch.Tensor, k: int, *, out_host: tuple | None = None,
                   stream=None, workspace: Workspace | None = None, device=None):
    """End-to-end call from host memory: copy the rows in, run top-k, copy the results out.

    x_host is a 2-D CPU tensor of fp16 values (float16, or int16/uint16 bit patterns),
    ideally pinned; out_host, if given, is a (values, indices) pair of CPU tensors
    [seg_num, k] (int16/float16 and int32).  Everything is queued on `stream` and this call
    returns after the results are on the host."""
    dev = torch.device(device or "cuda")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    seg_num, seg_len = x_host.shape
    with torch.cuda.device(dev):
        s = _launch_stream(dev, stream)
        key = (dev.index, s.cuda_stream)
        with torch.cuda.stream(s):
            buf = _staging.get(key)
            if buf is None or buf.numel() < x_host.numel():
                buf = torch.empty(x_host.numel(), dtype=torch.float16, device=dev)
                _staging[key] = buf
            xd = buf[: x_host.numel()].view(seg_num, seg_len)
            xd.view(torch.int16).copy_(x_host.view(torch.int16), non_blocking=True)
            vals, idx = topk(xd, k, workspace=workspace, stream=s)
            if out_host is None:
                out_host = (torch.empty((seg_num, k), dtype=torch.float16).pin_memory(),
                            torch.empty((seg_num, k), dtype=torch.int32).pin_memory())
            hv, hi = out_host
            hv.view(torch.int16).copy_(vals.view(torch.int16), non_blocking=True)
            hi.copy_(idx, non_blocking=True)
        s.synchronize()
    return hv, hi


# ---- PyTorch operator registration ---------------------------------------------------------
#
# torch.ops.batch_topk_b200.topk(x, k) and .topk_segmented(x, offsets, k): the same calls as
# topk / topk_segmented, registered as custom operators with fake (shape-only) kernels, so they
# trace under torch.compile and torch.export.  Each launch runs on the current stream.

@torch.library.custom_op("batch_topk_b200::topk", mutates_args=())
def _topk_op(x: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    return topk(x, k)


@_topk_op.register_fake
def _topk_op_fake(x: torch.Tensor, k: int):
    if x.dim() != 2 or x.dtype not in _ENTRY:
        raise ValueError("x must be a 2-D float16, bfloat16 or float32 tensor")
    return (x.new_empty((x.shape[0], k)), x.new_empty((x.shape[0], k), dtype=torch.int32))


@torch.library.custom_op("batch_topk_b200::topk_segmented", mutates_args=())
def _topk_segmented_op(x: torch.Tensor, offsets: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    return topk_segmented(x, offsets, k)


@_topk_segmented_op.register_fake
def _topk_segmented_op_fake(x: torch.Tensor, offsets: torch.Tensor, k: int):
    n = offsets.shape[0] - 1
    return (x.new_empty((n, k)), x.new_empty((n, k), dtype=torch.int32))
