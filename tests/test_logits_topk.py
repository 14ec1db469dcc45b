"""The logits producer and its fused top-k epilogue (bt_logits_f16, bt_logits_topk_f16).

No reference counterpart: the reference selects from logits already in memory.  The checks:
- the producer's fp16 logits against torch's fp32 matmul of the same fp16 inputs (within about
  one fp16 rounding step; exactly, when every product and sum is exact in fp32);
- the fused top-k, bit for bit (values and vocabulary indices), against the C checker applied to
  the producer's stored logits -- i.e. against the unfused path (producer, then top-k);
- on tie-heavy logits (quantised inputs: many exactly equal logits spread over every CTA's
  vocabulary range), where the lower-index rule has to hold across CTAs;
- argument errors.
"""
from __future__ import annotations

import numpy as np
import pytest

import batch_topk_b200 as bt

SHAPES = [  # M, V, D, k
    (1, 1000, 64, 1),
    (7, 5000, 128, 50),
    (33, 129, 8, 10),
    (128, 300, 72, 64),
    (64, 32000, 512, 50),
    (5, 70000, 256, 64),
    (64, 128256, 4096, 50),  # C2's batch and vocabulary at a 4096-wide hidden state
]


def _inputs(torch, M, V, D, seed, kind):
    g = torch.Generator(device="cuda").manual_seed(seed)
    H = torch.randn((M, D), generator=g, device="cuda", dtype=torch.float32)
    W = torch.randn((V, D), generator=g, device="cuda", dtype=torch.float32) / (D ** 0.5)
    if kind == "ties":  # small integers and quarters: exact fp32 sums, many equal logits
        H = H.round().clamp(-2, 2)
        W = (W * 4).round().clamp(-4, 4) / 4
    return H.half().contiguous(), W.half().contiguous()


def _stream(torch):
    return torch.cuda.current_stream().cuda_stream


def _logits(torch, H, W):
    M, D = H.shape
    V = W.shape[0]
    out = torch.empty((M, V), dtype=torch.float16, device="cuda")
    rc = bt.logits_f16(H.data_ptr(), W.data_ptr(), M, V, D, out.data_ptr(), _stream(torch))
    assert rc == 0, rc
    return out


def _fused(torch, H, W, k):
    M, D = H.shape
    V = W.shape[0]
    nb = bt.logits_topk_f16_workspace_size(M, V, D, k)
    assert nb > 0
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    ov = torch.empty((M, k), dtype=torch.int16, device="cuda")
    oi = torch.empty((M, k), dtype=torch.int32, device="cuda")
    rc = bt.logits_topk_f16(H.data_ptr(), W.data_ptr(), M, V, D, k, ov.data_ptr(), oi.data_ptr(),
                            ws.data_ptr(), nb, _stream(torch))
    assert rc == 0, rc
    assert bt.logits_topk_status(ws.data_ptr(), M, V, D, k, _stream(torch)) == 0
    return ov, oi


@pytest.mark.gpu
@pytest.mark.parametrize("M,V,D,k", SHAPES)
@pytest.mark.parametrize("kind", ["normal", "ties"])
def test_fused_topk_equals_unfused(orc, M, V, D, k, kind):
    import torch

    H, W = _inputs(torch, M, V, D, 1000 + 7 * M + V + D, kind)
    logits = _logits(torch, H, W)
    ref = H.float() @ W.float().T
    if kind == "ties":
        assert torch.equal(logits.float(), ref.half().float())
    else:
        torch.testing.assert_close(logits.float(), ref, rtol=2e-3, atol=2e-3)
    ov, oi = _fused(torch, H, W, k)
    torch.cuda.synchronize()
    ev, ei = orc.topk(logits.cpu().numpy().view(np.uint16), k)
    assert np.array_equal(oi.cpu().numpy(), ei)
    assert np.array_equal(ov.cpu().numpy().view(np.uint16), ev)


@pytest.mark.gpu
def test_fused_topk_repeated_calls_and_streams(orc):
    """Back-to-back calls on one workspace, then on a second stream, give the same answer."""
    import torch

    M, V, D, k = 16, 20000, 256, 32
    H, W = _inputs(torch, M, V, D, 77, "normal")
    logits = _logits(torch, H, W)
    ev, ei = orc.topk(logits.cpu().numpy().view(np.uint16), k)
    for _ in range(3):
        ov, oi = _fused(torch, H, W, k)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ov2, oi2 = _fused(torch, H, W, k)
    torch.cuda.synchronize()
    for v, i in ((ov, oi), (ov2, oi2)):
        assert np.array_equal(i.cpu().numpy(), ei)
        assert np.array_equal(v.cpu().numpy().view(np.uint16), ev)


@pytest.mark.gpu
def test_logits_argument_errors():
    import torch

    H = torch.zeros((4, 64), dtype=torch.float16, device="cuda")
    W = torch.zeros((100, 64), dtype=torch.float16, device="cuda")
    out = torch.empty((4, 100), dtype=torch.float16, device="cuda")
    s = _stream(torch)
    invalid = 1  # cudaErrorInvalidValue
    assert bt.logits_f16(H.data_ptr(), W.data_ptr(), 129, 100, 64, out.data_ptr(), s) == invalid
    assert bt.logits_f16(H.data_ptr(), W.data_ptr(), 4, 100, 60, out.data_ptr(), s) == invalid
    assert bt.logits_f16(H.data_ptr() + 2, W.data_ptr(), 4, 100, 64, out.data_ptr(), s) == invalid
    assert bt.logits_topk_f16_workspace_size(4, 100, 64, 65) == 0
    assert bt.logits_topk_f16_workspace_size(4, 10, 64, 11) == 0
    nb = bt.logits_topk_f16_workspace_size(4, 100, 64, 8)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    ov = torch.empty((4, 8), dtype=torch.int16, device="cuda")
    oi = torch.empty((4, 8), dtype=torch.int32, device="cuda")
    assert bt.logits_topk_f16(H.data_ptr(), W.data_ptr(), 4, 100, 64, 8, ov.data_ptr(),
                              oi.data_ptr(), ws.data_ptr(), nb - 1, s) == invalid
    torch.cuda.synchronize()
