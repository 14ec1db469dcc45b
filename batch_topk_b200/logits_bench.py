"""Timing command for the logits producer and its fused top-k.

    python -m batch_topk_b200.logits_bench [--shape M,V,D,k ...] [--iters N] [--once]

For each shape it builds H[M, D] and W[V, D] (seeded normal values, W scaled by 1/sqrt(D)) on
the device and prints one JSON line with the device time per call (CUDA events, after 3 warm-up
calls) of: the producer alone (bt_logits_f16), the producer followed by bt_topk_half on its
logits (unfused), the fused entry point (bt_logits_topk_f16), and torch.matmul for reference;
plus whether the fused and unfused answers agree bit for bit.  --once runs one unfused and one
fused call per shape, checks that they agree, and times nothing (a short command to profile).
"""
from __future__ import annotations

import argparse
import json

import torch

import batch_topk_b200 as bt

DEFAULT_SHAPES = ["64,128256,4096,50", "128,128256,4096,50", "1,128256,4096,50",
                  "64,32000,4096,50", "64,151936,8192,50"]


class Problem:
    def __init__(self, M: int, V: int, D: int, k: int, seed: int = 5):
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(seed)
        self.M, self.V, self.D, self.k = M, V, D, k
        self.H = torch.randn((M, D), generator=g, device=dev).half()
        self.W = (torch.randn((V, D), generator=g, device=dev) / D ** 0.5).half()
        self.logits = torch.empty((M, V), dtype=torch.float16, device=dev)
        self.nb_u = bt.batch_topk_half_workspace_size(M, V, k)
        self.ws_u = torch.empty(self.nb_u, dtype=torch.uint8, device=dev)
        self.nb_f = bt.logits_topk_f16_workspace_size(M, V, D, k)
        if self.nb_f == 0:
            raise ValueError(f"unsupported shape {M},{V},{D},{k}")
        self.ws_f = torch.empty(self.nb_f, dtype=torch.uint8, device=dev)
        self.ov_u = torch.empty((M, k), dtype=torch.int16, device=dev)
        self.oi_u = torch.empty((M, k), dtype=torch.int32, device=dev)
        self.ov_f = torch.empty_like(self.ov_u)
        self.oi_f = torch.empty_like(self.oi_u)

    def _stream(self) -> int:
        return torch.cuda.current_stream().cuda_stream

    def producer(self) -> None:
        rc = bt.logits_f16(self.H.data_ptr(), self.W.data_ptr(), self.M, self.V, self.D,
                           self.logits.data_ptr(), self._stream())
        if rc:
            raise bt.BatchTopkError(rc, "bt_logits_f16")

    def unfused(self) -> None:
        self.producer()
        rc = bt.batch_topk_half(self.logits.data_ptr(), self.M, self.V, self.k,
                                self.ov_u.data_ptr(), self.oi_u.data_ptr(), self.ws_u.data_ptr(),
                                self.nb_u, self._stream())
        if rc:
            raise bt.BatchTopkError(rc, "bt_topk_half")

    def fused(self) -> None:
        rc = bt.logits_topk_f16(self.H.data_ptr(), self.W.data_ptr(), self.M, self.V, self.D,
                                self.k, self.ov_f.data_ptr(), self.oi_f.data_ptr(),
                                self.ws_f.data_ptr(), self.nb_f, self._stream())
        if rc:
            raise bt.BatchTopkError(rc, "bt_logits_topk_f16")

    def cublas(self) -> None:
        torch.matmul(self.H, self.W.t())

    def agree(self) -> bool:
        return bool(torch.equal(self.ov_u, self.ov_f) and torch.equal(self.oi_u, self.oi_f))


def time_us(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / iters


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--shape", action="append", help="M,V,D,k (repeatable)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--once", action="store_true", help="one unfused and one fused call per shape")
    a = ap.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("a CUDA device is required")
    for spec in a.shape or DEFAULT_SHAPES:
        M, V, D, k = (int(x) for x in spec.split(","))
        pb = Problem(M, V, D, k)
        if a.once:
            pb.unfused()
            pb.fused()
            torch.cuda.synchronize()
            line = {"M": M, "V": V, "D": D, "k": k, "agree": pb.agree()}
        else:
            line = {"M": M, "V": V, "D": D, "k": k,
                    "producer_us": round(time_us(pb.producer, a.iters), 2),
                    "unfused_us": round(time_us(pb.unfused, a.iters), 2),
                    "fused_us": round(time_us(pb.fused, a.iters), 2),
                    "torch_matmul_us": round(time_us(pb.cublas, a.iters), 2)}
            line["weight_gbs_producer"] = round(V * D * 2 / line["producer_us"] / 1e3, 1)
            line["agree"] = pb.agree()
        line["status"] = bt.logits_topk_status(pb.ws_f.data_ptr(), M, V, D, k,
                                               torch.cuda.current_stream().cuda_stream)
        print(json.dumps(line), flush=True)
        if not line["agree"] or line["status"]:
            raise SystemExit(1)


if __name__ == "__main__":
    main()
