"""Device-side generation of the five benchmark configurations, bit-identical to the host
generators in workloads.py (the C ABI of include/batch_topk_b200_gen.h does the per-element
work on the GPU; the few per-row facts -- C3's level table, C2's 20 outliers, C5's row
constants -- come from workloads.py, and C5's ascending rows are sorted on the device).

Each function returns an int16 CUDA tensor of fp16 bit patterns with the same shape and
bits as its workloads.py counterpart, so a shard of any configuration is generated in place
on its own device without a host upload.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from . import workloads as wl

_bound = None


def _gen_lib():
    global _bound
    if _bound is None:
        lib = _lib.load()
        vp, i64, u64, dbl = C.c_void_p, C.c_longlong, C.c_ulonglong, C.c_double
        lib.bt_gen_normal.argtypes = [vp, i64, u64, u64, u64, dbl, vp]
        lib.bt_gen_uniform.argtypes = [vp, i64, u64, u64, u64, dbl, dbl, vp]
        lib.bt_gen_levels.argtypes = [vp, i64, u64, u64, u64, vp, vp]
        lib.bt_gen_mask.argtypes = [vp, i64, u64, u64, u64, dbl, C.c_ushort, vp]
        for f in (lib.bt_gen_normal, lib.bt_gen_uniform, lib.bt_gen_levels, lib.bt_gen_mask):
            f.restype = C.c_int
        _bound = lib
    return _bound


def _check(rc: int, what: str):
    if rc != 0:
        from . import BatchTopkError

        raise BatchTopkError(rc, what)


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _rows(cfg, rows):
    return [int(r) for r in wl._rows(cfg, rows)]


def _runs(rows):
    """Maximal runs of consecutive row numbers: (first row, count, output position)."""
    out, i = [], 0
    while i < len(rows):
        j = i
        while j + 1 < len(rows) and rows[j + 1] == rows[j] + 1:
            j += 1
        out.append((rows[i], j - i + 1, i))
        i = j + 1
    return out


def normal_(out: torch.Tensor, idx0: int, seed: int, stream_id: int, sigma: float = 1.0):
    _check(_gen_lib().bt_gen_normal(out.data_ptr(), out.numel(), idx0, seed, stream_id, sigma,
                                    _stream(out.device)), "bt_gen_normal")
    return out


def uniform_(out: torch.Tensor, idx0: int, seed: int, stream_id: int, lo: float, hi: float):
    _check(_gen_lib().bt_gen_uniform(out.data_ptr(), out.numel(), idx0, seed, stream_id, lo, hi,
                                     _stream(out.device)), "bt_gen_uniform")
    return out


def _rowwise(cfg, rows, seg_len, device, fill):
    """[len(rows), seg_len] int16 tensor; fill(view, first_flat_index) writes each run."""
    r = _rows(cfg, rows)
    out = torch.empty((len(r), seg_len), dtype=torch.int16, device=device)
    for row0, count, pos in _runs(r):
        fill(out[pos:pos + count].reshape(-1), row0 * seg_len)
    return out


def gen_c1(rows=None, seg_len=None, seed=None, device="cuda"):
    cfg = wl.CONFIGS["C1"]
    L, s = seg_len or cfg.seg_len, seed or cfg.seed
    return _rowwise(cfg, rows, L, device, lambda v, i0: normal_(v, i0, s, 0))


def gen_c2(rows=None, seg_len=None, seed=None, device="cuda"):
    cfg = wl.CONFIGS["C2"]
    L, s = seg_len or cfg.seg_len, seed or cfg.seed

    def fill(v, i0):
        normal_(v, i0, s, 0, 2.0)
        _check(_gen_lib().bt_gen_mask(v.data_ptr(), v.numel(), i0, s, 1, 0.05, 0xFC00,
                                      _stream(v.device)), "bt_gen_mask")

    out = _rowwise(cfg, rows, L, device, fill)
    for j, row in enumerate(_rows(cfg, rows)):  # the 20 planted outliers of each row
        pos, vals = wl.c2_outliers(row, L, s)
        out[j, torch.from_numpy(pos).to(out.device)] = torch.from_numpy(
            vals.view(np.int16).copy()).to(out.device)
    return out


def gen_c3(rows=None, seg_len=None, seed=None, device="cuda"):
    cfg = wl.CONFIGS["C3"]
    L, s = seg_len or cfg.seg_len, seed or cfg.seed
    levels = torch.from_numpy(wl.c3_levels(s).view(np.int16).copy()).to(device)

    def fill(v, i0):
        _check(_gen_lib().bt_gen_levels(v.data_ptr(), v.numel(), i0, s, 0, levels.data_ptr(),
                                        _stream(v.device)), "bt_gen_levels")

    return _rowwise(cfg, rows, L, device, fill)


def gen_c4_range(s0: int, s1: int, seed=None, device="cuda"):
    """Values of C4 segments [s0, s1) (1-D), as workloads.gen_c4_range."""
    s = seed or wl.CONFIGS["C4"].seed
    off = wl.c4_offsets(seed=s)
    b, e = int(off[s0]), int(off[s1])
    out = torch.empty((e - b,), dtype=torch.int16, device=device)
    return uniform_(out, b, s, 0, -1.0, 1.0)


def sort_ascending_bits_(rows: torch.Tensor):
    """In place, per row: fp16 bits ascending by value, equal values (+0/-0) by raw bits --
    workloads.sort_ascending_bits on the device."""
    b = rows.to(torch.int32) & 0xFFFF
    nan = ((b & 0x7C00) == 0x7C00) & ((b & 0x03FF) != 0)
    zero = (b & 0x7FFF) == 0
    norm = torch.where(nan, torch.full_like(b, 0xFFFF), torch.where(zero, torch.zeros_like(b), b))
    asc = torch.where((norm & 0x8000) != 0, (~norm) & 0xFFFF, norm ^ 0x8000)
    comp = (asc.to(torch.int64) << 16) | b.to(torch.int64)
    srt, _ = torch.sort(comp, dim=-1)
    rows.copy_((srt & 0xFFFF).to(torch.int32).to(torch.int16))
    return rows


def gen_c5(rows=None, seg_len=None, seed=None, device="cuda"):
    cfg = wl.CONFIGS["C5"]
    L, s = seg_len or cfg.seg_len, seed or cfg.seed
    r = _rows(cfg, rows)
    out = torch.empty((len(r), L), dtype=torch.int16, device=device)
    for j, row in enumerate(r):
        kind = row % 3
        if kind == 0:  # one constant per row
            c = int(wl.uniform_half(s, 30, np.array([row], np.int64), -4.0, 4.0)[0])
            out[j].fill_(c - 0x10000 if c >= 0x8000 else c)
        elif kind == 1:  # N(0,1), sorted ascending
            normal_(out[j], row * L, s, 0)
            sort_ascending_bits_(out[j])
        else:  # U[1,2)
            uniform_(out[j], row * L, s, 0, 1.0, 2.0)
    return out
