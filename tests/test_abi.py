"""The C ABI without a GPU: the library loads, exports every function include/ declares, and
keeps the reference's argument-error contract (src/batch_topk.cu:35-60 of
fire-emblem/batch_topk; test/test_batch_topk.cu:1168-1174 and :1340-1373).  Every call here
is rejected on the host before any CUDA work, so none needs a device.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess

import pytest

import batch_topk_b200 as bt
from batch_topk_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "batch_topk_b200.h")
INVALID = bt.CUDA_ERROR_INVALID_VALUE
FAKE = 1 << 20  # a 16-byte aligned address that is never dereferenced


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^[A-Za-z_][\w \*]*?\b(bt_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_bound_symbols():
    names = declared_functions()
    assert "bt_topk_half" in names and "bt_topk_half_workspace_size" in names
    assert sorted(_lib.EXPORTED) == names


def test_library_exports_every_declared_function():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", bt.library_path()], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\b[TW] (bt_\w+)$", out, flags=re.M))
    assert set(declared_functions()) <= exported


def test_workspace_size_contract():
    # the reference's zero cases that stay invalid here
    assert bt.batch_topk_half_workspace_size(0, 10000, 50) == 0
    assert bt.batch_topk_half_workspace_size(1, 10, 11) == 0
    assert bt.batch_topk_half_workspace_size(1, 0, 1) == 0
    assert bt.batch_topk_half_workspace_size(1, 10000, 0) == 0
    assert bt.batch_topk_half_workspace_size(1, 10000, bt.MAX_K + 1) == 0
    assert bt.batch_topk_half_workspace_size(1, bt.MAX_SEG_LEN + 1, 50) == 0
    # the reference rejects these (seg_len > 10000, k > 128); this library supports them
    assert bt.batch_topk_half_workspace_size(1, 10001, 50) > 0
    assert bt.batch_topk_half_workspace_size(1, 10000, 129) > 0
    # monotone in the batch size, 256-byte granular
    a = bt.batch_topk_half_workspace_size(1, 10000, 50)
    b = bt.batch_topk_half_workspace_size(1000, 10000, 50)
    assert 0 < a < b and a % 256 == 0 and b % 256 == 0
    assert bt.batch_topk_half_segmented_workspace_size(0, 10, 1) == 0
    assert bt.batch_topk_half_segmented_workspace_size(4, -1, 1) == 0
    assert bt.batch_topk_half_segmented_workspace_size(4, 100, 0) == 0
    assert bt.batch_topk_half_segmented_workspace_size(4, 0, 50) > 0  # all-empty batch is valid


def call_fixed(inp=FAKE, seg_num=2, seg_len=100, k=5, ov=FAKE, oi=FAKE, ws=FAKE, wsb=None):
    if wsb is None:
        wsb = bt.batch_topk_half_workspace_size(max(seg_num, 1), max(seg_len, 1), max(k, 1))
    return bt.batch_topk_half(inp, seg_num, seg_len, k, ov, oi, ws, wsb, 0)


def test_fixed_argument_errors():
    need = bt.batch_topk_half_workspace_size(2, 100, 5)
    assert call_fixed(inp=0) == INVALID
    assert call_fixed(ov=0) == INVALID
    assert call_fixed(oi=0) == INVALID
    assert call_fixed(ws=0) == INVALID
    assert call_fixed(seg_num=0) == INVALID
    assert call_fixed(seg_len=0) == INVALID
    assert call_fixed(k=0) == INVALID
    assert call_fixed(k=101) == INVALID  # k > seg_len
    assert call_fixed(k=bt.MAX_K + 1, seg_len=5000) == INVALID
    assert call_fixed(wsb=need - 1) == INVALID  # short workspace
    assert call_fixed(inp=FAKE + 1) == INVALID  # fp16 input must be 2-byte aligned
    assert call_fixed(oi=FAKE + 2) == INVALID  # int32 indices must be 4-byte aligned
    assert call_fixed(ws=FAKE + 8) == INVALID  # workspace must be 16-byte aligned


def test_segmented_argument_errors():
    need = bt.batch_topk_half_segmented_workspace_size(4, 1000, 8)

    def call(off=FAKE, seg_num=4, total=1000, k=8, ws=FAKE, wsb=need):
        return bt.batch_topk_half_segmented(FAKE, off, seg_num, total, k, FAKE, FAKE, ws, wsb, 0)

    assert call(off=0) == INVALID
    assert call(off=FAKE + 2) == INVALID
    assert call(seg_num=0) == INVALID
    assert call(total=-1) == INVALID
    assert call(total=1 << 31) == INVALID
    assert call(k=0) == INVALID
    assert call(ws=0) == INVALID
    assert call(wsb=need - 1) == INVALID


def test_error_strings_and_version():
    lib = _lib.load()
    assert lib.bt_error_string(0) == b"success"
    assert b"invalid" in lib.bt_error_string(INVALID)
    assert bt.version() == 100
    with pytest.raises(bt.BatchTopkError, match="invalid"):
        raise bt.BatchTopkError(INVALID, "bt_topk_half")


def test_workspace_status_rejects_null():
    stats = (C.c_uint * 6)()
    assert _lib.load().bt_workspace_status(None, 0, None, C.byref(stats)) == INVALID


def test_logits_argument_errors():
    """The logits producer rejects null or misaligned pointers before any CUDA work."""
    assert bt.logits_f16(0, FAKE, 4, 100, 64, FAKE, 0) == INVALID
    assert bt.logits_f16(FAKE, 0, 4, 100, 64, FAKE, 0) == INVALID
    assert bt.logits_f16(FAKE, FAKE, 4, 100, 64, 0, 0) == INVALID
    assert bt.logits_f16(FAKE + 2, FAKE, 4, 100, 64, FAKE, 0) == INVALID  # not 16-byte aligned
    assert bt.logits_f16(FAKE, FAKE, 4, 100, 64, FAKE + 1, 0) == INVALID  # not 2-byte aligned
    assert bt.logits_topk_f16(0, FAKE, 4, 100, 64, 8, FAKE, FAKE, FAKE, 1 << 20, 0) == INVALID
    assert bt.logits_topk_f16(FAKE, FAKE, 4, 100, 64, 8, FAKE, FAKE + 2, FAKE, 1 << 20, 0) == INVALID
    assert bt.logits_topk_f16(FAKE, FAKE, 4, 100, 64, 8, FAKE, FAKE, FAKE + 16, 1 << 20, 0) == INVALID
