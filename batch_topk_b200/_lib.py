"""ctypes binding of the C ABI declared in include/batch_topk_b200.h.

The shared library must exist (``python -m batch_topk_b200.build``); there is no fallback
implementation.  Loading it needs no GPU; calling the compute entry points does.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from .build import LIB

EXPORTED = (
    "bt_topk_half",
    "bt_topk_half_workspace_size",
    "bt_topk_half_segmented",
    "bt_topk_half_segmented_workspace_size",
    "bt_topk_half_noalloc",
    "bt_topk_bf16",
    "bt_topk_bf16_workspace_size",
    "bt_topk_bf16_segmented",
    "bt_topk_bf16_segmented_workspace_size",
    "bt_topk_f32",
    "bt_topk_f32_workspace_size",
    "bt_topk_f32_segmented",
    "bt_topk_f32_segmented_workspace_size",
    "bt_workspace_status",
    "bt_noalloc_status",
    "bt_logits_f16",
    "bt_logits_topk_f16_workspace_size",
    "bt_logits_topk_f16",
    "bt_logits_topk_status",
    "bt_set_handoff_wait_tries",
    "bt_set_profile_events",
    "bt_device_info",
    "bt_error_string",
    "bt_version",
)

_lock = threading.Lock()
_lib = None


class LibraryMissing(RuntimeError):
    pass


def load() -> C.CDLL:
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB):
            raise LibraryMissing(
                f"{LIB} is missing: build the CUDA library with `python -m batch_topk_b200.build`"
            )
        lib = C.CDLL(LIB)
        vp, sz, i32, i64 = C.c_void_p, C.c_size_t, C.c_int, C.c_longlong
        lib.bt_topk_half.argtypes = [vp, i32, i32, i32, vp, vp, vp, sz, vp]
        lib.bt_topk_half.restype = i32
        lib.bt_topk_half_workspace_size.argtypes = [i32, i32, i32]
        lib.bt_topk_half_workspace_size.restype = sz
        lib.bt_topk_half_segmented.argtypes = [vp, vp, i32, i64, i32, vp, vp, vp, sz, vp]
        lib.bt_topk_half_segmented.restype = i32
        lib.bt_topk_half_segmented_workspace_size.argtypes = [i32, i64, i32]
        lib.bt_topk_half_segmented_workspace_size.restype = sz
        lib.bt_topk_half_noalloc.argtypes = [vp, i32, i32, i32, vp, vp, vp]
        lib.bt_topk_half_noalloc.restype = i32
        lib.bt_topk_bf16.argtypes = [vp, i32, i32, i32, vp, vp, vp, sz, vp]
        lib.bt_topk_bf16.restype = i32
        lib.bt_topk_bf16_workspace_size.argtypes = [i32, i32, i32]
        lib.bt_topk_bf16_workspace_size.restype = sz
        lib.bt_topk_bf16_segmented.argtypes = [vp, vp, i32, i64, i32, vp, vp, vp, sz, vp]
        lib.bt_topk_bf16_segmented.restype = i32
        lib.bt_topk_bf16_segmented_workspace_size.argtypes = [i32, i64, i32]
        lib.bt_topk_bf16_segmented_workspace_size.restype = sz
        lib.bt_topk_f32.argtypes = [vp, i32, i32, i32, vp, vp, vp, sz, vp]
        lib.bt_topk_f32.restype = i32
        lib.bt_topk_f32_workspace_size.argtypes = [i32, i32, i32]
        lib.bt_topk_f32_workspace_size.restype = sz
        lib.bt_topk_f32_segmented.argtypes = [vp, vp, i32, i64, i32, vp, vp, vp, sz, vp]
        lib.bt_topk_f32_segmented.restype = i32
        lib.bt_topk_f32_segmented_workspace_size.argtypes = [i32, i64, i32]
        lib.bt_topk_f32_segmented_workspace_size.restype = sz
        lib.bt_workspace_status.argtypes = [vp, i32, vp, C.POINTER(C.c_uint * 6)]
        lib.bt_workspace_status.restype = i32
        lib.bt_noalloc_status.argtypes = [vp, C.POINTER(C.c_uint * 6)]
        lib.bt_noalloc_status.restype = i32
        lib.bt_logits_f16.argtypes = [vp, vp, i32, i32, i32, vp, vp]
        lib.bt_logits_f16.restype = i32
        lib.bt_logits_topk_f16_workspace_size.argtypes = [i32, i32, i32, i32]
        lib.bt_logits_topk_f16_workspace_size.restype = sz
        lib.bt_logits_topk_f16.argtypes = [vp, vp, i32, i32, i32, i32, vp, vp, vp, sz, vp]
        lib.bt_logits_topk_f16.restype = i32
        lib.bt_logits_topk_status.argtypes = [vp, i32, i32, i32, i32, vp]
        lib.bt_logits_topk_status.restype = i32
        lib.bt_set_handoff_wait_tries.argtypes = [i32]
        lib.bt_set_handoff_wait_tries.restype = None
        lib.bt_set_profile_events.argtypes = [vp, vp]
        lib.bt_set_profile_events.restype = None
        lib.bt_error_string.argtypes = [i32]
        lib.bt_error_string.restype = C.c_char_p
        lib.bt_device_info.argtypes = [C.POINTER(C.c_int), i32]
        lib.bt_device_info.restype = i32
        lib.bt_version.argtypes = []
        lib.bt_version.restype = i32
        _lib = lib
        return lib
