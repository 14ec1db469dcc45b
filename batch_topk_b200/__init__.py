"""batch_topk_b200 -- batched fp16 top-k for NVIDIA B200 (sm_100a).

Host-side mirror of fire-emblem/batch_topk's operator interface
(include/batch_topk.cuh:10-21): the same entry-point names, argument meaning and error
contract (cudaError_t codes, cudaErrorInvalidValue == 1 for bad arguments), called through
the C ABI of ``lib/libbatch_topk_b200.so``.  Pointers are device addresses (ints), the
stream is a cudaStream_t handle (int, 0 = default stream).

``batch_topk_b200.torch_api`` adds tensor-level helpers (``topk``, ``topk_segmented``).
"""
from __future__ import annotations

import ctypes as C

from . import _lib

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_VALUE = 1
MAX_K = 1024
MAX_SEG_LEN = 1 << 26
NOALLOC_SCRATCH_BYTES = 32 << 20  # BT_NOALLOC_SCRATCH_BYTES

STATUS_WAIT_TIMEOUT = 1
STATUS_BAD_OFFSETS = 2
STATUS_SEGMENT_TOO_LONG = 4
STATUS_CERTIFY_FAILED = 8
STATUS_FLAGS = {
    1: "a bounded device wait (bulk copy or hand-off) timed out",
    2: "CSR offsets decreasing or beyond max_total_len",
    4: "segment longer than the supported maximum",
    8: "candidate certification failed",
}


class BatchTopkError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = _lib.load().bt_error_string(code).decode()
        super().__init__(f"{what}: error {code}: {msg}" if what else f"error {code}: {msg}")


class DeviceStatusError(RuntimeError):
    """A device-side check of a call failed (its workspace status word holds STATUS_* flags)."""

    def __init__(self, flags: int, what: str = ""):
        self.flags = flags
        names = "; ".join(v for b, v in STATUS_FLAGS.items() if flags & b)
        super().__init__(f"{what}: device status {flags:#x} ({names})" if what
                         else f"device status {flags:#x} ({names})")


def batch_topk_half(d_input: int, seg_num: int, seg_len: int, k: int, d_output_values: int,
                    d_output_indices: int, d_workspace: int, workspace_bytes: int,
                    stream: int = 0) -> int:
    """radix_topk::batch_topk_half: returns a cudaError_t code; asynchronous on `stream`."""
    return _lib.load().bt_topk_half(d_input, seg_num, seg_len, k, d_output_values,
                                    d_output_indices, d_workspace, workspace_bytes, stream)


def batch_topk_half_workspace_size(seg_num: int, seg_len: int, k: int) -> int:
    """radix_topk::batch_topk_half_workspace_size: 0 for an unsupported shape."""
    return int(_lib.load().bt_topk_half_workspace_size(seg_num, seg_len, k))


def batch_topk_half_segmented(d_input: int, d_offsets: int, seg_num: int, max_total_len: int,
                              k: int, d_output_values: int, d_output_indices: int,
                              d_workspace: int, workspace_bytes: int, stream: int = 0) -> int:
    """CSR variant (no reference counterpart): int32 offsets[seg_num+1] on the device."""
    return _lib.load().bt_topk_half_segmented(d_input, d_offsets, seg_num, max_total_len, k,
                                              d_output_values, d_output_indices, d_workspace,
                                              workspace_bytes, stream)


def batch_topk_half_segmented_workspace_size(seg_num: int, max_total_len: int, k: int) -> int:
    return int(_lib.load().bt_topk_half_segmented_workspace_size(seg_num, max_total_len, k))


def batch_topk_bf16(d_input: int, seg_num: int, seg_len: int, k: int, d_output_values: int,
                    d_output_indices: int, d_workspace: int, workspace_bytes: int,
                    stream: int = 0) -> int:
    """batch_topk_half for bfloat16 rows (no reference counterpart): the same contract, with
    values ordered as bfloat16."""
    return _lib.load().bt_topk_bf16(d_input, seg_num, seg_len, k, d_output_values,
                                    d_output_indices, d_workspace, workspace_bytes, stream)


def batch_topk_bf16_workspace_size(seg_num: int, seg_len: int, k: int) -> int:
    return int(_lib.load().bt_topk_bf16_workspace_size(seg_num, seg_len, k))


def batch_topk_bf16_segmented(d_input: int, d_offsets: int, seg_num: int, max_total_len: int,
                              k: int, d_output_values: int, d_output_indices: int,
                              d_workspace: int, workspace_bytes: int, stream: int = 0) -> int:
    """CSR variant for bfloat16 values (no reference counterpart); -inf (0xFF80) pads."""
    return _lib.load().bt_topk_bf16_segmented(d_input, d_offsets, seg_num, max_total_len, k,
                                              d_output_values, d_output_indices, d_workspace,
                                              workspace_bytes, stream)


def batch_topk_bf16_segmented_workspace_size(seg_num: int, max_total_len: int, k: int) -> int:
    return int(_lib.load().bt_topk_bf16_segmented_workspace_size(seg_num, max_total_len, k))


def batch_topk_f32(d_input: int, seg_num: int, seg_len: int, k: int, d_output_values: int,
                   d_output_indices: int, d_workspace: int, workspace_bytes: int,
                   stream: int = 0) -> int:
    """batch_topk_half for float32 rows (no reference counterpart): 32-bit values in and out
    (4-byte aligned), the same contract and order (NaN last, -0 == +0, ties by index)."""
    return _lib.load().bt_topk_f32(d_input, seg_num, seg_len, k, d_output_values,
                                   d_output_indices, d_workspace, workspace_bytes, stream)


def batch_topk_f32_workspace_size(seg_num: int, seg_len: int, k: int) -> int:
    return int(_lib.load().bt_topk_f32_workspace_size(seg_num, seg_len, k))


def batch_topk_f32_segmented(d_input: int, d_offsets: int, seg_num: int, max_total_len: int,
                             k: int, d_output_values: int, d_output_indices: int,
                             d_workspace: int, workspace_bytes: int, stream: int = 0) -> int:
    """CSR variant for float32 values (no reference counterpart); -inf (0xFF800000) pads."""
    return _lib.load().bt_topk_f32_segmented(d_input, d_offsets, seg_num, max_total_len, k,
                                             d_output_values, d_output_indices, d_workspace,
                                             workspace_bytes, stream)


def batch_topk_f32_segmented_workspace_size(seg_num: int, max_total_len: int, k: int) -> int:
    return int(_lib.load().bt_topk_f32_segmented_workspace_size(seg_num, max_total_len, k))


def batch_topk_half_noalloc(d_input: int, seg_num: int, seg_len: int, k: int,
                            d_output_values: int, d_output_indices: int, stream: int = 0) -> int:
    """bt_topk_half_noalloc (no reference counterpart): batch_topk_half on the library's fixed
    scratch array instead of a caller workspace, for callers that may not allocate device
    memory at call time.  Returns cudaErrorInvalidValue when the shape's workspace exceeds
    NOALLOC_SCRATCH_BYTES.  Calls that can overlap on the GPU share that array and race."""
    return _lib.load().bt_topk_half_noalloc(d_input, seg_num, seg_len, k, d_output_values,
                                            d_output_indices, stream)


LOGITS_MAX_K = 64


def logits_f16(d_hidden: int, d_weight: int, M: int, V: int, D: int, d_logits: int,
               stream: int = 0) -> int:
    """bt_logits_f16 (no reference counterpart): logits[M, V] = hidden[M, D] . weight[V, D]^T in
    fp16 (fp32 accumulation on the tensor cores), stored row-major."""
    return _lib.load().bt_logits_f16(d_hidden, d_weight, M, V, D, d_logits, stream)


def logits_topk_f16_workspace_size(M: int, V: int, D: int, k: int) -> int:
    return int(_lib.load().bt_logits_topk_f16_workspace_size(M, V, D, k))


def logits_topk_f16(d_hidden: int, d_weight: int, M: int, V: int, D: int, k: int,
                    d_output_values: int, d_output_indices: int, d_workspace: int,
                    workspace_bytes: int, stream: int = 0) -> int:
    """bt_logits_topk_f16 (no reference counterpart): the top k of each row of the logits that
    logits_f16 would store, with batch_topk_half's order and layout, without storing them."""
    return _lib.load().bt_logits_topk_f16(d_hidden, d_weight, M, V, D, k, d_output_values,
                                          d_output_indices, d_workspace, workspace_bytes, stream)


def logits_topk_status(d_workspace: int, M: int, V: int, D: int, k: int, stream: int = 0) -> int:
    """Status flags of the last logits_topk_f16 call on this workspace (synchronous)."""
    rc = int(_lib.load().bt_logits_topk_status(d_workspace, M, V, D, k, stream))
    if rc < 0:
        raise BatchTopkError(-rc, "bt_logits_topk_status")
    return rc


def workspace_status(d_workspace: int, seg_num: int = 0, stream: int = 0):
    """Synchronously reads the device status of the last call on this workspace.

    Returns (flags, stats) where stats = (exact-select chunks, chunks with no candidate,
    group-max selects, rows emitted, verified first-chunk guesses, reserved); stats are only
    counted with BT_STATS=1."""
    stats = (C.c_uint * 6)()
    rc = _lib.load().bt_workspace_status(d_workspace, seg_num, stream, C.byref(stats))
    if rc < 0:
        raise BatchTopkError(-rc, "bt_workspace_status")
    return rc, tuple(int(v) for v in stats)


def noalloc_status(stream: int = 0):
    """workspace_status for batch_topk_half_noalloc: the status of the last no-alloc call on
    the current device, read from the library's fixed scratch array (allocates nothing)."""
    stats = (C.c_uint * 6)()
    rc = _lib.load().bt_noalloc_status(stream, C.byref(stats))
    if rc < 0:
        raise BatchTopkError(-rc, "bt_noalloc_status")
    return rc, tuple(int(v) for v in stats)


def set_handoff_wait_tries(tries: int | None) -> None:
    """Failure-path test hook: tries of each consumer <-> merger hand-off wait of later calls
    (0: fail at once, so the call ends with STATUS_WAIT_TIMEOUT; None: the default)."""
    _lib.load().bt_set_handoff_wait_tries(-1 if tries is None else int(tries))


def set_profile_events(ev_start: int | None, ev_stop: int | None) -> None:
    """Record cudaEvent_t handles around the streaming kernel of later calls (None: off)."""
    _lib.load().bt_set_profile_events(ev_start or None, ev_stop or None)


def device_info() -> dict:
    """SM count, resident blocks per SM and shared memory per block of the top-k kernel."""
    import ctypes as C

    buf = (C.c_int * 6)()
    rc = _lib.load().bt_device_info(buf, 6)
    if rc != 0:
        raise BatchTopkError(rc, "bt_device_info")
    keys = ("sms", "blocks_per_sm_small_k", "blocks_per_sm_large_k", "smem_small_k",
            "smem_large_k", "threads_per_block")
    return dict(zip(keys, list(buf)))


def version() -> int:
    return int(_lib.load().bt_version())


def library_path() -> str:
    from .build import LIB

    return LIB
