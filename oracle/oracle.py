"""ctypes bindings for the parity checker (test infrastructure only).

``Oracle`` wraps ``oracle/_build/liboracle.so`` (the C restatement in ``topk_oracle.c``).
``RefOracle`` wraps ``oracle/_ref/libref_oracle.so`` (the reference's own CPU top-k,
``include/batch_topk_types.cuh:50-92`` of fire-emblem/batch_topk), which only exists where
the reference tree was present at build time.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_oracle.so")
REF_GPU_LIB_PATH = os.path.join(HERE, "_ref", "libref_gpu.so")
_lock = threading.Lock()
_oracle = None
_ref = None

METHOD_SORT = 0  # the reference's algorithm: sort the index permutation
METHOD_COUNT = 1  # counting select on the descending key, same order, O(n)


def reference_dir() -> str | None:
    """The reference tree (fire-emblem/batch_topk) if it is present: the directory named by
    BT_REFERENCE_DIR, else a ``reference`` directory beside this repository; None otherwise."""
    cands = [os.environ.get("BT_REFERENCE_DIR"),
             os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for d in cands:
        if d and os.path.isfile(os.path.join(d, "include", "batch_topk_types.cuh")):
            return d
    return None


def build(ref: bool = True) -> None:
    """Compile the checker (and, when the reference tree exists, oracle/_ref)."""
    targets = ["all"] if ref else ["oracle"]
    cmd = ["make", "-s", "-C", HERE, *targets]
    rd = reference_dir() if ref else None
    if rd:
        cmd.append(f"REF={rd}")
    subprocess.run(cmd, check=True)


def encode_desc(bits: np.ndarray) -> np.ndarray:
    """Vectorised include/type_codec.cuh:13-38 (normalize, then desc = ~asc)."""
    b = np.asarray(bits, dtype=np.uint16)
    is_nan = ((b & 0x7C00) == 0x7C00) & ((b & 0x03FF) != 0)
    is_zero = (b & 0x7FFF) == 0
    norm = np.where(is_nan, np.uint16(0xFFFF), np.where(is_zero, np.uint16(0), b)).astype(np.uint16)
    asc = np.where(norm & 0x8000, ~norm, norm ^ np.uint16(0x8000)).astype(np.uint16)
    return (~asc).astype(np.uint16)


class Oracle:
    def __init__(self, path: str = LIB_PATH):
        lib = C.CDLL(path)
        u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
        u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
        lib.oracle_topk_batch.argtypes = [u16p, C.c_int64, C.c_int64, C.c_int, u16p, i32p, C.c_int, C.c_int]
        lib.oracle_topk_batch.restype = C.c_int
        lib.oracle_topk_csr.argtypes = [u16p, i64p, C.c_int64, C.c_int, u16p, i32p, C.c_int, C.c_int]
        lib.oracle_topk_csr.restype = C.c_int
        lib.oracle_topk_batch_bf16.argtypes = lib.oracle_topk_batch.argtypes
        lib.oracle_topk_batch_bf16.restype = C.c_int
        lib.oracle_topk_csr_bf16.argtypes = lib.oracle_topk_csr.argtypes
        lib.oracle_topk_csr_bf16.restype = C.c_int
        u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
        lib.oracle_topk_batch_f32.argtypes = [u32p, C.c_int64, C.c_int64, C.c_int, u32p, i32p, C.c_int, C.c_int]
        lib.oracle_topk_batch_f32.restype = C.c_int
        lib.oracle_topk_csr_f32.argtypes = [u32p, i64p, C.c_int64, C.c_int, u32p, i32p, C.c_int, C.c_int]
        lib.oracle_topk_csr_f32.restype = C.c_int
        lib.oracle_encode_desc_f32.argtypes = [C.c_uint32]
        lib.oracle_encode_desc_f32.restype = C.c_uint32
        lib.oracle_encode_desc_bf16.argtypes = [C.c_uint16]
        lib.oracle_encode_desc_bf16.restype = C.c_uint16
        lib.oracle_bf16_to_float.argtypes = [C.c_uint16]
        lib.oracle_bf16_to_float.restype = C.c_float
        lib.oracle_encode_desc.argtypes = [C.c_uint16]
        lib.oracle_encode_desc.restype = C.c_uint16
        lib.oracle_half_to_float.argtypes = [C.c_uint16]
        lib.oracle_half_to_float.restype = C.c_float
        lib.oracle_histogram_pass.argtypes = [u16p, C.c_int, C.c_int, C.c_uint16, C.c_uint16, u32p]
        lib.oracle_histogram_pass.restype = None
        lib.oracle_select_state.argtypes = [u16p, C.c_int, C.c_int, i32p]
        lib.oracle_select_state.restype = None
        self.lib = lib

    def topk(self, values_bits: np.ndarray, k: int, method: int = METHOD_COUNT,
             threads: int | None = None, bf16: bool = False):
        """Top-k of each row of a 2-D uint16 array of fp16 (or, with bf16, bfloat16) bits."""
        x = np.ascontiguousarray(values_bits, dtype=np.uint16)
        assert x.ndim == 2
        seg_num, seg_len = x.shape
        ov = np.empty((seg_num, k), np.uint16)
        oi = np.empty((seg_num, k), np.int32)
        fn = self.lib.oracle_topk_batch_bf16 if bf16 else self.lib.oracle_topk_batch
        rc = fn(x.reshape(-1), seg_num, seg_len, k, ov.reshape(-1), oi.reshape(-1), method,
                threads or os.cpu_count() or 1)
        if rc != 0:
            raise ValueError("oracle_topk_batch rejected the arguments")
        return ov, oi

    def topk_csr(self, values_bits: np.ndarray, offsets: np.ndarray, k: int,
                 method: int = METHOD_COUNT, threads: int | None = None, bf16: bool = False):
        x = np.ascontiguousarray(values_bits, dtype=np.uint16).reshape(-1)
        off = np.ascontiguousarray(offsets, dtype=np.int64)
        seg_num = off.shape[0] - 1
        ov = np.empty((seg_num, k), np.uint16)
        oi = np.empty((seg_num, k), np.int32)
        fn = self.lib.oracle_topk_csr_bf16 if bf16 else self.lib.oracle_topk_csr
        rc = fn(x, off, seg_num, k, ov.reshape(-1), oi.reshape(-1), method,
                threads or os.cpu_count() or 1)
        if rc != 0:
            raise ValueError("oracle_topk_csr rejected the arguments")
        return ov, oi

    def topk_f32(self, values_bits: np.ndarray, k: int, method: int = METHOD_COUNT,
                 threads: int | None = None):
        """Top-k of each row of a 2-D array of float32 bit patterns (uint32)."""
        x = np.ascontiguousarray(values_bits).view(np.uint32)
        assert x.ndim == 2
        seg_num, seg_len = x.shape
        ov = np.empty((seg_num, k), np.uint32)
        oi = np.empty((seg_num, k), np.int32)
        rc = self.lib.oracle_topk_batch_f32(x.reshape(-1), seg_num, seg_len, k, ov.reshape(-1),
                                            oi.reshape(-1), method, threads or os.cpu_count() or 1)
        if rc != 0:
            raise ValueError("oracle_topk_batch_f32 rejected the arguments")
        return ov, oi

    def topk_csr_f32(self, values_bits: np.ndarray, offsets: np.ndarray, k: int,
                     method: int = METHOD_COUNT, threads: int | None = None):
        x = np.ascontiguousarray(values_bits).view(np.uint32).reshape(-1)
        off = np.ascontiguousarray(offsets, dtype=np.int64)
        seg_num = off.shape[0] - 1
        ov = np.empty((seg_num, k), np.uint32)
        oi = np.empty((seg_num, k), np.int32)
        rc = self.lib.oracle_topk_csr_f32(x, off, seg_num, k, ov.reshape(-1), oi.reshape(-1),
                                          method, threads or os.cpu_count() or 1)
        if rc != 0:
            raise ValueError("oracle_topk_csr_f32 rejected the arguments")
        return ov, oi

    def histogram_pass(self, values_bits, shift, prefix, prefix_mask):
        x = np.ascontiguousarray(values_bits, dtype=np.uint16).reshape(-1)
        h = np.zeros(256, np.uint32)
        self.lib.oracle_histogram_pass(x, x.size, shift, prefix, prefix_mask, h)
        return h

    def select_state(self, values_bits, k):
        """{prefix, prefix_mask, cutoff_key, selected_count, live_count, boundary_digit,
        strictly_better_count, remaining_slots} as the reference's select kernels compute."""
        x = np.ascontiguousarray(values_bits, dtype=np.uint16).reshape(-1)
        out = np.zeros(8, np.int32)
        self.lib.oracle_select_state(x, x.size, k, out)
        keys = ["prefix", "prefix_mask", "cutoff_key", "selected_count", "live_count",
                "boundary_digit", "strictly_better_count", "remaining_slots"]
        return dict(zip(keys, (int(v) for v in out)))


class RefOracle:
    """The reference's own CPU implementation, built from its sources into oracle/_ref."""

    def __init__(self, path: str = REF_LIB_PATH):
        lib = C.CDLL(path)
        u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        lib.ref_cpu_topk.argtypes = [u16p, C.c_void_p, C.c_int64, C.c_int64, C.c_int, i32p, f32p,
                                     C.c_int, C.POINTER(C.c_double)]
        lib.ref_cpu_topk.restype = C.c_int
        lib.ref_simulate_radix_boundary.argtypes = [u16p, C.c_int, C.c_int, i32p]
        lib.ref_encode_half_desc.argtypes = [C.c_uint16]
        lib.ref_encode_half_desc.restype = C.c_uint16
        lib.ref_candidate_better.argtypes = [C.c_uint16, C.c_int, C.c_uint16, C.c_int]
        lib.ref_candidate_better.restype = C.c_int
        lib.ref_float_to_half_bits.argtypes = [C.c_float]
        lib.ref_float_to_half_bits.restype = C.c_uint16
        lib.ref_make_random_input.argtypes = [C.c_int, C.c_int, C.c_uint32, u16p]
        lib.ref_make_duplicate_heavy_input.argtypes = [C.c_int, C.c_int, u16p]
        lib.ref_make_special_values_input.argtypes = [C.c_int, C.c_int, u16p]
        self.lib = lib

    def topk(self, values_bits, k, offsets=None, threads=1):
        """Returns (indices[seg_num,k] with -1 padding, float values, timed seconds)."""
        x = np.ascontiguousarray(values_bits, dtype=np.uint16)
        if offsets is None:
            seg_num, seg_len = x.shape
            off_ptr = None
            off = None
        else:
            off = np.ascontiguousarray(offsets, dtype=np.int64)
            seg_num, seg_len = off.shape[0] - 1, 0
            off_ptr = off.ctypes.data_as(C.c_void_p)
        oi = np.empty((seg_num, k), np.int32)
        ov = np.empty((seg_num, k), np.float32)
        el = C.c_double(0.0)
        rc = self.lib.ref_cpu_topk(x.reshape(-1), off_ptr, seg_num, seg_len, k, oi.reshape(-1),
                                   ov.reshape(-1), threads, C.byref(el))
        if rc != 0:
            raise ValueError("ref_cpu_topk rejected the arguments")
        return oi, ov, el.value

    def simulate_radix_boundary(self, values_bits, k):
        x = np.ascontiguousarray(values_bits, dtype=np.uint16).reshape(-1)
        out = np.zeros(6, np.int32)
        self.lib.ref_simulate_radix_boundary(x, x.size, k, out)
        keys = ["prefix", "prefix_mask", "cutoff_key", "selected_count", "live_count",
                "boundary_digit"]
        return dict(zip(keys, (int(v) for v in out)))

    def make_random_input(self, seg_num, seg_len, seed):
        out = np.empty(seg_num * seg_len, np.uint16)
        self.lib.ref_make_random_input(seg_num, seg_len, seed, out)
        return out.reshape(seg_num, seg_len)

    def make_duplicate_heavy_input(self, seg_num, seg_len):
        out = np.empty(seg_num * seg_len, np.uint16)
        self.lib.ref_make_duplicate_heavy_input(seg_num, seg_len, out)
        return out.reshape(seg_num, seg_len)

    def make_special_values_input(self, seg_num, seg_len):
        out = np.empty(seg_num * seg_len, np.uint16)
        self.lib.ref_make_special_values_input(seg_num, seg_len, out)
        return out.reshape(seg_num, seg_len)


def load() -> Oracle:
    """Load the C restatement, compiling it first if the shared object is missing."""
    global _oracle
    with _lock:
        if _oracle is None:
            src = os.path.join(HERE, "topk_oracle.c")
            if not os.path.exists(LIB_PATH) or (
                    os.path.exists(src) and os.path.getmtime(src) > os.path.getmtime(LIB_PATH)):
                build(ref=False)
            _oracle = Oracle()
        return _oracle


class RefGpu:
    """The reference's own GPU path (its src/batch_topk.cu for sm_100a), built into
    oracle/_ref/libref_gpu.so: radix_topk::batch_topk_half behind a C ABI, for timing it next
    to this library on the reference's own supported shapes."""

    def __init__(self, path: str = REF_GPU_LIB_PATH):
        lib = C.CDLL(path)
        vp, i32 = C.c_void_p, C.c_int
        lib.ref_gpu_topk_half.argtypes = [vp, i32, i32, i32, vp, vp, vp, C.c_size_t, vp]
        lib.ref_gpu_topk_half.restype = i32
        lib.ref_gpu_workspace_size.argtypes = [i32, i32, i32]
        lib.ref_gpu_workspace_size.restype = C.c_size_t
        self.lib = lib

    def workspace_size(self, seg_num: int, seg_len: int, k: int) -> int:
        return int(self.lib.ref_gpu_workspace_size(seg_num, seg_len, k))

    def topk_half(self, d_in, seg_num, seg_len, k, d_vals, d_idx, d_ws, ws_bytes, stream=0) -> int:
        return int(self.lib.ref_gpu_topk_half(d_in, seg_num, seg_len, k, d_vals, d_idx, d_ws,
                                              ws_bytes, stream))


def load_ref_gpu() -> RefGpu | None:
    """Load the reference's GPU path if it was built here (None otherwise)."""
    if not os.path.exists(REF_GPU_LIB_PATH):
        return None
    return RefGpu()


def load_ref() -> RefOracle | None:
    """Load the reference's own CPU top-k if it was built here (None otherwise)."""
    global _ref
    with _lock:
        if _ref is None and os.path.exists(REF_LIB_PATH):
            _ref = RefOracle()
        return _ref
