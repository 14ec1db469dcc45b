"""Parity checker for batch_topk_b200 -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline and
``--impl reference`` legs) may import this package.  The product library never does.

* ``topk_oracle.c``   -- C restatement of the reference's CPU top-k and select state.
* ``ref_oracle.cpp``  -- C ABI over the reference's own header-only CPU implementation,
                         built in place from the reference tree into ``oracle/_ref``.
* ``ref_gpu.cu``      -- C ABI over the reference's own GPU path (its src/batch_topk.cu),
                         built in place for sm_100a into ``oracle/_ref``, for a same-box
                         timing comparison on the reference's supported shapes.
"""
from .oracle import (  # noqa: F401
    METHOD_COUNT,
    METHOD_SORT,
    Oracle,
    RefGpu,
    RefOracle,
    build,
    encode_desc,
    load,
    load_ref,
    load_ref_gpu,
    reference_dir,
)
