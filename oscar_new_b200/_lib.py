"""ctypes binding of ``liboscar_b200.so`` (C ABI in ``include/oscar_b200.h``).

There is no fallback: if the library is missing or fails to load, every operator
raises.  The library is built in-tree by ``oscar_new_b200.build``.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

_PATH = Path(__file__).resolve().parent / "liboscar_b200.so"
_lib = None

STATUS = {0: "ok", 1: "invalid argument", 2: "launch error", 3: "unsupported", 4: "device wait timeout"}
UNSUPPORTED = 3  # OSCAR_ERR_UNSUPPORTED: the caller may take another path


class Geometry(C.Structure):
    _fields_ = [
        ("kv_heads", C.c_int32),
        ("group", C.c_int32),
        ("head_dim", C.c_int32),
        ("block_tokens", C.c_int32),
        ("kernel_block", C.c_int32),
        ("slot_bytes", C.c_int32),
        ("vector_bytes", C.c_int32),
        ("sink", C.c_int32),
        ("recent", C.c_int32),
        ("ring", C.c_int32),
        ("table_stride", C.c_int32),
        ("query_tile", C.c_int32),
        ("page_bytes", C.c_int64),
    ]


class Clip(C.Structure):
    _fields_ = [
        ("enabled", C.c_int32),
        ("mode", C.c_int32),
        ("asc_lo", C.c_int32),
        ("asc_hi", C.c_int32),
        ("weight", C.c_float),
        ("factor", C.c_float),
    ]


P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
F32 = C.c_float

_SIGNATURES = {
    "oscar_version": [],
    "oscar_selftest_bounded_wait": [P, P],
    "oscar_test_set_wait_fault": [I32, C.c_uint32],
    "oscar_last_history_kernel": [],
    "oscar_prefill_attention": [P, I64, I64, P, I64, I64, P, I64, I64, P, I32, I32, I64, I32, I32, F32, P, I64, I64, P,
                                P],
    "oscar_rotate": [P, I64, I32, I64, I64, I64, P, I64, I64, P, P],
    "oscar_store_int2": [P, P, I64, P, P, P, Geometry, Clip, Clip, P],
    "oscar_rotate_store": [P, I64, I64, P, I64, I64, I64, P, P, P, P, P, Geometry, Clip, Clip, P, I64, I64, I32, P, P, P, P, P],
    "oscar_prepare_tasks": [P, P, P, P, I32, I32, I32, P, I64, P, I64, I32, P],
    "oscar_step_arena_layout": [I32, I32, I32, P],
    "oscar_stage_step_metadata": [P, P, P, I64, P, I32, I32, I32, I32, P, I32, I32, I32, P, I64, P],
    "oscar_attention_partials": [P, I64, I64, P, I64, I64, P, I64, I64, P, P, P, P, P, P, P, P, I32, I64, P, P, Geometry, F32, I32, I32, P, P],
    "oscar_merge_splits": [P, P, I64, I32, I32, P, P, P, P],
    "oscar_merge_paths": [P, P, P, I64, P, I64, I64, I32, P, P, P],
    "oscar_store_windows": [P, I64, I64, P, I64, I64, P, P, P, P, P, I32, Geometry, P],
    "oscar_unpack": [P, P, I64, Geometry, P, P, P],
    "oscar_decode_attention": [P, P, I64, I64, P, I64, I64, P, I64, I64, P, P, P, P, P, P, P, P, I32, I64, P, P, P, P, Geometry, F32, I32, I32, P, P],
    "oscar_accumulate_gram": [P, I64, I32, I64, I64, P, P, P],
    "oscar_sst_weights": [P, I64, I32, I64, I64, P, P, P, P],
    "oscar_accumulate_gram_grouped": [P, I64, I32, I64, I64, I32, P, P, P],
    "oscar_sst_weights_per_head": [P, I64, I32, I64, I64, P, P, P, P],
    "oscar_split_bf16x3": [P, I32, P, P],
    "oscar_sst_weights_split": [P, I64, I32, I64, I64, P, P, P, P, P],
    "oscar_normalize": [P, I64, P, F32, P, P],
    "oscar_jacobi_rotations": [P, I32, I32, F32, P, P, P, P],
    "oscar_decode_attention_noalloc": [P, P, I64, I64, P, I64, I64, P, I64, I64, P, P, P, P, P, P, P, P, I32, I64, P, P, Geometry, F32, I32, I32, P, P],
    "oscar_decode_attention_noalloc_max_rows": [],
}
_RESTYPES = {"oscar_decode_attention_noalloc_max_rows": C.c_int64}


def lib():
    """Load (once) and return the CUDA library; raise if it is absent."""
    global _lib
    if _lib is None:
        if not _PATH.exists():
            raise RuntimeError(
                f"OSCAR CUDA library not built ({_PATH}); run `python -m oscar_new_b200.build`"
            )
        handle = C.CDLL(str(_PATH))
        for name, args in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, C.c_int)
        _lib = handle
    return _lib


def exported_symbols():
    return list(_SIGNATURES)


def check(status: int, name: str):
    if status != 0:
        raise RuntimeError(f"{name} failed: {STATUS.get(status, status)}")


def call(name: str, *args):
    check(getattr(lib(), name)(*args), name)
