"""ctypes binding of libce_b200.so (declarations in include/ce_api.h).

This is the drop-in boundary: plain pointers, sizes and a cudaStream_t, no
torch types.  Loading fails loudly when the library has not been built; there
is no fallback implementation behind it.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

from . import build as _build

LIB_PATH = _build.LIB

CE_OK = 0
CE_ERR_ARG = -1
CE_ERR_UNSUPPORTED = -2
CE_ERR_CUDA = -3
CE_ERR_WORKSPACE = -4

CE_EW_INDEX = 0x01
CE_EW_CAPACITY = 0x02
CE_EW_TIMEOUT = 0x04
CE_EW_MODE = 0x08
CE_EW_PROTECTED = 0x10
CE_EW_SWA = 0x20
CE_EW_PACK = 0x40
CE_EW_SHAPE = 0x80

CE_POLICY_PREFIX_SLIDING = 0
CE_POLICY_RANDOM = 1
CE_POLICY_RESERVOIR = 2
CE_POLICY_HEAD_SUM = 3
CE_POLICY_HEAD_MAX = 4
CE_POLICY_H2O_GLOBAL = 5

CE_MODE_NONE, CE_MODE_SUM, CE_MODE_MAX = 0, 1, 2
CE_SCORE_DEFER = 4   # score_flags bit: leave the page scores to ce_decode_scores
CE_DTYPE_NONE, CE_DTYPE_F32, CE_DTYPE_F64, CE_DTYPE_BF16 = 0, 1, 2, 3

# size of the static scratch behind ce_decode_attn_score_static
CE_DECODE_STATIC_SCRATCH_BYTES = 32 << 20


class RowParams(C.Structure):
    """ce_row_params: one boundary's sizes in units (32 bytes)."""
    _fields_ = [("n", C.c_int32), ("budget", C.c_int32), ("prefix", C.c_int32),
                ("recent", C.c_int32), ("cursor", C.c_int32), ("policy", C.c_int32),
                ("seed", C.c_uint64)]


assert C.sizeof(RowParams) == 32

P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
F32 = C.c_float
U64 = C.c_uint64

SIGNATURES = {
    "ce_version": (C.c_char_p, []),
    "ce_status_string": (C.c_char_p, [C.c_int]),
    "ce_last_error": (C.c_char_p, []),
    "ce_prepare_device": (C.c_int, []),
    "ce_fill": (C.c_int, [P, I64, P, I64, P, P, P, P, I32, I32, P, P, I32, I64, P, P, P]),
    "ce_pool_alloc": (C.c_int, [P, P, P, I64, I64, P, P, I32, I32, P, P]),
    "ce_pool_push": (C.c_int, [P, P, I64, P, I64, P, I64, I32, P, P]),
    "ce_moe_gate_up": (C.c_int, [P, P, P, I32, I32, I32, I32, P, P, P]),
    "ce_moe_down": (C.c_int, [P, P, P, P, I32, I32, I32, I32, P, P, P]),
    "ce_decode_workspace_bytes": (I64, [I32, I64, I32, I32, I32, I32]),
    "ce_decode_attn_score": (C.c_int, [P, I64, I64, P, P, I64, P, P, P, I64, P, P, P, F32, I32,
                                       I32, I32, I32, I32, P, I64, I32, P, I32, I64, I64, P,
                                       I32, P, I64, P, P]),
    "ce_decode_scores": (C.c_int, [P, P, P, I64, I64, P, P, I32, I32, I32, I32, P, I64, I32, I32, P,
                                   I64, P, P]),
    "ce_decode_attn_score_static": (C.c_int, [P, I64, I64, P, P, I64, P, P, P, I64, P, P, P, F32,
                                              I32, I32, I32, I32, I32, P, I64, I32, P, I32, I64,
                                              I64, P, I32, P, P]),
    "ce_prefill_workspace_bytes": (I64, [I32, I32]),
    "ce_prefill_scores": (C.c_int, [P, I64, I64, P, I64, P, P, P, P, I64, P, P, P, F32, I32, I32,
                                    I32, I32, I32, I32, I32, I32, P, I64, I32, P, I64, P, P]),
    "ce_prefill_lost": (C.c_int, [P, I64, I64, P, I64, P, P, P, P, I64, P, F32, I32, I32, I32, I32,
                                  I32, I32, I32, P, I32, I64, P, I64, F32, P, I64, P, P]),
    "ce_replay_workspace_bytes": (I64, [I32, I32]),
    "ce_replay_error": (C.c_int, [P, I64, I64, P, P, I64, P, I64, P, F32, I32, I32, I32, I32, I32, P, P,
                                  P, I64, P, P]),
    "ce_selftest_wait": (C.c_int, [I32, I64, P, P, P]),
    "ce_choose_workspace_bytes": (I64, [I32, I32, I32]),
    "ce_choose": (C.c_int, [P, P, I32, P, I32, P, I32, I32, I32, I32, I32, P, I32, P, P, P,
                            I64, P, P]),
    "ce_boundary_workspace_bytes": (I64, [I32, I32, I32, I32, I32, I32, I32, I32, I64]),
    "ce_boundary": (C.c_int, [P, I64, I32, P, I64, I32, P, P, P, I64, I32, P, I64, I64, I64,
                              P, P, I32, I32, I32, I32, I32, P, I32, P, P, P, I32, P, I32, P,
                              I32, I32, I32, I32, I32, P, P, I64, P, I64, I64, P, I64, P, P, P]),
    "ce_gather_row_scores": (C.c_int, [P, I64, P, I64, P, P, P, I64, I64, I64, I32, I32, P,
                                       P, I32, I32, P, P, P]),
    "ce_reservoir_scores": (C.c_int, [P, I32, I32, I32, I32, U64, P, P]),
}

_lib = None
_lock = threading.Lock()


class CeError(RuntimeError):
    """A libce_b200 entry point returned a non-zero status."""


def load() -> C.CDLL:
    """Load the in-tree library; raise if it was never built."""
    global _lib
    with _lock:
        if _lib is None:
            if not Path(LIB_PATH).exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m cache_eviction_b200.build` "
                    "(there is no non-CUDA fallback)")
            lib = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != CE_OK:
        lib = load()
        raise CeError(f"{what}: {lib.ce_status_string(status).decode()} "
                      f"({lib.ce_last_error().decode()})")


def exported_symbols() -> list[str]:
    return sorted(SIGNATURES)
