"""ctypes binding of the sampler's C ABI (include/mstar_sampler.h).

The library is built in-tree (`python -m mstar_rs_b200.build`).  There is no
CPU fallback: if the library is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "_lib", "libmstar_sampler.so")

ABI_VERSION = 2
DTYPE_F32, DTYPE_BF16 = 0, 1
FLAG_UPDATE_HISTORY = 0x1
FLAG_UPDATE_SEEN = 0x2
FLAG_ADVANCE_OFFSET = 0x4
FLAG_FORCE_GENERAL = 0x8
FLAG_TEST_WITHHOLD = 0x10
STATUS_EMPTY = 0x1
STATUS_GENERAL = 0x2
STATUS_SPECIAL_OVERFLOW = 0x4
STATUS_TP_OVERFLOW = 0x8
STATUS_TIMEOUT = 0x10
STATUS_STOP = 0x20
STATUS_BAD_RECORD = 0x40
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3

P = ctypes.c_void_p
I32, I64, U32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32


class Params(ctypes.Structure):
    """Mirror of `mstar_sampler_params_t` (same field order and types)."""

    _fields_ = [
        ("logits", P), ("dtype", I32), ("B", I32), ("V", I32), ("num_slots", I32),
        ("ld", I64), ("vocab_offset", I64), ("slot_idx", P),
        ("temperature", P), ("top_k", P), ("top_p", P), ("min_p", P),
        ("rep_pen", P), ("pres_pen", P), ("freq_pen", P),
        ("hist_ids", P), ("hist_len", P), ("H", I32), ("seen_cap", I32),
        ("seen_bits", P), ("seen_words", I64),
        ("bias_ids", P), ("bias_vals", P), ("NB", I32), ("pad0", I32),
        ("allowed_bits", P), ("allowed_words", I64),
        ("uniforms", P), ("seed", P), ("offset", P),
        ("out_ids", P), ("out_ids32", P), ("out_status", P),
        ("out_x", P), ("out_kept", P), ("out_probs", P),
        ("flags", U32), ("cluster_size", I32),
        ("stop_ids", P), ("NS", I32), ("pad1", I32), ("stop_flags", P),
    ]


class SamplerError(RuntimeError):
    pass


_lib = None
_lock = threading.Lock()

EXPORTS = (
    "mstar_sampler_abi_version", "mstar_sampler_last_error", "mstar_sampler_plan",
    "mstar_sampler_step", "mstar_sampler_tp_record_words", "mstar_sampler_tp_local",
    "mstar_sampler_tp_merge", "mstar_sampler_philox_uniform", "mstar_sampler_commit",
    "mstar_lmhead_workspace_bytes", "mstar_lmhead_logits", "mstar_sampler_lmhead_step",
    "mstar_lmhead_logits_static", "mstar_sampler_tp_local2", "mstar_sampler_tp_merge1", "mstar_sampler_tp_mass",
    "mstar_sampler_tp_merge2",
)


def lib() -> ctypes.CDLL:
    """Load the in-tree CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise SamplerError(
                f"CUDA sampler library missing at {LIB_PATH}; build it with "
                "`python -m mstar_rs_b200.build` (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        L.mstar_sampler_abi_version.restype = ctypes.c_int
        L.mstar_sampler_last_error.restype = ctypes.c_char_p
        L.mstar_sampler_plan.argtypes = [ctypes.POINTER(Params), ctypes.POINTER(I32), ctypes.POINTER(I64)]
        L.mstar_sampler_plan.restype = ctypes.c_int
        L.mstar_sampler_step.argtypes = [ctypes.POINTER(Params), P]
        L.mstar_sampler_step.restype = ctypes.c_int
        L.mstar_sampler_tp_record_words.argtypes = [I32]
        L.mstar_sampler_tp_record_words.restype = I32
        L.mstar_sampler_tp_local.argtypes = [ctypes.POINTER(Params), I32, P, P]
        L.mstar_sampler_tp_local.restype = ctypes.c_int
        L.mstar_sampler_tp_merge.argtypes = [ctypes.POINTER(Params), I32, I32, I64, P, P]
        L.mstar_sampler_tp_merge.restype = ctypes.c_int
        L.mstar_sampler_commit.argtypes = [ctypes.POINTER(Params), P, P]
        L.mstar_sampler_commit.restype = ctypes.c_int
        L.mstar_sampler_tp_local2.argtypes = [ctypes.POINTER(Params), I32, P, P, P]
        L.mstar_sampler_tp_local2.restype = ctypes.c_int
        L.mstar_sampler_tp_merge1.argtypes = [ctypes.POINTER(Params), I32, I32, I64, P, P, P]
        L.mstar_sampler_tp_merge1.restype = ctypes.c_int
        L.mstar_sampler_tp_mass.argtypes = [ctypes.POINTER(Params), P, P, P, P]
        L.mstar_sampler_tp_mass.restype = ctypes.c_int
        L.mstar_sampler_tp_merge2.argtypes = [ctypes.POINTER(Params), I32, I32, I64, P, P, P, P]
        L.mstar_sampler_tp_merge2.restype = ctypes.c_int
        L.mstar_lmhead_workspace_bytes.argtypes = [I32]
        L.mstar_lmhead_workspace_bytes.restype = I64
        L.mstar_lmhead_logits.argtypes = [P, P, I32, I32, I32, P, I32, I64, P, I64, P, P]
        L.mstar_lmhead_logits.restype = ctypes.c_int
        L.mstar_sampler_lmhead_step.argtypes = [ctypes.POINTER(Params), P, P, I32, P, I64, P, P]
        L.mstar_sampler_lmhead_step.restype = ctypes.c_int
        L.mstar_lmhead_logits_static.argtypes = [P, P, I32, I32, I32, P, I32, I64, P, P]
        L.mstar_lmhead_logits_static.restype = ctypes.c_int
        L.mstar_sampler_philox_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.mstar_sampler_philox_uniform.restype = ctypes.c_float
        if L.mstar_sampler_abi_version() != ABI_VERSION:
            raise SamplerError("sampler library ABI version mismatch; rebuild it")
        _lib = L
        return L


def check(rc: int, what: str) -> None:
    if rc != OK:
        msg = lib().mstar_sampler_last_error().decode(errors="replace")
        raise SamplerError(f"{what} failed (code {rc}): {msg}")


def philox_uniform(seed: int, offset: int) -> float:
    return float(lib().mstar_sampler_philox_uniform(seed, offset))
