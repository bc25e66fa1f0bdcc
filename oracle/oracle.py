"""ctypes wrapper around the C oracle (`oracle/sampler_oracle.c`).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker / timed CPU arm, never by the
product package.  Parity with the reference's own sampler is UNPINNED (the
reference's sampler package `mstar.utils.sampling` is absent; see the C
file's header for the spec and the call sites it follows).

A batch is described by a plain dict of numpy arrays (`SamplerCase`), the
same layout the CUDA path takes through its C ABI.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
SRC = os.path.join(HERE, "sampler_oracle.c")


def build(force: bool = False) -> str:
    os.makedirs(os.path.dirname(LIB_PATH), exist_ok=True)
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(SRC):
        subprocess.check_call(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=c11",
                               "-o", LIB_PATH, SRC, "-lm"])
    return LIB_PATH


P = ctypes.c_void_p


class OrcArgs(ctypes.Structure):
    _fields_ = [
        ("logits", P), ("dtype", ctypes.c_int), ("ld", ctypes.c_int64),
        ("B", ctypes.c_int32), ("V", ctypes.c_int32), ("vocab_offset", ctypes.c_int64),
        ("slot_idx", P),
        ("temperature", P), ("top_p", P), ("min_p", P), ("rep_pen", P), ("pres_pen", P),
        ("freq_pen", P), ("top_k", P),
        ("hist_ids", P), ("hist_len", P), ("H", ctypes.c_int32),
        ("seen_bits", P), ("seen_words", ctypes.c_int64),
        ("bias_ids", P), ("bias_vals", P), ("NB", ctypes.c_int32),
        ("allowed_bits", P), ("allowed_words", ctypes.c_int64),
        ("uniforms", P), ("seed", P), ("offset", P),
        ("out_ids", P), ("out_status", P), ("out_probs", P), ("out_kept", P), ("out_x", P),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = LIB_PATH if os.path.exists(LIB_PATH) else build()
        _lib = ctypes.CDLL(path)
        _lib.orc_sample.argtypes = [ctypes.POINTER(OrcArgs), ctypes.c_int]
        _lib.orc_sample.restype = ctypes.c_int
        _lib.orc_args_size.restype = ctypes.c_int
        _lib.orc_exp_spec.argtypes = [ctypes.c_float]
        _lib.orc_exp_spec.restype = ctypes.c_float
        _lib.orc_philox_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        _lib.orc_philox_uniform.restype = ctypes.c_float
        assert _lib.orc_args_size() == ctypes.sizeof(OrcArgs), "oracle struct layout mismatch"
    return _lib


@dataclass
class SamplerCase:
    """One batch: logits [B, V] (f32 ndarray, or uint16 bf16 bit patterns with
    dtype='bf16') plus per-slot parameter arrays.  Optional arrays are None."""
    logits: np.ndarray
    dtype: str = "f32"
    slot_idx: np.ndarray | None = None
    temperature: np.ndarray | None = None
    top_k: np.ndarray | None = None
    top_p: np.ndarray | None = None
    min_p: np.ndarray | None = None
    rep_pen: np.ndarray | None = None
    pres_pen: np.ndarray | None = None
    freq_pen: np.ndarray | None = None
    hist_ids: np.ndarray | None = None      # [slots, H] int32 (global ids)
    hist_len: np.ndarray | None = None      # [slots] int32
    seen_bits: np.ndarray | None = None     # [slots, words] uint32
    bias_ids: np.ndarray | None = None      # [slots, NB] int32 (-1 = unused)
    bias_vals: np.ndarray | None = None     # [slots, NB] f32
    allowed_bits: np.ndarray | None = None  # [slots, words] uint32
    uniforms: np.ndarray | None = None      # [B] f32
    seed: np.ndarray | None = None          # [slots] uint64
    offset: np.ndarray | None = None        # [slots] uint64
    vocab_offset: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def B(self) -> int:
        return int(self.logits.shape[0])

    @property
    def V(self) -> int:
        return int(self.logits.shape[1])

    def logits_f32(self) -> np.ndarray:
        if self.dtype == "bf16":
            return (self.logits.astype(np.uint32) << 16).view(np.float32)
        return self.logits


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def run(case: SamplerCase, debug: bool = False, threads: int | None = None):
    """Run the C oracle; returns dict(ids, status[, probs, kept, x])."""
    L = lib()
    B, V = case.B, case.V
    c = lambda a, dt: None if a is None else np.ascontiguousarray(a, dtype=dt)  # noqa: E731
    arrs = dict(
        logits=np.ascontiguousarray(case.logits),
        slot_idx=c(case.slot_idx, np.int32), temperature=c(case.temperature, np.float32),
        top_p=c(case.top_p, np.float32), min_p=c(case.min_p, np.float32),
        rep_pen=c(case.rep_pen, np.float32), pres_pen=c(case.pres_pen, np.float32),
        freq_pen=c(case.freq_pen, np.float32), top_k=c(case.top_k, np.int32),
        hist_ids=c(case.hist_ids, np.int32), hist_len=c(case.hist_len, np.int32),
        seen_bits=c(case.seen_bits, np.uint32), bias_ids=c(case.bias_ids, np.int32),
        bias_vals=c(case.bias_vals, np.float32), allowed_bits=c(case.allowed_bits, np.uint32),
        uniforms=c(case.uniforms, np.float32), seed=c(case.seed, np.uint64),
        offset=c(case.offset, np.uint64))
    out = dict(ids=np.zeros(B, np.int64), status=np.zeros(B, np.int32))
    if debug:
        out.update(probs=np.zeros((B, V), np.float32), kept=np.zeros((B, V), np.uint8),
                   x=np.zeros((B, V), np.float32))
    a = OrcArgs()
    a.logits = _ptr(arrs["logits"])
    a.dtype = 1 if case.dtype == "bf16" else 0
    a.ld = arrs["logits"].shape[1]
    a.B, a.V, a.vocab_offset = B, V, case.vocab_offset
    for k in ("slot_idx", "temperature", "top_p", "min_p", "rep_pen", "pres_pen", "freq_pen",
              "top_k", "hist_ids", "hist_len", "seen_bits", "bias_ids", "bias_vals",
              "allowed_bits", "uniforms", "seed", "offset"):
        setattr(a, k, _ptr(arrs[k]))
    a.H = 0 if arrs["hist_ids"] is None else arrs["hist_ids"].shape[1]
    a.seen_words = 0 if arrs["seen_bits"] is None else arrs["seen_bits"].shape[1]
    a.NB = 0 if arrs["bias_ids"] is None else arrs["bias_ids"].shape[1]
    a.allowed_words = 0 if arrs["allowed_bits"] is None else arrs["allowed_bits"].shape[1]
    if arrs["uniforms"] is None and (arrs["seed"] is None or arrs["offset"] is None):
        raise ValueError("need uniforms or seed+offset")
    a.out_ids = _ptr(out["ids"])
    a.out_status = _ptr(out["status"])
    if debug:
        a.out_probs, a.out_kept, a.out_x = _ptr(out["probs"]), _ptr(out["kept"]), _ptr(out["x"])
    nt = threads if threads is not None else (os.cpu_count() or 1)
    L.orc_sample(ctypes.byref(a), nt)
    if debug:
        out["kept"] = out["kept"].astype(bool)
    return out


def run_np(case: SamplerCase):
    """Same batch through the numpy restatement (small cases only)."""
    from . import spec_np  # noqa: WPS433
    B, V = case.B, case.V
    lf = case.logits_f32()
    res = dict(ids=np.zeros(B, np.int64), status=np.zeros(B, np.int32),
               probs=np.zeros((B, V), np.float32), kept=np.zeros((B, V), bool),
               x=np.zeros((B, V), np.float32))
    g = lambda a, s, d: d if a is None else a[s]  # noqa: E731
    for r in range(B):
        s = int(case.slot_idx[r]) if case.slot_idx is not None else r
        if s < 0:
            res["ids"][r] = case.vocab_offset
            res["x"][r] = -np.inf
            continue
        hist = None
        if case.hist_ids is not None:
            n = min(int(case.hist_len[s]), case.hist_ids.shape[1])
            hist = case.hist_ids[s, :n]
        tok, st, x, kept, probs = spec_np.sample_row(
            lf[r], temperature=g(case.temperature, s, 1.0), top_k=int(g(case.top_k, s, 0)),
            top_p=g(case.top_p, s, 1.0), min_p=g(case.min_p, s, 0.0), rep=g(case.rep_pen, s, 1.0),
            pres=g(case.pres_pen, s, 0.0), freq=g(case.freq_pen, s, 0.0), hist=hist,
            seen_words=None if case.seen_bits is None else case.seen_bits[s],
            bias_ids=None if case.bias_ids is None else case.bias_ids[s],
            bias_vals=None if case.bias_vals is None else case.bias_vals[s],
            allowed_words=None if case.allowed_bits is None else case.allowed_bits[s],
            u=None if case.uniforms is None else case.uniforms[r],
            seed=int(g(case.seed, s, 0)), offset=int(g(case.offset, s, 0)),
            vocab_offset=case.vocab_offset)
        res["ids"][r], res["status"][r] = tok, st
        res["x"][r], res["kept"][r], res["probs"][r] = x, kept, probs
    return res


def stop_hits(ids, stop_ids) -> np.ndarray:
    """Rows whose sampled id is one of their stop ids (entries < 0 unused).

    Restates the engines' host-side stop test after a step,
    `int(tok.item()) == self.cfg.stop_token_id` (python/mstar_rs/models/
    orpheus.py:428-432, :518-519), widened to a short list of stop ids per
    request; `ignore_eos` requests carry none.  ids [n], stop_ids [n, NS]."""
    ids = np.asarray(ids, np.int64).reshape(-1, 1)
    st = np.asarray(stop_ids, np.int64)
    return ((st >= 0) & (st == ids)).any(axis=1)
