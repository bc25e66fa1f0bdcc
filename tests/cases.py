"""Seeded small sampling cases covering every knob and edge case of the spec.

Shared by the CPU oracle tests and the GPU parity tests."""
from __future__ import annotations

import numpy as np

from mstar_rs_b200.workloads import Batch, f32_to_bf16_bits, pack_bits


def random_case(seed: int, B: int = 8, V: int = 1000, dtype: str = "f32", *, penalty: str = "hist",
                bias: bool = True, mask: bool = True, ties: bool = False, greedy_frac: float = 0.15,
                specials: bool = True, philox: bool = False, pad_rows: bool = False,
                vocab_offset: int = 0, scale: float = 2.0, V_global: int | None = None,
                seen_density: float = 0.02) -> Batch:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, V)).astype(np.float32) * np.float32(scale)
    if ties:  # quantise hard so many exact ties exist
        x = np.round(x * 2.0).astype(np.float32) / np.float32(2.0)
    if specials:
        for r in range(B):
            k = rng.integers(0, 4)
            idx = rng.integers(0, V, k)
            choice = rng.integers(0, 4, k)
            for i, c in zip(idx, choice):
                x[r, i] = [np.nan, np.inf, -np.inf, 0.0][c] if c != 3 else -0.0
            if rng.random() < 0.05:
                x[r, :] = -np.inf  # all -inf row
    Vg = V_global if V_global is not None else vocab_offset + V
    logits = f32_to_bf16_bits(x) if dtype == "bf16" else x
    T = rng.uniform(0.2, 2.0, B).astype(np.float32)
    T[rng.random(B) < greedy_frac] = 0.0
    top_k = rng.choice(np.array([0, 0, 1, 2, 5, 20, 100, V + 5], np.int32), B)
    top_p = rng.choice(np.array([1.0, 0.9, 0.5, 0.0, 0.99], np.float32), B)
    min_p = rng.choice(np.array([0.0, 0.0, 0.05, 0.3, 1.5], np.float32), B)
    b = Batch(logits=logits, dtype=dtype, temperature=T, top_k=top_k, top_p=top_p, min_p=min_p,
              rep_pen=rng.uniform(0.7, 1.5, B).astype(np.float32),
              pres_pen=rng.uniform(-1.0, 1.0, B).astype(np.float32),
              freq_pen=rng.uniform(-0.5, 1.0, B).astype(np.float32),
              vocab_offset=vocab_offset, name=f"rand{seed}")
    if penalty == "hist":
        H = 64
        b.hist_ids = rng.integers(-2, Vg, (B, H)).astype(np.int32)
        b.hist_len = rng.integers(0, 2 * H, B).astype(np.int32)
    elif penalty == "seen":
        seen = rng.random((B, Vg)) < seen_density
        b.seen_bits = pack_bits(seen)
    if bias:
        NB = 6
        ids = rng.integers(-1, Vg, (B, NB)).astype(np.int32)
        ids[:, 1] = ids[:, 0]  # duplicate ids apply in list order
        b.bias_ids = ids
        b.bias_vals = rng.uniform(-5, 5, (B, NB)).astype(np.float32)
    if mask:
        allowed = rng.random((B, Vg)) < rng.uniform(0.05, 1.0, (B, 1))
        allowed[rng.random(B) < 0.05] = False  # some rows allow nothing
        b.allowed_bits = pack_bits(allowed)
    if philox:
        b.seed = rng.integers(0, 2**63, B, dtype=np.uint64)
        b.offset = rng.integers(0, 2**40, B, dtype=np.uint64)
    else:
        u = rng.random(B).astype(np.float32)
        u[0] = 0.0
        b.uniforms = u
    if pad_rows:
        slots = np.arange(B, dtype=np.int32)
        rng.shuffle(slots)
        slots[rng.random(B) < 0.2] = -1
        b.slot_idx = slots
    return b


def feature_grid():
    """(seed, kwargs) pairs the parity suites iterate over."""
    out = []
    s = 0
    for dtype in ("f32", "bf16"):
        for penalty in ("hist", "seen", None):
            for ties in (False, True):
                out.append((s, dict(dtype=dtype, penalty=penalty, ties=ties)))
                s += 1
    out.append((s, dict(V=37, B=5))); s += 1
    out.append((s, dict(V=1, B=3, bias=False, mask=False))); s += 1
    out.append((s, dict(V=5000, B=4, philox=True))); s += 1
    out.append((s, dict(V=3001, B=6, pad_rows=True))); s += 1
    out.append((s, dict(V=777, B=4, vocab_offset=1000, V_global=4000))); s += 1
    out.append((s, dict(V=20000, B=3, scale=0.05))); s += 1
    return out
