"""Seeded synthetic sampling workloads.

The reference publishes no sampler benchmark suite; these generators produce
inputs with the shapes, dtypes and value distributions of the five workloads
the sampler is measured on (Orpheus single-request, Qwen3 mixed continuous
batch, large-batch bucket sweep, vocab-sharded TP, constrained/biased
decoding).  A `Batch` is a plain bundle of numpy arrays in the layout of the
C ABI; `to_device` turns it into the tensors `kernel.sampler_step` takes.
"""
from __future__ import annotations

from dataclasses import dataclass, field, fields

import numpy as np


@dataclass
class Batch:
    logits: np.ndarray                      # [B, V] float32, or uint16 bf16 bit patterns
    dtype: str = "f32"                      # "f32" | "bf16"
    slot_idx: np.ndarray | None = None      # [B] int32
    temperature: np.ndarray | None = None   # [slots] f32
    top_k: np.ndarray | None = None         # [slots] i32
    top_p: np.ndarray | None = None
    min_p: np.ndarray | None = None
    rep_pen: np.ndarray | None = None
    pres_pen: np.ndarray | None = None
    freq_pen: np.ndarray | None = None
    hist_ids: np.ndarray | None = None      # [slots, H] i32 global ids
    hist_len: np.ndarray | None = None      # [slots] i32
    seen_bits: np.ndarray | None = None     # [slots, words] u32
    bias_ids: np.ndarray | None = None      # [slots, NB] i32 (-1 unused)
    bias_vals: np.ndarray | None = None     # [slots, NB] f32
    allowed_bits: np.ndarray | None = None  # [slots, words] u32
    uniforms: np.ndarray | None = None      # [B] f32
    seed: np.ndarray | None = None          # [slots] u64
    offset: np.ndarray | None = None        # [slots] u64
    vocab_offset: int = 0
    name: str = ""
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

    def row_slice(self, r0: int, r1: int) -> "Batch":
        """Rows [r0, r1) with their own slots (data-parallel shard)."""
        out = {}
        for f in fields(self):
            v = getattr(self, f.name)
            out[f.name] = v
        b = Batch(**out)
        b.logits = self.logits[r0:r1]
        if self.uniforms is not None:
            b.uniforms = self.uniforms[r0:r1]
        if self.slot_idx is not None:
            b.slot_idx = self.slot_idx[r0:r1]
        else:
            b.slot_idx = np.arange(r0, r1, dtype=np.int32)
        return b


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    nan = np.isnan(x)
    r = np.where(nan, np.uint32(0x7FC0), r)
    return r.astype(np.uint16)


def pack_bits(mask: np.ndarray) -> np.ndarray:
    """bool [rows, V] -> uint32 words [rows, ceil(V/32)], bit g&31 of word g>>5."""
    rows, V = mask.shape
    W = (V + 31) // 32
    padded = np.zeros((rows, W * 32), dtype=bool)
    padded[:, :V] = mask
    b = padded.reshape(rows, W, 32).astype(np.uint64)
    words = (b << np.arange(32, dtype=np.uint64)).sum(axis=2)
    return words.astype(np.uint32)


def zipf_ids(rng, V: int, n: tuple, a: float = 1.1, perm_seed: int = 1234) -> np.ndarray:
    """Ids drawn from a Zipf(a) law over ranks 1..V, ranks scattered over the
    vocabulary by a fixed permutation."""
    k = np.arange(1, V + 1, dtype=np.float64)
    cdf = np.cumsum(k ** -a)
    cdf /= cdf[-1]
    ranks = np.searchsorted(cdf, rng.random(n), side="right")
    perm = np.random.default_rng(perm_seed).permutation(V)
    return perm[np.minimum(ranks, V - 1)].astype(np.int32)


def orpheus_single(seed: int = 0) -> Batch:
    """B=1, V=156940 fp32 ~ N(0, 2^2); T 0.6, top_p 0.95, top_k off,
    repetition 1.1 over a 256-token uniform history; one pre-drawn uniform."""
    rng = np.random.default_rng(seed)
    B, V, H = 1, 156940, 256
    return Batch(
        logits=(rng.standard_normal((B, V), dtype=np.float32) * np.float32(2.0)),
        temperature=np.full(B, 0.6, np.float32), top_k=np.zeros(B, np.int32),
        top_p=np.full(B, 0.95, np.float32), min_p=np.zeros(B, np.float32),
        rep_pen=np.full(B, 1.1, np.float32), pres_pen=np.zeros(B, np.float32),
        freq_pen=np.zeros(B, np.float32),
        hist_ids=rng.integers(0, V, (B, H), dtype=np.int32), hist_len=np.full(B, H, np.int32),
        uniforms=rng.random(B, dtype=np.float32), name="orpheus_b1_v156940_f32")


def qwen_mixed(seed: int = 0, B: int = 64, V: int = 151936, H: int = 1024) -> Batch:
    """Mixed-parameter continuous batch: bf16 N(0, 3^2) with 0.5% of ids per
    row spiked by +U(4, 10); per-row T U[0.3,1.5], top_k from {0,20,50,200},
    top_p U[0.8,1], min_p U[0,0.1], presence/frequency U[0,1], repetition
    U[1,1.3]; 1024-token history per row from Zipf(1.1) over the vocabulary."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, V), dtype=np.float32) * np.float32(3.0)
    nspike = max(1, int(round(0.005 * V)))
    for r in range(B):
        ids = rng.choice(V, nspike, replace=False)
        x[r, ids] += rng.uniform(4.0, 10.0, nspike).astype(np.float32)
    return Batch(
        logits=f32_to_bf16_bits(x), dtype="bf16",
        temperature=rng.uniform(0.3, 1.5, B).astype(np.float32),
        top_k=rng.choice(np.array([0, 20, 50, 200], np.int32), B),
        top_p=rng.uniform(0.8, 1.0, B).astype(np.float32),
        min_p=rng.uniform(0.0, 0.1, B).astype(np.float32),
        pres_pen=rng.uniform(0.0, 1.0, B).astype(np.float32),
        freq_pen=rng.uniform(0.0, 1.0, B).astype(np.float32),
        rep_pen=rng.uniform(1.0, 1.3, B).astype(np.float32),
        hist_ids=zipf_ids(rng, V, (B, H)), hist_len=np.full(B, H, np.int32),
        uniforms=rng.random(B, dtype=np.float32),
        seed=rng.integers(0, 2**63, B, dtype=np.uint64), offset=np.zeros(B, np.uint64),
        name=f"qwen_mixed_b{B}_v{V}_bf16")


def bucket_sweep(B: int, seed: int = 0, V: int = 128256, base_seed: int = 1000) -> Batch:
    """Large-batch bucket: fp32 Gumbel(0,1)*2.5, top_k U[1,1024], top_p 0.9,
    T 1, no penalties; Philox keyed by base_seed (+ the step through offset)."""
    rng = np.random.default_rng(seed)
    g = -np.log(-np.log(rng.random((B, V), dtype=np.float32).clip(1e-12, 1 - 1e-7)))
    return Batch(
        logits=(g.astype(np.float32) * np.float32(2.5)),
        temperature=np.ones(B, np.float32), top_k=rng.integers(1, 1025, B, dtype=np.int32),
        top_p=np.full(B, 0.9, np.float32), min_p=np.zeros(B, np.float32),
        seed=np.full(B, base_seed, np.uint64), offset=np.zeros(B, np.uint64),
        name=f"bucket_b{B}_v{V}_f32")


def tp_sharded(tp: int, seed: int = 0, B: int = 128, V: int = 152064, H: int = 512) -> list[Batch]:
    """Vocab-sharded batch: shard q holds ids [q*V/tp, (q+1)*V/tp), bf16
    logits ~ N(0, 2.5^2) drawn from seed+q; top_k 50, top_p 0.9, T 0.7,
    repetition 1.05 over a 512-token uniform history (global ids)."""
    assert V % tp == 0
    Vs = V // tp
    prm = np.random.default_rng(seed + 7919)
    common = dict(
        temperature=np.full(B, 0.7, np.float32), top_k=np.full(B, 50, np.int32),
        top_p=np.full(B, 0.9, np.float32), min_p=np.zeros(B, np.float32),
        rep_pen=np.full(B, 1.05, np.float32), pres_pen=np.zeros(B, np.float32),
        freq_pen=np.zeros(B, np.float32),
        hist_ids=prm.integers(0, V, (B, H), dtype=np.int32), hist_len=np.full(B, H, np.int32),
        uniforms=prm.random(B, dtype=np.float32))
    shards = []
    for q in range(tp):
        rng = np.random.default_rng(seed + q)
        x = rng.standard_normal((B, Vs), dtype=np.float32) * np.float32(2.5)
        shards.append(Batch(logits=f32_to_bf16_bits(x), dtype="bf16", vocab_offset=q * Vs,
                            name=f"tp{tp}_shard{q}_b{B}_v{V}_bf16", **common))
    return shards


def tp_topk_off(tp: int, seed: int = 0, B: int = 32, V: int = 48000, H: int = 128, spike_frac: float = 0.003,
                top_p: tuple = (0.9, 1.0)) -> list[Batch]:
    """Vocab-sharded rows with top_k off, as the Thinker samples whenever a
    temperature is given (python/mstar_rs/models/qwen3_omni.py:440-443):
    bf16 N(0, 1) logits with spike_frac of each shard's ids spiked by
    +U(6, 10) (a peaked distribution), T 0.7, top_k 0, top_p cycling through
    `top_p` by row, repetition 1.05 over a uniform history."""
    assert V % tp == 0
    Vs = V // tp
    prm = np.random.default_rng(seed + 104729)
    common = dict(
        temperature=np.full(B, 0.7, np.float32), top_k=np.zeros(B, np.int32),
        top_p=np.array([top_p[r % len(top_p)] for r in range(B)], np.float32), min_p=np.zeros(B, np.float32),
        rep_pen=np.full(B, 1.05, np.float32), pres_pen=np.zeros(B, np.float32),
        freq_pen=np.zeros(B, np.float32),
        hist_ids=prm.integers(0, V, (B, H), dtype=np.int32), hist_len=np.full(B, H, np.int32),
        uniforms=prm.random(B, dtype=np.float32))
    shards = []
    nspike = max(1, int(round(spike_frac * Vs)))
    for q in range(tp):
        rng = np.random.default_rng(seed + 31 * q + 1)
        x = rng.standard_normal((B, Vs), dtype=np.float32)
        for r in range(B):
            ids = rng.choice(Vs, nspike, replace=False)
            x[r, ids] += rng.uniform(6.0, 10.0, nspike).astype(np.float32)
        shards.append(Batch(logits=f32_to_bf16_bits(x), dtype="bf16", vocab_offset=q * Vs,
                            name=f"tpk0_{tp}_shard{q}_b{B}_v{V}_bf16", **common))
    return shards


def tp_full(shards: list[Batch]) -> Batch:
    s0 = shards[0]
    b = Batch(**{f.name: getattr(s0, f.name) for f in fields(s0)})
    b.logits = np.concatenate([s.logits for s in shards], axis=1)
    b.vocab_offset = 0
    b.name = s0.name.split("_shard")[0] + "_full"
    return b


def constrained(seed: int = 0, B: int = 512, V: int = 257152, NB: int = 32, density: float = 0.05) -> Batch:
    """Constrained / biased decoding: fp32 N(0, 2^2); allowed-token bitmask of
    5% random density (>= 1 allowed id per row); logit_bias on 32 random ids
    per row with values U[-100, 100]; T 0.8, top_p 0.95, min_p 0.05."""
    rng = np.random.default_rng(seed)
    allowed = rng.random((B, V)) < density
    empty = ~allowed.any(axis=1)
    allowed[empty, rng.integers(0, V, int(empty.sum()))] = True
    return Batch(
        logits=(rng.standard_normal((B, V), dtype=np.float32) * np.float32(2.0)),
        temperature=np.full(B, 0.8, np.float32), top_k=np.zeros(B, np.int32),
        top_p=np.full(B, 0.95, np.float32), min_p=np.full(B, 0.05, np.float32),
        bias_ids=rng.integers(0, V, (B, NB), dtype=np.int32),
        bias_vals=rng.uniform(-100.0, 100.0, (B, NB)).astype(np.float32),
        allowed_bits=pack_bits(allowed), uniforms=rng.random(B, dtype=np.float32),
        name=f"constrained_b{B}_v{V}_f32")


def to_device(b: Batch, device="cuda", with_uniforms: bool = True) -> dict:
    """Device tensors for kernel.sampler_step (logits + parameter kwargs)."""
    import torch

    def t(a, dt):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a).view(dt)).to(device)

    if b.dtype == "bf16":
        logits = torch.from_numpy(np.ascontiguousarray(b.logits).view(np.int16)).to(device).view(torch.bfloat16)
    else:
        logits = torch.from_numpy(np.ascontiguousarray(b.logits, dtype=np.float32)).to(device)
    kw = dict(
        slot_idx=t(b.slot_idx, np.int32), temperature=t(b.temperature, np.float32),
        top_k=t(b.top_k, np.int32), top_p=t(b.top_p, np.float32), min_p=t(b.min_p, np.float32),
        rep_pen=t(b.rep_pen, np.float32), pres_pen=t(b.pres_pen, np.float32),
        freq_pen=t(b.freq_pen, np.float32), hist_ids=t(b.hist_ids, np.int32),
        hist_len=t(b.hist_len, np.int32), seen_bits=t(b.seen_bits, np.int32),
        bias_ids=t(b.bias_ids, np.int32), bias_vals=t(b.bias_vals, np.float32),
        allowed_bits=t(b.allowed_bits, np.int32),
        uniforms=t(b.uniforms, np.float32) if with_uniforms else None,
        seed=t(b.seed, np.int64), offset=t(b.offset, np.int64), vocab_offset=b.vocab_offset)
    return {"logits": logits, **kw}


def lmhead_operands(B: int = 64, V: int = 151936, d: int = 2048, seed: int = 0, device="cuda",
                    spike_frac: float = 0.005):
    """Seeded bf16 LM-head operands whose projection hidden @ weight.T has the
    mixed workload's logits: N(0, 3^2) per entry plus, for each row, a spike
    of U(4, 10) on spike_frac of the ids.  Dimensions [0, B) of hidden are
    one-hot row markers and weight's columns [0, B) carry the row spikes, so
    the spikes ride the projection itself; the rest is Gaussian (built on the
    device: the weight is V * d * 2 bytes)."""
    import torch

    if d < B + 64:
        raise ValueError("d must leave room for one marker dimension per row")
    g = torch.Generator(device=device).manual_seed(seed)
    hidden = torch.randn(B, d, generator=g, device=device)
    hidden[:, :B] = 0.0
    hidden[torch.arange(B, device=device), torch.arange(B, device=device)] = 1.0
    weight = torch.randn(V, d, generator=g, device=device).mul_(3.0 / (d - B) ** 0.5)
    weight[:, :B] = 0.0
    nspike = max(1, int(round(spike_frac * V)))
    for r in range(B):
        ids = torch.randperm(V, generator=g, device=device)[:nspike]
        weight[ids, r] = torch.empty(nspike, device=device).uniform_(4.0, 10.0, generator=g)
    return hidden.to(torch.bfloat16), weight.to(torch.bfloat16)
