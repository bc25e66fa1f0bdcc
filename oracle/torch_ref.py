"""Second CPU oracle: the sampler written the way a torch sampler is usually
written -- TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU-baseline leg load this module, as a checker or
as a timed CPU arm; the product package never imports it.

Parity status: UNPINNED, like the C oracle.  The reference's sampler
(`mstar.utils.sampling`, imported by python/mstar_rs/models/orpheus.py:78-83
and qwen3_omni.py:405, :906-911) is neither vendored nor installed, so no
reference output exists.  This module restates the same call-site semantics
(greedy = temperature 0 / top_k 1, orpheus.py:177-183; repetition penalty over
the generated tokens, orpheus.py:187, :500; per-request parameters,
qwen3_omni.py:1001-1009) in the common torch formulation, independently of
the C spec oracle:

    v        = logits (f32) + logit_bias; repetition / frequency / presence
               penalties on tokens with count > 0; disallowed ids -> -inf
    greedy   = argmax, lowest id among equal maxima
    x        = v * (1 / T)                                   (f32)
    p        = softmax(x) in float64                         (exp, not the spec's E)
    order    = stable sort by x descending (ties: lower id first)
    top_k    = first K of the order
    min_p    = p >= min_p * p_max
    top_p    = exclusive cumsum of the renormalised A-set mass < top_p
    draw     = first kept token whose inclusive cumsum exceeds u * W_K

Where it departs from the spec oracle on purpose, and what the comparison
tests allow for:
  - probabilities come from float64 `exp`, not from the spec's binary32
    polynomial E and 2^-32 fixed-point weights; boundaries (min_p cut, top_p
    cut, the draw) that fall within a small relative margin of a candidate's
    cumulative mass may land on the neighbouring token;
  - the spec gives weight 0 to tokens more than ~22.9 below the row maximum
    (E(x - m) * 2^32 rounds to 0); `drop_tiny=True` applies the same cut so
    the kept sets can be compared, `drop_tiny=False` keeps them (their total
    probability is below V * 1.2e-10).
"""
from __future__ import annotations

import numpy as np
import torch

TINY_LOG = float(np.log(2.0 ** -33))  # e^(x - m) below this rounds to weight 0 in the spec


def _philox_uniform(seed: int, offset: int) -> float:
    """Philox4x32-10 (Salmon et al., SC'11), first output word of counter
    (offset lo, offset hi, 0, 0) under key seed, as (w >> 8) * 2^-24."""
    M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
    c = [offset & 0xFFFFFFFF, (offset >> 32) & 0xFFFFFFFF, 0, 0]
    k0, k1 = seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF
    for _ in range(10):
        p0, p1 = M0 * c[0], M1 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k0) & 0xFFFFFFFF, p1 & 0xFFFFFFFF,
             ((p0 >> 32) ^ c[3] ^ k1) & 0xFFFFFFFF, p0 & 0xFFFFFFFF]
        k0, k1 = (k0 + W0) & 0xFFFFFFFF, (k1 + W1) & 0xFFFFFFFF
    return float(np.float32(c[0] >> 8) * np.float32(2.0 ** -24))


def _counts(case, slot: int, V: int, goff: int) -> torch.Tensor:
    """Occurrence count of every id of the row (history ring or seen bits)."""
    c = torch.zeros(V, dtype=torch.int64)
    if case.hist_ids is not None:
        n = min(int(case.hist_len[slot]), case.hist_ids.shape[1])
        ids = torch.from_numpy(case.hist_ids[slot, :n].astype(np.int64)) - goff
        ids = ids[(ids >= 0) & (ids < V)]
        c.index_add_(0, ids, torch.ones_like(ids))
    elif case.seen_bits is not None:
        words = case.seen_bits[slot].astype(np.uint32)
        bits = np.unpackbits(words.view(np.uint8), bitorder="little")
        c = torch.from_numpy(bits[goff:goff + V].astype(np.int64))
    return c


def _allowed(case, slot: int, V: int, goff: int) -> torch.Tensor | None:
    if case.allowed_bits is None:
        return None
    words = case.allowed_bits[slot].astype(np.uint32)
    bits = np.unpackbits(words.view(np.uint8), bitorder="little")
    return torch.from_numpy(bits[goff:goff + V].astype(bool))


def sample_row(case, r: int, drop_tiny: bool = True, nudge: tuple = (0.0, 0.0, 0.0)):
    """One row -> (token, kept bool[V], probs f64[V], x f32[V]); probs over
    the kept set; x the processed logits (NaN stays NaN, disallowed -inf).
    `nudge` = relative changes of (top_p, min_p, u): used to show that a
    disagreement with the spec oracle sits on a boundary."""
    V = case.V
    goff = case.vocab_offset
    slot = int(case.slot_idx[r]) if case.slot_idx is not None else r
    g = lambda a, d: d if a is None else a[slot]  # noqa: E731
    v = torch.from_numpy(np.ascontiguousarray(case.logits_f32()[r]).copy())
    if case.bias_ids is not None:
        for i, b in zip(case.bias_ids[slot], case.bias_vals[slot]):
            if 0 <= int(i) - goff < V:
                v[int(i) - goff] = v[int(i) - goff] + torch.tensor(b, dtype=torch.float32)
    cnt = _counts(case, slot, V, goff)
    R = torch.tensor(g(case.rep_pen, 1.0), dtype=torch.float32)
    F = torch.tensor(g(case.freq_pen, 0.0), dtype=torch.float32)
    P = torch.tensor(g(case.pres_pen, 0.0), dtype=torch.float32)
    hit = cnt > 0
    pen = torch.where(v > 0, v / R, v * R)
    pen = pen - F * cnt.to(torch.float32)
    pen = pen - P
    v = torch.where(hit, pen, v)
    nan = torch.isnan(v)
    ok = ~nan
    al = _allowed(case, slot, V, goff)
    if al is not None:
        ok &= al
    v = torch.where(ok, v, torch.tensor(-float("inf")))
    kept = torch.zeros(V, dtype=torch.bool)
    probs = torch.zeros(V, dtype=torch.float64)
    T = float(g(case.temperature, 1.0))
    K = int(g(case.top_k, 0))
    greedy = not (T >= 1e-5)
    x = v if greedy else v * torch.tensor(np.float32(1.0) / np.float32(T), dtype=torch.float32)
    xdbg = torch.where(nan, torch.tensor(float("nan")), x)
    if not ok.any() or not (v.max() > -float("inf")):
        return goff, kept, probs, xdbg
    if greedy or K == 1:
        tok = int(torch.argmax(x))  # first index of the maximum
        kept[tok] = True
        probs[tok] = 1.0
        return tok + goff, kept, probs, xdbg
    order = torch.sort(x, descending=True, stable=True).indices
    xs = x[order].to(torch.float64)
    m = xs[0]
    # log of the unnormalised probability relative to the max; tokens equal
    # to the max count as the max (this also defines rows whose max is +inf,
    # where plain softmax would give NaN)
    logp = torch.where(xs == m, torch.zeros_like(xs), xs - m)
    n = V
    if 0 < K < V:
        n = K
    live = torch.isfinite(logp[:n])
    if drop_tiny:
        live &= logp[:n] >= TINY_LOG
    Mp = float(g(case.min_p, 0.0)) * (1.0 + nudge[1])
    if Mp > 0:
        live &= logp[:n] >= np.log(min(Mp, 1.0))
    # A is the longest prefix of live members
    nA = int(torch.argmin(live.to(torch.int8))) if not bool(live.all()) else n
    if nA == 0:
        tok = int(order[0])
        return tok + goff, kept, probs, xdbg
    w = torch.exp(logp[:nA])
    pA = w / w.sum()
    Ptop = float(g(case.top_p, 1.0)) * (1.0 + nudge[0])
    nK = nA
    if Ptop < 1.0:
        excl = torch.cumsum(pA, 0) - pA
        keep = excl < Ptop
        keep[0] = True
        nK = int(keep.sum())
    wk = w[:nK]
    pk = wk / wk.sum()
    if case.uniforms is not None:
        u = float(case.uniforms[r])
    else:
        u = _philox_uniform(int(g(case.seed, 0)), int(g(case.offset, 0)))
    u = u * (1.0 + nudge[2])
    cum = torch.cumsum(pk, 0)
    j = int(torch.searchsorted(cum, torch.tensor([u], dtype=torch.float64), right=True)[0])
    j = min(j, nK - 1)
    ids = order[:nK]
    kept[ids] = True
    probs[ids] = pk
    return int(ids[j]) + goff, kept, probs, xdbg


def run(case, drop_tiny: bool = True):
    """All rows; returns dict(ids, kept, probs, x).  Padding rows (slot < 0)
    return vocab_offset with an empty kept set and x = -inf."""
    B, V = case.B, case.V
    ids = np.zeros(B, np.int64)
    kept = np.zeros((B, V), bool)
    probs = np.zeros((B, V), np.float64)
    x = np.full((B, V), -np.inf, np.float32)
    for r in range(B):
        if case.slot_idx is not None and int(case.slot_idx[r]) < 0:
            ids[r] = case.vocab_offset
            continue
        t, k, p, xr = sample_row(case, r, drop_tiny=drop_tiny)
        ids[r], kept[r], probs[r], x[r] = t, k.numpy(), p.numpy(), xr.numpy()
    return dict(ids=ids, kept=kept, probs=probs, x=x)


def run_batched(case, drop_tiny: bool = True):
    """The same formulation as `sample_row`, vectorised over the rows of the
    batch (batched sort, cumsum and searchsorted use torch's intra-op
    threads): the timed CPU baseline.  Its float64 sums run over whole rows,
    so on a boundary it may round differently from `sample_row`; the
    comparison tests use `sample_row`."""
    B, V = case.B, case.V
    goff = case.vocab_offset
    slots = np.arange(B) if case.slot_idx is None else case.slot_idx.astype(np.int64)
    live_row = slots >= 0
    sl = np.where(live_row, slots, 0)
    g = lambda a, d: np.full(B, d) if a is None else np.asarray(a)[sl]  # noqa: E731
    v = torch.from_numpy(np.ascontiguousarray(case.logits_f32()).copy())
    rows = torch.arange(B)
    if case.bias_ids is not None:
        for k in range(case.bias_ids.shape[1]):  # list order
            ids = case.bias_ids[sl, k].astype(np.int64) - goff
            ok = (ids >= 0) & (ids < V)
            r = rows[torch.from_numpy(ok)]
            c = torch.from_numpy(ids[ok])
            v[r, c] = v[r, c] + torch.from_numpy(case.bias_vals[sl, k][ok].astype(np.float32))
    cnt = torch.zeros(B, V, dtype=torch.int64)
    if case.hist_ids is not None:
        H = case.hist_ids.shape[1]
        hid = torch.from_numpy(case.hist_ids[sl].astype(np.int64)) - goff
        hl = torch.from_numpy(np.minimum(case.hist_len[sl], H).astype(np.int64))
        ok = (torch.arange(H)[None, :] < hl[:, None]) & (hid >= 0) & (hid < V)
        cnt.scatter_add_(1, torch.where(ok, hid, 0), ok.to(torch.int64))
    elif case.seen_bits is not None:
        bits = np.unpackbits(case.seen_bits[sl].astype(np.uint32).view(np.uint8), axis=1, bitorder="little")
        cnt = torch.from_numpy(bits[:, goff:goff + V].astype(np.int64))
    R = torch.from_numpy(g(case.rep_pen, 1.0).astype(np.float32))[:, None]
    F = torch.from_numpy(g(case.freq_pen, 0.0).astype(np.float32))[:, None]
    P = torch.from_numpy(g(case.pres_pen, 0.0).astype(np.float32))[:, None]
    pen = torch.where(v > 0, v / R, v * R) - F * cnt.to(torch.float32) - P
    v = torch.where(cnt > 0, pen, v)
    ok = ~torch.isnan(v)
    if case.allowed_bits is not None:
        bits = np.unpackbits(case.allowed_bits[sl].astype(np.uint32).view(np.uint8), axis=1, bitorder="little")
        ok &= torch.from_numpy(bits[:, goff:goff + V].astype(bool))
    v = torch.where(ok, v, torch.tensor(-float("inf")))
    T = g(case.temperature, 1.0).astype(np.float32)
    K = g(case.top_k, 0).astype(np.int64)
    greedy = ~(T >= 1e-5)
    invT = np.where(greedy, np.float32(1.0), np.float32(1.0) / np.where(greedy, np.float32(1.0), T))
    x = v * torch.from_numpy(invT.astype(np.float32))[:, None]
    ids = np.full(B, goff, np.int64)
    empty = ~(ok.any(1) & (v.max(1).values > -float("inf"))).numpy()
    one = greedy | (K == 1)
    am = torch.argmax(x, dim=1).numpy()
    ids[one & ~empty] = am[one & ~empty] + goff
    rest = live_row & ~one & ~empty
    if rest.any():
        ri = torch.from_numpy(np.flatnonzero(rest))
        xs, order = torch.sort(x[ri], dim=1, descending=True, stable=True)
        xs = xs.to(torch.float64)
        m = xs[:, :1]
        logp = torch.where(xs == m, torch.zeros_like(xs), xs - m)
        pos = torch.arange(V)[None, :]
        Kr = torch.from_numpy(np.where((K[rest] > 0) & (K[rest] < V), K[rest], V))[:, None]
        alive = torch.isfinite(logp) & (pos < Kr)
        if drop_tiny:
            alive &= logp >= TINY_LOG
        Mp = g(case.min_p, 0.0)[rest].astype(np.float64)
        lmp = torch.from_numpy(np.where(Mp > 0, np.log(np.minimum(np.where(Mp > 0, Mp, 1.0), 1.0)), -np.inf))[:, None]
        alive &= logp >= lmp
        nA = torch.cumprod(alive.to(torch.int64), dim=1).sum(1, keepdim=True)
        inA = pos < nA
        w = torch.where(inA, torch.exp(logp), torch.zeros_like(logp))
        pA = w / w.sum(1, keepdim=True).clamp_min(1e-300)
        Pt = torch.from_numpy(g(case.top_p, 1.0)[rest].astype(np.float64))[:, None]
        excl = torch.cumsum(pA, 1) - pA
        keep = ((excl < Pt) | (pos == 0)) & inA
        nK = torch.where(Pt < 1.0, keep.sum(1, keepdim=True), nA)
        wk = torch.where(pos < nK, w, torch.zeros_like(w))
        pk = wk / wk.sum(1, keepdim=True).clamp_min(1e-300)
        if case.uniforms is not None:
            u = case.uniforms[np.flatnonzero(rest)].astype(np.float64)
        else:
            u = np.array([_philox_uniform(int(g(case.seed, 0)[i]), int(g(case.offset, 0)[i]))
                          for i in np.flatnonzero(rest)], np.float64)
        cum = torch.cumsum(pk, 1)
        j = torch.searchsorted(cum, torch.from_numpy(u)[:, None], right=True)
        j = torch.minimum(j, (nK - 1).clamp_min(0))
        tok = torch.gather(order, 1, j)[:, 0]
        tok = torch.where(nA[:, 0] > 0, tok, order[:, 0])
        ids[rest] = tok.numpy() + goff
    return dict(ids=ids)
