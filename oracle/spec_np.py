"""Second, independent restatement of the sampler spec in numpy.

TEST INFRASTRUCTURE ONLY: used by tests/ to cross-check the C oracle
(`oracle/sampler_oracle.c`) and to generate golden fixtures.  It is written
separately from the C file (vectorised numpy, lexsort ordering, float64-free
weight path) so that the two restatements only agree if both follow the
spec stated in the C file's header.  Parity with the reference's own sampler
(`mstar.utils.sampling`, absent from the reference tree) is UNPINNED.

All float32 arithmetic is numpy binary32 ufuncs (one IEEE op each, no FMA).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
L2E = F32(float.fromhex("0x1.715476p+0"))
COEF = [F32(float.fromhex(h)) for h in (
    "0x1.0p+0", "0x1.62e43p-1", "0x1.ebfbep-3", "0x1.c6b08ep-5", "0x1.3b2ab6p-7",
    "0x1.5d87fep-10", "0x1.430912p-13", "0x1.ffcbfcp-17", "0x1.62c022p-20")]
TWO32 = F32(4294967296.0)
STATUS_EMPTY = 1


def exp_spec(y: np.ndarray) -> np.ndarray:
    """E(y) for y <= 0, vectorised (see the C oracle's header)."""
    y = np.asarray(y, dtype=F32)
    with np.errstate(invalid="ignore", over="ignore"):
        t = (y * L2E).astype(F32)
        live = t >= F32(-64.0)
        ts = np.where(live, t, F32(0.0)).astype(F32)
        n = np.floor(ts).astype(F32)
        f = (ts - n).astype(F32)
        p = np.full_like(f, COEF[8])
        for k in range(7, -1, -1):
            p = ((p * f).astype(F32) + COEF[k]).astype(F32)
        p = np.minimum(p, F32(2.0))
        out = np.ldexp(p, n.astype(np.int32)).astype(F32)
    out = np.where(live, out, F32(0.0)).astype(F32)
    return np.where(y == F32(0.0), F32(1.0), out).astype(F32)


def okey(x: np.ndarray) -> np.ndarray:
    b = np.asarray(x, dtype=F32).view(np.uint32).copy()
    b[b == np.uint32(0x80000000)] = 0
    neg = (b & np.uint32(0x80000000)) != 0
    return np.where(neg, ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def weights(x: np.ndarray, m: F32):
    with np.errstate(invalid="ignore"):
        e = np.where(x == m, F32(1.0), exp_spec((x - m).astype(F32))).astype(F32)
    w = np.rint((e * TWO32).astype(F32)).astype(np.uint64)
    return e, w


def philox4x32_10(ctr, key):
    """Philox4x32-10 (Salmon et al., SC'11) on python ints."""
    c = [int(v) & 0xFFFFFFFF for v in ctr]
    k0, k1 = int(key[0]) & 0xFFFFFFFF, int(key[1]) & 0xFFFFFFFF
    for _ in range(10):
        p0 = 0xD2511F53 * c[0]
        p1 = 0xCD9E8D57 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k0) & 0xFFFFFFFF, p1 & 0xFFFFFFFF,
             ((p0 >> 32) ^ c[3] ^ k1) & 0xFFFFFFFF, p0 & 0xFFFFFFFF]
        k0 = (k0 + 0x9E3779B9) & 0xFFFFFFFF
        k1 = (k1 + 0xBB67AE85) & 0xFFFFFFFF
    return c


def philox_uniform(seed: int, offset: int) -> F32:
    w = philox4x32_10([offset & 0xFFFFFFFF, offset >> 32, 0, 0], [seed & 0xFFFFFFFF, seed >> 32])[0]
    return F32(w >> 8) * F32(2.0 ** -24)


def bits_get(words: np.ndarray, ids: np.ndarray) -> np.ndarray:
    return ((words[ids >> 5] >> (ids & 31).astype(np.uint32)) & 1).astype(bool)


def sample_row(logits_row, *, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0,
               rep=1.0, pres=0.0, freq=0.0, hist=None, seen_words=None,
               bias_ids=None, bias_vals=None, allowed_words=None, u=None,
               seed=0, offset=0, vocab_offset=0):
    """One row of the spec.  `hist` holds the (already length-clipped) history
    ids as global ids; words arrays are indexed by global id.  Returns
    (token (global id), status, x (processed values), kept bool[V], probs f32[V])."""
    v = np.asarray(logits_row, dtype=F32).copy()
    V = v.shape[0]
    gid = np.arange(V, dtype=np.int64) + vocab_offset
    if bias_ids is not None:
        for i, b in zip(np.asarray(bias_ids).tolist(), np.asarray(bias_vals, dtype=F32).tolist()):
            j = i - vocab_offset
            if 0 <= j < V:
                v[j] = F32(v[j] + F32(b))
    cnt = np.zeros(V, dtype=np.int64)
    if hist is not None:
        h = np.asarray(hist, dtype=np.int64) - vocab_offset
        h = h[(h >= 0) & (h < V)]
        cnt = np.bincount(h, minlength=V).astype(np.int64)
    elif seen_words is not None:
        cnt = bits_get(np.asarray(seen_words, dtype=np.uint32), gid).astype(np.int64)
    pen = cnt > 0
    if pen.any():
        R, F, P = F32(rep), F32(freq), F32(pres)
        vp = v[pen]
        with np.errstate(invalid="ignore", over="ignore"):
            vp = np.where(vp > 0, (vp / R).astype(F32), (vp * R).astype(F32)).astype(F32)
            vp = (vp - (F * cnt[pen].astype(F32)).astype(F32)).astype(F32)
            vp = (vp - P).astype(F32)
        v[pen] = vp
    excl = np.isnan(v)
    if allowed_words is not None:
        excl |= ~bits_get(np.asarray(allowed_words, dtype=np.uint32), gid)
    kept = np.zeros(V, dtype=bool)
    probs = np.zeros(V, dtype=F32)
    T = F32(temperature)
    token = -1
    if not (T >= F32(1e-5)):
        x = v
        live = ~excl
        if live.any():
            k = okey(v)
            kl = np.where(live, k, 0)
            best = kl[live].max()
            cand = np.nonzero(live & (kl == best))[0]
            token = int(cand[0])
            if v[token] == -np.inf:
                token = -1
        if token >= 0:
            kept[token] = True
            probs[token] = 1.0
    else:
        invT = F32(F32(1.0) / T)
        with np.errstate(invalid="ignore", over="ignore"):
            x = (v * invT).astype(F32)
        excl = excl | np.isnan(x)
        live = ~excl
        if live.any():
            m = x[live].max()
            if m != -np.inf:
                ids = np.nonzero(live)[0]
                e, w = weights(x[ids], m)
                pos = w > 0
                ids, e, w = ids[pos], e[pos], w[pos]
                order = np.lexsort((ids, -x[ids].astype(np.float64)))  # x desc, id asc
                # okey ties (-0 == +0) are equal float64 values too, so lexsort agrees
                ids, e, w = ids[order], e[order], w[order]
                nA = ids.shape[0]
                if top_k > 0:
                    nA = min(nA, int(top_k))
                Mp = F32(min_p)
                if Mp > 0:
                    Mp = min(Mp, F32(1.0))
                    bad = np.nonzero(~(e[:nA] >= Mp))[0]
                    if bad.size:
                        nA = int(bad[0])
                w = w[:nA]
                WA = int(w.sum(dtype=np.uint64))
                nK = nA
                if F32(top_p) < F32(1.0):
                    thr = float(F32(top_p)) * float(WA)
                    S = np.concatenate([[0], np.cumsum(w, dtype=np.uint64)[:-1]]).astype(np.uint64)
                    keep = S.astype(np.float64) < thr
                    keep[0] = True
                    nK = int(np.argmin(keep)) if not keep.all() else nA
                wk = w[:nK]
                WK = int(wk.sum(dtype=np.uint64))
                uu = F32(u) if u is not None else philox_uniform(seed, offset)
                r = 0
                if uu > 0:
                    t = np.floor(float(uu) * float(WK))
                    r = WK - 1 if t >= float(WK) else int(t)
                incl = np.cumsum(wk, dtype=np.uint64)
                j = int(np.searchsorted(incl, np.uint64(r), side="right"))
                token = int(ids[j])
                kept[ids[:nK]] = True
                probs[ids[:nK]] = (wk.astype(np.float64) / float(WK)).astype(F32)
    xo = np.where(excl, np.where(np.isnan(x), x, F32(-np.inf)), x).astype(F32)
    status = 0
    if token < 0:
        status = STATUS_EMPTY
        token = 0
    return token + vocab_offset, status, xo, kept, probs
