"""Vocab-parallel sampling restated in numpy -- TEST INFRASTRUCTURE ONLY.

Only tests/ use this module, as the checker of the tensor-parallel record
format and of the merge; the product never imports it.

Parity status: UNPINNED (see oracle/sampler_oracle.c).  The reference keeps
Thinker ranks in agreement by broadcasting the sampled token
(python/mstar_rs/models/qwen3_omni.py:401-404); the vocab-parallel scheme
restated here replaces that broadcast: every rank samples its contiguous id
range, emits a fixed-size record, the records are all-gathered, and every
rank merges them the same way.

Record of one row (uint32 words, 4 + 2 * tp_cap of them):
  [0] bits of the shard's max transformed value m_q (-inf when the shard has
      no live token), [1] entry count (0 on overflow), [2] status bits,
  [3] 0, then (x bits, global id) pairs of the shard's value-A set computed
  against m_q, in order (x descending, id ascending), cut at top_k.  Greedy /
  top-1 rows carry one pair: (m_q, lowest id at m_q).

Merge: m = max_q m_q; the union of the pairs, re-weighted against m, goes
through the same A set / top_p / draw steps as a full row.  Because every
member of the row's A set in shard q is in shard q's record (weights against
m_q >= weights against m, and the row's first K are among each shard's first
K), the merge equals the full-row spec whenever no shard overflowed.
"""
from __future__ import annotations

import numpy as np

from . import spec_np as S

F32 = np.float32
STATUS_EMPTY = 0x1
STATUS_TP_OVERFLOW = 0x8


def _f2u(x) -> int:
    return int(np.asarray(x, dtype=F32).view(np.uint32))


def _u2f(u) -> F32:
    return np.asarray(u, dtype=np.uint32).view(F32)


def shard_values(logits_row, *, temperature, rep, pres, freq, hist, vocab_offset):
    """Processed values x of a shard row and its live mask, as the spec
    computes them (penalties only for history ids inside the shard)."""
    _, _, x, _, _ = S.sample_row(logits_row, temperature=temperature, rep=rep, pres=pres, freq=freq,
                                 hist=hist, u=F32(0.5), vocab_offset=vocab_offset)
    x = np.asarray(x, dtype=F32)
    live = ~np.isnan(x) & (x != -np.inf)
    return x, live


def shard_record(logits_row, tp_cap: int, *, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0,
                 rep=1.0, pres=0.0, freq=0.0, hist=None, vocab_offset=0) -> np.ndarray:
    rec = np.zeros(4 + 2 * tp_cap, dtype=np.uint32)
    x, live = shard_values(logits_row, temperature=temperature, rep=rep, pres=pres, freq=freq, hist=hist,
                           vocab_offset=vocab_offset)
    if not live.any():
        rec[0] = _f2u(-np.inf)
        rec[2] = STATUS_EMPTY
        return rec
    ids = np.nonzero(live)[0]
    m = x[ids].max()
    rec[0] = _f2u(m)
    greedy = not (F32(temperature) >= F32(1e-5))
    if greedy or int(top_k) == 1:
        best = ids[x[ids] == m].min()
        rec[1] = 1
        rec[4] = _f2u(m)
        rec[5] = int(best) + vocab_offset
        return rec
    e, w = S.weights(x[ids], m)
    keep = w > 0
    if F32(min_p) > 0:
        keep &= e >= min(F32(min_p), F32(1.0))
    ids = ids[keep]
    order = np.lexsort((ids, -x[ids].astype(np.float64)))
    ids = ids[order]
    if int(top_k) > 0:
        ids = ids[: int(top_k)]
    if ids.shape[0] > tp_cap:
        rec[1] = 0
        rec[2] = STATUS_TP_OVERFLOW
        return rec
    rec[1] = ids.shape[0]
    for j, i in enumerate(ids.tolist()):
        rec[4 + 2 * j] = _f2u(x[i])
        rec[5 + 2 * j] = i + vocab_offset
    return rec


def merge(records: np.ndarray, *, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, u=None) -> tuple[int, int]:
    """records: [tp_world, 4 + 2 * tp_cap] uint32 for one row -> (token, status)."""
    ms = _u2f(records[:, 0])
    status = int(np.bitwise_or.reduce(records[:, 2])) & ~STATUS_EMPTY
    m = ms.max()
    if not (m > -np.inf):
        return 0, status | STATUS_EMPTY
    xs, gs = [], []
    for r in records:
        n = int(r[1])
        xs.append(_u2f(r[4: 4 + 2 * n: 2]))
        gs.append(r[5: 5 + 2 * n: 2].astype(np.int64))
    x = np.concatenate(xs).astype(F32)
    g = np.concatenate(gs)
    greedy = not (F32(temperature) >= F32(1e-5))
    if greedy or int(top_k) == 1:
        return int(g[x == m].min()), status
    order = np.lexsort((g, -x.astype(np.float64)))
    x, g = x[order], g[order]
    e, w = S.weights(x, m)
    ok = w > 0
    if F32(min_p) > 0:
        ok &= e >= min(F32(min_p), F32(1.0))
    nA = int(np.argmin(ok)) if not ok.all() else ok.shape[0]
    if int(top_k) > 0:
        nA = min(nA, int(top_k))
    w = w[:nA].astype(np.uint64)
    S_ex = np.concatenate([[np.uint64(0)], np.cumsum(w, dtype=np.uint64)[:-1]]) if nA else np.zeros(0, np.uint64)
    WA = int(w.sum(dtype=np.uint64))
    nK = nA
    if F32(top_p) < F32(1.0):
        thr = float(np.float64(F32(top_p)) * np.float64(WA))
        keep = np.array([j == 0 or float(np.float64(S_ex[j])) < thr for j in range(nA)], dtype=bool)
        nK = max(int(keep.sum()), 1)
    WK = int(w[:nK].sum(dtype=np.uint64))
    uu = F32(0.0) if u is None else F32(u)
    if uu > 0 and WK > 0:
        r = int(np.floor(np.float64(uu) * np.float64(WK)))
        r = min(r, WK - 1)
    else:
        r = 0
    for j in range(nK):
        if int(S_ex[j]) + int(w[j]) > r:
            return int(g[j]), status
    return int(g[0]), status


# ---------------------------------------------------------------- two rounds
#
# Rows without top_k (or with one above tp_cap): round 1 sends the first
# tp_cap members of each shard's A set, flagged (word 3, bit 0) as possibly
# partial; a row with a partial shard (entry count == tp_cap) is deferred
# with the row max M of round 1; round 2 sends each shard's exact A mass
# against M; the second merge decides the row when its kept set (top_p) or
# its draw point (no top_p) lies among the members with keys up to k*, the
# smallest last-sent key of the partial shards (every key up to k* was sent).
# Otherwise the row is flagged STATUS_TP_OVERFLOW.


def shard_record2(logits_row, tp_cap: int, *, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, rep=1.0, pres=0.0,
                  freq=0.0, hist=None, vocab_offset=0) -> np.ndarray:
    greedy = not (F32(temperature) >= F32(1e-5))
    pseudo = (not greedy) and (int(top_k) <= 0 or int(top_k) > tp_cap) and tp_cap < len(logits_row)
    rec = shard_record(logits_row, tp_cap, temperature=temperature, top_k=tp_cap if pseudo else top_k, top_p=top_p,
                       min_p=min_p, rep=rep, pres=pres, freq=freq, hist=hist, vocab_offset=vocab_offset)
    if pseudo:
        rec[3] = 1
    return rec


def _partial(rec, tp_cap) -> bool:
    return bool(int(rec[3]) & 1) and int(rec[1]) >= tp_cap


def merge1(records: np.ndarray, tp_cap: int, *, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, u=None):
    """-> (token, status, deferred, M); token is None for a deferred row."""
    m = _u2f(records[:, 0]).max()
    one = (not (F32(temperature) >= F32(1e-5))) or int(top_k) == 1
    if any(_partial(r, tp_cap) for r in records) and not one and m > -np.inf:
        return None, 0, True, F32(m)
    tok, st = merge(records, temperature=temperature, top_k=top_k, top_p=top_p, min_p=min_p, u=u)
    return tok, st, False, F32(m)


def shard_mass(logits_row, M, *, temperature=1.0, min_p=0.0, rep=1.0, pres=0.0, freq=0.0, hist=None,
               vocab_offset=0) -> int:
    """Exact A mass (sum of the spec's fixed-point weights) of a shard row
    against the row max M."""
    x, live = shard_values(logits_row, temperature=temperature, rep=rep, pres=pres, freq=freq, hist=hist,
                           vocab_offset=vocab_offset)
    e, w = S.weights(x[live], F32(M))
    keep = w > 0
    if F32(min_p) > 0:
        keep &= e >= min(F32(min_p), F32(1.0))
    return int(w[keep].astype(np.uint64).sum(dtype=np.uint64))


def _key(km: int, x, g) -> int:
    return ((km - int(S.okey(np.asarray([x], dtype=F32))[0])) << 32) | int(g)


def merge2(records: np.ndarray, masses, tp_cap: int, M, *, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0,
           u=None, V_global=None) -> tuple[int, int]:
    status = int(np.bitwise_or.reduce(records[:, 2])) & ~STATUS_EMPTY
    M = F32(M)
    km = int(S.okey(np.asarray([M], dtype=F32))[0])
    kstar = None
    xs, gs = [], []
    for r in records:
        n = min(int(r[1]), tp_cap)
        x = _u2f(r[4: 4 + 2 * n: 2]).astype(F32)
        g = r[5: 5 + 2 * n: 2].astype(np.int64)
        if _partial(r, tp_cap) and n:
            last = max(_key(km, a, b) for a, b in zip(x.tolist(), g.tolist()))
            kstar = last if kstar is None else min(kstar, last)
        xs.append(x)
        gs.append(g)
    x = np.concatenate(xs).astype(F32)
    g = np.concatenate(gs)
    e, w = S.weights(x, M)
    ok_a = w > 0
    if F32(min_p) > 0:
        ok_a &= e >= min(F32(min_p), F32(1.0))
    x, g, w = x[ok_a], g[ok_a], w[ok_a].astype(np.uint64)
    order = np.lexsort((g, -x.astype(np.float64)))
    x, g, w = x[order], g[order], w[order]
    keys = [_key(km, a, b) for a, b in zip(x.tolist(), g.tolist())]
    nk = sum(1 for k in keys if kstar is None or k <= kstar)
    Sx = [0]
    for j in range(nk):
        Sx.append(Sx[-1] + int(w[j]))  # Sx[j] = exclusive prefix of member j; Sx[nk] = G
    ok = nk > 0
    K = int(top_k)
    if V_global is not None and K >= V_global:
        K = 0  # top_k covering the vocabulary is off
    if ok and K > 0:
        ok = K <= nk
        nA = K
        WA = Sx[K] if ok else 0
    else:
        nA = -1
        WA = int(sum(int(v) for v in masses))
    nK, WK = 0, 0
    if ok and F32(top_p) < F32(1.0):
        thr = float(np.float64(F32(top_p)) * np.float64(WA))
        lim = nA if nA >= 0 else nk
        for j in range(1, lim + 1):
            if not (float(np.float64(Sx[j])) < thr):
                nK = j
                break
        if nK == 0 and nA >= 0:
            nK = nA
        ok = nK > 0
        WK = Sx[nK] if ok else 0
    elif ok:
        nK = nA if nA >= 0 else nk
        WK = Sx[nA] if nA >= 0 else WA
    token = int(g[0]) if g.shape[0] else 0
    if ok and WK > 0:
        uu = F32(0.0) if u is None else F32(u)
        rr = min(int(np.floor(np.float64(uu) * np.float64(WK))), WK - 1) if uu > 0 else 0
        ok = False
        for j in range(min(nK, nk)):
            if Sx[j] <= rr < Sx[j] + int(w[j]):
                token = int(g[j])
                ok = True
                break
    if not ok:
        status |= STATUS_TP_OVERFLOW
    return token, status
