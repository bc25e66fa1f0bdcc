"""CPU: the vocab-parallel record format, exchange and merge.

Shard records come from the numpy restatement (oracle/tp_np.py), the
exchange is the product's own gather (mstar_rs_b200.tp._default_gather) over
a world-size-2 gloo group on 127.0.0.1, and the merged ids must equal the C
oracle's ids for the concatenated row."""
import os
import socket

import numpy as np
import pytest

from mstar_rs_b200 import workloads as W

TP_CAP = 64


def _shard_records(shard, tp_cap=TP_CAP):
    from oracle import tp_np

    recs = []
    for r in range(shard.B):
        lf = shard.logits_f32()[r]
        hist = shard.hist_ids[r, : int(shard.hist_len[r])] if shard.hist_ids is not None else None
        recs.append(tp_np.shard_record(
            lf, tp_cap, temperature=shard.temperature[r], top_k=shard.top_k[r], top_p=shard.top_p[r],
            min_p=shard.min_p[r], rep=shard.rep_pen[r], pres=shard.pres_pen[r], freq=shard.freq_pen[r],
            hist=hist, vocab_offset=shard.vocab_offset))
    return np.stack(recs)


def _merge_all(recv, case):
    from oracle import tp_np

    ids = []
    for r in range(case.B):
        tok, _ = tp_np.merge(recv[:, r], temperature=case.temperature[r], top_k=case.top_k[r],
                             top_p=case.top_p[r], min_p=case.min_p[r], u=case.uniforms[r])
        ids.append(tok)
    return np.array(ids, np.int64)


def _small_shards(tp, seed=3):
    return W.tp_sharded(tp, seed=seed, B=6, V=tp * 2500, H=64)


@pytest.mark.parametrize("tp", [2, 4])
def test_merge_equals_full_row(oracle_lib, tp):
    shards = _small_shards(tp)
    recv = np.stack([_shard_records(s) for s in shards])  # [tp, B, words]
    full = W.tp_full(shards)
    ref = oracle_lib.run(full)["ids"]
    np.testing.assert_array_equal(_merge_all(recv, full), ref)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    from mstar_rs_b200 import tp as TP

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = _small_shards(world)[rank]
        send = torch.from_numpy(_shard_records(shard).astype(np.int32).reshape(-1))
        recv = torch.zeros(world * send.numel(), dtype=torch.int32)
        TP._default_gather(None)(recv, send)
        np.save(os.path.join(out_dir, f"recv{rank}.npy"), recv.numpy())
    finally:
        dist.destroy_process_group()


def test_gloo_exchange_two_ranks(oracle_lib, tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    shards = _small_shards(world)
    full = W.tp_full(shards)
    ref = oracle_lib.run(full)["ids"]
    words = 4 + 2 * TP_CAP
    got = []
    for rank in range(world):
        recv = np.load(tmp_path / f"recv{rank}.npy").view(np.uint32).reshape(world, full.B, words)
        got.append(_merge_all(recv, full))
    np.testing.assert_array_equal(got[0], got[1])  # every rank draws the same ids
    np.testing.assert_array_equal(got[0], ref)


def _agree_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from mstar_rs_b200.sampling import _tp_agree, _tp_world

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ids = torch.tensor([1, 2, 3]) if rank == 0 else torch.tensor([9, 9, 9])
        _tp_agree(dist.group.WORLD, ids)
        q.put((rank, _tp_world(dist.group.WORLD), ids.tolist()))
    finally:
        dist.destroy_process_group()


def test_tp_group_broadcast_gloo():
    """The tp_group agreement step (rank 0's ids on every rank) over a
    world-size-2 gloo group on 127.0.0.1."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == [(0, 2, [1, 2, 3]), (1, 2, [1, 2, 3])]


# ------------------------------------------------------------ two rounds

def _shard_records2(shard, tp_cap=TP_CAP):
    from oracle import tp_np

    recs = []
    for r in range(shard.B):
        recs.append(tp_np.shard_record2(shard.logits_f32()[r], tp_cap, **_row_kw(shard, r)))
    return np.stack(recs)


def _row_kw(shard, r):
    return dict(temperature=shard.temperature[r], top_k=shard.top_k[r], top_p=shard.top_p[r], min_p=shard.min_p[r],
                rep=shard.rep_pen[r], pres=shard.pres_pen[r], freq=shard.freq_pen[r],
                hist=shard.hist_ids[r, : int(shard.hist_len[r])], vocab_offset=shard.vocab_offset)


def _shard_masses(shard, pend_m):
    """[B] exact A masses of a shard's deferred rows (0 for the others)."""
    from oracle import tp_np

    out = np.zeros(shard.B, np.uint64)
    for r, M in enumerate(pend_m):
        if M is not None:
            kw = _row_kw(shard, r)
            kw.pop("top_k")
            kw.pop("top_p")
            out[r] = tp_np.shard_mass(shard.logits_f32()[r], M, **kw)
    return out


def _merge_two_rounds(recv, case, masses_of):
    """Both merges of the two-round exchange over gathered records
    [tp, B, words]; masses_of(pend_m) -> [tp, B] exact masses."""
    from oracle import tp_np

    B = case.B
    ids = np.zeros(B, np.int64)
    status = np.zeros(B, np.int64)
    pend_m = [None] * B
    for r in range(B):
        kw = dict(temperature=case.temperature[r], top_k=case.top_k[r], top_p=case.top_p[r], min_p=case.min_p[r],
                  u=case.uniforms[r])
        tok, st, deferred, M = tp_np.merge1(recv[:, r], TP_CAP, **kw)
        if deferred:
            pend_m[r] = M
        else:
            ids[r], status[r] = tok, st
    masses = masses_of(pend_m)
    for r in range(B):
        if pend_m[r] is not None:
            kw = dict(temperature=case.temperature[r], top_k=case.top_k[r], top_p=case.top_p[r],
                      min_p=case.min_p[r], u=case.uniforms[r])
            ids[r], status[r] = tp_np.merge2(recv[:, r], [int(m) for m in masses[:, r]], TP_CAP, pend_m[r],
                                             V_global=case.V, **kw)
    return ids, status, sum(m is not None for m in pend_m)


@pytest.mark.parametrize("tp,spikes", [(2, 0.003), (4, 0.003), (2, 0.0), (4, 0.0)])
def test_two_round_merge_equals_full_row(oracle_lib, tp, spikes):
    """top_k off under vocab parallelism: every row the two rounds decide
    carries the full row's oracle id; the others are flagged (peaked rows:
    every row decided; flat rows: some flagged, none wrong)."""
    from oracle import tp_np

    shards = W.tp_topk_off(tp, seed=3, B=12, V=tp * 6000, H=64, spike_frac=spikes)
    full = W.tp_full(shards)
    ref = oracle_lib.run(full)["ids"]
    recv = np.stack([_shard_records2(s) for s in shards])
    ids, status, deferred = _merge_two_rounds(recv, full, lambda pm: np.stack([_shard_masses(s, pm) for s in shards]))
    assert deferred > 0
    decided = (status & tp_np.STATUS_TP_OVERFLOW) == 0
    np.testing.assert_array_equal(ids[decided], ref[decided])
    if spikes > 0:
        assert decided.all()
    else:
        assert decided.sum() >= 3


def _worker2(rank, world, port, out_dir):
    """Two-round exchange over gloo: records, then the deferred rows' masses,
    both through the product's gather."""
    import torch
    import torch.distributed as dist

    from mstar_rs_b200 import tp as TP

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shards = W.tp_topk_off(world, seed=5, B=8, V=world * 6000, H=64)
        shard = shards[rank]
        full = W.tp_full(shards)
        gather = TP._default_gather(None)
        send = torch.from_numpy(_shard_records2(shard).astype(np.int32).reshape(-1))
        recv = torch.zeros(world * send.numel(), dtype=torch.int32)
        gather(recv, send)
        recv_np = recv.numpy().view(np.uint32).reshape(world, full.B, -1)

        def masses_of(pm):
            mine = _shard_masses(shard, pm)
            send2 = torch.from_numpy(mine.view(np.int32).copy())
            recv2 = torch.zeros(world * send2.numel(), dtype=torch.int32)
            gather(recv2, send2)
            return recv2.numpy().view(np.uint64).reshape(world, full.B)

        ids, status, _ = _merge_two_rounds(recv_np, full, masses_of)
        np.save(os.path.join(out_dir, f"ids{rank}.npy"), ids)
        np.save(os.path.join(out_dir, f"status{rank}.npy"), status)
    finally:
        dist.destroy_process_group()


def test_gloo_two_round_exchange(oracle_lib, tmp_path):
    import torch.multiprocessing as mp

    from oracle import tp_np

    world = 2
    mp.spawn(_worker2, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    full = W.tp_full(W.tp_topk_off(world, seed=5, B=8, V=world * 6000, H=64))
    ref = oracle_lib.run(full)["ids"]
    ids = [np.load(tmp_path / f"ids{r}.npy") for r in range(world)]
    st = [np.load(tmp_path / f"status{r}.npy") for r in range(world)]
    np.testing.assert_array_equal(ids[0], ids[1])
    np.testing.assert_array_equal(st[0], st[1])
    assert not (st[0] & tp_np.STATUS_TP_OVERFLOW).any()
    np.testing.assert_array_equal(ids[0], ref)


def test_record_capacity_defaults():
    """Default record capacities: 64 members per shard for one round, 256 for
    two rounds, never more than the 2048 members a merge holds per row over
    all ranks; an explicit capacity beyond that is refused up front."""
    import pytest

    from mstar_rs_b200 import tp as TP

    def cap(world, two_round):
        return TP.VocabParallelSampler(4, 1000 * world, world, 0, "cpu", two_round=two_round,
                                       gather=lambda recv, send: None).tp_cap

    assert cap(1, False) == 64 and cap(8, False) == 64
    assert cap(2, True) == 256 and cap(8, True) == 256
    assert cap(16, True) == 128
    with pytest.raises(ValueError, match="2048"):
        TP.VocabParallelSampler(4, 32000, 16, 0, "cpu", tp_cap=256, gather=lambda recv, send: None)
