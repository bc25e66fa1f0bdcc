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
