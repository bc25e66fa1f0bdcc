"""GPU: vocab-parallel sampling through the C ABI, with the shards emulated
on one device.  Each shard's record must equal the numpy restatement's word
for word, and every shard's merge must return the full row's oracle ids."""
import numpy as np
import pytest

from mstar_rs_b200 import workloads as W

pytestmark = pytest.mark.gpu

TP_CAP = 64


def _records_np(shard):
    from tests.test_tp_exchange import _shard_records

    return _shard_records(shard, TP_CAP)


@pytest.mark.parametrize("tp", [2, 4])
@pytest.mark.parametrize("cluster", [0, 2])
def test_tp_local_merge(oracle_lib, tp, cluster):
    import torch

    from mstar_rs_b200 import tp as TP

    shards = W.tp_sharded(tp, seed=5, B=16, V=tp * 12000, H=128)
    full = W.tp_full(shards)
    ref = oracle_lib.run(full)["ids"]
    B = full.B
    recv_all = []

    def gather(recv, send):  # rank-major concatenation of every shard's send buffer
        recv.copy_(torch.cat(recv_all))

    samplers = [TP.VocabParallelSampler(B, full.V, tp, q, "cuda", tp_cap=TP_CAP, gather=gather) for q in range(tp)]
    devs = [W.to_device(s) for s in shards]
    for q, (smp, d) in enumerate(zip(samplers, devs)):
        logits = d.pop("logits")
        d["_logits"] = logits
        send = smp.local(logits, shards[q].vocab_offset, cluster_size=cluster, **d_params(d))
        torch.cuda.synchronize()
        got = send.cpu().numpy().view(np.uint32).reshape(B, -1).copy()
        got[:, 2] &= ~np.uint32(2)  # STATUS_GENERAL only says which path the shard took
        np.testing.assert_array_equal(got, _records_np(shards[q]), err_msg=f"shard {q} record")
        recv_all.append(send.clone())
    from mstar_rs_b200 import _native as N
    from oracle.oracle import stop_hits

    # stop ids: even rows stop on the id they sample, odd rows on another id
    stops = np.where(np.arange(B) % 2 == 0, ref, (ref + 1) % full.V).astype(np.int32).reshape(B, 1)
    hits = stop_hits(ref, stops)
    for q, (smp, d) in enumerate(zip(samplers, devs)):
        out = torch.zeros(B, dtype=torch.int64, device="cuda")
        status = torch.zeros(B, dtype=torch.int32, device="cuda")
        flags = torch.zeros(B, dtype=torch.int32, device="cuda")
        recv = smp.recv[: tp * B * smp.words]
        gather(recv, None)
        smp.merge(d["_logits"], shards[q].vocab_offset, recv, out_ids=out, out_status=status,
                  stop_ids=torch.from_numpy(stops).cuda(), stop_flags=flags, **d_params(d))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), ref, err_msg=f"merge on shard {q}")
        assert not TP.status_overflowed(status).any().item()
        np.testing.assert_array_equal((status.cpu().numpy() & N.STATUS_STOP) != 0, hits)
        np.testing.assert_array_equal(flags.cpu().numpy(), hits.astype(np.int32))


def d_params(d):
    return {k: v for k, v in d.items() if not k.startswith("_") and k != "vocab_offset"}


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_tp_full_size(oracle_lib, tp):
    """The vocab-sharded workload at its real size (B=128, V=152064, 512-token
    histories) through tp_local / tp_merge with the shards emulated on one
    device: every shard's record equals the numpy restatement's and every
    rank's merge returns the full row's oracle ids."""
    import torch

    from mstar_rs_b200 import tp as TP

    shards = W.tp_sharded(tp, seed=2)
    full = W.tp_full(shards)
    assert (full.B, full.V) == (128, 152064)
    ref = oracle_lib.run(full)["ids"]
    B = full.B
    sends = []
    samplers = [TP.VocabParallelSampler(B, full.V, tp, q, "cuda", tp_cap=TP_CAP, gather=None) for q in range(tp)]
    devs = [W.to_device(s) for s in shards]
    for q, (smp, d) in enumerate(zip(samplers, devs)):
        logits = d.pop("logits")
        d["_logits"] = logits
        send = smp.local(logits, shards[q].vocab_offset, **d_params(d))
        torch.cuda.synchronize()
        got = send.cpu().numpy().view(np.uint32).reshape(B, -1).copy()
        got[:, 2] &= ~np.uint32(2)
        np.testing.assert_array_equal(got, _records_np(shards[q]), err_msg=f"shard {q} record")
        sends.append(send.clone())
    recv = torch.cat(sends)
    for q, (smp, d) in enumerate(zip(samplers, devs)):
        out = torch.zeros(B, dtype=torch.int64, device="cuda")
        status = torch.zeros(B, dtype=torch.int32, device="cuda")
        smp.merge(d["_logits"], shards[q].vocab_offset, recv, out_ids=out, out_status=status, **d_params(d))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), ref, err_msg=f"merge on shard {q}")
        assert not TP.status_overflowed(status).any().item()


@pytest.mark.parametrize("tp,spikes", [(2, 0.003), (4, 0.003), (2, 0.0)])
def test_two_round_top_k_off(oracle_lib, tp, spikes):
    """top_k off under vocab parallelism through tp_local2 / tp_merge1 /
    tp_mass / tp_merge2 with the shards emulated on one device: records,
    shard values, deferred rows, masses, ids and overflow flags equal the
    numpy restatement's, and every decided row carries the full row's
    oracle id."""
    import torch

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import kernel
    from oracle import tp_np
    from tests.test_tp_exchange import _merge_two_rounds, _row_kw, _shard_masses, _shard_records2

    shards = W.tp_topk_off(tp, seed=3, B=12, V=tp * 6000, H=64, spike_frac=spikes)
    full = W.tp_full(shards)
    B, Vs = full.B, shards[0].V
    ref = oracle_lib.run(full)["ids"]
    devs = [W.to_device(s) for s in shards]
    words = kernel.tp_record_words(TP_CAP)
    logits = [d.pop("logits") for d in devs]
    sends, xbufs = [], []
    for q, d in enumerate(devs):
        send = torch.zeros(B * words, dtype=torch.int32, device="cuda")
        xbuf = torch.full((B, Vs), float("nan"), dtype=torch.float32, device="cuda")
        kernel.tp_local2(logits[q], TP_CAP, send, xbuf, **d)
        sends.append(send)
        xbufs.append(xbuf)
    torch.cuda.synchronize()
    recv_np = np.stack([_shard_records2(s) for s in shards])
    for q in range(tp):
        got = sends[q].cpu().numpy().view(np.uint32).reshape(B, -1).copy()
        got[:, 2] &= ~np.uint32(2)  # STATUS_GENERAL only says which path the shard took
        np.testing.assert_array_equal(got, recv_np[q], err_msg=f"shard {q} record")
        # shard values of the rows that sent a partial record, against the spec's
        xq = xbufs[q].cpu().numpy()
        for r in range(B):
            x_ref, live = tp_np.shard_values(shards[q].logits_f32()[r], **{k: v for k, v in _row_kw(shards[q], r).items()
                                                                          if k in ("temperature", "rep", "pres", "freq",
                                                                                   "hist", "vocab_offset")})
            np.testing.assert_array_equal(np.nan_to_num(xq[r][live]).view(np.uint32),
                                          np.nan_to_num(x_ref[live]).view(np.uint32), err_msg=f"shard {q} row {r}")
    recv = torch.cat(sends)
    want_ids, want_status, deferred = _merge_two_rounds(
        recv_np, full, lambda pm: np.stack([_shard_masses(s, pm) for s in shards]))
    assert deferred > 0
    pends, send2s, outs, stats = [], [], [], []
    for q, d in enumerate(devs):
        pend = torch.zeros(2 * B, dtype=torch.int32, device="cuda")
        out = torch.zeros(B, dtype=torch.int64, device="cuda")
        st = torch.zeros(B, dtype=torch.int32, device="cuda")
        kernel.tp_merge1(logits[q], TP_CAP, tp, full.V, recv, pend, **d, out_ids=out, out_status=st)
        send2 = torch.zeros(2 * B, dtype=torch.int32, device="cuda")
        kernel.tp_mass(logits[q], xbufs[q], pend, send2, **d)
        pends.append(pend)
        send2s.append(send2)
        outs.append(out)
        stats.append(st)
    torch.cuda.synchronize()
    pend_np = pends[0].cpu().numpy().view(np.uint32).reshape(B, 2)
    for q in range(1, tp):
        np.testing.assert_array_equal(pends[q].cpu().numpy(), pends[0].cpu().numpy())
    pm = [pend_np[r, 1].view(np.float32) if pend_np[r, 0] else None for r in range(B)]
    for q in range(tp):
        np.testing.assert_array_equal(send2s[q].cpu().numpy().view(np.uint64), _shard_masses(shards[q], pm),
                                      err_msg=f"shard {q} masses")
    recv2 = torch.cat(send2s)
    for q, d in enumerate(devs):
        kernel.tp_merge2(logits[q], TP_CAP, tp, full.V, recv, recv2, pends[q], **d, out_ids=outs[q],
                         out_status=stats[q])
    torch.cuda.synchronize()
    for q in range(tp):
        ids = outs[q].cpu().numpy()
        st = stats[q].cpu().numpy() & ~N.STATUS_GENERAL
        np.testing.assert_array_equal(ids, want_ids, err_msg=f"ids on shard {q}")
        np.testing.assert_array_equal((st & N.STATUS_TP_OVERFLOW) != 0, (want_status & N.STATUS_TP_OVERFLOW) != 0)
        decided = (st & N.STATUS_TP_OVERFLOW) == 0
        np.testing.assert_array_equal(ids[decided], ref[decided])
        if spikes > 0:
            assert decided.all()


def test_two_round_sampler_one_rank(oracle_lib):
    """VocabParallelSampler(two_round=True) end to end at one rank (the
    exchange is a copy): rows without top_k go through both rounds."""
    import torch

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import tp as TP

    shards = W.tp_topk_off(1, seed=9, B=16, V=20000, H=64)
    full = W.tp_full(shards)
    ref = oracle_lib.run(full)["ids"]
    d = W.to_device(shards[0])
    logits = d.pop("logits")
    d.pop("vocab_offset")
    smp = TP.VocabParallelSampler(16, full.V, 1, 0, "cuda", tp_cap=TP_CAP, two_round=True,
                                  gather=lambda recv, send: recv.copy_(send))
    out = torch.zeros(16, dtype=torch.int64, device="cuda")
    st = torch.zeros(16, dtype=torch.int32, device="cuda")
    smp.sample(logits, 0, out, out_status=st, **d)
    torch.cuda.synchronize()
    decided = (st.cpu().numpy() & N.STATUS_TP_OVERFLOW) == 0
    assert decided.all()
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("tp", [2, 4])
def test_two_round_full_size(oracle_lib, tp):
    """The two rounds at the vocab-parallel workload's full size (B=128,
    V=152064, peaked rows without top_k) with the sampler's default record
    capacity, shards emulated on one device (the exchange concatenates the
    shards' sends): every row is decided and every shard's ids equal the
    full row's oracle ids."""
    import torch

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import tp as TP

    B, V = 128, 152064
    shards = W.tp_topk_off(tp, seed=0, B=B, V=V, H=512)
    full = W.tp_full(shards)
    ref = oracle_lib.run(full)["ids"]
    devs = [W.to_device(s) for s in shards]
    logits = [d.pop("logits") for d in devs]
    offs = [d.pop("vocab_offset") for d in devs]
    smps = [TP.VocabParallelSampler(B, V, tp, q, "cuda", two_round=True, V_shard=shards[q].V,
                                    gather=lambda recv, send: None) for q in range(tp)]
    assert smps[0].tp_cap == TP.TWO_ROUND_TP_CAP
    outs = [torch.zeros(B, dtype=torch.int64, device="cuda") for _ in range(tp)]
    stats = [torch.zeros(B, dtype=torch.int32, device="cuda") for _ in range(tp)]
    # the step's kernels, shard by shard, with the two exchanges done by hand
    from mstar_rs_b200 import kernel
    for q in range(tp):
        kernel.tp_local2(logits[q], smps[q].tp_cap, smps[q].send[: B * smps[q].words], smps[q].xbuf[: B * shards[q].V],
                         vocab_offset=offs[q], **devs[q])
    recv = torch.cat([smps[q].send[: B * smps[q].words] for q in range(tp)])
    for q in range(tp):
        kernel.tp_merge1(logits[q], smps[q].tp_cap, tp, V, recv, smps[q].pend[: 2 * B], vocab_offset=offs[q],
                         out_ids=outs[q], out_status=stats[q], **devs[q])
        kernel.tp_mass(logits[q], smps[q].xbuf[: B * shards[q].V], smps[q].pend[: 2 * B], smps[q].send2[: 2 * B],
                       vocab_offset=offs[q], **devs[q])
    recv2 = torch.cat([smps[q].send2[: 2 * B] for q in range(tp)])
    for q in range(tp):
        kernel.tp_merge2(logits[q], smps[q].tp_cap, tp, V, recv, recv2, smps[q].pend[: 2 * B], vocab_offset=offs[q],
                         out_ids=outs[q], out_status=stats[q], **devs[q])
    torch.cuda.synchronize()
    for q in range(tp):
        st = stats[q].cpu().numpy()
        assert not (st & N.STATUS_TP_OVERFLOW).any(), f"shard {q}: {int(((st & N.STATUS_TP_OVERFLOW) != 0).sum())} rows"
        np.testing.assert_array_equal(outs[q].cpu().numpy(), ref, err_msg=f"ids on shard {q}")
