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
