"""GPU: the drop-in Python interface (mstar_rs_b200.sampling) against the
oracle, eager and replayed from a captured CUDA graph the way the Orpheus
engine captures its batched decode step (orpheus.py:322-366, :394-431)."""
import numpy as np
import pytest

from mstar_rs_b200.workloads import Batch, pack_bits

pytestmark = pytest.mark.gpu


def _cfg_rows(rng, n):
    return dict(temperature=rng.uniform(0.3, 1.4, n).astype(np.float32),
                top_k=rng.choice(np.array([0, 5, 40], np.int32), n),
                top_p=rng.uniform(0.6, 1.0, n).astype(np.float32),
                min_p=rng.choice(np.array([0.0, 0.02], np.float32), n),
                rep_pen=rng.uniform(1.0, 1.4, n).astype(np.float32),
                pres_pen=rng.uniform(0, 0.5, n).astype(np.float32),
                freq_pen=rng.uniform(0, 0.5, n).astype(np.float32))


def test_eager_sampler_matches_oracle(oracle_lib):
    import torch

    from mstar_rs_b200 import sampling

    rng = np.random.default_rng(5)
    n, V, H = 6, 5003, 32
    cfg = _cfg_rows(rng, n)
    seeds = rng.integers(0, 2**62, n).astype(np.uint64)
    hist = rng.integers(0, V, (n, H)).astype(np.int32)
    smp = sampling.Sampler(device="cuda", history=H)
    rids = [f"q{i}" for i in range(n)]
    for i, r in enumerate(rids):
        smp.add_request(r)
        smp.set_config(r, vocab_size=V, temperature=float(cfg["temperature"][i]), top_k=int(cfg["top_k"][i]),
                       top_p=float(cfg["top_p"][i]), min_p=float(cfg["min_p"][i]),
                       repetition_penalty=float(cfg["rep_pen"][i]),
                       presence_penalty=float(cfg["pres_pen"][i]), frequency_penalty=float(cfg["freq_pen"][i]))
        smp._sampling_config[r].set_seed(int(seeds[i]))
        smp.set_history(r, hist[i].tolist())
    hist_now = [list(h) for h in hist]
    for step in range(3):
        x = (rng.standard_normal((n, V)) * 2).astype(np.float32)
        order = rng.permutation(n)
        tok = smp.sample([rids[i] for i in order], torch.from_numpy(x[order]).cuda()).cpu().numpy()
        case = Batch(logits=x[order], temperature=cfg["temperature"][order], top_k=cfg["top_k"][order],
                     top_p=cfg["top_p"][order], min_p=cfg["min_p"][order], rep_pen=cfg["rep_pen"][order],
                     pres_pen=cfg["pres_pen"][order], freq_pen=cfg["freq_pen"][order],
                     hist_ids=np.array([hist_now[i][-H:] + [-1] * (H - len(hist_now[i][-H:])) for i in order],
                                       np.int32),
                     hist_len=np.array([min(len(hist_now[i]), H) for i in order], np.int32),
                     seed=seeds[order], offset=np.full(n, step, np.uint64))
        ref = oracle_lib.run(case)["ids"]
        np.testing.assert_array_equal(tok, ref, err_msg=f"step {step}")
        for j, i in enumerate(order):
            hist_now[i].append(int(tok[j]))


def test_graph_replay_matches_oracle(oracle_lib):
    """SamplerBuffers + CudaGraphableSampler captured in a CUDA graph; the
    per-row RNG offsets and seen bits advance in-graph across replays."""
    import torch

    from mstar_rs_b200 import sampling

    rng = np.random.default_rng(9)
    n, V = 4, 3001
    cfg = _cfg_rows(rng, n)
    seeds = rng.integers(0, 2**62, n).astype(np.uint64)
    sbuf = sampling.SamplerBuffers.allocate(8, "cuda", vocab_size=V)
    rids = [str(i) for i in range(n)]
    masks = []
    for i, r in enumerate(rids):
        c = sampling.SamplingConfig(vocab_size=V, temperature=float(cfg["temperature"][i]),
                                    top_k=int(cfg["top_k"][i]), top_p=float(cfg["top_p"][i]),
                                    min_p=float(cfg["min_p"][i]), repetition_penalty=float(cfg["rep_pen"][i]),
                                    presence_penalty=float(cfg["pres_pen"][i]),
                                    frequency_penalty=float(cfg["freq_pen"][i]))
        c.set_seed(int(seeds[i]))
        sbuf.register_request(r, c)
        m = sampling.SeenTokenMask.new(r, V, "cuda")
        m.add_tokens(torch.tensor(rng.integers(0, V, 5), device="cuda"))
        masks.append(m)
    g_logits = torch.zeros(n, V, device="cuda")
    g_out = torch.zeros(n, dtype=torch.int64, device="cuda")
    sbuf.stage_seen_token_masks(rids, masks)
    sampler = sbuf.gather_for_request_ids(rids, n, gather_seen_tokens=True)

    def dec():
        g_out.copy_(sampler.sample(rids, g_logits, apply_penalty=True))

    saved_off = sbuf.offset_buf[:n].clone()
    saved_seen = sbuf.seen_tokens.buf[:n].clone()
    torch.cuda.synchronize()
    for _ in range(2):
        dec()
    sbuf.offset_buf[:n].copy_(saved_off)
    sbuf.seen_tokens.buf[:n].copy_(saved_seen)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec()
    torch.cuda.synchronize()

    seen_host = [m.to_bool().cpu().numpy() for m in masks]
    for step in range(4):
        x = (rng.standard_normal((n, V)) * 2).astype(np.float32)
        g_logits.copy_(torch.from_numpy(x))
        graph.replay()
        tok = g_out.cpu().numpy()
        case = Batch(logits=x, **{k: v for k, v in cfg.items()}, seen_bits=pack_bits(np.stack(seen_host)),
                     seed=seeds, offset=np.full(n, step, np.uint64))
        ref = oracle_lib.run(case)["ids"]
        np.testing.assert_array_equal(tok, ref, err_msg=f"replay {step}")
        for i in range(n):
            seen_host[i][tok[i]] = True
    sampler.sync_seen_token_masks(masks)
    for i in range(n):
        np.testing.assert_array_equal(masks[i].to_bool().cpu().numpy(), seen_host[i])


def test_graph_buckets_match_oracle(oracle_lib):
    """Batches of 3, 1 and 6 requests through buckets (1, 2, 4, 8): pad rows
    are skipped, real rows match the oracle, RNG offsets advance per step."""
    import torch

    from mstar_rs_b200 import sampling

    rng = np.random.default_rng(21)
    V = 4099
    sbuf = sampling.SamplerBuffers.allocate(8, "cuda", vocab_size=V)
    cfg = _cfg_rows(rng, 8)
    seeds = rng.integers(0, 2**62, 8).astype(np.uint64)
    rids = [f"b{i}" for i in range(8)]
    cfgs = {}
    for i, r in enumerate(rids):
        c = sampling.SamplingConfig(vocab_size=V, temperature=float(cfg["temperature"][i]),
                                    top_k=int(cfg["top_k"][i]), top_p=float(cfg["top_p"][i]),
                                    min_p=float(cfg["min_p"][i]))
        c.set_seed(int(seeds[i]))
        sbuf.register_request(r, c)
        cfgs[r] = c
    gb = sampling.SamplerGraphBuckets(sbuf, buckets=(1, 2, 4, 8), dtype=torch.float32)
    gb.capture()
    step = {r: 0 for r in rids}
    for batch in ([0, 3, 5], [2], [1, 4, 6, 7, 0, 3]):
        rb = [rids[i] for i in batch]
        x = (rng.standard_normal((len(batch), V)) * 2).astype(np.float32)
        case = Batch(logits=x, temperature=cfg["temperature"][batch], top_k=cfg["top_k"][batch],
                     top_p=cfg["top_p"][batch], min_p=cfg["min_p"][batch], seed=seeds[batch],
                     offset=np.array([step[r] for r in rb], np.uint64))
        ref = oracle_lib.run(case)["ids"]
        # stop ids: rows at even positions stop on the id they will sample
        for j, r in enumerate(rb):
            cfgs[r].stop_token_ids = [int(ref[j]) if j % 2 == 0 else int((ref[j] + 1) % V)]
        tok = gb.sample(rb, torch.from_numpy(x).cuda()).cpu().numpy()
        gb.sync(rb)
        np.testing.assert_array_equal(tok, ref, err_msg=f"batch {batch}")
        assert gb.stopped(rb) == rb[::2], f"batch {batch}"
        for r in rb:
            step[r] += 1


def test_stop_flags(oracle_lib):
    """Stop tokens flagged on the device: the step's status bit, the eager
    Sampler's per-request flags and the captured step's per-row flags all
    equal the engines' host-side test (sampled id == a stop id) applied to
    the oracle's ids; ignore_eos requests are never flagged."""
    import torch

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import kernel, sampling
    from oracle.oracle import stop_hits

    rng = np.random.default_rng(33)
    n, V = 5, 3001
    cfg = _cfg_rows(rng, n)
    for k in ("rep_pen",):
        cfg[k] = np.ones(n, np.float32)
    for k in ("pres_pen", "freq_pen"):
        cfg[k] = np.zeros(n, np.float32)
    seeds = rng.integers(0, 2**62, n).astype(np.uint64)
    xs = [(rng.standard_normal((n, V)) * 2).astype(np.float32) for _ in range(2)]
    refs = [oracle_lib.run(Batch(logits=xs[s], **cfg, seed=seeds, offset=np.full(n, s, np.uint64)))["ids"]
            for s in range(2)]
    r0 = refs[0]
    # row 0 hits, row 1 hits but ignores EOS, row 2 misses, row 3 hits on its
    # second stop id, row 4 has none
    stops = [[int(r0[0])], [int(r0[1])], [int((r0[2] + 1) % V)], [int((r0[3] + 7) % V), int(r0[3])], None]
    ignore = [False, True, False, False, False]
    table = np.full((n, 4), -1, np.int64)
    for i, s in enumerate(stops):
        if s and not ignore[i]:
            table[i, : len(s)] = s

    def config(i):
        c = sampling.SamplingConfig(vocab_size=V, temperature=float(cfg["temperature"][i]),
                                    top_k=int(cfg["top_k"][i]), top_p=float(cfg["top_p"][i]),
                                    min_p=float(cfg["min_p"][i]), stop_token_ids=stops[i], ignore_eos=ignore[i])
        c.set_seed(int(seeds[i]))
        return c

    # C ABI: the status bit
    dev_x = torch.from_numpy(xs[0]).cuda()
    t = {k: torch.from_numpy(v).cuda() for k, v in cfg.items()}
    st = torch.zeros(n, dtype=torch.int32, device="cuda")
    ids = torch.zeros(n, dtype=torch.int64, device="cuda")
    flags = torch.zeros(n, dtype=torch.int32, device="cuda")
    kernel.sampler_step(dev_x, **t, seed=torch.from_numpy(seeds.view(np.int64)).cuda(),
                        offset=torch.zeros(n, dtype=torch.int64, device="cuda"),
                        stop_ids=torch.from_numpy(table.astype(np.int32)).cuda(), stop_flags=flags,
                        out_ids=ids, out_status=st)
    np.testing.assert_array_equal(ids.cpu().numpy(), r0)
    hit = stop_hits(r0, table)
    assert hit.tolist() == [True, False, False, True, False]
    np.testing.assert_array_equal((st.cpu().numpy() & N.STATUS_STOP) != 0, hit)
    np.testing.assert_array_equal(flags.cpu().numpy(), hit.astype(np.int32))

    # eager Sampler
    smp = sampling.Sampler(device="cuda", history=16)
    rids = [f"s{i}" for i in range(n)]
    for i, r in enumerate(rids):
        smp.add_request(r)
        c = config(i)
        smp.set_config(r, **{k: getattr(c, k) for k in ("vocab_size", "temperature", "top_k", "top_p", "min_p",
                                                         "stop_token_ids", "ignore_eos")})
        smp._sampling_config[r].set_seed(int(seeds[i]))
    tok = smp.sample(rids, dev_x, apply_penalty=False).cpu().numpy()
    np.testing.assert_array_equal(tok, r0)
    assert smp.stopped(rids) == [r for r, h in zip(rids, hit) if h]
    assert smp.stopped(rids) == []

    # captured step: per-row flags stay set across replays until read
    sbuf = sampling.SamplerBuffers.allocate(8, "cuda", vocab_size=V)
    for i, r in enumerate(rids):
        sbuf.register_request(r, config(i))
    g_logits = torch.zeros(n, V, device="cuda")
    sampler = sbuf.gather_for_request_ids(rids, n, gather_seen_tokens=False)
    out = torch.zeros(n, dtype=torch.int64, device="cuda")

    def dec():
        out.copy_(sampler.sample(rids, g_logits, apply_penalty=True))

    saved_off = sbuf.offset_buf[:n].clone()
    torch.cuda.synchronize()
    dec()
    sbuf.offset_buf[:n].copy_(saved_off)
    sbuf.seen_tokens.buf.zero_()
    sbuf.stop_flags.zero_()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec()
    torch.cuda.synchronize()
    seen = np.zeros(n, bool)
    for s in range(2):
        g_logits.copy_(torch.from_numpy(xs[s]))
        graph.replay()
        np.testing.assert_array_equal(out.cpu().numpy(), refs[s], err_msg=f"replay {s}")
        seen |= stop_hits(refs[s], table)
    assert sampler.stopped() == [r for r, h in zip(rids, seen) if h]
    assert sampler.stopped() == []


def test_captured_step_has_no_host_sync():
    """An Orpheus-shaped decode step (static hidden states -> LM head ->
    in-graph sampler) captured once and replayed 100 times with the
    engine's stage / gather / sync around every replay, under
    torch.cuda.set_sync_debug_mode("error"): no call on the path waits for
    the device, including the steps where a request leaves and another
    takes its row.  Every request's RNG offset then equals its step count."""
    import torch

    from mstar_rs_b200 import sampling

    n, V, d = 8, 4099, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    W = torch.randn(V, d, device="cuda", generator=g).to(torch.bfloat16)
    hidden = torch.zeros(n, d, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(n, dtype=torch.int64, device="cuda")
    sbuf = sampling.SamplerBuffers.allocate(n, "cuda", vocab_size=V)
    pool = [f"q{i}" for i in range(n + 6)]
    masks, steps = {}, {}

    def admit(rid):
        c = sampling.SamplingConfig(vocab_size=V, temperature=0.9, top_p=0.9, repetition_penalty=1.3)
        c.set_seed(hash(rid) & 0xFFFF)
        sbuf.register_request(rid, c)
        masks[rid] = sampling.SeenTokenMask.new(rid, V, "cuda")
        steps[rid] = 0

    rids = pool[:n]
    for r in rids:
        admit(r)
    sbuf.stage_seen_token_masks(rids, [masks[r] for r in rids])
    sampler = sbuf.gather_for_request_ids(rids, n, gather_seen_tokens=True)

    def dec():
        logits = hidden @ W.t()  # [n, V], the LM head
        out.copy_(sampler.sample(rids, logits, apply_penalty=True))

    saved_off = sbuf.offset_buf[:n].clone()
    saved_seen = sbuf.seen_tokens.buf[:n].clone()
    torch.cuda.synchronize()
    for _ in range(2):
        dec()
    sbuf.offset_buf[:n].copy_(saved_off)
    sbuf.seen_tokens.buf[:n].copy_(saved_seen)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec()
    torch.cuda.synchronize()
    waiting = pool[n:]
    torch.cuda.set_sync_debug_mode("error")
    try:
        for step in range(100):
            if step % 17 == 16 and waiting:  # a request leaves, another takes its row
                j = step % n
                gone = rids[j]
                sbuf.unregister_request(gone)
                rids[j] = waiting.pop(0)
                admit(rids[j])
            hidden.normal_(generator=g)
            cur = [masks[r] for r in rids]
            sbuf.stage_seen_token_masks(rids, cur)
            sbuf.gather_for_request_ids(rids, n, gather_seen_tokens=True)
            graph.replay()
            sampler.sync_seen_token_masks(cur)
            for r in rids:
                steps[r] += 1
    finally:
        torch.cuda.set_sync_debug_mode(0)
    torch.cuda.synchronize()
    off = sbuf.offset_buf[:n].cpu().tolist()
    assert off == [steps[r] for r in rids]
    tok = out.cpu().numpy()
    assert ((tok >= 0) & (tok < V)).all()
    for j, r in enumerate(rids):  # the last sampled id is in its request's seen mask
        assert bool(masks[r].to_bool()[int(tok[j])])


def test_tp_group_commit():
    """Under a tensor-parallel group the sampled ids are replaced by rank
    0's (here a stand-in group whose broadcast writes fixed ids) before the
    per-slot state takes them: history, seen bits and stop flags follow the
    broadcast ids, not the locally sampled ones."""
    import torch

    from mstar_rs_b200 import sampling

    n, V = 4, 3001
    forced = torch.tensor([5, 17, 2999, 1234], dtype=torch.int64, device="cuda")

    class Group:
        world_size = 2

        def broadcast(self, t, src):
            t.copy_(forced)

    # eager Sampler (history ring)
    smp = sampling.Sampler(device="cuda", tp_group=Group(), history=8)
    rids = [f"t{i}" for i in range(n)]
    for i, r in enumerate(rids):
        smp.add_request(r)
        smp.set_config(r, temperature=1.0, stop_token_ids=[int(forced[i])] if i % 2 == 0 else [3])
    x = torch.randn(n, V, device="cuda")
    tok = smp.sample(rids, x)
    assert tok.tolist() == forced.tolist()
    idx = [smp._slot[r] for r in rids]
    assert smp.hist[idx, 0].tolist() == forced.tolist()
    assert smp.hist_len[idx].tolist() == [1] * n
    assert smp.offset[idx].tolist() == [1] * n
    assert smp.stopped(rids) == rids[::2]
    # SamplerBuffers (seen bits)
    sbuf = sampling.SamplerBuffers(n, "cuda", tp_group=Group(), vocab_size=V)
    for r in rids:
        sbuf.register_request(r, sampling.SamplingConfig(vocab_size=V, temperature=1.0))
    masks = [sampling.SeenTokenMask.new(r, V, "cuda") for r in rids]
    sbuf.stage_seen_token_masks(rids, masks)
    s = sbuf.gather_for_request_ids(rids, n)
    tok = s.sample(rids, x)
    assert tok.tolist() == forced.tolist()
    s.sync_seen_token_masks(masks)
    for m, t in zip(masks, forced.tolist()):
        b = m.to_bool()
        assert bool(b[t]) and int(b.sum()) == 1
    assert sbuf.offset_buf[:n].tolist() == [1] * n
