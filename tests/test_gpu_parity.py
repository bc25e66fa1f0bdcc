"""GPU parity: the CUDA sampler through the C ABI against the oracle on the
same seeded inputs and the same pre-drawn uniforms (or Philox counters).

Token ids, kept-set membership, status and penalty-adjusted logits must be
bit-exact; probabilities within 1e-5 relative (fp32) / 2e-3 (bf16)."""
import numpy as np
import pytest

from tests.cases import feature_grid, random_case
from tests.gpu_util import assert_parity, run_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("seed,kw", feature_grid())
@pytest.mark.parametrize("cluster", [0, 1, 3])
def test_feature_grid(oracle_lib, seed, kw, cluster):
    case = random_case(seed, **kw)
    if cluster > 1 and case.V < 64 * cluster:
        pytest.skip("slice too small for this cluster size")
    o = oracle_lib.run(case, debug=True)
    g = run_gpu(case, cluster_size=cluster)
    assert_parity(g, o, case)


@pytest.mark.parametrize("seed,kw", feature_grid())
def test_general_path_matches(oracle_lib, seed, kw):
    """Force the multi-round histogram/compaction path on every row."""
    from mstar_rs_b200 import _native as N

    case = random_case(seed, **kw)
    o = oracle_lib.run(case, debug=True)
    g = run_gpu(case, flags=N.FLAG_FORCE_GENERAL, cluster_size=2 if case.V >= 128 else 1)
    assert_parity(g, o, case)


@pytest.mark.parametrize("seed", range(6))
def test_large_flat_rows(oracle_lib, seed):
    """Flat rows (top_k off, tiny min_p) whose value set exceeds the fast
    tail: exercises the per-query locate rounds with refinement."""
    case = random_case(100 + seed, B=4, V=60000, dtype=["f32", "bf16"][seed % 2], scale=0.3,
                       specials=False, greedy_frac=0.0)
    case.top_k[:] = [0, 0, 3000, 5000][: case.B]
    case.min_p[:] = 0.0
    case.top_p[:] = [0.95, 1.0, 0.7, 0.3][: case.B]
    o = oracle_lib.run(case, debug=True)
    for cl in (0, 4):
        g = run_gpu(case, cluster_size=cl)
        assert_parity(g, o, case)
        assert (g["status"] & 2).any(), "expected the general path"


@pytest.mark.parametrize("seed", range(4))
@pytest.mark.parametrize("cluster", [4, 8])
def test_cluster_topk_cut(oracle_lib, seed, cluster):
    """top_k rows whose K exceeds what one CTA may push (2048 / cluster) on
    flat rows where every id is a candidate: the CTAs cut at a value bin
    found from a histogram of all CTAs' vector maxima and specials summed in
    the leader, instead of taking the general path.  History penalties put
    specials into the histogram; odd seeds add the NaN / inf / -0 values."""
    case = random_case(400 + seed, B=6, V=60000, dtype=["f32", "bf16"][seed % 2], scale=1.0,
                       specials=bool(seed % 2), greedy_frac=0.0, mask=False)
    cap = 2048 // cluster
    case.temperature[:] = 1.0
    case.top_k[:] = [cap + 1, cap + 300, 900, 1200, 1536, cap + 60]
    case.top_p[:] = [1.0, 0.9, 0.95, 0.5, 1.0, 0.99]
    case.min_p[:] = 0.0
    o = oracle_lib.run(case, debug=True)
    g = run_gpu(case, cluster_size=cluster)
    assert_parity(g, o, case)
    if not seed % 2:  # finite rows take the cut, not the general path (a CTA holding
        # far more than its share of the cut's values may still overflow: at most one row)
        assert int(((g["status"] & 2) != 0).sum()) <= 1


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("cluster", [1, 2])
@pytest.mark.parametrize("mask", [False, True])
def test_many_seen_ids(oracle_lib, dtype, cluster, mask):
    """Seen-bit rows with far more seen ids in one slice than any fixed list
    would hold (about 12,000 and 24,000 of 40,000 ids): every seen id is
    penalised, none is dropped, and no overflow status is raised.  Bias ids
    that are also seen count once."""
    case = random_case(300 + cluster, B=4, V=40000, dtype=dtype, penalty="seen", mask=mask, specials=False,
                       seen_density=0.3 if cluster == 1 else 0.6, greedy_frac=0.0)
    case.bias_ids[:, 2] = np.flatnonzero(np.unpackbits(case.seen_bits[0].view(np.uint8), bitorder="little"))[5]
    from mstar_rs_b200 import _native as N

    o = oracle_lib.run(case, debug=True)
    for flags in (0, N.FLAG_FORCE_GENERAL):
        g = run_gpu(case, cluster_size=cluster, flags=flags)
        assert_parity(g, o, case)
        assert not (g["status"] & N.STATUS_SPECIAL_OVERFLOW).any()


def test_state_updates():
    """History append, seen-bit set and Philox offset advance happen on the
    device, exactly once per row."""
    import torch

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import kernel, workloads

    case = random_case(7, B=6, V=3000, philox=True, penalty="hist", mask=False)
    d = workloads.to_device(case)
    logits = d.pop("logits")
    out = torch.zeros(case.B, dtype=torch.int64, device="cuda")
    hist0 = d["hist_ids"].clone()
    len0 = d["hist_len"].clone()
    off0 = d["offset"].clone()
    kernel.sampler_step(logits, **d, out_ids=out,
                        flags=N.FLAG_UPDATE_HISTORY | N.FLAG_ADVANCE_OFFSET)
    torch.cuda.synchronize()
    ids = out.cpu().numpy()
    H = hist0.shape[1]
    assert torch.equal(d["offset"].cpu(), off0.cpu() + 1)
    assert torch.equal(d["hist_len"].cpu(), len0.cpu() + 1)
    h = d["hist_ids"].cpu().numpy()
    for r in range(case.B):
        pos = int(len0[r]) % H
        assert h[r, pos] == ids[r]
        rest = np.delete(h[r], pos)
        assert np.array_equal(rest, np.delete(hist0[r].cpu().numpy(), pos))


def test_seen_bits_update():
    import torch

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import kernel, workloads

    case = random_case(8, B=5, V=2000, penalty="seen", mask=False)
    d = workloads.to_device(case)
    logits = d.pop("logits")
    out = torch.zeros(case.B, dtype=torch.int64, device="cuda")
    before = d["seen_bits"].clone()
    kernel.sampler_step(logits, **d, out_ids=out, flags=N.FLAG_UPDATE_SEEN)
    torch.cuda.synchronize()
    after = d["seen_bits"].cpu().numpy().view(np.uint32)
    exp = before.cpu().numpy().view(np.uint32).copy()
    for r, t in enumerate(out.cpu().numpy()):
        exp[r, t >> 5] |= np.uint32(1) << np.uint32(t & 31)
    np.testing.assert_array_equal(after, exp)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("cluster", [0, 3])
def test_candidate_count_paths(oracle_lib, dtype, cluster):
    """Rows whose candidate set has an exact size: N ids near the top, the
    rest far below, min_p tiny.  The sizes straddle every tail variant (one
    warp with one or two candidates per lane, the block tail, the general
    path) and each row mixes top_k / top_p settings."""
    from mstar_rs_b200.workloads import Batch, f32_to_bf16_bits

    sizes = [1, 2, 31, 32, 33, 63, 64, 65, 200, 530, 2047, 2600]
    V, B = 24000, len(sizes)
    rng = np.random.default_rng(11 + cluster)
    x = np.full((B, V), -60.0, np.float32) + rng.standard_normal((B, V)).astype(np.float32)
    for r, n in enumerate(sizes):
        ids = rng.choice(V, n, replace=False)
        x[r, ids] = rng.uniform(0.0, 4.0, n).astype(np.float32)
    logits = f32_to_bf16_bits(x) if dtype == "bf16" else x
    case = Batch(logits=logits, dtype=dtype,
                 temperature=np.full(B, 0.9, np.float32),
                 top_k=np.array([0, 0, 20, 0, 50, 0, 0, 40, 0, 100, 0, 0], np.int32),
                 top_p=np.array([1.0, 0.9, 1.0, 0.8, 0.95, 1.0, 0.5, 0.99, 0.9, 0.85, 1.0, 0.97], np.float32),
                 min_p=np.full(B, 1e-6, np.float32),
                 uniforms=rng.random(B, dtype=np.float32),
                 name="candidate_counts")
    o = oracle_lib.run(case, debug=True)
    g = run_gpu(case, cluster_size=cluster)
    assert_parity(g, o, case)


@pytest.mark.parametrize("seed", range(4))
def test_general_value_bins(oracle_lib, seed):
    """General-path rows whose first histogram decides everything: top_k
    prefixes that fit the tail (placed by value bin, then ranked inside each
    bin), heavy exact ties (quantised logits: whole bins of equal values),
    and a flat row (every value in one bin: refined by id)."""
    from mstar_rs_b200 import _native as N
    from mstar_rs_b200.workloads import bucket_sweep

    case = bucket_sweep(6, seed=seed, V=40000)
    case.uniforms = np.random.default_rng(seed).random(case.B).astype(np.float32)
    case.seed = None
    case.offset = None
    case.top_k[:] = [120, 700, 1500, 1024, 65, 300]
    if seed % 2:
        x = case.logits_f32()
        x = (np.round(x * 1.0) / 1.0).astype(np.float32)  # integer logits: many exact ties
        x[5, :] = 1.5  # a flat row
        case.logits = x
    o = oracle_lib.run(case, debug=True)
    for cl in (0, 4):
        g = run_gpu(case, cluster_size=cl)
        assert_parity(g, o, case)
        g = run_gpu(case, cluster_size=cl, flags=N.FLAG_FORCE_GENERAL)
        assert_parity(g, o, case)


@pytest.mark.parametrize("B,V,K,P,dtype", [(1, 4096, 0, 1.0, "bf16"), (16, 4096, 0, 1.0, "f32"), (1, 2048, 50, 0.9, "bf16"),
                                            (8, 3072, 0, 0.8, "f32"), (4, 4096, 1, 1.0, "bf16")])
def test_small_vocab_rows(oracle_lib, B, V, K, P, dtype):
    """Talker-shaped rows (a codec vocabulary of at most 4096 ids: one CTA
    per row; temperature 1, repetition 1.1 over seen ids, top_k off and
    top_p 1 by default, so every id is a candidate) against the oracle, with
    history and seen-bit penalties, bias and a mask."""
    for penalty in ("seen", "hist"):
        case = random_case(400 + B + V, B=B, V=V, dtype=dtype, penalty=penalty, specials=False, greedy_frac=0.0,
                           scale=1.0)
        case.temperature[:] = 1.0
        case.top_k[:] = K
        case.top_p[:] = P
        case.min_p[:] = 0.0
        case.rep_pen[:] = 1.1
        o = oracle_lib.run(case, debug=True)
        g = run_gpu(case)
        assert_parity(g, o, case)


@pytest.mark.parametrize("K,dtype", [(0, "f32"), (20, "bf16"), (0, "bf16")])
def test_small_vocab_ties(oracle_lib, K, dtype):
    """Small rows whose logits take a dozen distinct values (long runs of
    exact ties, ordered by id): the value buckets overflow and the kernel
    sorts by order key instead."""
    from mstar_rs_b200.workloads import f32_to_bf16_bits

    case = random_case(77 + K, B=4, V=4096, dtype="f32", penalty="seen", specials=False, greedy_frac=0.0, scale=1.0)
    q = (np.round(case.logits * 2.0) / 2.0).astype(np.float32)
    case.logits = f32_to_bf16_bits(q) if dtype == "bf16" else q
    case.dtype = dtype
    case.temperature[:] = 1.0
    case.top_k[:] = K
    case.top_p[:] = 0.95
    case.min_p[:] = 0.0
    o = oracle_lib.run(case, debug=True)
    g = run_gpu(case)
    assert_parity(g, o, case)


def test_multi_head_step(oracle_lib):
    """Four codebook heads of three requests in one launch ([H, n, V] with a
    slot per (head, request), each slot with its own seen ids), against the
    oracle on the flattened rows."""
    import torch

    from mstar_rs_b200 import kernel
    from mstar_rs_b200.workloads import to_device

    H, n, V = 4, 3, 2048
    case = random_case(91, B=H * n, V=V, dtype="bf16", penalty="seen", specials=False, greedy_frac=0.0, scale=1.0)
    case.top_k[:] = 0
    case.top_p[:] = 1.0
    case.min_p[:] = 0.0
    o = oracle_lib.run(case)
    d = to_device(case)
    logits = d.pop("logits").reshape(H, n, V)
    ids = torch.zeros(H * n, dtype=torch.int64, device="cuda")
    kernel.sampler_step_heads(logits, **d, out_ids=ids)
    assert np.array_equal(ids.cpu().numpy(), o["ids"])
