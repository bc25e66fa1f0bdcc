"""CPU: the C oracle against the independent numpy restatement, Philox
known-answer vectors and the spec's exponential."""
import ctypes

import numpy as np
import pytest

from tests.cases import feature_grid, random_case


def _cmp(a, b, name):
    np.testing.assert_array_equal(a["ids"], b["ids"], err_msg=f"{name}: ids")
    np.testing.assert_array_equal(a["status"], b["status"], err_msg=f"{name}: status")
    np.testing.assert_array_equal(a["kept"], b["kept"], err_msg=f"{name}: kept")
    xa, xb = a["x"], b["x"]
    np.testing.assert_array_equal(np.isnan(xa), np.isnan(xb), err_msg=f"{name}: x NaN pattern")
    np.testing.assert_array_equal(np.where(np.isnan(xa), 0, xa).view(np.uint32),
                                  np.where(np.isnan(xb), 0, xb).view(np.uint32), err_msg=f"{name}: x bits")
    np.testing.assert_array_equal(a["probs"].view(np.uint32), b["probs"].view(np.uint32), err_msg=f"{name}: probs")


@pytest.mark.parametrize("seed,kw", feature_grid())
def test_c_oracle_matches_numpy_restatement(oracle_lib, seed, kw):
    case = random_case(seed, **kw)
    c = oracle_lib.run(case, debug=True, threads=2)
    n = oracle_lib.run_np(case)
    _cmp(c, n, case.name)


def test_philox_known_answers(oracle_lib):
    """Random123's published Philox4x32-10 test vectors."""
    from oracle import spec_np

    L = oracle_lib.lib()
    L.orc_philox4x32_10.argtypes = [ctypes.POINTER(ctypes.c_uint32)] * 3
    kat = [
        ([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
        ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2, [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
        ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
         [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]),
    ]
    for ctr, key, want in kat:
        c = (ctypes.c_uint32 * 4)(*ctr)
        k = (ctypes.c_uint32 * 2)(*key)
        o = (ctypes.c_uint32 * 4)()
        L.orc_philox4x32_10(c, k, o)
        assert list(o) == want
        assert spec_np.philox4x32_10(ctr, key) == want


def test_exp_spec_properties(oracle_lib):
    from oracle import spec_np

    L = oracle_lib.lib()
    assert L.orc_exp_spec(0.0) == 1.0
    assert L.orc_exp_spec(-0.0) == 1.0
    assert L.orc_exp_spec(float("-inf")) == 0.0
    rng = np.random.default_rng(0)
    y = -np.abs(rng.standard_normal(20000).astype(np.float32) * 15)
    y = np.sort(y)
    e_np = spec_np.exp_spec(y)
    e_c = np.array([L.orc_exp_spec(float(v)) for v in y[::97]], np.float32)
    np.testing.assert_array_equal(e_np[::97], e_c)
    assert np.all(np.diff(e_np) >= 0), "E must be monotone"
    ref = np.exp(y.astype(np.float64))
    live = y > -44.0  # E is defined as 0 once y*log2(e) < -64
    rel = np.abs(e_np[live] - ref[live]) / ref[live]
    assert rel.max() < 3e-6


def test_oracle_threads_deterministic(oracle_lib):
    case = random_case(99, B=16, V=4000, dtype="bf16")
    a = oracle_lib.run(case, debug=True, threads=1)
    b = oracle_lib.run(case, debug=True, threads=4)
    _cmp(a, b, "threads")


def test_oracle_statistics_small(oracle_lib):
    """Inverse-CDF draw over a grid of uniforms reproduces the kept-set
    probabilities (the draw is exact up to the uniform grid)."""
    from mstar_rs_b200.workloads import Batch

    V = 50
    rng = np.random.default_rng(3)
    row = (rng.standard_normal(V) * 1.5).astype(np.float32)
    n = 20000
    u = ((np.arange(n) + 0.5) / n).astype(np.float32)
    b = Batch(logits=np.tile(row, (n, 1)), temperature=np.full(n, 0.9, np.float32),
              top_p=np.full(n, 0.8, np.float32), top_k=np.full(n, 30, np.int32), uniforms=u)
    res = oracle_lib.run(b, debug=True)
    counts = np.bincount(res["ids"], minlength=V) / n
    np.testing.assert_allclose(counts, res["probs"][0], atol=2.0 / n)


def test_stop_hits():
    from oracle import oracle

    ids = [5, 7, 0, 9]
    st = [[5, -1], [-1, -1], [3, 0], [8, 10]]
    assert oracle.stop_hits(ids, st).tolist() == [True, False, True, False]
