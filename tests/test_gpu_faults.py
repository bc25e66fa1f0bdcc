"""Failure detection on the GPU without a fault: the kernel's bounded waits.

Slices larger than the register tile (160 KB) are bulk-copied into shared
memory and every thread waits on the copies' mbarriers with a 2 ms bound.
MSTAR_FLAG_TEST_WITHHOLD leaves each CTA's last bulk copy unissued, so the
barrier it would complete never does (no bad address, no copy in flight).
Every wait on it gives up after its limit, the row reports
MSTAR_STATUS_TIMEOUT, the launch returns, and the context stays usable.
The cases force cluster widths whose slices (164,000 bytes) exceed the tile."""
import numpy as np
import pytest

from tests.cases import random_case
from tests.gpu_util import assert_parity, run_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,V,cluster", [("f32", 41000, 1), ("bf16", 82000, 1), ("f32", 82000, 2)])
def test_withheld_copy_times_out(oracle_lib, dtype, V, cluster):
    from mstar_rs_b200 import _native as N

    case = random_case(41, B=3, V=V, dtype=dtype, penalty="hist", bias=False, mask=False, specials=False)
    g = run_gpu(case, debug=False, flags=N.FLAG_TEST_WITHHOLD, cluster_size=cluster)
    assert (g["status"] & N.STATUS_TIMEOUT).all(), g["status"]
    # the same context samples correctly right after
    o = oracle_lib.run(case)
    g = run_gpu(case, debug=False, cluster_size=cluster)
    assert not (g["status"] & N.STATUS_TIMEOUT).any()
    assert_parity(g, o, case, debug=False)
