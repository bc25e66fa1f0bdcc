"""Failure detection on the GPU without a fault: the kernel's bounded waits.

MSTAR_FLAG_TEST_WITHHOLD leaves each CTA's last bulk copy unissued, so the
barrier it would complete never does (no bad address, no copy in flight).
Every wait on it gives up after its 2 ms limit, the row reports
MSTAR_STATUS_TIMEOUT, the launch returns, and the context stays usable."""
import numpy as np
import pytest

from tests.cases import random_case
from tests.gpu_util import assert_parity, run_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cluster", [1, 2])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_withheld_copy_times_out(oracle_lib, cluster, dtype):
    from mstar_rs_b200 import _native as N

    case = random_case(41, B=3, V=30000, dtype=dtype, penalty="hist", bias=False, mask=False, specials=False)
    g = run_gpu(case, debug=False, flags=N.FLAG_TEST_WITHHOLD, cluster_size=cluster)
    assert (g["status"] & N.STATUS_TIMEOUT).all(), g["status"]
    # the same context samples correctly right after
    o = oracle_lib.run(case)
    g = run_gpu(case, debug=False, cluster_size=cluster)
    assert not (g["status"] & N.STATUS_TIMEOUT).any()
    assert_parity(g, o, case, debug=False)
