"""GPU parity at the full sizes of the five measured workloads."""
import numpy as np
import pytest

from tests.gpu_util import assert_parity, run_gpu

pytestmark = pytest.mark.gpu


def test_orpheus_single(oracle_lib):
    from mstar_rs_b200 import workloads

    case = workloads.orpheus_single(0)
    o = oracle_lib.run(case, debug=True)
    assert_parity(run_gpu(case), o, case)


@pytest.mark.parametrize("seed", [0, 1])
def test_qwen_mixed_batch(oracle_lib, seed):
    from mstar_rs_b200 import workloads

    case = workloads.qwen_mixed(seed)
    o = oracle_lib.run(case, debug=True)
    assert_parity(run_gpu(case), o, case)


@pytest.mark.parametrize("B", [1, 8, 32, 128, 256, 512])
def test_bucket_sweep(oracle_lib, B):
    from mstar_rs_b200 import workloads

    case = workloads.bucket_sweep(B, seed=B)
    o = oracle_lib.run(case, debug=False)
    assert_parity(run_gpu(case, debug=False, with_uniforms=False), o, case, debug=False)


def test_constrained(oracle_lib):
    from mstar_rs_b200 import workloads

    case = workloads.constrained(0, B=128)
    o = oracle_lib.run(case, debug=True)
    assert_parity(run_gpu(case), o, case)


def test_constrained_full_batch(oracle_lib):
    """All 512 rows of the constrained workload (ids and status)."""
    from mstar_rs_b200 import workloads

    case = workloads.constrained(1)
    assert case.B == 512
    o = oracle_lib.run(case, debug=False)
    assert_parity(run_gpu(case, debug=False), o, case, debug=False)


def test_tp_full_row_reference(oracle_lib):
    """The vocab-sharded workload's full row through the single-GPU path."""
    from mstar_rs_b200 import workloads

    case = workloads.tp_full(workloads.tp_sharded(4, seed=0))
    o = oracle_lib.run(case, debug=False)
    assert_parity(run_gpu(case, debug=False), o, case, debug=False)
