"""CPU: the C-ABI library builds, loads without a GPU, exports every symbol
include/mstar_sampler.h declares, matches the ctypes struct layout, and
rejects invalid arguments on the host before any launch."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mstar_sampler.h")


@pytest.fixture(scope="module")
def L():
    from mstar_rs_b200 import _native, build

    build.build()
    return _native.lib()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mstar_\w+)\s*\(", text)))


def test_exports_every_declared_symbol(L):
    names = declared_functions()
    assert len(names) >= 8
    for n in names:
        assert hasattr(L, n), f"library does not export {n}"
    from mstar_rs_b200 import _native

    assert set(_native.EXPORTS) == set(names)


def test_abi_version(L):
    from mstar_rs_b200 import _native

    assert L.mstar_sampler_abi_version() == _native.ABI_VERSION == 2


def test_struct_layout_matches_header():
    from mstar_rs_b200._native import Params

    fields = [f[0] for f in Params._fields_]
    src = ["#include <stdio.h>", "#include <stddef.h>", '#include "mstar_sampler.h"', "int main(void){",
           'printf("%zu\\n", sizeof(mstar_sampler_params_t));']
    for f in fields:
        src.append(f'printf("%zu\\n", offsetof(mstar_sampler_params_t, {f}));')
    src.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write("\n".join(src))
        exe = os.path.join(d, "t")
        subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), "-o", exe, c])
        out = [int(v) for v in subprocess.check_output([exe]).split()]
    assert out[0] == ctypes.sizeof(Params)
    for f, off in zip(fields, out[1:]):
        assert getattr(Params, f).offset == off, f


def test_host_philox_matches_oracle(L, oracle_lib):
    from mstar_rs_b200 import _native

    ol = oracle_lib.lib()
    for seed, off in [(0, 0), (1, 2), (2**63 + 5, 2**40 + 3), (123456789, 987654321)]:
        assert _native.philox_uniform(seed, off) == ol.orc_philox_uniform(seed, off)


def test_invalid_arguments_rejected_on_host(L):
    from mstar_rs_b200 import _native

    p = _native.Params()
    assert L.mstar_sampler_step(ctypes.byref(p), None) == _native.ERR_INVALID
    assert b"logits" in L.mstar_sampler_last_error()
    p.logits = 0x1000
    p.dtype = 7
    assert L.mstar_sampler_step(ctypes.byref(p), None) == _native.ERR_INVALID
    p.dtype, p.B, p.V, p.ld, p.num_slots = 0, 4, 100, 50, 4
    assert L.mstar_sampler_step(ctypes.byref(p), None) == _native.ERR_INVALID
    assert b"ld" in L.mstar_sampler_last_error()
    p.ld = 100
    assert L.mstar_sampler_step(ctypes.byref(p), None) == _native.ERR_INVALID  # no uniforms / seed
    assert L.mstar_sampler_tp_record_words(50) == 104


def test_stop_arguments_rejected_on_host(L):
    from mstar_rs_b200 import _native

    p = _native.Params()
    p.logits, p.dtype, p.B, p.V, p.ld, p.num_slots = 0x1000, 0, 4, 100, 100, 4
    p.uniforms, p.out_ids = 0x2000, 0x3000
    p.stop_flags = 0x4000  # flags without ids
    assert L.mstar_sampler_step(ctypes.byref(p), None) == _native.ERR_INVALID
    assert b"stop_flags" in L.mstar_sampler_last_error()
    p.stop_ids, p.NS = 0x5000, 0
    assert L.mstar_sampler_step(ctypes.byref(p), None) == _native.ERR_INVALID
    assert b"NS" in L.mstar_sampler_last_error()


def test_stop_ids_in_the_parameter_table():
    """SamplingConfig.stop_token_ids fill the per-slot stop table (-1 =
    unused); ignore_eos clears them; more than the table holds is refused."""
    import numpy as np

    from mstar_rs_b200 import sampling

    t = sampling._ParamTable(3, "cpu")
    t.write(0, sampling.SamplingConfig(stop_token_ids=[7, 9]))
    t.write(1, sampling.SamplingConfig(stop_token_ids=7, ignore_eos=True))
    t.write(2, sampling.SamplingConfig(stop_token_ids=11))
    np.testing.assert_array_equal(t.host_stop, [[7, 9, -1, -1], [-1] * 4, [11, -1, -1, -1]])
    t.write(2, sampling.SamplingConfig())
    np.testing.assert_array_equal(t.host_stop[2], [-1] * 4)
    t.upload()
    assert t.kwargs()["stop_ids"].tolist() == t.host_stop.tolist()
    with pytest.raises(ValueError):
        t.write(0, sampling.SamplingConfig(temperature=0.5, stop_token_ids=[1, 2, 3, 4, 5]))
    assert t.host["temperature"][0] == 1.0  # a refused config changes nothing
    with pytest.raises(ValueError):
        t.write(0, sampling.SamplingConfig(stop_token_ids=[-3]))


def test_python_front_end_rejects_cpu_tensors():
    import torch

    from mstar_rs_b200 import kernel

    with pytest.raises(ValueError, match="CUDA"):
        kernel.build_params(torch.zeros(2, 10))


def _plan(L, B, V, dtype, H=0, cluster_size=0):
    from mstar_rs_b200 import _native

    p = _native.Params()
    p.logits, p.dtype, p.B, p.V, p.ld, p.num_slots = 0x1000, dtype, B, V, V, B
    p.uniforms, p.out_ids = 0x2000, 0x3000  # never dereferenced by the planner
    if H:
        p.hist_ids, p.hist_len, p.H = 0x4000, 0x5000, H
    p.cluster_size = cluster_size
    cs, sm = _native.I32(), _native.I64()
    rc = L.mstar_sampler_plan(ctypes.byref(p), ctypes.byref(cs), ctypes.byref(sm))
    return rc, cs.value, sm.value


def test_planner_cluster_widths(L):
    """The launch planner (no GPU needed): single-wave grids widen each row's
    cluster while SMs would sit idle; a grid of several waves keeps a width
    that holds the row; an explicit width is honoured or refused."""
    from mstar_rs_b200 import _native

    optin = 227 * 1024
    # headline: 64 bf16 rows of 151936 with 1024-token histories -> pairs (128 CTAs)
    assert _plan(L, 64, 151936, _native.DTYPE_BF16, H=1024) == (0, 2, 223104)
    # one f32 row (Orpheus) and eight (bucket of 8): eight CTAs per row
    rc, s, smem = _plan(L, 1, 156940, _native.DTYPE_F32, H=256)
    assert (rc, s) == (0, 8) and smem <= optin
    rc, s, smem = _plan(L, 8, 128256, _native.DTYPE_F32)
    assert (rc, s) == (0, 8) and smem <= optin
    # 128 f32 rows: more than one wave; the narrowest width whose slices fit
    # the register tile (160 KB) is 4, the narrowest that fits shared memory 3
    rc, s, smem = _plan(L, 128, 128256, _native.DTYPE_F32)
    assert rc == 0 and 4 <= s <= 8 and smem <= optin
    assert _plan(L, 128, 128256, _native.DTYPE_F32, cluster_size=3) == (0, 3, 229888)
    # a whole f32 row does not fit one CTA; widths above 16 are invalid
    assert _plan(L, 8, 128256, _native.DTYPE_F32, cluster_size=1)[0] == _native.ERR_UNSUPPORTED
    assert _plan(L, 8, 128256, _native.DTYPE_F32, cluster_size=17)[0] == _native.ERR_INVALID
