"""The LM-head projection entry point that allocates nothing
(mstar_lmhead_logits_static, scratch in a static device array) against
mstar_lmhead_logits with a caller workspace, called through the C ABI.

Collected last, so it runs both after every other test and alone in a fresh
process."""
import ctypes

import pytest

from mstar_rs_b200 import _native as N


def _args(hidden, weight, out):
    B, d = hidden.shape
    V = weight.shape[0]
    dt = N.DTYPE_BF16 if out.dtype.is_floating_point and out.element_size() == 2 else N.DTYPE_F32
    return (ctypes.c_void_p(hidden.data_ptr()), ctypes.c_void_p(weight.data_ptr()), B, V, d,
            ctypes.c_void_p(out.data_ptr()), dt, out.stride(0))


@pytest.mark.gpu
@pytest.mark.parametrize("B,V,d,out_dtype", [(64, 151936, 2048, "f32"), (5, 4099, 136, "f32"),
                                             (96, 50000, 1024, "bf16"), (3, 1000, 4096, "f32")])
def test_static_scratch_matches_workspace_entry(B, V, d, out_dtype):
    import torch

    L = N.lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(B + V + d)
    hidden = torch.randn(B, d, device=dev, generator=g).to(torch.bfloat16)
    weight = (torch.randn(V, d, device=dev, generator=g) * (3.0 / d ** 0.5)).to(torch.bfloat16)
    tdt = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    wsn = int(L.mstar_lmhead_workspace_bytes(B))
    ws = torch.empty(wsn, dtype=torch.uint8, device=dev)
    ref = torch.empty(B, V, dtype=tdt, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    N.check(L.mstar_lmhead_logits(*_args(hidden, weight, ref), ctypes.c_void_p(ws.data_ptr()), wsn,
                                  ctypes.c_void_p(st.data_ptr()), stream), "mstar_lmhead_logits")
    # tolerance of the projection tests: two fp32 summation orders over d terms
    bound = (hidden.float().abs() @ weight.float().abs().T) * 1e-5 + 1e-6
    if tdt == torch.bfloat16:
        bound = bound + ref.float().abs() * 2.0 ** -8  # one bf16 rounding step either way
    for _ in range(2):  # two calls in a row share the static scratch
        out = torch.full((B, V), float("nan"), dtype=tdt, device=dev)
        N.check(L.mstar_lmhead_logits_static(*_args(hidden, weight, out), ctypes.c_void_p(st.data_ptr()), stream),
                "mstar_lmhead_logits_static")
        torch.cuda.synchronize(dev)
        assert st.item() == 0
        diff = (out.float() - ref.float()).abs()
        assert bool((diff <= bound).all()), float((diff / bound).max())


def test_static_scratch_refuses_rows_past_its_size():
    """More rows than the static array's partial tiles hold (97 on a 148-SM
    GPU, the count assumed without one) are refused before any launch."""
    L = N.lib()
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: the size check comes first
    rc = L.mstar_lmhead_logits_static(fake, fake, 256, 1000, 64, fake, N.DTYPE_F32, 1000, None, None)
    assert rc == N.ERR_INVALID
    assert b"static workspace" in L.mstar_sampler_last_error()
