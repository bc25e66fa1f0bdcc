"""GPU: the tcgen05 LM-head projection against a float32 matmul of the same
bf16 operands (fp32 accumulation in both; the sums differ only in order),
and its bf16 output against its own fp32 output rounded to nearest even."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ws", ["auto", None])
@pytest.mark.parametrize("B,V,d", [(1, 1000, 64), (7, 4099, 136), (64, 151936, 2048), (33, 50000, 1024),
                                   (256, 8192, 512), (16, 128, 8), (3, 1000, 4096)])
def test_lmhead_logits_match_fp32_matmul(B, V, d, ws):
    """With the workspace every SM takes an equal share of (tile, k-block)
    units, so tiles are split over up to 19 CTAs (V=1000, d=4096) and summed
    through it; without it each CTA takes whole tiles."""
    import torch

    from mstar_rs_b200 import kernel

    g = torch.Generator(device="cuda").manual_seed(B * 7 + V + d)
    hidden = (torch.randn(B, d, device="cuda", generator=g)).to(torch.bfloat16)
    weight = (torch.randn(V, d, device="cuda", generator=g) * (3.0 / d ** 0.5)).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = kernel.lmhead_logits(hidden, weight, status=status, workspace=ws)
    ref = hidden.float() @ weight.float().T
    torch.cuda.synchronize()
    assert status.item() == 0
    # |error| of two fp32 summation orders over d terms: well below 1e-5 of the
    # sum of |terms|
    bound = (hidden.float().abs() @ weight.float().abs().T) * 1e-5 + 1e-6
    assert bool(((out - ref).abs() <= bound).all()), float(((out - ref).abs() / bound).max())
    ob = kernel.lmhead_logits(hidden, weight, dtype=torch.bfloat16, workspace=ws)
    assert torch.equal(ob, out.to(torch.bfloat16))
    again = kernel.lmhead_logits(hidden, weight, workspace=ws)  # the workspace is reused call to call
    assert torch.equal(again, out)


def test_lmhead_logits_into_a_wider_buffer():
    """Rows of an output with a leading dimension past V: only [:, :V] is
    written."""
    import torch

    from mstar_rs_b200 import kernel

    B, V, d = 5, 1000, 256
    hidden = torch.randn(B, d, device="cuda").to(torch.bfloat16)
    weight = torch.randn(V, d, device="cuda").to(torch.bfloat16)
    buf = torch.full((B, V + 24), 7.0, device="cuda")
    kernel.lmhead_logits(hidden, weight, out=buf[:, :V])
    torch.cuda.synchronize()
    assert bool((buf[:, V:] == 7.0).all())
    ref = hidden.float() @ weight.float().T
    assert torch.allclose(buf[:, :V], ref, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("B,V,d,dtype", [(64, 151936, 2048, "bf16"), (1, 156940, 3072, "f32"), (24, 32000, 512, "bf16")])
def test_lmhead_step_matches_unfused_and_oracle(oracle_lib, B, V, d, dtype):
    """Projection + sampling in one call (the mixed workload's per-row
    parameters and 1024-token histories) against the two calls made in turn,
    and the sampled ids against the oracle run on the projection's logits."""
    import numpy as np
    import torch

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import kernel
    from mstar_rs_b200 import workloads as W

    case = W.qwen_mixed(seed=5, B=B, V=V)
    case.dtype = dtype
    g = torch.Generator(device="cuda").manual_seed(11)
    hidden = torch.randn(B, d, device="cuda", generator=g).to(torch.bfloat16)
    weight = (torch.randn(V, d, device="cuda", generator=g) * (3.0 / d ** 0.5)).to(torch.bfloat16)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    kw = W.to_device(case)
    kw.pop("logits")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, V, dtype=tdt, device="cuda")
    ids = torch.zeros(B, dtype=torch.int64, device="cuda")
    status = torch.zeros(B, dtype=torch.int32, device="cuda")
    kernel.lmhead_step(hidden, weight, logits, status=st, **kw, out_ids=ids, out_status=status)
    ref = kernel.lmhead_logits(hidden, weight, dtype=tdt)
    ids2 = torch.zeros_like(ids)
    kernel.sampler_step(ref, **kw, out_ids=ids2)
    torch.cuda.synchronize()
    assert st.item() == 0
    assert torch.equal(logits, ref)
    assert torch.equal(ids, ids2)
    assert int((status & (N.STATUS_TIMEOUT | N.STATUS_BAD_RECORD)).max()) == 0
    if dtype == "bf16":
        case.logits = ref.view(torch.int16).cpu().numpy().view(np.uint16)
    else:
        case.logits = ref.cpu().numpy()
    o = oracle_lib.run(case)
    assert np.array_equal(ids.cpu().numpy(), o["ids"])
