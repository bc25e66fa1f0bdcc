"""GPU: the sampled distribution over 1e6 Philox draws against the oracle's
normalised kept distribution (chi-square goodness of fit)."""
import numpy as np
import pytest

from mstar_rs_b200.workloads import Batch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_chi_square_1e6_draws(oracle_lib, dtype):
    import torch
    from scipy import stats

    from mstar_rs_b200 import kernel
    from mstar_rs_b200.workloads import f32_to_bf16_bits

    rng = np.random.default_rng(17)
    V = 96
    row = (rng.standard_normal(V) * 1.5).astype(np.float32)
    params = dict(temperature=0.8, top_k=40, top_p=0.95, min_p=0.01)
    one = Batch(logits=(f32_to_bf16_bits(row[None]) if dtype == "bf16" else row[None]), dtype=dtype,
                temperature=np.array([params["temperature"]], np.float32),
                top_k=np.array([params["top_k"]], np.int32), top_p=np.array([params["top_p"]], np.float32),
                min_p=np.array([params["min_p"]], np.float32), uniforms=np.array([0.5], np.float32))
    probs = oracle_lib.run(one, debug=True)["probs"][0].astype(np.float64)
    kept = np.nonzero(probs > 0)[0]
    assert kept.size > 5

    B, launches = 65535, 16  # 1,048,560 draws (B is at most 65535)
    src = torch.from_numpy(one.logits.view(np.int16) if dtype == "bf16" else one.logits).cuda()
    logits = src.repeat(B, 1)
    if dtype == "bf16":
        logits = logits.view(torch.bfloat16)
    dev = logits.device
    full = lambda v, dt: torch.full((B,), v, dtype=dt, device=dev)  # noqa: E731
    seed = full(0x5EED, torch.int64)
    offset = torch.arange(B, dtype=torch.int64, device=dev)
    out = torch.zeros(B, dtype=torch.int64, device=dev)
    counts = torch.zeros(V, dtype=torch.int64, device=dev)
    for _ in range(launches):
        kernel.sampler_step(logits, temperature=full(params["temperature"], torch.float32),
                            top_k=full(params["top_k"], torch.int32), top_p=full(params["top_p"], torch.float32),
                            min_p=full(params["min_p"], torch.float32), seed=seed, offset=offset, out_ids=out)
        counts += torch.bincount(out, minlength=V)
        offset += B
    counts = counts.cpu().numpy()
    n = B * launches
    assert counts.sum() == n
    assert counts[probs == 0].sum() == 0, "a token outside the kept set was drawn"
    expected = probs[kept] * n
    chi2 = float(((counts[kept] - expected) ** 2 / expected).sum())
    p = float(stats.chi2.sf(chi2, df=kept.size - 1))
    assert p > 1e-3, f"chi2={chi2:.1f} over {kept.size - 1} dof, p={p:.2e}"
