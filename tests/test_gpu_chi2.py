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


@pytest.mark.parametrize("general", [False, True])
def test_chi_square_headline_row(oracle_lib, general):
    """1,048,576 Philox draws of one row of the mixed workload's shape
    (V=151936 bf16, 1024-token Zipf history, cluster of 2), on the fast path
    and forced onto the general path, against the probabilities of the
    torch-formulated oracle (float64 softmax), which is written
    independently of the kernel's fixed-point arithmetic."""
    import torch
    from scipy import stats

    from mstar_rs_b200 import _native as N
    from mstar_rs_b200 import kernel
    from mstar_rs_b200 import workloads as W
    from oracle import torch_ref

    one = W.qwen_mixed(seed=9, B=1)
    one.temperature[:] = 1.2
    one.top_k[:] = 0
    one.top_p[:] = 0.95
    one.min_p[:] = 0.005
    spec = oracle_lib.run(one, debug=True)
    kept = np.flatnonzero(spec["kept"][0])
    _, tkept, tprobs, _ = torch_ref.sample_row(one, 0)
    assert np.array_equal(np.flatnonzero(tkept.numpy()), kept), "the two oracles keep different sets"
    probs = tprobs.numpy()[kept]
    assert 20 <= kept.size <= 2000, kept.size

    B, launches = 512, 2048
    d = W.to_device(one, with_uniforms=False)
    src = d.pop("logits")
    logits = src.repeat(B, 1)
    dev = logits.device
    rep = {k: (v.repeat(B, *([1] * (v.dim() - 1))) if torch.is_tensor(v) else v) for k, v in d.items()}
    rep.pop("vocab_offset", None)
    rep["seed"] = torch.full((B,), 0xC0FFEE, dtype=torch.int64, device=dev)
    rep["offset"] = torch.arange(B, dtype=torch.int64, device=dev) * launches
    out = torch.zeros(B, dtype=torch.int64, device=dev)
    counts = torch.zeros(one.V, dtype=torch.int64, device=dev)
    flags = N.FLAG_ADVANCE_OFFSET | (N.FLAG_FORCE_GENERAL if general else 0)
    p = kernel.build_params(logits, **rep, out_ids=out, flags=flags, cluster_size=2)
    for _ in range(launches):
        kernel.launch_step(p, dev)
        counts += torch.bincount(out, minlength=one.V)
    counts = counts.cpu().numpy()
    n = B * launches
    assert counts.sum() == n
    outside = np.ones(one.V, bool)
    outside[kept] = False
    assert counts[outside].sum() == 0, "a token outside the kept set was drawn"
    expected = probs * n
    obs = counts[kept].astype(np.float64)
    small = expected < 5  # pool the rare tokens into one bin
    e = np.append(expected[~small], expected[small].sum())
    o = np.append(obs[~small], obs[small].sum())
    if e[-1] == 0:
        e, o = e[:-1], o[:-1]
    chi2 = float(((o - e) ** 2 / e).sum())
    pv = float(stats.chi2.sf(chi2, df=e.size - 1))
    assert pv > 1e-3, f"chi2={chi2:.1f} over {e.size - 1} dof, p={pv:.2e}"
