"""Helpers for the GPU parity tests: run a Batch through the C ABI and
compare against the oracle."""
from __future__ import annotations

import numpy as np


def run_gpu(case, debug=True, flags=0, cluster_size=0, with_uniforms=True):
    import torch

    from mstar_rs_b200 import kernel, workloads

    d = workloads.to_device(case, with_uniforms=with_uniforms)
    logits = d.pop("logits")
    B, V = case.B, case.V
    dev = logits.device
    out = dict(out_ids=torch.full((B,), -7, dtype=torch.int64, device=dev),
               out_status=torch.full((B,), -7, dtype=torch.int32, device=dev))
    if debug:
        out.update(out_x=torch.full((B, V), 123.0, device=dev),
                   out_kept=torch.full((B, V), 7, dtype=torch.uint8, device=dev),
                   out_probs=torch.full((B, V), 9.0, device=dev))
    ns = None
    if case.slot_idx is not None:
        ns = max(int(case.slot_idx.max()) + 1, 1)
        for a in (case.temperature, case.seed, case.hist_len, case.top_k):
            if a is not None:
                ns = a.shape[0]
                break
    kernel.sampler_step(logits, **d, **out, flags=flags, cluster_size=cluster_size, num_slots=ns)
    torch.cuda.synchronize()
    res = dict(ids=out["out_ids"].cpu().numpy(), status=out["out_status"].cpu().numpy())
    if debug:
        res.update(x=out["out_x"].cpu().numpy(), kept=out["out_kept"].cpu().numpy().astype(bool),
                   probs=out["out_probs"].cpu().numpy())
    res["_dev"] = d
    return res


def assert_parity(g, o, case, debug=True, status_mask=0x1):
    name = case.name
    np.testing.assert_array_equal(g["ids"], o["ids"], err_msg=f"{name}: token ids")
    np.testing.assert_array_equal(g["status"] & status_mask, o["status"] & status_mask,
                                  err_msg=f"{name}: status")
    if not debug:
        return
    np.testing.assert_array_equal(g["kept"], o["kept"], err_msg=f"{name}: kept set")
    xa, xb = g["x"], o["x"]
    np.testing.assert_array_equal(np.isnan(xa), np.isnan(xb), err_msg=f"{name}: processed NaN pattern")
    np.testing.assert_array_equal(np.where(np.isnan(xa), 0, xa).view(np.uint32),
                                  np.where(np.isnan(xb), 0, xb).view(np.uint32),
                                  err_msg=f"{name}: penalty-adjusted logits (bit-exact)")
    # probabilities: the spec's tolerance (1e-5 relative fp32, 2e-3 bf16)
    tol = 2e-3 if case.dtype == "bf16" else 1e-5
    np.testing.assert_allclose(g["probs"], o["probs"], rtol=tol, atol=0, err_msg=f"{name}: probabilities")
