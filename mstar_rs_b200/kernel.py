"""Torch-tensor front end of the sampler kernel.

`sampler_step` fills a `Params` struct from device tensors and launches one
sampling step on the current CUDA stream.  It allocates nothing, never
synchronises and never reads device memory on the host, so it can be called
inside `torch.cuda.graph` capture.  Shapes, dtypes, devices and contiguity are
validated here (before any launch) and again by the C ABI.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N

_DT = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16}
_U64 = (torch.int64, torch.uint64)  # seed / offset: 64-bit words, read as unsigned


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _need(t, name, dtype, dev, shape0=None, ndim=1):
    if t is None:
        return
    ok = dtype if isinstance(dtype, tuple) else (dtype,)
    if t.dtype not in ok:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.device != dev:
        raise ValueError(f"{name} must live on {dev}, got {t.device}")
    if t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if shape0 is not None and t.shape[0] < shape0:
        raise ValueError(f"{name} has {t.shape[0]} rows, need >= {shape0}")


def build_params(logits: torch.Tensor, *, slot_idx=None, num_slots=None, temperature=None, top_k=None,
                 top_p=None, min_p=None, rep_pen=None, pres_pen=None, freq_pen=None, hist_ids=None,
                 hist_len=None, seen_bits=None, seen_cap=0, bias_ids=None, bias_vals=None,
                 allowed_bits=None, uniforms=None, seed=None, offset=None, out_ids=None, out_ids32=None,
                 out_status=None, out_x=None, out_kept=None, out_probs=None, flags=0, cluster_size=0,
                 vocab_offset=0, stop_ids=None, stop_flags=None) -> N.Params:
    if logits.dim() != 2:
        raise ValueError("logits must be [B, V]")
    if logits.dtype not in _DT:
        raise TypeError(f"logits must be float32 or bfloat16, got {logits.dtype}")
    if not logits.is_cuda:
        raise ValueError("logits must be a CUDA tensor (there is no CPU path)")
    if logits.stride(1) != 1:
        raise ValueError("logits rows must be contiguous")
    dev = logits.device
    B, V = logits.shape
    ns = num_slots
    if ns is None:
        for t in (temperature, top_k, top_p, min_p, rep_pen, pres_pen, freq_pen, seed, offset, hist_len):
            if t is not None:
                ns = t.shape[0]
                break
        else:
            ns = B
    _need(slot_idx, "slot_idx", torch.int32, dev, B)
    for name, t, dt in (("temperature", temperature, torch.float32), ("top_k", top_k, torch.int32),
                        ("top_p", top_p, torch.float32), ("min_p", min_p, torch.float32),
                        ("rep_pen", rep_pen, torch.float32), ("pres_pen", pres_pen, torch.float32),
                        ("freq_pen", freq_pen, torch.float32), ("hist_len", hist_len, torch.int32),
                        ("seed", seed, _U64), ("offset", offset, _U64)):
        _need(t, name, dt, dev, ns)
    _need(hist_ids, "hist_ids", torch.int32, dev, ns, 2)
    _need(seen_bits, "seen_bits", torch.int32, dev, ns, 2)
    _need(bias_ids, "bias_ids", torch.int32, dev, ns, 2)
    _need(bias_vals, "bias_vals", torch.float32, dev, ns, 2)
    _need(allowed_bits, "allowed_bits", torch.int32, dev, ns, 2)
    _need(stop_ids, "stop_ids", torch.int32, dev, ns, 2)
    _need(stop_flags, "stop_flags", torch.int32, dev, ns)
    if stop_flags is not None and stop_ids is None:
        raise ValueError("stop_flags needs stop_ids")
    _need(uniforms, "uniforms", torch.float32, dev, B)
    _need(out_ids, "out_ids", torch.int64, dev, B)
    _need(out_ids32, "out_ids32", torch.int32, dev, B)
    _need(out_status, "out_status", torch.int32, dev, B)
    for name, t, dt in (("out_x", out_x, torch.float32), ("out_kept", out_kept, torch.uint8),
                        ("out_probs", out_probs, torch.float32)):
        if t is not None:
            _need(t, name, dt, dev, B, 2)
            if t.shape[1] != V:
                raise ValueError(f"{name} must be [B, V]")
    p = N.Params()
    p.logits = logits.data_ptr()
    p.dtype = _DT[logits.dtype]
    p.B, p.V, p.num_slots = B, V, ns
    p.ld = logits.stride(0)
    p.vocab_offset = vocab_offset
    p.slot_idx = _ptr(slot_idx)
    p.temperature, p.top_k, p.top_p, p.min_p = _ptr(temperature), _ptr(top_k), _ptr(top_p), _ptr(min_p)
    p.rep_pen, p.pres_pen, p.freq_pen = _ptr(rep_pen), _ptr(pres_pen), _ptr(freq_pen)
    p.hist_ids, p.hist_len = _ptr(hist_ids), _ptr(hist_len)
    p.H = 0 if hist_ids is None else hist_ids.shape[1]
    p.seen_cap = seen_cap
    p.seen_bits = _ptr(seen_bits)
    p.seen_words = 0 if seen_bits is None else seen_bits.shape[1]
    p.bias_ids, p.bias_vals = _ptr(bias_ids), _ptr(bias_vals)
    p.NB = 0 if bias_ids is None else bias_ids.shape[1]
    p.allowed_bits = _ptr(allowed_bits)
    p.allowed_words = 0 if allowed_bits is None else allowed_bits.shape[1]
    p.uniforms, p.seed, p.offset = _ptr(uniforms), _ptr(seed), _ptr(offset)
    p.out_ids, p.out_ids32, p.out_status = _ptr(out_ids), _ptr(out_ids32), _ptr(out_status)
    p.out_x, p.out_kept, p.out_probs = _ptr(out_x), _ptr(out_kept), _ptr(out_probs)
    p.flags = flags
    p.cluster_size = cluster_size
    p.stop_ids = _ptr(stop_ids)
    p.NS = 0 if stop_ids is None else stop_ids.shape[1]
    p.stop_flags = _ptr(stop_flags)
    return p


def launch_step(p: N.Params, device: torch.device) -> None:
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        N.check(N.lib().mstar_sampler_step(ctypes.byref(p), ctypes.c_void_p(stream)), "mstar_sampler_step")


def sampler_step(logits: torch.Tensor, **kw) -> N.Params:
    """Launch one sampling step; returns the Params used (keep it to relaunch)."""
    p = build_params(logits, **kw)
    launch_step(p, logits.device)
    return p


def sampler_step_heads(logits: torch.Tensor, **kw) -> N.Params:
    """One launch for H heads of n rows each (logits [H, n, V], e.g. the
    codebook heads of a multi-codebook decoder sampled together): row h * n + i
    of the flattened [H * n, V] batch is head h's row i, and slot_idx [H * n]
    (or the row number) picks its parameters and per-slot state, so each
    (head, request) pair keeps its own history, seen mask and RNG offset."""
    if logits.dim() != 3:
        raise ValueError("logits must be [H, n, V]")
    H, n, V = logits.shape
    if logits.stride(2) != 1 or logits.stride(0) != n * logits.stride(1):
        raise ValueError("logits heads must be stacked rows of one [H * n, V] matrix")
    return sampler_step(logits.reshape(H * n, V), **kw)


def plan(logits: torch.Tensor, **kw):
    p = build_params(logits, **kw)
    cs, sm = N.I32(), N.I64()
    N.check(N.lib().mstar_sampler_plan(ctypes.byref(p), ctypes.byref(cs), ctypes.byref(sm)), "mstar_sampler_plan")
    return cs.value, sm.value


def tp_record_words(tp_cap: int) -> int:
    return int(N.lib().mstar_sampler_tp_record_words(tp_cap))


def tp_local(logits: torch.Tensor, tp_cap: int, send: torch.Tensor, **kw) -> None:
    p = build_params(logits, **kw)
    if send.dtype != torch.int32 or not send.is_contiguous() or send.device != logits.device:
        raise ValueError("send must be a contiguous int32 tensor on the logits device")
    if send.numel() < logits.shape[0] * tp_record_words(tp_cap):
        raise ValueError("send buffer too small")
    with torch.cuda.device(logits.device):
        stream = torch.cuda.current_stream(logits.device).cuda_stream
        N.check(N.lib().mstar_sampler_tp_local(ctypes.byref(p), tp_cap, ctypes.c_void_p(send.data_ptr()),
                                               ctypes.c_void_p(stream)), "mstar_sampler_tp_local")


def tp_merge(logits: torch.Tensor, tp_cap: int, tp_world: int, V_global: int, recv: torch.Tensor, **kw) -> None:
    p = build_params(logits, **kw)
    if recv.dtype != torch.int32 or not recv.is_contiguous() or recv.device != logits.device:
        raise ValueError("recv must be a contiguous int32 tensor on the logits device")
    if recv.numel() < tp_world * logits.shape[0] * tp_record_words(tp_cap):
        raise ValueError("recv buffer too small")
    with torch.cuda.device(logits.device):
        stream = torch.cuda.current_stream(logits.device).cuda_stream
        N.check(N.lib().mstar_sampler_tp_merge(ctypes.byref(p), tp_cap, tp_world, V_global,
                                               ctypes.c_void_p(recv.data_ptr()), ctypes.c_void_p(stream)),
                "mstar_sampler_tp_merge")


def _u32(t, name, dev, n):
    if t.dtype != torch.int32 or t.device != dev or not t.is_contiguous() or t.numel() < n:
        raise ValueError(f"{name} must be a contiguous int32 tensor of >= {n} words on {dev}")


def tp_local2(logits: torch.Tensor, tp_cap: int, send: torch.Tensor, xbuf: torch.Tensor, **kw) -> None:
    """Two-round shard records (mstar_sampler_tp_local2): rows without a
    usable top_k send their first tp_cap members and leave their shard
    values in xbuf [B, V] float32."""
    p = build_params(logits, **kw)
    dev = logits.device
    _u32(send, "send", dev, logits.shape[0] * tp_record_words(tp_cap))
    if xbuf.dtype != torch.float32 or xbuf.device != dev or not xbuf.is_contiguous() or \
            xbuf.numel() < logits.shape[0] * logits.shape[1]:
        raise ValueError("xbuf must be a contiguous float32 [B, V] tensor on the logits device")
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        N.check(N.lib().mstar_sampler_tp_local2(ctypes.byref(p), tp_cap, _ptr(send), _ptr(xbuf),
                                                ctypes.c_void_p(stream)), "mstar_sampler_tp_local2")


def tp_merge1(logits: torch.Tensor, tp_cap: int, tp_world: int, V_global: int, recv: torch.Tensor,
              pend: torch.Tensor, **kw) -> None:
    """First merge of the two-round exchange (mstar_sampler_tp_merge1): decides
    the rows no shard cut short, defers the others into pend [B, 2] int32."""
    p = build_params(logits, **kw)
    dev = logits.device
    B = logits.shape[0]
    _u32(recv, "recv", dev, tp_world * B * tp_record_words(tp_cap))
    _u32(pend, "pend", dev, 2 * B)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        N.check(N.lib().mstar_sampler_tp_merge1(ctypes.byref(p), tp_cap, tp_world, V_global, _ptr(recv), _ptr(pend),
                                                ctypes.c_void_p(stream)), "mstar_sampler_tp_merge1")


def tp_mass(logits: torch.Tensor, xbuf: torch.Tensor, pend: torch.Tensor, send2: torch.Tensor, **kw) -> None:
    """The shard's exact A mass of every deferred row (mstar_sampler_tp_mass)
    into send2 [B, 2] int32 (a little-endian u64 per row)."""
    p = build_params(logits, **kw)
    dev = logits.device
    B = logits.shape[0]
    _u32(pend, "pend", dev, 2 * B)
    _u32(send2, "send2", dev, 2 * B)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        N.check(N.lib().mstar_sampler_tp_mass(ctypes.byref(p), _ptr(xbuf), _ptr(pend), _ptr(send2),
                                              ctypes.c_void_p(stream)), "mstar_sampler_tp_mass")


def tp_merge2(logits: torch.Tensor, tp_cap: int, tp_world: int, V_global: int, recv: torch.Tensor,
              recv2: torch.Tensor, pend: torch.Tensor, **kw) -> None:
    """Second merge of the two-round exchange (mstar_sampler_tp_merge2)."""
    p = build_params(logits, **kw)
    dev = logits.device
    B = logits.shape[0]
    _u32(recv, "recv", dev, tp_world * B * tp_record_words(tp_cap))
    _u32(recv2, "recv2", dev, tp_world * 2 * B)
    _u32(pend, "pend", dev, 2 * B)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        N.check(N.lib().mstar_sampler_tp_merge2(ctypes.byref(p), tp_cap, tp_world, V_global, _ptr(recv), _ptr(recv2),
                                                _ptr(pend), ctypes.c_void_p(stream)), "mstar_sampler_tp_merge2")


def commit(ids: torch.Tensor, *, V: int, num_slots: int, slot_idx=None, hist_ids=None, hist_len=None,
           seen_bits=None, stop_ids=None, stop_flags=None, offset=None, flags=0, vocab_offset=0) -> None:
    """Per-slot state updates for ids chosen elsewhere (mstar_sampler_commit):
    history append / seen bit / RNG offset as `flags` selects, stop flags."""
    if ids.dtype != torch.int64 or ids.dim() != 1 or not ids.is_cuda or not ids.is_contiguous():
        raise ValueError("ids must be a contiguous 1-D int64 CUDA tensor")
    dev = ids.device
    B = ids.shape[0]
    _need(slot_idx, "slot_idx", torch.int32, dev, B)
    _need(hist_len, "hist_len", torch.int32, dev, num_slots)
    _need(offset, "offset", _U64, dev, num_slots)
    _need(stop_flags, "stop_flags", torch.int32, dev, num_slots)
    _need(hist_ids, "hist_ids", torch.int32, dev, num_slots, 2)
    _need(seen_bits, "seen_bits", torch.int32, dev, num_slots, 2)
    _need(stop_ids, "stop_ids", torch.int32, dev, num_slots, 2)
    p = N.Params()
    p.B, p.V, p.num_slots, p.vocab_offset = B, V, num_slots, vocab_offset
    p.slot_idx = _ptr(slot_idx)
    p.hist_ids, p.hist_len = _ptr(hist_ids), _ptr(hist_len)
    p.H = 0 if hist_ids is None else hist_ids.shape[1]
    p.seen_bits = _ptr(seen_bits)
    p.seen_words = 0 if seen_bits is None else seen_bits.shape[1]
    p.stop_ids, p.stop_flags = _ptr(stop_ids), _ptr(stop_flags)
    p.NS = 0 if stop_ids is None else stop_ids.shape[1]
    p.offset = _ptr(offset)
    p.flags = flags
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        N.check(N.lib().mstar_sampler_commit(ctypes.byref(p), ctypes.c_void_p(ids.data_ptr()),
                                             ctypes.c_void_p(stream)), "mstar_sampler_commit")


def _check_lmhead(hidden: torch.Tensor, weight: torch.Tensor):
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("hidden and weight must be bfloat16")
    if not hidden.is_cuda or weight.device != hidden.device:
        raise ValueError("hidden and weight must be CUDA tensors on one device")
    if hidden.dim() != 2 or weight.dim() != 2 or hidden.shape[1] != weight.shape[1]:
        raise ValueError("hidden must be [B, d] and weight [V, d]")
    if not hidden.is_contiguous() or not weight.is_contiguous():
        raise ValueError("hidden and weight must be contiguous")
    return hidden.shape[0], weight.shape[0], hidden.shape[1]


_WS: dict = {}


def lmhead_workspace(B: int, device: torch.device) -> torch.Tensor:
    """Scratch for projections of up to B rows on `device`
    (mstar_lmhead_workspace_bytes), kept per device and reused: calls on one
    stream share it; give each concurrent stream its own."""
    dev = torch.device(device)
    with torch.cuda.device(dev):
        n = int(N.lib().mstar_lmhead_workspace_bytes(B))
    if n <= 0:
        raise ValueError(f"B={B} is outside [1, 256]")
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _WS.get(key)
    if ws is None or ws.numel() < n:
        ws = torch.empty(n, dtype=torch.uint8, device=dev)
        _WS[key] = ws
    return ws


def _check_ws(ws, dev):
    if ws is None:
        return None, 0
    if ws.dtype != torch.uint8 or ws.device != dev or not ws.is_contiguous():
        raise ValueError("workspace must be a contiguous uint8 tensor on the hidden device")
    return _ptr(ws), ws.numel()


def lmhead_logits(hidden: torch.Tensor, weight: torch.Tensor, *, out: torch.Tensor | None = None,
                  dtype=torch.float32, status: torch.Tensor | None = None, workspace="auto") -> torch.Tensor:
    """hidden [B, d] @ weight[V, d]^T on the tensor cores (mstar_lmhead_logits),
    fp32 accumulation, stored as float32 or bfloat16.  workspace: "auto" (the
    device's cached lmhead_workspace), a uint8 tensor, or None (whole-tile
    shares, no scratch)."""
    B, V, d = _check_lmhead(hidden, weight)
    dev = hidden.device
    if out is None:
        out = torch.empty(B, V, dtype=dtype, device=dev)
    if out.dtype not in _DT or out.device != dev or out.dim() != 2 or out.shape[0] != B or out.shape[1] < V \
            or out.stride(1) != 1:
        raise ValueError("out must be [B, >= V] float32 / bfloat16 with contiguous rows on the hidden device")
    if status is not None and (status.dtype != torch.int32 or status.device != dev or status.numel() < 1):
        raise ValueError("status must be an int32 tensor on the hidden device")
    if isinstance(workspace, str):
        workspace = lmhead_workspace(B, dev)
    wp, wn = _check_ws(workspace, dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        N.check(N.lib().mstar_lmhead_logits(_ptr(hidden), _ptr(weight), B, V, d, _ptr(out), _DT[out.dtype],
                                            out.stride(0), wp, wn, _ptr(status), ctypes.c_void_p(stream)),
                "mstar_lmhead_logits")
    return out


def lmhead_step(hidden: torch.Tensor, weight: torch.Tensor, logits: torch.Tensor, *, status=None,
                workspace="auto", **kw) -> N.Params:
    """Project hidden [B, d] by weight [V, d] into `logits` [B, V] (float32 or
    bfloat16, written) and sample from it (mstar_sampler_lmhead_step).  The
    sampling keywords are sampler_step's; workspace as for lmhead_logits."""
    B, V, d = _check_lmhead(hidden, weight)
    if logits.shape[0] != B or logits.dim() != 2 or logits.shape[1] != V:
        raise ValueError("logits must be [B, V] for hidden [B, d] and weight [V, d]")
    if status is not None and (status.dtype != torch.int32 or status.device != hidden.device or status.numel() < 1):
        raise ValueError("status must be an int32 tensor on the hidden device")
    p = build_params(logits, **kw)
    if isinstance(workspace, str):
        workspace = lmhead_workspace(B, hidden.device)
    wp, wn = _check_ws(workspace, hidden.device)
    with torch.cuda.device(logits.device):
        stream = torch.cuda.current_stream(logits.device).cuda_stream
        N.check(N.lib().mstar_sampler_lmhead_step(ctypes.byref(p), _ptr(hidden), _ptr(weight), d, wp, wn,
                                                  _ptr(status), ctypes.c_void_p(stream)),
                "mstar_sampler_lmhead_step")
    return p
