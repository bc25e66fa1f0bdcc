"""Drop-in sampler interface for the mstar-rs engines.

Mirrors the classes the reference's engines import from the external
`mstar.utils.sampling` package (python/mstar_rs/models/orpheus.py:78-83,
python/mstar_rs/models/qwen3_omni.py:405, :906-911), with the call-site
semantics those engines rely on:

  SamplingConfig(vocab_size=, temperature=, top_k=, top_p=,
                 repetition_penalty=, ignore_eos=) + .set_seed(seed)
                                   orpheus.py:177-185, qwen3_omni.py:440-447, :1001-1009
  Sampler(device, tp_group=): add_request / set_config / _sampling_config[rid]
      .set_seed / sample([rid], logits, apply_penalty=) / remove_request
                                   orpheus.py:93, :196-207, :517; qwen3_omni.py:457-466, :483
  SamplerBuffers.allocate(max_bs, device, tp_group=, vocab_size=):
      register_request / unregister_request / stage_seen_token_masks /
      gather_for_request_ids(rids, n, gather_seen_tokens=) / offset_buf /
      seen_tokens.buf               orpheus.py:101-103, :186, :229, :341-359, :419-426
  CudaGraphableSampler.sample(rids, logits, apply_penalty=True) /
      sync_seen_token_masks(masks)  orpheus.py:350, :426; qwen3_omni.py:518
  SeenTokenMask.new(rid, V, device) / add_tokens(tok)   orpheus.py:187, :500

One addition: `SamplingConfig.stop_token_ids` (ignored under `ignore_eos`)
lets the kernel flag the rows that sampled a stop token, so an engine reads
one small flag vector per step (`Sampler.stopped`, `SamplerBuffers.stopped`)
instead of reading every sampled id back to compare it with the stop id
(orpheus.py:428-432, :518-519).

Every sampling call runs the sm_100a kernel through the C ABI; nothing here
computes a token on the host.  Greedy is temperature 0 (or top_k 1).  The
in-graph sampler advances the per-row RNG offset and the seen-token bits on
the device, so a captured decode graph replays with no host involvement.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _native as N
from . import kernel

_SAMPLING_EPS = 1e-5


@dataclass
class SamplingConfig:
    vocab_size: int | None = None
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    logit_bias: dict | None = None
    ignore_eos: bool = False
    seed: int | None = None
    stop_token_ids: tuple | list | None = None
    _owner: object = field(default=None, repr=False, compare=False)

    def set_seed(self, seed) -> None:
        self.seed = None if seed is None else int(seed)
        if self._owner is not None:
            self._owner._mark_dirty()

    @property
    def greedy(self) -> bool:
        return self.temperature < _SAMPLING_EPS or self.top_k == 1


def _words(V: int) -> int:
    return (V + 31) // 32


class SeenTokenMask:
    """Per-request set of generated token ids, bit-packed on the device
    (bit id & 31 of word id >> 5).  Prompt tokens are not added."""

    def __init__(self, rid, vocab_size: int, device):
        self.rid = rid
        self.vocab_size = vocab_size
        self.bits = torch.zeros(_words(vocab_size), dtype=torch.int32, device=device)

    @classmethod
    def new(cls, rid, vocab_size: int, device) -> "SeenTokenMask":
        return cls(rid, vocab_size, device)

    def add_tokens(self, tok: torch.Tensor) -> None:
        t = tok.reshape(-1).to(device=self.bits.device, dtype=torch.int64)
        w = t >> 5
        b = torch.bitwise_left_shift(torch.ones_like(t, dtype=torch.int32), (t & 31).to(torch.int32))
        self.bits.index_put_((w,), self.bits.index_select(0, w) | b)

    def to_bool(self) -> torch.Tensor:
        ar = torch.arange(32, device=self.bits.device, dtype=torch.int32)
        m = ((self.bits.unsqueeze(1) >> ar) & 1).bool().reshape(-1)
        return m[: self.vocab_size]


class _ParamTable:
    """Host mirror + device copy of the per-slot parameter arrays."""

    NAMES = ("temperature", "top_p", "min_p", "rep_pen", "pres_pen", "freq_pen")
    NSTOP = 4  # stop ids per slot

    def __init__(self, n: int, device):
        self.n = n
        self.device = device
        self.host = {k: np.zeros(n, np.float32) for k in self.NAMES}
        self.host["temperature"][:] = 1.0
        self.host["top_p"][:] = 1.0
        self.host["rep_pen"][:] = 1.0
        self.host_k = np.zeros(n, np.int32)
        self.host_seed = np.zeros(n, np.int64)
        self.host_stop = np.full((n, self.NSTOP), -1, np.int32)
        self.dev = {k: torch.from_numpy(v.copy()).to(device) for k, v in self.host.items()}
        self.dev_k = torch.zeros(n, dtype=torch.int32, device=device)
        self.dev_seed = torch.zeros(n, dtype=torch.int64, device=device)
        self.dev_stop = torch.full((n, self.NSTOP), -1, dtype=torch.int32, device=device)
        self.dirty = True

    def write(self, i: int, cfg: SamplingConfig) -> None:
        stops = () if cfg.ignore_eos or cfg.stop_token_ids is None else cfg.stop_token_ids
        if isinstance(stops, int):
            stops = (stops,)
        stops = [int(t) for t in stops]
        if len(stops) > self.NSTOP or any(t < 0 for t in stops):  # checked before any field changes
            raise ValueError(f"stop_token_ids takes at most {self.NSTOP} non-negative ids, got {stops}")
        greedy = cfg.temperature < _SAMPLING_EPS
        self.host["temperature"][i] = 0.0 if greedy else cfg.temperature
        self.host_k[i] = 1 if greedy else int(cfg.top_k)
        self.host["top_p"][i] = cfg.top_p
        self.host["min_p"][i] = cfg.min_p
        self.host["rep_pen"][i] = cfg.repetition_penalty
        self.host["pres_pen"][i] = cfg.presence_penalty
        self.host["freq_pen"][i] = cfg.frequency_penalty
        s = 0 if cfg.seed is None else cfg.seed
        self.host_seed[i] = np.int64(np.uint64(s & 0xFFFFFFFFFFFFFFFF).view(np.int64))
        self.host_stop[i] = -1
        self.host_stop[i, : len(stops)] = stops
        self.dirty = True

    def upload(self) -> None:
        if not self.dirty:
            return
        for k, v in self.host.items():
            self.dev[k].copy_(torch.from_numpy(v))
        self.dev_k.copy_(torch.from_numpy(self.host_k))
        self.dev_seed.copy_(torch.from_numpy(self.host_seed))
        self.dev_stop.copy_(torch.from_numpy(self.host_stop))
        self.dirty = False

    def kwargs(self) -> dict:
        return dict(temperature=self.dev["temperature"], top_k=self.dev_k, top_p=self.dev["top_p"],
                    min_p=self.dev["min_p"], rep_pen=self.dev["rep_pen"], pres_pen=self.dev["pres_pen"],
                    freq_pen=self.dev["freq_pen"], seed=self.dev_seed, stop_ids=self.dev_stop)


class Sampler:
    """Eager per-request sampler (prefill and non-graph decode).

    Each request owns a slot: parameters, RNG (seed, offset) and a ring of
    its last `history` generated ids (repetition / presence / frequency
    penalties count over it).  `sample` reads the slots through an index
    vector, so requests can be sampled in any order or subset."""

    def __init__(self, device=None, tp_group=None, max_requests: int = 256, history: int = 1024,
                 vocab_size: int | None = None):
        self.device = torch.device(device if device is not None else "cuda")
        if self.device.type != "cuda":
            raise ValueError("the sampler runs on CUDA devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.tp_group = tp_group
        self.max_requests = max_requests
        self.H = history
        self.vocab_size = vocab_size
        self.params = _ParamTable(max_requests, self.device)
        self.offset = torch.zeros(max_requests, dtype=torch.int64, device=self.device)
        self.hist = torch.full((max_requests, history), -1, dtype=torch.int32, device=self.device)
        self.hist_len = torch.zeros(max_requests, dtype=torch.int32, device=self.device)
        self.stop_flags = torch.zeros(max_requests, dtype=torch.int32, device=self.device)
        self._slot: dict = {}
        self._free = list(range(max_requests - 1, -1, -1))
        self._sampling_config: dict = {}
        self._idx_cache: dict = {}

    def _mark_dirty(self) -> None:
        for rid, cfg in self._sampling_config.items():
            self.params.write(self._slot[rid], cfg)

    def add_request(self, rid) -> None:
        if rid in self._slot:
            return
        if not self._free:
            raise RuntimeError(f"sampler full ({self.max_requests} requests)")
        s = self._free.pop()
        self._slot[rid] = s
        cfg = SamplingConfig(vocab_size=self.vocab_size, _owner=self)
        self._sampling_config[rid] = cfg
        self.params.write(s, cfg)
        self.offset[s] = 0
        self.hist_len[s] = 0
        self.stop_flags[s] = 0
        self._idx_cache.clear()

    def set_config(self, rid, **kw) -> None:
        cfg = self._sampling_config[rid]
        for k in kw:
            if not hasattr(cfg, k) or k.startswith("_"):
                raise TypeError(f"unknown sampling option {k!r}")
        old = {k: getattr(cfg, k) for k in kw}
        for k, v in kw.items():
            setattr(cfg, k, v)
        try:
            self.params.write(self._slot[rid], cfg)
        except ValueError:
            for k, v in old.items():  # a refused option leaves the request as it was
                setattr(cfg, k, v)
            raise

    def set_history(self, rid, ids) -> None:
        """Seed a request's generated-token history (penalty state)."""
        s = self._slot[rid]
        ids = list(ids)[-self.H:]
        row = torch.full((self.H,), -1, dtype=torch.int32)
        if ids:
            row[: len(ids)] = torch.tensor(ids, dtype=torch.int32)
        self.hist[s].copy_(row)
        self.hist_len[s] = len(ids)

    def remove_request(self, rid) -> None:
        s = self._slot.pop(rid, None)
        self._sampling_config.pop(rid, None)
        if s is not None:
            self._free.append(s)
        self._idx_cache.clear()

    def _index(self, rids) -> torch.Tensor:
        key = tuple(rids)
        t = self._idx_cache.get(key)
        if t is None:
            t = torch.tensor([self._slot[r] for r in rids], dtype=torch.int32, device=self.device)
            self._idx_cache[key] = t
        return t

    def sample(self, rids, logits: torch.Tensor, apply_penalty: bool = True) -> torch.Tensor:
        """logits [n, V] (bf16 or fp32, on this sampler's device) -> ids [n] int64."""
        n = len(rids)
        if logits.dim() == 1:
            logits = logits.unsqueeze(0)
        if logits.shape[0] != n:
            raise ValueError(f"{n} request ids for {logits.shape[0]} logits rows")
        self.params.upload()
        out = torch.empty(n, dtype=torch.int64, device=self.device)
        flags = N.FLAG_ADVANCE_OFFSET | N.FLAG_UPDATE_HISTORY
        kernel.sampler_step(logits, slot_idx=self._index(rids), num_slots=self.max_requests,
                            **self.params.kwargs(), offset=self.offset,
                            hist_ids=self.hist if apply_penalty else None,
                            hist_len=self.hist_len if apply_penalty else None,
                            out_ids=out, stop_flags=self.stop_flags,
                            flags=flags if apply_penalty else N.FLAG_ADVANCE_OFFSET)
        return out

    def stopped(self, rids) -> list:
        """The requests among `rids` that have sampled one of their stop
        tokens (one device read for all of them); their flags are cleared."""
        if not rids:
            return []
        idx = self._index(rids).long()
        hit = self.stop_flags.index_select(0, idx).tolist()
        out = [r for r, h in zip(rids, hit) if h]
        if out:
            self.stop_flags.index_fill_(0, idx, 0)
        return out


class _SeenTokens:
    def __init__(self, max_bs: int, V: int, device):
        self.buf = torch.zeros(max_bs, _words(V), dtype=torch.int32, device=device)


class CudaGraphableSampler:
    """Samples rows [0, n) of a SamplerBuffers' step buffers.  `sample` is
    capturable: fixed buffers, no allocation, no host sync."""

    def __init__(self, sbuf: "SamplerBuffers", n: int):
        self.sbuf = sbuf
        self.n = n
        self.out = torch.zeros(n, dtype=torch.int64, device=sbuf.device)
        self.slot_idx: torch.Tensor | None = None  # [n] int32; -1 marks a padding row
        self._rids: list = []

    def sample(self, rids, logits: torch.Tensor, apply_penalty: bool = True) -> torch.Tensor:
        sb = self.sbuf
        n = self.n
        if logits.shape[0] != n:
            raise ValueError(f"sampler gathered for {n} rows, logits has {logits.shape[0]}")
        kw = sb.params.kwargs()
        if not apply_penalty:  # seen bits still advance; the penalties are neutral
            kw.update(rep_pen=None, pres_pen=None, freq_pen=None)
        kernel.sampler_step(logits, num_slots=sb.max_bs, **kw, offset=sb.offset_buf,
                            seen_bits=sb.seen_tokens.buf, seen_cap=sb.seen_cap, out_ids=self.out,
                            slot_idx=self.slot_idx, stop_flags=sb.stop_flags,
                            flags=N.FLAG_ADVANCE_OFFSET | N.FLAG_UPDATE_SEEN)
        return self.out

    def stopped(self) -> list:
        """The gathered requests that sampled a stop token since the flags
        were last read (see SamplerBuffers.stopped)."""
        return self.sbuf.stopped(self._rids)

    def sync_seen_token_masks(self, masks) -> None:
        """Copy the step rows' seen bits (updated in-graph) back to the
        per-request masks, and the advanced RNG offsets to the requests."""
        sb = self.sbuf
        for j, m in enumerate(masks):
            m.bits.copy_(sb.seen_tokens.buf[j])
        sb._store_offsets(self._rids)


class SamplerBuffers:
    """Fixed-shape step buffers for in-graph sampling of up to max_bs rows.

    Requests register a config; `gather_for_request_ids` writes the configs
    and RNG offsets of a batch into rows [0, n) (outside the graph), and the
    returned CudaGraphableSampler samples those rows in-graph."""

    def __init__(self, max_bs: int, device, tp_group=None, vocab_size: int | None = None, seen_cap: int = 2048):
        self.max_bs = max_bs
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.tp_group = tp_group
        self.vocab_size = vocab_size or 1
        self.seen_cap = seen_cap
        self.params = _ParamTable(max_bs, self.device)
        self.offset_buf = torch.zeros(max_bs, dtype=torch.int64, device=self.device)
        self.seen_tokens = _SeenTokens(max_bs, self.vocab_size, self.device)
        self.stop_flags = torch.zeros(max_bs, dtype=torch.int32, device=self.device)  # per step row
        self._rows: list = []
        self._cfg: dict = {}
        self._req_offset: dict = {}
        self._samplers: dict = {}

    @classmethod
    def allocate(cls, max_bs: int, device, tp_group=None, vocab_size: int | None = None) -> "SamplerBuffers":
        return cls(max_bs, device, tp_group=tp_group, vocab_size=vocab_size)

    def _mark_dirty(self) -> None:
        pass

    def register_request(self, rid, cfg: SamplingConfig) -> None:
        self._cfg[rid] = cfg
        self._req_offset.setdefault(rid, 0)

    def unregister_request(self, rid) -> None:
        self._cfg.pop(rid, None)
        self._req_offset.pop(rid, None)

    def stage_seen_token_masks(self, rids, masks) -> None:
        for j, m in enumerate(masks):
            self.seen_tokens.buf[j].copy_(m.bits)

    def gather_for_request_ids(self, rids, n: int, gather_seen_tokens: bool = True) -> CudaGraphableSampler:
        if len(rids) != n or n > self.max_bs:
            raise ValueError(f"gather of {len(rids)} ids into {n} rows (max {self.max_bs})")
        for j, rid in enumerate(rids):
            self.params.write(j, self._cfg[rid])
        self.params.upload()
        offs = torch.tensor([self._req_offset.get(r, 0) for r in rids], dtype=torch.int64)
        self.offset_buf[:n].copy_(offs)
        if not gather_seen_tokens:
            self.seen_tokens.buf[:n].zero_()
        if list(rids) != self._rows:  # rows now hold other requests: their stop flags start clear
            self.stop_flags.zero_()
            self._rows = list(rids)
        s = self._samplers.get(n)
        if s is None:
            s = CudaGraphableSampler(self, n)
            self._samplers[n] = s
        s._rids = list(rids)
        return s

    def stopped(self, rids) -> list:
        """The requests among the gathered `rids` (row j = rids[j]) whose row
        sampled one of their stop tokens in a step since the flags were last
        read: one device read of the step rows' flags, which are then cleared.
        The flags stay set across replays, so an engine may read them every
        few steps instead of after every step."""
        n = len(rids)
        if n == 0:
            return []
        hit = self.stop_flags[:n].tolist()
        out = [r for r, h in zip(rids, hit) if h]
        if out:
            self.stop_flags[:n].zero_()
        return out

    def _store_offsets(self, rids) -> None:
        vals = self.offset_buf[: len(rids)].tolist()
        for r, v in zip(rids, vals):
            if r in self._req_offset:
                self._req_offset[r] = int(v)


class SamplerGraphBuckets:
    """One captured CUDA graph per bucket size over fixed buffers, the way
    the reference's batched decode graphs pad a batch to the next bucket and
    discard the pad rows (python/mstar_rs/batched_graph.py:26-80,
    orpheus.py:322-366).  Pad rows carry slot -1: the kernel skips them (no
    sampling work, no state update).

    Usage: ``capture()`` once after ``SamplerBuffers.allocate``; then every
    step ``sample(rids, logits)`` stages the rows (outside any graph),
    replays the smallest bucket that holds them and returns the ids of the
    real rows.  ``sync(rids, masks)`` copies seen bits and RNG offsets back."""

    def __init__(self, sbuf: SamplerBuffers, buckets=(1, 2, 4, 8, 16, 32, 64), dtype=torch.bfloat16):
        self.sbuf = sbuf
        self.buckets = sorted(b for b in set(buckets) if 1 <= b <= sbuf.max_bs)
        if not self.buckets:
            raise ValueError("no bucket fits max_bs")
        top = self.buckets[-1]
        self.logits = torch.zeros(top, sbuf.vocab_size, dtype=dtype, device=sbuf.device)
        self.slot_idx = torch.full((top,), -1, dtype=torch.int32, device=sbuf.device)
        self._samplers = {}
        self._graphs = {}
        self._last = None

    def capture(self) -> None:
        sb = self.sbuf
        saved_off = sb.offset_buf.clone()
        saved_seen = sb.seen_tokens.buf.clone()
        self.slot_idx.fill_(-1)  # capture with every row padded: no state changes
        stream = torch.cuda.Stream(device=sb.device)
        stream.wait_stream(torch.cuda.current_stream(sb.device))
        for b in self.buckets:
            s = CudaGraphableSampler(sb, b)
            s.slot_idx = self.slot_idx[:b]
            with torch.cuda.stream(stream):
                s.sample(None, self.logits[:b])  # warm-up outside capture
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                s.sample(None, self.logits[:b])
            self._samplers[b], self._graphs[b] = s, g
        torch.cuda.current_stream(sb.device).wait_stream(stream)
        torch.cuda.synchronize(sb.device)
        sb.offset_buf.copy_(saved_off)
        sb.seen_tokens.buf.copy_(saved_seen)

    def bucket_for(self, n: int) -> int:
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(f"batch {n} exceeds the largest bucket {self.buckets[-1]}")

    def sample(self, rids, logits: torch.Tensor, masks=None) -> torch.Tensor:
        n = len(rids)
        b = self.bucket_for(n)
        self.sbuf.gather_for_request_ids(rids, n, gather_seen_tokens=masks is not None)
        if masks is not None:
            self.sbuf.stage_seen_token_masks(rids, masks)
        self.logits[:n].copy_(logits)
        self.slot_idx[:n].copy_(torch.arange(n, dtype=torch.int32))
        self.slot_idx[n:b].fill_(-1)
        self._graphs[b].replay()
        self._last = list(rids)
        return self._samplers[b].out[:n]

    def stopped(self, rids) -> list:
        """The requests of the last `sample` batch that sampled a stop token
        (SamplerBuffers.stopped over the bucket's rows)."""
        return self.sbuf.stopped(rids)

    def sync(self, rids, masks=None) -> None:
        sb = self.sbuf
        if masks is not None:
            for j, m in enumerate(masks):
                m.bits.copy_(sb.seen_tokens.buf[j])
        sb._store_offsets(list(rids))
