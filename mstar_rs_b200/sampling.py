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

    def __setattr__(self, name, value) -> None:
        object.__setattr__(self, name, value)
        owner = self.__dict__.get("_owner")
        if owner is not None and not name.startswith("_"):  # the sampler re-reads this config
            owner._mark_dirty()

    def set_seed(self, seed) -> None:
        self.seed = None if seed is None else int(seed)

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
        self._row = None  # (SamplerBuffers, row) while the bits live in a step row

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
    """Per-slot sampling parameters: a host mirror and one packed device
    table whose sections are the kernel's per-slot arrays (temperature,
    top_k, top_p, min_p, repetition / presence / frequency penalties, seed,
    stop ids).  An upload copies the whole table from pinned memory without
    blocking the host (torch's pinned allocator keeps the buffer alive until
    the copy has run), so it may sit between CUDA-graph replays."""

    NAMES = ("temperature", "top_p", "min_p", "rep_pen", "pres_pen", "freq_pen")
    NSTOP = 4  # stop ids per slot
    _F32 = {"temperature": 0, "top_p": 2, "min_p": 3, "rep_pen": 4, "pres_pen": 5, "freq_pen": 6}
    _K, _SEED, _STOP = 1, 8, 10  # section starts, in rows of n int32 words

    def __init__(self, n: int, device):
        self.n = n
        self.device = device
        words = (self._STOP + self.NSTOP) * n
        self.host_words = np.zeros(words, np.int32)
        self.dev_words = torch.zeros(words, dtype=torch.int32, device=device)
        sec = lambda i, k=1: self.host_words[i * n:(i + k) * n]  # noqa: E731
        self.host = {k: sec(i).view(np.float32) for k, i in self._F32.items()}
        self.host["temperature"][:] = 1.0
        self.host["top_p"][:] = 1.0
        self.host["rep_pen"][:] = 1.0
        self.host_k = sec(self._K)
        self.host_seed = sec(self._SEED, 2).view(np.int64)
        self.host_stop = sec(self._STOP, self.NSTOP).reshape(n, self.NSTOP)
        self.host_stop[:] = -1
        dsec = lambda i, k=1: self.dev_words[i * n:(i + k) * n]  # noqa: E731
        self.dev = {k: dsec(i).view(torch.float32) for k, i in self._F32.items()}
        self.dev_k = dsec(self._K)
        self.dev_seed = dsec(self._SEED, 2).view(torch.int64)
        self.dev_stop = dsec(self._STOP, self.NSTOP).view(n, self.NSTOP)
        self._keys = [None] * n
        self.dirty = True

    @staticmethod
    def key(cfg: SamplingConfig) -> tuple:
        stops = () if cfg.ignore_eos or cfg.stop_token_ids is None else cfg.stop_token_ids
        if isinstance(stops, int):
            stops = (stops,)
        return (float(cfg.temperature), int(cfg.top_k), float(cfg.top_p), float(cfg.min_p),
                float(cfg.repetition_penalty), float(cfg.presence_penalty), float(cfg.frequency_penalty),
                cfg.seed, tuple(int(t) for t in stops))

    def write(self, i: int, cfg: SamplingConfig) -> None:
        k = self.key(cfg)
        if self._keys[i] == k:
            return
        T, top_k, top_p, min_p, rep, pres, freq, seed, stops = k
        if len(stops) > self.NSTOP or any(t < 0 for t in stops):  # checked before any field changes
            raise ValueError(f"stop_token_ids takes at most {self.NSTOP} non-negative ids, got {list(stops)}")
        greedy = T < _SAMPLING_EPS
        self.host["temperature"][i] = 0.0 if greedy else T
        self.host_k[i] = 1 if greedy else top_k
        self.host["top_p"][i] = top_p
        self.host["min_p"][i] = min_p
        self.host["rep_pen"][i] = rep
        self.host["pres_pen"][i] = pres
        self.host["freq_pen"][i] = freq
        s = 0 if seed is None else seed
        self.host_seed[i] = np.int64(np.uint64(s & 0xFFFFFFFFFFFFFFFF).view(np.int64))
        self.host_stop[i] = -1
        self.host_stop[i, : len(stops)] = stops
        self._keys[i] = k
        self.dirty = True

    def upload(self) -> None:
        if not self.dirty:
            return
        src = torch.from_numpy(self.host_words)
        if self.dev_words.is_cuda:
            self.dev_words.copy_(src.pin_memory(), non_blocking=True)
        else:  # (a host table, for tests without a device)
            self.dev_words.copy_(src)
        self.dirty = False

    def kwargs(self) -> dict:
        return dict(temperature=self.dev["temperature"], top_k=self.dev_k, top_p=self.dev["top_p"],
                    min_p=self.dev["min_p"], rep_pen=self.dev["rep_pen"], pres_pen=self.dev["pres_pen"],
                    freq_pen=self.dev["freq_pen"], seed=self.dev_seed, stop_ids=self.dev_stop)


def _pinned(values, dtype) -> torch.Tensor:
    """A pinned host tensor holding `values` (a source for a non-blocking
    upload: torch's pinned allocator keeps it alive until the copy ran)."""
    return torch.tensor(values, dtype=dtype).pin_memory()


def _tp_world(group) -> int:
    """World size of a tensor-parallel group (None or a one-rank group: 1)."""
    if group is None:
        return 1
    import torch.distributed as dist

    if isinstance(group, dist.ProcessGroup):
        return dist.get_world_size(group)
    size = getattr(group, "world_size", None)
    if isinstance(size, int):
        return size
    if callable(getattr(group, "size", None)):
        return int(group.size())
    import torch.distributed as dist

    try:
        return dist.get_world_size(group) if dist.is_initialized() else 1
    except (RuntimeError, ValueError, TypeError):  # not a process group: a one-rank stand-in
        return 1


def _tp_agree(group, ids: torch.Tensor) -> None:
    """Make every rank of `group` hold rank 0's sampled ids: the reference's
    tp_group broadcast (python/mstar_rs/models/qwen3_omni.py:401-404), which
    keeps Thinker ranks from drifting apart on tied logits.  One broadcast
    of the [n] ids, capturable in a CUDA graph with NCCL."""
    import torch.distributed as dist

    if isinstance(group, dist.ProcessGroup):
        dist.broadcast(ids, src=dist.get_global_rank(group, 0), group=group)
    else:  # a communicator object of the engine's own (broadcast(tensor, src))
        group.broadcast(ids, 0)


class Sampler:
    """Eager per-request sampler (prefill and non-graph decode).

    Each request owns a slot: parameters, RNG (seed, offset) and a ring of
    its last `history` generated ids (repetition / presence / frequency
    penalties count over it).  `sample` reads the slots through an index
    vector, so requests can be sampled in any order or subset.  Nothing here
    waits for the device: parameter and index uploads go out from pinned
    memory.  With a `tp_group` of more than one rank, rank 0's ids are
    broadcast before the per-slot state takes them (`mstar_sampler_commit`)."""

    def __init__(self, device=None, tp_group=None, max_requests: int = 256, history: int = 1024,
                 vocab_size: int | None = None):
        self.device = torch.device(device if device is not None else "cuda")
        if self.device.type != "cuda":
            raise ValueError("the sampler runs on CUDA devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.tp_group = tp_group
        self.tp_world = _tp_world(tp_group)
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
        self._dirty = False

    def _mark_dirty(self) -> None:
        self._dirty = True  # a request's config changed: its row is rewritten before the next step

    def _flush(self) -> None:
        if self._dirty:
            for rid, cfg in self._sampling_config.items():
                self.params.write(self._slot[rid], cfg)
            self._dirty = False

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
        # (fills, not element assignments: those copy a host scalar and wait)
        self.offset[s:s + 1].zero_()
        self.hist_len[s:s + 1].zero_()
        self.stop_flags[s:s + 1].zero_()
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
        row = [-1] * self.H
        row[: len(ids)] = [int(t) for t in ids]
        self.hist[s].copy_(_pinned(row, torch.int32), non_blocking=True)
        self.hist_len[s:s + 1].fill_(len(ids))

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
            t = torch.empty(len(rids), dtype=torch.int32, device=self.device)
            t.copy_(_pinned([self._slot[r] for r in rids], torch.int32), non_blocking=True)
            self._idx_cache[key] = t
        return t

    def sample(self, rids, logits: torch.Tensor, apply_penalty: bool = True) -> torch.Tensor:
        """logits [n, V] (bf16 or fp32, on this sampler's device) -> ids [n] int64."""
        n = len(rids)
        if logits.dim() == 1:
            logits = logits.unsqueeze(0)
        if logits.shape[0] != n:
            raise ValueError(f"{n} request ids for {logits.shape[0]} logits rows")
        self._flush()
        self.params.upload()
        out = torch.empty(n, dtype=torch.int64, device=self.device)
        idx = self._index(rids)
        state = N.FLAG_UPDATE_HISTORY if apply_penalty else 0
        hist = dict(hist_ids=self.hist, hist_len=self.hist_len) if apply_penalty else {}
        pk = self.params.kwargs()
        if self.tp_world == 1:
            kernel.sampler_step(logits, slot_idx=idx, num_slots=self.max_requests, **pk, offset=self.offset,
                                **hist, out_ids=out, stop_flags=self.stop_flags,
                                flags=N.FLAG_ADVANCE_OFFSET | state)
            return out
        stop_ids = pk.pop("stop_ids")
        kernel.sampler_step(logits, slot_idx=idx, num_slots=self.max_requests, **pk, offset=self.offset,
                            **hist, out_ids=out, flags=N.FLAG_ADVANCE_OFFSET)
        _tp_agree(self.tp_group, out)
        kernel.commit(out, slot_idx=idx, num_slots=self.max_requests, V=logits.shape[1], **hist,
                      stop_ids=stop_ids, stop_flags=self.stop_flags, flags=state)
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
        if sb.tp_world == 1:
            kernel.sampler_step(logits, num_slots=sb.max_bs, **kw, offset=sb.offset_buf,
                                seen_bits=sb.seen_tokens.buf, out_ids=self.out, slot_idx=self.slot_idx,
                                stop_flags=sb.stop_flags, flags=N.FLAG_ADVANCE_OFFSET | N.FLAG_UPDATE_SEEN)
            return self.out
        stop_ids = kw.pop("stop_ids")
        kernel.sampler_step(logits, num_slots=sb.max_bs, **kw, offset=sb.offset_buf, seen_bits=sb.seen_tokens.buf,
                            out_ids=self.out, slot_idx=self.slot_idx, flags=N.FLAG_ADVANCE_OFFSET)
        _tp_agree(sb.tp_group, self.out)
        kernel.commit(self.out, slot_idx=self.slot_idx, num_slots=sb.max_bs, V=logits.shape[1],
                      seen_bits=sb.seen_tokens.buf, stop_ids=stop_ids, stop_flags=sb.stop_flags,
                      flags=N.FLAG_UPDATE_SEEN)
        return self.out

    def stopped(self) -> list:
        """The gathered requests that sampled a stop token since the flags
        were last read (see SamplerBuffers.stopped)."""
        return self.sbuf.stopped(self._rids)

    def sync_seen_token_masks(self, masks) -> None:
        """Hand the step rows' seen bits (updated in-graph) back to the
        per-request masks.  Masks staged by this SamplerBuffers already live
        in their rows (SeenTokenMask.bits is a view of the row), so there is
        nothing to copy; RNG offsets stay in the rows while their requests do."""
        self.sbuf._sync_masks(self._rids, masks)


class SamplerBuffers:
    """Fixed-shape step buffers for in-graph sampling of up to max_bs rows.

    The rows hold the in-graph state the kernel reads and advances: per-row
    parameters, RNG offsets (`offset_buf`), seen bits (`seen_tokens.buf`) and
    stop flags, as in the reference (orpheus.py:341-359, :419-426).  The
    state stays in a row while the same request occupies it: staging,
    gathering and syncing the same requests again (every decode step) copies
    nothing and never waits for the device.  A request's state moves only when
    its row changes: its RNG offset goes to a per-request table on the device
    and comes back from it, and its SeenTokenMask is bound to the row it is
    staged into (`mask.bits` becomes a view of that row, so the engine's own
    `add_tokens` writes reach the kernel) and given its own copy when it
    leaves the row."""

    def __init__(self, max_bs: int, device, tp_group=None, vocab_size: int | None = None, seen_cap: int = 0,
                 max_requests: int = 4096):
        self.max_bs = max_bs
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.tp_group = tp_group
        self.tp_world = _tp_world(tp_group)
        self.vocab_size = vocab_size or 1
        self.seen_cap = seen_cap
        self.max_requests = max_requests
        self.params = _ParamTable(max_bs, self.device)
        self.offset_buf = torch.zeros(max_bs, dtype=torch.int64, device=self.device)
        self.seen_tokens = _SeenTokens(max_bs, self.vocab_size, self.device)
        self.stop_flags = torch.zeros(max_bs, dtype=torch.int32, device=self.device)  # per step row
        self._req_off = torch.zeros(max_requests, dtype=torch.int64, device=self.device)
        self._req_slot: dict = {}
        self._free = list(range(max_requests - 1, -1, -1))
        self._row_rid: list = [None] * max_bs   # the request whose state a row holds
        self._row_mask: list = [None] * max_bs  # the mask bound to a row
        self._rows: list = []
        self._cfg: dict = {}
        self._cfg_dirty = True
        self._samplers: dict = {}

    @classmethod
    def allocate(cls, max_bs: int, device, tp_group=None, vocab_size: int | None = None) -> "SamplerBuffers":
        return cls(max_bs, device, tp_group=tp_group, vocab_size=vocab_size)

    def _mark_dirty(self) -> None:
        self._cfg_dirty = True  # a registered config changed: rows are compared at the next gather

    def register_request(self, rid, cfg: SamplingConfig) -> None:
        if cfg._owner is None:
            object.__setattr__(cfg, "_owner", self)
        self._cfg[rid] = cfg
        self._cfg_dirty = True
        if rid not in self._req_slot:
            if not self._free:
                raise RuntimeError(f"SamplerBuffers full ({self.max_requests} requests)")
            s = self._free.pop()
            self._req_slot[rid] = s
            self._req_off[s:s + 1].zero_()  # a fixed seed reproduces per request

    def unregister_request(self, rid) -> None:
        self._cfg.pop(rid, None)
        s = self._req_slot.pop(rid, None)
        if s is not None:
            self._free.append(s)
        for j, r in enumerate(self._row_rid):
            if r == rid:
                self._row_rid[j] = None
                self._release_row(j)

    def _release_row(self, j: int) -> None:
        """Give the mask bound to row j its own storage (rare: the row is
        about to hold another request, or its request left)."""
        m = self._row_mask[j]
        if m is not None:
            m.bits = m.bits.clone()
            m._row = None
            self._row_mask[j] = None

    def stage_seen_token_masks(self, rids, masks) -> None:
        masks = list(masks)
        if masks == self._row_mask[: len(masks)]:  # every mask already lives in its row
            return
        rows = self.seen_tokens.buf
        moving = [j for j, m in enumerate(masks) if self._row_mask[j] is not m]
        if not moving:
            return
        # every mask that moves, and every mask a moving one displaces, first
        # gets its own storage; then the moving masks enter their rows
        for j in moving:
            m = masks[j]
            k = getattr(m, "_row", None)
            if k is not None and k[0] is self:
                self._release_row(k[1])
            self._release_row(j)
        for j in moving:
            m = masks[j]
            rows[j].copy_(m.bits)
            m.bits = rows[j]
            m._row = (self, j)
            self._row_mask[j] = m

    def _sync_masks(self, rids, masks) -> None:
        masks = list(masks)
        if masks == self._row_mask[: len(masks)]:
            return
        rows = self.seen_tokens.buf
        for j, m in enumerate(masks):
            if self._row_mask[j] is not m:  # not staged here: copy the row back
                m.bits.copy_(rows[j])

    def gather_for_request_ids(self, rids, n: int, gather_seen_tokens: bool = True) -> CudaGraphableSampler:
        if len(rids) != n or n > self.max_bs:
            raise ValueError(f"gather of {len(rids)} ids into {n} rows (max {self.max_bs})")
        rids = list(rids)
        same = rids == self._rows
        if not same or self._cfg_dirty:
            for j, rid in enumerate(rids):
                self.params.write(j, self._cfg[rid])
            self.params.upload()
            self._cfg_dirty = False
        moved = [] if same else [j for j, rid in enumerate(rids) if self._row_rid[j] != rid]
        if moved:
            # RNG offsets: a row's previous request keeps its offset in the
            # per-request table, the arriving request brings its own
            old = [(j, self._req_slot[self._row_rid[j]]) for j in moved
                   if self._row_rid[j] is not None and self._row_rid[j] in self._req_slot]
            if old:
                rows_t = torch.empty(len(old), dtype=torch.int64, device=self.device)
                rows_t.copy_(_pinned([j for j, _ in old], torch.int64), non_blocking=True)
                slots_t = torch.empty(len(old), dtype=torch.int64, device=self.device)
                slots_t.copy_(_pinned([s for _, s in old], torch.int64), non_blocking=True)
                self._req_off.index_copy_(0, slots_t, self.offset_buf.index_select(0, rows_t))
            rows_t = torch.empty(len(moved), dtype=torch.int64, device=self.device)
            rows_t.copy_(_pinned(moved, torch.int64), non_blocking=True)
            slots_t = torch.empty(len(moved), dtype=torch.int64, device=self.device)
            slots_t.copy_(_pinned([self._req_slot[rids[j]] for j in moved], torch.int64), non_blocking=True)
            self.offset_buf.index_copy_(0, rows_t, self._req_off.index_select(0, slots_t))
            self.stop_flags.index_fill_(0, rows_t, 0)  # rows now hold other requests: their stop flags start clear
            for j in moved:
                self._row_rid[j] = rids[j]
        if not gather_seen_tokens:  # the step starts from empty seen sets; the masks keep theirs
            for j in range(n):
                self._release_row(j)
            self.seen_tokens.buf[:n].zero_()
        self._rows = rids
        s = self._samplers.get(n)
        if s is None:
            s = CudaGraphableSampler(self, n)
            self._samplers[n] = s
        s._rids = rids
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


class SamplerGraphBuckets:
    """One captured CUDA graph per bucket size over fixed buffers, the way
    the reference's batched decode graphs pad a batch to the next bucket and
    discard the pad rows (python/mstar_rs/batched_graph.py:26-80,
    orpheus.py:322-366).  Pad rows carry slot -1: the kernel skips them (no
    sampling work, no state update).

    Usage: ``capture()`` once after ``SamplerBuffers.allocate``; then every
    step ``sample(rids, logits)`` stages the rows (outside any graph),
    replays the smallest bucket that holds them and returns the ids of the
    real rows.  The producer of the logits (the LM head) may write them
    straight into ``logits_for(n)``, in which case nothing is copied.
    ``sync(rids, masks)`` hands seen bits back to unbound masks."""

    def __init__(self, sbuf: SamplerBuffers, buckets=(1, 2, 4, 8, 16, 32, 64), dtype=torch.bfloat16):
        self.sbuf = sbuf
        self.buckets = sorted(b for b in set(buckets) if 1 <= b <= sbuf.max_bs)
        if not self.buckets:
            raise ValueError("no bucket fits max_bs")
        top = self.buckets[-1]
        self.logits = torch.zeros(top, sbuf.vocab_size, dtype=dtype, device=sbuf.device)
        self.slot_idx = torch.full((top,), -1, dtype=torch.int32, device=sbuf.device)
        # slot_idx pattern for n real rows in its bucket: 0 .. n-1, then -1
        ar = torch.arange(top, dtype=torch.int32, device=sbuf.device)
        self._patterns = torch.where(ar[None, :] < ar[:, None] + 1, ar[None, :], -1).to(torch.int32)
        self._n = None
        self._samplers = {}
        self._graphs = {}
        self._last = None

    def logits_for(self, n: int) -> torch.Tensor:
        """The buffer rows the graph of n requests reads: write logits here
        to skip the copy in `sample`."""
        return self.logits[:n]

    def capture(self) -> None:
        sb = self.sbuf
        saved_off = sb.offset_buf.clone()
        saved_seen = sb.seen_tokens.buf.clone()
        self.slot_idx.fill_(-1)  # capture with every row padded: no state changes
        self._n = None
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
        if logits.data_ptr() != self.logits.data_ptr() or logits.shape[0] != n:
            self.logits[:n].copy_(logits)
        if self._n != n:
            self.slot_idx.copy_(self._patterns[n - 1])
            self._n = n
        self._graphs[b].replay()
        self._last = list(rids)
        return self._samplers[b].out[:n]

    def stopped(self, rids) -> list:
        """The requests of the last `sample` batch that sampled a stop token
        (SamplerBuffers.stopped over the bucket's rows)."""
        return self.sbuf.stopped(rids)

    def sync(self, rids, masks=None) -> None:
        if masks is not None:
            self.sbuf._sync_masks(list(rids), masks)
