"""Vocab-parallel (tensor-parallel) sampling over a process group.

Each rank holds the logits of a contiguous vocabulary range (ids
[vocab_offset, vocab_offset + V_shard)).  One step is

  1. ``mstar_sampler_tp_local``: this shard's candidate record per row (its
     max, and its value-A set against that max, cut at top_k, as
     (value, global id) pairs);
  2. an all-gather of the fixed-size records over the group (52 KB per rank
     at B=128, top_k 50);
  3. ``mstar_sampler_tp_merge`` on every rank: the same merge, draw and state
     updates everywhere, so the sampled ids agree without a broadcast.

This replaces the reference's token broadcast across Thinker ranks
(python/mstar_rs/models/qwen3_omni.py:401-404, :408, :431).  All buffers are
allocated once, so a step can be captured in a CUDA graph together with the
NCCL all-gather.

With ``two_round=True`` rows without top_k (the Thinker's default whenever a
temperature is given, qwen3_omni.py:440-443) are sampled too: such a row's
shards send their first ``tp_cap`` members; rows with a shard cut short are
deferred by the first merge, every shard sends its exact A mass against the
row max (a second, 8-byte-per-row all-gather), and the second merge decides
them whenever the kept set or the draw lies among the members every shard
sent.  Rows it cannot decide report ``STATUS_TP_OVERFLOW``; with one round,
so does every row whose shard set exceeds ``tp_cap``.
"""
from __future__ import annotations

from typing import Callable

import torch

from . import _native as N
from . import kernel


# Default record capacities (members per shard and row).  One round: a row's
# top_k members must fit, and the Thinker's top_k rarely exceeds 64.  Two
# rounds: rows without top_k send their first members in order; 256 decide
# every row of a peaked 152k-vocabulary batch at tp 2 where 64 leave about one
# in ten to the overflow flag (the numpy restatement and the GPU agree on
# which rows), and the record stays under 2 KB per row.
TP_CAP = 64
TWO_ROUND_TP_CAP = 256


def _default_gather(group) -> Callable[[torch.Tensor, torch.Tensor], None]:
    import torch.distributed as dist

    def gather(recv: torch.Tensor, send: torch.Tensor) -> None:
        if dist.get_backend(group) == "nccl":
            dist.all_gather_into_tensor(recv, send, group=group)
        else:  # gloo has no all_gather_into_tensor for every dtype / device
            parts = list(recv.view(-1, send.numel()).unbind(0))
            dist.all_gather(parts, send, group=group)

    return gather


class VocabParallelSampler:
    """Fixed-shape vocab-parallel sampler for up to ``max_bs`` rows.

    ``tp_cap`` defaults to TP_CAP (one round) or TWO_ROUND_TP_CAP (two
    rounds), at most 2048 // world; world * tp_cap must not exceed 2048.  ``gather(recv, send)`` all-gathers ``send`` ([B * words] int32) from every
    rank into ``recv`` ([world, B * words], rank-major); by default it is a
    torch.distributed all-gather over ``group``.
    """

    def __init__(self, max_bs: int, V_global: int, world: int, rank: int, device, tp_cap: int | None = None,
                 group=None, gather: Callable[[torch.Tensor, torch.Tensor], None] | None = None,
                 two_round: bool = False, V_shard: int | None = None):
        if tp_cap is None:  # the merge holds at most 2048 members per row over all ranks
            tp_cap = min(TWO_ROUND_TP_CAP if two_round else TP_CAP, 2048 // max(1, world))
        if world * tp_cap > 2048:
            raise ValueError(f"world * tp_cap = {world * tp_cap} exceeds the 2048 members a merge holds per row")
        if tp_cap < 1:
            raise ValueError("tp_cap must be >= 1")
        if two_round and world > 16:
            raise ValueError("the two-round exchange takes at most 16 ranks")
        self.max_bs, self.V_global, self.world, self.rank = max_bs, V_global, world, rank
        self.tp_cap = tp_cap
        self.device = torch.device(device)
        self.words = kernel.tp_record_words(tp_cap)
        self.send = torch.zeros(max_bs * self.words, dtype=torch.int32, device=self.device)
        self.recv = torch.zeros(world * max_bs * self.words, dtype=torch.int32, device=self.device)
        self.gather = gather if gather is not None else _default_gather(group)
        self.two_round = two_round
        if two_round:
            vs = V_shard if V_shard is not None else -(-V_global // world)
            self.xbuf = torch.empty(max_bs * vs, dtype=torch.float32, device=self.device)
            self.pend = torch.zeros(2 * max_bs, dtype=torch.int32, device=self.device)
            self.send2 = torch.zeros(2 * max_bs, dtype=torch.int32, device=self.device)
            self.recv2 = torch.zeros(world * 2 * max_bs, dtype=torch.int32, device=self.device)

    def local(self, logits: torch.Tensor, vocab_offset: int, **params) -> torch.Tensor:
        """Step 1: this shard's records for the rows of ``logits``."""
        B = logits.shape[0]
        if B > self.max_bs:
            raise ValueError(f"batch {B} exceeds max_bs {self.max_bs}")
        send = self.send[: B * self.words]
        kernel.tp_local(logits, self.tp_cap, send, vocab_offset=vocab_offset, **params)
        return send

    def merge(self, logits: torch.Tensor, vocab_offset: int, recv: torch.Tensor, **params) -> None:
        """Step 3: merge the gathered records (``recv`` = [world, B * words])."""
        kernel.tp_merge(logits, self.tp_cap, self.world, self.V_global, recv, vocab_offset=vocab_offset, **params)

    def sample(self, logits: torch.Tensor, vocab_offset: int, out_ids: torch.Tensor, **params) -> torch.Tensor:
        """One vocab-parallel step; ``params`` are the per-slot parameters and
        state of ``kernel.sampler_step`` (temperature, top_k, ..., seed/offset
        or uniforms, history, flags)."""
        B = logits.shape[0]
        local = {k: v for k, v in params.items() if k not in ("flags", "out_status", "stop_ids", "stop_flags")}
        if not self.two_round:
            send = self.local(logits, vocab_offset, **local)
            recv = self.recv[: self.world * B * self.words]  # contiguous [world, B * words]
            self.gather(recv, send)
            self.merge(logits, vocab_offset, recv, out_ids=out_ids, **params)
            return out_ids
        if B > self.max_bs:
            raise ValueError(f"batch {B} exceeds max_bs {self.max_bs}")
        V = logits.shape[1]
        if self.xbuf.numel() < B * V:
            raise ValueError(f"shard of {V} ids exceeds the V_shard the sampler was built for")
        send = self.send[: B * self.words]
        xbuf = self.xbuf[: B * V]
        kernel.tp_local2(logits, self.tp_cap, send, xbuf, vocab_offset=vocab_offset, **local)
        recv = self.recv[: self.world * B * self.words]
        self.gather(recv, send)
        pend = self.pend[: 2 * B]
        kernel.tp_merge1(logits, self.tp_cap, self.world, self.V_global, recv, pend, vocab_offset=vocab_offset,
                         out_ids=out_ids, **params)
        send2 = self.send2[: 2 * B]
        kernel.tp_mass(logits, xbuf, pend, send2, vocab_offset=vocab_offset, **local)
        recv2 = self.recv2[: self.world * 2 * B]
        self.gather(recv2, send2)
        kernel.tp_merge2(logits, self.tp_cap, self.world, self.V_global, recv, recv2, pend,
                         vocab_offset=vocab_offset, out_ids=out_ids, **params)
        return out_ids


def status_overflowed(status: torch.Tensor) -> torch.Tensor:
    return (status & N.STATUS_TP_OVERFLOW) != 0
