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
NCCL all-gather.  Rows whose shard set exceeds ``tp_cap`` (top_k off over a
flat shard) report ``STATUS_TP_OVERFLOW``; size ``tp_cap`` to the largest
top_k in use.
"""
from __future__ import annotations

from typing import Callable

import torch

from . import _native as N
from . import kernel


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

    ``gather(recv, send)`` all-gathers ``send`` ([B * words] int32) from every
    rank into ``recv`` ([world, B * words], rank-major); by default it is a
    torch.distributed all-gather over ``group``.
    """

    def __init__(self, max_bs: int, V_global: int, world: int, rank: int, device, tp_cap: int = 64,
                 group=None, gather: Callable[[torch.Tensor, torch.Tensor], None] | None = None):
        if tp_cap < 1:
            raise ValueError("tp_cap must be >= 1")
        self.max_bs, self.V_global, self.world, self.rank = max_bs, V_global, world, rank
        self.tp_cap = tp_cap
        self.device = torch.device(device)
        self.words = kernel.tp_record_words(tp_cap)
        self.send = torch.zeros(max_bs * self.words, dtype=torch.int32, device=self.device)
        self.recv = torch.zeros(world * max_bs * self.words, dtype=torch.int32, device=self.device)
        self.gather = gather if gather is not None else _default_gather(group)

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
        send = self.local(logits, vocab_offset, **{k: v for k, v in params.items() if k != "flags"})
        recv = self.recv[: self.world * B * self.words]  # contiguous [world, B * words]
        self.gather(recv, send)
        self.merge(logits, vocab_offset, recv, out_ids=out_ids, **params)
        return out_ids


def status_overflowed(status: torch.Tensor) -> torch.Tensor:
    return (status & N.STATUS_TP_OVERFLOW) != 0
