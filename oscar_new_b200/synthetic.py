"""Seeded synthetic inputs in the shapes of the OSCAR benchmark configurations.

No dataset or checkpoint is available offline, so the measurement and parity harness
use these generators (seeds are part of every result):

* Q/K/V: bf16 N(0,1); channels 0..7 of K scaled by 20 (outlier channels).
* rotations: Q of a seeded Gaussian QR with the sign of diag(R) folded in, composed with
  the normalised Sylvester Hadamard matrix (K seed 1, V seed 2 by default).
* paging: physical pages of ``Bp`` tokens handed out through a seeded permutation; a
  request's kernel blocks run consecutively inside each of its pages, and its first
  block starts a page (the window owner).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from types import SimpleNamespace

import torch

from .config import task_capacity


def hadamard(dim: int = 256) -> torch.Tensor:
    h = torch.ones(1, 1)
    while h.shape[0] < dim:
        h = torch.cat((torch.cat((h, h), 1), torch.cat((h, -h), 1)), 0)
    return h / math.sqrt(dim)


def orthogonal(seed: int, dim: int = 256) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    q, r = torch.linalg.qr(torch.randn(dim, dim, generator=gen))
    return q * torch.sign(torch.diagonal(r))[None, :]


def rotation(seed: int, dim: int = 256) -> torch.Tensor:
    """fp32 orthogonal * Hadamard."""
    return orthogonal(seed, dim) @ hadamard(dim)


def outlier_bf16(gen: torch.Generator, *shape, channels: int = 8, factor: float = 20.0, device="cpu"):
    x = torch.randn(*shape, generator=gen)
    x[..., :channels] *= factor
    return x.bfloat16().to(device)


@dataclass
class PagedPlan:
    """Page ownership and per-step metadata for a batch of requests (host tensors)."""

    seq_lens: list
    query_lens: list
    block_tables: torch.Tensor  # int32 [max_reqs, cols]
    query_start_loc: torch.Tensor  # int32 [max_reqs + 1]
    slot_mapping: torch.Tensor  # int64 [num_tokens] (slots of the current tokens)
    counts: torch.Tensor  # int32 [2]
    num_pages: int
    max_reqs: int

    def meta(self, device, query_tile: int = 4, tasks_capacity: int | None = None):
        n = int(self.counts[1])
        cap = tasks_capacity or task_capacity(max(n, 1), self.max_reqs, query_tile)
        seq = torch.zeros(self.max_reqs, dtype=torch.int32)
        seq[: len(self.seq_lens)] = torch.tensor(self.seq_lens, dtype=torch.int32)
        return SimpleNamespace(
            query_start_loc=self.query_start_loc.to(device),
            seq_lens=seq.to(device),
            block_tables=self.block_tables.to(device),
            slot_mapping=self.slot_mapping.to(device),
            counts=self.counts.to(device),
            num_reqs=len(self.seq_lens),
            max_num_reqs=self.max_reqs,
            max_query_len=max(self.query_lens) if self.query_lens else 0,
            tasks=torch.full((cap, 2), -1, dtype=torch.int32, device=device),
            task_count=torch.zeros(1, dtype=torch.int32, device=device),
        )

    def slots_of(self, req: int, positions) -> torch.Tensor:
        row = self.block_tables[req]
        pos = torch.as_tensor(positions, dtype=torch.int64)
        return row[pos // 128].long() * 128 + pos % 128


def plan_pages(seq_lens, query_lens, block_tokens: int, seed: int = 0, spare_pages: int = 1,
               max_reqs: int | None = None) -> PagedPlan:
    """Seeded random page permutation; page 0 is never handed out."""
    per_page = block_tokens // 128
    need = [-(-s // block_tokens) for s in seq_lens]
    num_pages = sum(need) + spare_pages + 1
    gen = torch.Generator().manual_seed(seed)
    perm = (torch.randperm(num_pages - 1, generator=gen) + 1).tolist()
    max_reqs = max_reqs or len(seq_lens) + 1
    cols = max(1, max(need, default=1) * per_page)
    table = torch.zeros((max_reqs, cols), dtype=torch.int32)
    qstarts = [0]
    slots = []
    for i, (s, q) in enumerate(zip(seq_lens, query_lens)):
        own, perm = perm[: need[i]], perm[need[i] :]
        blocks = [p * per_page + j for p in own for j in range(per_page)]
        if blocks:
            table[i, : len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
        for t in range(s - q, s):
            slots.append(blocks[t // 128] * 128 + t % 128)
        qstarts.append(qstarts[-1] + q)
    qs = torch.full((max_reqs + 1,), qstarts[-1], dtype=torch.int32)
    qs[: len(qstarts)] = torch.tensor(qstarts, dtype=torch.int32)
    return PagedPlan(
        seq_lens=list(seq_lens),
        query_lens=list(query_lens),
        block_tables=table,
        query_start_loc=qs,
        slot_mapping=torch.tensor(slots, dtype=torch.int64),
        counts=torch.tensor([len(seq_lens), qstarts[-1]], dtype=torch.int32),
        num_pages=num_pages,
        max_reqs=max_reqs,
    )


def cache_stripes(num_pages: int, block_tokens: int, kv_heads: int, device, sentinel: int = 0x5A):
    """Native vLLM-style cache [2, num_blocks, 128, H, 256] bf16, filled with a byte
    sentinel so that untouched bytes can be checked."""
    blocks = num_pages * (block_tokens // 128)
    raw = torch.full((2 * blocks * 128 * kv_heads * 256 * 2,), sentinel, dtype=torch.uint8, device=device)
    return raw.view(torch.bfloat16).view(2, blocks, 128, kv_heads, 256)
