"""OSCAR INT2 KV-cache parameters and the small host-side policies around them.

The parameter names, environment variables, validation rules and derived sizes
follow the reference plugin's ``oscar_ascend/config.py:8-106`` so that a
deployment configured for the Ascend plugin keeps its meaning here:

* one quantisation group per D=256 vector: 64 code bytes + fp16 scale + fp16 zero
  (``data_bytes`` = 64, ``vector_bytes`` = 68), K then V, padded to a 32-byte
  multiple (``slot_bytes`` = 160);
* a BF16 window of ``sink_tokens`` + a ring of ``recent + speculative + 1`` tokens;
* percentile clipping with ``torch.quantile`` (linear interpolation) semantics.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass


@dataclass(frozen=True)
class OscarConfig:
    """Static OSCAR parameters (reference ``config.py:8-63``)."""

    head_dim: int = 256
    group_size: int = 256
    sink_tokens: int = 64
    recent_tokens: int = 256
    speculative_tokens: int = 3
    k_clip_ratio: float = 0.96
    v_clip_ratio: float = 0.92
    clip_mode: str = "percentile"
    k_clip_factor: float = 1.0
    v_clip_factor: float = 1.0
    k_rotation_path: str = ""
    v_rotation_path: str = ""
    block_n: int = 32
    queries_per_tile: int = 4

    def __post_init__(self):
        # Same acceptance rules as reference config.py:25-43.
        if self.head_dim != 256 or self.group_size < self.head_dim:
            raise ValueError("OSCAR INT2 requires D=256 with a single quantisation group")
        if min(self.sink_tokens, self.recent_tokens, self.speculative_tokens) < 0:
            raise ValueError("sink/recent/speculative token counts must be >= 0")
        if self.speculative_tokens > 15:
            raise ValueError("at most 15 speculative tokens are supported")
        if self.clip_mode not in ("percentile", "factor"):
            raise ValueError("clip mode must be 'percentile' or 'factor'")
        for ratio in (self.k_clip_ratio, self.v_clip_ratio):
            if not math.isfinite(ratio) or not (ratio == 0 or 0.875 <= ratio <= 1):
                raise ValueError("clip percentile must be 0 (off) or within [0.875, 1]")
        for factor in (self.k_clip_factor, self.v_clip_factor):
            if not math.isfinite(factor) or not 0 < factor <= 1:
                raise ValueError("fixed clip factors must lie in (0, 1]")
        if self.block_n not in (16, 32):
            raise ValueError("block_n must be 16 or 32")
        if self.queries_per_tile not in (1, 2, 4):
            raise ValueError("queries_per_tile must be 1, 2 or 4")

    # --- derived byte geometry -------------------------------------------------
    @property
    def data_bytes(self) -> int:
        """Packed code bytes of one vector: 4 two-bit codes per byte."""
        return self.head_dim // 4

    @property
    def vector_bytes(self) -> int:
        """Codes + fp16 scale + fp16 zero."""
        return self.data_bytes + 4

    @property
    def slot_bytes(self) -> int:
        """K vector + V vector, rounded up to a 32-byte multiple (160 at D=256)."""
        return -(-2 * self.vector_bytes // 32) * 32

    @property
    def ring_tokens(self) -> int:
        return self.recent_tokens + self.speculative_tokens + 1

    @property
    def window_tokens(self) -> int:
        return self.sink_tokens + self.ring_tokens

    @classmethod
    def from_env(cls, speculative_tokens: int = 3) -> "OscarConfig":
        """Read the reference's environment names (reference ``config.py:66-81``)."""
        env = os.environ.get
        return cls(
            group_size=int(env("VLLM_OSCAR_GROUP_SIZE", "256")),
            sink_tokens=int(env("VLLM_OSCAR_SINK_TOKENS", "64")),
            recent_tokens=int(env("VLLM_OSCAR_RECENT_TOKENS", "256")),
            speculative_tokens=speculative_tokens,
            k_clip_ratio=float(env("VLLM_OSCAR_K_CLIP_RATIO", "0.96")),
            v_clip_ratio=float(env("VLLM_OSCAR_V_CLIP_RATIO", "0.92")),
            clip_mode=env("OSCAR_ASCEND_CLIP_MODE", "percentile"),
            k_clip_factor=float(env("OSCAR_ASCEND_K_CLIP_FACTOR", "1")),
            v_clip_factor=float(env("OSCAR_ASCEND_V_CLIP_FACTOR", "1")),
            k_rotation_path=env("VLLM_OSCAR_K_ROTATION_PATH", ""),
            v_rotation_path=env("VLLM_OSCAR_V_ROTATION_PATH", ""),
            block_n=int(env("OSCAR_ASCEND_BLOCK_N", "32")),
            queries_per_tile=int(env("OSCAR_ASCEND_QUERY_TILE", "4")),
        )


def choose_splits(num_requests: int, num_kv_heads: int, max_query_len: int) -> int:
    """Split-KV count (reference ``config.py:84-89``): scratch is bounded by the
    current tokens, never by the device-resident context length."""
    if max_query_len > 16:
        return 1
    parallel = num_requests * num_kv_heads
    if parallel <= 8:
        return 32
    if parallel <= 32:
        return 16
    return 8


def decode_split_cap(num_requests: int, num_kv_heads: int, max_query_len: int, num_tokens: int,
                     num_q_heads: int, scratch_bytes: int = 256 << 20) -> int:
    """Most KV splits a decode / verify step may use.  The device balances splits per
    request (a long request gets more, a short one fewer, all splits of similar
    length), so the cap only bounds the fp32 split scratch [tokens, Hq, splits+1, 256]:
    the reference policy (``choose_splits``) is the floor, raised up to 64 while the
    scratch stays under ``scratch_bytes``."""
    base = choose_splits(num_requests, num_kv_heads, max_query_len)
    if max_query_len > 16:
        return base
    fit = scratch_bytes // max(num_tokens * num_q_heads * 256 * 4, 1) - 1
    return max(base, min(64, fit))


def percentile_selection(ratio: float, dim: int = 256):
    """Descending ranks (low, high) and weight of the linear quantile
    (reference ``config.py:92-97``).

    ``torch.quantile`` interpolates between ascending-sorted elements
    ``floor(r)`` and ``ceil(r)`` with ``r = (dim-1)*ratio``; in descending order
    those are ranks ``dim-1-floor(r)`` (the smaller value) and ``dim-1-ceil(r)``.
    """
    index = (dim - 1) * ratio
    lower, upper = math.floor(index), math.ceil(index)
    return dim - 1 - lower, dim - 1 - upper, index - lower


def quantile_weight_f32(ratio: float, dim: int = 256):
    """The exact fp32 interpolation weight ``torch.quantile`` uses.

    ATen converts the quantile to the input dtype (fp32) before multiplying by
    ``dim-1``; the weight is that fp32 rank minus its floor, in fp32.  Returns
    ``(ascending_low_index, ascending_high_index, weight_f32)``.
    """
    import numpy as np

    rank = np.float32(ratio) * np.float32(dim - 1)
    lo = int(np.floor(rank))
    hi = int(np.ceil(rank))
    return lo, hi, float(np.float32(rank - np.float32(lo)))


def task_capacity(tokens: int, requests: int, query_tile: int) -> int:
    """Upper bound of (request, query-tile) tasks (reference ``config.py:100-101``)."""
    return min(tokens, (tokens + query_tile - 1) // query_tile + requests - 1)


def attention_programs(tokens: int, requests: int, query_tile: int) -> int:
    """Task slots a launch must cover (reference ``config.py:104-106``)."""
    return max(1, task_capacity(tokens, requests, query_tile))
