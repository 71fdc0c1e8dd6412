"""Byte geometry of the paged OSCAR cache over vLLM's native BF16 K/V stripes.

The format must stay byte-compatible with the reference (``oscar_ascend/layout.py:8-95``,
``docs/design.md:82-118``):

* INT2 history lives in the K stripe.  Token slot ``s`` of KV head ``h`` sits at
  ``(s // Bp) * J + ((s % Bp) * H + h) * 160`` bytes, with ``J = Bp * H * D * 2`` the
  stripe bytes of one physical page of ``Bp`` tokens.  Bytes 0..63 are K codes
  (4 per byte, LSB first), 64..65 K scale (fp16 LE), 66..67 K zero, 68..135 the same
  for V, 136..159 untouched padding.
* The BF16 window (sink + ring) of a request lives in the V stripe of the request's
  first physical page (``owner = block_table[0] // (Bp // 128)``), element offset
  ``owner * J/2 + ((idx * 2 + kv) * H + h) * D`` with ``idx = t`` for ``t < S`` and
  ``S + t % C`` otherwise.
* The page table is in 128-token kernel blocks: logical token ``t`` maps to slot
  ``table[t // 128] * 128 + t % 128``.

No tensor is allocated here; ``tensor_views`` reinterprets existing stripes.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .config import OscarConfig

KERNEL_BLOCK_TOKENS = 128


@dataclass(frozen=True)
class CacheLayout:
    physical_block_tokens: int
    kv_heads: int = 1
    kernel_block_tokens: int = KERNEL_BLOCK_TOKENS
    config: OscarConfig = field(default_factory=OscarConfig)

    def __post_init__(self):
        # Capacity rules of reference layout.py:15-28.
        if self.kv_heads <= 0 or self.physical_block_tokens <= 0:
            raise ValueError("invalid physical cache geometry")
        if self.physical_block_tokens % self.kernel_block_tokens:
            raise ValueError("physical block must be a multiple of the 128-token kernel block")
        if self.history_page_bytes > self.stripe_page_bytes:
            raise ValueError("INT2 slots do not fit the native K stripe page")
        if self.window_page_bytes > self.stripe_page_bytes:
            raise ValueError(
                f"the BF16 window needs {self.window_page_bytes} bytes per owner page but a "
                f"native V stripe page holds {self.stripe_page_bytes}; use a physical block "
                f"of at least {2 * self.config.window_tokens} tokens"
            )

    # --- sizes -------------------------------------------------------------
    @property
    def stripe_page_bytes(self) -> int:
        return self.physical_block_tokens * self.kv_heads * self.config.head_dim * 2

    @property
    def history_page_bytes(self) -> int:
        return self.physical_block_tokens * self.kv_heads * self.config.slot_bytes

    @property
    def window_page_bytes(self) -> int:
        return self.config.window_tokens * 2 * self.kv_heads * self.config.head_dim * 2

    @property
    def blocks_per_page(self) -> int:
        return self.physical_block_tokens // self.kernel_block_tokens

    # --- addresses -----------------------------------------------------------
    def slot_offset(self, slot: int, head: int = 0) -> int:
        """Byte offset of (slot, head) in the K stripe."""
        if slot < 0 or not 0 <= head < self.kv_heads:
            raise ValueError("invalid slot/head")
        page, position = divmod(slot, self.physical_block_tokens)
        return page * self.stripe_page_bytes + (position * self.kv_heads + head) * self.config.slot_bytes

    def logical_slot(self, block_table, position: int) -> int:
        block, token = divmod(position, self.kernel_block_tokens)
        return int(block_table[block]) * self.kernel_block_tokens + token

    def window_index(self, position: int) -> int:
        cfg = self.config
        return position if position < cfg.sink_tokens else cfg.sink_tokens + position % cfg.ring_tokens

    def window_offset(self, first_kernel_block: int, position: int, kv: int = 0, head: int = 0) -> int:
        """Byte offset of window token ``position`` (kv 0 = K, 1 = V) in the V stripe."""
        if position < 0 or kv not in (0, 1) or not 0 <= head < self.kv_heads:
            raise ValueError("invalid window position/head")
        if first_kernel_block < 0 or first_kernel_block % self.blocks_per_page:
            raise ValueError("the first kernel block must start a physical page")
        owner = first_kernel_block // self.blocks_per_page
        index = self.window_index(position)
        return (
            owner * self.stripe_page_bytes
            + ((index * 2 + kv) * self.kv_heads + head) * self.config.head_dim * 2
        )

    # --- views -------------------------------------------------------------
    def tensor_views(self, kv_cache):
        """(history bytes, window bf16) flat views over the native (K, V) stripes.

        Accepts a ``(K, V)`` pair or a tensor whose leading dimension is 2, each
        stripe contiguous BF16 ``[num_blocks, 128, H, D]`` (reference layout.py:75-95).
        """
        import torch

        if isinstance(kv_cache, torch.Tensor):
            if kv_cache.ndim != 5 or kv_cache.shape[0] != 2:
                raise ValueError("expected a (2, num_blocks, 128, H, D) cache tensor")
            kv_cache = (kv_cache[0], kv_cache[1])
        if not isinstance(kv_cache, (tuple, list)) or len(kv_cache) != 2:
            raise ValueError("expected native (K, V) cache views")
        k, v = kv_cache
        expect = (self.kernel_block_tokens, self.kv_heads, self.config.head_dim)
        for tensor in (k, v):
            if tensor.dtype != torch.bfloat16 or not tensor.is_contiguous():
                raise ValueError("OSCAR needs contiguous BF16 K/V stripes")
            if tensor.ndim != 4 or tuple(tensor.shape[1:]) != expect:
                raise ValueError(f"unexpected native cache shape {tuple(tensor.shape)}")
            if tensor.numel() * tensor.element_size() % self.stripe_page_bytes:
                raise ValueError("native stripe is not a whole number of physical pages")
        if k.shape != v.shape:
            raise ValueError("K/V stripes must have identical geometry")
        return k.view(torch.uint8).view(-1), v.view(-1)
