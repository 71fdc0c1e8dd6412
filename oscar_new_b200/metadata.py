"""Per-step device metadata of the OSCAR backend: vLLM's attention metadata builder.

Contract kept from the reference builder (``oscar_ascend/metadata.py:36-170``):

* capacities fixed at start-up so CUDA graphs replay with new contents: ``max_num_seqs + 1``
  requests (graph padding may add a dummy row), the batched-token budget plus
  ``(speculative + 4)`` tail slots per request, ``ceil(max_model_len / 128) +
  blocks_per_page + 1`` block-table columns, and the task table those imply;
* the device counts ``[requests, active tokens]`` bound every kernel, and a step built
  inside :func:`dummy_run_scope` (graph capture, warm-up) stages zero counts, so its
  recorded kernels touch no cache page;
* steps with shared prefixes, non-causal attention, more requests / tokens / table
  columns than the capacities, or metadata that is not on the GPU are refused.

Structure here: the fixed metadata lives in ONE int32 arena on the device
(``StepBuffers``; counts, task count, query starts, sequence lengths, block table, task
table) plus one int64 slot buffer, and each step is staged by ONE native launch
(``oscar_stage_step_metadata``) instead of separate copies, fills and a task-table
kernel.  The builder never reads device memory on the host.
"""

from __future__ import annotations

import contextlib
import contextvars
import math
from dataclasses import dataclass

import torch
from vllm.v1.attention.backend import AttentionCGSupport, AttentionMetadataBuilder

from . import kernels
from .config import OscarConfig, task_capacity
from .layout import CacheLayout

_dummy_step = contextvars.ContextVar("oscar_dummy_step", default=False)


@contextlib.contextmanager
def dummy_run_scope(capturing: bool = False):
    """Steps built inside this scope own no cache pages (reference startup.py:24-33)."""
    mark = _dummy_step.set(True)
    try:
        yield
    finally:
        _dummy_step.reset(mark)


def in_dummy_run() -> bool:
    return _dummy_step.get()


@dataclass(frozen=True)
class StepCapacity:
    """Fixed sizes of one builder's device metadata."""

    requests: int
    tokens: int
    columns: int
    query_tile: int

    @property
    def tasks(self) -> int:
        return task_capacity(self.tokens, self.requests, self.query_tile)

    @classmethod
    def for_engine(cls, vllm_config, layout: CacheLayout, cfg: OscarConfig) -> "StepCapacity":
        requests = vllm_config.scheduler_config.max_num_seqs + 1
        tail = (cfg.speculative_tokens + 4) * requests
        columns = math.ceil(vllm_config.model_config.max_model_len / 128) + layout.blocks_per_page + 1
        return cls(requests, vllm_config.scheduler_config.max_num_batched_tokens + tail, columns,
                   cfg.queries_per_tile)


class StepBuffers:
    """The arena and slot buffer of one builder, with named views into the arena."""

    def __init__(self, cap: StepCapacity, device):
        self.cap = cap
        off = kernels.step_arena_layout(cap.requests, cap.columns, cap.tasks)
        self.arena = torch.zeros(off["words"], dtype=torch.int32, device=device)
        self.slot_mapping = torch.full((cap.tokens,), -1, dtype=torch.int64, device=device)
        a = self.arena
        self.counts = a[0:2]
        self.task_count = a[2:3]
        self.query_start_loc = a[off["qstarts"]:off["qstarts"] + cap.requests + 1]
        self.seq_lens = a[off["seq_lens"]:off["seq_lens"] + cap.requests]
        self.block_tables = a[off["table"]:off["table"] + cap.requests * cap.columns].view(cap.requests, cap.columns)
        self.tasks = a[off["tasks"]:off["tasks"] + 2 * cap.tasks].view(cap.tasks, 2)

    def stage(self, source=None, num_reqs: int = 0, num_tokens: int = 0, copy_columns: int = 0):
        """One launch: the step's counts, starts, lengths, reachable table columns, slots
        and task table (``source`` None: a dummy step with zero counts)."""
        c = self.cap
        if source is None:
            kernels.stage_step_metadata(self.arena, self.slot_mapping, c.requests, c.columns, c.tasks, c.query_tile)
            return
        kernels.stage_step_metadata(self.arena, self.slot_mapping, c.requests, c.columns, c.tasks, c.query_tile,
                                    num_reqs=num_reqs, num_tokens=num_tokens, qstarts=source.query_start_loc,
                                    seq_lens=source.seq_lens, table=source.block_table_tensor,
                                    slots=source.slot_mapping, copy_columns=copy_columns)


@dataclass(frozen=True)
class OscarMetadata:
    """One step's metadata: device views of the builder's buffers plus host scalars."""

    buffers: StepBuffers
    num_reqs: int
    num_actual_tokens: int
    max_query_len: int
    layout: CacheLayout
    is_dummy: bool = False
    # host query starts when every request of the step is a first prefill (no history,
    # no window yet); the forward then runs the causal attention over the current tokens
    # with the tcgen05 prefill kernel (the reference hands it to the vendor's fused
    # attention, backend.py:175-193)
    prefill_starts: torch.Tensor | None = None
    causal: bool = True

    query_start_loc = property(lambda self: self.buffers.query_start_loc)
    seq_lens = property(lambda self: self.buffers.seq_lens)
    block_tables = property(lambda self: self.buffers.block_tables)
    slot_mapping = property(lambda self: self.buffers.slot_mapping)
    counts = property(lambda self: self.buffers.counts)
    tasks = property(lambda self: self.buffers.tasks)
    task_count = property(lambda self: self.buffers.task_count)
    max_num_reqs = property(lambda self: self.buffers.cap.requests)
    prefill_only = property(lambda self: self.prefill_starts is not None)
    query_start_loc_cpu = property(lambda self: self.prefill_starts)


def _first_prefill_starts(cm, num_reqs: int):
    """Host query starts if the scheduler's host data proves every request starts at
    position 0, else None.  ``seq_lens_cpu_upper_bound`` is exact for prefill rows and
    never below a true length, so bound == query length means an empty prefix; nothing
    on the device is read."""
    bound = getattr(cm, "seq_lens_cpu_upper_bound", None)
    starts = getattr(cm, "query_start_loc_cpu", None)
    if bound is None or starts is None or num_reqs == 0 or cm.max_query_len <= 16:
        return None
    starts = starts[: num_reqs + 1].to(torch.int64)
    if torch.equal(bound[:num_reqs].to(torch.int64), starts[1:] - starts[:-1]):
        return starts
    return None


def _page_tokens(kv_cache_spec, vllm_config) -> int:
    """Tokens per physical cache page.  vLLM hands the builder a spec in the backend's
    128-token kernel blocks when the engine's cache block (e.g. 768) is larger; the
    kernel blocks of one engine block are consecutive in memory, so the engine block is
    the page that holds a request's history and BF16 window."""
    spec = kv_cache_spec.block_size
    engine = getattr(getattr(vllm_config, "cache_config", None), "block_size", None)
    if isinstance(engine, int) and engine > spec and engine % spec == 0:
        return engine
    return spec


class OscarMetadataBuilder(AttentionMetadataBuilder[OscarMetadata]):
    supports_update_block_table = False
    _cudagraph_support = AttentionCGSupport.UNIFORM_BATCH

    def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)
        from .backend import OscarAttentionImpl

        forward_ctx = getattr(getattr(vllm_config, "compilation_config", None), "static_forward_context", None) or {}
        replaced = [n for n in layer_names
                    if n in forward_ctx and not isinstance(getattr(forward_ctx[n], "impl", None), OscarAttentionImpl)]
        if replaced:
            raise TypeError(f"OSCAR attention implementation replaced on layers {replaced}")
        spec = vllm_config.speculative_config
        cfg = OscarConfig.from_env(spec.num_speculative_tokens if spec else 0)
        self.layout = CacheLayout(_page_tokens(kv_cache_spec, vllm_config), kv_cache_spec.num_kv_heads, config=cfg)
        self.capacity = StepCapacity.for_engine(vllm_config, self.layout, cfg)
        self.buffers = StepBuffers(self.capacity, device)
        self.reorder_batch_threshold = cfg.speculative_tokens + 1

    # capacity views kept for callers that size their own inputs from the builder
    max_reqs = property(lambda self: self.capacity.requests)
    max_tokens = property(lambda self: self.capacity.tokens)
    table = property(lambda self: self.buffers.block_tables)
    counts = property(lambda self: self.buffers.counts)

    @classmethod
    def get_cudagraph_support(cls, vllm_config, kv_cache_spec):
        return AttentionCGSupport.UNIFORM_BATCH

    def reorder_batch(self, input_batch, scheduler_output):
        return False

    def _check(self, common_prefix_len, cm):
        cap = self.capacity
        if common_prefix_len:
            raise ValueError("OSCAR keeps one BF16 ring per request: shared prefixes (cascade attention) "
                             "are not supported")
        if not cm.causal:
            raise ValueError("OSCAR implements causal decoder attention only")
        if cm.num_reqs > cap.requests or cm.num_actual_tokens > cap.tokens:
            raise ValueError(f"step of {cm.num_reqs} requests / {cm.num_actual_tokens} tokens is larger than "
                             f"the metadata capacity ({cap.requests} / {cap.tokens})")
        if cm.block_table_tensor.shape[1] > cap.columns:
            raise ValueError(f"block table of {cm.block_table_tensor.shape[1]} columns is wider than the "
                             f"{cap.columns} this builder holds")
        for name in ("query_start_loc", "seq_lens", "block_table_tensor", "slot_mapping"):
            if getattr(cm, name).device.type != "cuda":
                raise ValueError(f"{name} must be a CUDA tensor")

    def _reachable_columns(self, cm) -> int:
        """Block-table columns a step can reach: all of them, or fewer when the host knows
        the longest sequence (``max_seq_len``, a scheduler value, not a device read)."""
        columns = cm.block_table_tensor.shape[1]
        longest = getattr(cm, "max_seq_len", None)
        if not isinstance(longest, int):
            return columns
        return min(columns, max(1, -(-longest // self.layout.kernel_block_tokens)))

    def build(self, common_prefix_len, common_attn_metadata, fast_build=False):
        cm = common_attn_metadata
        self._check(common_prefix_len, cm)
        if in_dummy_run():
            self.buffers.stage()
            return OscarMetadata(self.buffers, cm.num_reqs, cm.num_actual_tokens, cm.max_query_len, self.layout,
                                 is_dummy=True)
        self.buffers.stage(cm, cm.num_reqs, cm.num_actual_tokens, self._reachable_columns(cm))
        return OscarMetadata(self.buffers, cm.num_reqs, cm.num_actual_tokens, cm.max_query_len, self.layout,
                             prefill_starts=_first_prefill_starts(cm, cm.num_reqs))

    def build_for_cudagraph_capture(self, common_attn_metadata):
        with dummy_run_scope(capturing=True):
            return self.build(0, common_attn_metadata)
