"""Graph-stable device metadata for the OSCAR backend, without device-to-host reads.

Mirrors the reference's ``oscar_ascend/metadata.py:36-170`` on vLLM's CUDA worker:
fixed device buffers sized once (``max_num_seqs + 1`` requests, the batched-token
budget plus the MTP tail, ``ceil(max_model_len/128) + r + 1`` table columns) so CUDA
graphs replay with new contents; ``counts = [num_reqs, num_actual_tokens]`` bound every
kernel on the device; a dummy / capture scope zeroes ``counts`` so recorded kernels
touch no cache page.
"""

from __future__ import annotations

import contextlib
import contextvars
import math
from dataclasses import dataclass

import torch
from vllm.v1.attention.backend import AttentionCGSupport, AttentionMetadataBuilder

from .config import OscarConfig, task_capacity
from .layout import CacheLayout

_dummy = contextvars.ContextVar("oscar_dummy_run", default=False)


@contextlib.contextmanager
def dummy_run_scope(capturing: bool = False):
    """Metadata built inside this scope owns no cache pages (reference startup.py:24-33)."""
    token = _dummy.set(True)
    try:
        yield
    finally:
        _dummy.reset(token)


def in_dummy_run() -> bool:
    return _dummy.get()


@dataclass
class OscarMetadata:
    query_start_loc: torch.Tensor
    seq_lens: torch.Tensor
    block_tables: torch.Tensor
    slot_mapping: torch.Tensor
    counts: torch.Tensor
    num_reqs: int
    num_actual_tokens: int
    max_query_len: int
    max_num_reqs: int
    layout: CacheLayout
    causal: bool = True
    is_dummy: bool = False
    tasks: torch.Tensor | None = None
    task_count: torch.Tensor | None = None
    # host-known first prefill: every request starts at position 0 (no history, no
    # window yet); the forward then uses a library flash-attention kernel for the
    # causal current-token attention (the reference hands this case to the vendor's
    # fused attention, backend.py:175-193)
    prefill_only: bool = False
    query_start_loc_cpu: torch.Tensor | None = None


class OscarMetadataBuilder(AttentionMetadataBuilder[OscarMetadata]):
    supports_update_block_table = False
    _cudagraph_support = AttentionCGSupport.UNIFORM_BATCH

    def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)
        from .backend import OscarAttentionImpl

        ctx = getattr(getattr(vllm_config, "compilation_config", None), "static_forward_context", None)
        if ctx is not None:
            for name in layer_names:
                impl = getattr(ctx.get(name), "impl", None)
                if impl is not None and not isinstance(impl, OscarAttentionImpl):
                    raise TypeError(f"OSCAR implementation was replaced for {name}")
        spec = vllm_config.speculative_config
        cfg = OscarConfig.from_env(spec.num_speculative_tokens if spec else 0)
        self.query_tile = cfg.queries_per_tile
        self.layout = CacheLayout(kv_cache_spec.block_size, kv_cache_spec.num_kv_heads, config=cfg)
        self.reorder_batch_threshold = cfg.speculative_tokens + 1
        sched = vllm_config.scheduler_config
        self.max_reqs = sched.max_num_seqs + 1  # graph padding may add a dummy row
        self.max_tokens = sched.max_num_batched_tokens + (cfg.speculative_tokens + 4) * self.max_reqs
        cols = math.ceil(vllm_config.model_config.max_model_len / 128) + self.layout.blocks_per_page + 1
        self.qstarts = torch.zeros(self.max_reqs + 1, dtype=torch.int32, device=device)
        self.seqs = torch.zeros(self.max_reqs, dtype=torch.int32, device=device)
        self.table = torch.zeros((self.max_reqs, cols), dtype=torch.int32, device=device)
        self.slots = torch.full((self.max_tokens,), -1, dtype=torch.int64, device=device)
        self.counts = torch.zeros(2, dtype=torch.int32, device=device)
        self.tasks = torch.empty((task_capacity(self.max_tokens, self.max_reqs, self.query_tile), 2),
                                 dtype=torch.int32, device=device)
        self.task_count = torch.zeros(1, dtype=torch.int32, device=device)

    @classmethod
    def get_cudagraph_support(cls, vllm_config, kv_cache_spec):
        return AttentionCGSupport.UNIFORM_BATCH

    def reorder_batch(self, input_batch, scheduler_output):
        return False

    def build(self, common_prefix_len, common_attn_metadata, fast_build=False):
        cm = common_attn_metadata
        if common_prefix_len:
            raise ValueError("Prefix sharing is unsupported by the request-owned BF16 ring")
        if not cm.causal:
            raise ValueError("OSCAR supports causal decoder attention only")
        nr, nt = cm.num_reqs, cm.num_actual_tokens
        if nr > self.max_reqs or nt > self.max_tokens:
            raise ValueError("OSCAR metadata capacity exceeded")
        columns = cm.block_table_tensor.shape[1]
        if columns > self.table.shape[1]:
            raise ValueError("Native block table exceeds the configured OSCAR buffer")
        for name in ("query_start_loc", "seq_lens", "block_table_tensor", "slot_mapping"):
            if getattr(cm, name).device.type != "cuda":
                raise ValueError(f"Expected CUDA metadata for {name}")
        dummy = in_dummy_run()
        copy_columns = 0
        if dummy:
            # A dummy/capture step owns no pages: zero counts mask every access on device.
            self.counts.zero_()
        else:
            self.qstarts[: nr + 1].copy_(cm.query_start_loc[: nr + 1], non_blocking=True)
            self.seqs[:nr].copy_(cm.seq_lens[:nr], non_blocking=True)
            copy_columns = columns
            max_seq_len = getattr(cm, "max_seq_len", None)
            if isinstance(max_seq_len, int):
                copy_columns = min(columns, max(1, -(-max_seq_len // self.layout.kernel_block_tokens)))
            self.slots[:nt].copy_(cm.slot_mapping[:nt], non_blocking=True)
            self.counts[0].fill_(nr)
            self.counts[1].fill_(nt)
        from .kernels import prepare_tasks

        prepare_tasks(self.qstarts, self.counts, self.tasks, self.task_count, self.max_reqs, self.query_tile,
                      source_table=cm.block_table_tensor, table=self.table, copy_columns=copy_columns)
        prefill_only, qcpu = False, None
        bound = getattr(cm, "seq_lens_cpu_upper_bound", None)
        qcpu_src = getattr(cm, "query_start_loc_cpu", None)
        if not dummy and bound is not None and qcpu_src is not None and nr > 0 and cm.max_query_len > 16:
            # the bound is exact for prefill rows and never below the true length, so
            # bound == query length proves a zero-length prefix
            qcpu = qcpu_src[: nr + 1].to(torch.int64)
            prefill_only = bool(torch.equal(bound[:nr].to(torch.int64), qcpu[1:] - qcpu[:-1]))
        return OscarMetadata(self.qstarts, self.seqs, self.table, self.slots, self.counts, nr, nt,
                             cm.max_query_len, self.max_reqs, self.layout, is_dummy=dummy, tasks=self.tasks,
                             task_count=self.task_count, prefill_only=prefill_only,
                             query_start_loc_cpu=qcpu if prefill_only else None)

    def build_for_cudagraph_capture(self, common_attn_metadata):
        with dummy_run_scope(capturing=True):
            return self.build(0, common_attn_metadata)
