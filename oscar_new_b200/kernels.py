"""OSCAR INT2 KV-cache operators on B200, behind the reference's operator names.

Each function keeps the name, argument order and meaning of the reference's
``oscar_ascend/kernels.py`` (Triton-Ascend) and calls the sm_100a CUDA library through
its C ABI.  There is deliberately no CPU fallback: tensors must live on a CUDA device
and the library must be built, otherwise the call raises.

Fused entry points that the reference does not have (``rotate_store``,
``decode_attention``) implement the same arithmetic in fewer launches; the backend
uses them.
"""

from __future__ import annotations

import ctypes as C
import os

import torch

from . import _lib
from .config import attention_programs, quantile_weight_f32

LOG2E = 1.4426950408889634

# Device status words (one int32 per device).  Kernels with bounded device waits store
# 4 (device wait timeout) into their device's word when a wait gives up; the library
# never clears it.  With OSCAR_CHECK_STATUS=1 every such call synchronises and raises
# on a nonzero word (debug mode); otherwise `read_status` reports it on demand.
_STATUS_WORDS: dict = {}
_CHECK_STATUS = os.environ.get("OSCAR_CHECK_STATUS", "0") not in ("", "0")


def status_word(device) -> torch.Tensor:
    """The int32[1] device status word that this module passes to ``device``'s launches."""
    device = torch.device(device)
    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _STATUS_WORDS.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=f"cuda:{index}")
        _STATUS_WORDS[index] = word
    return word


def read_status(device=None, clear: bool = True) -> int:
    """Synchronise ``device`` and return its status word (0 = no device wait gave up)."""
    word = status_word(device if device is not None else torch.device("cuda"))
    torch.cuda.synchronize(word.device)
    value = int(word.item())
    if clear and value:
        word.zero_()
    return value


def _status(t: torch.Tensor):
    return status_word(t.device).data_ptr()


def _checked(name: str, t: torch.Tensor):
    """Debug mode: a launch whose device wait gave up raises instead of leaving stale outputs."""
    if _CHECK_STATUS:
        value = read_status(t.device)
        if value:
            raise RuntimeError(f"{name} failed on the device: {_lib.STATUS.get(value, value)}")


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("OSCAR kernels run on a CUDA device only (no CPU fallback)")


def _rows(x: torch.Tensor):
    """[n, h, 256] bf16 view with unit inner stride and 16-byte aligned rows."""
    if x.dtype != torch.bfloat16 or x.ndim != 3 or x.shape[-1] != 256:
        raise ValueError(f"expected bf16 [n, h, 256], got {tuple(x.shape)} {x.dtype}")
    if x.stride(2) != 1 or x.stride(0) % 8 or x.stride(1) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


def geometry(layout, hq: int, table_stride: int) -> _lib.Geometry:
    cfg = layout.config
    if hq % layout.kv_heads:
        raise ValueError("query heads must be a multiple of KV heads")
    return _lib.Geometry(
        kv_heads=layout.kv_heads,
        group=hq // layout.kv_heads,
        head_dim=cfg.head_dim,
        block_tokens=layout.physical_block_tokens,
        kernel_block=layout.kernel_block_tokens,
        slot_bytes=cfg.slot_bytes,
        vector_bytes=cfg.vector_bytes,
        sink=cfg.sink_tokens,
        recent=cfg.recent_tokens,
        ring=cfg.ring_tokens,
        table_stride=table_stride,
        query_tile=cfg.queries_per_tile,
        page_bytes=layout.stripe_page_bytes,
    )


def clip_params(cfg, kind: str) -> _lib.Clip:
    """torch.quantile semantics (fp32 rank/weight) or fixed max-abs factor."""
    ratio = cfg.k_clip_ratio if kind == "k" else cfg.v_clip_ratio
    factor = cfg.k_clip_factor if kind == "k" else cfg.v_clip_factor
    if cfg.clip_mode == "factor":
        return _lib.Clip(enabled=1, mode=1, asc_lo=0, asc_hi=0, weight=0.0, factor=factor)
    if not ratio:
        return _lib.Clip(enabled=0, mode=0, asc_lo=0, asc_hi=0, weight=0.0, factor=1.0)
    lo, hi, w = quantile_weight_f32(ratio, cfg.head_dim)
    return _lib.Clip(enabled=1, mode=0, asc_lo=lo, asc_hi=hi, weight=w, factor=1.0)


def _rotation(r: torch.Tensor):
    if r.dtype != torch.bfloat16 or r.shape != (256, 256):
        raise ValueError("rotation must be bf16 [256, 256]")
    s0, s1 = r.stride()
    if not ((s1 == 1 and s0 % 8 == 0) or (s0 == 1 and s1 % 8 == 0)) or r.data_ptr() % 16:
        r = r.contiguous()
    return r


# ----------------------------------------------------------------------------
# reference operators (oscar_ascend/kernels.py)
# ----------------------------------------------------------------------------


def rotate(x: torch.Tensor, rotation: torch.Tensor) -> torch.Tensor:
    """``bf16(x) @ bf16(R)`` with fp32 accumulation -> bf16 (reference kernels.py:51-66)."""
    _require_cuda(x, rotation)
    n, h, d = x.shape
    out = torch.empty((n, h, d), device=x.device, dtype=torch.bfloat16)
    if n == 0:
        return out
    x = _rows(x)
    r = _rotation(rotation)
    _lib.call("oscar_rotate", x.data_ptr(), n, h, x.stride(0), x.stride(1), x.stride(2), r.data_ptr(),
              r.stride(0), r.stride(1), out.data_ptr(), _stream(x))
    return out


def store_int2(key_rot, value_rot, history, slots, counts, layout):
    """Clip + INT2 pack + masked scatter (reference kernels.py:175-202)."""
    _require_cuda(key_rot, value_rot, history, slots, counts)
    cfg = layout.config
    n = key_rot.shape[0]
    kr, vr = key_rot.contiguous(), value_rot.contiguous()
    geo = geometry(layout, layout.kv_heads, 1)
    _lib.call("oscar_store_int2", kr.data_ptr(), vr.data_ptr(), n, history.data_ptr(), slots.data_ptr(),
              counts.data_ptr(), geo, clip_params(cfg, "k"), clip_params(cfg, "v"), _stream(history))


def rotate_store(key, value, rk, rv, history, slots, counts, layout, query=None, debug_rotated=False):
    """Fused ``rotate(K,Rk)``, ``rotate(V,Rv)``, ``store_int2`` and optionally
    ``rotate(Q,Rk)`` in one launch.  Returns ``qrot`` (or None) and, with
    ``debug_rotated``, the bf16 rotated K/V rows that were quantised."""
    _require_cuda(key, value, rk, rv, history, slots, counts, query)
    cfg = layout.config
    n = key.shape[0]
    key, value = _rows(key), _rows(value)
    rk, rv = rk.contiguous(), rv.contiguous()
    qrot = kout = vout = None
    qargs = (None, 0, 0, 0, None)
    if query is not None:
        query = _rows(query)
        qrot = torch.empty(query.shape, device=query.device, dtype=torch.bfloat16)
        qargs = (query.data_ptr(), query.stride(0), query.stride(1), query.shape[1], qrot.data_ptr())
    if debug_rotated:
        kout = torch.empty((n, layout.kv_heads, 256), device=key.device, dtype=torch.bfloat16)
        vout = torch.empty_like(kout)
    geo = geometry(layout, layout.kv_heads, 1)
    _lib.call("oscar_rotate_store", key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(),
              value.stride(0), value.stride(1), n, rk.data_ptr(), rv.data_ptr(), history.data_ptr(),
              slots.data_ptr(), counts.data_ptr(), geo, clip_params(cfg, "k"), clip_params(cfg, "v"),
              *qargs, _ptr(kout), _ptr(vout), _status(key), _stream(key))
    _checked("oscar_rotate_store", key)
    if debug_rotated:
        return qrot, kout, vout
    return qrot


def prepare_tasks(qstarts, counts, tasks, task_count, max_reqs, query_tile, num_reqs=None, source_table=None,
                  table=None, copy_columns=0):
    """Compact (request, query offset) task table (reference kernels.py:262-287)."""
    _require_cuda(qstarts, counts, tasks, task_count, source_table, table)
    copy = source_table is not None and table is not None and copy_columns > 0
    if copy and source_table.stride(1) != 1:
        source_table = source_table.contiguous()
    _lib.call("oscar_prepare_tasks", qstarts.data_ptr(), counts.data_ptr(), tasks.data_ptr(),
              task_count.data_ptr(), tasks.shape[0], max_reqs, query_tile,
              source_table.data_ptr() if copy else None, source_table.stride(0) if copy else 0,
              table.data_ptr() if copy else None, table.stride(0) if copy else 0, copy_columns if copy else 0,
              _stream(counts))


def step_arena_layout(max_reqs: int, columns: int, task_capacity: int) -> dict:
    """Word offsets of the fixed per-step metadata arena (host-only call, no device)."""
    off = (C.c_int64 * 5)()
    _lib.call("oscar_step_arena_layout", max_reqs, columns, task_capacity, C.addressof(off))
    return dict(zip(("qstarts", "seq_lens", "table", "tasks", "words"), (int(x) for x in off)))


def stage_step_metadata(arena, slot_out, max_reqs, columns, task_capacity, query_tile, num_reqs=0, num_tokens=0,
                        qstarts=None, seq_lens=None, table=None, slots=None, copy_columns=0):
    """Stage one step's metadata into the fixed arena in one launch (counts, query starts,
    sequence lengths, reachable block-table columns, slot mapping, task table).  No
    sources and zero requests / tokens stage a dummy step: counts and task count 0,
    nothing else."""
    _require_cuda(arena, slot_out, qstarts, seq_lens, table, slots)
    if arena.dtype != torch.int32 or slot_out.dtype != torch.int64:
        raise ValueError("the arena is int32 and the slot buffer int64")
    if qstarts is not None:
        qstarts = qstarts.to(torch.int32)
    if not num_reqs:
        seq_lens = table = None
    if seq_lens is not None:
        seq_lens = seq_lens.to(torch.int32)
    if table is None or not copy_columns:
        table, copy_columns = None, 0
    elif table.dtype != torch.int32 or table.stride(1) != 1:
        table = table.to(torch.int32).contiguous()
    slots = slots.to(torch.int64) if num_tokens else None
    _lib.call("oscar_stage_step_metadata", _ptr(qstarts), _ptr(seq_lens), _ptr(table),
              0 if table is None else table.stride(0), _ptr(slots), num_reqs, num_tokens, copy_columns, query_tile,
              arena.data_ptr(), max_reqs, columns, task_capacity, slot_out.data_ptr(), slot_out.shape[0],
              _stream(arena))


def prefill_attention(query, key, value, query_start_loc, num_reqs: int, max_query_len: int, scale: float,
                      out=None):
    """Causal attention of a first prefill over the current tokens only (tcgen05 kernel):
    query [n, Hq, 256], key / value [n, Hkv, 256] bf16, device query starts
    [num_reqs + 1]; returns / fills out [n, Hq, 256] bf16."""
    _require_cuda(query, key, value, query_start_loc, out)
    n, hq, d = query.shape
    if out is None:
        out = torch.empty((n, hq, d), dtype=torch.bfloat16, device=query.device)
    if n == 0 or num_reqs == 0:
        return out
    query, key, value = _rows(query), _rows(key), _rows(value)
    _lib.call("oscar_prefill_attention", query.data_ptr(), query.stride(0), query.stride(1), key.data_ptr(),
              key.stride(0), key.stride(1), value.data_ptr(), value.stride(0), value.stride(1),
              query_start_loc.data_ptr(), num_reqs, max_query_len, n, hq, key.shape[1], float(scale), out.data_ptr(),
              out.stride(0), out.stride(1), _status(out), _stream(query))
    return out


def _meta_common(meta, layout, hq):
    geo = geometry(layout, hq, meta.block_tables.stride(0))
    if meta.block_tables.stride(1) != 1:
        raise ValueError("block table rows must be contiguous")
    # Launch only the query-row tiles this step can use: a task never holds more than
    # min(queries_per_tile, max_query_len) queries (host scheduler value, no device read).
    max_q = getattr(meta, "max_query_len", None)
    if isinstance(max_q, int) and max_q > 0:
        geo.query_tile = min(geo.query_tile, max_q)
    return geo


def attention_partials(query, key, value, history, window, meta, layout, scale, splits, raw):
    """Split-KV attention partials (reference kernels.py:439-482)."""
    _require_cuda(query, key, value, history, window)
    n, hq, d = query.shape
    partials = torch.empty((n, hq, splits, d), dtype=torch.float32, device=query.device)
    lse = torch.empty((n, hq, splits), dtype=torch.float32, device=query.device)
    if n == 0:
        return partials, lse
    query = _rows(query)
    key, value = _rows(key), _rows(value)
    geo = _meta_common(meta, layout, hq)
    programs = attention_programs(n, meta.max_num_reqs, layout.config.queries_per_tile)
    _lib.call("oscar_attention_partials", query.data_ptr(), query.stride(0), query.stride(1), key.data_ptr(),
              key.stride(0), key.stride(1), value.data_ptr(), value.stride(0), value.stride(1),
              history.data_ptr(), window.data_ptr(), meta.query_start_loc.data_ptr(), meta.seq_lens.data_ptr(),
              meta.block_tables.data_ptr(), meta.counts.data_ptr(), meta.tasks.data_ptr(),
              meta.task_count.data_ptr(), min(programs, meta.tasks.shape[0]), n, partials.data_ptr(),
              lse.data_ptr(), geo, float(scale), int(splits), int(bool(raw)), _status(query), _stream(query))
    _checked("oscar_attention_partials", query)
    return partials, lse


def merge_splits(partials, lse, counts):
    """LSE merge of split partials (reference kernels.py:506-511)."""
    _require_cuda(partials, lse, counts)
    n, hq, splits, d = partials.shape
    out = torch.empty((n, hq, d), dtype=torch.bfloat16, device=partials.device)
    logsum = torch.empty((n, hq), dtype=torch.float32, device=partials.device)
    if n:
        _lib.call("oscar_merge_splits", partials.contiguous().data_ptr(), lse.contiguous().data_ptr(), n, hq, splits,
                  counts.data_ptr(), out.data_ptr(), logsum.data_ptr(), _stream(partials))
    return out, logsum


def merge_paths(history_out, history_lse, raw_partials, raw_lse, counts, output):
    """LSE merge of the history and raw paths into ``output`` (reference kernels.py:530-541)."""
    _require_cuda(history_out, history_lse, raw_partials, raw_lse, counts, output)
    n, hq, d = history_out.shape
    if n == 0:
        return
    if not output.is_contiguous():
        raise ValueError("output must be contiguous")
    a = history_out.contiguous()
    b = raw_partials.contiguous()
    lb = raw_lse.contiguous()
    b_stride = b.shape[2] * d if b.ndim == 4 else d
    lb_stride = lb.shape[2] if lb.ndim == 3 else 1
    _lib.call("oscar_merge_paths", a.data_ptr(), history_lse.contiguous().data_ptr(), b.data_ptr(), b_stride,
              lb.data_ptr(), lb_stride, n, hq, counts.data_ptr(), output.data_ptr(), _stream(a))


def store_windows(key, value, window, meta, layout):
    """Write current BF16 K/V into the sink/ring window (reference kernels.py:598-620)."""
    _require_cuda(key, value, window)
    key, value = _rows(key), _rows(value)
    geo = _meta_common(meta, layout, layout.kv_heads)
    programs = min(key.shape[0], meta.max_num_reqs)
    _lib.call("oscar_store_windows", key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(),
              value.stride(0), value.stride(1), window.data_ptr(), meta.query_start_loc.data_ptr(),
              meta.seq_lens.data_ptr(), meta.block_tables.data_ptr(), meta.counts.data_ptr(), programs, geo,
              _stream(key))


def dequant_inverse_rotate(history, slots, rk, rv, layout):
    """Diagnostic finite tile only (reference kernels.py:651-672)."""
    _require_cuda(history, slots, rk, rv)
    n, h = slots.numel(), layout.kv_heads
    if n > 4096:
        raise ValueError("diagnostic dequant is limited to 4096 tokens; use fused attention")
    k = torch.empty((n, h, 256), device=history.device, dtype=torch.bfloat16)
    v = torch.empty_like(k)
    geo = geometry(layout, h, 1)
    _lib.call("oscar_unpack", history.data_ptr(), slots.contiguous().data_ptr(), n, geo, k.data_ptr(),
              v.data_ptr(), _stream(history))
    return rotate(k, rk.T), rotate(v, rv.T)


# ----------------------------------------------------------------------------
# fused decode step
# ----------------------------------------------------------------------------


class DecodeScratch:
    """Caller-owned split scratch: fp32 partials [n, Hq, splits+1, 256] and lse."""

    def __init__(self, max_tokens: int, hq: int, splits: int, device):
        self.splits = splits
        self.partials = torch.empty((max_tokens, hq, splits + 1, 256), dtype=torch.float32, device=device)
        self.lse = torch.empty((max_tokens, hq, splits + 1), dtype=torch.float32, device=device)


def decode_attention(qrot, query, key, value, history, window, meta, layout, scale, splits, rv, output, scratch=None,
                     store_window=True):
    """History + raw attention, split merge, inverse V rotation, path merge and the
    window store of one decode / MTP-verify step (reference backend.py:195-226)."""
    _require_cuda(qrot, query, key, value, history, window, rv, output)
    n, hq, _ = query.shape
    if n == 0:
        return output
    if scratch is None or scratch.partials.shape[0] < n or scratch.splits != splits:
        scratch = DecodeScratch(n, hq, splits, query.device)
    query, key, value = _rows(query), _rows(key), _rows(value)
    qrot = qrot.contiguous()
    rv = rv.contiguous()
    geo = _meta_common(meta, layout, hq)
    programs = min(attention_programs(n, meta.max_num_reqs, layout.config.queries_per_tile), meta.tasks.shape[0])
    window_programs = min(n, meta.max_num_reqs) if store_window else 0
    _lib.call("oscar_decode_attention", qrot.data_ptr(), query.data_ptr(), query.stride(0), query.stride(1),
              key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(), value.stride(0), value.stride(1),
              history.data_ptr(), window.data_ptr(), meta.query_start_loc.data_ptr(), meta.seq_lens.data_ptr(),
              meta.block_tables.data_ptr(), meta.counts.data_ptr(), meta.tasks.data_ptr(),
              meta.task_count.data_ptr(), programs, n, rv.data_ptr(), scratch.partials.data_ptr(),
              scratch.lse.data_ptr(), output.data_ptr(), geo, float(scale), int(splits), window_programs,
              _status(query), _stream(query))
    _checked("oscar_decode_attention", query)
    return output
