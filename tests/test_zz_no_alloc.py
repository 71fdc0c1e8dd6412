"""The no-allocation decode entry point agrees with the regular one.

`oscar_decode_attention_noalloc` serves callers that cannot allocate device memory at
decode time (an engine whose memory plan already gave the free memory to the KV cache,
or an FFI host without a device allocator).  It keeps its split scratch in fixed device
arrays inside the library instead of taking a caller buffer.  This file is collected
last on purpose, and passes both on its own and after the rest of the suite.
"""

import pytest
import torch

from oscar_new_b200 import _lib, kernels
from oscar_new_b200.config import attention_programs
from tests.helpers import Scenario, make_config

pytestmark = pytest.mark.gpu


def call_noalloc(sc, qrot, q, k, v, out, splits, status=None):
    m = sc.meta
    geo = kernels._meta_common(m, sc.layout, sc.hq)
    programs = min(attention_programs(q.shape[0], m.max_num_reqs, sc.cfg.queries_per_tile), m.tasks.shape[0])
    return _lib.lib().oscar_decode_attention_noalloc(
        qrot.data_ptr(), q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
        v.data_ptr(), v.stride(0), v.stride(1), sc.history.data_ptr(), sc.window.data_ptr(),
        m.query_start_loc.data_ptr(), m.seq_lens.data_ptr(), m.block_tables.data_ptr(), m.counts.data_ptr(),
        m.tasks.data_ptr(), m.task_count.data_ptr(), programs, q.shape[0], sc.rv.to("cuda").data_ptr(),
        out.data_ptr(), geo, 1 / 16, splits, 0, None if status is None else status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def _prepared(sc):
    q, k, v = sc.current()
    sc.prepare_tasks()
    qrot = kernels.rotate_store(k, v, sc.rk.to("cuda"), sc.rv.to("cuda"), sc.history, sc.meta.slot_mapping,
                                sc.meta.counts, sc.layout, query=q)
    return qrot, q, k, v


def _regular(sc, qrot, q, k, v, splits):
    ref = torch.empty((q.shape[0], sc.hq * 256), dtype=torch.bfloat16, device="cuda")
    kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, sc.meta, sc.layout, 1 / 16, splits,
                             sc.rv.to("cuda"), ref, store_window=False)
    return ref


def test_noalloc_decode_matches_regular_entry_point_larger_then_smaller(cuda_lib):
    """A larger call (more tokens, more splits) leaves its partials in the shared arrays;
    the smaller call after it must not read any of them."""
    big = Scenario([5200, 3000, 700, 4100], [4, 1, 2, 3], hq=24, h=4, cfg=make_config(4, 128, 3), seed=77)
    small = Scenario([1200, 900], [1, 2], hq=24, h=4, cfg=make_config(4, 128, 3), seed=78)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for sc, splits in ((big, 16), (small, 4), (small, 4)):
        qrot, q, k, v = _prepared(sc)
        ref = _regular(sc, qrot, q, k, v, splits)
        out = torch.full_like(ref, float("nan"))
        assert call_noalloc(sc, qrot, q, k, v, out, splits, status) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        torch.testing.assert_close(out.float(), ref.float(), atol=0.035, rtol=0.04)


def test_noalloc_accepts_exactly_its_capacity_and_rejects_one_row_more(cuda_lib):
    cap = _lib.lib().oscar_decode_attention_noalloc_max_rows()
    assert cap == 32768
    # 8 requests x 4 query tokens x 16 query heads x (63 + 1) split slots = 32768 rows
    sc = Scenario([900 + 37 * i for i in range(8)], [4] * 8, hq=16, h=4, cfg=make_config(4, 64, 3), seed=5)
    qrot, q, k, v = _prepared(sc)
    assert q.shape[0] * sc.hq * (63 + 1) == cap
    ref = _regular(sc, qrot, q, k, v, 63)
    out = torch.full_like(ref, float("nan"))
    assert call_noalloc(sc, qrot, q, k, v, out, 63) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), ref.float(), atol=0.035, rtol=0.04)
    # one token more at the same head and split count is one row group beyond capacity
    sc2 = Scenario([900 + 37 * i for i in range(8)] + [500], [4] * 8 + [1], hq=16, h=4, cfg=make_config(4, 64, 3),
                   seed=6)
    qrot2, q2, k2, v2 = _prepared(sc2)
    assert q2.shape[0] * sc2.hq * 64 > cap
    out2 = torch.empty((q2.shape[0], 16 * 256), dtype=torch.bfloat16, device="cuda")
    assert call_noalloc(sc2, qrot2, q2, k2, v2, out2, 63) == 1
    # split counts beyond the merge's 64 are refused before any size arithmetic
    assert call_noalloc(sc2, qrot2, q2, k2, v2, out2, 65) == 1
