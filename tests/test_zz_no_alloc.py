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


def call_noalloc(sc, qrot, q, k, v, out, splits):
    m = sc.meta
    geo = kernels._meta_common(m, sc.layout, sc.hq)
    programs = min(attention_programs(q.shape[0], m.max_num_reqs, sc.cfg.queries_per_tile), m.tasks.shape[0])
    status = _lib.lib().oscar_decode_attention_noalloc(
        qrot.data_ptr(), q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
        v.data_ptr(), v.stride(0), v.stride(1), sc.history.data_ptr(), sc.window.data_ptr(),
        m.query_start_loc.data_ptr(), m.seq_lens.data_ptr(), m.block_tables.data_ptr(), m.counts.data_ptr(),
        m.tasks.data_ptr(), m.task_count.data_ptr(), programs, q.shape[0], sc.rv.to("cuda").data_ptr(),
        out.data_ptr(), geo, 1 / 16, splits, 0, torch.cuda.current_stream().cuda_stream)
    return status


def test_noalloc_decode_matches_regular_entry_point_twice(cuda_lib):
    splits = 8
    sc = Scenario([1200, 3000, 700], [1, 4, 2], hq=24, h=4, cfg=make_config(4, 128, 3), seed=77)
    q, k, v = sc.current()
    sc.prepare_tasks()
    qrot = kernels.rotate_store(k, v, sc.rk.to("cuda"), sc.rv.to("cuda"), sc.history, sc.meta.slot_mapping,
                                sc.meta.counts, sc.layout, query=q)
    ref = torch.empty((q.shape[0], sc.hq * 256), dtype=torch.bfloat16, device="cuda")
    kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, sc.meta, sc.layout, 1 / 16, splits,
                             sc.rv.to("cuda"), ref, store_window=False)
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        assert call_noalloc(sc, qrot, q, k, v, out, splits) == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), atol=0.035, rtol=0.04)


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_lib):
    cap = _lib.lib().oscar_decode_attention_noalloc_max_rows()
    assert cap == 32768
    sc = Scenario([600], [1], hq=24, h=4, cfg=make_config(4, 128, 0), seed=5)
    q, k, v = sc.current()
    out = torch.empty((1, 24 * 256), dtype=torch.bfloat16, device="cuda")
    # 1 token x 24 heads x (splits + 1) rows: pick splits so the rows exceed the capacity
    too_many = cap // 24 + 1
    assert call_noalloc(sc, q, q, k, v, out, too_many) == 1
