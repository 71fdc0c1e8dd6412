"""The 8-bit tcgen05 decode history kernel (history_f8_kernel) against the CPU oracle.

It covers launches with at most 8 query rows per KV head (decode, and short MTP rows at
small GQA groups) and is selected with OSCAR_HISTORY_F8=1.  Which kernel ran is asserted by name through the CUDA
profiler.  Tolerances as elsewhere: output atol .035 / rtol .04 and rel 1e-2 in norm
(reference tests/test_npu_kernels.py:194), LSE within 1e-3 abs.
"""

import pytest
import torch

from oracle import int2_oracle as oo
from oscar_new_b200 import _lib, kernels
from oscar_new_b200.config import task_capacity
from oscar_new_b200.layout import CacheLayout
from tests.golden.fixtures import load, unzpack
from tests.helpers import Scenario, make_config

pytestmark = pytest.mark.gpu
DEV = "cuda"
F8 = "history_f8_kernel"


@pytest.fixture(autouse=True)
def f8_selected(monkeypatch):
    """The kernel is opt-in (OSCAR_HISTORY_F8=1, read at every launch)."""
    monkeypatch.setenv("OSCAR_HISTORY_F8", "1")


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


def kernel_names(fn):
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        out = fn()
        torch.cuda.synchronize()
    return out, {e.name for e in prof.events()}


def history_lse(scratch, n, splits):
    """Logsumexp over the history split slots of a decode step's scratch (the raw path's
    slot, index `splits`, left out)."""
    return torch.logsumexp(scratch.lse[:n, :, :splits].float(), dim=-1).cpu()


def oracle_history_lse(sc, qrot, k, v):
    """History-path LSE of the kernel-faithful CPU oracle on the same bf16 rotated query
    (the dense hybrid reference rotates the query in fp32, which moves logits by about
    2^-9 relative and is not a 1e-3 LSE reference)."""
    meta_cpu = type("M", (), {})()
    for nm in ("query_start_loc", "seq_lens", "block_tables", "counts"):
        setattr(meta_cpu, nm, getattr(sc.meta, nm).cpu())
    _, lse = oo.attention_partials(qrot.cpu(), k.cpu(), v.cpu(), sc.history.cpu(), sc.window.cpu(), meta_cpu,
                                   sc.layout, 1 / 16, 1, False)
    return lse[:, :, 0]


@pytest.mark.parametrize("index", [0, 2])
def test_f8_partials_match_reference_kernel_body(cuda_lib, index):
    """Reference split semantics (32-token granules, `splits` per task): partials and
    split LSEs against the reference kernel body run on CPU (golden fixture); case 0 is
    one KV head with 8 query heads, case 2 two KV heads x 2 groups x 4 query tokens."""
    case = load("attention_kernel.pt")[index]
    cfg = make_config(case["sink"], case["recent"], case["mtp"])
    layout = CacheLayout(case["bp"], kv_heads=case["h"], config=cfg)
    hist = unzpack(case["history"]).to(DEV)
    win = unzpack(case["window"]).to(DEV)
    m = case["meta"]
    meta = type("M", (), {})()
    for name in ("query_start_loc", "seq_lens", "block_tables", "counts"):
        setattr(meta, name, m[name].to(DEV))
    qs = m["query_start_loc"]
    meta.max_query_len = int((qs[1:] - qs[:-1]).max())
    n = case["q"].shape[0]
    meta.max_num_reqs = m["block_tables"].shape[0]
    meta.tasks = torch.full((task_capacity(n, meta.max_num_reqs, 4), 2), -1, dtype=torch.int32, device=DEV)
    meta.task_count = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.prepare_tasks(meta.query_start_loc, meta.counts, meta.tasks, meta.task_count, meta.max_num_reqs, 4)
    qrot, k, v = (case[x].to(DEV) for x in ("qrot", "k", "v"))
    (hp, hl), names = kernel_names(
        lambda: kernels.attention_partials(qrot, k, v, hist, win, meta, layout, 1 / 16, case["splits"], False))
    assert any(F8 in nm for nm in names), names
    live = ~torch.isnan(case["hist_lse"])
    ref_l, got_l = case["hist_lse"][live], hl.cpu()[live]
    assert torch.equal(torch.isinf(ref_l), torch.isinf(got_l))
    fin = torch.isfinite(ref_l)
    torch.testing.assert_close(got_l[fin], ref_l[fin], atol=1e-3, rtol=0)
    torch.testing.assert_close(hp.cpu()[live], case["hist_partials"][live], atol=0.035, rtol=0.04)


@pytest.mark.parametrize(
    "name,seq,qlen,hq,h,cfg,splits",
    [
        # 4 KV heads per CTA (GQA 6), decode
        ("gqa24x4", [700, 1500, 3000, 130], [1, 1, 1, 1], 24, 4, make_config(4, 128, 0), 16),
        # one KV head, 8 query heads (the reference's CPU-oracle configuration)
        ("config1", [300, 1000, 2500, 4096], [1, 1, 1, 1], 8, 1, make_config(4, 64, 0), 4),
        # two KV heads per CTA; 2 query tokens x GQA 4 = 8 rows per head
        ("pairs_mtp1", [900, 2300], [2, 2], 8, 2, make_config(4, 128, 1), 8),
        # 8 KV heads: two head groups of 4
        ("heads8", [1300, 2600, 517], [1, 1, 1], 32, 8, make_config(4, 128, 0), 8),
        # skewed lengths: the balanced split gives the long request most of the splits
        ("skewed", [140, 9000, 333, 5, 1500, 20000], [1, 1, 1, 1, 1, 1], 24, 4, make_config(4, 128, 0), 64),
    ],
)
def test_f8_decode_step_matches_hybrid_reference(cuda_lib, name, seq, qlen, hq, h, cfg, splits):
    sc = Scenario(seq, qlen, hq=hq, h=h, cfg=cfg, seed=len(name) + 40)
    n = sum(qlen)
    scratch = kernels.DecodeScratch(n, hq, splits, DEV)
    q, k, v = sc.current()
    sc.prepare_tasks()
    qrot = kernels.rotate_store(k, v, sc.rk.to(DEV), sc.rv.to(DEV), sc.history, sc.meta.slot_mapping,
                                sc.meta.counts, sc.layout, query=q)

    def step():
        out = torch.empty((n, hq * 256), dtype=torch.bfloat16, device=DEV)
        kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, sc.meta, sc.layout, 1 / 16, splits,
                                 sc.rv.to(DEV), out, scratch, store_window=False)
        return out.view(n, hq, 256)

    out, names = kernel_names(step)
    assert any(F8 in nm for nm in names), names
    expect, _ = sc.expected()
    assert rel_err(out.cpu(), expect) < 1e-2, rel_err(out.cpu(), expect)
    torch.testing.assert_close(out.float().cpu(), expect, atol=0.035, rtol=0.04)
    got, want = history_lse(scratch, n, splits), oracle_history_lse(sc, qrot, k, v)
    assert torch.equal(torch.isinf(got), torch.isinf(want))
    fin = torch.isfinite(want)
    torch.testing.assert_close(got[fin], want[fin], atol=1e-3, rtol=0)


def test_f8_config3_full_context(cuda_lib):
    """BASELINE config 3 at full per-request size: 32768-token contexts (4 sink, 128
    recent, 32635 INT2 history tokens each), 24 query / 4 KV heads, 16 splits; output
    against the oracle's dense hybrid reference, history LSE against the oracle's
    paged history attention."""
    seq = [32768] * 4
    sc = Scenario(seq, [1] * 4, hq=24, h=4, cfg=make_config(4, 128, 0), seed=33)
    scratch = kernels.DecodeScratch(4, 24, 16, DEV)
    q, k, v = sc.current()
    sc.prepare_tasks()

    qrot = kernels.rotate_store(k, v, sc.rk.to(DEV), sc.rv.to(DEV), sc.history, sc.meta.slot_mapping,
                                sc.meta.counts, sc.layout, query=q)

    def step():
        out = torch.empty((4, 24 * 256), dtype=torch.bfloat16, device=DEV)
        kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, sc.meta, sc.layout, 1 / 16, 16,
                                 sc.rv.to(DEV), out, scratch, store_window=False)
        return out.view(4, 24, 256)

    out, names = kernel_names(step)
    assert any(F8 in nm for nm in names), names
    expect, _ = sc.expected()
    assert rel_err(out.cpu(), expect) < 1e-2, rel_err(out.cpu(), expect)
    torch.testing.assert_close(out.float().cpu(), expect, atol=0.035, rtol=0.04)
    torch.testing.assert_close(history_lse(scratch, 4, 16), oracle_history_lse(sc, qrot, k, v), atol=1e-3, rtol=0)


def test_f8_wait_timeout_reports_status_and_context_recovers(cuda_lib):
    """The timeout path of the product kernel: with the test hook, CTA 0 never issues the
    copy of its second tile and waits give up after 4096 probes.  The launch must return,
    store OSCAR_ERR_TIMEOUT (4) in the status word and leave the context usable: the next
    step, without the hook, matches the oracle with a clear status word."""
    sc = Scenario([1500, 2600], [1, 1], hq=24, h=4, cfg=make_config(4, 128, 0), seed=91)
    q, k, v = sc.current()
    sc.prepare_tasks()
    rk, rv = sc.rk.to(DEV), sc.rv.to(DEV)
    qrot = kernels.rotate_store(k, v, rk, rv, sc.history, sc.meta.slot_mapping, sc.meta.counts, sc.layout, query=q)
    kernels.read_status(DEV)  # start from a clear word
    out = torch.empty((2, 24 * 256), dtype=torch.bfloat16, device=DEV)
    lib = _lib.lib()
    assert lib.oscar_test_set_wait_fault(1, 4096) == 0
    try:
        kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, sc.meta, sc.layout, 1 / 16, 8, rv, out,
                                 store_window=False)
        torch.cuda.synchronize()
    finally:
        assert lib.oscar_test_set_wait_fault(-1, 0) == 0
    assert kernels.read_status(DEV) == 4
    kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, sc.meta, sc.layout, 1 / 16, 8, rv, out,
                             store_window=False)
    assert kernels.read_status(DEV) == 0
    expect, _ = sc.expected()
    torch.testing.assert_close(out.view(2, 24, 256).float().cpu(), expect, atol=0.035, rtol=0.04)
