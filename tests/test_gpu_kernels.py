"""GPU parity of every CUDA operator against the CPU oracle (tests/oracle.py restated).

Tolerances follow the reference's device tests and the project targets:
packed bytes / scales bit-exact given identical bf16 rotated inputs; rotation within
bf16 rounding (atol 2^-5, rtol 1.5e-2); attention output within atol .035 / rtol .04
(reference tests/test_npu_kernels.py:194) and rel 1e-2 in norm; LSE within 1e-3 abs.
"""

from dataclasses import replace

import numpy as np
import pytest
import torch

from oracle import calibration_oracle as co
from oracle import int2_oracle as oo
from oscar_new_b200 import _lib
from oscar_new_b200 import calibration_kernels as ck
from oscar_new_b200 import kernels
from oscar_new_b200.config import OscarConfig, task_capacity
from oscar_new_b200.layout import CacheLayout
from oscar_new_b200.synthetic import cache_stripes, rotation
from tests.golden.fixtures import load, unzpack
from tests.helpers import Scenario, make_config

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


# ----------------------------------------------------------------------------
# store / rotate
# ----------------------------------------------------------------------------


@pytest.mark.parametrize(
    "kr,vr,mode",
    [(0.96, 0.92, "percentile"), (0.0, 0.0, "percentile"), (1.0, 1.0, "percentile"), (0.875, 0.92, "percentile"),
     (0.96, 0.92, "factor")],
)
def test_store_int2_bytes_exact(cuda_lib, kr, vr, mode):
    cfg = replace(OscarConfig(), k_clip_ratio=kr, v_clip_ratio=vr, clip_mode=mode, k_clip_factor=0.9,
                  v_clip_factor=0.75)
    h = 4
    layout = CacheLayout(768, kv_heads=h, config=cfg)
    gen = torch.Generator().manual_seed(3)
    n = 700
    k = torch.randn(n, h, 256, generator=gen)
    k[..., :8] *= 20
    k = k.bfloat16()
    v = torch.randn(n, h, 256, generator=gen).bfloat16()
    k[0].zero_()
    k[1].fill_(0.5)
    k[2].fill_(1e-12)
    v[3].fill_(-3)
    k[4, 0] = (torch.arange(256).float().remainder(11) - 5).bfloat16()
    v[5] = (torch.randn(h, 256, generator=gen) * 3000 - 70000).bfloat16()  # fp16 zero -inf: codes 0
    pages = 4
    cache = cache_stripes(pages, 768, h, DEV)
    history, _ = layout.tensor_views(cache)
    perm = torch.randperm(pages * 768 - 768, generator=gen)[:n] + 768  # page 0 untouched
    slots = perm.long()
    slots[::64] = -1
    active = n - 5  # the last 5 tokens are beyond counts[1]
    counts = torch.tensor([1, active], dtype=torch.int32)
    kernels.store_int2(k.to(DEV), v.to(DEV), history, slots.to(DEV), counts.to(DEV), layout)
    got = history.cpu().numpy()
    expect = oo.packed_slots(k, v, cfg).numpy()
    ref = np.full_like(got, 0x5A)
    for t in range(active):
        s = int(slots[t])
        if s < 0:
            continue
        for hh in range(h):
            off = layout.slot_offset(s, hh)
            ref[off : off + 136] = expect[t, hh, :136]
    mism = np.nonzero(got != ref)[0]
    assert mism.size == 0, f"{mism.size} bytes differ, first at {mism[:5]}"


def test_rotate_strided_matches_torch(cuda_lib):
    torch.manual_seed(7)
    x = torch.randn(23, 12, 256, device=DEV, dtype=torch.bfloat16)[:, ::2]
    r = torch.linalg.qr(torch.randn(256, 256))[0].bfloat16().to(DEV).T
    out = kernels.rotate(x, r)
    ref = (x.float() @ r.float()).bfloat16().float()
    torch.testing.assert_close(out.float(), ref, atol=0.03125, rtol=0.015)


def test_rotate_store_fused_bytes_and_rotation(cuda_lib):
    cfg = OscarConfig()
    h, hq = 4, 24
    layout = CacheLayout(768, kv_heads=h, config=cfg)
    gen = torch.Generator().manual_seed(11)
    n = 300
    k = torch.randn(n, h, 256, generator=gen)
    k[..., :8] *= 20
    k = k.bfloat16()
    v = torch.randn(n, h, 256, generator=gen).bfloat16()
    q = torch.randn(n, hq, 256, generator=gen).bfloat16()
    rk, rv = rotation(1).bfloat16(), rotation(2).bfloat16()
    cache = cache_stripes(3, 768, h, DEV)
    history, _ = layout.tensor_views(cache)
    slots = (torch.randperm(2 * 768, generator=gen)[:n] + 768).long()
    slots[7] = -1
    counts = torch.tensor([1, n], dtype=torch.int32)
    qrot, krot, vrot = kernels.rotate_store(k.to(DEV), v.to(DEV), rk.to(DEV), rv.to(DEV), history, slots.to(DEV),
                                            counts.to(DEV), layout, query=q.to(DEV), debug_rotated=True)
    torch.testing.assert_close(krot.float().cpu(), (k.float() @ rk.float()).bfloat16().float(), atol=0.03125,
                               rtol=0.015)
    torch.testing.assert_close(vrot.float().cpu(), (v.float() @ rv.float()).bfloat16().float(), atol=0.03125,
                               rtol=0.015)
    torch.testing.assert_close(qrot.float().cpu(), (q.float() @ rk.float()).bfloat16().float(), atol=0.03125,
                               rtol=0.015)
    # bytes: bit-exact given the kernel's own bf16 rotated rows
    expect = oo.packed_slots(krot.cpu(), vrot.cpu(), cfg).numpy()
    got = history.cpu().numpy()
    for t in range(n):
        s = int(slots[t])
        for hh in range(h):
            if s < 0:
                continue
            off = layout.slot_offset(s, hh)
            assert (got[off : off + 136] == expect[t, hh, :136]).all(), (t, hh)
            assert (got[off + 136 : off + 160] == 0x5A).all()


def _check_store_bytes(history, layout, slots, krot, vrot, cfg):
    """Every written slot bit-exact vs the oracle quantiser on the kernel's own bf16
    rotated rows; every other byte of the stripe still holds the 0x5A sentinel."""
    expect = oo.packed_slots(krot.cpu(), vrot.cpu(), cfg).numpy()  # [n, H, 160]
    got = history.cpu().numpy()
    written = np.zeros(got.shape[0], dtype=bool)
    s = slots.cpu().numpy()
    live = np.nonzero(s >= 0)[0]
    for hh in range(layout.kv_heads):
        addr = oo.slot_addresses(s[live], hh, layout)
        idx = addr[:, None] + np.arange(136)[None, :]
        np.testing.assert_array_equal(got[idx], expect[live, hh, :136])
        written[idx.reshape(-1)] = True
    assert (got[~written] == 0x5A).all()


def test_rotate_store_config2_tcgen05(cuda_lib):
    """Config 2 at full size: 16384 tokens x 4 heads (tcgen05 + TMA tiles), K/V clip
    .96/.92, a seeded shuffle of distinct slots in 22 pages with every 64th slot -1."""
    cfg = OscarConfig()
    h, n, pages = 4, 16384, 22
    layout = CacheLayout(768, kv_heads=h, config=cfg)
    gen = torch.Generator().manual_seed(202)
    k = torch.randn(n, h, 256, generator=gen)
    k[..., :8] *= 20
    k = k.bfloat16().to(DEV)
    v = torch.randn(n, h, 256, generator=gen).bfloat16().to(DEV)
    rk, rv = rotation(1).bfloat16().to(DEV), rotation(2).bfloat16().to(DEV)
    slots = torch.randperm(pages * 768, generator=gen)[:n].long()
    slots[::64] = -1
    cache = cache_stripes(pages, 768, h, DEV)
    history, _ = layout.tensor_views(cache)
    counts = torch.tensor([1, n], dtype=torch.int32, device=DEV)
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        _, krot, vrot = kernels.rotate_store(k, v, rk, rv, history, slots.to(DEV), counts, layout,
                                             debug_rotated=True)
        torch.cuda.synchronize()
    names = {e.name for e in prof.events()}
    assert any("rotate_tc_kernel" in nm for nm in names), names  # the tcgen05 path ran
    torch.testing.assert_close(krot.float(), (k.float() @ rk.float()).bfloat16().float(), atol=0.03125, rtol=0.015)
    torch.testing.assert_close(vrot.float(), (v.float() @ rv.float()).bfloat16().float(), atol=0.03125, rtol=0.015)
    assert rel_err(krot, k.float() @ rk.float()) < 1e-2
    _check_store_bytes(history, layout, slots, krot, vrot, cfg)


def test_rotate_store_prefill_chunk_with_query_tcgen05(cuda_lib):
    """K, V and Q jobs in one tcgen05 launch (Q: 24 heads -> 120-row tiles), strided
    fused-QKV views, a token count that is not a tile multiple, counts below n."""
    cfg = OscarConfig()
    h, hq, n = 4, 24, 1031
    layout = CacheLayout(768, kv_heads=h, config=cfg)
    gen = torch.Generator().manual_seed(203)
    qkv = torch.randn(n, hq + 2 * h, 256, generator=gen)
    qkv[:, hq : hq + h, :8] *= 20
    qkv = qkv.bfloat16().to(DEV)
    q, k, v = qkv[:, :hq], qkv[:, hq : hq + h], qkv[:, hq + h :]
    rk, rv = rotation(3).bfloat16().to(DEV), rotation(4).bfloat16().to(DEV)
    slots = torch.randperm(2 * 768, generator=gen)[:n].long() + 768
    cache = cache_stripes(3, 768, h, DEV)
    history, _ = layout.tensor_views(cache)
    active = n - 5
    counts = torch.tensor([1, active], dtype=torch.int32, device=DEV)
    qrot, krot, vrot = kernels.rotate_store(k, v, rk, rv, history, slots.to(DEV), counts, layout, query=q,
                                            debug_rotated=True)
    for got, x, r in ((qrot, q, rk), (krot, k, rk), (vrot, v, rv)):
        torch.testing.assert_close(got.float().view(n, -1, 256), (x.float() @ r.float()).bfloat16().float(),
                                   atol=0.03125, rtol=0.015)
    masked = slots.clone()
    masked[active:] = -1  # tokens at or beyond counts[1] are not stored
    _check_store_bytes(history, layout, masked, krot.view(n, h, 256), vrot.view(n, h, 256), cfg)


def _edge_rows(gen, count):
    """[count, 256] fp32 rows that stress the exact quantiser: the middle code boundary
    at zero (symmetric data), ties at the percentile ranks, constant rows, tiny and
    huge magnitudes (a minimum below -65504 makes the fp16 zero -inf: every reference
    code is 0), mixed binades, a lone outlier."""
    kinds = [
        lambda: torch.rand(256, generator=gen) * 3 - 1.5,
        lambda: torch.randint(-4, 5, (256,), generator=gen).float() * 0.25,
        lambda: torch.full((256,), 0.0),
        lambda: torch.full((256,), 0.5),
        lambda: torch.full((256,), -3.0),
        lambda: torch.full((256,), 1e-12),
        lambda: torch.randn(256, generator=gen) * 1e-20,
        lambda: torch.randn(256, generator=gen) * 3000 + 20000,
        lambda: torch.randn(256, generator=gen) * 3000 - 70000,
        lambda: torch.randn(256, generator=gen) * 3000 + 70000,
        lambda: torch.randn(256, generator=gen) * torch.logspace(-6, 4, 256),
        lambda: torch.cat([torch.full((1,), 5000.0), torch.randn(255, generator=gen) * 1e-3]),
        lambda: torch.cat([torch.full((24,), -2.0), torch.full((24,), 2.0), torch.randn(208, generator=gen)]),
        lambda: (torch.arange(256).float().remainder(11) - 5),
        lambda: torch.randn(256, generator=gen),
    ]
    pick = torch.randint(0, len(kinds), (count,), generator=gen)
    return torch.stack([kinds[int(i)]()[torch.randperm(256, generator=gen)] for i in pick])


@pytest.mark.parametrize("n", [600, 3000])  # 16-row mma.sync tiles / tcgen05 tiles
@pytest.mark.parametrize("kr,vr,mode", [(0.96, 0.92, "percentile"), (0.875, 0.0, "percentile"),
                                        (1.0, 1.0, "percentile"), (0.96, 0.92, "factor")])
def test_rotate_store_quantiser_edge_rows(cuda_lib, n, kr, vr, mode):
    """Identity rotations hand the epilogue the input rows unchanged, so adversarial
    rows reach the exact quantiser directly; bytes bit-exact vs the oracle."""
    cfg = replace(OscarConfig(), k_clip_ratio=kr, v_clip_ratio=vr, clip_mode=mode, k_clip_factor=0.9,
                  v_clip_factor=0.75)
    h = 4
    layout = CacheLayout(768, kv_heads=h, config=cfg)
    gen = torch.Generator().manual_seed(n + int(kr * 100))
    k = _edge_rows(gen, n * h).view(n, h, 256).bfloat16()
    v = _edge_rows(gen, n * h).view(n, h, 256).bfloat16()
    eye = torch.eye(256).bfloat16().to(DEV)
    pages = (n + 767) // 768 + 1
    slots = torch.randperm(pages * 768, generator=gen)[:n].long()
    slots[::97] = -1
    cache = cache_stripes(pages, 768, h, DEV)
    history, _ = layout.tensor_views(cache)
    counts = torch.tensor([1, n], dtype=torch.int32, device=DEV)
    _, krot, vrot = kernels.rotate_store(k.to(DEV), v.to(DEV), eye, eye, history, slots.to(DEV), counts, layout,
                                         debug_rotated=True)
    assert torch.equal(krot.cpu(), k) and torch.equal(vrot.cpu(), v)
    _check_store_bytes(history, layout, slots, k, v, cfg)


def test_rotate_large_column_major_rotation_tcgen05(cuda_lib):
    """Plain rotation with a transposed (column-major) rotation view: the K-major B
    operand path of the tcgen05 kernel; 6 heads per token (126-row tiles)."""
    torch.manual_seed(8)
    x = torch.randn(4096, 12, 256, device=DEV, dtype=torch.bfloat16)[:, ::2]
    r = torch.linalg.qr(torch.randn(256, 256))[0].bfloat16().to(DEV).T
    out = kernels.rotate(x, r)
    ref = (x.float() @ r.float()).bfloat16().float()
    torch.testing.assert_close(out.float(), ref, atol=0.03125, rtol=0.015)


def test_unpack_matches_golden(cuda_lib):
    fx = load("unpack.pt")
    layout = CacheLayout(768, kv_heads=1)
    rows = fx["vectors"].shape[0]
    cache = cache_stripes(1, 768, 1, DEV)
    history, _ = layout.tensor_views(cache)
    for r in range(rows):
        off = layout.slot_offset(r)
        history[off : off + 68] = fx["vectors"][r].to(DEV)
        history[off + 68 : off + 136] = fx["vectors"][r].to(DEV)
    eye = torch.eye(256, dtype=torch.bfloat16, device=DEV)
    kd, vd = kernels.dequant_inverse_rotate(history, torch.arange(rows, device=DEV), eye, eye, layout)
    assert torch.equal(kd[:, 0].cpu().view(torch.int16), fx["decoded"].view(torch.int16))
    assert torch.equal(vd[:, 0].cpu().view(torch.int16), fx["decoded"].view(torch.int16))


# ----------------------------------------------------------------------------
# tasks / windows / merges
# ----------------------------------------------------------------------------


def test_prepare_tasks_matches_reference_body(cuda_lib):
    for case in load("tasks.pt"):
        tasks = torch.full((case["capacity"], 2), -7, dtype=torch.int32, device=DEV)
        count = torch.zeros(1, dtype=torch.int32, device=DEV)
        kernels.prepare_tasks(case["qstarts"].to(DEV), case["counts"].to(DEV), tasks, count,
                              case["qstarts"].numel() - 1, case["query_tile"])
        c = int(count.item())
        assert c == case["count"]
        assert torch.equal(tasks[:c].cpu(), case["tasks"][:c])


def test_prepare_tasks_copies_table_columns(cuda_lib):
    src = torch.arange(5 * 40, dtype=torch.int32, device=DEV).view(5, 40)
    dst = torch.full((8, 64), -1, dtype=torch.int32, device=DEV)
    qs = torch.tensor([0, 1, 2, 3, 3, 3, 3, 3, 3], dtype=torch.int32, device=DEV)
    counts = torch.tensor([3, 3], dtype=torch.int32, device=DEV)
    tasks = torch.zeros((task_capacity(3, 8, 4), 2), dtype=torch.int32, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.prepare_tasks(qs, counts, tasks, cnt, 8, 4, source_table=src, table=dst, copy_columns=17)
    assert torch.equal(dst[:3, :17], src[:3, :17])
    assert (dst[3:] == -1).all() and (dst[:, 17:] == -1).all()


def _stage(bufs_cap, **kw):
    from oscar_new_b200.metadata import StepBuffers

    bufs = StepBuffers(bufs_cap, DEV)
    bufs.arena.fill_(-7)
    bufs.slot_mapping.fill_(-9)
    bufs.stage(**kw)
    return bufs


def test_stage_step_metadata_matches_reference_task_body(cuda_lib):
    """One staging launch: counts, starts, lengths, reachable table columns, slots, and
    the task table of the reference kernel body (golden fixture)."""
    from types import SimpleNamespace

    from oscar_new_b200.metadata import StepCapacity

    for case in load("tasks.pt"):
        nr, nt = int(case["counts"][0]), int(case["counts"][1])
        cap = StepCapacity(requests=nr + 1, tokens=max(nt, 1) + 3, columns=23, query_tile=case["query_tile"])
        assert cap.tasks >= case["count"]
        g = torch.Generator().manual_seed(nr)
        src = SimpleNamespace(query_start_loc=case["qstarts"][:nr + 1].to(DEV),
                              seq_lens=torch.randint(1, 1 << 20, (nr,), generator=g, dtype=torch.int32).to(DEV),
                              block_table_tensor=torch.randint(0, 1 << 30, (nr, 40), generator=g,
                                                               dtype=torch.int32).to(DEV)[:, 3:31],
                              slot_mapping=torch.randint(-1, 1 << 40, (nt,), generator=g).to(DEV))
        b = _stage(cap, source=src, num_reqs=nr, num_tokens=nt, copy_columns=17)
        assert b.counts.tolist() == [nr, nt]
        assert torch.equal(b.query_start_loc[:nr + 1], src.query_start_loc)
        assert torch.equal(b.seq_lens[:nr], src.seq_lens)
        assert torch.equal(b.block_tables[:nr, :17], src.block_table_tensor[:, :17])
        assert (b.block_tables[:, 17:] == -7).all() and (b.block_tables[nr:] == -7).all()
        assert torch.equal(b.slot_mapping[:nt], src.slot_mapping)
        assert (b.slot_mapping[nt:] == -9).all()
        c = int(b.task_count.item())
        assert c == case["count"]
        assert torch.equal(b.tasks[:c].cpu(), case["tasks"][:c])
        want, wc = oo.prepare_tasks(case["qstarts"], case["counts"], case["query_tile"], cap.tasks)
        assert wc == c and torch.equal(b.tasks[:c].cpu(), want[:c])


def test_stage_dummy_step_zeroes_counts_and_touches_nothing_else(cuda_lib):
    from oscar_new_b200.metadata import StepCapacity

    b = _stage(StepCapacity(requests=5, tokens=40, columns=9, query_tile=4))
    assert b.counts.tolist() == [0, 0] and int(b.task_count.item()) == 0
    assert (b.arena[3:] == -7).all() and (b.slot_mapping == -9).all()


@pytest.mark.parametrize("seq,qlen", [([30, 70, 5], [20, 4, 5]), ([1500, 40, 700], [1200, 40, 3])])
def test_store_windows_matches_oracle(cuda_lib, seq, qlen):
    """Sink and ring slots (latest writer only), short and prefill-sized chunks."""
    cfg = make_config(sink=4, recent=16, mtp=3)
    sc = Scenario(seq, qlen, hq=6, h=2, cfg=cfg, block_tokens=256, seed=5)
    q, k, v = sc.current()
    before = sc.window.cpu()
    kernels.store_windows(k, v, sc.window, sc.meta, sc.layout)
    meta_cpu = type("M", (), {})()
    for name in ("query_start_loc", "seq_lens", "block_tables", "counts"):
        setattr(meta_cpu, name, getattr(sc.meta, name).cpu())
    expect = oo.store_windows(k.cpu(), v.cpu(), before.clone(), meta_cpu, sc.layout, min(k.shape[0], sc.meta.max_num_reqs))
    assert torch.equal(sc.window.cpu().view(torch.int16), expect.view(torch.int16))


def test_merge_splits_and_paths_match_oracle(cuda_lib):
    gen = torch.Generator().manual_seed(4)
    n, hq, s = 9, 6, 5
    part = torch.randn(n, hq, s, 256, generator=gen)
    lse = torch.randn(n, hq, s, generator=gen) * 3
    lse[0, 0] = -float("inf")  # empty row
    lse[1, :, 2] = -float("inf")  # empty split
    counts = torch.tensor([3, 7], dtype=torch.int32)
    out, ls = kernels.merge_splits(part.to(DEV), lse.to(DEV), counts.to(DEV))
    eo, el = oo.merge_splits(part, lse, counts)
    torch.testing.assert_close(out.float().cpu(), eo.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(ls.cpu(), el, atol=1e-5, rtol=1e-5)
    raw = torch.randn(n, hq, 1, 256, generator=gen)
    rl = torch.randn(n, hq, 1, generator=gen)
    dst = torch.empty(n, hq * 256, dtype=torch.bfloat16, device=DEV)
    kernels.merge_paths(out, ls, raw.to(DEV), rl.to(DEV), counts.to(DEV), dst)
    expect = oo.merge_paths(out.cpu(), ls.cpu(), raw[:, :, 0], rl[:, :, 0], counts)
    torch.testing.assert_close(dst.view(n, hq, 256).float().cpu(), expect.float(), atol=1e-2, rtol=1e-2)
    assert (dst.view(n, hq, 256)[7:] == 0).all()


# ----------------------------------------------------------------------------
# attention partials against the reference kernel body (golden)
# ----------------------------------------------------------------------------


@pytest.mark.parametrize("index", [0, 1, 2])
def test_attention_partials_match_reference_kernel(cuda_lib, index):
    case = load("attention_kernel.pt")[index]
    cfg = make_config(case["sink"], case["recent"], case["mtp"])
    layout = CacheLayout(case["bp"], kv_heads=case["h"], config=cfg)
    hist = unzpack(case["history"]).to(DEV)
    win = unzpack(case["window"]).to(DEV)
    m = case["meta"]
    meta = type("M", (), {})()
    for name in ("query_start_loc", "seq_lens", "block_tables", "counts"):
        setattr(meta, name, m[name].to(DEV))
    n = case["q"].shape[0]
    meta.max_num_reqs = m["block_tables"].shape[0]
    meta.tasks = torch.full((task_capacity(n, meta.max_num_reqs, 4), 2), -1, dtype=torch.int32, device=DEV)
    meta.task_count = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels.prepare_tasks(meta.query_start_loc, meta.counts, meta.tasks, meta.task_count, meta.max_num_reqs, 4)
    q, qrot, k, v = (case[x].to(DEV) for x in ("q", "qrot", "k", "v"))
    hp, hl = kernels.attention_partials(qrot, k, v, hist, win, meta, layout, 1 / 16, case["splits"], False)
    live = ~torch.isnan(case["hist_lse"])
    ref_l, got_l = case["hist_lse"][live], hl.cpu()[live]
    assert torch.equal(torch.isinf(ref_l), torch.isinf(got_l))
    fin = torch.isfinite(ref_l)
    torch.testing.assert_close(got_l[fin], ref_l[fin], atol=1e-3, rtol=0)
    torch.testing.assert_close(hp.cpu()[live], case["hist_partials"][live], atol=0.035, rtol=0.04)
    rp, rl = kernels.attention_partials(q, k, v, hist, win, meta, layout, 1 / 16, 1, True)
    live = ~torch.isnan(case["raw_lse"])
    torch.testing.assert_close(rl.cpu()[live], case["raw_lse"][live], atol=1e-3, rtol=0)
    torch.testing.assert_close(rp.cpu()[live], case["raw_partials"][live], atol=0.035, rtol=0.04)


# ----------------------------------------------------------------------------
# end-to-end decode / verify against the reference's dense hybrid oracle
# ----------------------------------------------------------------------------


@pytest.mark.parametrize(
    "name,seq,qlen,hq,h,cfg,splits",
    [
        ("config1", [300, 1000, 2500, 4096], [1, 1, 1, 1], 8, 1, make_config(4, 64, 0), 4),
        ("gqa24x4", [700, 1500, 3000], [1, 1, 1], 24, 4, make_config(4, 128, 0), 16),
        ("mtp_verify", [900, 2049, 1400], [4, 4, 3], 24, 4, make_config(4, 128, 3), 8),
        ("prefill_chunk", [1700], [900], 6, 1, make_config(64, 256, 3), 1),
        ("empty_history", [4], [4], 6, 1, make_config(64, 256, 3), 32),
        ("ragged_overlap", [69, 263], [4, 3], 6, 1, make_config(64, 256, 3), 16),
        # skewed lengths: balanced splits give the long request most of the 64 splits
        ("skewed_balanced", [140, 9000, 333, 2, 1500], [4, 4, 1, 2, 4], 24, 4, make_config(4, 128, 3), 64),
        # launch shapes: 8 KV heads x 2 row tiles (8-warp CTAs), 2 KV heads x 3 row tiles
        # (12-warp CTA, two warps per unit), 8 row tiles per KV head (GQA 16 at MTP verify)
        ("wide_8heads", [1300, 2600], [4, 4], 32, 8, make_config(4, 128, 3), 8),
        ("mid_2heads", [1100, 3100], [4, 3], 12, 2, make_config(4, 128, 3), 8),
        ("group16_mtp", [800, 1900], [4, 4], 32, 2, make_config(4, 128, 3), 4),
    ],
)
def test_decode_step_matches_hybrid_reference(cuda_lib, name, seq, qlen, hq, h, cfg, splits):
    sc = Scenario(seq, qlen, hq=hq, h=h, cfg=cfg, seed=len(name))
    out = sc.run_step(splits).float().cpu()
    expect, _ = sc.expected()
    assert rel_err(out, expect) < 1e-2, rel_err(out, expect)
    torch.testing.assert_close(out, expect, atol=0.035, rtol=0.04)


@pytest.mark.parametrize(
    "name,seq,qlen,hq,h,cfg,splits",
    [
        ("mtp_verify", [900, 2049, 1400], [4, 4, 3], 24, 4, make_config(4, 128, 3), 8),
        ("skewed_balanced", [140, 9000, 333, 2, 1500], [4, 4, 1, 2, 4], 24, 4, make_config(4, 128, 3), 64),
        ("group4_16rows", [1300, 2600], [4, 4], 16, 4, make_config(4, 128, 3), 8),
        ("mid_2heads", [1100, 3100], [4, 3], 12, 2, make_config(4, 128, 3), 8),
    ],
)
@pytest.mark.parametrize("mtp_env,kernel", [("1", "history_mtp_kernel"), ("0", "history_attention_kernel")])
def test_decode_step_mtp_kernel_choice(cuda_lib, monkeypatch, mtp_env, kernel, name, seq, qlen, hq, h, cfg, splits):
    """16 and 24 rows per KV head: the shared-operand MTP kernel (the default; four warps
    per KV head) and, with OSCAR_HISTORY_MTP=0, the per-row-tile kernel, both against the
    dense hybrid reference; which kernel ran is asserted by name."""
    monkeypatch.setenv("OSCAR_HISTORY_MTP", mtp_env)
    sc = Scenario(seq, qlen, hq=hq, h=h, cfg=cfg, seed=len(name))
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        out = sc.run_step(splits).float().cpu()
        torch.cuda.synchronize()
    names = {e.name for e in prof.events()}
    assert any(kernel in nm for nm in names), names
    expect, _ = sc.expected()
    assert rel_err(out, expect) < 1e-2, rel_err(out, expect)
    torch.testing.assert_close(out, expect, atol=0.035, rtol=0.04)


def test_history_lse_matches_oracle(cuda_lib):
    sc = Scenario([3000, 1200], [1, 1], hq=24, h=4, cfg=make_config(4, 128, 0), seed=9)
    q, k, v = sc.current()
    sc.prepare_tasks()
    qrot = kernels.rotate(q, sc.rk.to(DEV))
    hp, hl = kernels.attention_partials(qrot, k, v, sc.history, sc.window, sc.meta, sc.layout, 1 / 16, 16, False)
    hrot, hls = kernels.merge_splits(hp, hl, sc.meta.counts)
    meta_cpu = type("M", (), {})()
    for nm in ("query_start_loc", "seq_lens", "block_tables", "counts"):
        setattr(meta_cpu, nm, getattr(sc.meta, nm).cpu())
    ep, el = oo.attention_partials(qrot.cpu(), k.cpu(), v.cpu(), sc.history.cpu(), sc.window.cpu(), meta_cpu,
                                   sc.layout, 1 / 16, 1, False)
    torch.testing.assert_close(hls.cpu(), el[:, :, 0], atol=1e-3, rtol=0)
    assert rel_err(hrot.cpu(), ep[:, :, 0]) < 1e-2


def test_graph_capture_with_zero_counts_then_replay(cuda_lib):
    """Reference tests/test_npu_kernels.py:197-245 on a CUDA graph."""
    cfg = make_config(64, 256, 3)
    sc = Scenario([4], [4], hq=6, h=1, cfg=cfg, seed=10, max_reqs=4)
    q, k, v = sc.current()
    rk = rv = torch.eye(256, device=DEV, dtype=torch.bfloat16)
    sc.rk = sc.rv = rk.cpu()
    m = sc.meta
    out = torch.empty((4, 6 * 256), dtype=torch.bfloat16, device=DEV)
    scratch = kernels.DecodeScratch(4, 6, 8, DEV)

    def step():
        kernels.prepare_tasks(m.query_start_loc, m.counts, m.tasks, m.task_count, m.max_num_reqs, 4)
        qrot = kernels.rotate_store(k, v, rk, rv, sc.history, m.slot_mapping, m.counts, sc.layout, query=q)
        kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, m, sc.layout, 1 / 16, 8, rv, out, scratch)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    m.counts.zero_()
    before = sc.history.clone(), sc.window.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    torch.cuda.synchronize()
    assert torch.equal(sc.history, before[0]) and torch.equal(sc.window, before[1])
    # replay with two requests of two tokens each on new pages
    m.query_start_loc.copy_(torch.tensor([0, 2, 4, 4, 4], dtype=torch.int32, device=DEV))
    m.seq_lens[:2].fill_(2)
    m.counts.copy_(torch.tensor([2, 4], dtype=torch.int32, device=DEV))
    m.block_tables[0, :6].copy_(torch.arange(6, 12, dtype=torch.int32, device=DEV))
    m.block_tables[1, :6].copy_(torch.arange(12, 18, dtype=torch.int32, device=DEV))
    m.slot_mapping.copy_(torch.tensor([6 * 128, 6 * 128 + 1, 12 * 128, 12 * 128 + 1], device=DEV))
    q.normal_(), k.normal_(), v.normal_()
    graph.replay()
    torch.cuda.synchronize()
    expect = torch.cat([
        oo.hybrid_reference(q[i : i + 2].cpu(), k[i : i + 2].cpu(), v[i : i + 2].cpu(), 0, rk.cpu(), rv.cpu(), cfg)
        for i in (0, 2)
    ])
    torch.testing.assert_close(out.view(4, 6, 256).float().cpu(), expect, atol=0.035, rtol=0.04)


def test_ring_survives_mtp_rejection(cuda_lib):
    """Reference tests/test_npu_kernels.py:248-290: prefix written by the device store
    kernels, then verify steps whose rejected drafts roll back."""
    cfg = make_config(64, 256, 3)
    layout = CacheLayout(768, kv_heads=1, config=cfg)
    from oscar_new_b200.synthetic import plan_pages

    plan = plan_pages([1600], [1600], 768, seed=81, max_reqs=2)
    cache = cache_stripes(plan.num_pages, 768, 1, DEV)
    hist, win = layout.tensor_views(cache)
    rk = rv = torch.eye(256, device=DEV, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(81)
    keys = torch.randn(1600, 1, 256, generator=gen).bfloat16()
    values = torch.randn(1600, 1, 256, generator=gen).bfloat16()
    meta = plan.meta(DEV)
    prefix = 900
    # prefix via the device kernels
    meta.query_start_loc[:2] = torch.tensor([0, prefix], dtype=torch.int32)
    meta.seq_lens[0] = prefix
    meta.counts.copy_(torch.tensor([1, prefix], dtype=torch.int32))
    slots = plan.slots_of(0, range(prefix)).to(DEV)
    kernels.rotate_store(keys[:prefix].to(DEV), values[:prefix].to(DEV), rk, rv, hist, slots, meta.counts, layout)
    kernels.store_windows(keys[:prefix].to(DEV), values[:prefix].to(DEV), win, meta, layout)
    for rejected in (3, 2, 0, 3, 1):
        keys[prefix : prefix + 4] = torch.randn(4, 1, 256, generator=gen).bfloat16()
        values[prefix : prefix + 4] = torch.randn(4, 1, 256, generator=gen).bfloat16()
        q = torch.randn(4, 6, 256, generator=gen).bfloat16()
        meta.query_start_loc[:2] = torch.tensor([0, 4], dtype=torch.int32)
        meta.seq_lens[0] = prefix + 4
        meta.counts.copy_(torch.tensor([1, 4], dtype=torch.int32))
        slots = plan.slots_of(0, range(prefix, prefix + 4)).to(DEV)
        k, v = keys[prefix : prefix + 4].to(DEV), values[prefix : prefix + 4].to(DEV)
        kernels.prepare_tasks(meta.query_start_loc, meta.counts, meta.tasks, meta.task_count, meta.max_num_reqs, 4)
        qrot = kernels.rotate_store(k, v, rk, rv, hist, slots, meta.counts, layout, query=q.to(DEV))
        out = torch.empty(4, 6 * 256, dtype=torch.bfloat16, device=DEV)
        kernels.decode_attention(qrot, q.to(DEV), k, v, hist, win, meta, layout, 1 / 16, 16, rv, out)
        expect = oo.hybrid_reference(q, keys[: prefix + 4], values[: prefix + 4], prefix, rk.cpu(), rv.cpu(), cfg)
        torch.testing.assert_close(out.view(4, 6, 256).float().cpu(), expect, atol=0.035, rtol=0.04)
        prefix += 4 - rejected


# ----------------------------------------------------------------------------
# calibration
# ----------------------------------------------------------------------------


def test_streamed_covariances_against_fp64(cuda_lib):
    """Reference tests/test_npu_calibration.py:18-37, generalised to 4 KV heads."""
    torch.manual_seed(88)
    q = torch.randn(137, 6, 256).bfloat16()
    k, v = torch.randn(137, 4, 256).bfloat16(), torch.randn(137, 4, 256).bfloat16()
    qsum = torch.zeros((256, 256), device=DEV)
    for chunk in q.split(32):
        ck.accumulate_gram(chunk.to(DEV), qsum)
    qcov = ck.normalize(qsum, 137 * 6)
    expect_q = co.gram(q) / (137 * 6)
    torch.testing.assert_close(qcov.cpu().double(), expect_q, atol=2e-5, rtol=2e-5)
    vsum = torch.zeros_like(qsum)
    den = torch.zeros((), device=DEV)
    for kc, vc in zip(k.split(32), v.split(32)):
        w = ck.sst_weights(kc.to(DEV), qcov, den)
        ck.accumulate_gram(vc.to(DEV), vsum, w)
    got = ck.normalize(vsum, den).cpu().double()
    w = co.sst_weights(k, expect_q)
    expect_v = co.weighted_gram(v, w) / w.sum()
    torch.testing.assert_close(got, expect_v, atol=2e-4, rtol=2e-4)


@pytest.mark.parametrize("weighted", [False, True])
def test_gram_tcgen05_matches_fp64_and_the_mma_sync_gram(cuda_lib, monkeypatch, weighted):
    """The tcgen05 Gram (default) on grouped rows: 24 query heads in 4 groups of 6 (a
    64-row block holds 60 rows), or 4 KV heads one per group with per-row weights;
    1003 tokens (not a multiple of a block), a strided view, outlier channels.  Against
    fp64 and against the mma.sync Gram (OSCAR_GRAM_MMA=1)."""
    torch.manual_seed(57 + weighted)
    n, h, groups = (1003, 4, 4) if weighted else (1003, 24, 4)
    x = torch.randn(n, 2 * h, 256)
    x[..., :8] *= 20
    x = x.bfloat16()[:, ::2]
    w = torch.rand(n * h) * 3 if weighted else None
    hpg = h // groups
    xd = x.double().view(n, groups, hpg, 256)
    wd = None if w is None else w.double().view(n, groups, hpg, 1)
    expect = torch.einsum("ngpi,ngpj->gij", xd, xd if wd is None else xd * wd)

    def run():
        cov = torch.zeros((groups, 256, 256), device=DEV)
        ck.accumulate_gram_grouped(x.to(DEV), cov, None if w is None else w.to(DEV))
        return cov

    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        got = run()
        torch.cuda.synchronize()
    assert any("gram_tc_kernel" in e.name for e in prof.events())
    scale = float(expect.abs().max())
    torch.testing.assert_close(got.cpu().double(), expect, rtol=1e-5, atol=2e-6 * scale)
    monkeypatch.setenv("OSCAR_GRAM_MMA", "1")
    ref = run()
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=2e-6 * scale)


def test_sst_weights_match_fp64(cuda_lib):
    """w = max(k C k^T, 0) per row and the weight totals against fp64: per-head and
    shared covariances (outlier channels), 150 tokens (not a multiple of the 64-row
    tile), a strided key view."""
    torch.manual_seed(31)
    n, h = 150, 4
    k = torch.randn(n, 2 * h, 256).bfloat16()[:, ::2]
    x = torch.randn(h, 600, 256)
    x[..., :8] *= 20
    covs = x.transpose(-1, -2) @ x / 600
    kd = k.double()
    expect = torch.einsum("nhi,hij,nhj->nh", kd, covs.double(), kd).clamp_min(0)
    totals = torch.zeros(h, device=DEV)
    w = ck.sst_weights_per_head(k.to(DEV), covs.to(DEV), totals)
    scale = float(expect.abs().max())
    torch.testing.assert_close(w.cpu().double().view(n, h), expect, rtol=1e-5, atol=1e-6 * scale)
    torch.testing.assert_close(totals.cpu().double(), expect.sum(0), rtol=1e-5, atol=0.0)
    total = torch.zeros((), device=DEV)
    w1 = ck.sst_weights(k.to(DEV), covs[1].to(DEV), total)
    expect1 = torch.einsum("nhi,ij,nhj->nh", kd, covs[1].double(), kd).clamp_min(0).reshape(-1)
    torch.testing.assert_close(w1.cpu().double(), expect1, rtol=1e-5, atol=1e-6 * float(expect1.max()))
    torch.testing.assert_close(total.cpu().double(), expect1.sum(), rtol=1e-5, atol=0.0)


@pytest.mark.parametrize("n,strided", [(300, True), (1024, False)])
def test_sst_weights_tcgen05_from_split_covariances(cuda_lib, n, strided):
    """The exact three-part bf16 split of the covariances, and the tcgen05 SST kernel
    fed by it (called through the C ABI, so a fallback cannot hide) against fp64: 300
    rows (not a multiple of the 128-row tile) of a strided key view, and the config-5
    call shape (1024 tokens x 4 KV heads)."""
    torch.manual_seed(37 + n)
    h = 4
    k = torch.randn(n, 2 * h, 256).bfloat16()[:, ::2] if strided else torch.randn(n, h, 256).bfloat16()
    x = torch.randn(h, 700, 256)
    x[..., :8] = 20 * torch.distributions.StudentT(3.0).sample((h, 700, 8))
    covs = (x.transpose(-1, -2) @ x / 700).to(DEV)
    parts = ck.prepare_sst_covariances(covs)
    assert torch.equal(parts.double().sum(1), covs.double())  # hi + mid + lo == C exactly
    kd = k.double()
    expect = torch.einsum("nhi,hij,nhj->nh", kd, covs.cpu().double(), kd).clamp_min(0)
    kdev = k.to(DEV)
    totals = torch.zeros(h, device=DEV)
    w = torch.empty(n * h, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = _lib.lib().oscar_sst_weights_split(kdev.data_ptr(), n, h, kdev.stride(0), kdev.stride(1), parts.data_ptr(),
                                            w.data_ptr(), totals.data_ptr(), status.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    scale = float(expect.abs().max())
    torch.testing.assert_close(w.cpu().double().view(n, h), expect, rtol=1e-5, atol=1e-6 * scale)
    torch.testing.assert_close(totals.cpu().double(), expect.sum(0), rtol=1e-5, atol=0.0)
    # the wrapper takes the same path when given the prepared parts
    totals2 = torch.zeros(h, device=DEV)
    w2 = ck.sst_weights_per_head(kdev, covs, totals2, prepared=parts)
    assert torch.equal(w2, w)


def test_device_eigensolver_reconstructs_and_matches_eigvalsh(cuda_lib):
    """Reference tests/test_npu_calibration.py:39-57 plus the project targets
    (eigenvalues rel 1e-4, ||R^T R - I|| < 1e-5)."""
    torch.manual_seed(23)
    x = torch.randn(3, 320, 256)
    x[..., :8] *= 5
    cov = x.transpose(-1, -2) @ x / 320
    r, ev, info = ck.calibrated_rotations(cov.to(DEV))
    r, ev = r.cpu().double(), ev.cpu().double()
    assert info["relative_off_diagonal"] < 1e-6
    ref = torch.linalg.eigvalsh(cov.double())
    assert float(((ev - ref).abs() / ref.abs()).max()) < 1e-4
    eye = torch.eye(256, dtype=torch.float64)
    assert float((r.transpose(-1, -2) @ r - eye).norm(dim=(-2, -1)).max()) < 1e-5
    u = r @ co.pbr(256).T @ co.hadamard(256).T
    recon = (u * ev[:, None, :]) @ u.transpose(-1, -2)
    torch.testing.assert_close(recon, cov.double(), atol=2e-4, rtol=2e-3)


def test_bounded_wait_times_out_and_context_stays_usable(cuda_lib):
    """A device wait that nothing can satisfy ends with OSCAR_ERR_TIMEOUT in the status
    word (no hang), and the context keeps working afterwards."""
    import time

    from oscar_new_b200 import _lib

    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    t0 = time.time()
    _lib.call("oscar_selftest_bounded_wait", status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert int(status.item()) == 4, int(status.item())
    assert elapsed < 60, elapsed
    x = torch.randn(16, 2, 256).bfloat16().to(DEV)
    r = rotation(1).bfloat16().to(DEV)
    torch.testing.assert_close(kernels.rotate(x, r).float(), (x.float() @ r.float()).bfloat16().float(),
                               atol=0.03125, rtol=0.015)


def _capture_first_call_check():
    """Body of the next test, run in a fresh process: no eager step before the capture."""
    cfg = make_config(64, 256, 3)
    sc = Scenario([300, 700], [1, 1], hq=6, h=1, cfg=cfg, seed=12, max_reqs=4)
    q, k, v = sc.current()
    m = sc.meta
    rk, rv = sc.rk.to(DEV).bfloat16(), sc.rv.to(DEV).bfloat16()
    out = torch.zeros((q.shape[0], 6 * 256), dtype=torch.bfloat16, device=DEV)
    scratch = kernels.DecodeScratch(q.shape[0], 6, 8, DEV)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        kernels.prepare_tasks(m.query_start_loc, m.counts, m.tasks, m.task_count, m.max_num_reqs, 4)
        qrot = kernels.rotate_store(k, v, rk, rv, sc.history, m.slot_mapping, m.counts, sc.layout, query=q)
        kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, m, sc.layout, 1 / 16, 8, rv, out, scratch)
    graph.replay()
    torch.cuda.synchronize()
    expect, _ = sc.expected()
    torch.testing.assert_close(out.view(-1, 6, 256).float().cpu(), expect, atol=0.035, rtol=0.04)


def test_graph_capture_as_first_decode_call(cuda_lib):
    """The first decode call of a process may come inside a CUDA-graph capture (an engine
    can capture before any eager decode step): the step is captured without the side
    stream, which is only created outside a capture, and replays correctly."""
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    r = subprocess.run([sys.executable, "-c", "import tests.test_gpu_kernels as t; t._capture_first_call_check()"],
                       cwd=root, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
