"""BASELINE config 4 (MTP target verification) at full context lengths against the CPU
oracle: 4 query tokens per request (1 + 3 draft) on the 24 query / 4 KV head D256
layer, ragged contexts from 2048 to 262144 tokens (past 131072, more than 1024 kernel
blocks per request), a padded -1 slot, a zero-length padded row closing the batch, and
balanced splits whose unused slots hold lse -inf.  The cache is written by the product
store kernels (their bytes equal the oracle's, store parity tests); the oracle's decode
step then reads that cache on the host.  Tolerances: output rel 1e-2 in norm and atol
.035 / rtol .04; history LSE 1e-3 abs."""

import math

import pytest
import torch

from oracle import int2_oracle as oo
from oscar_new_b200 import kernels
from oscar_new_b200.config import decode_split_cap
from oscar_new_b200.layout import CacheLayout
from oscar_new_b200.synthetic import cache_stripes, plan_pages, rotation
from tests.helpers import fill_prefixes_on_device, make_config

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_config4_long_ragged_verify_step_matches_oracle(cuda_lib):
    seqs = [262144, 2048, 140001, 33000, 7100, 91234, 0]
    qlens = [4, 4, 4, 4, 4, 4, 0]
    cfg = make_config(4, 128, 3)
    layout = CacheLayout(768, kv_heads=4, config=cfg)
    plan = plan_pages(seqs, qlens, 768, seed=404, max_reqs=8)
    cache = cache_stripes(plan.num_pages, 768, 4, DEV)
    history, window = layout.tensor_views(cache)
    rk, rv = rotation(1).bfloat16().to(DEV), rotation(2).bfloat16().to(DEV)
    fill_prefixes_on_device(plan, layout, history, window, rk, rv, seed=404)
    meta = plan.meta(DEV, cfg.queries_per_tile)
    meta.slot_mapping[1 * 4 + 3] = -1  # the 2048-token request's last draft token is padding
    n = sum(qlens)
    gen = torch.Generator(device=DEV).manual_seed(405)
    q = torch.randn(n, 24, 256, device=DEV, generator=gen).bfloat16()
    k = torch.randn(n, 4, 256, device=DEV, generator=gen)
    k[..., :8] *= 20
    k = k.bfloat16()
    v = torch.randn(n, 4, 256, device=DEV, generator=gen).bfloat16()
    kernels.prepare_tasks(meta.query_start_loc, meta.counts, meta.tasks, meta.task_count, meta.max_num_reqs,
                          cfg.queries_per_tile)
    # oracle inputs: the cache before this step's store (the step's own tokens come from q/k/v)
    hist_cpu = history.cpu().numpy()
    win_cpu = window.cpu()
    qrot = kernels.rotate_store(k, v, rk, rv, history, meta.slot_mapping, meta.counts, layout, query=q)
    splits = decode_split_cap(6, 4, 4, n, 24)
    scratch = kernels.DecodeScratch(n, 24, splits, DEV)
    out = torch.empty((n, 24 * 256), dtype=torch.bfloat16, device=DEV)
    scale = 1 / math.sqrt(256)
    kernels.decode_attention(qrot, q, k, v, history, window, meta, layout, scale, splits, rv, out, scratch,
                             store_window=False)
    torch.cuda.synchronize()

    mh = type("M", (), {})()
    for name in ("query_start_loc", "seq_lens", "block_tables", "counts"):
        setattr(mh, name, getattr(meta, name).cpu())
    want, want_hlse, _ = oo.decode_reference(qrot.cpu(), q.cpu(), k.cpu(), v.cpu(), hist_cpu, win_cpu, mh, layout,
                                             scale, rv.cpu())
    got = out.view(n, 24, 256).float().cpu()
    err = float((got - want.float()).norm() / want.float().norm())
    assert err < 1e-2, err
    torch.testing.assert_close(got, want.float(), atol=0.035, rtol=0.04)

    lse = scratch.lse[:n, :, :splits].cpu()
    got_hlse = torch.logsumexp(lse, dim=-1)
    torch.testing.assert_close(got_hlse, want_hlse.float(), atol=1e-3, rtol=0)
    # balanced splits: the used slots of a row come first, the rest hold -inf
    used = torch.isfinite(lse)
    assert torch.equal(used, used.int().cummin(dim=-1).values.bool())
    per_req = used.sum(-1)[torch.tensor([0, 4, 8, 12, 16, 20])][:, 0]
    assert int(per_req[1]) < int(per_req[0]) <= splits  # the 2048-token request uses fewer splits
    assert int(per_req[1]) >= 1
