"""Test-side helpers: build paged OSCAR caches whose contents come from the CPU oracle."""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import torch

from oracle import int2_oracle as oo
from oscar_new_b200 import kernels
from oscar_new_b200.config import OscarConfig
from oscar_new_b200.layout import CacheLayout
from oscar_new_b200.synthetic import cache_stripes, plan_pages


def make_config(sink=4, recent=64, mtp=0, **kw):
    return replace(OscarConfig(), sink_tokens=sink, recent_tokens=recent, speculative_tokens=mtp, **kw)


def populate_prefix_cpu(history_cpu: np.ndarray, window_cpu: torch.Tensor, plan, layout, ks, vs, rk, rv, prefixes):
    """Write oracle-packed rotated history bytes and the BF16 window of every prefix."""
    cfg = layout.config
    for req, (k, v, p) in enumerate(zip(ks, vs, prefixes)):
        if p == 0:
            continue
        kr = (k[:p].float() @ rk.float()).bfloat16()
        vr = (v[:p].float() @ rv.float()).bfloat16()
        packed = oo.packed_slots(kr, vr, cfg).numpy()  # [p, H, 160]
        slots = plan.slots_of(req, range(p)).numpy()
        for h in range(layout.kv_heads):
            addr = oo.slot_addresses(slots, h, layout)
            idx = addr[:, None] + np.arange(136)[None, :]
            history_cpu[idx] = packed[:, h, :136]
        owner = int(plan.block_tables[req, 0]) // layout.blocks_per_page
        for t in range(p):
            idx = t if t < cfg.sink_tokens else cfg.sink_tokens + t % cfg.ring_tokens
            for h in range(layout.kv_heads):
                for kv, src in ((0, k), (1, v)):
                    off = owner * (layout.stripe_page_bytes // 2) + ((idx * 2 + kv) * layout.kv_heads + h) * 256
                    window_cpu[off : off + 256] = src[t, h]


class Scenario:
    """A batch of requests with full K/V sequences, a paged cache and step metadata."""

    def __init__(self, seq_lens, query_lens, hq, h, cfg, block_tokens=768, seed=0, device="cuda", fill="oracle",
                 rk=None, rv=None, max_reqs=None, data=None):
        self.cfg = cfg
        self.layout = CacheLayout(block_tokens, kv_heads=h, config=cfg)
        self.plan = plan_pages(seq_lens, query_lens, block_tokens, seed=seed, max_reqs=max_reqs)
        gen = torch.Generator().manual_seed(1000 + seed)
        self.hq, self.h = hq, h
        if data is None:
            self.ks = [oo_outlier(gen, s, h) for s in seq_lens]
            self.vs = [torch.randn(s, h, 256, generator=gen).bfloat16() for s in seq_lens]
            self.qs = [torch.randn(q, hq, 256, generator=gen).bfloat16() for q in query_lens]
        else:  # given per-request K/V [s, h, 256] and Q [q, hq, 256] (e.g. one rank's shard)
            self.ks, self.vs, self.qs = (list(x) for x in data)
        self.prefixes = [s - q for s, q in zip(seq_lens, query_lens)]
        from oscar_new_b200.synthetic import rotation

        self.rk = (rotation(1) if rk is None else rk).bfloat16()
        self.rv = (rotation(2) if rv is None else rv).bfloat16()
        self.cache = cache_stripes(self.plan.num_pages, block_tokens, h, device)
        self.history, self.window = self.layout.tensor_views(self.cache)
        if fill == "oracle":
            hist = self.history.cpu().numpy()
            win = self.window.cpu()
            populate_prefix_cpu(hist, win, self.plan, self.layout, self.ks, self.vs, self.rk, self.rv, self.prefixes)
            self.history.copy_(torch.from_numpy(hist))
            self.window.copy_(win)
        self.meta = self.plan.meta(device, cfg.queries_per_tile)
        self.device = device

    def current(self):
        q = torch.cat(self.qs).to(self.device)
        k = torch.cat([x[p:] for x, p in zip(self.ks, self.prefixes)]).to(self.device)
        v = torch.cat([x[p:] for x, p in zip(self.vs, self.prefixes)]).to(self.device)
        return q, k, v

    def expected(self):
        outs, lses = [], []
        for q, k, v, p in zip(self.qs, self.ks, self.vs, self.prefixes):
            o, l = oo.hybrid_reference(q, k, v, p, self.rk, self.rv, self.cfg, with_lse=True)
            outs.append(o)
            lses.append(l)
        return torch.cat(outs), torch.cat(lses)

    def prepare_tasks(self):
        m = self.meta
        kernels.prepare_tasks(m.query_start_loc, m.counts, m.tasks, m.task_count, m.max_num_reqs,
                              self.cfg.queries_per_tile)

    def run_step(self, splits, scale=1 / 16):
        q, k, v = self.current()
        self.prepare_tasks()
        qrot = kernels.rotate_store(k, v, self.rk.to(self.device), self.rv.to(self.device), self.history,
                                    self.meta.slot_mapping, self.meta.counts, self.layout, query=q)
        out = torch.empty((q.shape[0], self.hq * 256), dtype=torch.bfloat16, device=self.device)
        kernels.decode_attention(qrot, q, k, v, self.history, self.window, self.meta, self.layout, scale, splits,
                                 self.rv.to(self.device), out)
        return out.view(q.shape[0], self.hq, 256)


def oo_outlier(gen, n, h):
    x = torch.randn(n, h, 256, generator=gen)
    x[..., :8] *= 20
    return x.bfloat16()


def shard_scenario(sc, shard, seed=0):
    """The Scenario one rank of a KV head x request partition holds: its requests (in
    shard order) and its KV heads with their query heads, same rotations and config."""
    g = sc.hq // sc.h
    hb, he = shard.head_begin, shard.head_end
    reqs = list(shard.requests)
    data = ([sc.ks[r][:, hb:he].contiguous() for r in reqs], [sc.vs[r][:, hb:he].contiguous() for r in reqs],
            [sc.qs[r][:, hb * g:he * g].contiguous() for r in reqs])
    return Scenario([sc.plan.seq_lens[r] for r in reqs], [sc.plan.query_lens[r] for r in reqs], hq=(he - hb) * g,
                    h=he - hb, cfg=sc.cfg, block_tokens=sc.layout.physical_block_tokens, seed=seed,
                    device=sc.device, rk=sc.rk, rv=sc.rv, data=data)


def fill_prefixes_on_device(plan, layout, history, window, rk, rv, seed, chunk=16384):
    """Write every request's prefix (seeded bf16 K/V, K channels 0-7 x20, generated on
    the device chunk by chunk) with the product store kernels: INT2 history through
    rotate_store, the BF16 sink / ring window through store_windows.  For contexts too
    long to pack on the host; the store kernels' bytes equal the oracle's (store parity
    tests), and the oracle then reads the cache these calls wrote."""
    device = history.device
    gen = torch.Generator(device=device).manual_seed(seed)
    h = layout.kv_heads
    for req, (sq, ql) in enumerate(zip(plan.seq_lens, plan.query_lens)):
        prefix = sq - ql
        for s0 in range(0, prefix, chunk):
            n = min(chunk, prefix - s0)
            k = torch.randn(n, h, 256, device=device, generator=gen)
            k[..., :8] *= 20
            k = k.bfloat16()
            v = torch.randn(n, h, 256, device=device, generator=gen).bfloat16()
            slots = plan.slots_of(req, range(s0, s0 + n)).to(device)
            counts = torch.tensor([1, n], dtype=torch.int32, device=device)
            kernels.rotate_store(k, v, rk, rv, history, slots, counts, layout)
            m1 = plan.meta(device)
            m1.query_start_loc = torch.tensor([0, n], dtype=torch.int32, device=device)
            m1.seq_lens = torch.tensor([s0 + n], dtype=torch.int32, device=device)
            m1.block_tables = plan.block_tables[req: req + 1].to(device).contiguous()
            m1.counts = counts
            m1.max_num_reqs = 1
            kernels.store_windows(k, v, window, m1, layout)
