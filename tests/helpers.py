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
                 rk=None, rv=None, max_reqs=None):
        self.cfg = cfg
        self.layout = CacheLayout(block_tokens, kv_heads=h, config=cfg)
        self.plan = plan_pages(seq_lens, query_lens, block_tokens, seed=seed, max_reqs=max_reqs)
        gen = torch.Generator().manual_seed(1000 + seed)
        self.hq, self.h = hq, h
        self.ks = [oo_outlier(gen, s, h) for s in seq_lens]
        self.vs = [torch.randn(s, h, 256, generator=gen).bfloat16() for s in seq_lens]
        self.qs = [torch.randn(q, hq, 256, generator=gen).bfloat16() for q in query_lens]
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
