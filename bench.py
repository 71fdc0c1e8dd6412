"""Benchmark of the OSCAR INT2 decode-attention layer on B200.

Workload: one FULL attention layer, 24 query heads / 4 KV heads,
D=256, batch 64 requests per GPU with 32768 context tokens each (4 BF16 sink tokens,
128-token BF16 recent window, 1 current token, INT2 history for the rest), physical
pages of 768 tokens handed out by a seeded random permutation, 16 KV splits with LSE
merge.  A step is one layer forward of the drop-in path: task table, fused rotation +
INT2 store of the current K/V (+ Q rotation), paged split-KV history attention, BF16
sink/recent/current attention, split merge + inverse V rotation + path merge, window
store.  Synthetic seeded data (no dataset offline); the cache is filled by the same
store kernels.  Weak scaling: every rank owns its own 64 requests; ranks share nothing
on the data path (torch.distributed is used only for the barrier and max-over-ranks
timing).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from dataclasses import replace
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

B, H, G, D, SEQ, SINK, RECENT, SPLITS, BP = 64, 4, 6, 256, 32768, 4, 128, 16, 768
METRIC = "int2_decode_attention_kv_tokens_per_s"
UNIT = "KV tokens/s"
HISTORY_BYTES_PER_TOKEN_HEAD = 136  # packed K + V vectors of one (token, KV head)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def decode_config():
    """The decode workload both arms report (config 3)."""
    return {"workload": "config3 single-query paged INT2 decode attention layer (store + attention + merge)",
            "requests_per_gpu": B, "context": SEQ, "q_heads": H * G, "kv_heads": H, "head_dim": D,
            "sink": SINK, "recent": RECENT, "kv_splits": SPLITS, "page_tokens": BP}


def workload_sizes(requests=None, kv_heads=None):
    """Per-GPU sizes of a decode step of `requests` x `kv_heads` (default: config 3)."""
    nr = B if requests is None else requests
    h = H if kv_heads is None else kv_heads
    hist_tokens = SEQ - 1 - SINK - RECENT  # prefix minus sink and recent
    hist_bytes = nr * h * hist_tokens * HISTORY_BYTES_PER_TOKEN_HEAD
    window_bytes = nr * h * (SINK + RECENT) * 2 * D * 2
    current = nr * (h * G + 2 * h) * D * 2
    out = nr * h * G * D * 2
    return dict(
        kv_tokens=nr * SEQ * h,
        history_bytes=hist_bytes,
        footprint_bytes=nr * h * hist_tokens * 160,
        algorithmic_bytes=hist_bytes + window_bytes + current + out,
    )


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------


def build_state(device, seed, requests=None, kv_heads=None):
    """One GPU's share of the decode workload: `requests` x `kv_heads` (default config 3:
    64 x 4), 32768-token contexts whose prefixes are written by the device store kernels."""
    from oscar_new_b200 import kernels
    from oscar_new_b200.config import OscarConfig
    from oscar_new_b200.layout import CacheLayout
    from oscar_new_b200.synthetic import cache_stripes, plan_pages, rotation

    nr = B if requests is None else requests
    h = H if kv_heads is None else kv_heads
    cfg = replace(OscarConfig(), sink_tokens=SINK, recent_tokens=RECENT, speculative_tokens=0)
    layout = CacheLayout(BP, kv_heads=h, config=cfg)
    plan = plan_pages([SEQ] * nr, [1] * nr, BP, seed=seed)
    cache = cache_stripes(plan.num_pages, BP, h, device)
    history, window = layout.tensor_views(cache)
    rk = rotation(1).bfloat16().to(device)
    rv = rotation(2).bfloat16().to(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    prefix = SEQ - 1
    # fill every request's prefix with the device store kernels (history + window)
    for req in range(nr):
        k = torch.randn(prefix, h, D, device=device, generator=gen)
        k[..., :8] *= 20
        k = k.bfloat16()
        v = torch.randn(prefix, h, D, device=device, generator=gen).bfloat16()
        slots = plan.slots_of(req, range(prefix)).to(device)
        counts = torch.tensor([1, prefix], dtype=torch.int32, device=device)
        kernels.rotate_store(k, v, rk, rv, history, slots, counts, layout)
        meta1 = plan.meta(device)
        meta1.query_start_loc = torch.tensor([0, prefix], dtype=torch.int32, device=device)
        meta1.seq_lens = torch.tensor([prefix], dtype=torch.int32, device=device)
        meta1.block_tables = plan.block_tables[req : req + 1].to(device).contiguous()
        meta1.counts = counts
        meta1.max_num_reqs = 1
        kernels.store_windows(k, v, window, meta1, layout)
        del k, v
    meta = plan.meta(device, cfg.queries_per_tile)
    q = torch.randn(nr, h * G, D, device=device, generator=gen).bfloat16()
    k = torch.randn(nr, h, D, device=device, generator=gen)
    k[..., :8] *= 20
    k = k.bfloat16()
    v = torch.randn(nr, h, D, device=device, generator=gen).bfloat16()
    torch.cuda.synchronize(device)
    return dict(cfg=cfg, layout=layout, plan=plan, cache=cache, history=history, window=window, rk=rk, rv=rv,
                meta=meta, q=q, k=k, v=v, requests=nr, kv_heads=h)


def layer_step(st, out, scratch):
    """One layer forward through the kernel wrappers (used for spot parity and ncu runs;
    the timed legs go through OscarMetadataBuilder.build + OscarAttentionImpl.forward)."""
    from oscar_new_b200 import kernels

    m = st["meta"]
    kernels.prepare_tasks(m.query_start_loc, m.counts, m.tasks, m.task_count, m.max_num_reqs,
                          st["cfg"].queries_per_tile)
    qrot = kernels.rotate_store(st["k"], st["v"], st["rk"], st["rv"], st["history"], m.slot_mapping, m.counts,
                                st["layout"], query=st["q"])
    kernels.decode_attention(qrot, st["q"], st["k"], st["v"], st["history"], st["window"], m, st["layout"],
                             1.0 / math.sqrt(D), SPLITS, st["rv"], out, scratch)
    return qrot


LAYER = "model.layers.0.self_attn.attn"


def plugin_for(st, device, workdir):
    """What a vLLM worker holds for one OSCAR layer: the attention impl (rotations loaded
    from .pt files after "weight loading"), the metadata builder, and the step's common
    attention metadata (vLLM's per-step device tensors)."""
    from types import SimpleNamespace

    from oscar_new_b200.backend import OscarAttentionImpl
    from oscar_new_b200.metadata import OscarMetadataBuilder

    nr, h = st["requests"], st["kv_heads"]
    for name, rot in (("K", st["rk"]), ("V", st["rv"])):
        path = os.path.join(workdir, f"{name.lower()}_rotation.pt")
        torch.save({"layers": {0: {"rotation": rot.float().cpu()}}}, path)
        os.environ[f"VLLM_OSCAR_{name}_ROTATION_PATH"] = path
    os.environ["VLLM_OSCAR_SINK_TOKENS"] = str(SINK)
    os.environ["VLLM_OSCAR_RECENT_TOKENS"] = str(RECENT)
    vc = SimpleNamespace(
        cache_config=SimpleNamespace(enable_prefix_caching=False, cache_dtype="auto"),
        model_config=SimpleNamespace(dtype=torch.bfloat16, hf_text_config=SimpleNamespace(head_dim=D),
                                     max_model_len=SEQ),
        kv_transfer_config=None,
        parallel_config=SimpleNamespace(decode_context_parallel_size=1, prefill_context_parallel_size=1,
                                        enable_dbo=False),
        speculative_config=None,
        scheduler_config=SimpleNamespace(max_num_seqs=nr, max_num_batched_tokens=nr),
        compilation_config=SimpleNamespace(static_forward_context={}),
    )
    impl = OscarAttentionImpl(h * G, D, 1.0 / math.sqrt(D), num_kv_heads=h, vllm_config=vc)
    impl.initialize_layer(SimpleNamespace(layer_name=LAYER))
    builder = OscarMetadataBuilder(SimpleNamespace(block_size=BP, num_kv_heads=h), [LAYER], vc, device)
    if impl.cfg.sink_tokens != SINK or impl.cfg.recent_tokens != RECENT:
        raise RuntimeError("plugin configuration differs from the workload")
    m = st["meta"]
    cm = SimpleNamespace(query_start_loc=m.query_start_loc[: nr + 1].clone(), seq_lens=m.seq_lens[:nr].clone(),
                         block_table_tensor=m.block_tables[:nr].clone(), slot_mapping=m.slot_mapping[:nr].clone(),
                         num_reqs=nr, num_actual_tokens=nr, max_query_len=1, max_seq_len=SEQ, causal=True)
    return impl, builder, cm


def count_launches(fn, device):
    """Kernels of this library (namespace oscar) that one call of `fn` launches, from
    the CUDA profiler; None if the profiler is unavailable (e.g. under ncu)."""
    try:
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize(device)
        names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
        return sum(1 for nm in names if "oscar::" in nm)
    except Exception:  # noqa: BLE001 - a profiler clash must not end the bench
        return None


class ClockSampler:
    """nvidia-smi samples (every 20 ms) of this GPU's SM clock and throttle reasons;
    `mark()` brackets the timed region and `summary()` keeps the samples inside it.
    Every GPU is sampled and the rows are matched to this device by PCI bus id, since
    nvidia-smi's index need not equal the CUDA ordinal (CUDA_VISIBLE_DEVICES); the
    ordinal is the fallback when no row matches."""

    def __init__(self, device):
        device = torch.device(device)
        self.index = device.index if device.index is not None else torch.cuda.current_device()
        try:
            prop = torch.cuda.get_device_properties(self.index)
            self.bus = (prop.pci_domain_id, prop.pci_bus_id, prop.pci_device_id)
        except (RuntimeError, AttributeError, AssertionError):
            self.bus = None
        self.proc = None
        self.path = None
        self.window = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("timestamp,index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def mark(self, start, end):
        self.window = (start, end)

    def __exit__(self, *exc):
        time.sleep(0.05)
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        import datetime

        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        by_bus, by_index = [], []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 11:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                row = (ts, float(parts[3]), float(parts[4]),
                       {n for n, v in zip(names, parts[7:11]) if v.lower() == "active"})
                dom, bus, devfn = parts[2].split(":")
                if self.bus is not None and (int(dom, 16), int(bus, 16), int(devfn.split(".")[0], 16)) == self.bus:
                    by_bus.append(row)
                if int(parts[1]) == self.index:
                    by_index.append(row)
            except ValueError:
                continue
        os.unlink(self.path)
        samples = by_bus or by_index
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        inside = samples
        where = "timed region"
        if self.window is not None:
            lo, hi = self.window
            inside = [x for x in samples if lo <= x[0] <= hi]
            if not inside:  # region shorter than the sampling period: nearest samples
                inside = sorted(samples, key=lambda x: min(abs(x[0] - lo), abs(x[0] - hi)))[:2]
                where = "nearest to a timed region shorter than the 20 ms sampling period"
        reasons = sorted(set().union(*(x[3] for x in inside)))
        return {"sm_mhz": statistics.median(x[1] for x in inside), "sm_max_mhz": max(x[2] for x in samples),
                "reasons": reasons, "samples": len(inside), "window": where}


def traffic_per_launch(requests):
    """DRAM bytes per history-kernel launch: the committed ncu capture (a smaller batch,
    one launch), scaled to `requests` x the captured kv heads by the units processed."""
    p = ROOT / "profiles" / "history_attention_traffic.json"
    if not p.exists():
        return None, None
    d = json.loads(p.read_text())
    captured = d["dram_bytes_read_captured"] + d["dram_bytes_write_captured"]
    n = d["requests_captured"]
    return captured * requests / n, (f"not measured in this run: ncu capture of {n} requests x 4 KV heads "
                                     f"({captured} B), scaled by {requests}/{n} ({p.name})")


TARGET_REGION_S = 3.0  # each timed leg runs about this long, whatever --steps is
MIN_HEADS_PER_RANK = 2


def run_gpu(args):
    from oscar_new_b200 import _lib, kernels
    from oscar_new_b200.config import decode_split_cap
    from oscar_new_b200.partition import head_split, shard_of

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    _lib.lib()
    # One global batch of B * world config-3 requests, split by KV head (tensor parallel,
    # as the model shards its heads) down to 2 KV heads per rank, then by request: every
    # rank gets B * tp requests x H / tp KV heads, the per-GPU work of N = 1.  (On one
    # B200 a 128-request x 2-head shard runs a forward in 510 us like 64 x 4, a 256 x 1
    # shard in 557 us: the raw path and the merges grow with the requests.)
    tp = head_split(H, world, MIN_HEADS_PER_RANK)
    shard = shard_of(rank, [SEQ] * (B * world), H, world, MIN_HEADS_PER_RANK)
    st = build_state(device, seed=1234 + rank, requests=len(shard.requests), kv_heads=shard.kv_heads)
    nr, h = st["requests"], st["kv_heads"]
    sizes = workload_sizes(nr, h)
    workdir = tempfile.mkdtemp(prefix="oscar_bench_")
    impl, builder, cm = plugin_for(st, device, workdir)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / steps)

    out = torch.empty((nr, h * G * D), dtype=torch.bfloat16, device=device)
    q2, k2, v2 = (st[x].view(nr, -1) for x in ("q", "k", "v"))

    def forward(q, k, v, o, meta):
        impl.forward(None, q, k, v, st["cache"], meta, o)

    # ---- inner repeats: a step is one metadata build + R layer forwards, R chosen from
    # the warm-up so that every timed leg runs about TARGET_REGION_S seconds ----
    meta = builder.build(0, cm)
    for _ in range(args.warmup):
        forward(q2, k2, v2, out, meta)
    layer_ms = timed(lambda: forward(q2, k2, v2, out, meta), max(args.warmup, 3))
    repeats = max(1, math.ceil(TARGET_REGION_S * 1e3 / (args.steps * layer_ms)))
    repeats = int(max_over_ranks(repeats))

    def step():
        m = builder.build(0, cm)
        for _ in range(repeats):
            forward(q2, k2, v2, out, m)

    launches = count_launches(step, device)
    for _ in range(args.warmup):
        step()
    with ClockSampler(device) as clocks:
        t0 = time.time()
        step_ms = timed(step, args.steps)
        clocks.mark(t0, time.time())
    if not bool(torch.isfinite(out.float()).all()):
        raise RuntimeError("non-finite attention output")

    # ---- dominant kernel alone: history split-KV attention, CUDA events on its stream ----
    m = st["meta"]
    kernels.prepare_tasks(m.query_start_loc, m.counts, m.tasks, m.task_count, m.max_num_reqs,
                          st["cfg"].queries_per_tile)
    qrot = kernels.rotate(st["q"], st["rk"])

    def history():
        kernels.attention_partials(qrot, st["k"], st["v"], st["history"], st["window"], m, st["layout"],
                                   1.0 / math.sqrt(D), SPLITS, False)

    for _ in range(3):
        history()
    kern_ms = timed(history, max(5, math.ceil(TARGET_REGION_S * 1e3 / max(layer_ms, 1e-3))))

    # ---- end to end through the plugin with host buffers ----
    # Per step: vLLM's per-step metadata (query starts, sequence lengths, slot mapping)
    # goes host -> device and the builder stages it; per layer forward: that layer's
    # Q/K/V go host -> device and its output device -> host.  Two device input / output
    # sets: a copy stream moves call c+1's inputs in while call c computes, another
    # reads call c's output back.  The block table stays device-resident, as in the
    # runner (it changes only when a request gains a page).
    pin = {x: st[x].view(nr, -1).cpu().pin_memory() for x in ("q", "k", "v")}
    meta_pin = {x: getattr(cm, x).cpu().pin_memory() for x in ("query_start_loc", "seq_lens", "slot_mapping")}
    dev_in = [{x: torch.empty_like(t, device=device) for x, t in pin.items()} for _ in range(2)]
    dev_cm = []
    for _ in range(2):
        c2 = type(cm)(**vars(cm))
        for x, t in meta_pin.items():
            setattr(c2, x, torch.empty_like(t, device=device))
        dev_cm.append(c2)
    dev_out = [torch.empty_like(out) for _ in range(2)]
    host_out = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    layer_h2d = sum(t.numel() * t.element_size() for t in pin.values())
    step_h2d = sum(t.numel() * t.element_size() for t in meta_pin.values())
    layer_d2h = host_out[0].numel() * host_out[0].element_size()

    def upload(b, with_meta):
        with torch.cuda.stream(up):
            for x, t in pin.items():
                dev_in[b][x].copy_(t, non_blocking=True)
            if with_meta:
                for x, t in meta_pin.items():
                    getattr(dev_cm[b], x).copy_(t, non_blocking=True)
            h2d_done[b].record(up)

    def e2e_run(steps):
        calls = steps * repeats
        up.wait_stream(stream)
        down.wait_stream(stream)
        upload(0, True)
        meta_now = None
        for c in range(calls):
            b = c & 1
            stream.wait_event(h2d_done[b])
            if c >= 2:
                stream.wait_event(d2h_done[b])  # call c-2's output has been read back
            if c % repeats == 0:
                meta_now = builder.build(0, dev_cm[b])
            forward(dev_in[b]["q"], dev_in[b]["k"], dev_in[b]["v"], dev_out[b], meta_now)
            done[b].record(stream)
            if c + 1 < calls:
                if c >= 1:
                    up.wait_event(done[1 - b])  # call c-1, the other set's user, is done
                upload(1 - b, (c + 1) % repeats == 0)
            with torch.cuda.stream(down):
                down.wait_event(done[b])
                host_out[b].copy_(dev_out[b], non_blocking=True)
                d2h_done[b].record(down)
        stream.wait_stream(up)
        stream.wait_stream(down)

    e2e_run(max(1, args.warmup // repeats + 1))
    e2e_ms = timed(lambda: e2e_run(args.steps), 1) / args.steps
    torch.cuda.synchronize(device)
    last = host_out[(args.steps * repeats - 1) & 1].float()
    ref_out = out.float().cpu()
    e2e_rel = float((last - ref_out).norm() / ref_out.norm().clamp_min(1e-30))
    if not e2e_rel < 1e-3:
        raise RuntimeError(f"end-to-end output differs from the device-resident step (rel {e2e_rel})")

    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = sizes["history_bytes"] / (kern_ms * 1e-3) / 1e9
        traffic, traffic_note = traffic_per_launch(nr * h // H)
        kv_per_step = world * sizes["kv_tokens"] * repeats
        line = {
            "metric": METRIC,
            "value": kv_per_step / (step_ms * 1e-3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": step_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int2-kv/bf16",
            "data": "synthetic (seeded N(0,1) bf16, K channels 0-7 x20, random-permutation pages)",
            "config": {
                **decode_config(),
                "global_batch": B * world,
                "partition": f"KV heads tensor-parallel x{tp}, requests x{world // tp} (partition.py); "
                             f"{nr} requests x {h} KV heads per GPU, no data-path collective",
                "inner_repeats": repeats,
                "step": f"one metadata build + {repeats} layer forwards (OscarMetadataBuilder.build, "
                        f"OscarAttentionImpl.forward)",
                "kv_splits": f"balanced per request, at most "
                             f"{decode_split_cap(nr, h, 1, nr, h * G)} (forward's cap); roofline leg {SPLITS}",
                "l2": "inputs larger than L2 (packed history 1.14 GB per GPU)",
                "us_per_layer": step_ms * 1e3 / repeats,
                "hbm_gbs_algorithmic": sizes["algorithmic_bytes"] * repeats / (step_ms * 1e-3) / 1e9,
                "frac_of_8tbs_packed_history": sizes["history_bytes"] * repeats / (step_ms * 1e-3) / 8e12,
                "parallelism": f"weak x{world}",
            },
            "roofline": {
                "kernel": "history_attention_kernel",
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "peak_kind": f"{peak_kind} hbm copy GB/s",
                "unit": "GB/s",
                "frac": achieved / peak,
                "us_per_launch": kern_ms * 1e3,
                "algorithmic_bytes_per_launch": sizes["history_bytes"],
                "traffic": traffic,
                "traffic_source": traffic_note,
            },
            "e2e": {
                "value": kv_per_step / (e2e_ms * 1e-3),
                "unit": UNIT,
                "h2d_bytes_per_step": step_h2d + repeats * layer_h2d,
                "d2h_bytes_per_step": repeats * layer_d2h,
                "ms_per_step": e2e_ms,
                "path": "OscarMetadataBuilder.build + OscarAttentionImpl.forward with pinned host inputs/outputs",
                "rel_err_vs_device_step": e2e_rel,
                "pipelining": "call c+1's host->device inputs (one copy stream) and call c's device->host output "
                              "(another) overlap call c (two device input/output sets)",
            },
            "gpu_launches": None if launches is None else launches * args.steps,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            scratch = kernels.DecodeScratch(nr, h * G, SPLITS, device)
            line["cpu_baseline"] = cpu_baseline(st, scratch, budget_s=args.cpu_budget)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------
# CPU reference arm: the oracle port of the reference's algorithm on the host cores
# ----------------------------------------------------------------------------


def oracle_decode_sample(history, window, meta, layout, qrot, q, k, v, rv, requests):
    """Decode step of `requests` through the CPU oracle (history in the rotated space,
    raw BF16 path, merges, inverse rotation).  Inputs are host tensors."""
    from types import SimpleNamespace

    from oracle import int2_oracle as oo

    outs = []
    for req in requests:
        sub = SimpleNamespace(
            query_start_loc=torch.tensor([0, 1], dtype=torch.int32),
            seq_lens=meta.seq_lens[req : req + 1].clone(),
            block_tables=meta.block_tables[req : req + 1].clone(),
            counts=torch.tensor([1, 1], dtype=torch.int32),
        )
        out, _, _ = oo.decode_reference(qrot[req : req + 1], q[req : req + 1], k[req : req + 1], v[req : req + 1],
                                        history, window, sub, layout, 1.0 / math.sqrt(D), rv)
        outs.append(out)
    return torch.cat(outs)


def cpu_baseline(st, scratch, budget_s=20.0):
    torch.set_num_threads(os.cpu_count() or 1)
    from oscar_new_b200 import kernels

    hist = st["history"].cpu().numpy()
    win = st["window"].cpu()
    meta = st["meta"]
    mh = type("M", (), {})()
    mh.seq_lens = meta.seq_lens.cpu()
    mh.block_tables = meta.block_tables.cpu()
    qrot = kernels.rotate(st["q"], st["rk"]).cpu()
    q, k, v, rv = st["q"].cpu(), st["k"].cpu(), st["v"].cpu(), st["rv"].cpu()
    done = 0
    t0 = time.perf_counter()
    out = None
    while done < B and time.perf_counter() - t0 < budget_s:
        out = oracle_decode_sample(hist, win, mh, st["layout"], qrot, q, k, v, rv, [done])
        done += 1
    dt = time.perf_counter() - t0
    check = None
    if out is not None:
        # spot parity of the last sampled request against the GPU output
        gpu = torch.empty((B, H * G * D), dtype=torch.bfloat16, device=st["q"].device)
        layer_step(st, gpu, scratch)
        g = gpu.view(B, H * G, D)[done - 1].float().cpu()
        check = float((g - out[0]).norm() / out[0].norm())
    return {
        "value": done * SEQ * H / dt,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"{done} of {B} config-3 requests through the CPU oracle decode step ({dt:.1f} s)",
        "gpu_vs_oracle_rel_err": check,
    }


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    from oracle import int2_oracle as oo
    from oscar_new_b200.config import OscarConfig
    from oscar_new_b200.layout import CacheLayout
    from oscar_new_b200.synthetic import plan_pages, rotation

    cfg = replace(OscarConfig(), sink_tokens=SINK, recent_tokens=RECENT, speculative_tokens=0)
    layout = CacheLayout(BP, kv_heads=H, config=cfg)
    # one request of the config, built with the oracle's own packer on the host
    plan = plan_pages([SEQ], [1], BP, seed=7)
    pages = plan.num_pages
    hist = torch.full((pages * layout.stripe_page_bytes,), 0x5A, dtype=torch.uint8).numpy()
    win = torch.zeros(pages * layout.stripe_page_bytes // 2, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(7)
    rk, rv = rotation(1).bfloat16(), rotation(2).bfloat16()
    prefix = SEQ - 1
    chunk = 4096
    for s0 in range(0, prefix, chunk):
        n = min(chunk, prefix - s0)
        kk = torch.randn(n, H, D, generator=gen)
        kk[..., :8] *= 20
        kr = (kk.bfloat16().float() @ rk.float()).bfloat16()
        vr = (torch.randn(n, H, D, generator=gen).bfloat16().float() @ rv.float()).bfloat16()
        packed = oo.packed_slots(kr, vr, cfg).numpy()
        slots = plan.slots_of(0, range(s0, s0 + n)).numpy()
        for h in range(H):
            addr = oo.slot_addresses(slots, h, layout)
            hist[addr[:, None] + torch.arange(136).numpy()[None, :]] = packed[:, h, :136]
    q = torch.randn(1, H * G, D, generator=gen).bfloat16()
    k = torch.randn(1, H, D, generator=gen).bfloat16()
    v = torch.randn(1, H, D, generator=gen).bfloat16()
    qrot = (q.float() @ rk.float()).bfloat16()
    mh = type("M", (), {})()
    mh.seq_lens = torch.tensor([SEQ], dtype=torch.int32)
    mh.block_tables = plan.block_tables
    for _ in range(args.warmup):
        oracle_decode_sample(hist, win, mh, layout, qrot, q, k, v, rv, [0])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle_decode_sample(hist, win, mh, layout, qrot, q, k, v, rv, [0])
    dt = (time.perf_counter() - t0) / args.steps
    value = SEQ * H / dt
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int2-kv/fp32",
        "data": "synthetic (seeded, same generators as the GPU arm)",
        "config": {**decode_config(),
                   "sample": f"one of the {B} requests per step (bounded CPU sample): attention, merges and inverse "
                             f"rotation through the CPU oracle; the INT2 and window stores of the current token (1 "
                             f"of the request's {SEQ}) are not in it",
                   "parallelism": f"{torch.get_num_threads()} host threads, rank 0 only"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": "1 config-3 request (32768 tokens x 4 KV heads) per step through the CPU oracle"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# secondary workloads (configs 2, 4, 5): their own JSON lines, not the headline
# ----------------------------------------------------------------------------


def _flush_l2(buf):
    buf.add_(1)  # 256 MiB write: evicts the 126 MB L2 between timed iterations


def _timed_each(fn, steps, warmup, device, flush):
    """Sum of per-iteration CUDA-event durations on the launching stream, with an L2
    flush (outside the timed interval) before every iteration."""
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in events:
        _flush_l2(flush)
        e0.record(stream)
        fn()
        e1.record(stream)
    torch.cuda.synchronize(device)
    return sum(e0.elapsed_time(e1) for e0, e1 in events) / steps


def config2_state(device, seed=202):
    """Config 2: 16384 tokens x 4 heads, K channels 0-7 x20, distinct seeded slots in 22
    pages with every 64th slot -1, counts = [1, 16384], K/V clip .96/.92."""
    from oscar_new_b200.config import OscarConfig
    from oscar_new_b200.layout import CacheLayout
    from oscar_new_b200.synthetic import cache_stripes, rotation

    cfg = OscarConfig()
    n, pages = 16384, 22
    layout = CacheLayout(BP, kv_heads=H, config=cfg)
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn(n, H, D, generator=gen)
    k[..., :8] *= 20
    v = torch.randn(n, H, D, generator=gen)
    slots = torch.randperm(pages * BP, generator=gen)[:n].long()
    slots[::64] = -1
    cache = cache_stripes(pages, BP, H, device)
    history, _ = layout.tensor_views(cache)
    return dict(cfg=cfg, layout=layout, n=n, pages=pages, k=k.bfloat16().to(device), v=v.bfloat16().to(device),
                rk=rotation(1).bfloat16().to(device), rv=rotation(2).bfloat16().to(device), slots=slots.to(device),
                counts=torch.tensor([1, n], dtype=torch.int32, device=device), history=history)


def run_rotate_store(args):
    from oscar_new_b200 import _lib, kernels

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    _lib.lib()
    st = config2_state(device)
    n = st["n"]
    flush = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device=device)

    def step():
        kernels.rotate_store(st["k"], st["v"], st["rk"], st["rv"], st["history"], st["slots"], st["counts"],
                             st["layout"])

    with ClockSampler(device) as clocks:
        t0 = time.time()
        ms = _timed_each(step, args.steps, args.warmup, device, flush)
        clocks.mark(t0, time.time())
    live = int((st["slots"] >= 0).sum())
    read_bytes = 2 * n * H * D * 2 + n * 8 + 2 * D * D * 2
    write_bytes = 2 * live * H * 68
    alg = read_bytes + write_bytes
    flops = 2 * (2 * n * H * D * D)
    peak, peak_kind = measured_peaks()
    tflops_peak = _measured_tflops()
    # end to end: pinned host K/V/slots in, the packed K stripe of the 22 pages out
    pin = {name: st[name].cpu().pin_memory() for name in ("k", "v", "slots")}
    hist_host = torch.empty(st["history"].shape, dtype=torch.uint8).pin_memory()

    def e2e():
        for name, t in pin.items():
            st[name].copy_(t, non_blocking=True)
        step()
        hist_host.copy_(st["history"], non_blocking=True)

    e2e_ms = _timed_each(e2e, args.steps, args.warmup, device, flush)
    h2d = sum(t.numel() * t.element_size() for t in pin.values())
    achieved = alg / (ms * 1e-3) / 1e9
    line = {
        "metric": "int2_rotate_store_token_heads_per_s", "value": n * H / (ms * 1e-3), "unit": "token-heads/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16->int2", "data": "synthetic (seeded, config 2)",
        "config": {"workload": "config2 fused K/V rotation + clip + INT2 pack/scatter (tcgen05 + TMA tiles)",
                   "tokens": n, "kv_heads": H, "head_dim": D, "pages": st["pages"], "page_tokens": BP,
                   "l2": "flushed (256 MiB write) before every timed iteration",
                   "tensor_tflops": flops / (ms * 1e-3) / 1e12,
                   "tensor_frac_of_measured_bf16": (flops / (ms * 1e-3) / 1e12) / tflops_peak},
        "roofline": {"kernel": "rotate_tc_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
                     "peak_kind": f"{peak_kind} hbm copy GB/s", "unit": "GB/s", "frac": achieved / peak,
                     "us_per_launch": ms * 1e3, "algorithmic_bytes_per_launch": alg, "traffic": None},
        "e2e": {"value": n * H / (e2e_ms * 1e-3), "unit": "token-heads/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": hist_host.numel(), "ms_per_step": e2e_ms},
        "gpu_launches": args.steps, "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def config4_contexts(seed=404):
    """The 32 context lengths of config 4: exp(U(ln 2048, ln 262144)), seeded."""
    gen = torch.Generator().manual_seed(seed)
    u = torch.rand(32, generator=gen, dtype=torch.float64)
    return [int(math.exp(math.log(2048) + x * (math.log(262144) - math.log(2048)))) for x in u.tolist()]


def config4_state(device, seed=404, nreq=32, requests=None, kv_heads=None):
    """Config 4 (MTP verify): 32 requests with qlen 4 (1 + 3 draft tokens) and seq_len
    ~ exp(U(ln 2048, ln 262144)) seeded; S=4, R=128, MTP=3; the sixth request's last
    draft has a padded -1 slot and a zero-length padded row closes the batch.  ``nreq``
    < 32 keeps the first requests only (small ncu captures); ``requests`` / ``kv_heads``
    build one rank's shard (its requests, its number of KV heads)."""
    from oscar_new_b200 import kernels
    from oscar_new_b200.config import OscarConfig
    from oscar_new_b200.layout import CacheLayout
    from oscar_new_b200.synthetic import cache_stripes, plan_pages, rotation

    all_seqs = config4_contexts(seed)
    chosen = list(range(nreq)) if requests is None else list(requests)
    seqs = [all_seqs[r] for r in chosen]
    nreq = len(seqs)
    h = H if kv_heads is None else kv_heads
    seqs.append(0)
    qlens = [4] * nreq + [0]
    cfg = replace(OscarConfig(), sink_tokens=SINK, recent_tokens=RECENT, speculative_tokens=3)
    layout = CacheLayout(BP, kv_heads=h, config=cfg)
    plan = plan_pages(seqs, qlens, BP, seed=seed, max_reqs=nreq + 2)
    cache = cache_stripes(plan.num_pages, BP, h, device)
    history, window = layout.tensor_views(cache)
    rk, rv = rotation(1).bfloat16().to(device), rotation(2).bfloat16().to(device)
    dgen = torch.Generator(device=device).manual_seed(seed)
    chunk = 16384
    for req, (sq, ql) in enumerate(zip(seqs, qlens)):
        prefix = sq - ql
        for s0 in range(0, prefix, chunk):
            n = min(chunk, prefix - s0)
            k = torch.randn(n, h, D, device=device, generator=dgen)
            k[..., :8] *= 20
            k = k.bfloat16()
            v = torch.randn(n, h, D, device=device, generator=dgen).bfloat16()
            slots = plan.slots_of(req, range(s0, s0 + n)).to(device)
            counts = torch.tensor([1, n], dtype=torch.int32, device=device)
            kernels.rotate_store(k, v, rk, rv, history, slots, counts, layout)
            m1 = plan.meta(device)
            m1.query_start_loc = torch.tensor([0, n], dtype=torch.int32, device=device)
            m1.seq_lens = torch.tensor([s0 + n], dtype=torch.int32, device=device)
            m1.block_tables = plan.block_tables[req : req + 1].to(device).contiguous()
            m1.counts = counts
            m1.max_num_reqs = 1
            kernels.store_windows(k, v, window, m1, layout)
    meta = plan.meta(device, cfg.queries_per_tile)
    if nreq > 5:
        meta.slot_mapping[5 * 4 + 3] = -1
    t = sum(qlens)
    q = torch.randn(t, h * G, D, device=device, generator=dgen).bfloat16()
    k = torch.randn(t, h, D, device=device, generator=dgen)
    k[..., :8] *= 20
    v = torch.randn(t, h, D, device=device, generator=dgen).bfloat16()
    torch.cuda.synchronize(device)
    hist_heads = 0
    for sq, ql in zip(seqs, qlens):
        prefix = sq - ql
        sink_len = min(SINK, prefix)
        hist_heads += h * max(0, max(sink_len, prefix - RECENT) - sink_len)
    return dict(cfg=cfg, layout=layout, plan=plan, cache=cache, history=history, window=window, rk=rk, rv=rv,
                meta=meta, q=q, k=k.bfloat16(), v=v, seqs=seqs, qlens=qlens, hist_token_heads=hist_heads, kv_heads=h,
                requests=nreq)


def run_mtp_verify(args):
    """Config 4 on N GPUs: the fixed batch of 32 requests split by KV head (at least 2 per
    rank) and by request, balanced by total context (partition.py); strong scaling."""
    from oscar_new_b200 import _lib, kernels
    from oscar_new_b200.config import decode_split_cap
    from oscar_new_b200.partition import head_split, shard_of

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    _lib.lib()
    contexts = config4_contexts()
    tp = head_split(H, world, MIN_HEADS_PER_RANK)
    shard = shard_of(rank, contexts, H, world, MIN_HEADS_PER_RANK)
    st = config4_state(device, requests=shard.requests, kv_heads=shard.kv_heads)
    h, nr = st["kv_heads"], st["requests"]
    m = st["meta"]
    t = st["q"].shape[0]
    splits = decode_split_cap(nr, h, 4, t, h * G)
    out = torch.empty((t, h * G * D), dtype=torch.bfloat16, device=device)
    scratch = kernels.DecodeScratch(t, h * G, splits, device)
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)

    def max_over_ranks(x):
        if dist is None:
            return x
        v = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return float(v.item())

    def step():
        kernels.prepare_tasks(m.query_start_loc, m.counts, m.tasks, m.task_count, m.max_num_reqs,
                              st["cfg"].queries_per_tile)
        qrot = kernels.rotate_store(st["k"], st["v"], st["rk"], st["rv"], st["history"], m.slot_mapping, m.counts,
                                    st["layout"], query=st["q"])
        kernels.decode_attention(qrot, st["q"], st["k"], st["v"], st["history"], st["window"], m, st["layout"],
                                 scale, splits, st["rv"], out, scratch)

    def timed(fn, steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / steps)

    for _ in range(args.warmup):
        step()
    with ClockSampler(device) as clocks:
        t0 = time.time()
        ms = timed(step, args.steps)
        clocks.mark(t0, time.time())
    qrot = kernels.rotate(st["q"], st["rk"])

    def history():
        kernels.attention_partials(qrot, st["k"], st["v"], st["history"], st["window"], m, st["layout"], scale,
                                   splits, False)

    for _ in range(3):
        history()
    kern_ms = timed(history, args.steps)
    hist_bytes = st["hist_token_heads"] * HISTORY_BYTES_PER_TOKEN_HEAD
    total_kv = sum(contexts) * H
    own_ctx = sum(contexts[r] for r in shard.requests)
    ctx_max = max_over_ranks(float(own_ctx * shard.kv_heads))
    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = hist_bytes / (kern_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": total_kv / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int2-kv/bf16", "data": "synthetic (seeded, config 4)",
            "config": {"workload": "config4 MTP verify (qlen 4) paged INT2 decode attention layer",
                       "requests": 32, "padded_rows": 1, "sum_seq_len": sum(contexts),
                       "partition": f"KV heads tensor-parallel x{tp}, requests x{world // tp} balanced by context "
                                    f"(partition.py); rank 0: {nr} requests x {h} KV heads",
                       "kv_heads_x_context_max_over_ranks_vs_mean": ctx_max / (total_kv / world),
                       "kv_splits": f"balanced per request, at most {splits}",
                       "history_token_heads_rank0": st["hist_token_heads"], "l2": "inputs larger than L2",
                       "us_per_layer": ms * 1e3},
            "roofline": {"kernel": "history_mtp_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
                         "peak_kind": f"{peak_kind} hbm copy GB/s", "unit": "GB/s", "frac": achieved / peak,
                         "us_per_launch": kern_ms * 1e3, "algorithmic_bytes_per_launch": hist_bytes,
                         "traffic": None, "traffic_source": "not measured in this run (see profiles/)"},
            "gpu_launches": 6 * args.steps, "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    del scratch
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_calibration(args):
    """Config 5: 16 layers x 4 KV heads (6 query heads each), 16 segments x 1024 tokens,
    channels 0-7 = 20 * Student-t(3); both passes, the covariance all-reduce and the
    rank-0 eigensolve + publication.  Segments are sharded over ranks (strong scaling:
    the job is fixed); one NCCL all-reduce in second_pass and one in finish."""
    from oscar_new_b200 import _lib
    from oscar_new_b200 import calibration_kernels as ck
    from oscar_new_b200.calibration_worker import CalibrationSession

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        group = dist.group.WORLD
    _lib.lib()
    layers, segments, tokens = 16, 16, 1024
    gen = torch.Generator(device=device).manual_seed(505)

    def student(shape):
        chi2 = torch.randn(*shape, 3, device=device, generator=gen).square().sum(-1)
        return 20 * torch.randn(*shape, device=device, generator=gen) / (chi2 / 3).sqrt()

    data = {}
    for layer in range(layers):
        for seg in range(segments):
            if seg % world != rank:
                continue
            q = torch.randn(tokens, H * G, D, device=device, generator=gen)
            k = torch.randn(tokens, H, D, device=device, generator=gen)
            v = torch.randn(tokens, H, D, device=device, generator=gen)
            for x in (q, k, v):
                x[..., :8] = student(x[..., :8].shape)
            data[(layer, seg)] = (q.bfloat16(), k.bfloat16(), v.bfloat16())
    outdir = tempfile.mkdtemp(prefix="oscar_calib_")

    def job():
        s = CalibrationSession(range(layers), 10**9, device, H, G, shard="tokens", group=group)
        for phase in (1, 2):
            for (layer, _), (q, k, v) in data.items():
                s.observe(layer, q.view(tokens, -1), k.view(tokens, -1), v.view(tokens, -1), tokens)
            if phase == 1:
                s.second_pass()
        return s.finish(outdir, {"model_fingerprint": "synthetic-config5"}, 12)

    for _ in range(1):
        job()  # warm-up (first-call setup)
    torch.cuda.synchronize(device)
    times, info = [], None
    steps = max(1, min(args.steps, 5))
    for _ in range(steps):
        if group is not None:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        info = job()
        torch.cuda.synchronize(device)
        times.append(time.perf_counter() - t0)
    job_s = statistics.median(times)
    if group is not None:
        t = torch.tensor([job_s], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        job_s = float(t.item())
    # component timings on this rank: Gram over one (layer, segment) and the eigensolve
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    q0 = next(iter(data.values()))[0]
    cov = torch.zeros((D, D), dtype=torch.float32, device=device)
    for _ in range(3):
        ck.accumulate_gram(q0[:, :G], cov)
    e0.record(stream)
    for _ in range(20):
        ck.accumulate_gram(q0[:, :G], cov)
    e1.record(stream)
    torch.cuda.synchronize(device)
    gram_ms = e0.elapsed_time(e1) / 20
    gram_tflops = 2 * tokens * G * D * D / (gram_ms * 1e-3) / 1e12
    stack = torch.randn(2 * layers, D, D, device=device)
    stack = stack @ stack.transpose(-1, -2) / D
    e0.record(stream)
    _, _, einfo = ck.calibrated_rotations(stack)
    e1.record(stream)
    torch.cuda.synchronize(device)
    eig_ms = e0.elapsed_time(e1)
    if rank == 0:
        line = {
            "metric": "calibration_job_seconds", "value": job_s, "unit": "s", "n_gpus": world, "steps": steps,
            "warmup": 1, "ms_per_step": job_s * 1e3, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16->fp32 (Gram), fp64 (Jacobi)", "data": "synthetic (seeded, config 5)",
            "config": {"workload": "config5 calibration: 16 layers x 16 segments x 1024 tokens, both passes, "
                                   "NCCL all-reduce, device Jacobi + U H P_br, checkpoint write",
                       "layers": layers, "segments": segments, "tokens_per_segment": tokens, "kv_heads": H,
                       "q_heads_per_kv": G, "shard": "tokens (segments round-robin over ranks)",
                       "sweeps": info["sweeps"], "relative_off_diagonal": info["relative_off_diagonal"],
                       "gram_us_per_1024x6_rows": gram_ms * 1e3, "gram_tflops": gram_tflops,
                       "gram_frac_of_measured_bf16": gram_tflops / _measured_tflops(),
                       "eigensolve_32_matrices_ms": eig_ms, "eigensolve_sweeps": einfo["sweeps"]},
            "gpu_launches": None,
        }
        print(json.dumps(line), flush=True)
    if group is not None:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def _measured_tflops(kind="bf16_tflops"):
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if kind in d:
            return float(d[kind])
    return 1590.0


def set_requests(n):
    global B
    B = int(n)


def profile_only(what):
    """Small, self-ending workload for ncu captures (no timing, no JSON)."""
    from oscar_new_b200 import kernels

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    if what == "calibration":
        from oscar_new_b200.calibration_worker import CalibrationSession

        gen = torch.Generator(device=device).manual_seed(505)
        layers, segments, tokens = 4, 4, 1024
        data = {}
        for layer in range(layers):
            for seg in range(segments):
                q = torch.randn(tokens, H * G, D, device=device, generator=gen)
                k = torch.randn(tokens, H, D, device=device, generator=gen)
                v = torch.randn(tokens, H, D, device=device, generator=gen)
                for x in (q, k, v):
                    x[..., :8] *= 20
                data[(layer, seg)] = (q.bfloat16(), k.bfloat16(), v.bfloat16())
        s = CalibrationSession(range(layers), 10**9, device, H, G, shard="tokens", group=None)
        for phase in (1, 2):
            for (layer, _), (q, k, v) in data.items():
                s.observe(layer, q.view(tokens, -1), k.view(tokens, -1), v.view(tokens, -1), tokens)
            if phase == 1:
                s.second_pass()
        s.finish(tempfile.mkdtemp(prefix="oscar_calib_"), {"model_fingerprint": "profile"}, 12)
        torch.cuda.synchronize(device)
        print("profile run done: calibration job (4 layers x 4 segments x 1024 tokens)")
        return
    if what == "mtp-verify":
        from oscar_new_b200.config import decode_split_cap

        st = config4_state(device, nreq=8)
        m = st["meta"]
        t = st["q"].shape[0]
        splits = decode_split_cap(32, H, 4, t, H * G)
        kernels.prepare_tasks(m.query_start_loc, m.counts, m.tasks, m.task_count, m.max_num_reqs,
                              st["cfg"].queries_per_tile)
        qrot = kernels.rotate(st["q"], st["rk"])
        for _ in range(4):
            kernels.attention_partials(qrot, st["k"], st["v"], st["history"], st["window"], m, st["layout"],
                                       1.0 / math.sqrt(D), splits, False)
        torch.cuda.synchronize(device)
        print("profile run done: config 4 (8 requests) history")
        return
    if what == "prefill":
        # first prefill of one 8192-token request, 24 query / 4 KV heads (tcgen05 kernel)
        gen = torch.Generator(device=device).manual_seed(8)
        n = 8192
        q = torch.randn(n, H * G, D, device=device, generator=gen).bfloat16()
        k = torch.randn(n, H, D, device=device, generator=gen).bfloat16()
        v = torch.randn(n, H, D, device=device, generator=gen).bfloat16()
        starts = torch.tensor([0, n], dtype=torch.int32, device=device)
        for _ in range(4):
            kernels.prefill_attention(q, k, v, starts, 1, n, 1.0 / math.sqrt(D))
        torch.cuda.synchronize(device)
        print("profile run done: prefill 8192 tokens")
        return
    if what == "rotate-store":
        cs = config2_state(device)
        for _ in range(4):
            kernels.rotate_store(cs["k"], cs["v"], cs["rk"], cs["rv"], cs["history"], cs["slots"], cs["counts"],
                                 cs["layout"])
        torch.cuda.synchronize(device)
        print("profile run done: config 2 rotate-store")
        return
    st = build_state(device, seed=1234)
    m = st["meta"]
    out = torch.empty((B, H * G * D), dtype=torch.bfloat16, device=device)
    if what == "forward":
        # the timed decode step: one metadata build + one layer forward, four times
        impl, builder, cm = plugin_for(st, device, tempfile.mkdtemp(prefix="oscar_prof_"))
        q2, k2, v2 = (st[x].view(B, -1) for x in ("q", "k", "v"))
        for _ in range(4):
            impl.forward(None, q2, k2, v2, st["cache"], builder.build(0, cm), out)
        torch.cuda.synchronize(device)
        print("profile run done", B, "requests, build + forward")
        return
    scratch = kernels.DecodeScratch(B, H * G, SPLITS, device)
    kernels.prepare_tasks(m.query_start_loc, m.counts, m.tasks, m.task_count, m.max_num_reqs,
                          st["cfg"].queries_per_tile)
    qrot = kernels.rotate(st["q"], st["rk"])
    for _ in range(4):
        if what == "history":
            kernels.attention_partials(qrot, st["k"], st["v"], st["history"], st["window"], m, st["layout"],
                                       1.0 / math.sqrt(D), SPLITS, False)
        else:
            layer_step(st, out, scratch)
    torch.cuda.synchronize(device)
    print("profile run done", B, "requests", what)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="oscar", choices=["oscar", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--requests", type=int, default=B, help="requests per GPU (profiling runs use fewer)")
    ap.add_argument("--profile-kernel", choices=["history", "step", "forward", "prefill", "rotate-store",
                                                 "mtp-verify", "calibration"],
                    default=None,
                    help="build the state, run 4 launches of the kernel (or 4 layer steps) and exit")
    ap.add_argument("--workload", choices=["decode", "rotate-store", "mtp-verify", "calibration"], default="decode",
                    help="decode: config 3 (the headline); rotate-store: config 2; mtp-verify: config 4; "
                         "calibration: config 5")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    set_requests(args.requests)
    if args.profile_kernel:
        profile_only(args.profile_kernel)
        return
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "rotate-store":
        run_rotate_store(args)
    elif args.workload == "mtp-verify":
        run_mtp_verify(args)
    elif args.workload == "calibration":
        run_calibration(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
