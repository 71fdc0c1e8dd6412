"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout exists (read-only):

    python tests/golden/make_golden.py --reference /path/to/Oscar_new

It imports the reference's own ``tests/oracle.py`` (``quantize``, ``packed_slots``,
``hybrid_reference``), ``oscar_ascend/config.py`` and ``tests/test_calibration_math.py``
(``jacobi_oracle``, ``hadamard``, ``pbr``), and executes the reference's Triton kernel
bodies ``_prepare_tasks_kernel``, ``_attention_kernel`` and ``_load_vec`` on CPU with a
torch-backed ``tl`` namespace -- the same technique as the reference's
``tests/test_attention_empty_tasks.py:34-169`` and ``tests/test_packed_load.py:43-88``.
Outputs are small ``.pt`` files next to this script.  Nothing at test time reads the
reference; the fixtures carry inputs and expected outputs.
"""

from __future__ import annotations

import argparse
import ast
import math
import sys
from dataclasses import replace
from pathlib import Path
from types import SimpleNamespace

import torch

HERE = Path(__file__).resolve().parent


def outlier_bf16(gen, *shape, scale_channels=8, factor=20.0):
    x = torch.randn(*shape, generator=gen)
    x[..., :scale_channels] *= factor
    return x.bfloat16()


def orth(seed, dim=256):
    gen = torch.Generator().manual_seed(seed)
    q, r = torch.linalg.qr(torch.randn(dim, dim, generator=gen))
    return q * torch.sign(torch.diagonal(r))[None, :]


def hadamard_n(dim):
    h = torch.ones(1, 1)
    while h.shape[0] < dim:
        h = torch.cat((torch.cat((h, h), 1), torch.cat((h, -h), 1)), 0)
    return h / math.sqrt(dim)


class Bitcast(ast.NodeTransformer):
    """Rewrite ``x.to(dtype, bitcast=True)`` into ``bitcast(x, dtype)`` (as the reference test)."""

    def visit_Call(self, node):
        self.generic_visit(node)
        if (
            isinstance(node.func, ast.Attribute)
            and node.func.attr == "to"
            and any(kw.arg == "bitcast" and ast.literal_eval(kw.value) for kw in node.keywords)
        ):
            return ast.copy_location(
                ast.Call(func=ast.Name(id="bitcast", ctx=ast.Load()), args=[node.func.value] + node.args, keywords=[]),
                node,
            )
        return node


def load_kernel_bodies(ref: Path, names):
    tree = ast.parse((ref / "oscar_ascend/kernels.py").read_text())
    fns = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            node.decorator_list = []
            for arg in node.args.args:
                arg.annotation = None
            fns.append(Bitcast().visit(node))
    return ast.fix_missing_locations(ast.Module(body=fns, type_ignores=[]))


def tl_namespace(Pointer):
    def load(ptr, mask=True, other=0):
        offsets, mask, indices = ptr.indices(mask)
        result = torch.full(offsets.shape, other, dtype=ptr.data.dtype)
        result[mask] = ptr.data[indices]
        return result

    def store(ptr, value, mask=True):
        offsets, mask, indices = ptr.indices(mask)
        ptr.data[indices] = torch.broadcast_to(torch.as_tensor(value), offsets.shape)[mask].to(ptr.data.dtype)

    def as_t(x):
        return torch.as_tensor(x)

    return SimpleNamespace(
        load=load,
        store=store,
        dot=lambda a, b: a.float() @ b.float(),
        program_id=None,
        arange=torch.arange,
        minimum=lambda a, b: torch.minimum(as_t(a), as_t(b)),
        maximum=lambda a, b: torch.maximum(as_t(a), as_t(b)),
        cdiv=lambda a, b: (a + b - 1) // b,
        sum=torch.sum,
        where=lambda c, a, b: torch.where(as_t(c), as_t(a), as_t(b)),
        full=lambda shape, value, dtype: torch.full(shape, value, dtype=dtype),
        max=lambda x, axis: x.max(dim=axis).values,
        trans=lambda x: x.T,
        exp=torch.exp,
        log=torch.log,
        int32=torch.int32,
        int64=torch.int64,
        uint16=torch.int32,
        float16=torch.float16,
        float32=torch.float32,
        bfloat16=torch.bfloat16,
    )


def run_reference_attention(ref, Pointer, inputs, geometry, splits, raw):
    """Execute the reference ``_attention_kernel`` body for every program on CPU."""
    module = load_kernel_bodies(ref, {"_attention_kernel", "_load_vec"})
    tl = tl_namespace(Pointer)
    pid = [0, 0, 0]
    tl.program_id = lambda axis: torch.tensor(pid[axis], dtype=torch.int32)
    ns = {"tl": tl, "bitcast": lambda x, dtype: x.to(torch.uint16).contiguous().view(dtype)}
    exec(compile(module, "reference_attention_body", "exec"), ns)
    q = inputs["Query"]
    n, hq, d = q.shape
    partials = torch.full((n, hq, splits, d), float("nan"))
    lse = torch.full((n, hq, splits), float("nan"))
    accesses = []
    ptrs = {k: Pointer(v, k, accesses) for k, v in inputs.items()}
    ptrs["Partials"] = Pointer(partials, "Partials", accesses)
    ptrs["LSE"] = Pointer(lse, "LSE", accesses)
    k, v = inputs["CurrentK"], inputs["CurrentV"]
    for task in range(geometry["programs"]):
        for head in range(geometry["H"]):
            for split in range(splits):
                pid[:] = [task, head, split]
                ns["_attention_kernel"](
                    **ptrs,
                    H=geometry["H"],
                    G=geometry["G"],
                    D=256,
                    QT=geometry["QT"],
                    BM=max(16, 1 << (geometry["QT"] * geometry["G"] - 1).bit_length()),
                    BN=32,
                    BK=128,
                    BP=geometry["BP"],
                    PAGE_BYTES=geometry["PAGE_BYTES"],
                    SLOT=160,
                    VECTOR=68,
                    TABLE_STRIDE=inputs["Table"].stride(0),
                    SINK=geometry["SINK"],
                    RECENT=geometry["RECENT"],
                    RING=geometry["RING"],
                    QS0=q.stride(0),
                    QS1=q.stride(1),
                    QS2=q.stride(2),
                    KS0=k.stride(0),
                    KS1=k.stride(1),
                    KS2=k.stride(2),
                    VS0=v.stride(0),
                    VS1=v.stride(1),
                    VS2=v.stride(2),
                    SPLITS=splits,
                    SCALE=1 / 16,
                    RAW=raw,
                )
    return partials, lse


def run_reference_tasks(ref, Pointer, qstarts, counts, capacity, max_reqs, query_tile, num_reqs):
    module = load_kernel_bodies(ref, {"_prepare_tasks_kernel"})
    tl = tl_namespace(Pointer)
    pid = [0]
    tl.program_id = lambda axis: torch.tensor(pid[0], dtype=torch.int32)
    ns = {"tl": tl}
    exec(compile(module, "reference_tasks_body", "exec"), ns)
    tasks = torch.full((capacity, 2), -1, dtype=torch.int32)
    total = torch.full((1,), -1, dtype=torch.int32)
    acc = []
    for pid[0] in range(max(1, num_reqs)):
        ns["_prepare_tasks_kernel"](
            Pointer(qstarts, "qstarts", acc),
            Pointer(counts, "counts", acc),
            Pointer(tasks, "tasks", acc),
            Pointer(total, "task_count", acc),
            query_tile,
            1 << (max_reqs - 1).bit_length(),
        )
    return tasks, int(total.item())


def zpack(t):
    """Losslessly compress a (mostly sentinel-filled) CPU tensor for the fixture."""
    import zlib

    raw = t.contiguous().view(torch.uint8).numpy().tobytes()
    return dict(dtype=str(t.dtype).replace("torch.", ""), shape=tuple(t.shape), z=zlib.compress(raw, 9))


def build_paged_case(cfg_mod, oracle, lengths, prefixes, hq, h, sink, recent, mtp, seed, bp=256):
    """A small paged cache built with the reference oracle's own packed bytes."""
    cfg = replace(cfg_mod.OscarConfig(), sink_tokens=sink, recent_tokens=recent, speculative_tokens=mtp)
    gen = torch.Generator().manual_seed(seed)
    rk = (orth(seed + 1) @ hadamard_n(256)).bfloat16()
    rv = (orth(seed + 2) @ hadamard_n(256)).bfloat16()
    pages = sum(-(-n // bp) for n in lengths) + 2
    page_elems = bp * h * 256
    hist = torch.full((pages * page_elems * 2,), 0x5A, dtype=torch.uint8)
    window = torch.full((pages * page_elems,), 0, dtype=torch.bfloat16)
    per_page = bp // 128
    avail = list(range(1, pages))
    avail = avail[::2] + avail[1::2]
    cols = pages * per_page
    table = torch.zeros((len(lengths) + 1, cols), dtype=torch.int32)
    ks, vs, qs = [], [], []
    qstarts = [0]
    slots = []
    ring = sink + recent + mtp + 1 - sink  # recent + mtp + 1
    for i, (n, p) in enumerate(zip(lengths, prefixes)):
        need = -(-n // bp)
        own, avail = avail[:need], avail[need:]
        blocks = [pg * per_page + j for pg in own for j in range(per_page)]
        table[i, : len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
        k = outlier_bf16(gen, n, h, 256)
        v = torch.randn(n, h, 256, generator=gen).bfloat16()
        q = torch.randn(n - p, hq, 256, generator=gen).bfloat16()
        ks.append(k), vs.append(v), qs.append(q)
        kr = (k.float() @ rk.float()).bfloat16()
        vr = (v.float() @ rv.float()).bfloat16()
        packed = oracle.packed_slots(kr[:p], vr[:p], cfg)  # [p, h, 160]
        for t in range(p):
            slot = blocks[t // 128] * 128 + t % 128
            for hh in range(h):
                off = (slot // bp) * page_elems * 2 + ((slot % bp) * h + hh) * 160
                hist[off : off + 136] = packed[t, hh, :136]
            # window: sink + ring entries of the prefix (latest writer per ring slot)
            idx = t if t < sink else sink + t % ring
            owner = blocks[0] // per_page
            for hh in range(h):
                base = owner * page_elems + ((idx * 2) * h + hh) * 256
                window[base : base + 256] = k[t, hh]
                base = owner * page_elems + ((idx * 2 + 1) * h + hh) * 256
                window[base : base + 256] = v[t, hh]
        slots.extend(blocks[t // 128] * 128 + t % 128 for t in range(p, n))
        qstarts.append(qstarts[-1] + n - p)
    meta = dict(
        query_start_loc=torch.tensor(qstarts + [qstarts[-1]], dtype=torch.int32),
        seq_lens=torch.tensor(list(lengths) + [0], dtype=torch.int32),
        block_tables=table,
        counts=torch.tensor([len(lengths), qstarts[-1]], dtype=torch.int32),
        slot_mapping=torch.tensor(slots, dtype=torch.int64),
    )
    return cfg, rk, rv, ks, vs, qs, hist, window, meta, bp


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout (read-only)")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref))
    from oscar_ascend import config as cfg_mod  # noqa: E402
    from tests import oracle  # noqa: E402
    from tests.test_attention_empty_tasks import Pointer  # noqa: E402
    from tests.test_calibration_math import hadamard, jacobi_oracle, pbr  # noqa: E402

    gen = torch.Generator().manual_seed(20261201)

    # 1. quantize at every accepted clip setting, incl. constant / tiny / tie rows
    x = outlier_bf16(gen, 40, 2, 256)
    x[0, 0].zero_()
    x[1, 0].fill_(0.5)
    x[2, 0].fill_(1e-12)
    x[3, 0].fill_(-3)
    x[4, 0] = (torch.arange(256).float().remainder(11) - 5).bfloat16()
    x[5, 1] = torch.randn(256, generator=gen).bfloat16() * 1e-3
    quant = {"x": x, "cases": []}
    for mode, ratio, factor in (
        ("percentile", 0.0, 1.0),
        ("percentile", 0.875, 1.0),
        ("percentile", 0.92, 1.0),
        ("percentile", 0.96, 1.0),
        ("percentile", 1.0, 1.0),
        ("factor", 0.0, 0.9),
    ):
        packed, scale, zero, decoded = oracle.quantize(x, ratio, mode, factor)
        quant["cases"].append(dict(mode=mode, ratio=ratio, factor=factor, packed=packed, scale=scale, zero=zero, decoded=decoded))
    torch.save(quant, HERE / "quantize.pt")

    # 2. packed slot bytes (reference tests/test_npu_kernels.py:71-96 template)
    k = outlier_bf16(gen, 40, 2, 256)
    v = torch.randn(40, 2, 256, generator=gen).bfloat16()
    k[0].zero_()
    k[1].fill_(0.5)
    k[2].fill_(1e-12)
    slots = {"k": k, "v": v, "cases": []}
    for kr, vr in ((0.96, 0.92), (0.0, 0.0), (1.0, 1.0), (0.92, 0.96)):
        cfg = replace(cfg_mod.OscarConfig(), k_clip_ratio=kr, v_clip_ratio=vr)
        slots["cases"].append(dict(k_ratio=kr, v_ratio=vr, bytes=oracle.packed_slots(k, v, cfg)))
    torch.save(slots, HERE / "packed_slots.pt")

    # 3. exact unpack vectors (reference tests/test_packed_load.py:13-32)
    rows = 16
    vec = torch.zeros(rows, 68, dtype=torch.uint8)
    expect = torch.zeros(rows, 256, dtype=torch.bfloat16)
    for row in range(rows):
        codes = (torch.arange(256) + row) % 4
        vec[row, :64] = (codes.reshape(64, 4) << (torch.arange(4) * 2)).sum(1).byte()
        s = torch.tensor([0.125 * (row + 1)], dtype=torch.float16)
        z = torch.tensor([-0.25 * row], dtype=torch.float16)
        vec[row, 64:66] = s.view(torch.uint8)
        vec[row, 66:68] = z.view(torch.uint8)
        expect[row] = (codes.float() * s.float() + z.float()).bfloat16()
    torch.save({"vectors": vec, "decoded": expect}, HERE / "unpack.pt")

    # 4. hybrid reference (config-1 geometry, scaled down) with the oracle's output
    cases = []
    for lengths, prefixes, hq, h, sink, recent, mtp in (
        ([200, 300], [199, 299], 8, 1, 4, 64, 0),
        ([160, 233], [156, 230], 6, 1, 4, 64, 3),
        ([290], [286], 8, 2, 4, 64, 3),
    ):
        cfg, rk, rv, ks, vs, qs, hist, window, meta, bp = build_paged_case(
            cfg_mod, oracle, lengths, prefixes, hq, h, sink, recent, mtp, seed=len(cases) + 5
        )
        outs = [oracle.hybrid_reference(q, kk, vv, p, rk, rv, cfg) for q, kk, vv, p in zip(qs, ks, vs, prefixes)]
        cases.append(
            dict(lengths=lengths, prefixes=prefixes, hq=hq, h=h, sink=sink, recent=recent, mtp=mtp, rk=rk, rv=rv, k=ks, v=vs, q=qs, expected=outs)
        )
    torch.save(cases, HERE / "hybrid.pt")

    # 5. the reference attention kernel body on a real paged cache (history + raw paths)
    att = []
    for lengths, prefixes, hq, h, sink, recent, mtp, splits in (
        ([300, 200], [299, 199], 8, 1, 4, 64, 0, 4),
        ([260, 200], [256, 197], 6, 1, 4, 64, 3, 3),
        ([300], [296], 4, 2, 4, 32, 3, 2),
    ):
        cfg, rk, rv, ks, vs, qs, hist, window, meta, bp = build_paged_case(
            cfg_mod, oracle, lengths, prefixes, hq, h, sink, recent, mtp, seed=100 + len(att)
        )
        q = torch.cat(qs)
        qrot = (q.float() @ rk.float()).bfloat16()
        kcur = torch.cat([kk[p:] for kk, p in zip(ks, prefixes)])
        vcur = torch.cat([vv[p:] for vv, p in zip(vs, prefixes)])
        qt = 4
        n = q.shape[0]
        cap = cfg_mod.task_capacity(n, len(lengths) + 1, qt)
        tasks, count = run_reference_tasks(ref, Pointer, meta["query_start_loc"], meta["counts"], cap, len(lengths) + 1, qt, len(lengths))
        base = dict(
            CurrentK=kcur,
            CurrentV=vcur,
            History=hist,
            Window=window,
            QStarts=meta["query_start_loc"],
            SeqLens=meta["seq_lens"],
            Table=meta["block_tables"],
            Counts=meta["counts"],
            Tasks=tasks,
            TaskCount=torch.tensor([count], dtype=torch.int32),
        )
        geo = dict(H=h, G=hq // h, QT=qt, BP=bp, PAGE_BYTES=bp * h * 512, SINK=sink, RECENT=recent, RING=recent + mtp + 1, programs=cap)
        hp, hl = run_reference_attention(ref, Pointer, dict(base, Query=qrot), geo, splits, False)
        rp, rl = run_reference_attention(ref, Pointer, dict(base, Query=q), geo, 1, True)
        att.append(
            dict(
                lengths=lengths, prefixes=prefixes, hq=hq, h=h, sink=sink, recent=recent, mtp=mtp, splits=splits,
                rk=rk, rv=rv, q=q, qrot=qrot, k=kcur, v=vcur, history=zpack(hist), window=zpack(window), meta=meta, bp=bp,
                hist_partials=hp, hist_lse=hl, raw_partials=rp, raw_lse=rl,
            )
        )
    torch.save(att, HERE / "attention_kernel.pt")

    # 6. the reference task-table kernel body
    tcases = []
    for lengths, active, qt in (([], 0, 4), ([0, 0], 0, 4), ([4] * 9, 36, 4), ([7, 0, 1, 11], 19, 4), ([7, 0, 1, 11], 10, 2), ([5, 3], 8, 1)):
        max_reqs = 12
        starts = [0]
        for s in lengths:
            starts.append(starts[-1] + s)
        qstarts = torch.zeros(max_reqs + 1, dtype=torch.int32)
        qstarts[: len(starts)] = torch.tensor(starts, dtype=torch.int32)
        counts = torch.tensor([len(lengths), active], dtype=torch.int32)
        cap = cfg_mod.task_capacity(max(active, 1), max_reqs, qt)
        tasks, count = run_reference_tasks(ref, Pointer, qstarts, counts, cap, max_reqs, qt, max(1, len(lengths)))
        tcases.append(dict(qstarts=qstarts, counts=counts, query_tile=qt, capacity=cap, tasks=tasks, count=count))
    torch.save(tcases, HERE / "tasks.pt")

    # 7. calibration math (reference tests/test_calibration_math.py)
    g14 = torch.Generator().manual_seed(14)
    xx = torch.randn(48, 16, dtype=torch.float64, generator=g14)
    cov = xx.T @ xx
    u, ev = jacobi_oracle(cov)
    torch.save(dict(cov=cov, u=u, eigenvalues=ev, hadamard16=hadamard(16), pbr16=pbr(16), pbr256=pbr(256)), HERE / "calibration.pt")

    # 8. geometry constants straight from the reference classes
    from oscar_ascend.layout import CacheLayout  # noqa: E402

    lay = CacheLayout(768)
    lay4 = CacheLayout(768, kv_heads=4, config=replace(cfg_mod.OscarConfig(), sink_tokens=4, recent_tokens=128, speculative_tokens=3))
    geo = dict(
        vector_bytes=lay.config.vector_bytes,
        slot_bytes=lay.config.slot_bytes,
        stripe_page_bytes=lay.stripe_page_bytes,
        history_page_bytes=lay.history_page_bytes,
        window_page_bytes=lay.window_page_bytes,
        blocks_per_page=lay.blocks_per_page,
        slot_offsets=[(s, hh, lay4.slot_offset(s, hh)) for s in (0, 1, 127, 128, 767, 768, 5000) for hh in range(4)],
        window_offsets=[(b, t, kv, hh, lay4.window_offset(b, t, kv, hh)) for b in (0, 6, 42) for t in (0, 3, 4, 135, 136, 1000) for kv in (0, 1) for hh in (0, 3)],
        selections={r: cfg_mod.percentile_selection(r) for r in (0.875, 0.92, 0.96, 1.0)},
        splits=[(b, hh, ql, cfg_mod.choose_splits(b, hh, ql)) for b in (1, 2, 8, 16, 64) for hh in (1, 4) for ql in (1, 4, 17)],
        capacity=[(t, r, qt, cfg_mod.task_capacity(t, r, qt)) for t in (1, 64, 512, 16000) for r in (1, 33, 129) for qt in (1, 2, 4)],
    )
    torch.save(geo, HERE / "geometry.pt")
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
