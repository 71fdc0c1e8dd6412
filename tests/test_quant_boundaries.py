"""The device quantiser's exact code boundaries, restated in numpy, against the oracle.

The packed quantiser (`oscar_new_b200/csrc/quant.cuh`, `code_boundaries`) codes a bf16
value x as #{c in 1..3 : x >= B_c}, with B_c the smallest bf16 whose reference code
clamp(trunc(RN(RN(RN(x - z) / s) + 0.5)), 0, 3) is >= c.  It finds B_c without a
division by inverting the three roundings through their midpoints in fp64, then checks
the candidate with two exact evaluations (bisection if the check fails).  This test runs
the same steps in numpy (IEEE float32 / float64, round to nearest) on adversarial
vectors and requires (a) codes identical to the oracle's and (b) that the check never
fails on them, i.e. that the fallback is never needed.  The device path itself is
checked byte for byte on a B200 by tests/test_gpu_kernels.py.
"""

import numpy as np
import torch

from oracle.int2_oracle import clip_threshold, quantize

F32, F64 = np.float32, np.float64


def _pred32(x):
    return np.nextafter(x, F32(-np.inf))


def _ru32(y):  # smallest float32 >= y (float64 array)
    f = y.astype(F32)
    low = f.astype(F64) < y
    f[low] = np.nextafter(f[low], F32(np.inf))
    return f


def _bf16_ru(f):  # smallest bf16 >= f (finite float32 array)
    b = f.view(np.uint32).copy()
    frac = (b & 0xFFFF) != 0
    pos = (b >> 31) == 0
    b[frac & pos] = (b[frac & pos] & 0xFFFF0000) + 0x10000
    b[frac & ~pos] &= 0xFFFF0000
    return b.view(F32)


def _bf16_step(x, d):  # neighbouring bf16 (d = +1 up, -1 down)
    b = (x.view(np.uint32) >> 16).astype(np.int64)
    key = np.where(b & 0x8000, 0x7FFF - (b & 0x7FFF), b + 0x8000) + d
    nb = np.where(key >= 0x8000, key - 0x8000, 0x8000 | (0x7FFF - key))
    return (nb.astype(np.uint32) << 16).view(F32)


def _r(y, z, s):  # RN(RN(RN(y - z) / s) + 0.5)
    with np.errstate(all="ignore"):
        return (((y - z).astype(F32) / s).astype(F32) + F32(0.5)).astype(F32)


# smallest float32 q with RN(q + 0.5) >= c, and whether it is odd (strict midpoint)
Q = {1: np.uint32(0x3EFFFFFF).view(F32), 2: F32(1.5), 3: F32(2.5)}


def boundaries(lo, hi, z, s):
    """B_c [N, 3] (NaN: no value reaches c; -inf: every value does) and the number of
    candidates whose exact check failed."""
    rlo, rhi = _r(lo, z, s), _r(hi, z, s)
    bad = ~np.isfinite(z) | ~np.isfinite(s)
    out = np.zeros((len(z), 3), F32)
    failed = 0
    for c in (1, 2, 3):
        q = np.float32(Q[c])
        mq = (F64(_pred32(q)) + F64(q)) / 2
        sm = s.astype(F64) * mq
        d = _ru32(sm)
        if int(q.view(np.uint32)) & 1:
            eq = d.astype(F64) == sm
            d[eq] = np.nextafter(d[eq], F32(np.inf))
        md = (_pred32(d).astype(F64) + d.astype(F64)) / 2
        y = z.astype(F64) + md
        b = _bf16_ru(_ru32(y))
        strict = ((d.view(np.uint32) & 1) == 1) & (b.astype(F64) == y)
        b[strict] = _bf16_step(b[strict], +1)
        ok = (_r(b, z, s) >= c) & (_r(_bf16_step(b, -1), z, s) < c)
        none = bad | (rhi < c)
        every = ~none & (rlo >= c)
        res = b.copy()
        res[none] = np.nan
        res[every] = -np.inf
        failed += int((~ok & ~none & ~every).sum())
        out[:, c - 1] = res
    return out, failed


def _rows(gen, n):
    kinds = [
        lambda: torch.randn(n, 256, generator=gen) * torch.where(torch.arange(256) < 8, 20.0, 1.0),
        lambda: torch.rand(n, 256, generator=gen) * 3 - 1.5,
        lambda: torch.randint(-4, 5, (n, 256), generator=gen).float() * 0.25,
        lambda: torch.randn(n, 256, generator=gen) * 1e-20,
        lambda: torch.randn(n, 256, generator=gen) * torch.logspace(-6, 4, 256),
        lambda: torch.randn(n, 256, generator=gen) * 3000 + torch.randn(n, 1, generator=gen) * 20000,
    ]
    return torch.cat([k() for k in kinds]).bfloat16()


def test_exact_boundaries_match_oracle_codes():
    gen = torch.Generator().manual_seed(11)
    xb = _rows(gen, 1500)
    x = xb.float()
    xn = x.numpy().astype(F32)
    total_failed = 0
    for ratio, mode, factor in ((0.96, "percentile", 1.0), (0.92, "percentile", 1.0), (0.0, "percentile", 1.0),
                                (0.96, "factor", 0.9)):
        packed, scale, zero, _ = quantize(xb, ratio, mode, factor)
        lo, hi = xn.min(1), xn.max(1)
        if mode == "factor":
            thr = (x.abs().amax(-1) * factor).numpy().astype(F32)
        elif ratio:
            thr = clip_threshold(x.abs(), ratio).numpy()[:, 0].astype(F32)
        else:
            thr = None
        if thr is not None:  # min / max of the clipped values
            lo, hi = np.minimum(np.maximum(lo, -thr), thr), np.maximum(np.minimum(hi, thr), -thr)
        z = zero.float().numpy()[:, 0].astype(F32)
        s = scale.float().numpy()[:, 0].astype(F32)
        b, failed = boundaries(lo.astype(F32), hi.astype(F32), z, s)
        total_failed += failed
        with np.errstate(invalid="ignore"):
            codes = (xn >= b[:, None, 0]).astype(np.int64) + (xn >= b[:, None, 1]) + (xn >= b[:, None, 2])
        p = packed.numpy()
        ref = np.stack([(p >> (2 * k)) & 3 for k in range(4)], -1).reshape(len(p), 256)
        bad = np.nonzero((codes != ref).any(1))[0]
        assert bad.size == 0, (ratio, mode, bad[:5])
    assert total_failed == 0
