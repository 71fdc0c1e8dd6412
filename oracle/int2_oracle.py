"""CPU oracle for the OSCAR INT2 KV-cache path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and
``--impl reference``) may import this module, and only as the checker / the timed CPU
reference.  The product package ``oscar_new_b200`` never imports it.

It restates, in plain numpy / torch-CPU code, the arithmetic of the reference
(jpl123123/Oscar_new v0.3.2, Triton-Ascend):

* ``quantize`` / ``packed_slots``  — reference ``tests/oracle.py:6-39`` and the byte
  order of ``oscar_ascend/kernels.py:104-137`` (clip, fp16 scale/zero, codes, pack).
* ``dense_attention`` / ``hybrid_reference`` — ``tests/oracle.py:42-65``, plus the
  natural-log LSE of the same masked, scaled fp32 scores
  (``tests/test_attention_empty_tasks.py:203`` computes it the same way).
* paged-kernel semantics: ``attention_partials`` — ``kernels.py:290-436`` (history and
  raw BF16 path, split ranges of ``BN``-token tiles, empty split -> 0 / -inf);
  ``merge_splits`` — ``kernels.py:485-503``; ``merge_paths`` — ``kernels.py:514-527``;
  ``store_windows`` — ``kernels.py:544-595``; ``prepare_tasks`` — ``kernels.py:222-259``;
  ``unpack`` — ``kernels.py:205-219``.

Parity pin: ``tests/test_oracle_golden.py`` checks these functions against fixtures in
``tests/golden/`` that ``tests/golden/make_golden.py`` produced by importing the
reference's own ``tests/oracle.py`` and ``config.py`` and running its test vectors.
"""

from __future__ import annotations

import math

import numpy as np
import torch

# ----------------------------------------------------------------------------
# quantisation (reference tests/oracle.py:6-21, kernels.py:69-137)
# ----------------------------------------------------------------------------


def clip_threshold(absx: torch.Tensor, ratio: float) -> torch.Tensor:
    """``torch.quantile(absx, ratio, dim=-1, keepdim=True)`` restated.

    ATen sorts ascending, takes fp32 rank ``r = f32(ratio) * 255`` and interpolates
    ``lerp(sorted[floor r], sorted[ceil r], r - floor r)``; CPU ``lerp`` is a fused
    multiply-add: ``fma(w, hi-lo, lo)`` for ``w < 0.5`` else ``fma(w-1, hi-lo, hi)``.
    ``torch.lerp`` is that exact kernel.
    """
    n = absx.shape[-1]
    rank = np.float32(ratio) * np.float32(n - 1)
    lo_i, hi_i = int(np.floor(rank)), int(np.ceil(rank))
    weight = float(np.float32(rank - np.float32(lo_i)))
    s = absx.float().sort(-1).values
    lo = s[..., lo_i : lo_i + 1]
    hi = s[..., hi_i : hi_i + 1]
    return torch.lerp(lo, hi, torch.full_like(lo, weight))


def quantize(x: torch.Tensor, ratio: float = 0.0, mode: str = "percentile", factor: float = 1.0):
    """Clip + asymmetric 2-bit quantisation of the last (D=256) axis.

    Returns ``(packed uint8 [..., D/4], scale fp16 [...,1], zero fp16 [...,1], decoded bf16)``.
    """
    x = x.float()
    if mode == "factor":
        thr = x.abs().amax(-1, keepdim=True) * factor
        x = torch.minimum(torch.maximum(x, -thr), thr)
    elif ratio:
        thr = clip_threshold(x.abs(), ratio)
        x = torch.minimum(torch.maximum(x, -thr), thr)
    lo = x.amin(-1, keepdim=True)
    hi = x.amax(-1, keepdim=True)
    zero = lo.half()
    scale = ((hi - lo) / 3).clamp_min(2.0**-14).half()
    code = ((x - zero.float()) / scale.float() + 0.5).to(torch.int32).clamp(0, 3)
    c = code.reshape(*code.shape[:-1], -1, 4)
    packed = (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).to(torch.uint8)
    decoded = (code.float() * scale.float() + zero.float()).bfloat16()
    return packed, scale, zero, decoded


def packed_slots(k: torch.Tensor, v: torch.Tensor, cfg) -> torch.Tensor:
    """[..., slot_bytes] uint8: K vector at +0, V vector at +68, padding left 0."""
    out = torch.zeros((*k.shape[:-1], cfg.slot_bytes), dtype=torch.uint8)
    for val, off, ratio, factor in (
        (k, 0, cfg.k_clip_ratio, cfg.k_clip_factor),
        (v, cfg.vector_bytes, cfg.v_clip_ratio, cfg.v_clip_factor),
    ):
        codes, scale, zero, _ = quantize(val, ratio, cfg.clip_mode, factor)
        db = cfg.data_bytes
        out[..., off : off + db] = codes
        out[..., off + db : off + db + 2] = scale.contiguous().view(torch.uint8)
        out[..., off + db + 2 : off + db + 4] = zero.contiguous().view(torch.uint8)
    return out


def unpack(vec_bytes: np.ndarray, dim: int = 256) -> torch.Tensor:
    """[N, 68] uint8 vectors -> bf16 [N, dim] (reference kernels.py:205-219)."""
    vb = np.ascontiguousarray(vec_bytes, dtype=np.uint8)
    data = vb[:, : dim // 4]
    codes = np.stack([(data >> (2 * p)) & 3 for p in range(4)], axis=-1).reshape(len(vb), dim)
    scale = vb[:, dim // 4 : dim // 4 + 2].copy().view(np.float16).astype(np.float32)
    zero = vb[:, dim // 4 + 2 : dim // 4 + 4].copy().view(np.float16).astype(np.float32)
    return (torch.from_numpy(codes.astype(np.float32)) * torch.from_numpy(scale) + torch.from_numpy(zero)).bfloat16()


# ----------------------------------------------------------------------------
# dense references (reference tests/oracle.py:42-65)
# ----------------------------------------------------------------------------


def dense_attention(q, k, v, prefix: int, with_lse: bool = False):
    """fp32 causal attention of ``q`` [nq,Hq,D] over ``k,v`` [nk,Hk,D] (GQA).

    Query ``i`` sees keys ``j <= prefix + i``; scale ``1/sqrt(D)``; natural-log LSE.
    """
    hq, hk = q.shape[1], k.shape[1]
    keys = k.float().repeat_interleave(hq // hk, 1)
    vals = v.float().repeat_interleave(hq // hk, 1)
    scores = torch.einsum("qhd,khd->hqk", q.float(), keys) / math.sqrt(q.shape[-1])
    qi = torch.arange(q.shape[0]) + prefix
    kj = torch.arange(k.shape[0])
    scores.masked_fill_(kj[None, None, :] > qi[None, :, None], -math.inf)
    out = torch.einsum("hqk,khd->qhd", scores.softmax(-1), vals)
    if with_lse:
        return out, scores.logsumexp(-1).transpose(0, 1)
    return out


def hybrid_reference(q, k, v, prefix: int, rk, rv, cfg, with_lse: bool = False):
    """Dense attention where history tokens [S, max(min(S,P), P-R)) are replaced by
    their rotate -> quantise -> dequantise -> inverse-rotate reconstruction."""
    end = max(min(cfg.sink_tokens, prefix), prefix - cfg.recent_tokens)
    kr = (k.float() @ rk.float()).bfloat16()
    vr = (v.float() @ rv.float()).bfloat16()
    kd = quantize(kr, cfg.k_clip_ratio, cfg.clip_mode, cfg.k_clip_factor)[3]
    vd = quantize(vr, cfg.v_clip_ratio, cfg.clip_mode, cfg.v_clip_factor)[3]
    keys, vals = k.float().clone(), v.float().clone()
    keys[cfg.sink_tokens : end] = kd[cfg.sink_tokens : end].float() @ rk.float().T
    vals[cfg.sink_tokens : end] = vd[cfg.sink_tokens : end].float() @ rv.float().T
    return dense_attention(q, keys, vals, prefix, with_lse)


# ----------------------------------------------------------------------------
# paged-cache semantics (reference layout.py:46-73, kernels.py)
# ----------------------------------------------------------------------------


def slot_addresses(slots: np.ndarray, head: int, layout) -> np.ndarray:
    slots = np.asarray(slots, dtype=np.int64)
    bp = layout.physical_block_tokens
    return (slots // bp) * layout.stripe_page_bytes + ((slots % bp) * layout.kv_heads + head) * layout.config.slot_bytes


def history_vectors(history: np.ndarray, table_row, positions, head: int, layout, kv: int):
    """Dequantised rotated K (kv=0) or V (kv=1) rows of logical ``positions``."""
    positions = np.asarray(positions, dtype=np.int64)
    table_row = np.asarray(table_row, dtype=np.int64)
    slots = table_row[positions // layout.kernel_block_tokens] * layout.kernel_block_tokens + positions % layout.kernel_block_tokens
    base = slot_addresses(slots, head, layout) + kv * layout.config.vector_bytes
    idx = base[:, None] + np.arange(layout.config.vector_bytes)[None, :]
    return unpack(history[idx], layout.config.head_dim)


def window_rows(window: torch.Tensor, first_block: int, positions, head: int, layout, kv: int):
    cfg = layout.config
    owner = int(first_block) // layout.blocks_per_page
    out = []
    for p in positions:
        p = int(p)
        idx = p if p < cfg.sink_tokens else cfg.sink_tokens + p % cfg.ring_tokens
        off = owner * (layout.stripe_page_bytes // 2) + ((idx * 2 + kv) * layout.kv_heads + head) * cfg.head_dim
        out.append(window[off : off + cfg.head_dim])
    if not out:
        return torch.zeros((0, cfg.head_dim), dtype=torch.bfloat16)
    return torch.stack(out)


def _softmax_partial(q, keys, vals, scale, mask=None):
    """Normalised fp32 output and natural LSE of ``q`` [R,D] over ``keys`` [N,D]."""
    if keys.shape[0] == 0:
        return torch.zeros(q.shape[0], q.shape[1]), torch.full((q.shape[0],), -math.inf)
    s = (q.float() @ keys.float().T) * scale
    if mask is not None:
        s = s.masked_fill(~mask, -math.inf)
    lse = torch.logsumexp(s, -1)
    w = torch.exp(s - torch.where(torch.isinf(lse), torch.zeros_like(lse), lse)[:, None])
    w = torch.nan_to_num(w, nan=0.0)
    o = w @ vals.float()
    return o, lse


def attention_partials(query, key, value, history, window, meta, layout, scale, splits, raw, block_n=32):
    """Restated ``_attention_kernel`` semantics (reference kernels.py:290-436).

    ``meta`` holds host tensors ``query_start_loc``, ``seq_lens``, ``block_tables``,
    ``counts``.  Returns ``partials`` [n,Hq,splits,D] fp32 and ``lse`` [n,Hq,splits];
    entries of rows that are not live are NaN (the kernel leaves them unwritten).
    """
    cfg = layout.config
    n, hq, d = query.shape
    h = layout.kv_heads
    g = hq // h
    hist = history.numpy() if isinstance(history, torch.Tensor) else history
    part = torch.full((n, hq, splits, d), math.nan)
    lse = torch.full((n, hq, splits), math.nan)
    qs = meta.query_start_loc.tolist()
    seqs = meta.seq_lens.tolist()
    nr, active = int(meta.counts[0]), int(meta.counts[1])
    for req in range(nr):
        qstart = qs[req]
        qend = min(qs[req + 1], active)
        qlen = qend - qstart
        if qlen <= 0:
            continue
        prefix = seqs[req] - qlen
        sink_len = min(cfg.sink_tokens, prefix)
        recent_begin = max(sink_len, prefix - cfg.recent_tokens)
        table = meta.block_tables[req].tolist()
        for head in range(h):
            q = query[qstart:qend, head * g : (head + 1) * g].reshape(qlen * g, d)
            qi = torch.arange(qlen).repeat_interleave(g)
            if raw:
                positions = list(range(sink_len)) + list(range(recent_begin, prefix)) + list(range(prefix, prefix + qlen))
                nprev = sink_len + prefix - recent_begin
                ks = torch.cat([window_rows(window, table[0], positions[:nprev], head, layout, 0).float(), key[qstart:qend, head].float()])
                vs = torch.cat([window_rows(window, table[0], positions[:nprev], head, layout, 1).float(), value[qstart:qend, head].float()])
                pos = torch.tensor(positions)
                mask = pos[None, :] <= (prefix + qi)[:, None]
                o, l = _softmax_partial(q, ks, vs, scale, mask)
                for r in range(qlen * g):
                    part[qstart + r // g, head * g + r % g, 0] = o[r]
                    lse[qstart + r // g, head * g + r % g, 0] = l[r]
                continue
            length = recent_begin - sink_len
            tiles = -(-length // block_n)
            per_split = -(-tiles // splits)
            for s in range(splits):
                begin = s * per_split * block_n
                end = min((s + 1) * per_split * block_n, length)
                pos = np.arange(sink_len + begin, sink_len + max(end, begin))
                ks = history_vectors(hist, table, pos, head, layout, 0)
                vs = history_vectors(hist, table, pos, head, layout, 1)
                o, l = _softmax_partial(q, ks, vs, scale)
                for r in range(qlen * g):
                    part[qstart + r // g, head * g + r % g, s] = o[r]
                    lse[qstart + r // g, head * g + r % g, s] = l[r]
    return part, lse


def merge_splits(partials, lse, counts):
    """(reference kernels.py:485-503) -> bf16 [n,Hq,D], fp32 [n,Hq]; every row written."""
    n, hq, s, d = partials.shape
    valid = (torch.arange(n) < int(counts[1]))[:, None, None].expand(n, hq, s)
    ls = torch.where(valid, lse, torch.full_like(lse, -math.inf))
    m = ls.amax(-1)
    safe = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m), m)
    w = torch.exp(ls - safe[..., None])
    den = w.sum(-1)
    vals = torch.where(valid[..., None], torch.nan_to_num(partials, nan=0.0), torch.zeros_like(partials))
    out = (vals * w[..., None]).sum(-2) / den.clamp_min(1e-30)[..., None]
    logsum = torch.where(den > 0, m + torch.log(den.clamp_min(1e-30)), torch.full_like(m, -math.inf))
    return out.bfloat16(), logsum


def merge_paths(a, la, b, lb, counts):
    """(reference kernels.py:514-527): LSE-weighted average, invalid rows -> 0."""
    n = a.shape[0]
    valid = (torch.arange(n) < int(counts[1]))[:, None]
    la = torch.where(valid, la, torch.full_like(la, -math.inf))
    lb = torch.where(valid, lb, torch.full_like(lb, -math.inf))
    m = torch.maximum(la, lb)
    m = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m), m)
    wa, wb = torch.exp(la - m), torch.exp(lb - m)
    af = torch.where(valid[..., None], a.float(), torch.zeros_like(a.float()))
    bf = torch.where(valid[..., None], torch.nan_to_num(b.float(), nan=0.0), torch.zeros_like(b.float()))
    return (wa[..., None] * af + wb[..., None] * bf) / (wa + wb).clamp_min(1e-30)[..., None]


def prepare_tasks(qstarts, counts, query_tile: int, capacity: int):
    """(reference kernels.py:222-259): ``(tasks [capacity,2] with -1 fill, task_count)``."""
    nr, active = int(counts[0]), int(counts[1])
    tasks = []
    for req in range(nr):
        start = min(int(qstarts[req]), active)
        end = min(int(qstarts[req + 1]), active)
        for off in range(0, max(end - start, 0), query_tile):
            tasks.append((req, off))
    out = torch.full((capacity, 2), -1, dtype=torch.int32)
    if tasks:
        out[: len(tasks)] = torch.tensor(tasks, dtype=torch.int32)
    return out, len(tasks)


def store_windows(key, value, window, meta, layout, num_programs: int):
    """(reference kernels.py:544-595): write current BF16 K/V into sink/ring slots;
    each ring slot gets only its latest writer.  Mutates ``window`` in place."""
    cfg = layout.config
    qs = meta.query_start_loc.tolist()
    seqs = meta.seq_lens.tolist()
    nr, active = int(meta.counts[0]), int(meta.counts[1])
    ring, sink = cfg.ring_tokens, cfg.sink_tokens
    for req in range(min(num_programs, nr)):
        qstart = qs[req]
        qend = min(qs[req + 1], active)
        seq = seqs[req]
        prefix = seq - (qend - qstart)
        owner = int(meta.block_tables[req, 0]) // layout.blocks_per_page
        for idx in range(sink + ring):
            if idx < sink:
                pos = idx
            else:
                residue = idx - sink
                pos = seq - 1 - ((seq - 1 - residue) % ring)
            ok = pos >= prefix and pos < seq and qend > qstart and (idx < sink or pos >= sink)
            if not ok:
                continue
            cur = qstart + pos - prefix
            for head in range(layout.kv_heads):
                for kv, src in ((0, key), (1, value)):
                    off = owner * (layout.stripe_page_bytes // 2) + ((idx * 2 + kv) * layout.kv_heads + head) * cfg.head_dim
                    window[off : off + cfg.head_dim] = src[cur, head]
    return window


def decode_reference(query_rot, query, key, value, history, window, meta, layout, scale, rv):
    """End-to-end output of one decode/verify step over a paged cache.

    History attention in the rotated space (the reference kernel's arithmetic), merged
    over the whole history, inverse-rotated with ``rv``, LSE-merged with the raw BF16
    path.  Returns ``(output [n,Hq,D] fp32, history_lse [n,Hq], raw_lse [n,Hq])``.
    """
    hp, hl = attention_partials(query_rot, key, value, history, window, meta, layout, scale, 1, False)
    rp, rl = attention_partials(query, key, value, history, window, meta, layout, scale, 1, True)
    hrot, hls = merge_splits(hp, hl, meta.counts)
    hout = (hrot.float() @ rv.float().T).bfloat16()
    out = merge_paths(hout, hls, rp[:, :, 0], rl[:, :, 0], meta.counts)
    return out, hls, rl[:, :, 0]
