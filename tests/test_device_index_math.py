"""Index and bit arithmetic of the device kernels, restated on the CPU.

The device code itself runs in the GPU tests; these tests pin the small exact
arithmetic those kernels rely on, over every case rather than a sample:
  * the history kernels' key operands (history_common.cuh `key_lut` and the PRMT
    selectors `x * 0x11 + 0x40404040`) fetch exactly the reference's bf16 key levels,
    for every byte of four 2-bit codes;
  * the packed quantiser's counts (quant.cuh `count_ge_bf16`) stay exact small integers
    in bf16 and read back from the low 7 bits of 128 + n;
  * the MTP kernel's value byte lanes (history_mtp.cu) split the 256 dims among the four
    warps of a head and extract the codes the reference's unpack assigns to those dims;
  * the Jacobi ring (calibration.cu): the register moves between rounds keep every pair
    on the columns of the reference's round-robin schedule, and the partial-sum reads of
    a quarter warp fall on distinct shared-memory banks;
  * the rotation epilogue's row -> (token, head) split by multiply-high (rotate.cuh);
  * the window store (attention.cu `window_store_kernel`) visits exactly the reference's
    per-slot latest writers, each slot once.
"""

import numpy as np
import torch

from oracle.calibration_oracle import round_robin_pairs
from oracle.int2_oracle import unpack


def prmt(a: int, b: int, sel: int) -> int:
    """PTX prmt.b32 (default mode): byte i of the result is byte (nibble i & 7) of the
    eight bytes b:a, or that byte's sign replicated when nibble bit 3 is set."""
    pool = [(a >> (8 * k)) & 0xFF for k in range(4)] + [(b >> (8 * k)) & 0xFF for k in range(4)]
    out = 0
    for i in range(4):
        nib = (sel >> (4 * i)) & 0xF
        byte = pool[nib & 7]
        if nib & 8:
            byte = 0xFF if byte & 0x80 else 0x00
        out |= byte << (8 * i)
    return out


def half_bits(x: float) -> int:
    return int(np.array([x], dtype=np.float16).view(np.uint16)[0])


def bf16(x):
    return torch.tensor(x, dtype=torch.float32).bfloat16().float().numpy()


def key_table(s: np.float16, z: np.float16):
    """key_lut: the four levels bf16(c*s + z), scaled by 2^e into [2^14, 2^15), as fp16
    byte planes (lo = low bytes, hi = high bytes); returns (lo, hi, scaled levels)."""
    sf, zf = np.float32(s), np.float32(z)
    v = bf16([zf, np.float32(sf + zf), np.float32(np.float32(2) * sf + zf), np.float32(np.float32(3) * sf + zf)])
    ex = (np.array([max(abs(v[0]), abs(v[3]))], dtype=np.float32).view(np.uint32)[0] >> 23) & 0xFF
    exc = max(int(ex), 16)
    up = np.array([(268 - exc) << 23], dtype=np.uint32).view(np.float32)[0]
    scaled = (v * up).astype(np.float32)
    h = [half_bits(x) for x in scaled]
    h01, h23 = h[0] | (h[1] << 16), h[2] | (h[3] << 16)
    return prmt(h01, h23, 0x6420), prmt(h01, h23, 0x7531), scaled


def test_key_selectors_fetch_the_bf16_levels_for_every_code_byte():
    rng = np.random.default_rng(7)
    cases = [(np.float16(0.5), np.float16(-0.75)), (np.float16(2.0 ** -14), np.float16(0.0)),
             (np.float16(3000.0), np.float16(-60000.0))]
    cases += [(np.float16(abs(rng.normal()) * 10 ** rng.uniform(-3, 2) + 2 ** -14), np.float16(rng.normal() * 30))
              for _ in range(40)]
    for s, z in cases:
        lo, hi, levels = key_table(s, z)
        # the scaled levels are exact in fp16
        assert np.array_equal(levels.astype(np.float16).astype(np.float32), levels)
        for word in range(256):
            codes = [(word >> (2 * p)) & 3 for p in range(4)]
            x = sum(c << (8 * k) for k, c in enumerate(codes))  # codes of one position, bytes 0..3
            sel = (x * 0x11 + 0x40404040) & 0xFFFFFFFF
            for half, pair in ((sel & 0xFFFF, codes[:2]), (sel >> 16, codes[2:])):
                r = prmt(lo, hi, half)
                got = np.array([r & 0xFFFF, r >> 16], dtype=np.uint16).view(np.float16).astype(np.float32)
                assert np.array_equal(got, levels[pair]), (s, z, word)


def test_bf16_counts_are_exact_small_integers():
    one, zero = torch.tensor(1.0).bfloat16(), torch.tensor(0.0).bfloat16()
    for lo_counts in np.ndindex(5, 5):
        for hi_counts in np.ndindex(5, 5):
            halves = []
            for c0, c1 in (lo_counts, hi_counts):
                a0 = torch.tensor(32.0).bfloat16()
                a1 = torch.tensor(32.0).bfloat16()
                for i in range(4):
                    a0 = a0 + (one if i < c0 else zero)
                    a1 = a1 + (one if i < c1 else zero)
                halves.append(a0 + a1)
            total = halves[0] + halves[1]
            bits = int(total.view(torch.int16).item()) & 0xFFFF
            assert bits & 0x7F == sum(lo_counts) + sum(hi_counts)


def test_mtp_value_byte_lanes_partition_the_dims():
    dims = [32 * gi + 16 * half + 4 * w + p for w in range(4) for gi in range(8) for half in range(2)
            for p in range(4)]
    assert sorted(dims) == list(range(256))
    # warp w's operand: prmt(word of token a, same word of token b, vsel) >> vshift, then
    # mask 0x00030003 << 2p: token a's code in bits 2p..2p+1, token b's 16 bits higher
    rng = np.random.default_rng(11)
    vecs = np.zeros((2, 68), dtype=np.uint8)
    vecs[:, :64] = rng.integers(0, 256, size=(2, 64), dtype=np.uint8)
    vecs[:, 64:66] = np.array([1.0], dtype=np.float16).view(np.uint8)  # scale 1, zero 0
    codes = unpack(vecs).float().numpy().astype(int)
    words = vecs[:, :64].copy().view("<u4")
    for w in range(4):
        vsel = 0x7632 if w >> 1 else 0x5410
        vshift = 8 if w & 1 else 0
        for gi in range(8):
            for half in range(2):
                x = prmt(int(words[0, 2 * gi + half]), int(words[1, 2 * gi + half]), vsel) >> vshift
                for p in range(4):
                    d = 32 * gi + 16 * half + 4 * w + p
                    assert (x >> (2 * p)) & 3 == codes[0, d]
                    assert (x >> (16 + 2 * p)) & 3 == codes[1, d]


def test_jacobi_ring_moves_follow_the_round_robin_schedule():
    """jacobi_kernel: group m (lanes 4(m % 8) .. + 3 of warp m // 8) holds pairs 2m and
    2m + 1.  Between rounds: p0 <- p1 (pair 0 keeps column 255), q0 <- group m - 1's q1
    (pair 0: its own p1), p1 <- group m + 1's p0 (pair 127: its own q1), q1 <- q0; a
    move from another group is a shuffle by 4 lanes, or a shared-memory hand-over when
    the groups sit in different warps."""
    d, groups = 256, 64
    pairs = [round_robin_pairs(d, r) for r in range(d - 1)]

    def seat(r):
        p, q = (t.tolist() for t in pairs[r % (d - 1)])
        return ([p[2 * m] for m in range(groups)], [q[2 * m] for m in range(groups)],
                [p[2 * m + 1] for m in range(groups)], [q[2 * m + 1] for m in range(groups)])

    p0, q0, p1, q1 = seat(0)
    crossings = 0
    for r in range(3 * (d - 1)):
        assert (p0, q0, p1, q1) == seat(r), r
        n = ([None] * groups, [None] * groups, [None] * groups, [None] * groups)
        for m in range(groups):
            n[0][m] = p0[m] if m == 0 else p1[m]
            n[1][m] = p1[m] if m == 0 else q1[m - 1]
            n[2][m] = q1[m] if m == groups - 1 else p0[m + 1]
            n[3][m] = q0[m]
            crossings += (m % 8 == 0 and m > 0) + (m % 8 == 7 and m < groups - 1)
        p0, q0, p1, q1 = n
    assert crossings == 3 * (d - 1) * 14  # 7 warp boundaries, both directions


def test_jacobi_partial_sum_reads_are_bank_conflict_free():
    """JacobiSmem::all: group stride 560 B, pair k at 272 k, CTA c at 32 c; lane g of group
    m reads CTAs g and g + 4 as 16-byte loads.  Each quarter warp (8 lanes: two groups x
    four lanes) must touch 8 distinct 16-byte bank groups in every load."""
    group_stride, pair_stride = (2 * 34 + 2) * 8, 34 * 8
    for k in range(2):
        for load in (0, 16, 128, 144):  # (a_pp, a_qq), (a_pq, pad) of CTAs g and g + 4
            for quarter in range(4):
                lanes = range(8 * quarter, 8 * quarter + 8)
                addr = [(lane >> 2) * group_stride + k * pair_stride + 32 * (lane & 3) + load for lane in lanes]
                assert all(a % 16 == 0 for a in addr)
                assert len({(a % 128) // 16 for a in addr}) == 8, (k, load, quarter)
    # the bytes a CTA expects per round: 8 CTAs x 64 groups x 2 pairs x (16 + 8) bytes
    assert 8 * 64 * 2 * 24 == 24576 < (1 << 20)


def test_row_to_token_division_by_multiply_high():
    # rotate.cuh: floor(t / h) = umulhi(t, floor((2^32 - 1) / h) + 1) for t < 2^16 (t is
    # a tile's first head plus a row offset); every head count a token can have
    t = np.arange(1 << 16, dtype=np.uint64)
    for h in range(2, 257):
        hm = np.uint64(0xFFFFFFFF // h + 1)
        tq = (t * hm) >> np.uint64(32)
        assert np.array_equal(tq, t // np.uint64(h)), h
        assert np.array_equal(t - tq * np.uint64(h), t % np.uint64(h)), h


def window_positions_visited(seq, qlen, sink, ring):
    """window_store_kernel's loop: sink [lo, min(seq, S)), ring [max(lo, S, seq - C), seq)."""
    if qlen <= 0:
        return []
    lo = max(seq - qlen, 0)
    n_sink = max(0, min(seq, sink) - lo)
    ring_lo = max(lo, sink, seq - ring)
    n_ring = max(0, seq - ring_lo)
    out = []
    for k in range(n_sink + n_ring):
        pos = lo + k if k < n_sink else ring_lo + (k - n_sink)
        out.append((pos if pos < sink else sink + pos % ring, pos))
    return out


def window_positions_reference(seq, qlen, sink, ring):
    """Per-slot latest-writer rule of int2_oracle.store_windows."""
    prefix = seq - qlen
    out = []
    for idx in range(sink + ring):
        pos = idx if idx < sink else seq - 1 - ((seq - 1 - (idx - sink)) % ring)
        if pos >= prefix and pos < seq and qlen > 0 and (idx < sink or pos >= sink):
            out.append((idx, pos))
    return out


def test_window_store_visits_each_slots_latest_writer_once():
    for sink in (0, 1, 4, 16):
        for ring in (1, 3, 8, 32):
            for seq in range(0, 90):
                for qlen in sorted({0, 1, 2, 3, 5, 8, 17, 40, seq}):
                    if qlen > seq:
                        continue
                    got = window_positions_visited(seq, qlen, sink, ring)
                    assert len({idx for idx, _ in got}) == len(got)  # no slot written twice
                    assert sorted(got) == window_positions_reference(seq, qlen, sink, ring), (
                        sink, ring, seq, qlen)
