// Exact percentile clip + INT2 quantise + pack of D=256 vectors, two per warp.
//
// The arithmetic reproduces the reference oracle bit for bit (tests/oracle.py:6-21 with
// kernels.py:104-137 byte order):
//   thr   = torch.quantile(|x|, ratio) = lerp(asc[lo], asc[hi], w) as a CPU fused
//           multiply-add (w < .5 ? fma(w, b-a, a) : fma(w-1, b-a, b)), or max|x|*factor
//   x     = min(max(x, -thr), thr)
//   zero  = fp16_rn(min x), scale = fp16_rn(max((max x - min x) / 3, 2^-14))
//   code  = clamp(trunc((x - zero) / scale + 0.5), 0, 3), IEEE ops, no contraction; an
//           infinite or NaN quotient (zero or scale beyond fp16) converts to INT_MIN on
//           the reference's x86 host, i.e. code 0
//   bytes = codes LSB-first, 4 per byte; then scale, zero as little-endian fp16.
// The order statistics are found exactly by counting passes over the 15-bit magnitude
// keys of the (bf16-valued) inputs, with warp-wide integer reductions.
#pragma once

#include "common.cuh"

namespace oscar {

// ----------------------------------------------------------------------------
// Two vectors per warp, on the bf16 values as they are stored: lanes 0-15 quantise
// vector A, lanes 16-31 vector B; lane l = lane & 15 owns dims [16l, 16l+16) as eight
// bf16 pairs (element 2i in the low half of word i), computed with packed bf16x2
// compares:
//  * order statistics: counts of magnitudes >= t, two per compare, added as exact small
//    integers in bf16 (count_ge_bf16);
//  * min / max of the clipped vector: min / max of the raw values, then clipped (the
//    clip is monotone; with a factor below 1 every value may lie above thr);
//  * codes: the reference code of a value, clamp(trunc(RN(RN(RN(x - z) / s) + 0.5)),
//    0, 3) of the clipped x, is a non-decreasing function of the bf16 input x, so
//    code(x) = #{c in 1..3 : x >= B_c} with B_c the smallest bf16 of code >= c
//    (code_boundaries).  Three packed compares then give the codes of two values.
// The per-half sums of the bisection share one warp reduction (the upper half's count
// is carried in the high 16 bits); min / max reductions stay inside each half.
// ----------------------------------------------------------------------------
// sh = 16 on the upper half's lanes, 0 on the lower half's (half_shift()).
OSCAR_DEVINL uint32_t half_shift() { return (threadIdx.x & 16u); }
OSCAR_DEVINL uint32_t half_sum(uint32_t c, uint32_t sh) {
  const uint32_t total = __reduce_add_sync(0xffffffffu, c << sh);
  return (total >> sh) & 0xffffu;
}

OSCAR_DEVINL float half_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

OSCAR_DEVINL float half_min(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

OSCAR_DEVINL uint32_t half_umax(uint32_t v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

OSCAR_DEVINL __nv_bfloat162 as_bf2(uint32_t u) { return *reinterpret_cast<const __nv_bfloat162 *>(&u); }
OSCAR_DEVINL uint32_t bf2_bits(__nv_bfloat162 b) { return *reinterpret_cast<const uint32_t *>(&b); }

// Number of the lane's 16 magnitudes (non-negative bf16, packed in pairs) >= the 15-bit
// key t.  For non-negative bf16 bit patterns, value order is integer order (a NaN
// pattern t compares false everywhere, so t = 0x7fff counts nothing).  Each compare
// gives 1.0 / 0.0 per half; two accumulators start at 32 (exact up to 36 in bf16), their
// sum lies in [64, 72] and the sum of both halves in [128, 144], where 128 + n has n in
// its low 7 bits.
OSCAR_DEVINL uint32_t count_ge_bf16(const uint32_t (&mag)[8], uint32_t t) {
  const __nv_bfloat162 T = as_bf2(t * 0x00010001u);
  __nv_bfloat162 a0 = as_bf2(0x42004200u), a1 = a0;  // 32.0
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    a0 = __hadd2(a0, __hge2(as_bf2(mag[i]), T));
    a1 = __hadd2(a1, __hge2(as_bf2(mag[i + 1]), T));
  }
  const uint32_t s = bf2_bits(__hadd2(a0, a1));
  return bf2_bits(__hadd2(as_bf2(s), as_bf2(prmt(s, 0u, 0x1032u)))) & 0x7fu;
}

// k-th largest (1-indexed) 15-bit key of each half's 256 magnitudes.  A key is a bf16
// magnitude: exponent in bits 7-14, mantissa in bits 0-6.  The binade of the answer is
// found first by counting keys >= e << 7 for e = the half's largest exponent and below
// (usually one or two probes); the 7 mantissa bits follow by bisection.  A half that
// has not found its binade after 4 probes falls back to a 15-bit bisection.  Both
// halves run the same number of counting steps (their counts share each reduction).
// *count receives the number of keys >= the result.
OSCAR_DEVINL uint32_t half_kth_largest_bf16(const uint32_t (&mag)[8], int k, uint32_t *count) {
  __nv_bfloat162 m2 = __hmax2(__hmax2(as_bf2(mag[0]), as_bf2(mag[1])), __hmax2(as_bf2(mag[2]), as_bf2(mag[3])));
  m2 = __hmax2(m2, __hmax2(__hmax2(as_bf2(mag[4]), as_bf2(mag[5])), __hmax2(as_bf2(mag[6]), as_bf2(mag[7]))));
  const uint32_t mb = bf2_bits(m2);
  const int e = (int)(half_umax(max(mb & 0xffffu, mb >> 16)) >> 7);
  const uint32_t sh = half_shift();
  bool found = false;
  uint32_t v = 0, cv = 256;
#pragma unroll 1
  for (int p = 0; p < 4; ++p) {
    const uint32_t t = (uint32_t)max(e - p, 0) << 7;
    const uint32_t c = half_sum(count_ge_bf16(mag, t), sh);
    if (!found && c >= (uint32_t)k) {
      found = true;
      v = t;
      cv = c;
    }
    if (__all_sync(0xffffffffu, found)) break;
  }
  if (__all_sync(0xffffffffu, found)) {
    // the usual case: both halves know their binade; the 7 mantissa bits, unrolled
#pragma unroll
    for (int b = 6; b >= 0; --b) {
      const uint32_t t = v | (1u << b);
      const uint32_t c = half_sum(count_ge_bf16(mag, t), sh);
      if (c >= (uint32_t)k) {
        v = t;
        cv = c;
      }
    }
    *count = cv;
    return v;
  }
  const int nb = found ? 7 : 15;
  const int steps = __reduce_max_sync(0xffffffffu, (unsigned)nb);
#pragma unroll 1
  for (int s = 0; s < steps; ++s) {
    const int b = nb - 1 - s;
    const uint32_t t = b >= 0 ? (v | (1u << b)) : 0x7fffu;  // 0x7fff: counts nothing
    const uint32_t c = half_sum(count_ge_bf16(mag, t), sh);
    if (c >= (uint32_t)k && b >= 0) {
      v = t;
      cv = c;
    }
  }
  *count = cv;
  return v;
}

// The reference's code test for c >= 1: trunc(RN(RN(RN(y - z) / s) + 0.5)) >= c, i.e.
// RN(RN(RN(y - z) / s) + 0.5) >= c (y, z, s finite, s > 0).
OSCAR_DEVINL bool code_at_least(float y, float zf, float sf, int c) {
  return __fadd_rn(__fdiv_rn(__fsub_rn(y, zf), sf), 0.5f) >= (float)c;
}

// Order-preserving index of a bf16 pattern (-0 directly below +0) and its inverse.
OSCAR_DEVINL uint32_t bf16_order(uint32_t b) { return (b & 0x8000u) ? (0x7fffu - (b & 0x7fffu)) : (b + 0x8000u); }
OSCAR_DEVINL uint32_t bf16_from_order(uint32_t k) { return k >= 0x8000u ? (k - 0x8000u) : (0x8000u | (0x7fffu - k)); }

constexpr uint32_t kBf16None = 0x7fc0u;  // NaN: no value compares >=
constexpr uint32_t kBf16All = 0xff80u;   // -inf: every (non-NaN) value compares >=

// B_c (c = 1, 2, 3) as bf16 patterns for the half's vector: the smallest bf16 x whose
// code (clipped to [lo, hi] as the data are) is >= c.  The three IEEE roundings of the
// code test are inverted through their midpoints, exactly, in fp64 (no division):
//  * RN(q + 0.5) >= c  <=>  q >= Q_c, with Q_1 = 0.5 - 2^-25, Q_2 = 1.5, Q_3 = 2.5;
//  * RN(d / s) >= Q    <=>  d / s >= m(Q) (> when Q is odd), m(Q) = (Q^- + Q) / 2 with
//    Q^- the float below Q, so D = the smallest float >= s m(Q) (exact product);
//  * RN(y - z) >= D    <=>  y >= z + m(D) (> when D is odd), and B_c = the smallest bf16
//    >= z + m(D) (next one up when equal and D is odd).
// z + m(D) is exact in fp64 unless it spans more than 53 bits; the candidate is then
// checked by the exact test at B_c and at the bf16 below it (one division per lane,
// lanes 0-5 of the half), and a bisection over all bf16 values takes over if the check
// fails.  Every code is >= c when lo's is (B_c = -inf) and none when hi's is below c,
// or when z or s is not finite: the reference then converts an infinite or NaN quotient
// to int32, which gives INT_MIN on the x86 host (code 0).
OSCAR_DEVINL void code_boundaries(float lo, float hi, float zf, float sf, uint32_t (&B)[3]) {
  const int lane = threadIdx.x & 31, l = lane & 15, base = lane & 16;
  const int cl = l % 3 + 1;  // lanes 0-2: B_c, lanes 3-5: the bf16 below B_c
  const float q = cl == 1 ? __uint_as_float(0x3effffffu) : (cl == 2 ? 1.5f : 2.5f);
  const double mq = ((double)__uint_as_float(__float_as_uint(q) - 1u) + (double)q) * 0.5;
  const double sm = (double)sf * mq;
  float d = __double2float_ru(sm);
  if (cl == 1 && (double)d == sm) d = __uint_as_float(__float_as_uint(d) + 1u);  // Q_1 is odd
  const double md = ((double)__uint_as_float(__float_as_uint(d) - 1u) + (double)d) * 0.5;
  const double y = (double)zf + md;
  const uint32_t fb = __float_as_uint(__double2float_ru(y));
  uint32_t bb = fb >> 16;                                   // smallest bf16 >= the float:
  if ((fb & 0xffffu) != 0u && (fb >> 31) == 0u) bb += 1u;   // positive: round up
  if ((__float_as_uint(d) & 1u) && (double)__uint_as_float(bb << 16) == y)
    bb = bf16_from_order(bf16_order(bb) + 1u);              // strict: the next one up
  // the check: each of lanes 0-7 evaluates one point
  uint32_t pt = bb;
  if (l >= 3 && l < 6) pt = bf16_from_order(bf16_order(bb) - 1u);
  float yv = __uint_as_float(pt << 16);
  if (l == 6) yv = lo;
  if (l >= 7) yv = hi;
  const float r = __fadd_rn(__fdiv_rn(__fsub_rn(yv, zf), sf), 0.5f);
  const bool pass = l < 3 ? r >= (float)cl : r < (float)cl;
  const uint32_t bal = __ballot_sync(0xffffffffu, pass) >> base;
  const float rlo = __shfl_sync(0xffffffffu, r, base + 6);
  const float rhi = __shfl_sync(0xffffffffu, r, base + 7);
  const bool bad = !isfinite(zf) || !isfinite(sf);
  bool need = false;
#pragma unroll
  for (int c = 1; c <= 3; ++c) {
    const uint32_t cand = __shfl_sync(0xffffffffu, bb, base + c - 1);
    const bool ok = ((bal >> (c - 1)) & 1u) && ((bal >> (c + 2)) & 1u);
    if (bad || rhi < (float)c) {
      B[c - 1] = kBf16None;
    } else if (rlo >= (float)c) {
      B[c - 1] = kBf16All;
    } else if (ok) {
      B[c - 1] = cand;
    } else {
      B[c - 1] = 0u;
      need = true;
    }
  }
  if (__any_sync(0xffffffffu, need)) {
    // bisection over the order of all finite bf16 values (-max .. +max), per lane
#pragma unroll
    for (int c = 1; c <= 3; ++c) {
      if (B[c - 1] != 0u || bad || rhi < (float)c || rlo >= (float)c) continue;
      uint32_t a = 0x0080u, b = 0xff80u;  // [a, b): b = one past +max (none)
#pragma unroll 1
      for (int it = 0; it < 17 && a < b; ++it) {
        const uint32_t m = (a + b) >> 1;
        if (code_at_least(__uint_as_float(bf16_from_order(m) << 16), zf, sf, c))
          b = m;
        else
          a = m + 1u;
      }
      B[c - 1] = a >= 0xff80u ? kBf16None : bf16_from_order(a);
    }
  }
}

// w: the lane's 16 bf16 values (pairs).  Writes 4 code bytes per lane and, from lane 0
// of the half, scale / zero -- only when `write` (the half still takes part in the
// reductions otherwise).  Both halves must use the same clip settings.
OSCAR_DEVINL void quantize_pack_half(const uint32_t (&w)[8], const oscar_clip &clip, uint8_t *dst, bool write) {
  const int l = threadIdx.x & 15;
  uint32_t mag[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mag[i] = w[i] & 0x7fff7fffu;
  float thr = INFINITY;
  if (clip.enabled) {
    if (clip.mode == 1) {
      __nv_bfloat162 m2 = as_bf2(mag[0]);
#pragma unroll
      for (int i = 1; i < 8; ++i) m2 = __hmax2(m2, as_bf2(mag[i]));
      const uint32_t mb = bf2_bits(m2);
      thr = __fmul_rn(__uint_as_float(half_umax(max(mb & 0xffffu, mb >> 16)) << 16), clip.factor);
    } else {
      const int k_hi = 256 - clip.asc_hi;
      uint32_t ge = 0;
      const uint32_t hi_key = half_kth_largest_bf16(mag, k_hi, &ge);
      uint32_t lo_key = hi_key;
      if (clip.asc_lo != clip.asc_hi) {
        // the next order statistic: hi_key again when it occurs more than k_hi times,
        // else the largest key below it
        const __nv_bfloat162 H = as_bf2(hi_key * 0x00010001u);
        __nv_bfloat162 b2 = as_bf2(0u);
#pragma unroll
        for (int i = 0; i < 8; ++i) b2 = __hmax2(b2, as_bf2(mag[i] & __hlt2_mask(as_bf2(mag[i]), H)));
        const uint32_t bb = bf2_bits(b2);
        const uint32_t below = half_umax(max(bb & 0xffffu, bb >> 16));
        if (ge < (uint32_t)(k_hi + 1)) lo_key = below;
      }
      const float a = __uint_as_float(lo_key << 16);
      const float b = __uint_as_float(hi_key << 16);
      const float d = __fsub_rn(b, a);
      thr = clip.weight < 0.5f ? __fmaf_rn(clip.weight, d, a) : __fmaf_rn(__fsub_rn(clip.weight, 1.0f), d, b);
    }
  }
  __nv_bfloat162 mn = as_bf2(w[0]), mx = mn;
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    mn = __hmin2(mn, as_bf2(w[i]));
    mx = __hmax2(mx, as_bf2(w[i]));
  }
  const uint32_t mnb = bf2_bits(mn), mxb = bf2_bits(mx);
  float lo = half_min(fminf(bf16_bits_to_float(mnb & 0xffffu), bf16_bits_to_float(mnb >> 16)));
  float hi = half_max(fmaxf(bf16_bits_to_float(mxb & 0xffffu), bf16_bits_to_float(mxb >> 16)));
  if (clip.enabled) {  // min / max of the clipped values: the clipped min / max
    lo = fminf(fmaxf(lo, -thr), thr);
    hi = fmaxf(fminf(hi, thr), -thr);
  }
  const uint16_t zero_h = float_to_half_bits(lo);
  const uint16_t scale_h = float_to_half_bits(fmaxf(__fdiv_rn(__fsub_rn(hi, lo), 3.0f), 6.103515625e-05f));
  uint32_t B[3];
  code_boundaries(lo, hi, half_bits_to_float(zero_h), half_bits_to_float(scale_h), B);
  const __nv_bfloat162 B1 = as_bf2(B[0] * 0x00010001u), B2 = as_bf2(B[1] * 0x00010001u),
                       B3 = as_bf2(B[2] * 0x00010001u);
  // pair i: codes of elements 2i, 2i+1 in bits 0-1 and 16-17 (B_1 <= B_2 <= B_3, so
  // the three masks are nested: bit 0 = m1 ^ m2 ^ m3, bit 1 = m2)
  uint32_t u[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __nv_bfloat162 x = as_bf2(w[i]);
    const uint32_t m1 = __hge2_mask(x, B1), m2 = __hge2_mask(x, B2), m3 = __hge2_mask(x, B3);
    // the masks are all-ones or all-zeros per half, so the code bits go straight to
    // their packed position: bit 0 (m1 ^ m2 ^ m3) and bit 1 (m2) of element pair i
    const uint32_t lo_bit = 0x00010001u << (4 * (i & 3)), hi_bit = 0x00020002u << (4 * (i & 3));
    u[i >> 2] |= ((m1 ^ m2 ^ m3) & lo_bit) | (m2 & hi_bit);
  }
  // element 2i at bit 4i, element 2i+1 at bit 16 + 4i -> 4i + 2
  const uint32_t packed = ((u[0] | (u[0] >> 14)) & 0xffffu) | (((u[1] | (u[1] >> 14)) & 0xffffu) << 16);
  if (write) {
    reinterpret_cast<uint32_t *>(dst)[l] = packed;
    if (l == 0) *reinterpret_cast<uint32_t *>(dst + kDataBytes) = (uint32_t)scale_h | ((uint32_t)zero_h << 16);
  }
}

}  // namespace oscar
