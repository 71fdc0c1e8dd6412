// Exact percentile clip + INT2 quantise + pack of one D=256 vector per warp.
//
// Each lane owns dims [8*lane, 8*lane+8).  The arithmetic reproduces the reference
// oracle bit for bit (tests/oracle.py:6-21 with kernels.py:104-137 byte order):
//   thr   = torch.quantile(|x|, ratio) = lerp(asc[lo], asc[hi], w) as a CPU fused
//           multiply-add (w < .5 ? fma(w, b-a, a) : fma(w-1, b-a, b)), or max|x|*factor
//   x     = min(max(x, -thr), thr)
//   zero  = fp16_rn(min x), scale = fp16_rn(max((max x - min x) / 3, 2^-14))
//   code  = clamp(trunc((x - zero) / scale + 0.5), 0, 3), IEEE ops, no contraction
//   bytes = codes LSB-first, 4 per byte; then scale, zero as little-endian fp16.
// The order statistics are found exactly by a bisection over the 15-bit magnitude
// keys of the (bf16-valued) inputs, with warp-wide integer reductions.
#pragma once

#include "common.cuh"

namespace oscar {

// k-th largest (1-indexed) 15-bit key among the 256 keys of the warp.
OSCAR_DEVINL uint32_t warp_kth_largest(const uint32_t (&key)[8], int k) {
  uint32_t v = 0;
#pragma unroll 1
  for (int b = 14; b >= 0; --b) {
    const uint32_t t = v | (1u << b);
    uint32_t c = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) c += key[i] >= t ? 1u : 0u;
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= (uint32_t)k) v = t;
  }
  return v;
}

// Quantise the warp's vector x (fp32 copies of bf16 values) and write the 68-byte
// packed vector at dst (only when `write`; the warp still participates otherwise).
OSCAR_DEVINL void quantize_pack_warp(float (&x)[8], const oscar_clip &clip, uint8_t *dst, bool write) {
  const int lane = threadIdx.x & 31;
  if (clip.enabled) {
    float thr;
    if (clip.mode == 1) {
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(x[i]));
      thr = __fmul_rn(warp_max(m), clip.factor);
    } else {
      uint32_t key[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) key[i] = (__float_as_uint(x[i]) & 0x7fffffffu) >> 16;
      const int k_hi = 256 - clip.asc_hi;  // rank of the larger interpolation point
      const uint32_t hi_key = warp_kth_largest(key, k_hi);
      uint32_t lo_key = hi_key;
      if (clip.asc_lo != clip.asc_hi) {
        uint32_t ge = 0, below = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          ge += key[i] >= hi_key ? 1u : 0u;
          if (key[i] < hi_key) below = max(below, key[i]);
        }
        ge = __reduce_add_sync(0xffffffffu, ge);
        below = __reduce_max_sync(0xffffffffu, below);
        if (ge < (uint32_t)(k_hi + 1)) lo_key = below;
      }
      const float a = __uint_as_float(lo_key << 16);
      const float b = __uint_as_float(hi_key << 16);
      const float d = __fsub_rn(b, a);
      thr = clip.weight < 0.5f ? __fmaf_rn(clip.weight, d, a) : __fmaf_rn(__fsub_rn(clip.weight, 1.0f), d, b);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = fminf(fmaxf(x[i], -thr), thr);
  }
  float lo = x[0], hi = x[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    lo = fminf(lo, x[i]);
    hi = fmaxf(hi, x[i]);
  }
  lo = warp_min(lo);
  hi = warp_max(hi);
  const uint16_t zero_h = float_to_half_bits(lo);
  const uint16_t scale_h = float_to_half_bits(fmaxf(__fdiv_rn(__fsub_rn(hi, lo), 3.0f), 6.103515625e-05f));
  const float zf = half_bits_to_float(zero_h);
  const float sf = half_bits_to_float(scale_h);
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float q = __fadd_rn(__fdiv_rn(__fsub_rn(x[i], zf), sf), 0.5f);
    int c = (int)q;  // truncation toward zero (torch .to(int32))
    c = min(max(c, 0), 3);
    packed |= (uint32_t)c << (2 * i);
  }
  if (write) {
    reinterpret_cast<uint16_t *>(dst)[lane] = (uint16_t)packed;
    if (lane == 0) *reinterpret_cast<uint32_t *>(dst + kDataBytes) = (uint32_t)scale_h | ((uint32_t)zero_h << 16);
  }
}

// ----------------------------------------------------------------------------
// Two vectors per warp: lanes 0-15 quantise vector A, lanes 16-31 vector B; lane
// l = lane & 15 owns dims [16l, 16l+16).  Same arithmetic as quantize_pack_warp; the
// per-half sums of the bisection share one warp reduction (the upper half's count is
// carried in the high 16 bits), and the min / max reductions stay inside each half.
// ----------------------------------------------------------------------------
OSCAR_DEVINL uint32_t half_sum(uint32_t c) {
  const bool upper = (threadIdx.x & 16) != 0;
  const uint32_t total = __reduce_add_sync(0xffffffffu, upper ? (c << 16) : c);
  return upper ? (total >> 16) : (total & 0xffffu);
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

// Number of the 16 keys >= t, as four independent partial sums (short dependency chains).
OSCAR_DEVINL uint32_t count_ge16(const uint32_t (&key)[16], uint32_t t) {
  uint32_t c[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 16; ++i) c[i & 3] += key[i] >= t ? 1u : 0u;
  return (c[0] + c[1]) + (c[2] + c[3]);
}

// k-th largest (1-indexed) 15-bit key of each half's 256 keys.  A key is a bf16
// magnitude: exponent in bits 7-14, mantissa in bits 0-6.  The binade of the answer is
// found first by counting keys >= e << 7 for e = the half's largest exponent and below
// (usually one or two probes); the 7 mantissa bits follow by bisection.  A half that
// has not found its binade after 4 probes falls back to a 15-bit bisection.  Both
// halves run the same number of counting steps (their counts share each reduction).
OSCAR_DEVINL uint32_t half_kth_largest(const uint32_t (&key)[16], int k) {
  uint32_t m4[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 16; ++i) m4[i & 3] = max(m4[i & 3], key[i]);
  const int e = (int)(half_umax(max(max(m4[0], m4[1]), max(m4[2], m4[3]))) >> 7);
  bool found = false;
  uint32_t v = 0;
#pragma unroll 1
  for (int p = 0; p < 4; ++p) {
    const uint32_t t = (uint32_t)max(e - p, 0) << 7;
    const uint32_t c = half_sum(count_ge16(key, t));
    if (!found && c >= (uint32_t)k) {
      found = true;
      v = t;
    }
    if (__all_sync(0xffffffffu, found)) break;
  }
  const int nb = found ? 7 : 15;
  const int steps = __reduce_max_sync(0xffffffffu, (unsigned)nb);
#pragma unroll 1
  for (int s = 0; s < steps; ++s) {
    const int b = nb - 1 - s;
    const uint32_t t = b >= 0 ? (v | (1u << b)) : 0xffffffffu;  // no key reaches 0xffffffff
    if (half_sum(count_ge16(key, t)) >= (uint32_t)k && b >= 0) v = t;
  }
  return v;
}

// x: the lane's 16 values (fp32 copies of bf16).  Writes 4 code bytes per lane and,
// from lane 0 of the half, scale / zero -- only when `write` (the half still takes
// part in the reductions otherwise).  Both halves must use the same clip settings.
OSCAR_DEVINL void quantize_pack_half(float (&x)[16], const oscar_clip &clip, uint8_t *dst, bool write) {
  const int l = threadIdx.x & 15;
  if (clip.enabled) {
    float thr;
    if (clip.mode == 1) {
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(x[i]));
      thr = __fmul_rn(half_max(m), clip.factor);
    } else {
      uint32_t key[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) key[i] = (__float_as_uint(x[i]) & 0x7fffffffu) >> 16;
      const int k_hi = 256 - clip.asc_hi;
      const uint32_t hi_key = half_kth_largest(key, k_hi);
      uint32_t lo_key = hi_key;
      if (clip.asc_lo != clip.asc_hi) {
        uint32_t b4[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (key[i] < hi_key) b4[i & 3] = max(b4[i & 3], key[i]);
        const uint32_t ge = half_sum(count_ge16(key, hi_key));
        const uint32_t below = half_umax(max(max(b4[0], b4[1]), max(b4[2], b4[3])));
        if (ge < (uint32_t)(k_hi + 1)) lo_key = below;
      }
      const float a = __uint_as_float(lo_key << 16);
      const float b = __uint_as_float(hi_key << 16);
      const float d = __fsub_rn(b, a);
      thr = clip.weight < 0.5f ? __fmaf_rn(clip.weight, d, a) : __fmaf_rn(__fsub_rn(clip.weight, 1.0f), d, b);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = fminf(fmaxf(x[i], -thr), thr);
  }
  float lo4[4] = {x[0], x[1], x[2], x[3]}, hi4[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
  for (int i = 4; i < 16; ++i) {
    lo4[i & 3] = fminf(lo4[i & 3], x[i]);
    hi4[i & 3] = fmaxf(hi4[i & 3], x[i]);
  }
  float lo = half_min(fminf(fminf(lo4[0], lo4[1]), fminf(lo4[2], lo4[3])));
  float hi = half_max(fmaxf(fmaxf(hi4[0], hi4[1]), fmaxf(hi4[2], hi4[3])));
  const uint16_t zero_h = float_to_half_bits(lo);
  const uint16_t scale_h = float_to_half_bits(fmaxf(__fdiv_rn(__fsub_rn(hi, lo), 3.0f), 6.103515625e-05f));
  const float zf = half_bits_to_float(zero_h);
  const float sf = half_bits_to_float(scale_h);
  // code = trunc(RN(RN((x - z) / s) + 0.5)).  The quotient is taken as d * RN(1/s),
  // within 4e-7 of the IEEE quotient for |d / s| <= 3.01, so the truncation agrees
  // whenever q lies more than 1e-5 from an integer; otherwise (and for q < 0) the
  // IEEE division is done.
  const float inv = __frcp_rn(sf);
  uint32_t pk[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float d = __fsub_rn(x[i], zf);
    float q = __fadd_rn(__fmul_rn(d, inv), 0.5f);
    if (fabsf(__fsub_rn(__fsub_rn(q, truncf(q)), 0.5f)) > 0.49999f) q = __fadd_rn(__fdiv_rn(d, sf), 0.5f);
    int c = (int)q;  // truncation toward zero (torch .to(int32))
    c = min(max(c, 0), 3);
    pk[i & 3] |= (uint32_t)c << (2 * i);
  }
  const uint32_t packed = (pk[0] | pk[1]) | (pk[2] | pk[3]);
  if (write) {
    reinterpret_cast<uint32_t *>(dst)[l] = packed;
    if (l == 0) *reinterpret_cast<uint32_t *>(dst + kDataBytes) = (uint32_t)scale_h | ((uint32_t)zero_h << 16);
  }
}

}  // namespace oscar
