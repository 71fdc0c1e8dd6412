// Definitions shared by the INT2 history attention kernels (attention.cu and
// history_mtp.cu: mma.sync with register-built operands; history_f8.cu: tcgen05 with
// 8-bit operands): launch parameters, task decoding (reference
// oscar_ascend/kernels.py:290-330) and the per-token byte tables of the four bf16 key
// levels (mma.sync kernels).
#pragma once

#include "common.cuh"

namespace oscar {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kTwo24 = 16777216.0f;
constexpr float kRescaleSlack = 3.0f;  // lazily re-base the running max (p <= 2^3)

struct HistParams {
  const __nv_bfloat16 *query;  // rotated query rows, unit inner stride
  int64_t qs0, qs1;
  const uint8_t *history;
  const int32_t *qstarts, *seq_lens, *table, *counts, *tasks, *task_count;
  int32_t num_tasks;
  float *partials;  // [n, Hq, split_slots, 256]
  float *lse;       // [n, Hq, split_slots]
  int32_t split_slots;
  int32_t splits;
  oscar_geometry geo;
  float scale_log2;
  // launch shape
  int32_t heads_per_cta;  // HPC
  int32_t ntiles;         // 8-row n-tiles per head
  int32_t units;          // HPC * ntiles
  int32_t warps_per_unit; // R_tok
  int32_t consumers;      // units * warps_per_unit
  int32_t chunk_tokens;   // CT
  int32_t stage_bytes;
  int32_t *status;        // nullable error word
  // balanced splits (decode path): a request of L history tokens uses
  // clamp(ceil(L / span), 1, splits) splits, span = max(kMinSplitTokens,
  // total history * head groups / target_ctas); empty splits write only lse = -inf
  int32_t balanced;
  int32_t target_ctas;
  // test hook (oscar_test_set_wait_fault): CTA 0 never issues the copy of this chunk / tile
  // (-1: none); every bounded device wait gives up after wait_probes probes
  int32_t withhold;
  uint32_t wait_probes;
};

constexpr int kMinSplitTokens = 1024;

struct TaskInfo {
  bool live;
  int req, qoff, qstart, qlen, prefix, sink_len, recent_begin;
};

OSCAR_DEVINL TaskInfo load_task(int task, const int32_t *tasks, const int32_t *task_count,
                                const int32_t *qstarts, const int32_t *seq_lens, const int32_t *counts,
                                const oscar_geometry &g) {
  TaskInfo ti{};
  ti.live = task < task_count[0];
  if (!ti.live) return ti;
  ti.req = tasks[2 * task];
  ti.qoff = tasks[2 * task + 1];
  ti.qstart = qstarts[ti.req];
  const int qend = min(qstarts[ti.req + 1], counts[1]);
  ti.qlen = qend - ti.qstart;
  const int seq = seq_lens[ti.req];
  ti.prefix = seq - ti.qlen;
  ti.sink_len = min(g.sink, ti.prefix);
  ti.recent_begin = max(ti.sink_len, ti.prefix - g.recent);
  return ti;
}

// The four bf16 key levels v_c = bf16(c*s + z) of one token as an fp16 byte table for
// PRMT: levels scaled by 2^e (max |v| in [2^14, 2^15)), which fp16 holds exactly (a
// level smaller than 2^-31 max |v| may lose low bits).  lo = low bytes of the four
// halves, hi = high bytes, so selector nibbles (c, 4 + c) fetch level c.  inv = 2^-e.
struct KeyLut {
  uint32_t lo, hi;
  float inv;
};

OSCAR_DEVINL KeyLut key_lut(uint32_t sz) {
  const float s = half_bits_to_float(sz & 0xffffu), z = half_bits_to_float(sz >> 16);
  const float v0 = round_bf16(z);
  const float v1 = round_bf16(__fadd_rn(s, z));
  const float v2 = round_bf16(__fadd_rn(2.f * s, z));
  const float v3 = round_bf16(__fadd_rn(3.f * s, z));
  // s >= 2^-14 for every written slot, so the levels increase and max |v| is at an end
  const uint32_t ex = (__float_as_uint(fmaxf(fabsf(v0), fabsf(v3))) >> 23) & 0xffu;
  const uint32_t exc = ex < 16u ? 16u : ex;  // unwritten slots (masked later) stay finite
  // 2^(141 - ex) scales [2^(ex-127), 2^(ex-126)) to [2^14, 2^15)
  const float up = __uint_as_float((268u - exc) << 23);
  const uint32_t h01 = pack_half2(v0 * up, v1 * up), h23 = pack_half2(v2 * up, v3 * up);
  KeyLut k;
  k.lo = prmt(h01, h23, 0x6420u);
  k.hi = prmt(h01, h23, 0x7531u);
  k.inv = __uint_as_float((exc - 14u) << 23);
  return k;
}

// PRMT selectors: for codes in bits 0-1 of each byte of x, x * 0x11 + 0x40404040 holds
// the nibbles (c0, 4 + c0, c1, 4 + c1) in its low half and (c2, 4 + c2, c3, 4 + c3) in
// its high half; (c, 4 + c) fetches level c from (lo, hi).

// Query operands of one 8-row n-tile for the fp16 key MMAs, in the contraction order
// the key tables are read in (lane t owns dims [64t, 64t+64); k16-step j = 4w + p covers
// dims 16(4t+w) + {p, 4+p} in the first register and 16(4t+w) + {8+p, 12+p} in the
// second):
//  * qf: q * 2^e in fp16 (row max scaled into [2^14, 2^15)), exact for bf16 queries;
//  * qm: 2^-e * log2(e) * softmax scale of the rows 2t, 2t+1 this lane accumulates.
struct QueryFrags {
  uint32_t qf[16][2];
  float qm[2];
};

OSCAR_DEVINL void load_query_frags(QueryFrags &Q, const __nv_bfloat16 *qrow, bool valid, float scale_log2) {
  const int lane = threadIdx.x & 31, t = lane & 3;
  uint32_t w[32];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 v = valid ? *reinterpret_cast<const uint4 *>(qrow + 64 * t + 8 * c) : make_uint4(0, 0, 0, 0);
    w[4 * c] = v.x, w[4 * c + 1] = v.y, w[4 * c + 2] = v.z, w[4 * c + 3] = v.w;
  }
  auto dim = [&](int d) {  // bf16 value of local dim d (0..63)
    const uint32_t word = w[d >> 1];
    return bf16_bits_to_float((d & 1) ? (word >> 16) : (word & 0xffffu));
  };
  float amax = 0.f;
#pragma unroll
  for (int d = 0; d < 64; ++d) amax = fmaxf(amax, fabsf(dim(d)));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const uint32_t ex = (__float_as_uint(amax) >> 23) & 0xffu;
  const uint32_t exc = ex < 16u ? 16u : ex;
  const bool any = amax > 0.f;
  const float up = any ? __uint_as_float((268u - exc) << 23) : 0.f;
  const float down = any ? __uint_as_float((exc - 14u) << 23) * scale_log2 : 0.f;
#pragma unroll
  for (int wd = 0; wd < 4; ++wd)
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int d = 16 * wd + p;
      Q.qf[4 * wd + p][0] = pack_half2(dim(d) * up, dim(d + 4) * up);
      Q.qf[4 * wd + p][1] = pack_half2(dim(d + 8) * up, dim(d + 12) * up);
    }
  // down is a row-gi value on all four t lanes; the S fragment needs rows 2t, 2t+1.
  Q.qm[0] = __shfl_sync(0xffffffffu, down, 8 * t);
  Q.qm[1] = __shfl_sync(0xffffffffu, down, 8 * t + 4);
}

// 8-bit tcgen05 history kernel (history_f8.cu): up to 8 query rows per KV head (decode),
// persistent CTAs (at most `sm_count`); OSCAR_ERR_UNSUPPORTED for other geometries.
int history_f8_launch(const HistParams &P, int32_t num_tasks, int sm_count, cudaStream_t stream, int priority);

// History kernel for 9..24 query rows per KV head (MTP verify; history_mtp.cu): four
// warps per KV head build every key and value operand once for all the head's rows.
// OSCAR_ERR_UNSUPPORTED for other row counts and for more than 4 KV heads.
int history_mtp_launch(HistParams P, int32_t num_tasks, cudaStream_t stream, int priority);

}  // namespace oscar
