// Paged split-KV decode attention over the OSCAR cache (reference
// oscar_ascend/kernels.py:290-482), split LSE merge (:485-511), path merge (:514-541),
// BF16 window store (:544-620) and the compact task table (:222-287).
//
// History kernel (INT2, rotated space).  One CTA = one (task, split, head group).
// The warps stream chunks of the paged K stripe (at most one 128-token kernel block)
// into a 3- or 4-stage shared-memory ring with 1-D bulk copies (cp.async.bulk, mbarrier
// completion; contiguous [chunk tokens x heads x 160 B] runs, no multicast); the copy
// of chunk c + stages - 1 is issued by warp c % warps after its part of chunk c (there
// is no separate producer warp).  The warps own (KV head,
// 8 query rows) units and two 16-token m-tiles each.  Narrow launches (all KV heads x
// row tiles in 4 warps) run 3 CTAs per SM at <= 168 registers, wider ones 8 warps per
// CTA at up to 255 registers.
//
// Keys: the reference rounds the dequantised key to bf16, so a token's 256 key
// elements take only its four levels v_c = bf16(c*s + z).  Each token gets an 8-byte
// table of those levels in fp16 (scaled by a power of two, which keeps them exact);
// one PRMT whose selector nibbles come from one IMAD of two codes turns them into an
// fp16 MMA operand register, and m16n8k16 MMAs against the (also power-of-two scaled,
// exact) fp16 query give q.k_bf16 in fp32.  Values: sum_t p_t v_t =
// sum_t (p_t s_t) c_t + sum_t p_t z_t; the 2-bit codes enter the fp16 MMA as
// subnormals: one AND of a packed word with 0x00030003 << 2p leaves the fp16 values
// c * 4^p * 2^-24 exactly, and the output is multiplied back by 4^p.  The contraction
// dimension is permuted (a bijection over the 256 dims) so that each lane reads only
// its own 16 bytes of a token vector; the query fragments use the same permutation.
// MMAs use the swapped orientation (tokens / dims as M = 16, query rows as N = 8).
#include <algorithm>
#include <cstdlib>
#include <atomic>
#include <mutex>

#include "history_common.cuh"
#include "tasks.cuh"
#include "rowgemm.cuh"

namespace oscar {

constexpr int kMaxConsumerWarps = 8;  // wider CTAs spill the O accumulator
// Narrow launch (every KV head x row tile of a task fits in 4 warps, e.g. decode with
// 4 KV heads): 4-warp CTAs at <= 168 registers, 3 resident per SM (12 warps instead of
// 8 hide more of the operand-building latency).
constexpr int kNarrowWarps = 4;
constexpr int kNarrowCtasPerSm = 3;
// Middle launch (all KV heads x row tiles of a task in at most 12 warps, e.g. MTP verify
// with 3 row tiles x 4 KV heads): one 12-warp CTA per SM at <= 170 registers, every KV
// head in the CTA so each chunk is one contiguous copy.
constexpr int kMidWarps = 12;
template <int MAXW, int NM, int STAGES, int MINB>
__global__ void __launch_bounds__(32 * MAXW, MINB) history_attention_kernel(HistParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const oscar_geometry &g = P.geo;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int task = blockIdx.x, split = blockIdx.y;
  const int h0 = blockIdx.z * P.heads_per_cta;
  const TaskInfo ti = load_task(task, P.tasks, P.task_count, P.qstarts, P.seq_lens, P.counts, g);
  if (!ti.live || ti.qlen <= 0) return;
  const int rows_valid = min(g.query_tile, ti.qoff < ti.qlen ? ti.qlen - ti.qoff : 0) * g.group;
  const int length = ti.recent_begin - ti.sink_len;
  const int tiles = (length + 31) / 32;
  int nsplit = P.splits;
  if (P.balanced) {
    __shared__ int s_span;
    if (warp == 0) {
      int64_t total = 0;
      const int nt = min(P.task_count[0], P.num_tasks);
      for (int t2 = lane; t2 < nt; t2 += 32) {
        const TaskInfo tj = load_task(t2, P.tasks, P.task_count, P.qstarts, P.seq_lens, P.counts, g);
        if (tj.live && tj.qlen > 0) total += max(0, tj.recent_begin - tj.sink_len);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
      if (lane == 0) {
        const int64_t span = (total * gridDim.z + P.target_ctas - 1) / max(P.target_ctas, 1);
        s_span = (int)(span < kMinSplitTokens ? (int64_t)kMinSplitTokens : (span > (1 << 30) ? (int64_t)(1 << 30) : span));
      }
    }
    __syncthreads();
    nsplit = max(1, min(P.splits, (length + s_span - 1) / s_span));
  }
  const int per_split = (tiles + nsplit - 1) / nsplit;
  const int begin = split * per_split * 32;
  const int end = min((split + 1) * per_split * 32, length);
  const int lo = ti.sink_len + begin, hi = ti.sink_len + max(end, begin);  // absolute positions
  if (P.balanced && hi <= lo) {
    // unused split of a balanced launch: only the lse marker (the merge skips it)
    for (int i = threadIdx.x; i < P.heads_per_cta * rows_valid; i += blockDim.x) {
      const int hl = i / rows_valid, row = i % rows_valid;
      const int tok = ti.qstart + ti.qoff + row / g.group;
      const int qh = (h0 + hl) * g.group + row % g.group;
      P.lse[((int64_t)tok * g.kv_heads * g.group + qh) * P.split_slots + split] = -INFINITY;
    }
    return;
  }
  const int CT = P.chunk_tokens;
  const int first_chunk = lo / CT;
  const int nchunks = hi > lo ? (hi - 1) / CT - first_chunk + 1 : 0;

  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + STAGES;
  uint8_t *stages = smem + 128;
  __shared__ int32_t s_abort;  // any warp's wait gave up: the CTA's partials are not valid
  __shared__ int32_t s_stage_chunk[STAGES];  // last chunk whose copy went into each stage
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], P.consumers);
    }
    s_abort = 0;
    for (int s = 0; s < STAGES; ++s) s_stage_chunk[s] = -1;
    fence_mbarrier_init();
  }
  __syncthreads();

  const int hpc = P.heads_per_cta;
  const int token_bytes = hpc * g.slot_bytes;
  // Copies: thread 0 issues chunks 0 .. STAGES-2; then, after its own part of chunk c,
  // warp c % consumers issues chunk c + STAGES - 1 into the stage chunk c - 1 used
  // (bounded wait for its release).  Rotating the issuer keeps any one warp from being
  // the slowest of the CTA, which every stage release waits for.
  const int32_t *trow = P.table + (int64_t)ti.req * g.table_stride;
  auto issue_one = [&](int c) {
    const int s = c % STAGES;
    const int pos = (first_chunk + c) * CT;
    const int64_t slot0 = (int64_t)trow[pos / kKernelBlock] * kKernelBlock + pos % kKernelBlock;
    const uint8_t *src = P.history + (slot0 / g.block_tokens) * g.page_bytes +
                         ((slot0 % g.block_tokens) * g.kv_heads + h0) * (int64_t)g.slot_bytes;
    if (c == P.withhold && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) return;  // test hook
    const uint32_t dst = smem_u32(stages + s * P.stage_bytes);
    s_stage_chunk[s] = c;
    mbar_arrive_expect_tx(&full[s], CT * token_bytes);
    if (hpc == g.kv_heads) {
      bulk_copy_g2s(dst, src, CT * token_bytes, &full[s]);
    } else {
      for (int tk = 0; tk < CT; ++tk)
        bulk_copy_g2s(dst + tk * token_bytes, src + (int64_t)tk * g.kv_heads * g.slot_bytes, token_bytes, &full[s]);
    }
  };
  if (warp >= P.consumers) return;
  if (threadIdx.x == 0)
    for (int c = 0; c < min(STAGES - 1, nchunks); ++c) issue_one(c);

  // ---------------- consumer warps ----------------
  const int unit = warp % P.units, sub = warp / P.units;
  const int head_local = unit / P.ntiles, ntile = unit % P.ntiles;
  const int head = h0 + head_local;
  const int gi = lane >> 2, t = lane & 3;
  // query row of this thread's B fragment: row index r = 8*ntile + gi
  const int r_mine = 8 * ntile + gi;
  const bool rvalid = r_mine < rows_valid;
  const int qtok = ti.qstart + ti.qoff + r_mine / g.group;
  const int qhead = head * g.group + r_mine % g.group;
  QueryFrags Q;
  load_query_frags(Q, P.query + (int64_t)qtok * P.qs0 + (int64_t)qhead * P.qs1, rvalid, P.scale_log2);

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f}, zp_run[2] = {0.f, 0.f};
  bool ok = true;

#pragma unroll 1
  for (int c = 0; c < nchunks && ok; ++c) {
    const int s = c % STAGES;
    if (!mbar_wait_bounded(&full[s], (c / STAGES) & 1, P.wait_probes)) {
      ok = false;
      if (lane == 0) {
        atomicExch(&s_abort, 1);
        if (P.status) atomicExch(P.status, OSCAR_ERR_TIMEOUT);
      }
      break;
    }
    const uint8_t *stage = stages + s * P.stage_bytes;
    const int cpos = (first_chunk + c) * CT;
    // this warp's NM consecutive 16-token m-tiles of the chunk
    const int mt0 = sub * NM;
    if (cpos + 16 * (mt0 + NM) > lo && cpos + 16 * mt0 < hi) {  // warp-uniform
      const uint8_t *tl[NM];
      bool va[NM], vb[NM];
#pragma unroll
      for (int j = 0; j < NM; ++j) {
        const int tpos = cpos + 16 * (mt0 + j);
        tl[j] = stage + (16 * (mt0 + j)) * token_bytes + head_local * g.slot_bytes;
        va[j] = tpos + gi >= lo && tpos + gi < hi;
        vb[j] = tpos + gi + 8 >= lo && tpos + gi + 8 < hi;
      }
      // ---- S^T (tokens x rows) on fp16 tensor cores.  Each 2-bit key code becomes its
      // bf16 level (exact in fp16 after the token's power-of-two scale) through the
      // token's byte table: one PRMT turns two codes into an MMA operand register. ----
      uint32_t kaw[NM][4], kbw[NM][4];
      KeyLut lA[NM], lB[NM];
      uint32_t vsz[NM][2];
      static_assert(NM == 2, "one key table per lane covers two 16-token m-tiles");
      {
        // lane 4gi + 2j + h builds the table of token (m-tile j, row gi + 8h) once; the
        // four lanes of row group gi fetch the four tables they use
        const uint8_t *own = ((t >> 1) ? tl[1] : tl[0]) + (gi + 8 * (t & 1)) * token_bytes;
        const KeyLut mine = key_lut(*reinterpret_cast<const uint32_t *>(own + 64));
#pragma unroll
        for (int j = 0; j < NM; ++j) {
          const int la = 4 * gi + 2 * j;
          lA[j].lo = __shfl_sync(0xffffffffu, mine.lo, la);
          lA[j].hi = __shfl_sync(0xffffffffu, mine.hi, la);
          lA[j].inv = __shfl_sync(0xffffffffu, mine.inv, la);
          lB[j].lo = __shfl_sync(0xffffffffu, mine.lo, la + 1);
          lB[j].hi = __shfl_sync(0xffffffffu, mine.hi, la + 1);
          lB[j].inv = __shfl_sync(0xffffffffu, mine.inv, la + 1);
        }
      }
#pragma unroll
      for (int j = 0; j < NM; ++j) {
        const uint8_t *ra = tl[j] + gi * token_bytes, *rb = ra + 8 * token_bytes;
        const uint4 ka = *reinterpret_cast<const uint4 *>(ra + 16 * t);
        const uint4 kb = *reinterpret_cast<const uint4 *>(rb + 16 * t);
        kaw[j][0] = ka.x, kaw[j][1] = ka.y, kaw[j][2] = ka.z, kaw[j][3] = ka.w;
        kbw[j][0] = kb.x, kbw[j][1] = kb.y, kbw[j][2] = kb.z, kbw[j][3] = kb.w;
        vsz[j][0] = *reinterpret_cast<const uint32_t *>(ra + g.vector_bytes + 64);
        vsz[j][1] = *reinterpret_cast<const uint32_t *>(rb + g.vector_bytes + 64);
      }
      float sc[NM][2][4];  // [m-tile][chain (even / odd code position)][fragment]
#pragma unroll
      for (int j = 0; j < NM; ++j)
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[j][u][e] = 0.f;
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) {
#pragma unroll
        for (int p = 0; p < 4; ++p) {
#pragma unroll
          for (int j = 0; j < NM; ++j) {
            // codes of position p of the four bytes, in bits 0-1 of each byte; one IMAD
            // gives the PRMT selectors of bytes (0, 1) in its low and (2, 3) in its high half
            const uint32_t xa = (kaw[j][wd] >> (2 * p)) & 0x03030303u;
            const uint32_t xb = (kbw[j][wd] >> (2 * p)) & 0x03030303u;
            const uint32_t sa = xa * 0x11u + 0x40404040u, sb = xb * 0x11u + 0x40404040u;
            const uint32_t a0 = prmt(lA[j].lo, lA[j].hi, sa);
            const uint32_t a1 = prmt(lB[j].lo, lB[j].hi, sb);
            const uint32_t a2 = prmt(lA[j].lo, lA[j].hi, sa >> 16);
            const uint32_t a3 = prmt(lB[j].lo, lB[j].hi, sb >> 16);
            mma_f16_16816(sc[j][p & 1], a0, a1, a2, a3, Q.qf[4 * wd + p][0], Q.qf[4 * wd + p][1]);
          }
        }
      }
      // ---- logits (log2 domain) ----
      float lg[NM][4];
#pragma unroll
      for (int j = 0; j < NM; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float dot = sc[j][0][e] + sc[j][1][e];
          const float mul = (e < 2 ? lA[j].inv : lB[j].inv) * Q.qm[e & 1];
          lg[j][e] = ((e < 2) ? va[j] : vb[j]) ? dot * mul : -INFINITY;
        }
      }
      // ---- online softmax over the warp's 16*NM tokens, lazy re-basing ----
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < NM; ++j) {
        mx[0] = fmaxf(mx[0], fmaxf(lg[j][0], lg[j][2]));
        mx[1] = fmaxf(mx[1], fmaxf(lg[j][1], lg[j][3]));
      }
#pragma unroll
      for (int o2 = 4; o2 <= 16; o2 <<= 1) {
        mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], o2));
        mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], o2));
      }
      const bool need0 = mx[0] > m_run[0] + kRescaleSlack || (m_run[0] == -INFINITY && mx[0] > -INFINITY);
      const bool need1 = mx[1] > m_run[1] + kRescaleSlack || (m_run[1] == -INFINITY && mx[1] > -INFINITY);
      if (__any_sync(0xffffffffu, need0 || need1)) {
        const float a0 = need0 ? (m_run[0] == -INFINITY ? 0.f : ex2(m_run[0] - mx[0])) : 1.f;
        const float a1 = need1 ? (m_run[1] == -INFINITY ? 0.f : ex2(m_run[1] - mx[1])) : 1.f;
        if (need0) m_run[0] = mx[0];
        if (need1) m_run[1] = mx[1];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o[i][0] *= a0, o[i][1] *= a1, o[i][2] *= a0, o[i][3] *= a1;
        }
        l_run[0] *= a0, l_run[1] *= a1, zp_run[0] *= a0, zp_run[1] *= a1;
      }
      const float ms0 = m_run[0] == -INFINITY ? 0.f : m_run[0];
      const float ms1 = m_run[1] == -INFINITY ? 0.f : m_run[1];
      uint32_t pb[NM][2];
#pragma unroll
      for (int j = 0; j < NM; ++j) {
        const float p0 = ex2(lg[j][0] - ms0), p1 = ex2(lg[j][1] - ms1);
        const float p2 = ex2(lg[j][2] - ms0), p3 = ex2(lg[j][3] - ms1);
        const float vsA = va[j] ? half_bits_to_float(vsz[j][0] & 0xffffu) : 0.f;
        const float vzA = va[j] ? half_bits_to_float(vsz[j][0] >> 16) : 0.f;
        const float vsB = vb[j] ? half_bits_to_float(vsz[j][1] & 0xffffu) : 0.f;
        const float vzB = vb[j] ? half_bits_to_float(vsz[j][1] >> 16) : 0.f;
        l_run[0] += p0 + p2;
        l_run[1] += p1 + p3;
        zp_run[0] = fmaf(p0, vzA, fmaf(p2, vzB, zp_run[0]));
        zp_run[1] = fmaf(p1, vzA, fmaf(p3, vzB, zp_run[1]));
        // P'^T fragments: (token, row) -> transposed to (row, token)
        pb[j][0] = movmatrix_trans(pack_half2(p0 * vsA, p1 * vsA));
        pb[j][1] = movmatrix_trans(pack_half2(p2 * vsB, p3 * vsB));
      }
      // ---- O^T += Vc^T . P'^T (dims x rows) ----
#pragma unroll
      for (int j = 0; j < NM; ++j) {
        const uint8_t *vt = tl[j] + g.vector_bytes;
        uint32_t vw[4][2];  // [token 2t,2t+1,2t+8,2t+9][word 2gi, 2gi+1]
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int tok = 2 * t + (q & 1) + (q >> 1) * 8;
          const uint32_t *src = reinterpret_cast<const uint32_t *>(vt + tok * token_bytes) + 2 * gi;
          vw[q][0] = src[0];
          vw[q][1] = src[1];
        }
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          // bytes (2hb, 2hb+1) of token a in the low half, of token b in the high half
          const uint32_t sel = hb ? 0x7632u : 0x5410u;
          const uint32_t x0 = prmt(vw[0][0], vw[1][0], sel);  // word 2gi, tokens 2t,2t+1
          const uint32_t x1 = prmt(vw[0][1], vw[1][1], sel);  // word 2gi+1
          const uint32_t x2 = prmt(vw[2][0], vw[3][0], sel);  // word 2gi, tokens 2t+8,2t+9
          const uint32_t x3 = prmt(vw[2][1], vw[3][1], sel);
          const uint32_t y0 = x0 >> 8, y1 = x1 >> 8, y2 = x2 >> 8, y3 = x3 >> 8;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const uint32_t msk = 0x00030003u << (2 * p);
            mma_f16_16816(o[4 * (2 * hb) + p], x0 & msk, x1 & msk, x2 & msk, x3 & msk, pb[j][0], pb[j][1]);
            mma_f16_16816(o[4 * (2 * hb + 1) + p], y0 & msk, y1 & msk, y2 & msk, y3 & msk, pb[j][0], pb[j][1]);
          }
        }
      }
    }
    {
      // copy issue rotates over the warps: after its part of chunk c, warp c % consumers
      // issues chunk c + STAGES - 1 into the stage that chunk c - 1 used
      const int cn = c + STAGES - 1;
      int good = 1;
      if (warp == c % P.consumers && lane == 0 && cn < nchunks) {
        if (cn >= STAGES && !mbar_wait_bounded(&empty[cn % STAGES], ((cn / STAGES) - 1) & 1, P.wait_probes)) {
          good = 0;
          atomicExch(&s_abort, 1);
          if (P.status) atomicExch(P.status, OSCAR_ERR_TIMEOUT);
        } else {
          issue_one(cn);
        }
      }
      if (!__shfl_sync(0xffffffffu, good, 0)) ok = false;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---------------- combine the warps of a unit, write the partial ----------------
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 4);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 8);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 16);
    zp_run[r] += __shfl_xor_sync(0xffffffffu, zp_run[r], 4);
    zp_run[r] += __shfl_xor_sync(0xffffffffu, zp_run[r], 8);
    zp_run[r] += __shfl_xor_sync(0xffffffffu, zp_run[r], 16);
  }
  // every consumer warp is past its last stage read; reuse the stage ring
  asm volatile("bar.sync 1, %0;" ::"r"(P.consumers * 32));
  if (*reinterpret_cast<volatile int32_t *>(&s_abort) != 0) {
    // an aborted loop may leave copies in flight: no warp issues any more, so the last
    // chunk copied into each stage is final; let those land before the ring is reused
    // and the CTA exits
    if (threadIdx.x == 0)
      for (int s = 0; s < STAGES; ++s) {
        const int cc = s_stage_chunk[s];
        if (cc >= 0) (void)mbar_wait_bounded(&full[s], (cc / STAGES) & 1, P.wait_probes);
      }
    asm volatile("bar.sync 1, %0;" ::"r"(P.consumers * 32));
  }
  // exchange area over the stage ring: one record (O^T fragment + running max) per
  // non-leader warp, then l / zp of every consumer warp
  float *xch = reinterpret_cast<float *>(stages);
  constexpr int kSlot = 16 * 4 * 32 + 2 * 32;  // floats per warp record
  if (sub > 0) {
    float *rec = xch + (size_t)(warp - P.units) * kSlot;
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q) rec[(i * 4 + q) * 32 + lane] = o[i][q];
    rec[2048 + lane] = m_run[0];
    rec[2048 + 32 + lane] = m_run[1];
  }
  float *aux = xch + (size_t)(P.consumers - P.units) * kSlot;  // [warp][4][32]
  aux[(warp * 4 + 0) * 32 + lane] = l_run[0];
  aux[(warp * 4 + 1) * 32 + lane] = l_run[1];
  aux[(warp * 4 + 2) * 32 + lane] = zp_run[0];
  aux[(warp * 4 + 3) * 32 + lane] = zp_run[1];
  asm volatile("bar.sync 1, %0;" ::"r"(P.consumers * 32));
  if (sub > 0) return;
  const bool aborted = *reinterpret_cast<volatile int32_t *>(&s_abort) != 0;
  float mtot[2] = {m_run[0], m_run[1]};
  for (int w2 = warp + P.units; w2 < P.consumers; w2 += P.units) {
    const float *rec = xch + (size_t)(w2 - P.units) * kSlot;
    mtot[0] = fmaxf(mtot[0], rec[2048 + lane]);
    mtot[1] = fmaxf(mtot[1], rec[2048 + 32 + lane]);
  }
  float f0 = m_run[0] == -INFINITY ? 0.f : ex2(m_run[0] - mtot[0]);
  float f1 = m_run[1] == -INFINITY ? 0.f : ex2(m_run[1] - mtot[1]);
  float L[2] = {l_run[0] * f0, l_run[1] * f1}, Z[2] = {zp_run[0] * f0, zp_run[1] * f1};
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] *= f0, o[i][1] *= f1, o[i][2] *= f0, o[i][3] *= f1;
  for (int w2 = warp + P.units; w2 < P.consumers; w2 += P.units) {
    const float *rec = xch + (size_t)(w2 - P.units) * kSlot;
    const float mw0 = rec[2048 + lane], mw1 = rec[2048 + 32 + lane];
    const float e0 = mw0 == -INFINITY ? 0.f : ex2(mw0 - mtot[0]);
    const float e1 = mw1 == -INFINITY ? 0.f : ex2(mw1 - mtot[1]);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] = fmaf(e0, rec[(i * 4 + 0) * 32 + lane], o[i][0]);
      o[i][1] = fmaf(e1, rec[(i * 4 + 1) * 32 + lane], o[i][1]);
      o[i][2] = fmaf(e0, rec[(i * 4 + 2) * 32 + lane], o[i][2]);
      o[i][3] = fmaf(e1, rec[(i * 4 + 3) * 32 + lane], o[i][3]);
    }
    L[0] = fmaf(e0, aux[(w2 * 4 + 0) * 32 + lane], L[0]);
    L[1] = fmaf(e1, aux[(w2 * 4 + 1) * 32 + lane], L[1]);
    Z[0] = fmaf(e0, aux[(w2 * 4 + 2) * 32 + lane], Z[0]);
    Z[1] = fmaf(e1, aux[(w2 * 4 + 3) * 32 + lane], Z[1]);
  }
  // rows of this thread: 8*ntile + 2t + {0,1}; dims 32gi + {0..15} and 32gi + 16 + {0..15}
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = 8 * ntile + 2 * t + r;
    if (row >= rows_valid) continue;
    const int tok = ti.qstart + ti.qoff + row / g.group;
    const int qh = head * g.group + row % g.group;
    const int64_t orow = ((int64_t)tok * g.kv_heads * g.group + qh) * P.split_slots + split;
    // an aborted CTA marks its rows empty (-inf) so no merge reads a partial sum
    const bool any = L[r] > 0.f && !aborted;
    // lse (natural log): m is in log2 units
    if (gi == 0) P.lse[orow] = any ? (mtot[r] * 0.69314718055994531f + logf(L[r])) : -INFINITY;
    if (!any && (P.balanced || aborted)) continue;  // the merge skips -inf splits without reading them
    const float inv = any ? 1.0f / L[r] : 0.f;
    const float zterm = any ? Z[r] * inv : 0.f;
    float *dst = P.partials + orow * kDim + 32 * gi;
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int mv = 4 * q4 + e;  // dim offset delta = mv, position p = e
          const float mul = kTwo24 / (float)(1 << (2 * e));
          v[e] = fmaf(o[mv][2 * half + r] * mul, inv, zterm);
        }
        *reinterpret_cast<float4 *>(dst + 16 * half + 4 * q4) = make_float4(v[0], v[1], v[2], v[3]);
      }
  }
}

// ----------------------------------------------------------------------------
// BF16 raw path: sink + recent (window) + causal current tokens, one split.
// One CTA = (task, KV head, 8-row n-tile); 4 warps split the token list.
// ----------------------------------------------------------------------------
struct RawParams {
  const __nv_bfloat16 *query;
  int64_t qs0, qs1;
  const __nv_bfloat16 *key, *value;
  int64_t ks0, ks1, vs0, vs1;
  const __nv_bfloat16 *window;
  const int32_t *qstarts, *seq_lens, *table, *counts, *tasks, *task_count;
  float *partials, *lse;
  int32_t split_slots, split_index;
  oscar_geometry geo;
  float scale_log2;
  int32_t ntiles;
};

constexpr int kRawWarps = 4;
constexpr int kRawSmem = kRawWarps * 2 * 16 * kDim * 2;  // per warp K and V 16-token tiles

OSCAR_DEVINL const __nv_bfloat16 *raw_token_row(const RawParams &P, const TaskInfo &ti, int64_t owner,
                                                int idx, int kv, int head) {
  // idx-th token of the raw list: sink | prefix recent | current
  const oscar_geometry &g = P.geo;
  const int nprev = ti.sink_len + ti.prefix - ti.recent_begin;
  if (idx < nprev) {
    const int pos = idx < ti.sink_len ? idx : ti.recent_begin + idx - ti.sink_len;
    return P.window + window_elem_offset(owner, window_index(pos, g), kv, head, g);
  }
  const int cur = ti.qstart + idx - nprev;
  return kv == 0 ? P.key + (int64_t)cur * P.ks0 + (int64_t)head * P.ks1
                 : P.value + (int64_t)cur * P.vs0 + (int64_t)head * P.vs1;
}

__global__ void __launch_bounds__(32 * kRawWarps) raw_attention_kernel(RawParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const oscar_geometry &g = P.geo;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gi = lane >> 2, t = lane & 3;
  const int task = blockIdx.x, head = blockIdx.y, ntile = blockIdx.z;
  const TaskInfo ti = load_task(task, P.tasks, P.task_count, P.qstarts, P.seq_lens, P.counts, g);
  if (!ti.live || ti.qlen <= 0) return;
  const int rows_valid = min(g.query_tile, ti.qlen - ti.qoff) * g.group;
  if (8 * ntile >= rows_valid) return;
  const int nprev = ti.sink_len + ti.prefix - ti.recent_begin;
  const int total = nprev + ti.qlen;
  const int64_t owner = (int64_t)P.table[(int64_t)ti.req * g.table_stride] / (g.block_tokens / kKernelBlock);
  // query fragment (unrotated bf16), row r = 8*ntile + gi
  const int r_mine = 8 * ntile + gi;
  const bool rvalid = r_mine < rows_valid;
  const int qi_mine = ti.qoff + r_mine / g.group;
  const __nv_bfloat16 *qrow = P.query + (int64_t)(ti.qstart + qi_mine) * P.qs0 +
                              (int64_t)(head * g.group + r_mine % g.group) * P.qs1;
  uint32_t qf[16][2];
#pragma unroll
  for (int js = 0; js < 16; ++js) {
    qf[js][0] = rvalid ? *reinterpret_cast<const uint32_t *>(qrow + 16 * js + 2 * t) : 0u;
    qf[js][1] = rvalid ? *reinterpret_cast<const uint32_t *>(qrow + 16 * js + 8 + 2 * t) : 0u;
  }
  // causal limit for rows 2t, 2t+1 (query index of the row)
  int qlim[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = 8 * ntile + 2 * t + r;
    qlim[r] = ti.prefix + ti.qoff + row / g.group;
  }
  __nv_bfloat16 *sk = reinterpret_cast<__nv_bfloat16 *>(smem) + warp * 2 * 16 * kDim;
  __nv_bfloat16 *sv = sk + 16 * kDim;
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
#pragma unroll 1
  for (int base = 16 * warp; base < total; base += 16 * kRawWarps) {
    // stage 16 K and V rows (swizzled 16-byte chunks)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int c = lane + 32 * i;  // 16 rows x 32 chunks
      const int r = c >> 5, ch = c & 31;
      const int idx = base + r;
      __nv_bfloat16 *dk = sk + r * kDim + ((ch ^ (r & 7)) << 3);
      __nv_bfloat16 *dv = sv + r * kDim + ((ch ^ (r & 7)) << 3);
      if (idx < total) {
        cp_async_16(smem_u32(dk), raw_token_row(P, ti, owner, idx, 0, head) + ch * 8);
        cp_async_16(smem_u32(dv), raw_token_row(P, ti, owner, idx, 1, head) + ch * 8);
      } else {
        *reinterpret_cast<uint4 *>(dk) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(dv) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int js = 0; js < 16; ++js) {
      uint32_t a[4];
      const int row = lane & 15, k = 16 * js + (lane >> 4) * 8;
      ldmatrix_x4(a, smem_u32(sk + row * kDim + (((k >> 3) ^ (row & 7)) << 3)));
      mma_bf16_16816(sc, a[0], a[1], a[2], a[3], qf[js][0], qf[js][1]);
    }
    // positions of tokens gi, gi+8
    float lg[4];
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
      const int idx = base + gi + 8 * hb;
      int pos;
      if (idx < ti.sink_len) pos = idx;
      else if (idx < nprev) pos = ti.recent_begin + idx - ti.sink_len;
      else pos = ti.prefix + idx - nprev;
      const bool ok = idx < total;
#pragma unroll
      for (int r = 0; r < 2; ++r)
        lg[2 * hb + r] = (ok && pos <= qlim[r]) ? sc[2 * hb + r] * P.scale_log2 : -INFINITY;
    }
    float mx[2] = {fmaxf(lg[0], lg[2]), fmaxf(lg[1], lg[3])};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 4));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 8));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 16));
    }
    float a[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mn = fmaxf(m_run[r], mx[r]);
      a[r] = (m_run[r] == -INFINITY) ? 0.f : ex2(m_run[r] - mn);
      m_run[r] = mn;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] *= a[0], o[i][1] *= a[1], o[i][2] *= a[0], o[i][3] *= a[1];
    const float ms0 = m_run[0] == -INFINITY ? 0.f : m_run[0];
    const float ms1 = m_run[1] == -INFINITY ? 0.f : m_run[1];
    const float p0 = ex2(lg[0] - ms0), p1 = ex2(lg[1] - ms1), p2 = ex2(lg[2] - ms0), p3 = ex2(lg[3] - ms1);
    l_run[0] = l_run[0] * a[0] + p0 + p2;
    l_run[1] = l_run[1] * a[1] + p1 + p3;
    const uint32_t pb0 = movmatrix_trans(pack_bf162(p0, p1));
    const uint32_t pb1 = movmatrix_trans(pack_bf162(p2, p3));
#pragma unroll
    for (int mv = 0; mv < 16; ++mv) {
      uint32_t av[4];
      const int tok = (lane & 7) + ((lane >> 4) << 3);
      const int d = 16 * mv + ((lane >> 3) & 1) * 8;
      ldmatrix_x4_trans(av, smem_u32(sv + tok * kDim + (((d >> 3) ^ (tok & 7)) << 3)));
      mma_bf16_16816(o[mv], av[0], av[1], av[2], av[3], pb0, pb1);
    }
    __syncwarp();
  }
  // combine the 4 warps
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 4);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 8);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 16);
  }
  __syncthreads();
  float *xch = reinterpret_cast<float *>(smem);  // [warp][64 + 4][32]
  float *rec = xch + warp * (68 * 32);
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int q = 0; q < 4; ++q) rec[(i * 4 + q) * 32 + lane] = o[i][q];
  rec[64 * 32 + lane] = m_run[0];
  rec[65 * 32 + lane] = m_run[1];
  rec[66 * 32 + lane] = l_run[0];
  rec[67 * 32 + lane] = l_run[1];
  __syncthreads();
  if (warp != 0) return;
  float M[2] = {-INFINITY, -INFINITY};
  for (int w = 0; w < kRawWarps; ++w) {
    M[0] = fmaxf(M[0], xch[w * 68 * 32 + 64 * 32 + lane]);
    M[1] = fmaxf(M[1], xch[w * 68 * 32 + 65 * 32 + lane]);
  }
  float L[2] = {0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  for (int w = 0; w < kRawWarps; ++w) {
    const float *rw = xch + w * 68 * 32;
    const float mw0 = rw[64 * 32 + lane], mw1 = rw[65 * 32 + lane];
    const float e0 = mw0 == -INFINITY ? 0.f : ex2(mw0 - M[0]);
    const float e1 = mw1 == -INFINITY ? 0.f : ex2(mw1 - M[1]);
    L[0] = fmaf(e0, rw[66 * 32 + lane], L[0]);
    L[1] = fmaf(e1, rw[67 * 32 + lane], L[1]);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] = fmaf(e0, rw[(i * 4 + 0) * 32 + lane], o[i][0]);
      o[i][1] = fmaf(e1, rw[(i * 4 + 1) * 32 + lane], o[i][1]);
      o[i][2] = fmaf(e0, rw[(i * 4 + 2) * 32 + lane], o[i][2]);
      o[i][3] = fmaf(e1, rw[(i * 4 + 3) * 32 + lane], o[i][3]);
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = 8 * ntile + 2 * t + r;
    if (row >= rows_valid) continue;
    const int tok = ti.qstart + ti.qoff + row / g.group;
    const int qh = head * g.group + row % g.group;
    const int64_t orow = ((int64_t)tok * g.kv_heads * g.group + qh) * P.split_slots + P.split_index;
    const bool any = L[r] > 0.f;
    const float inv = any ? 1.0f / L[r] : 0.f;
    float *dst = P.partials + orow * kDim;
    // O^T fragment: m-tile mv rows (dims) 16mv + gi and 16mv + gi + 8
#pragma unroll
    for (int mv = 0; mv < 16; ++mv) {
      dst[16 * mv + gi] = o[mv][r] * inv;
      dst[16 * mv + gi + 8] = o[mv][2 + r] * inv;
    }
    if (gi == 0) P.lse[orow] = any ? (M[r] * 0.69314718055994531f + logf(L[r])) : -INFINITY;
  }
}

// ----------------------------------------------------------------------------
// split merge (reference _merge_splits_kernel): warp per row
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256) merge_splits_kernel(const float *__restrict__ partials,
                                                           const float *__restrict__ lse, int64_t rows,
                                                           int32_t hq, int32_t splits, int32_t slot_stride,
                                                           const int32_t *__restrict__ counts,
                                                           __nv_bfloat16 *__restrict__ out,
                                                           float *__restrict__ logsum) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bool valid = row / hq < counts[1];
  float m = -INFINITY;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, valid ? lse[row * slot_stride + s] : -INFINITY);
  const float safe = m == -INFINITY ? 0.f : m;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float den = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float l = valid ? lse[row * slot_stride + s] : -INFINITY;
    const float w = expf(l - safe);
    den += w;
    if (w != 0.f) {
      const float4 *src = reinterpret_cast<const float4 *>(partials + (row * slot_stride + s) * kDim + lane * 8);
      const float4 x0 = src[0], x1 = src[1];
      acc[0] = fmaf(w, x0.x, acc[0]), acc[1] = fmaf(w, x0.y, acc[1]), acc[2] = fmaf(w, x0.z, acc[2]);
      acc[3] = fmaf(w, x0.w, acc[3]), acc[4] = fmaf(w, x1.x, acc[4]), acc[5] = fmaf(w, x1.y, acc[5]);
      acc[6] = fmaf(w, x1.z, acc[6]), acc[7] = fmaf(w, x1.w, acc[7]);
    }
  }
  const float inv = 1.0f / fmaxf(den, 1e-30f);
  uint4 o;
  o.x = pack_bf162(acc[0] * inv, acc[1] * inv);
  o.y = pack_bf162(acc[2] * inv, acc[3] * inv);
  o.z = pack_bf162(acc[4] * inv, acc[5] * inv);
  o.w = pack_bf162(acc[6] * inv, acc[7] * inv);
  *reinterpret_cast<uint4 *>(out + row * kDim + lane * 8) = o;
  if (lane == 0) logsum[row] = den > 0.f ? m + logf(fmaxf(den, 1e-30f)) : -INFINITY;
}

// path merge (reference _merge_paths_kernel): warp per row
__global__ void __launch_bounds__(256) merge_paths_kernel(const __nv_bfloat16 *__restrict__ a,
                                                          const float *__restrict__ la,
                                                          const float *__restrict__ b, int64_t b_stride,
                                                          const float *__restrict__ lb, int64_t lb_stride,
                                                          int64_t rows, int32_t hq,
                                                          const int32_t *__restrict__ counts,
                                                          __nv_bfloat16 *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bool valid = row / hq < counts[1];
  const float xa = valid ? la[row] : -INFINITY;
  const float xb = valid ? lb[row * lb_stride] : -INFINITY;
  float m = fmaxf(xa, xb);
  m = m == -INFINITY ? 0.f : m;
  const float wa = expf(xa - m), wb = expf(xb - m);
  const float inv = 1.0f / fmaxf(wa + wb, 1e-30f);
  uint4 araw = valid ? *reinterpret_cast<const uint4 *>(a + row * kDim + lane * 8) : make_uint4(0, 0, 0, 0);
  float4 b0 = make_float4(0, 0, 0, 0), b1 = b0;
  if (valid && wb != 0.f) {
    b0 = *reinterpret_cast<const float4 *>(b + row * b_stride + lane * 8);
    b1 = *reinterpret_cast<const float4 *>(b + row * b_stride + lane * 8 + 4);
  }
  const uint32_t aw[4] = {araw.x, araw.y, araw.z, araw.w};
  const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  uint32_t ow[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float r0 = (wa * bf16_bits_to_float(aw[i] & 0xffffu) + wb * bv[2 * i]) * inv;
    const float r1 = (wa * bf16_bits_to_float(aw[i] >> 16) + wb * bv[2 * i + 1]) * inv;
    ow[i] = pack_bf162(r0, r1);
  }
  *reinterpret_cast<uint4 *>(out + row * kDim + lane * 8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

// ----------------------------------------------------------------------------
// fused epilogue of a decode step: split merge -> bf16 hrot -> hrot @ Rv^T (bf16
// rounding, as the reference rotate) -> LSE path merge with the raw partial.
// One CTA = 64 rows of [n*Hq]; the row-tile GEMM core does the inverse rotation.
// ----------------------------------------------------------------------------
struct FinalParams {
  const float *partials, *lse;
  int32_t split_slots, splits;
  int64_t rows;
  int32_t hq;
  const int32_t *counts;
  const __nv_bfloat16 *rv;
  __nv_bfloat16 *out;
};

// 4 output rows per CTA on a 16-row GEMM tile (rows 4..15 of the tile are zero), 4 warps,
// one row each: a decode step (n * Hq rows) spreads over n * Hq / 4 CTAs (the merge is
// latency-bound: a row reads one 1 KB partial per used split, four at a time).
constexpr int kFinRows = 16;
constexpr int kFinLive = 4;
constexpr int kFinThreads = 128;
constexpr int kFinSmem = (kFinRows * kDim + 2 * kBStageElems) * 2 + 2 * kFinRows * 4;

__global__ void __launch_bounds__(kFinThreads) finalize_kernel(FinalParams P) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16 *sA = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *sB = sA + kFinRows * kDim;
  float *s_la = reinterpret_cast<float *>(sB + 2 * kBStageElems);  // [16]
  float *s_lb = s_la + kFinRows;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row0 = (int64_t)blockIdx.x * kFinLive;
  const int32_t active = P.counts[1];
  // zero tile rows 8..15 (16 bytes per thread)
  for (int i = threadIdx.x; i < (kFinRows - kFinLive) * kDim / 8; i += kFinThreads)
    reinterpret_cast<uint4 *>(sA + kFinLive * kDim)[i] = make_uint4(0, 0, 0, 0);
  constexpr int RW = kFinLive / 4;  // rows per warp
  float m[RW], w0[RW], w1[RW], den[RW];
  bool valid[RW];
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    const int64_t row = row0 + warp * RW + i;
    valid[i] = row < P.rows && row / P.hq < active;
    // lane s holds split s's lse (splits <= 64: two per lane); warp max / weights
    const float *lrow = P.lse + row * P.split_slots;
    const float l0 = valid[i] && lane < P.splits ? lrow[lane] : -INFINITY;
    const float l1 = valid[i] && lane + 32 < P.splits ? lrow[lane + 32] : -INFINITY;
    float mm = fmaxf(l0, l1);
#pragma unroll
    for (int o = 16; o; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
    const float safe = mm == -INFINITY ? 0.f : mm;
    w0[i] = expf(l0 - safe), w1[i] = expf(l1 - safe);
    float d = w0[i] + w1[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    m[i] = mm, den[i] = d;
  }
  float macc[RW][8];
#pragma unroll
  for (int i = 0; i < RW; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) macc[i][e] = 0.f;
  // four splits of every row per group: all loads of the group are in flight before any is used
  for (int s0 = 0; s0 < P.splits; s0 += 4) {
    float w[RW][4];
    float4 x[RW][4][2];
#pragma unroll
    for (int i = 0; i < RW; ++i) {
      const int64_t row = row0 + warp * RW + i;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int sp = s0 + u;
        const float ws = __shfl_sync(0xffffffffu, sp < 32 ? w0[i] : w1[i], sp & 31);
        w[i][u] = sp < P.splits ? ws : 0.f;
        if (w[i][u] != 0.f) {
          const float4 *src = reinterpret_cast<const float4 *>(P.partials + (row * P.split_slots + sp) * kDim + lane * 8);
          x[i][u][0] = src[0], x[i][u][1] = src[1];
        } else {
          x[i][u][0] = x[i][u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < RW; ++i)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float wu = w[i][u];
        macc[i][0] = fmaf(wu, x[i][u][0].x, macc[i][0]), macc[i][1] = fmaf(wu, x[i][u][0].y, macc[i][1]);
        macc[i][2] = fmaf(wu, x[i][u][0].z, macc[i][2]), macc[i][3] = fmaf(wu, x[i][u][0].w, macc[i][3]);
        macc[i][4] = fmaf(wu, x[i][u][1].x, macc[i][4]), macc[i][5] = fmaf(wu, x[i][u][1].y, macc[i][5]);
        macc[i][6] = fmaf(wu, x[i][u][1].z, macc[i][6]), macc[i][7] = fmaf(wu, x[i][u][1].w, macc[i][7]);
      }
  }
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    const int r = warp * RW + i;
    const int64_t row = row0 + r;
    const float inv = 1.0f / fmaxf(den[i], 1e-30f);
    uint4 o;
    o.x = pack_bf162(macc[i][0] * inv, macc[i][1] * inv);
    o.y = pack_bf162(macc[i][2] * inv, macc[i][3] * inv);
    o.z = pack_bf162(macc[i][4] * inv, macc[i][5] * inv);
    o.w = pack_bf162(macc[i][6] * inv, macc[i][7] * inv);
    *reinterpret_cast<uint4 *>(sA + r * kDim + ((lane ^ (r & 7)) << 3)) = o;
    if (lane == 0) {
      s_la[r] = den[i] > 0.f ? m[i] + logf(fmaxf(den[i], 1e-30f)) : -INFINITY;
      s_lb[r] = valid[i] ? P.lse[row * P.split_slots + P.splits] : -INFINITY;
    }
  }
  float acc[1][8][4];
  rowgemm_mainloop<1, kFinThreads>(acc, sA, sB, BMatrix{P.rv, 1, 256});  // B(k, n) = Rv[n][k]
  const int wn = warp & 3, gq = lane >> 2, t = lane & 3;
  {
    const int hb = 0;  // tile rows 0..kFinLive-1 are this CTA's rows
    const int r = gq;
    if (r >= kFinLive) return;
    const int64_t row = row0 + r;
    if (row >= P.rows) return;
    const float xa = s_la[r], xb = s_lb[r];
    float m = fmaxf(xa, xb);
    m = m == -INFINITY ? 0.f : m;
    const float wa = expf(xa - m), wb = expf(xb - m);
    const float inv = 1.0f / fmaxf(wa + wb, 1e-30f);
    const float *braw = P.partials + (row * P.split_slots + P.splits) * kDim;
#pragma unroll
    for (int nj = 0; nj < 8; ++nj) {
      const int col = wn * 64 + nj * 8 + 2 * t;
      // hout is rounded to bf16 (the reference rotate writes bf16)
      const float h0 = round_bf16(acc[0][nj][2 * hb]);
      const float h1 = round_bf16(acc[0][nj][2 * hb + 1]);
      float b0 = 0.f, b1 = 0.f;
      if (wb != 0.f) {
        const float2 bb = *reinterpret_cast<const float2 *>(braw + col);
        b0 = bb.x, b1 = bb.y;
      }
      const float r0 = (wa * h0 + wb * b0) * inv, r1 = (wa * h1 + wb * b1) * inv;
      *reinterpret_cast<uint32_t *>(P.out + row * kDim + col) = pack_bf162(r0, r1);
    }
  }
}

// ----------------------------------------------------------------------------
// window store (reference _window_store_kernel): CTA per request, warp per
// (window index, head) pair, 16-byte lanes.
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256) window_store_kernel(const __nv_bfloat16 *__restrict__ key,
                                                           int64_t ks0, int64_t ks1,
                                                           const __nv_bfloat16 *__restrict__ value,
                                                           int64_t vs0, int64_t vs1,
                                                           __nv_bfloat16 *__restrict__ window,
                                                           const int32_t *__restrict__ qstarts,
                                                           const int32_t *__restrict__ seq_lens,
                                                           const int32_t *__restrict__ table,
                                                           const int32_t *__restrict__ counts,
                                                           oscar_geometry g) {
  const int req = blockIdx.x;
  if (req >= counts[0]) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qstart = qstarts[req];
  const int qend = min(qstarts[req + 1], counts[1]);
  const int seq = seq_lens[req];
  const int prefix = seq - (qend - qstart);
  if (qend <= qstart) return;
  const int64_t owner = (int64_t)table[(int64_t)req * g.table_stride] / (g.block_tokens / kKernelBlock);
  // Positions this step writes: sink positions in [prefix, min(seq, S)) and, for the
  // ring, each slot's latest writer, i.e. pos >= S with pos + C >= seq.  Same set as
  // the reference's per-slot latest-writer rule (kernels.py:576-582).
  // Only those positions are visited (a prefill chunk of thousands of tokens writes at
  // most sink + ring of them): sink [lo, min(seq, S)), ring [max(lo, S, seq - C), seq).
  const int lo = max(prefix, 0);
  const int n_sink = max(0, min(seq, g.sink) - lo);
  const int ring_lo = max(max(lo, g.sink), seq - g.ring);
  const int n_ring = max(0, seq - ring_lo);
  const int entries = (n_sink + n_ring) * g.kv_heads;
  for (int e = warp; e < entries; e += 8) {
    const int k = e / g.kv_heads, head = e % g.kv_heads;
    const int pos = k < n_sink ? lo + k : ring_lo + (k - n_sink);
    const int idx = pos < g.sink ? pos : g.sink + pos % g.ring;
    const int cur = qstart + pos - prefix;
    const uint4 kv0 = *reinterpret_cast<const uint4 *>(key + (int64_t)cur * ks0 + (int64_t)head * ks1 + lane * 8);
    const uint4 kv1 = *reinterpret_cast<const uint4 *>(value + (int64_t)cur * vs0 + (int64_t)head * vs1 + lane * 8);
    *reinterpret_cast<uint4 *>(window + window_elem_offset(owner, idx, 0, head, g) + lane * 8) = kv0;
    *reinterpret_cast<uint4 *>(window + window_elem_offset(owner, idx, 1, head, g) + lane * 8) = kv1;
  }
}

// ----------------------------------------------------------------------------
// task table (reference _prepare_tasks_kernel): block 0 builds the table (tasks.cuh);
// other blocks copy page-table columns.
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) prepare_tasks_kernel(const int32_t *__restrict__ qstarts,
                                                             const int32_t *__restrict__ counts,
                                                             int32_t *__restrict__ tasks,
                                                             int32_t *__restrict__ task_count, int32_t capacity,
                                                             int32_t query_tile, const int32_t *__restrict__ src,
                                                             int64_t src_stride, int32_t *__restrict__ dst,
                                                             int64_t dst_stride, int32_t copy_cols) {
  const int nr = counts[0], active = counts[1];
  if (blockIdx.x > 0) {
    const int64_t total = (int64_t)nr * copy_cols;
    for (int64_t i = (int64_t)(blockIdx.x - 1) * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)(gridDim.x - 1) * blockDim.x) {
      const int64_t r = i / copy_cols, c = i % copy_cols;
      dst[r * dst_stride + c] = src[r * src_stride + c];
    }
    return;
  }
  build_task_table(qstarts, nr, active, tasks, task_count, capacity, query_tile);
}

// ----------------------------------------------------------------------------
// launch helpers
// ----------------------------------------------------------------------------
static bool geo_ok(const oscar_geometry &g) {
  return g.head_dim == kDim && g.kv_heads > 0 && g.group > 0 && g.kernel_block == kKernelBlock &&
         g.block_tokens % kKernelBlock == 0 && g.slot_bytes % 16 == 0 && g.vector_bytes == kDataBytes + 4 &&
         g.page_bytes == (int64_t)g.block_tokens * g.kv_heads * kDim * 2 && g.ring > 0 && g.sink >= 0 &&
         g.recent >= 0 && g.query_tile > 0 && g.table_stride > 0;
}

// priority != 0: launch priority of the grid (the decode step gives the history grid the
// device's greatest priority, so a concurrently queued lower-priority grid only takes
// the SM slots that history blocks leave free, i.e. the tail of the last wave)
template <int MAXW, int NM, int STAGES, int MINB>
static int launch_history(const HistParams &P, dim3 grid, size_t smem, cudaStream_t stream, int priority) {
  if (!ensure_dynamic_smem<history_attention_kernel<MAXW, NM, STAGES, MINB>>(smem)) return OSCAR_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(32 * P.consumers);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributePriority;
  attr[0].val.priority = priority;
  cfg.attrs = attr;
  cfg.numAttrs = priority != 0 ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, history_attention_kernel<MAXW, NM, STAGES, MINB>, P) != cudaSuccess)
    return OSCAR_ERR_LAUNCH;
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

// Launch shape: each consumer warp owns one (KV head, 8-row) unit and NM = 2
// consecutive 16-token m-tiles of every chunk; a chunk is all heads of
// 16 * NM * warps_per_unit tokens (at most one 128-token kernel block).
// SM count of the current device (cached per device).
static int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int v = 0;
    cache[dev] = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0 ? v : 148;
  }
  return cache[dev];
}

// The shared-operand MTP kernel serves 9..24 rows per KV head (at most 4 KV heads) by
// default; OSCAR_HISTORY_MTP=0 (read at every launch) sends those launches to
// history_attention_kernel, for comparisons.
static bool history_mtp_enabled() {
  const char *v = getenv("OSCAR_HISTORY_MTP");
  return v == nullptr || v[0] != '0';
}

// The 8-bit tcgen05 kernel (history_f8.cu) is opt-in: OSCAR_HISTORY_F8=1, read at every
// launch.  It is parity-green but slower than history_attention_kernel on config 3
// (1208 against 454 us per launch on B200): its warp roles run one warp per
// sub-partition, each a latency-bound chain over thin (N = 16) tensor-core tiles.
static bool history_f8_enabled() {
  const char *v = getenv("OSCAR_HISTORY_F8");
  return v != nullptr && v[0] == '1';
}

// The history kernel of the latest successful history launch (oscar_last_history_kernel).
static std::atomic<int32_t> g_last_history{0};

// Test hook state (oscar_test_set_wait_fault), read at every history launch.
static std::atomic<int32_t> g_withhold{-1};
static std::atomic<uint32_t> g_wait_probes{kWaitLimit};
int32_t test_hook_withhold() { return g_withhold.load(); }
uint32_t test_hook_wait_probes() { return g_wait_probes.load(); }

static int history_launch(HistParams P, int32_t num_tasks, cudaStream_t stream, int priority = 0) {
  P.withhold = g_withhold.load();
  P.wait_probes = g_wait_probes.load();
  if (history_f8_enabled()) {
    const int rc = history_f8_launch(P, num_tasks, sm_count(), stream, priority);
    if (rc == OSCAR_OK) g_last_history.store(OSCAR_HISTORY_F8_KERNEL);
    if (rc != OSCAR_ERR_UNSUPPORTED) return rc;
  }
  if (history_mtp_enabled()) {
    const int rc = history_mtp_launch(P, num_tasks, stream, priority);
    if (rc == OSCAR_OK) g_last_history.store(OSCAR_HISTORY_MTP_KERNEL);
    if (rc != OSCAR_ERR_UNSUPPORTED) return rc;
  }
  const oscar_geometry &g = P.geo;
  const int rows = g.query_tile * g.group;
  P.ntiles = (rows + 7) / 8;
  if (P.ntiles > kMaxConsumerWarps) return OSCAR_ERR_UNSUPPORTED;
  constexpr int NM = 2;
  const bool narrow = P.ntiles * g.kv_heads <= kNarrowWarps;
  const bool mid = !narrow && P.ntiles * g.kv_heads <= kMidWarps;
  const int max_warps = narrow ? kNarrowWarps : (mid ? kMidWarps : kMaxConsumerWarps);
  int hpc = g.kv_heads;
  while (hpc * P.ntiles > max_warps) hpc = (hpc + 1) / 2;
  if (g.kv_heads % hpc) hpc = 1;
  P.heads_per_cta = hpc;
  P.units = hpc * P.ntiles;
  int wpu = P.units >= max_warps ? 1 : max_warps / P.units;
  while (wpu > 1 && 16 * NM * wpu > kKernelBlock) wpu >>= 1;
  P.warps_per_unit = wpu;
  P.consumers = P.units * wpu;
  P.chunk_tokens = 16 * NM * wpu;
  P.stage_bytes = P.chunk_tokens * hpc * g.slot_bytes;
  const int stages = narrow ? 3 : 4;
  const size_t xch = ((size_t)(P.consumers - P.units) * (16 * 4 * 32 + 2 * 32) + (size_t)P.consumers * 4 * 32) * 4;
  size_t smem = 128 + (size_t)stages * P.stage_bytes;
  if (smem < 128 + xch) smem = 128 + xch;
  if (smem > 227 * 1024) return OSCAR_ERR_UNSUPPORTED;
  dim3 grid(num_tasks, P.splits, g.kv_heads / hpc);
  const int rc = narrow ? launch_history<kNarrowWarps, NM, 3, kNarrowCtasPerSm>(P, grid, smem, stream, priority)
                 : mid    ? launch_history<kMidWarps, NM, 4, 1>(P, grid, smem, stream, priority)
                          : launch_history<kMaxConsumerWarps, NM, 4, 1>(P, grid, smem, stream, priority);
  if (rc == OSCAR_OK) g_last_history.store(OSCAR_HISTORY_ATTENTION_KERNEL);
  return rc;
}

// Side stream of the decode step's BF16 raw path (one per device, created on first use):
// the raw grid is small and latency-bound, so it runs beside the history grid, which
// gets the greatest launch priority; `mu` keeps the fork / launch / join sequence of
// concurrent host callers on one device from interleaving on the shared events.
struct RawSide {
  std::once_flag once;
  std::mutex mu;
  std::atomic<bool> tried{false};
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  int priority = 0;
  bool ok = false;
};

// `caller` is the stream of the call: while it is being captured into a graph and the
// side stream does not exist yet, the call goes without it (creating a stream inside a
// capture could invalidate the capture) and a later eager call creates it.
static RawSide *raw_side(cudaStream_t caller) {
  static RawSide cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  RawSide &c = cache[dev];
  if (!c.tried.load(std::memory_order_acquire)) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(caller, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
      cudaGetLastError();
      return nullptr;
    }
  }
  std::call_once(c.once, [&c] {
    c.tried.store(true, std::memory_order_release);
    int least = 0, greatest = 0;
    if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) return;
    if (cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking) != cudaSuccess) return;
    if (cudaEventCreateWithFlags(&c.fork, cudaEventDisableTiming) != cudaSuccess) return;
    if (cudaEventCreateWithFlags(&c.join, cudaEventDisableTiming) != cudaSuccess) return;
    c.priority = greatest;
    c.ok = true;
  });
  if (!c.ok) cudaGetLastError();  // a failed set-up leaves the single-stream order
  return c.ok ? &c : nullptr;
}

static int raw_launch(const RawParams &P, int32_t num_tasks, cudaStream_t stream) {
  if (!ensure_dynamic_smem<raw_attention_kernel>(kRawSmem)) return OSCAR_ERR_LAUNCH;
  dim3 grid(num_tasks, P.geo.kv_heads, P.ntiles);
  raw_attention_kernel<<<grid, 32 * kRawWarps, kRawSmem, stream>>>(P);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

}  // namespace oscar

using namespace oscar;

extern "C" int oscar_prepare_tasks(const int32_t *qstarts, const int32_t *counts, int32_t *tasks,
                                   int32_t *task_count, int32_t capacity, int32_t max_reqs, int32_t query_tile,
                                   const int32_t *source_table, int64_t source_stride, int32_t *table,
                                   int64_t table_stride, int32_t copy_columns, void *stream) {
  if (!qstarts || !counts || !tasks || !task_count || capacity <= 0 || max_reqs <= 0 || query_tile <= 0)
    return OSCAR_ERR_INVALID;
  if (copy_columns > 0 && (!source_table || !table)) return OSCAR_ERR_INVALID;
  int copy_blocks = 0;
  if (copy_columns > 0) {
    const int64_t total = (int64_t)max_reqs * copy_columns;
    copy_blocks = (int)std::min<int64_t>((total + 1023) / 1024, 1024);
  }
  prepare_tasks_kernel<<<1 + copy_blocks, 1024, 0, (cudaStream_t)stream>>>(
      qstarts, counts, tasks, task_count, capacity, query_tile, source_table, source_stride, table, table_stride,
      copy_columns > 0 ? copy_columns : 0);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_attention_partials(const void *query, int64_t qs0, int64_t qs1, const void *key, int64_t ks0,
                                        int64_t ks1, const void *value, int64_t vs0, int64_t vs1,
                                        const uint8_t *history, const void *window, const int32_t *qstarts,
                                        const int32_t *seq_lens, const int32_t *table, const int32_t *counts,
                                        const int32_t *tasks, const int32_t *task_count, int32_t num_tasks,
                                        int64_t n, float *partials, float *lse, oscar_geometry geo, float scale,
                                        int32_t splits, int32_t raw, int32_t *status, void *stream) {
  if (!geo_ok(geo) || splits <= 0 || num_tasks < 0 || n < 0) return OSCAR_ERR_INVALID;
  if (n == 0 || num_tasks == 0) return OSCAR_OK;
  if (!query || !qstarts || !seq_lens || !table || !counts || !tasks || !task_count || !partials || !lse)
    return OSCAR_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(query) & 15) || qs0 % 8 || qs1 % 8) return OSCAR_ERR_INVALID;
  if (raw) {
    if (splits != 1 || !key || !value || !window) return OSCAR_ERR_INVALID;
    if (((reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value)) & 15) || ks0 % 8 || ks1 % 8 ||
        vs0 % 8 || vs1 % 8)
      return OSCAR_ERR_INVALID;
    RawParams P{};
    P.query = reinterpret_cast<const __nv_bfloat16 *>(query);
    P.qs0 = qs0, P.qs1 = qs1;
    P.key = reinterpret_cast<const __nv_bfloat16 *>(key);
    P.value = reinterpret_cast<const __nv_bfloat16 *>(value);
    P.ks0 = ks0, P.ks1 = ks1, P.vs0 = vs0, P.vs1 = vs1;
    P.window = reinterpret_cast<const __nv_bfloat16 *>(window);
    P.qstarts = qstarts, P.seq_lens = seq_lens, P.table = table, P.counts = counts;
    P.tasks = tasks, P.task_count = task_count;
    P.partials = partials, P.lse = lse, P.split_slots = 1, P.split_index = 0;
    P.geo = geo;
    P.scale_log2 = scale * kLog2e;
    P.ntiles = (geo.query_tile * geo.group + 7) / 8;
    return raw_launch(P, num_tasks, (cudaStream_t)stream);
  }
  if (!history) return OSCAR_ERR_INVALID;
  HistParams P{};
  P.query = reinterpret_cast<const __nv_bfloat16 *>(query);
  P.qs0 = qs0, P.qs1 = qs1;
  P.history = history;
  P.qstarts = qstarts, P.seq_lens = seq_lens, P.table = table, P.counts = counts;
  P.tasks = tasks, P.task_count = task_count, P.num_tasks = num_tasks;
  P.partials = partials, P.lse = lse, P.split_slots = splits, P.splits = splits;
  P.geo = geo;
  P.scale_log2 = scale * kLog2e;
  P.status = status;
  return history_launch(P, num_tasks, (cudaStream_t)stream);
}

extern "C" int oscar_merge_splits(const float *partials, const float *lse, int64_t n, int32_t hq, int32_t splits,
                                  const int32_t *counts, void *out, float *logsum, void *stream) {
  if (n < 0 || hq <= 0 || splits <= 0) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!partials || !lse || !counts || !out || !logsum) return OSCAR_ERR_INVALID;
  const int64_t rows = n * hq;
  merge_splits_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      partials, lse, rows, hq, splits, splits, counts, reinterpret_cast<__nv_bfloat16 *>(out), logsum);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_merge_paths(const void *a, const float *la, const float *b, int64_t b_row_stride,
                                 const float *lb, int64_t lb_stride, int64_t n, int32_t hq, const int32_t *counts,
                                 void *out, void *stream) {
  if (n < 0 || hq <= 0) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!a || !la || !b || !lb || !counts || !out || b_row_stride % 4) return OSCAR_ERR_INVALID;
  const int64_t rows = n * hq;
  merge_paths_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16 *>(a), la, b, b_row_stride, lb, lb_stride, rows, hq, counts,
      reinterpret_cast<__nv_bfloat16 *>(out));
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_store_windows(const void *key, int64_t ks0, int64_t ks1, const void *value, int64_t vs0,
                                   int64_t vs1, void *window, const int32_t *qstarts, const int32_t *seq_lens,
                                   const int32_t *table, const int32_t *counts, int32_t num_programs,
                                   oscar_geometry geo, void *stream) {
  if (!geo_ok(geo) || num_programs < 0) return OSCAR_ERR_INVALID;
  if (num_programs == 0) return OSCAR_OK;
  if (!key || !value || !window || !qstarts || !seq_lens || !table || !counts) return OSCAR_ERR_INVALID;
  if (((reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value)) & 15) || ks0 % 8 || ks1 % 8 ||
      vs0 % 8 || vs1 % 8)
    return OSCAR_ERR_INVALID;
  window_store_kernel<<<num_programs, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16 *>(key), ks0, ks1, reinterpret_cast<const __nv_bfloat16 *>(value), vs0,
      vs1, reinterpret_cast<__nv_bfloat16 *>(window), qstarts, seq_lens, table, counts, geo);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_decode_attention(const void *qrot, const void *query, int64_t qs0, int64_t qs1, const void *key,
                                      int64_t ks0, int64_t ks1, const void *value, int64_t vs0, int64_t vs1,
                                      const uint8_t *history, void *window, const int32_t *qstarts,
                                      const int32_t *seq_lens, const int32_t *table, const int32_t *counts,
                                      const int32_t *tasks, const int32_t *task_count, int32_t num_tasks, int64_t n,
                                      const void *rv, float *scratch_partials, float *scratch_lse, void *output,
                                      oscar_geometry geo, float scale, int32_t splits, int32_t window_programs,
                                      int32_t *status, void *stream) {
  if (!geo_ok(geo) || splits <= 0 || splits > 64 || num_tasks < 0 || n < 0 || window_programs < 0)
    return OSCAR_ERR_INVALID;  // the fused merge holds at most 64 split LSEs per row in one warp
  if (n == 0) return OSCAR_OK;
  if (!qrot || !query || !key || !value || !history || !window || !qstarts || !seq_lens || !table || !counts ||
      !tasks || !task_count || !rv || !scratch_partials || !scratch_lse || !output)
    return OSCAR_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(qrot) | reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(key) |
       reinterpret_cast<uintptr_t>(value) | reinterpret_cast<uintptr_t>(rv) | reinterpret_cast<uintptr_t>(output)) &
      15)
    return OSCAR_ERR_INVALID;
  if (qs0 % 8 || qs1 % 8 || ks0 % 8 || ks1 % 8 || vs0 % 8 || vs1 % 8) return OSCAR_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  const int hq = geo.kv_heads * geo.group;
  bool window_done = false;
  if (num_tasks > 0) {
    HistParams H{};
    H.query = reinterpret_cast<const __nv_bfloat16 *>(qrot);
    H.qs0 = (int64_t)hq * kDim, H.qs1 = kDim;  // qrot is contiguous [n, Hq, 256]
    H.history = history;
    H.qstarts = qstarts, H.seq_lens = seq_lens, H.table = table, H.counts = counts;
    H.tasks = tasks, H.task_count = task_count, H.num_tasks = num_tasks;
    H.partials = scratch_partials, H.lse = scratch_lse, H.split_slots = splits + 1, H.splits = splits;
    H.geo = geo;
    H.scale_log2 = scale * kLog2e;
    H.balanced = 1;
    H.target_ctas = 8 * sm_count();
    H.status = status;
    // history on the caller's stream at the greatest priority, the raw path and then the
    // window store beside it on the side stream (joined before the merge); without a side
    // stream, one after the other
    RawSide *side = raw_side(st);
    std::unique_lock<std::mutex> side_lock;
    if (side) {
      side_lock = std::unique_lock<std::mutex>(side->mu);
      if (cudaEventRecord(side->fork, st) != cudaSuccess || cudaStreamWaitEvent(side->stream, side->fork, 0) != cudaSuccess)
        return OSCAR_ERR_LAUNCH;
    }
    int rc = history_launch(H, num_tasks, st, side ? side->priority : 0);
    if (rc) return rc;
    RawParams R{};
    R.query = reinterpret_cast<const __nv_bfloat16 *>(query);
    R.qs0 = qs0, R.qs1 = qs1;
    R.key = reinterpret_cast<const __nv_bfloat16 *>(key);
    R.value = reinterpret_cast<const __nv_bfloat16 *>(value);
    R.ks0 = ks0, R.ks1 = ks1, R.vs0 = vs0, R.vs1 = vs1;
    R.window = reinterpret_cast<const __nv_bfloat16 *>(window);
    R.qstarts = qstarts, R.seq_lens = seq_lens, R.table = table, R.counts = counts;
    R.tasks = tasks, R.task_count = task_count;
    R.partials = scratch_partials, R.lse = scratch_lse, R.split_slots = splits + 1, R.split_index = splits;
    R.geo = geo;
    R.scale_log2 = scale * kLog2e;
    R.ntiles = (geo.query_tile * geo.group + 7) / 8;
    rc = raw_launch(R, num_tasks, side ? side->stream : st);
    if (rc) return rc;
    if (side && window_programs > 0) {
      // the window store overwrites ring slots the raw path reads: after it, same stream
      window_store_kernel<<<window_programs, 256, 0, side->stream>>>(
          reinterpret_cast<const __nv_bfloat16 *>(key), ks0, ks1, reinterpret_cast<const __nv_bfloat16 *>(value),
          vs0, vs1, reinterpret_cast<__nv_bfloat16 *>(window), qstarts, seq_lens, table, counts, geo);
      OSCAR_CHECK_LAUNCH();
      window_done = true;
    }
    if (side && (cudaEventRecord(side->join, side->stream) != cudaSuccess ||
                 cudaStreamWaitEvent(st, side->join, 0) != cudaSuccess))
      return OSCAR_ERR_LAUNCH;
  }
  if (!ensure_dynamic_smem<finalize_kernel>(kFinSmem)) return OSCAR_ERR_LAUNCH;
  FinalParams F{};
  F.partials = scratch_partials, F.lse = scratch_lse, F.split_slots = splits + 1, F.splits = splits;
  F.rows = n * hq, F.hq = hq, F.counts = counts;
  F.rv = reinterpret_cast<const __nv_bfloat16 *>(rv);
  F.out = reinterpret_cast<__nv_bfloat16 *>(output);
  finalize_kernel<<<(unsigned)((F.rows + kFinLive - 1) / kFinLive), kFinThreads, kFinSmem, st>>>(F);
  OSCAR_CHECK_LAUNCH();
  if (window_programs > 0 && !window_done) {
    window_store_kernel<<<window_programs, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16 *>(key), ks0, ks1, reinterpret_cast<const __nv_bfloat16 *>(value), vs0,
        vs1, reinterpret_cast<__nv_bfloat16 *>(window), qstarts, seq_lens, table, counts, geo);
    OSCAR_CHECK_LAUNCH();
  }
  return OSCAR_OK;
}

// Test hook, no counterpart in the reference: CTA (0, 0, 0) of every later history launch
// skips the copy of its chunk / tile `withhold` (-1: none), CTA 0 of the first matrix of
// every later eigensolver launch skips its partial-sum pushes of round `withhold`, and
// every bounded device wait of those launches gives up after `wait_probes` probes (0: the
// default limit).  The skipped copy's consumers then time out, which exercises the
// timeout path (status word / info status, -inf rows, clean exit).
extern "C" int oscar_test_set_wait_fault(int32_t withhold, uint32_t wait_probes) {
  g_withhold.store(withhold < 0 ? -1 : withhold);
  g_wait_probes.store(wait_probes == 0 ? kWaitLimit : wait_probes);
  return OSCAR_OK;
}

extern "C" int oscar_last_history_kernel(void) { return g_last_history.load(); }
