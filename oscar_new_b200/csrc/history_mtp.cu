// INT2 history attention for MTP verify and other launches with 9..24 query rows per
// KV head (reference oscar_ascend/kernels.py:290-436, RAW=False; same partials, LSE and
// split ranges as history_attention_kernel in attention.cu).  The default for those
// launches (OSCAR_HISTORY_MTP=0 selects history_attention_kernel instead).
//
// history_attention_kernel gives every 8-row n-tile its own warp, and each of those warps
// rebuilds the key and value operands of every token: at 24 rows per KV head (4 query
// tokens x 6 heads) that is three times the operand work of a decode step.  Here four
// warps share a KV head and every operand is built once:
//  * chunks of 64 tokens (all heads of the CTA, one bulk copy, a 3-stage ring; the next
//    chunk is issued without blocking by whichever warp finds its stage released);
//  * scores: warp w builds the key operands of tokens 16w..16w+15 (per-token fp16 level
//    tables, PRMT, exactly as the decode kernel) and runs them against the query
//    fragments of all NT n-tiles, read from shared memory;
//  * softmax: the four warps agree on the chunk's row maxima through shared memory
//    (named barrier per head), so P' = p * s_v shares one scale per row; each warp turns
//    its scores into P' fragments (movmatrix) and stores them;
//  * values: warp w owns one byte lane of the value codes (64 of the 256 dims) for all
//    rows and all 64 tokens of the chunk: O^T += Vc^T . P'^T with the 2-bit codes as fp16
//    subnormals, NT MMAs per built operand.
// Row sums l and sum p * z_v are partial per warp (one common scale) and summed at the
// end; each warp writes its 64 dims of every row.  Every wait is bounded; a timeout sets
// an abort word that the four warps of a head read after the same named barrier, so they
// leave the chunk loop together and none is left waiting at a barrier.
#include "history_common.cuh"

namespace oscar {
namespace {

constexpr int kMtpChunk = 64;  // tokens per chunk: one 16-token m-tile per warp of a head
constexpr int kMtpStages = 3;
// All KV heads of a token in one CTA (up to 4): a chunk is then one contiguous run and one
// bulk copy; with fewer heads per CTA every token of the chunk needs its own copy.
constexpr int kMtpHeadsPerCta = 4;
constexpr int kMtpThreads = 128 * kMtpHeadsPerCta;

// per-head shared-memory block (bytes)
template <int NT>
struct MtpLayout {
  static constexpr int qfrag = 0;                       // [NT][8 k-step pairs][32 lanes] uint4
  static constexpr int qm = qfrag + NT * 16 * 32 * 8;   // [NT * 8] row scales
  static constexpr int xmax = qm + 32 * 4;              // [NT][4 t][2 r][4 warps] chunk row maxima
  static constexpr int pbuf = xmax + 4 * NT * 8 * 4;    // [4 k-steps][NT][32 lanes] uint2 P' fragments
  static constexpr int lz = pbuf + 4 * NT * 32 * 8;     // [4 warps][NT][4 t][2 r][2] l, sum p z
  static constexpr int bytes = (lz + 4 * NT * 8 * 2 * 4 + 127) / 128 * 128;
};

OSCAR_DEVINL void head_bar(int hl) { asm volatile("bar.sync %0, 128;" ::"r"(1 + hl) : "memory"); }

template <int NT>
__global__ void __launch_bounds__(kMtpThreads, 1) history_mtp_kernel(HistParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  using L = MtpLayout<NT>;
  const oscar_geometry &g = P.geo;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gi = lane >> 2, t = lane & 3;
  const int hl = warp >> 2, w = warp & 3;  // KV head within the CTA, warp within the head
  const int task = blockIdx.x, split = blockIdx.y;
  const int h0 = blockIdx.z * P.heads_per_cta;
  const int head = h0 + hl;
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
  const int lo = ti.sink_len + begin, hi = ti.sink_len + max(end, begin);
  if (P.balanced && hi <= lo) {
    for (int i = threadIdx.x; i < P.heads_per_cta * rows_valid; i += blockDim.x) {
      const int hh = i / rows_valid, row = i % rows_valid;
      const int tok = ti.qstart + ti.qoff + row / g.group;
      const int qh = (h0 + hh) * g.group + row % g.group;
      P.lse[((int64_t)tok * g.kv_heads * g.group + qh) * P.split_slots + split] = -INFINITY;
    }
    return;
  }
  const int first_chunk = lo / kMtpChunk;
  const int nchunks = hi > lo ? (hi - 1) / kMtpChunk - first_chunk + 1 : 0;

  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kMtpStages;
  int32_t *abort_word = reinterpret_cast<int32_t *>(empty + kMtpStages);
  int32_t *next_issue = abort_word + 1;  // first chunk not yet issued
  uint8_t *stages = smem + 128;
  uint8_t *hs = stages + kMtpStages * P.stage_bytes + hl * L::bytes;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMtpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], P.consumers);
    }
    *abort_word = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  const int hpc = P.heads_per_cta;
  const int token_bytes = hpc * g.slot_bytes;
  const int32_t *trow = P.table + (int64_t)ti.req * g.table_stride;
  auto issue_one = [&](int c) {
    const int s = c % kMtpStages;
    const int pos = (first_chunk + c) * kMtpChunk;
    const int64_t slot0 = (int64_t)trow[pos / kKernelBlock] * kKernelBlock + pos % kKernelBlock;
    const uint8_t *src = P.history + (slot0 / g.block_tokens) * g.page_bytes +
                         ((slot0 % g.block_tokens) * g.kv_heads + h0) * (int64_t)g.slot_bytes;
    if (c == P.withhold && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) return;  // test hook
    const uint32_t dst = smem_u32(stages + s * P.stage_bytes);
    mbar_arrive_expect_tx(&full[s], kMtpChunk * token_bytes);
    if (hpc == g.kv_heads) {
      bulk_copy_g2s(dst, src, kMtpChunk * token_bytes, &full[s]);
    } else {
      for (int tk = 0; tk < kMtpChunk; ++tk)
        bulk_copy_g2s(dst + tk * token_bytes, src + (int64_t)tk * g.kv_heads * g.slot_bytes, token_bytes, &full[s]);
    }
  };
  if (threadIdx.x == 0) {
    for (int c = 0; c < min(kMtpStages - 1, nchunks); ++c) issue_one(c);
    *next_issue = min(kMtpStages - 1, nchunks);
  }
  // Non-blocking copy issue (lane 0 of any warp): the next unissued chunk goes out as soon
  // as every warp has released its stage (the previous occupant, STAGES chunks back).  A
  // warp that is ahead never waits for another head's warps here; the atomic claim keeps
  // each chunk to one issuer.  The empty-barrier parity test is unambiguous: chunk nx - S
  // was issued, so phase nx / S - 2 of that barrier has completed.
  auto try_issue = [&]() {
#pragma unroll 1
    for (int k = 0; k < kMtpStages; ++k) {
      const int nx = *reinterpret_cast<volatile int32_t *>(next_issue);
      if (nx >= nchunks) return;
      if (nx >= kMtpStages && !mbar_test(&empty[nx % kMtpStages], ((nx / kMtpStages) - 1) & 1)) return;
      if (atomicCAS(next_issue, nx, nx + 1) == nx) issue_one(nx);
    }
  };

  // ---- query fragments of the head: warp w < NT computes n-tile w ----
  // k-steps 2m and 2m + 1 of a lane side by side: one 16-byte load feeds two MMAs
  uint4 *qfrag = reinterpret_cast<uint4 *>(hs + L::qfrag);
  float *qm_row = reinterpret_cast<float *>(hs + L::qm);
  if (w < NT && nchunks > 0) {
    const int r_mine = 8 * w + gi;
    const bool rvalid = r_mine < rows_valid;
    const int qtok = ti.qstart + ti.qoff + (rvalid ? r_mine / g.group : 0);
    const int qhead = head * g.group + (rvalid ? r_mine % g.group : 0);
    QueryFrags Q;
    load_query_frags(Q, P.query + (int64_t)qtok * P.qs0 + (int64_t)qhead * P.qs1, rvalid, P.scale_log2);
#pragma unroll
    for (int m = 0; m < 8; ++m)
      qfrag[(w * 8 + m) * 32 + lane] = make_uint4(Q.qf[2 * m][0], Q.qf[2 * m][1], Q.qf[2 * m + 1][0], Q.qf[2 * m + 1][1]);
    if (gi == 0) {
      qm_row[8 * w + 2 * t] = Q.qm[0];
      qm_row[8 * w + 2 * t + 1] = Q.qm[1];
    }
  }
  __syncthreads();

  float *xmax = reinterpret_cast<float *>(hs + L::xmax);
  uint2 *pbuf = reinterpret_cast<uint2 *>(hs + L::pbuf);
  // value side: this warp's byte lane of the code words (dims 32gi + 16 half + 4w + p)
  const uint32_t vsel = (w >> 1) ? 0x7632u : 0x5410u;
  const int vshift = (w & 1) ? 8 : 0;

  float o[NT][4][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int p = 0; p < 4; ++p) o[n][p][0] = o[n][p][1] = o[n][p][2] = o[n][p][3] = 0.f;
  float m_run[NT][2], l_run[NT][2], zp_run[NT][2];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int r = 0; r < 2; ++r) m_run[n][r] = -INFINITY, l_run[n][r] = 0.f, zp_run[n][r] = 0.f;
  bool ok = true;

#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    const int s = c % kMtpStages;
    // lane 0 waits for the chunk and issues pending copies meanwhile; then every lane
    // observes the completed phase itself (acquire of the copied bytes)
    uint32_t got = 0;
    if (lane == 0) {
#pragma unroll 1
      for (uint32_t it = 0, lim = P.wait_probes ? P.wait_probes : kWaitLimit; it < lim; ++it) {
        if (mbar_try_wait(&full[s], (c / kMtpStages) & 1)) {
          got = 1;
          break;
        }
        try_issue();
      }
    }
    const bool have = __shfl_sync(0xffffffffu, got, 0) != 0 && mbar_wait_bounded(&full[s], (c / kMtpStages) & 1, P.wait_probes);
    if (!have) {
      if (lane == 0) {
        atomicExch(abort_word, 1);
        if (P.status) atomicExch(P.status, OSCAR_ERR_TIMEOUT);
      }
    }
    const uint8_t *stage = stages + s * P.stage_bytes;
    const int cpos = (first_chunk + c) * kMtpChunk;

    // ---------------- scores of tokens cpos + 16w + {gi, gi+8}, all rows ----------------
    const int tpos = cpos + 16 * w;
    const uint8_t *tl = stage + 16 * w * token_bytes + hl * g.slot_bytes;
    const bool va = tpos + gi >= lo && tpos + gi < hi;
    const bool vb = tpos + gi + 8 >= lo && tpos + gi + 8 < hi;
    const bool live = have && tpos + 16 > lo && tpos < hi;  // warp-uniform
    float lg[NT][4];
    uint32_t vsz0 = 0, vsz1 = 0;
    if (live) {
      // lanes t = 0, 1 of row group gi build the tables of tokens gi and gi + 8
      const KeyLut mine = key_lut(*reinterpret_cast<const uint32_t *>(tl + (gi + 8 * (t & 1)) * token_bytes + 64));
      KeyLut lA, lB;
      lA.lo = __shfl_sync(0xffffffffu, mine.lo, 4 * gi);
      lA.hi = __shfl_sync(0xffffffffu, mine.hi, 4 * gi);
      lA.inv = __shfl_sync(0xffffffffu, mine.inv, 4 * gi);
      lB.lo = __shfl_sync(0xffffffffu, mine.lo, 4 * gi + 1);
      lB.hi = __shfl_sync(0xffffffffu, mine.hi, 4 * gi + 1);
      lB.inv = __shfl_sync(0xffffffffu, mine.inv, 4 * gi + 1);
      const uint8_t *ra = tl + gi * token_bytes, *rb = ra + 8 * token_bytes;
      const uint4 ka = *reinterpret_cast<const uint4 *>(ra + 16 * t);
      const uint4 kb = *reinterpret_cast<const uint4 *>(rb + 16 * t);
      const uint32_t kaw[4] = {ka.x, ka.y, ka.z, ka.w}, kbw[4] = {kb.x, kb.y, kb.z, kb.w};
      vsz0 = *reinterpret_cast<const uint32_t *>(ra + g.vector_bytes + 64);
      vsz1 = *reinterpret_cast<const uint32_t *>(rb + g.vector_bytes + 64);
      float sc[NT][4];
#pragma unroll
      for (int n = 0; n < NT; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) {
        uint4 qp[NT];  // query fragments of k-steps 4 wd + p, p of one pair
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          if ((p & 1) == 0) {
#pragma unroll
            for (int n = 0; n < NT; ++n) qp[n] = qfrag[(n * 8 + 2 * wd + (p >> 1)) * 32 + lane];
          }
          const uint32_t xa = (kaw[wd] >> (2 * p)) & 0x03030303u;
          const uint32_t xb = (kbw[wd] >> (2 * p)) & 0x03030303u;
          const uint32_t sa = xa * 0x11u + 0x40404040u, sb = xb * 0x11u + 0x40404040u;
          const uint32_t a0 = prmt(lA.lo, lA.hi, sa);
          const uint32_t a1 = prmt(lB.lo, lB.hi, sb);
          const uint32_t a2 = prmt(lA.lo, lA.hi, sa >> 16);
          const uint32_t a3 = prmt(lB.lo, lB.hi, sb >> 16);
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            mma_f16_16816(sc[n], a0, a1, a2, a3, (p & 1) ? qp[n].z : qp[n].x, (p & 1) ? qp[n].w : qp[n].y);
          }
        }
      }
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const float2 qmn = *reinterpret_cast<const float2 *>(qm_row + 8 * n + 2 * t);  // rows 2t, 2t+1
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mul = (e < 2 ? lA.inv : lB.inv) * ((e & 1) ? qmn.y : qmn.x);
          lg[n][e] = ((e < 2) ? va : vb) ? sc[n][e] * mul : -INFINITY;
        }
      }
    } else {
#pragma unroll
      for (int n = 0; n < NT; ++n) lg[n][0] = lg[n][1] = lg[n][2] = lg[n][3] = -INFINITY;
    }
    // chunk row maxima: over this warp's 16 tokens, then over the head's four warps
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float mx = fmaxf(lg[n][r], lg[n][r + 2]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        if (gi == 0) xmax[((n * 4 + t) * 2 + r) * 4 + w] = mx;  // the head's 4 warps side by side
      }
    head_bar(hl);
    // Abort snapshot: every write of the word (a full-barrier timeout of this chunk, a
    // copy-issue timeout of the previous one) precedes its writer's arrival at the barrier
    // above, and no warp of the head can write it again before all four have passed the
    // next barrier, so the four warps read the same value and leave together.
    if (*reinterpret_cast<volatile int32_t *>(abort_word) != 0) {
      ok = false;
      break;
    }
    float mc[NT][2];
    bool need_any = false;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float4 xw = *reinterpret_cast<const float4 *>(xmax + ((n * 4 + t) * 2 + r) * 4);
        const float mx = fmaxf(fmaxf(xw.x, xw.y), fmaxf(xw.z, xw.w));
        mc[n][r] = mx;
        need_any |= mx > m_run[n][r] + kRescaleSlack || (m_run[n][r] == -INFINITY && mx > -INFINITY);
      }
    // every warp of the head sees the same maxima, so all re-base together
    if (__any_sync(0xffffffffu, need_any)) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const float mx = mc[n][r];
          const bool need = mx > m_run[n][r] + kRescaleSlack || (m_run[n][r] == -INFINITY && mx > -INFINITY);
          const float a = need ? (m_run[n][r] == -INFINITY ? 0.f : ex2(m_run[n][r] - mx)) : 1.f;
          if (need) m_run[n][r] = mx;
#pragma unroll
          for (int p = 0; p < 4; ++p) o[n][p][r] *= a, o[n][p][r + 2] *= a;
          l_run[n][r] *= a;
          zp_run[n][r] *= a;
        }
    }
    // P' = p * s_v of this warp's tokens as B fragments of the value MMAs
    {
      const float vsA = va && live ? half_bits_to_float(vsz0 & 0xffffu) : 0.f;
      const float vzA = va && live ? half_bits_to_float(vsz0 >> 16) : 0.f;
      const float vsB = vb && live ? half_bits_to_float(vsz1 & 0xffffu) : 0.f;
      const float vzB = vb && live ? half_bits_to_float(vsz1 >> 16) : 0.f;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const float ms0 = m_run[n][0] == -INFINITY ? 0.f : m_run[n][0];
        const float ms1 = m_run[n][1] == -INFINITY ? 0.f : m_run[n][1];
        const float p0 = ex2(lg[n][0] - ms0), p1 = ex2(lg[n][1] - ms1);
        const float p2 = ex2(lg[n][2] - ms0), p3 = ex2(lg[n][3] - ms1);
        l_run[n][0] += p0 + p2;
        l_run[n][1] += p1 + p3;
        zp_run[n][0] = fmaf(p0, vzA, fmaf(p2, vzB, zp_run[n][0]));
        zp_run[n][1] = fmaf(p1, vzA, fmaf(p3, vzB, zp_run[n][1]));
        pbuf[(w * NT + n) * 32 + lane] = make_uint2(movmatrix_trans(pack_half2(p0 * vsA, p1 * vsA)),
                                                    movmatrix_trans(pack_half2(p2 * vsB, p3 * vsB)));
      }
    }
    head_bar(hl);

    // ---------------- O^T += Vc^T . P'^T over the chunk's 64 tokens ----------------
    if (have) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (cpos + 16 * kk + 16 <= lo || cpos + 16 * kk >= hi) continue;  // uniform: no live token
        const uint8_t *vt = stage + 16 * kk * token_bytes + hl * g.slot_bytes + g.vector_bytes;
        uint32_t vw[4][2];  // [token 2t, 2t+1, 2t+8, 2t+9][word 2gi, 2gi+1]
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int tok = 2 * t + (q & 1) + (q >> 1) * 8;
          const uint32_t *src = reinterpret_cast<const uint32_t *>(vt + tok * token_bytes) + 2 * gi;
          vw[q][0] = src[0];
          vw[q][1] = src[1];
        }
        const uint32_t x0 = prmt(vw[0][0], vw[1][0], vsel) >> vshift;
        const uint32_t x1 = prmt(vw[0][1], vw[1][1], vsel) >> vshift;
        const uint32_t x2 = prmt(vw[2][0], vw[3][0], vsel) >> vshift;
        const uint32_t x3 = prmt(vw[2][1], vw[3][1], vsel) >> vshift;
        uint2 pb[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n) pb[n] = pbuf[(kk * NT + n) * 32 + lane];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const uint32_t msk = 0x00030003u << (2 * p);
#pragma unroll
          for (int n = 0; n < NT; ++n)
            mma_f16_16816(o[n][p], x0 & msk, x1 & msk, x2 & msk, x3 & msk, pb[n].x, pb[n].y);
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&empty[s]);
      try_issue();
    }
  }
  if (!ok && lane == 0) {
    // Aborted: let the copies this warp may have issued land before it can exit.  This
    // lane issues nothing more, so its chunks are below the claim counter `snap`; a chunk
    // below snap - S has landed (the claim of snap - 1 needed every consumer past
    // snap - 1 - S).  A chunk c also has landed once chunk c + S is claimed, which stops
    // the wait before the stage's barrier can complete a second phase.
    const int snap = *reinterpret_cast<volatile int32_t *>(next_issue);
    const bool hooked = blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
    const uint32_t lim = P.wait_probes ? P.wait_probes : kWaitLimit;
    for (int cc = max(0, snap - kMtpStages); cc < snap; ++cc) {
      if (hooked && cc == P.withhold) continue;
#pragma unroll 1
      for (uint32_t it = 0; it < lim; ++it)
        if (mbar_try_wait(&full[cc % kMtpStages], (cc / kMtpStages) & 1) ||
            *reinterpret_cast<volatile int32_t *>(next_issue) > cc + kMtpStages)
          break;
    }
  }

  // ---------------- row sums over the head's warps, write the partials ----------------
  float *lz = reinterpret_cast<float *>(hs + L::lz);
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float lsum = l_run[n][r], zsum = zp_run[n][r];
#pragma unroll
      for (int o2 = 4; o2 <= 16; o2 <<= 1) {
        lsum += __shfl_xor_sync(0xffffffffu, lsum, o2);
        zsum += __shfl_xor_sync(0xffffffffu, zsum, o2);
      }
      if (gi == 0) {
        lz[(((w * NT + n) * 4 + t) * 2 + r) * 2 + 0] = lsum;
        lz[(((w * NT + n) * 4 + t) * 2 + r) * 2 + 1] = zsum;
      }
    }
  head_bar(hl);
  if (!ok) {
    // aborted: mark the rows empty (-inf) so the merge never reads a partial sum
    if (w == 0 && gi == 0)
      for (int n = 0; n < NT; ++n)
        for (int r = 0; r < 2; ++r) {
          const int row = 8 * n + 2 * t + r;
          if (row >= rows_valid) continue;
          const int tok = ti.qstart + ti.qoff + row / g.group;
          const int qh = head * g.group + row % g.group;
          P.lse[((int64_t)tok * g.kv_heads * g.group + qh) * P.split_slots + split] = -INFINITY;
        }
    return;
  }
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = 8 * n + 2 * t + r;
      float Lr = 0.f, Zr = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < 4; ++w2) {
        Lr += lz[(((w2 * NT + n) * 4 + t) * 2 + r) * 2 + 0];
        Zr += lz[(((w2 * NT + n) * 4 + t) * 2 + r) * 2 + 1];
      }
      if (row >= rows_valid) continue;
      const int tok = ti.qstart + ti.qoff + row / g.group;
      const int qh = head * g.group + row % g.group;
      const int64_t orow = ((int64_t)tok * g.kv_heads * g.group + qh) * P.split_slots + split;
      const bool any = Lr > 0.f;
      if (w == 0 && gi == 0) P.lse[orow] = any ? (m_run[n][r] * 0.69314718055994531f + logf(Lr)) : -INFINITY;
      if (!any && P.balanced) continue;  // the merge skips -inf splits without reading them
      const float inv = any ? 1.0f / Lr : 0.f;
      const float zterm = any ? Zr * inv : 0.f;
      float *dst = P.partials + orow * kDim + 32 * gi + 4 * w;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float v[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) v[p] = fmaf(o[n][p][2 * half + r] * (kTwo24 / (float)(1 << (2 * p))), inv, zterm);
        *reinterpret_cast<float4 *>(dst + 16 * half) = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
}

template <int NT>
int launch_mtp(HistParams P, int32_t num_tasks, cudaStream_t stream, int priority) {
  const oscar_geometry &g = P.geo;
  if (g.kv_heads > kMtpHeadsPerCta) return OSCAR_ERR_UNSUPPORTED;
  const int hpc = g.kv_heads;
  P.heads_per_cta = hpc;
  P.ntiles = NT;
  P.units = hpc * NT;
  P.warps_per_unit = 1;
  P.consumers = 4 * hpc;
  P.chunk_tokens = kMtpChunk;
  P.stage_bytes = kMtpChunk * hpc * g.slot_bytes;
  const size_t smem = 128 + (size_t)kMtpStages * P.stage_bytes + (size_t)hpc * MtpLayout<NT>::bytes;
  if (smem > 227 * 1024) return OSCAR_ERR_UNSUPPORTED;
  if (!ensure_dynamic_smem<history_mtp_kernel<NT>>(smem)) return OSCAR_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_tasks, P.splits, g.kv_heads / hpc);
  cfg.blockDim = dim3(128 * hpc);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributePriority;
  attr[0].val.priority = priority;
  cfg.attrs = attr;
  cfg.numAttrs = priority != 0 ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, history_mtp_kernel<NT>, P) != cudaSuccess) return OSCAR_ERR_LAUNCH;
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

}  // namespace

int history_mtp_launch(HistParams P, int32_t num_tasks, cudaStream_t stream, int priority) {
  const oscar_geometry &g = P.geo;
  const int ntiles = (g.query_tile * g.group + 7) / 8;
  if (g.slot_bytes % 16 != 0 || g.vector_bytes != 68) return OSCAR_ERR_UNSUPPORTED;
  if (ntiles == 2) return launch_mtp<2>(P, num_tasks, stream, priority);
  if (ntiles == 3) return launch_mtp<3>(P, num_tasks, stream, priority);
  return OSCAR_ERR_UNSUPPORTED;
}

}  // namespace oscar
