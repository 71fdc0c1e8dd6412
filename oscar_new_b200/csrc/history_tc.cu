// INT2 history split-KV attention with the key side on the 5th-generation tensor cores.
// Reference: oscar_ascend/kernels.py:290-436 (RAW=False), same split / mask / LSE
// semantics as history_attention_kernel (attention.cu).
//
// One CTA = (task, split, KV head); the history of the split is walked in 128-token
// tiles (one kernel block each).
// * Warp 4 lane 0 streams tiles with a 3-D TMA load (box {160 B, 128 tokens, 1 page}
//   out of the [pages][page tokens][heads x 160 B] history stripe: the head's slots,
//   strided in HBM, land contiguous in shared memory) into a 4-stage ring.  No multicast.
// * Warps 0-3 ("key warps", thread = token = TMEM lane) expand the token's 2-bit key
//   codes into one fp16 A operand in tensor memory: the token's four bf16 key levels
//   (exact in fp16 after a power-of-two scale) looked up by PRMT, two codes per
//   instruction, 128 columns.  One thread issues 16 tcgen05.mma (M = 128 tokens, N = 16
//   or 32 query rows, K = 16) against a single query tile B (q times a per-row power
//   of two, fp16, 128-byte swizzle) in shared memory: all query rows of the task share
//   the operand work.  The key warps read the accumulators back (logit = D * 2^-e_token *
//   2^-e_row), take each row's warp maximum with one integer reduction, run the online
//   softmax (log2 domain, lazy re-basing) and write P' = p * s_v as fp16 and the
//   re-basing factors to shared memory.
// * Warps 4-7 ("value warps") each own 64 of the 256 dims: O^T += Vc^T . P'^T on
//   mma.sync m16n8k16 with the V codes as fp16 subnormals (byte pairs of two tokens by
//   prmt, one AND per two codes) for every 8-row tile of the task's query rows.
// Tensor memory: 128 columns of A operand + N accumulator columns (256 allocated, one
// CTA per SM).  Every mbarrier wait is bounded; a timeout sets the
// status word, the warps leave their loops at the next common point and the CTA frees
// its tensor memory.
#include <cstring>

#include "history_common.cuh"
#include "tcgen05.cuh"

namespace oscar {
namespace {

constexpr int kTcTile = 128;
constexpr int kTcStages = 4;
constexpr int kTcSlot = 160;
constexpr int kTcStageBytes = kTcTile * kTcSlot;  // 20 KiB
constexpr int kTcThreads = 256;
constexpr int kTcMaxRows = 32;
constexpr int kPRowBytes = kTcTile * 2 + 16;  // P' row: 128 fp16 + 16 B pad (ldmatrix rows hit distinct banks)
constexpr int kColD = 128;  // A operand (key levels) in columns 0..127, accumulators after it
constexpr uint32_t kTcTmemCols = 256;
constexpr int kOffB = kTcStages * kTcStageBytes;               // query tile (1024-aligned)
constexpr int kOffP = kOffB + kTcMaxRows * kDim * 2;           // P' double buffer
constexpr int kOffSmall = kOffP + 2 * kTcMaxRows * kPRowBytes;  // scalars and barriers

struct TcSmall {
  float alpha[2][kTcMaxRows];
  float mrun[2][kTcMaxRows];
  float qup[kTcMaxRows];  // per-row power-of-two scale of the fp16 query tile
  float qm[kTcMaxRows];   // its inverse times log2(e) * softmax scale
  float wmax[4][kTcMaxRows];
  float wl[4][kTcMaxRows];
  float wz[4][kTcMaxRows];
  float lsum[kTcMaxRows], zsum[kTcMaxRows], mfin[kTcMaxRows];
  uint64_t full[kTcStages], empty[kTcStages], mma, pfull[2], pempty[2];
  uint32_t tmem;
  int32_t span;
  int32_t abort;
};
constexpr int kSmemHistTc = kOffSmall + (int)sizeof(TcSmall) + 1024;

struct HistTcParams {
  CUtensorMap hmap;  // [pages][page tokens][kv_heads * 160 B], uint8
  HistParams P;
  int32_t ncols;     // MMA N: 16 or 32
};

// Instruction descriptor, kind::f16: fp32 accumulator, A and B fp16, both K-major,
// N >> 3 at [17,23), M = 128 -> 8 at [24,29).
OSCAR_DEVINL uint32_t idesc_f16_m128(int n) { return (1u << 4) | ((uint32_t)(n >> 3) << 17) | (8u << 24); }

OSCAR_DEVINL void named_sync(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }

OSCAR_DEVINL void ldmatrix_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

OSCAR_DEVINL bool aborted(const TcSmall &S) { return *reinterpret_cast<const volatile int32_t *>(&S.abort) != 0; }

OSCAR_DEVINL void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__global__ void __launch_bounds__(kTcThreads, 1) history_tc_kernel(const __grid_constant__ HistTcParams T) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  TcSmall &S = *reinterpret_cast<TcSmall *>(smem + kOffSmall);
  const HistParams &P = T.P;
  const oscar_geometry &g = P.geo;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int task = blockIdx.x, split = blockIdx.y, head = blockIdx.z;
  const TaskInfo ti = load_task(task, P.tasks, P.task_count, P.qstarts, P.seq_lens, P.counts, g);
  if (!ti.live || ti.qlen <= 0) return;
  const int R = min(g.query_tile, ti.qoff < ti.qlen ? ti.qlen - ti.qoff : 0) * g.group;
  const int length = ti.recent_begin - ti.sink_len;
  const int tiles32 = (length + 31) / 32;
  int nsplit = P.splits;
  if (P.balanced) {
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
        S.span = (int)(span < kMinSplitTokens ? (int64_t)kMinSplitTokens : (span > (1 << 30) ? (int64_t)(1 << 30) : span));
      }
    }
    __syncthreads();
    nsplit = max(1, min(P.splits, (length + S.span - 1) / S.span));
  }
  const int per_split = (tiles32 + nsplit - 1) / nsplit;
  const int begin = split * per_split * 32;
  const int end = min((split + 1) * per_split * 32, length);
  const int lo = ti.sink_len + begin, hi = ti.sink_len + max(end, begin);
  auto out_row = [&](int r) {
    const int tok = ti.qstart + ti.qoff + r / g.group;
    const int qh = head * g.group + r % g.group;
    return ((int64_t)tok * g.kv_heads * g.group + qh) * P.split_slots + split;
  };
  if (P.balanced && hi <= lo) {
    for (int r = tid; r < R; r += kTcThreads) P.lse[out_row(r)] = -INFINITY;
    return;
  }
  const int first_blk = lo / kTcTile;
  const int nblk = hi > lo ? (hi - 1) / kTcTile - first_blk + 1 : 0;
  const int N = T.ncols;

  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 8);
    }
    mbar_init(&S.mma, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.pfull[b], 128);
      mbar_init(&S.pempty[b], 4);
    }
    S.abort = 0;
    fence_mbarrier_init();
  }
  if (tid < kTcMaxRows) S.mrun[0][tid] = -INFINITY;
  if (warp == 0) tmem_alloc(&S.tmem, kTcTmemCols);
  // per-row scale of the query: max |q| into [2^14, 2^15), exact in fp16
  if (tid < kTcMaxRows) {
    float amax = 0.f;
    if (tid < R) {
      const uint16_t *qrow = reinterpret_cast<const uint16_t *>(
          P.query + (int64_t)(ti.qstart + ti.qoff + tid / g.group) * P.qs0 +
          (int64_t)(head * g.group + tid % g.group) * P.qs1);
      for (int d = 0; d < kDim; ++d) amax = fmaxf(amax, fabsf(bf16_bits_to_float(qrow[d])));
    }
    const uint32_t ex = (__float_as_uint(amax) >> 23) & 0xffu, exc = ex < 16u ? 16u : ex;
    S.qup[tid] = amax > 0.f ? __uint_as_float((268u - exc) << 23) : 0.f;
    S.qm[tid] = amax > 0.f ? __uint_as_float((exc - 14u) << 23) * P.scale_log2 : 0.f;
  }
  __syncthreads();
  // query tile B: row n, contraction index k = 16 W + 4 p + 2 h + s holds q[16 W + p + 8 h + 4 s]
  // (the order the key levels are expanded in: column 8 W + 2 p + h of the A operand
  // holds the levels of code position p of bytes {2h, 2h + 1} of word W), K-major in four
  // 64-wide blocks, 128-byte swizzle
  for (int e = tid; e < N * 32; e += kTcThreads) {
    const int n = e >> 5, ch = e & 31;
    uint32_t wv[4] = {0u, 0u, 0u, 0u};
    if (n < R) {
      const uint16_t *qrow = reinterpret_cast<const uint16_t *>(
          P.query + (int64_t)(ti.qstart + ti.qoff + n / g.group) * P.qs0 + (int64_t)(head * g.group + n % g.group) * P.qs1);
      const float up = S.qup[n];
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) {
        float v2[2];
#pragma unroll
        for (int s2 = 0; s2 < 2; ++s2) {
          const int k = 8 * ch + 2 * e2 + s2;
          const int dim = 16 * (k >> 4) + ((k >> 2) & 3) + 8 * ((k >> 1) & 1) + 4 * (k & 1);
          v2[s2] = bf16_bits_to_float(qrow[dim]) * up;
        }
        wv[e2] = pack_half2(v2[0], v2[1]);
      }
    }
    const int kb = ch >> 3, c = ch & 7;
    *reinterpret_cast<uint4 *>(smem + kOffB + kb * (N * 128) + n * 128 + ((c ^ (n & 7)) << 4)) =
        make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;

  if (warp < 4) {
    // ================= key warps: thread = token = TMEM lane =================
    const int i = tid;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
    float lp[kTcMaxRows], zp[kTcMaxRows], lg[kTcMaxRows];
#pragma unroll
    for (int r = 0; r < kTcMaxRows; ++r) lp[r] = zp[r] = 0.f;
    const uint32_t idesc = idesc_f16_m128(N);
    for (int t = 0; t < nblk; ++t) {
      const int s = t % kTcStages, b = t & 1;
      bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&S.full[s], (t / kTcStages) & 1));
      uint32_t w[16];
      uint32_t ksz = 0, vsz = 0;
      float kinv = 0.f;
      if (ok) {
        const uint8_t *row = smem + s * kTcStageBytes + i * kTcSlot;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 v = *reinterpret_cast<const uint4 *>(row + 16 * c);
          w[4 * c] = v.x, w[4 * c + 1] = v.y, w[4 * c + 2] = v.z, w[4 * c + 3] = v.w;
        }
        ksz = *reinterpret_cast<const uint32_t *>(row + 64);
        vsz = *reinterpret_cast<const uint32_t *>(row + 132);
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);
        // the A operand: the token's bf16 key levels (exact in fp16 after its power-of-two
        // scale) through its byte table, column 8 W + 2 p + h = code position p of bytes
        // {2h, 2h + 1} of word W; one IMAD builds both PRMT selectors of a word position
        const KeyLut lt = key_lut(ksz);
        kinv = lt.inv;
#pragma unroll
        for (int bt = 0; bt < 4; ++bt) {
          uint32_t v[32];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const uint32_t ww = w[4 * bt + jj];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const uint32_t sel = ((ww >> (2 * p)) & 0x03030303u) * 0x11u + 0x40404040u;
              v[8 * jj + 2 * p] = prmt(lt.lo, lt.hi, sel);
              v[8 * jj + 2 * p + 1] = prmt(lt.lo, lt.hi, sel >> 16);
            }
          }
          tmem_store32(lane_base + (uint32_t)(32 * bt), v);
        }
        tmem_store_wait();
      } else {
        atomicExch(&S.abort, 1);
      }
      tc_fence_before();
      named_sync(1, 128);
      if (aborted(S)) break;
      if (tid == 0) {
        tc_fence_after();
#pragma unroll 1
        for (int j = 0; j < 16; ++j) {
          const uint64_t bd = smem_desc(smem_u32(smem + kOffB) + (j >> 2) * (N * 128) + (j & 3) * 32, 16, 1024);
          umma_f16_ts(tmem + kColD, tmem + 8 * j, bd, idesc, j > 0 ? 1u : 0u);
        }
        umma_commit(&S.mma);
      }
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(&S.mma, t & 1));
      tc_fence_after();
      const int pos = (first_blk + t) * kTcTile + i;
      const bool valid = pos >= lo && pos < hi;
      if (ok) {
#pragma unroll
        for (int g0 = 0; g0 < kTcMaxRows; g0 += 16) {
          if (g0 < N) {
            uint32_t dm[16];
            tmem_load16(lane_base + (uint32_t)(kColD + g0), dm);
#pragma unroll
            for (int rr = 0; rr < 16; ++rr) {
              const int r = g0 + rr;
              lg[r] = (valid && r < R) ? __uint_as_float(dm[rr]) * (kinv * S.qm[r]) : -INFINITY;
            }
          }
        }
        // per-row max over the warp's 32 tokens: one integer reduction on an order-preserving
        // image of the float
#pragma unroll
        for (int r = 0; r < kTcMaxRows; ++r) {
          if (r >= R) break;
          const int key = __float_as_int(lg[r]);
          const int mk = __reduce_max_sync(0xffffffffu, key >= 0 ? key : key ^ 0x7fffffff);
          if (lane == 0) S.wmax[warp][r] = __int_as_float(mk >= 0 ? mk : mk ^ 0x7fffffff);
        }
      } else {
        atomicExch(&S.abort, 1);
      }
      named_sync(1, 128);
      if (aborted(S)) break;
      // running max per row (the same decision in every key thread), P' and the sums
      if (t >= 2 && !mbar_wait_bounded(&S.pempty[b], ((t >> 1) - 1) & 1)) atomicExch(&S.abort, 1);
      const float *mold = S.mrun[t & 1];
      float *mnew = S.mrun[(t + 1) & 1];
      const float vs = half_bits_to_float(vsz & 0xffffu), vz = half_bits_to_float(vsz >> 16);
      uint8_t *pb = smem + kOffP + b * (kTcMaxRows * kPRowBytes);
#pragma unroll
      for (int r = 0; r < kTcMaxRows; ++r) {
        if (r >= R) break;
        const float tm = fmaxf(fmaxf(S.wmax[0][r], S.wmax[1][r]), fmaxf(S.wmax[2][r], S.wmax[3][r]));
        const float mo = mold[r];
        const bool need = tm > mo + kRescaleSlack || (mo == -INFINITY && tm > -INFINITY);
        const float mn = need ? tm : mo;
        const float al = need ? (mo == -INFINITY ? 0.f : ex2(mo - mn)) : 1.f;
        if (i == r) {
          mnew[r] = mn;
          S.alpha[b][r] = al;
        }
        const float pr = ex2(lg[r] - (mn == -INFINITY ? 0.f : mn));
        lp[r] = fmaf(lp[r], al, pr);
        zp[r] = fmaf(zp[r], al, pr * vz);
        *reinterpret_cast<__half *>(pb + r * kPRowBytes + i * 2) = __float2half_rn(pr * vs);
      }
      mbar_arrive(&S.pfull[b]);
    }
    // row sums over the 128 token lanes
#pragma unroll
    for (int r = 0; r < kTcMaxRows; ++r) {
      if (r >= R) break;
      float l = lp[r], z = zp[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        l += __shfl_xor_sync(0xffffffffu, l, o);
        z += __shfl_xor_sync(0xffffffffu, z, o);
      }
      if (lane == 0) S.wl[warp][r] = l, S.wz[warp][r] = z;
    }
    named_sync(1, 128);
    if (tid < R) {
      S.lsum[tid] = (S.wl[0][tid] + S.wl[1][tid]) + (S.wl[2][tid] + S.wl[3][tid]);
      S.zsum[tid] = (S.wz[0][tid] + S.wz[1][tid]) + (S.wz[2][tid] + S.wz[3][tid]);
      S.mfin[tid] = S.mrun[nblk & 1][tid];
    }
  } else {
    // ================= value warps: 64 dims each, all 8-row tiles of the task =================
    const int v = warp - 4;
    const int gi = lane >> 2, tq = lane & 3, bg = gi & 3;
    const int wlo = 4 * v + (gi >> 2), whi = wlo + 2;  // V words (16 dims each) of rows gi and gi + 8
    const uint32_t sel = (uint32_t)bg | ((uint32_t)bg << 4) | ((uint32_t)(4 + bg) << 8) | ((uint32_t)(4 + bg) << 12);
    const int NT = (R + 7) >> 3;
    float o[4][4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[a][p][e] = 0.f;
    // producer state (warp 4 lane 0): tile t + kTcStages - 1 is issued as soon as its
    // stage is free (non-blocking probe), tile t at the latest before it is needed
    const int32_t *trow = P.table + (int64_t)ti.req * g.table_stride;
    int issued = 0;
    auto issue_one = [&](int t) {
      const int s = t % kTcStages;
      const int64_t slot0 = (int64_t)trow[(first_blk + t)] * kKernelBlock;
      mbar_arrive_expect_tx(&S.full[s], kTcStageBytes);
      tma_load_3d(smem_u32(smem + s * kTcStageBytes), &T.hmap, head * g.slot_bytes, (int)(slot0 % g.block_tokens),
                  (int)(slot0 / g.block_tokens), &S.full[s]);
    };
    auto pump = [&](int t) -> bool {
      while (issued <= t && issued < nblk) {
        if (issued >= kTcStages &&
            !mbar_wait_bounded(&S.empty[issued % kTcStages], ((issued / kTcStages) - 1) & 1))
          return false;
        issue_one(issued++);
      }
      while (issued < nblk && issued < t + kTcStages) {
        if (issued >= kTcStages && !mbar_test(&S.empty[issued % kTcStages], ((issued / kTcStages) - 1) & 1)) break;
        issue_one(issued++);
      }
      return true;
    };
    for (int t = 0; t < nblk; ++t) {
      const int s = t % kTcStages, b = t & 1;
      if (warp == 4) {
        bool pumped = true;
        if (lane == 0) pumped = pump(t);
        if (!__shfl_sync(0xffffffffu, (int)pumped, 0)) {
          atomicExch(&S.abort, 1);
          break;
        }
      }
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&S.pfull[b], (t >> 1) & 1)) ||
          !__all_sync(0xffffffffu, mbar_wait_bounded(&S.full[s], (t / kTcStages) & 1))) {
        atomicExch(&S.abort, 1);
        break;
      }
      // re-base the accumulators of the rows whose running max moved
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        if (nt >= NT) break;
        const int r0 = 8 * nt + 2 * tq;
        const float a0 = r0 < R ? S.alpha[b][r0] : 1.f, a1 = r0 + 1 < R ? S.alpha[b][r0 + 1] : 1.f;
        if (a0 != 1.f || a1 != 1.f) {
#pragma unroll
          for (int p = 0; p < 4; ++p) o[nt][p][0] *= a0, o[nt][p][1] *= a1, o[nt][p][2] *= a0, o[nt][p][3] *= a1;
        }
      }
      const uint8_t *stage = smem + s * kTcStageBytes + 68;  // V vectors
      const uint32_t pb = smem_u32(smem + kOffP + b * (kTcMaxRows * kPRowBytes));
#pragma unroll 2
      for (int mt = 0; mt < kTcTile / 16; ++mt) {
        const uint8_t *r0 = stage + (16 * mt + 2 * tq) * kTcSlot;
        const uint8_t *r8 = r0 + 8 * kTcSlot;
        const uint32_t x0 = prmt(*reinterpret_cast<const uint32_t *>(r0 + 4 * wlo),
                                 *reinterpret_cast<const uint32_t *>(r0 + kTcSlot + 4 * wlo), sel);
        const uint32_t x1 = prmt(*reinterpret_cast<const uint32_t *>(r0 + 4 * whi),
                                 *reinterpret_cast<const uint32_t *>(r0 + kTcSlot + 4 * whi), sel);
        const uint32_t x2 = prmt(*reinterpret_cast<const uint32_t *>(r8 + 4 * wlo),
                                 *reinterpret_cast<const uint32_t *>(r8 + kTcSlot + 4 * wlo), sel);
        const uint32_t x3 = prmt(*reinterpret_cast<const uint32_t *>(r8 + 4 * whi),
                                 *reinterpret_cast<const uint32_t *>(r8 + kTcSlot + 4 * whi), sel);
        uint32_t pf[4][2];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          if (nt < NT)
            ldmatrix_x2(pf[nt], pb + (uint32_t)((8 * nt + (lane & 7)) * kPRowBytes + (16 * mt + 8 * ((lane >> 3) & 1)) * 2));
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const uint32_t msk = 0x00030003u << (2 * p);
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            if (nt < NT) mma_f16_16816(o[nt][p], x0 & msk, x1 & msk, x2 & msk, x3 & msk, pf[nt][0], pf[nt][1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&S.empty[s]);
        mbar_arrive(&S.pempty[b]);
      }
    }
    if (warp == 4 && lane == 0) {
      // the newest copy of every stage may still be in flight after an abort: let it land
      // (a phase that already completed passes at once)
      for (int t = max(0, issued - kTcStages); t < issued; ++t)
        (void)mbar_wait_bounded(&S.full[t % kTcStages], (t / kTcStages) & 1);
    }
    named_sync(2, kTcThreads);  // row sums of the key warps (pairs with the key warps' barrier 2)
    if (!aborted(S)) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        if (nt >= NT) break;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = 8 * nt + 2 * tq + (e & 1);
          if (r >= R) continue;
          const float L = S.lsum[r];
          const bool any = L > 0.f;
          if (!any && P.balanced) continue;
          const float inv = any ? 1.0f / L : 0.f;
          const float zterm = any ? S.zsum[r] * inv : 0.f;
          const int dbase = 16 * (e < 2 ? wlo : whi) + 4 * bg;
          float4 val;
          val.x = fmaf(o[nt][0][e] * kTwo24, inv, zterm);
          val.y = fmaf(o[nt][1][e] * (kTwo24 / 4.f), inv, zterm);
          val.z = fmaf(o[nt][2][e] * (kTwo24 / 16.f), inv, zterm);
          val.w = fmaf(o[nt][3][e] * (kTwo24 / 64.f), inv, zterm);
          *reinterpret_cast<float4 *>(P.partials + out_row(r) * kDim + dbase) = val;
        }
      }
    }
  }
  if (warp < 4) {
    named_sync(2, kTcThreads);  // pairs with the value warps' barrier 2
    if (tid < R) {  // an aborted CTA marks its rows empty so the merge skips them
      const float L = aborted(S) ? 0.f : S.lsum[tid];
      P.lse[out_row(tid)] = L > 0.f ? (S.mfin[tid] * 0.69314718055994531f + logf(L)) : -INFINITY;
    }
  }
  if (aborted(S) && tid == 0 && P.status) atomicExch(P.status, OSCAR_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

}  // namespace

// History stripe as a [pages][page tokens][kv_heads * 160 B] byte tensor.  The page
// extent only bounds out-of-range fill; every box requested is a block of the request's
// page table, which the caller keeps inside the cache (as for the mma.sync kernel).
int history_tc_launch(const HistParams &P, int32_t num_tasks, cudaStream_t stream) {
  const oscar_geometry &g = P.geo;
  const int rows = g.query_tile * g.group;
  if (rows > kTcMaxRows || g.slot_bytes != kTcSlot || g.block_tokens % kTcTile || encode_fn() == nullptr)
    return OSCAR_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(P.history) & 15) || g.page_bytes % 16) return OSCAR_ERR_UNSUPPORTED;
  HistTcParams T;
  memset(&T, 0, sizeof(T));
  T.P = P;
  T.ncols = rows <= 16 ? 16 : 32;
  cuuint64_t dims[3] = {(cuuint64_t)g.kv_heads * kTcSlot, (cuuint64_t)g.block_tokens, (cuuint64_t)1 << 20};
  cuuint64_t strides[2] = {(cuuint64_t)g.kv_heads * kTcSlot, (cuuint64_t)g.page_bytes};
  cuuint32_t box[3] = {(cuuint32_t)kTcSlot, (cuuint32_t)kTcTile, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  if (encode_fn()(&T.hmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(P.history), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return OSCAR_ERR_UNSUPPORTED;
  if (!ensure_dynamic_smem<history_tc_kernel>(kSmemHistTc)) return OSCAR_ERR_LAUNCH;
  dim3 grid(num_tasks, P.splits, g.kv_heads);
  history_tc_kernel<<<grid, kTcThreads, kSmemHistTc, stream>>>(T);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

}  // namespace oscar
