// INT2 history split-KV attention on the 5th-generation tensor cores with 8-bit
// operands: the decode history kernel (reference oscar_ascend/kernels.py:290-436,
// RAW=False; same split, mask and LSE semantics as history_attention_kernel).
//
// Arithmetic.
// * Keys.  The reference rounds every dequantised key element to bf16, so a token's 256
//   key elements take only its four levels v_c = bf16(c*s + z).  Scaled by a power of
//   two (largest |v_c| in [128, 256)), each level is the exact sum of two e4m3 numbers
//   hi_c + lo_c (an 8-bit significand split 4 + 4).  The token's two 4-byte tables
//   (hi_0..hi_3, lo_0..lo_3) turn four 2-bit codes into four e4m3 operand bytes with one
//   PRMT each: nibble selectors x & 0x33333333 (even code positions) and
//   (x >> 2) & 0x33333333 (odd ones), 13 integer instructions per 16 codes for both
//   parts.  Thread = token = TMEM lane writes its 512 operand bytes (hi for the 256
//   dims, then lo) into tensor memory, the A operand of a TS-form tcgen05.mma
//   (kind::f8f6f4, M = 128 tokens, N = 16, K = 32 per instruction, 16 instructions).
//   The query row r is split the same way (q * 2^e = qhi + qlo exactly for bf16 q) into
//   B columns r (qhi) and 8 + r (qlo), so S[t][r] + S[t][8 + r] = q_r . k_t * 2^(e_r+e_t)
//   with all four cross products, in fp32.
// * Values.  sum_t p_t v_t = sum_t (p_t s_t) c_t + sum_t p_t z_t.  A code byte masked
//   with 0x03030303 or 0x0C0C0C0C (before or after >> 4) is an e4m3 bit pattern in
//   0..15, where e4m3 is exactly linear: pattern k is k * 2^-9, so the masked codes are
//   c * 2^-9 or c * 2^-7.  One 16-byte chunk per code word holds its 16 codes; the V^T
//   tile (M = dims in that permuted order, K = tokens, MN-major, no swizzle, 16-byte pad
//   per M group so the stores hit distinct banks) is the A operand of an SS-form
//   tcgen05.mma whose B operand is P'^T with P'_t = p_t s_t split into two e4m3 parts
//   (columns r and 8 + r).  P' is formed as 2^(logit + log2 s_t - m) with m the row's
//   running maximum of logit + log2 s minus 4, re-based lazily when a logit passes
//   m + 4: P' stays in (0, 256], inside e4m3 range, and l = sum P' / s, zp = sum P' z/s
//   are accumulated in fp32 from the unrounded P'.
//
// Work.  Persistent CTAs (one per SM) walk work items (task, split, KV-head group);
// splits are 128-token-block aligned in the balanced (decode step) mode, so every block
// is read by one CTA.  A tile is one 128-token kernel block of one KV head (20 KiB of
// slots, one 3-D TMA copy, no multicast); the heads of a block are consecutive tiles so
// the four heads of a token row are fetched together.  Warp roles:
//   0-3   softmax (thread = TMEM lane = token): scores, lazy max, P', l, zp; item epilogue
//   4-7   key operands (thread = token = TMEM lane)
//   8-9   value operands (lane = one code word of one token; conflict-free loads/stores)
//   10    producer (lane 0: TMA copies into a 5-stage ring)
//   11    query operands (double buffered, one item ahead) and the -inf marks of unused splits
//   12-15 MMA issuers, one per KV head of the CTA (lane 0), one per SM sub-partition: a
//         small tcgen05.mma keeps its issuing thread busy for tens of cycles, and four
//         issuers working at once raise the rate about fourfold (measured on B200).
//         Each polls its head's score and value streams and issues whichever is ready.
// Tensor memory: key A operand x2 (256 columns), scores x2 (32), O^T per head (2 M
// tiles x 16 columns), and each softmax thread's running l / zp per head (16 columns
// per head, loaded and stored with the scores of every tile instead of held in registers).  Every mbarrier wait is bounded; a timeout raises a CTA abort
// flag and the device status word, every role leaves at its next wait, copies in flight
// land, issued MMAs complete, tensor memory is freed, and the CTA marks its rows -inf.
#include <cstring>

#include "history_common.cuh"
#include "tcgen05.cuh"

namespace oscar {
namespace {

constexpr int kF8Tile = 128;  // tokens per tile: one kernel block of one KV head
constexpr int kF8Slot = 160;
constexpr int kF8StageBytes = kF8Tile * kF8Slot;  // 20 KiB
constexpr int kF8Stages = 5;
constexpr int kF8Rows = 8;         // query rows per KV head (padded)
constexpr int kF8N = 2 * kF8Rows;  // MMA N: rows x {hi, lo} part
constexpr int kF8MaxHeads = 4;
constexpr int kF8MaxTasks = 1024;
constexpr int kF8Warps = 16;  // 4 per SM sub-partition: 128 registers per thread
constexpr int kF8Threads = 32 * kF8Warps;
constexpr int kWarpKey0 = 4, kWarpVal0 = 8, kWarpProd = 10, kWarpQ = 11, kWarpMma0 = 12;
constexpr int kValWarps = kWarpProd - kWarpVal0;
constexpr float kF8Slack = 4.f;   // re-base when a logit passes the running max by 2^4
constexpr float kF8Offset = 4.f;  // P' = 2^(x - (m - 4)) <= 2^8 right after a re-base

constexpr uint32_t kColA = 0;  // 2 x 128 columns
constexpr uint32_t kColS = 256;
constexpr uint32_t kColO = kColS + 2 * kF8N;
constexpr uint32_t kColL = kColO + kF8MaxHeads * 2 * kF8N;  // per-lane running row sums l, zp
constexpr uint32_t kTmemCols = 512;

constexpr int kQHeadBytes = 256 * kF8N;  // K-major B: 16 chunks of [16 rows x 16 bytes]
constexpr int kQBufBytes = kF8MaxHeads * kQHeadBytes;
constexpr int kOffQ = 0;  // two buffers
constexpr int kOffStage = kOffQ + 2 * kQBufBytes;
constexpr int kVtSbo = 2064;  // stride of the 16-byte M groups of a V^T tile (16 B pad)
constexpr int kVtTileBytes = 8 * kVtSbo;
constexpr int kVtBufBytes = 2 * kVtTileBytes;
constexpr int kOffVt = kOffStage + kF8Stages * kF8StageBytes;
constexpr int kPBufBytes = kF8Tile * kF8N;
constexpr int kOffP = kOffVt + 2 * kVtBufBytes;
constexpr int kOffTok = kOffP + 2 * kPBufBytes;  // per-token softmax inputs, float4 x 128, x2
constexpr int kOffSmall = kOffTok + 2 * kF8Tile * 16;

struct F8Small {
  uint64_t full[kF8Stages], empty[kF8Stages];
  // per-tile barriers, set t % 4, phase t / 4: one issuer's tiles of a set are consecutive
  // phases, and every wait on another tile's set is at most one phase behind (its previous
  // phase was already waited on), so parity waits are never ambiguous
  uint64_t akey[4], sfull[4], sempty[4], vfull[4], pfull[4], vdone[4];
  uint64_t qfull[2], qempty[2], ofree;
  uint64_t hvdone[kF8MaxHeads];  // phase k: the k-th value MMA group of head h has completed
  uint64_t mmadone[kF8MaxHeads];
  float qfac[2][kF8MaxHeads][kF8Rows];
  float mrun[kF8MaxHeads][kF8Rows];
  float wmax[4][kF8Rows];
  float red[4][kF8MaxHeads][kF8Rows][2];
  float fin[kF8MaxHeads][kF8Rows][2];
  int32_t flags[2][4];
  uint32_t tmem;
  int32_t abort;
  int32_t span;
  int32_t n_items;
  int32_t pref[kF8MaxTasks + 1];
};
constexpr int kF8Smem = kOffSmall + (int)sizeof(F8Small);
static_assert(kF8Smem <= 227 * 1024, "shared memory budget");
static_assert(kColL + kF8MaxHeads * 2 * kF8Rows <= kTmemCols, "tensor memory budget");

struct F8Params {
  CUtensorMap hmap;  // history stripe as [pages][page tokens][kv_heads * 160 B], uint8
  HistParams P;
  int32_t nhg;            // KV-head groups (kv_heads / HG)
  int32_t withhold_tile;  // test hook: CTA 0's producer never issues this tile (-1: none)
  uint32_t wait_probes;   // bounded-wait limit
};

struct F8Item {
  TaskInfo ti;
  int split, hgrp, rows;
  int lo, hi, blk0, nblk;
};

OSCAR_DEVINL volatile int32_t &abort_word(F8Small &S) { return *reinterpret_cast<volatile int32_t *>(&S.abort); }

// Bounded wait on an mbarrier phase.  Each probe may suspend the thread for up to 4 us
// (it wakes when the phase completes), so waiting warps do not spin; the wait gives up at
// the probe limit (about 4 s at the default), raising the CTA abort flag and the status
// word, or as soon as another role has raised the flag.
constexpr uint32_t kF8ProbeNs = 4000;
OSCAR_DEVINL bool f8_wait(uint64_t *bar, uint32_t parity, F8Small &S, const F8Params &T) {
  for (uint32_t i = 0; i < T.wait_probes; ++i) {
    if (mbar_try_wait_sleep(bar, parity, kF8ProbeNs)) return true;
    if ((i & 7u) == 7u && abort_word(S) != 0) return false;
  }
  atomicExch(&S.abort, 1);
  if (T.P.status) atomicExch(T.P.status, OSCAR_ERR_TIMEOUT);
  return false;
}

// Every lane waits (each gets the acquire); the warp proceeds only if all lanes did.
OSCAR_DEVINL bool f8_warp_wait(uint64_t *bar, uint32_t parity, F8Small &S, const F8Params &T) {
  return __all_sync(0xffffffffu, f8_wait(bar, parity, S, T));
}

// Wait that ignores the abort flag: used on the way out so copies and MMAs in flight
// finish before shared or tensor memory is released.
OSCAR_DEVINL void f8_drain(uint64_t *bar, uint32_t parity, uint32_t probes) {
  for (uint32_t i = 0; i < probes; ++i)
    if (mbar_try_wait(bar, parity)) return;
}

OSCAR_DEVINL void named_sync128() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

OSCAR_DEVINL int blocks_of(const TaskInfo &ti) {
  const int length = ti.recent_begin - ti.sink_len;
  return length > 0 ? (ti.recent_begin - 1) / kKernelBlock - ti.sink_len / kKernelBlock + 1 : 0;
}

// Balanced mode: splits of whole 128-token blocks, ceil(length / span) of them (at most
// `splits`), trimmed so that none is empty.  Returns the blocks per split in *per.
OSCAR_DEVINL int balanced_splits(const TaskInfo &ti, int span, int splits, int *per) {
  *per = 0;
  if (!ti.live || ti.qlen <= 0) return 0;
  const int length = ti.recent_begin - ti.sink_len;
  const int nb = blocks_of(ti);
  if (nb <= 0) return 0;
  const int want = max(1, min(splits, (length + span - 1) / span));
  const int ps = (nb + want - 1) / want;
  *per = ps;
  return (nb + ps - 1) / ps;
}

OSCAR_DEVINL F8Item f8_item(const F8Params &T, const F8Small &S, int j, int HG) {
  const HistParams &P = T.P;
  const oscar_geometry &g = P.geo;
  F8Item it{};
  int task;
  if (P.balanced) {
    const int nt = min(P.task_count[0], P.num_tasks);
    int lo = 0, hi = nt;  // largest task with pref[task] <= j
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (S.pref[mid] <= j) lo = mid;
      else hi = mid;
    }
    task = lo;
    const int r = j - S.pref[task];
    it.split = r / T.nhg;
    it.hgrp = r % T.nhg;
  } else {
    task = j / (P.splits * T.nhg);
    it.split = (j / T.nhg) % P.splits;
    it.hgrp = j % T.nhg;
  }
  it.ti = load_task(task, P.tasks, P.task_count, P.qstarts, P.seq_lens, P.counts, g);
  const TaskInfo &ti = it.ti;
  if (!ti.live || ti.qlen <= 0) return it;  // rows = 0, nblk = 0: nothing to write
  it.rows = min(g.query_tile, ti.qoff < ti.qlen ? ti.qlen - ti.qoff : 0) * g.group;
  if (P.balanced) {
    int per = 0;
    balanced_splits(ti, S.span, P.splits, &per);
    const int b_first = ti.sink_len / kKernelBlock;
    const int nb = blocks_of(ti);
    it.blk0 = b_first + it.split * per;
    it.nblk = min(per, nb - it.split * per);
    it.lo = max(ti.sink_len, it.blk0 * kKernelBlock);
    it.hi = min(ti.recent_begin, (it.blk0 + it.nblk) * kKernelBlock);
  } else {
    // the reference's split of [sink_len, recent_begin): 32-token granules
    const int length = ti.recent_begin - ti.sink_len;
    const int tiles32 = (length + 31) / 32;
    const int per_split = ((tiles32 + P.splits - 1) / P.splits) * 32;
    const int begin = it.split * per_split;
    const int end = min(begin + per_split, length);
    it.lo = ti.sink_len + begin;
    it.hi = ti.sink_len + max(end, begin);
    if (it.hi > it.lo) {
      it.blk0 = it.lo / kKernelBlock;
      it.nblk = (it.hi - 1) / kKernelBlock - it.blk0 + 1;
    }
  }
  return it;
}

OSCAR_DEVINL int64_t f8_out_row(const F8Item &it, const oscar_geometry &g, int HG, int h, int r, int split_slots) {
  const int tok = it.ti.qstart + it.ti.qoff + r / g.group;
  const int qh = (it.hgrp * HG + h) * g.group + r % g.group;
  return ((int64_t)tok * g.kv_heads * g.group + qh) * split_slots + it.split;
}

// Walks this CTA's tiles of one KV head in order: items blockIdx.x, blockIdx.x +
// gridDim.x, ... that have blocks, each nblk blocks x HG heads (head fastest).  t is the
// CTA-wide tile index, i the tile index within the item, kq the ordinal of the item.
struct F8Cursor {
  int j, kq, ntile, i, t;
  bool done;
  OSCAR_DEVINL void seek(const F8Params &T, const F8Small &S, int n_items, int HG) {
    while (j < n_items) {
      const F8Item it = f8_item(T, S, j, HG);
      if (it.nblk > 0) {
        ntile = it.nblk * HG;
        return;
      }
      j += gridDim.x;
    }
    done = true;
  }
  OSCAR_DEVINL void start(const F8Params &T, const F8Small &S, int n_items, int HG, int head) {
    j = blockIdx.x, kq = 0, ntile = 0, i = head, t = head, done = false;
    seek(T, S, n_items, HG);
  }
  OSCAR_DEVINL void next(const F8Params &T, const F8Small &S, int n_items, int HG, int head) {
    t += HG;
    i += HG;
    if (i < ntile) return;
    ++kq;
    i = head;
    j += gridDim.x;
    seek(T, S, n_items, HG);
  }
};

// The token's two e4m3 tables of its four bf16 key levels (bytes c = level c) and the
// power of two that undoes their scale.  Invalid tokens get zero tables.
OSCAR_DEVINL void key_tables(uint32_t ksz, bool valid, uint32_t &thi, uint32_t &tlo, float &tokfac) {
  const float s = half_bits_to_float(ksz & 0xffffu), z = half_bits_to_float(ksz >> 16);
  const float v0 = round_bf16(z);
  const float v1 = round_bf16(__fadd_rn(s, z));
  const float v2 = round_bf16(__fadd_rn(2.f * s, z));
  const float v3 = round_bf16(__fadd_rn(3.f * s, z));
  // s >= 2^-14 for every written slot, so the levels increase and max |v| is at an end
  const uint32_t ex = (__float_as_uint(fmaxf(fabsf(v0), fabsf(v3))) >> 23) & 0xffu;
  const uint32_t exc = ex < 16u ? 16u : (ex > 250u ? 250u : ex);
  const float up = __uint_as_float((261u - exc) << 23);  // 2^(134 - ex): max |v| -> [128, 256)
  const uint32_t w01 = pack_half2(v0 * up, v1 * up), w23 = pack_half2(v2 * up, v3 * up);
  const uint32_t h01 = e4m3x2_from_f16x2(w01), h23 = e4m3x2_from_f16x2(w23);
  const uint32_t l01 = e4m3x2_from_f16x2(hsub2_bits(w01, f16x2_from_e4m3x2(h01)));
  const uint32_t l23 = e4m3x2_from_f16x2(hsub2_bits(w23, f16x2_from_e4m3x2(h23)));
  thi = valid ? (h01 | (h23 << 16)) : 0u;
  tlo = valid ? (l01 | (l23 << 16)) : 0u;
  tokfac = valid ? __uint_as_float((exc - 7u) << 23) : 0.f;  // 2^(ex - 134)
}

// M index m (0..127) of V^T tile mt -> head dimension, and the e4m3 code scale to undo.
OSCAR_DEVINL int vt_dim(int m, int mt) {
  const int w = 8 * mt + (m >> 4), i = m & 15;
  return 16 * w + 4 * (i & 3) + (i >> 2);
}
OSCAR_DEVINL float vt_fac(int m) { return ((m >> 2) & 1) ? 128.f : 512.f; }

// ---------------------------------------------------------------------------------
template <int HG>
__global__ void __launch_bounds__(kF8Threads, 1) history_f8_kernel(const __grid_constant__ F8Params T) {
  // used directly (no integer round trip for alignment), so the compiler keeps every
  // access in the shared address space; no layout here needs more than 128-byte alignment
  extern __shared__ __align__(128) uint8_t smem[];
  F8Small &S = *reinterpret_cast<F8Small *>(smem + kOffSmall);
  const HistParams &P = T.P;
  const oscar_geometry &g = P.geo;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kF8Stages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 4 + kValWarps);  // key + value warps
    }
    for (int b = 0; b < 2; ++b) {

      mbar_init(&S.qfull[b], 1);
      mbar_init(&S.qempty[b], HG + 4);  // each issuer's last score MMA of the item + 4 softmax warps
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&S.akey[b], 4);
      mbar_init(&S.sfull[b], 1);
      mbar_init(&S.sempty[b], 4);
      mbar_init(&S.vfull[b], kValWarps);
      mbar_init(&S.pfull[b], 4);
      mbar_init(&S.vdone[b], 1);
    }
    mbar_init(&S.ofree, 4);
    for (int h = 0; h < kF8MaxHeads; ++h) {
      mbar_init(&S.hvdone[h], 1);
      mbar_init(&S.mmadone[h], 1);
    }
    S.abort = 0;
    fence_mbarrier_init();
  }
  if (tid < kF8MaxHeads * kF8Rows) S.mrun[tid / kF8Rows][tid % kF8Rows] = -INFINITY;
  if (warp == 0) {
    // work items: balanced mode counts each live task's splits (prefix sums in shared
    // memory); the reference mode has `splits` per task
    const int nt = min(P.task_count[0], P.num_tasks);
    if (P.balanced) {
      int64_t total = 0;
      for (int t2 = lane; t2 < nt; t2 += 32) {
        const TaskInfo tj = load_task(t2, P.tasks, P.task_count, P.qstarts, P.seq_lens, P.counts, g);
        if (tj.live && tj.qlen > 0) total += max(0, tj.recent_begin - tj.sink_len);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
      const int64_t span0 = (total * T.nhg + P.target_ctas - 1) / max(P.target_ctas, 1);
      const int span = (int)(span0 < kMinSplitTokens ? (int64_t)kMinSplitTokens
                                                     : (span0 > (1 << 30) ? (int64_t)(1 << 30) : span0));
      int run = 0;
      for (int base = 0; base < nt; base += 32) {
        const int t2 = base + lane;
        int cnt = 0, per = 0;
        if (t2 < nt) {
          const TaskInfo tj = load_task(t2, P.tasks, P.task_count, P.qstarts, P.seq_lens, P.counts, g);
          cnt = balanced_splits(tj, span, P.splits, &per) * T.nhg;
        }
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        if (t2 < nt) S.pref[t2 + 1] = run + incl;
        run += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) {
        S.pref[0] = 0;
        S.span = span;
        S.n_items = run;
      }
    } else if (lane == 0) {
      S.span = 0;
      S.n_items = nt * P.splits * T.nhg;
    }
  }
  if (warp == kWarpMma0) tmem_alloc(&S.tmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;
  const int n_items = S.n_items;
  const int step = gridDim.x;

  if (warp == kWarpProd) {
    // ===================== producer: one TMA copy per tile =====================
    if (lane == 0) {
      int t = 0;
      bool ok = true;
      for (int j = blockIdx.x; j < n_items && ok; j += step) {
        const F8Item it = f8_item(T, S, j, HG);
        if (it.nblk <= 0) continue;
        const int32_t *trow = P.table + (int64_t)it.ti.req * g.table_stride;
        for (int b = 0; b < it.nblk && ok; ++b) {
          const int64_t slot0 = (int64_t)trow[it.blk0 + b] * kKernelBlock;
          const int page = (int)(slot0 / g.block_tokens), y = (int)(slot0 % g.block_tokens);
          for (int h = 0; h < HG; ++h, ++t) {
            const int s = t % kF8Stages;
            if (t >= kF8Stages && !f8_wait(&S.empty[s], ((t / kF8Stages) - 1) & 1, S, T)) {
              ok = false;
              break;
            }
            if (blockIdx.x == 0 && t == T.withhold_tile) continue;  // test hook
            mbar_arrive_expect_tx(&S.full[s], kF8StageBytes);
            tma_load_3d(smem_u32(smem + kOffStage + s * kF8StageBytes), &T.hmap, (it.hgrp * HG + h) * kF8Slot, y,
                        page, &S.full[s]);
          }
        }
      }
      // copies still in flight land before the CTA can exit (phases already complete pass)
      for (int u = max(0, t - kF8Stages); u < t; ++u)
        if (!(blockIdx.x == 0 && u == T.withhold_tile)) f8_drain(&S.full[u % kF8Stages], (u / kF8Stages) & 1, T.wait_probes);
    }
  } else if (warp >= kWarpMma0) {
    // ===================== MMA issuers: one per KV head =====================
    // Issuer h handles the tiles of head h.  Scores (16 MMAs of tile t) need A(t) and the
    // S buffer back from the softmax of tile t - 2; values (8 MMAs of tile t) need P'(t),
    // V^T(t) and, on an item's first block, the O columns back from the last epilogue.
    // The two streams are polled, never waited on one after the other.
    const int hi = warp - kWarpMma0;
    if (lane == 0 && hi < HG) {
      const uint32_t idk = idesc_e4m3_m128(kF8N, false, false);
      const uint32_t idv = idesc_e4m3_m128(kF8N, true, true);
      F8Cursor kc, vc;
      kc.start(T, S, n_items, HG, hi);
      vc.start(T, S, n_items, HG, hi);
      uint32_t idle = 0;
      const uint32_t idle_limit = T.wait_probes * 8u;  // backed-off polls, a few seconds at the default limit
      while (!vc.done) {
        bool did = false;
        if (!kc.done) {
          const int t = kc.t, a = t & 1;
          if (mbar_test(&S.akey[t & 3], (t >> 2) & 1) && (t < 2 || mbar_test(&S.sempty[(t - 2) & 3], ((t - 2) >> 2) & 1)) &&
              (kc.i >= HG || mbar_test(&S.qfull[kc.kq & 1], (kc.kq >> 1) & 1))) {
            tc_fence_after();
            const uint32_t d = tmem + kColS + (uint32_t)(a * kF8N);
            const uint32_t at = tmem + kColA + (uint32_t)(a * 128);
            // the start-address field (bits 0-13, 16-byte units) advances by 32 per 32-byte
            // K step; the other fields of a descriptor are fixed
            const uint64_t qd =
                smem_desc_plain(smem_u32(smem + kOffQ + (kc.kq & 1) * kQBufBytes + hi * kQHeadBytes), kF8N * 16, 128);
#pragma unroll
            for (int k = 0; k < 16; ++k) umma_f8_ts(d, at + 8 * k, qd + (uint64_t)(32 * (k & 7)), idk, k > 0 ? 1u : 0u);
            umma_commit(&S.sfull[t & 3]);
            if (kc.i >= kc.ntile - HG) umma_commit(&S.qempty[kc.kq & 1]);
            kc.next(T, S, n_items, HG, hi);
            did = true;
          }
        }
        if (vc.t < kc.t) {
          const int t = vc.t, a = t & 1;
          const bool first = vc.i < HG;
          if ((!first || vc.kq == 0 || mbar_test(&S.ofree, (vc.kq - 1) & 1)) && mbar_test(&S.pfull[t & 3], (t >> 2) & 1) &&
              mbar_test(&S.vfull[t & 3], (t >> 2) & 1)) {
            tc_fence_after();
            const uint64_t pd = smem_desc_plain(smem_u32(smem + kOffP + a * kPBufBytes), 128, 2048);
            const uint64_t vd = smem_desc_plain(smem_u32(smem + kOffVt + a * kVtBufBytes), 128, kVtSbo);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              const uint32_t d = tmem + kColO + (uint32_t)((hi * 2 + mt) * kF8N);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_f8(d, vd + (uint64_t)(mt * (kVtTileBytes >> 4) + 32 * k), pd + (uint64_t)(32 * k), idv,
                        (first && k == 0) ? 0u : 1u);
            }
            umma_commit(&S.vdone[t & 3]);
            umma_commit(&S.hvdone[hi]);
            vc.next(T, S, n_items, HG, hi);
            did = true;
          }
        }
        if (did) {
          idle = 0;
        } else if (++idle >= idle_limit) {
          atomicExch(&S.abort, 1);
          if (P.status) atomicExch(P.status, OSCAR_ERR_TIMEOUT);
          break;
        } else if ((idle & 63u) == 0u && abort_word(S) != 0) {
          break;
        } else {
          // nothing ready: back off, so the polling thread does not take issue slots from
          // the softmax and key warps of its sub-partition
          __nanosleep(idle < 4 ? 32u : (idle < 16 ? 128u : 512u));
        }
      }
      umma_commit(&S.mmadone[hi]);
      f8_drain(&S.mmadone[hi], 0, T.wait_probes);  // this issuer's MMAs complete before teardown
    }
  } else if (warp == kWarpQ) {
    // ===================== query operands (+ unused-split marks) =====================
    if (P.balanced) {
      const int nt = min(P.task_count[0], P.num_tasks);
      for (int u = blockIdx.x; u < nt * P.splits; u += step) {
        const int t2 = u / P.splits, sp = u % P.splits;
        if (sp * T.nhg < S.pref[t2 + 1] - S.pref[t2]) continue;
        const TaskInfo tj = load_task(t2, P.tasks, P.task_count, P.qstarts, P.seq_lens, P.counts, g);
        if (!tj.live || tj.qlen <= 0) continue;
        const int rows = min(g.query_tile, tj.qoff < tj.qlen ? tj.qlen - tj.qoff : 0) * g.group;
        for (int i = lane; i < g.kv_heads * rows; i += 32) {
          const int h = i / rows, r = i % rows;
          const int tok = tj.qstart + tj.qoff + r / g.group;
          const int qh = h * g.group + r % g.group;
          P.lse[((int64_t)tok * g.kv_heads * g.group + qh) * P.split_slots + sp] = -INFINITY;
        }
      }
    }
    int kq = 0;
    for (int j = blockIdx.x; j < n_items; j += step) {
      const F8Item it = f8_item(T, S, j, HG);
      if (it.nblk <= 0) continue;
      const int qb = kq & 1;
      if (kq >= 2 && !f8_warp_wait(&S.qempty[qb], ((kq >> 1) - 1) & 1, S, T)) break;
      uint8_t *qbuf = smem + kOffQ + qb * kQBufBytes;
      for (int h = 0; h < HG; ++h)
        for (int r = 0; r < kF8Rows; ++r) {
          // lane: dims 8*lane .. 8*lane+7 of row r (word lane/2 of the key operand order)
          uint4 raw = make_uint4(0, 0, 0, 0);
          const bool valid = r < it.rows;
          if (valid) {
            const int tok = it.ti.qstart + it.ti.qoff + r / g.group;
            const int qh = (it.hgrp * HG + h) * g.group + r % g.group;
            raw = *reinterpret_cast<const uint4 *>(P.query + (int64_t)tok * P.qs0 + (int64_t)qh * P.qs1 + 8 * lane);
          }
          float q[8];
          q[0] = bf16_bits_to_float(raw.x & 0xffffu), q[1] = bf16_bits_to_float(raw.x >> 16);
          q[2] = bf16_bits_to_float(raw.y & 0xffffu), q[3] = bf16_bits_to_float(raw.y >> 16);
          q[4] = bf16_bits_to_float(raw.z & 0xffffu), q[5] = bf16_bits_to_float(raw.z >> 16);
          q[6] = bf16_bits_to_float(raw.w & 0xffffu), q[7] = bf16_bits_to_float(raw.w >> 16);
          float amax = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(q[e]));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
          const uint32_t ex = (__float_as_uint(amax) >> 23) & 0xffu;
          const uint32_t exc = ex < 16u ? 16u : (ex > 250u ? 250u : ex);
          const bool any = valid && amax > 0.f;
          const float up = any ? __uint_as_float((261u - exc) << 23) : 0.f;
          // even dims of this lane -> word A (q index 0 / 1), odd dims -> word B (2 / 3)
          uint32_t hA = 0, hB = 0, lA = 0, lB = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float xa = q[2 * e] * up, xb = q[2 * e + 1] * up;
            const uint32_t hh = e4m3x2_from_f32(xa, xb);  // bits 0-7: even dim, 8-15: odd dim
            const uint32_t hf = f16x2_from_e4m3x2(hh);
            const float ra = xa - __half2float(__ushort_as_half((unsigned short)(hf & 0xffffu)));
            const float rb = xb - __half2float(__ushort_as_half((unsigned short)(hf >> 16)));
            const uint32_t ll = e4m3x2_from_f32(ra, rb);
            hA |= (hh & 0xffu) << (8 * e), hB |= ((hh >> 8) & 0xffu) << (8 * e);
            lA |= (ll & 0xffu) << (8 * e), lB |= ((ll >> 8) & 0xffu) << (8 * e);
          }
          const int w = lane >> 1, qa = (lane & 1) ? 1 : 0, qbq = qa + 2;
          uint8_t *chunk = qbuf + h * kQHeadBytes + w * (kF8N * 16);
          *reinterpret_cast<uint32_t *>(chunk + r * 16 + 4 * qa) = hA;
          *reinterpret_cast<uint32_t *>(chunk + r * 16 + 4 * qbq) = hB;
          *reinterpret_cast<uint32_t *>(chunk + (kF8Rows + r) * 16 + 4 * qa) = lA;
          *reinterpret_cast<uint32_t *>(chunk + (kF8Rows + r) * 16 + 4 * qbq) = lB;
          if (lane == 0) S.qfac[qb][h][r] = any ? __uint_as_float((exc - 7u) << 23) * P.scale_log2 : 0.f;
        }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.qfull[qb]);
      ++kq;
    }
  } else if (warp >= kWarpKey0 && warp < kWarpVal0) {
    // ===================== key operands: thread = token = TMEM lane =====================
    const int tau = 32 * (warp & 3) + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    float4 *tokbuf = reinterpret_cast<float4 *>(smem + kOffTok);
    int t = 0;
    bool ok = true;
    for (int j = blockIdx.x; j < n_items && ok; j += step) {
      const F8Item it = f8_item(T, S, j, HG);
      if (it.nblk <= 0) continue;
      for (int b = 0; b < it.nblk && ok; ++b) {
        const int pos = (it.blk0 + b) * kF8Tile + tau;
        const bool valid = pos >= it.lo && pos < it.hi;
        for (int h = 0; h < HG; ++h, ++t) {
          const int s = t % kF8Stages, a = t & 1;
          if (!f8_warp_wait(&S.full[s], (t / kF8Stages) & 1, S, T)) {
            ok = false;
            break;
          }
          const uint8_t *row = smem + kOffStage + s * kF8StageBytes + tau * kF8Slot;
          const uint32_t ksz = *reinterpret_cast<const uint32_t *>(row + 64);
          const uint32_t vsz = *reinterpret_cast<const uint32_t *>(row + 132);
          if (t >= 2 && !f8_warp_wait(&S.sempty[(t - 2) & 3], ((t - 2) >> 2) & 1, S, T)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t thi, tlo;
          float tokfac;
          key_tables(ksz, valid, thi, tlo, tokfac);
          const float vs = half_bits_to_float(vsz & 0xffffu), vz = half_bits_to_float(vsz >> 16);
          const float rvs = valid ? __fdividef(1.f, vs) : 0.f;
          float4 info;
          info.x = tokfac;
          info.y = valid ? __log2f(vs) : -INFINITY;
          info.z = rvs;
          info.w = valid ? vz * rvs : 0.f;
          tokbuf[a * kF8Tile + tau] = info;
          // the codes are read group by group (a compact loop), so the stage is released
          // after the last group
#pragma unroll 1
          for (int grp = 0; grp < 4; ++grp) {
            uint32_t hv[16], lv[16];
            const uint4 kq4 = *reinterpret_cast<const uint4 *>(row + 16 * grp);
            const uint32_t kw[4] = {kq4.x, kq4.y, kq4.z, kq4.w};
#pragma unroll
            for (int w2 = 0; w2 < 4; ++w2) {
              const uint32_t x = kw[w2];
              const uint32_t sa = x & 0x33333333u, sb = (x >> 2) & 0x33333333u;
              const uint32_t sa2 = sa >> 16, sb2 = sb >> 16;
              hv[4 * w2 + 0] = prmt(thi, thi, sa), hv[4 * w2 + 1] = prmt(thi, thi, sa2);
              hv[4 * w2 + 2] = prmt(thi, thi, sb), hv[4 * w2 + 3] = prmt(thi, thi, sb2);
              lv[4 * w2 + 0] = prmt(tlo, tlo, sa), lv[4 * w2 + 1] = prmt(tlo, tlo, sa2);
              lv[4 * w2 + 2] = prmt(tlo, tlo, sb), lv[4 * w2 + 3] = prmt(tlo, tlo, sb2);
            }
            tmem_store16(lane_base + kColA + (uint32_t)(a * 128 + 16 * grp), hv);
            tmem_store16(lane_base + kColA + (uint32_t)(a * 128 + 64 + 16 * grp), lv);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.empty[s]);
          tmem_store_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.akey[t & 3]);
        }
      }
    }
  } else if (warp >= kWarpVal0 && warp < kWarpProd) {
    // ===================== value operands: V^T tile in shared memory =====================
    // lane = (token, code word): rounds of 4 tokens; warp wv takes tokens {wv, wv + 2}
    // of each round, so the two tokens of one load are 320 bytes apart and the 32 loads
    // hit 32 distinct banks
    const int wv = warp - kWarpVal0;
    const int word = lane & 15;
    const int tok_off = wv + 2 * (lane >> 4);
    int t = 0;
    bool ok = true;
    for (int j = blockIdx.x; j < n_items && ok; j += step) {
      const F8Item it = f8_item(T, S, j, HG);
      if (it.nblk <= 0) continue;
      const int ntile = it.nblk * HG;
      for (int i = 0; i < ntile; ++i, ++t) {
        const int s = t % kF8Stages, a = t & 1;
        if (!f8_warp_wait(&S.full[s], (t / kF8Stages) & 1, S, T)) {
          ok = false;
          break;
        }
        if (t >= 2 && !f8_warp_wait(&S.vdone[(t - 2) & 3], ((t - 2) >> 2) & 1, S, T)) {
          ok = false;
          break;
        }
        const uint8_t *src = smem + kOffStage + s * kF8StageBytes + 68 + 4 * word;
        uint8_t *dst = smem + kOffVt + a * kVtBufBytes + (word >> 3) * kVtTileBytes + (word & 7) * kVtSbo;
        // four chunks of 8 rounds (a compact loop); the stage is released after the last
#pragma unroll 1
        for (int r0 = 0; r0 < 32; r0 += 8) {
          uint32_t x[8];
#pragma unroll
          for (int r = 0; r < 8; ++r)
            x[r] = *reinterpret_cast<const uint32_t *>(src + (4 * (r0 + r) + tok_off) * kF8Slot);
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const uint32_t xs = x[r] >> 4;
            *reinterpret_cast<uint4 *>(dst + (4 * (r0 + r) + tok_off) * 16) =
                make_uint4(x[r] & 0x03030303u, x[r] & 0x0C0C0C0Cu, xs & 0x03030303u, xs & 0x0C0C0C0Cu);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.vfull[t & 3]);
      }
    }
  } else {
    // ===================== softmax: thread = token = TMEM lane (warps 0-3) =====================
    // The four warps meet at named barriers, so no warp may leave alone: a failed wait
    // only clears this warp's `ok`; the decision to stop is taken from the votes that all
    // four read after the same barrier (vote slots alternate, so a slot is rewritten only
    // after every warp has passed the barrier that follows its reading).
    const int tau = tid;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
    const float4 *tokbuf = reinterpret_cast<const float4 *>(smem + kOffTok);
    int t = 0, kq = 0, vc = 0;
    int blocks_done = 0;  // blocks of every item before the current one and of this item so far
    bool ok = true, stop = false;
    int jfail = n_items;
    // all four warps: returns the OR of their `bits` (bit 0: failed wait, bit 1: re-base)
    auto vote = [&](int bits) -> int {
      if (lane == 0) S.flags[vc & 1][warp] = bits;
      named_sync128();
      const int v = S.flags[vc & 1][0] | S.flags[vc & 1][1] | S.flags[vc & 1][2] | S.flags[vc & 1][3];
      ++vc;
      return v;
    };
    for (int j = blockIdx.x; j < n_items && !stop; j += step) {
      const F8Item it = f8_item(T, S, j, HG);
      if (it.rows <= 0) continue;
      if (it.nblk <= 0) {
        // reference mode, empty split range: zero partials, lse -inf
        for (int e = tau; e < HG * it.rows * kDim; e += 128) {
          const int hr = e / kDim, d = e % kDim;
          const int64_t orow = f8_out_row(it, g, HG, hr / it.rows, hr % it.rows, P.split_slots);
          P.partials[orow * kDim + d] = 0.f;
          if (d == 0) P.lse[orow] = -INFINITY;
        }
        continue;
      }
      const int qb = kq & 1;
      if (ok && !f8_warp_wait(&S.qfull[qb], (kq >> 1) & 1, S, T)) ok = false;
      {
        uint32_t zero[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) zero[e] = 0u;
#pragma unroll
        for (int h = 0; h < HG; ++h) tmem_store16(lane_base + kColL + (uint32_t)(16 * h), zero);
      }
      const int item_blocks0 = blocks_done;
      for (int b = 0; b < it.nblk && !stop; ++b, ++blocks_done) {
#pragma unroll 1
        for (int h = 0; h < HG; ++h) {
          if (stop) break;
          const int a = t & 1;
          if (ok && (!f8_warp_wait(&S.akey[t & 3], (t >> 2) & 1, S, T) || !f8_warp_wait(&S.sfull[t & 3], (t >> 2) & 1, S, T)))
            ok = false;
          float lg[kF8Rows], m[kF8Rows];
          float4 info = make_float4(0.f, -INFINITY, 0.f, 0.f);
          uint32_t lz[16];  // this thread's running l (0..7) and zp (8..15) of head h
          bool need = false;
          if (ok) {
            tc_fence_after();
            uint32_t sv[16];
            tmem_store_wait();  // the previous store of the l / zp columns has landed
            tmem_load16x2(lane_base + kColS + (uint32_t)(a * kF8N), sv, lane_base + kColL + (uint32_t)(16 * h), lz);
            info = tokbuf[a * kF8Tile + tau];
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.sempty[t & 3]);
#pragma unroll
            for (int r = 0; r < kF8Rows; ++r) {
              const float dot = __uint_as_float(sv[r]) + __uint_as_float(sv[kF8Rows + r]);
              lg[r] = fmaf(dot, info.x * S.qfac[qb][h][r], info.y);
              m[r] = S.mrun[h][r];
              if (r < it.rows) need |= lg[r] > m[r] + kF8Slack || (m[r] == -INFINITY && lg[r] > -INFINITY);
            }
          } else {
#pragma unroll
            for (int r = 0; r < kF8Rows; ++r) lg[r] = -INFINITY, m[r] = -INFINITY;
#pragma unroll
            for (int e = 0; e < 16; ++e) lz[e] = 0u;
          }
          const int v = vote((ok ? 0 : 1) | (__any_sync(0xffffffffu, need) ? 2 : 0));
          if (v & 1) {
            stop = true;
            break;
          }
          if (v & 2) {
            // re-base: exact row maxima of this tile over the 128 tokens
#pragma unroll
            for (int r = 0; r < kF8Rows; ++r) {
              const int key = __float_as_int(lg[r]);
              const int mk = __reduce_max_sync(0xffffffffu, key >= 0 ? key : key ^ 0x7fffffff);
              if (lane == 0) S.wmax[warp][r] = __int_as_float(mk >= 0 ? mk : mk ^ 0x7fffffff);
            }
            named_sync128();
            float alpha[kF8Rows];
            bool resc = false;
#pragma unroll
            for (int r = 0; r < kF8Rows; ++r) {
              const float tm = fmaxf(fmaxf(S.wmax[0][r], S.wmax[1][r]), fmaxf(S.wmax[2][r], S.wmax[3][r]));
              const float mo = m[r];
              const bool up = r < it.rows && (tm > mo + kF8Slack || (mo == -INFINITY && tm > -INFINITY));
              const float mn = up ? tm : mo;
              alpha[r] = (up && mo != -INFINITY) ? ex2(mo - mn) : 1.f;
              resc |= alpha[r] != 1.f;
              m[r] = mn;
            }
            if (resc) {
              // the head's earlier value MMAs complete before its O columns are re-based in
              // place (m was finite, so this item has an earlier block of head h)
              if (blocks_done > item_blocks0 &&
                  !f8_warp_wait(&S.hvdone[h], (blocks_done - 1) & 1, S, T))
                ok = false;
              if (ok) {
                tc_fence_after();
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                  uint32_t ov[16];
                  const uint32_t oaddr = lane_base + kColO + (uint32_t)((h * 2 + mt) * kF8N);
                  tmem_load16(oaddr, ov);
#pragma unroll
                  for (int r = 0; r < kF8Rows; ++r) {
                    ov[r] = __float_as_uint(__uint_as_float(ov[r]) * alpha[r]);
                    ov[kF8Rows + r] = __float_as_uint(__uint_as_float(ov[kF8Rows + r]) * alpha[r]);
                  }
                  tmem_store16(oaddr, ov);
                }
                tmem_store_wait();
              }
#pragma unroll
              for (int r = 0; r < kF8Rows; ++r) {
                lz[r] = __float_as_uint(__uint_as_float(lz[r]) * alpha[r]);
                lz[kF8Rows + r] = __float_as_uint(__uint_as_float(lz[kF8Rows + r]) * alpha[r]);
              }
            }
            if (tau < kF8Rows) S.mrun[h][tau] = m[tau];
            if (vote(ok ? 0 : 1) & 1) {
              stop = true;
              break;
            }
          }
          uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
#pragma unroll
          for (int r = 0; r < kF8Rows; r += 2) {
            const float ms0 = m[r] == -INFINITY ? 0.f : m[r] - kF8Offset;
            const float ms1 = m[r + 1] == -INFINITY ? 0.f : m[r + 1] - kF8Offset;
            const float p0 = ex2(lg[r] - ms0), p1 = ex2(lg[r + 1] - ms1);
            lz[r] = __float_as_uint(fmaf(p0, info.z, __uint_as_float(lz[r])));
            lz[r + 1] = __float_as_uint(fmaf(p1, info.z, __uint_as_float(lz[r + 1])));
            lz[kF8Rows + r] = __float_as_uint(fmaf(p0, info.w, __uint_as_float(lz[kF8Rows + r])));
            lz[kF8Rows + r + 1] = __float_as_uint(fmaf(p1, info.w, __uint_as_float(lz[kF8Rows + r + 1])));
            const uint32_t ph = pack_half2(p0, p1);
            const uint32_t eh = e4m3x2_from_f16x2(ph);
            const uint32_t el = e4m3x2_from_f16x2(hsub2_bits(ph, f16x2_from_e4m3x2(eh)));
            hw[r >> 2] |= eh << (16 * ((r >> 1) & 1));
            lw[r >> 2] |= el << (16 * ((r >> 1) & 1));
          }
          if (ok) tmem_store16(lane_base + kColL + (uint32_t)(16 * h), lz);
          if (ok && t >= 2 && !f8_warp_wait(&S.vdone[(t - 2) & 3], ((t - 2) >> 2) & 1, S, T)) ok = false;
          if (ok) {
            *reinterpret_cast<uint4 *>(smem + kOffP + a * kPBufBytes + tau * 16) =
                make_uint4(hw[0], hw[1], lw[0], lw[1]);
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.pfull[t & 3]);
          }
          ++t;
        }
      }
      if (stop) {
        jfail = j;
        break;
      }
      // ---- item epilogue: row sums over the 128 token lanes, O^T -> partials ----
      tmem_store_wait();
#pragma unroll 1
      for (int h = 0; h < HG; ++h) {
        uint32_t lzh[16];
        tmem_load16(lane_base + kColL + (uint32_t)(16 * h), lzh);
#pragma unroll
        for (int r = 0; r < kF8Rows; ++r) {
          float lv = __uint_as_float(lzh[r]), zv = __uint_as_float(lzh[kF8Rows + r]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            lv += __shfl_xor_sync(0xffffffffu, lv, o);
            zv += __shfl_xor_sync(0xffffffffu, zv, o);
          }
          if (lane == 0) S.red[warp][h][r][0] = lv, S.red[warp][h][r][1] = zv;
        }
      }
      // every head's last value MMAs of the item
      for (int h = 0; h < HG && ok; ++h)
        if (!f8_warp_wait(&S.hvdone[h], (blocks_done - 1) & 1, S, T)) ok = false;
      if (vote(ok ? 0 : 1) & 1) {
        jfail = j;
        break;
      }
      tc_fence_after();
      if (tau < HG * kF8Rows) {
        const int h = tau / kF8Rows, r = tau % kF8Rows;
        S.fin[h][r][0] = (S.red[0][h][r][0] + S.red[1][h][r][0]) + (S.red[2][h][r][0] + S.red[3][h][r][0]);
        S.fin[h][r][1] = (S.red[0][h][r][1] + S.red[1][h][r][1]) + (S.red[2][h][r][1] + S.red[3][h][r][1]);
      }
      named_sync128();
      const int d0 = vt_dim(tau, 0), d1 = vt_dim(tau, 1);
      const float fac = vt_fac(tau);
#pragma unroll 1
      for (int h = 0; h < HG; ++h) {
        uint32_t o0[16], o1[16];
        tmem_load16(lane_base + kColO + (uint32_t)((h * 2 + 0) * kF8N), o0);
        tmem_load16(lane_base + kColO + (uint32_t)((h * 2 + 1) * kF8N), o1);
#pragma unroll
        for (int r = 0; r < kF8Rows; ++r) {
          if (r >= it.rows) break;
          const float L = S.fin[h][r][0];
          const bool any = L > 0.f;
          if (!any && P.balanced) continue;  // the merge skips -inf splits without reading them
          const float inv = any ? 1.f / L : 0.f;
          const float zt = any ? S.fin[h][r][1] * inv : 0.f;
          float *dst = P.partials + f8_out_row(it, g, HG, h, r, P.split_slots) * kDim;
          dst[d0] = fmaf((__uint_as_float(o0[r]) + __uint_as_float(o0[kF8Rows + r])) * fac, inv, zt);
          dst[d1] = fmaf((__uint_as_float(o1[r]) + __uint_as_float(o1[kF8Rows + r])) * fac, inv, zt);
        }
      }
      if (tau < HG * it.rows) {
        const int h = tau / it.rows, r = tau % it.rows;
        const float L = S.fin[h][r][0];
        const float ms = S.mrun[h][r] == -INFINITY ? 0.f : S.mrun[h][r] - kF8Offset;
        P.lse[f8_out_row(it, g, HG, h, r, P.split_slots)] =
            L > 0.f ? (ms + __log2f(L)) * 0.69314718055994531f : -INFINITY;
      }
      tc_fence_before();
      named_sync128();
      if (tau < kF8MaxHeads * kF8Rows) S.mrun[tau / kF8Rows][tau % kF8Rows] = -INFINITY;
      named_sync128();
      if (lane == 0) {
        mbar_arrive(&S.ofree);
        mbar_arrive(&S.qempty[qb]);
      }
      ++kq;
    }
    if (jfail < n_items) {
      // aborted: mark every row of the remaining items empty, so no merge reads a stale partial
      for (int j = jfail; j < n_items; j += step) {
        const F8Item it = f8_item(T, S, j, HG);
        for (int e = tau; e < HG * it.rows; e += 128)
          P.lse[f8_out_row(it, g, HG, e / it.rows, e % it.rows, P.split_slots)] = -INFINITY;
      }
    }
  }

  __syncwarp();  // lanes that skipped a lane-0 role rejoin before the block barrier
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int HG>
int launch_f8(F8Params &T, int grid, cudaStream_t stream, int priority) {
  if (!ensure_dynamic_smem<history_f8_kernel<HG>>(kF8Smem)) return OSCAR_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kF8Threads);
  cfg.dynamicSmemBytes = kF8Smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributePriority;
  attr[0].val.priority = priority;
  cfg.attrs = attr;
  cfg.numAttrs = priority != 0 ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, history_f8_kernel<HG>, T) != cudaSuccess) return OSCAR_ERR_LAUNCH;
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

}  // namespace

int history_f8_launch(const HistParams &P, int32_t num_tasks, int sm_count, cudaStream_t stream, int priority) {
  const oscar_geometry &g = P.geo;
  const int rows = g.query_tile * g.group;
  if (rows > kF8Rows || g.slot_bytes != kF8Slot || g.head_dim != kDim || g.kernel_block != kKernelBlock ||
      g.block_tokens % kF8Tile || num_tasks > kF8MaxTasks || encode_fn() == nullptr)
    return OSCAR_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(P.history) & 15) || g.page_bytes % 16) return OSCAR_ERR_UNSUPPORTED;
  const int hg = g.kv_heads % 4 == 0 ? 4 : (g.kv_heads % 2 == 0 ? 2 : 1);
  F8Params T;
  memset(&T, 0, sizeof(T));
  T.P = P;
  T.nhg = g.kv_heads / hg;
  T.withhold_tile = P.withhold;
  T.wait_probes = P.wait_probes;
  // work items per CTA: the balanced split span targets `target_ctas` items in all
  if (P.balanced) T.P.target_ctas = sm_count * 6;
  cuuint64_t dims[3] = {(cuuint64_t)g.kv_heads * kF8Slot, (cuuint64_t)g.block_tokens, (cuuint64_t)1 << 20};
  cuuint64_t strides[2] = {(cuuint64_t)g.kv_heads * kF8Slot, (cuuint64_t)g.page_bytes};
  cuuint32_t box[3] = {(cuuint32_t)kF8Slot, (cuuint32_t)kF8Tile, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  if (encode_fn()(&T.hmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(P.history), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return OSCAR_ERR_UNSUPPORTED;
  // an upper bound of the items is enough for the grid: surplus CTAs find no item
  const int64_t max_items = (int64_t)num_tasks * P.splits * T.nhg;
  const int grid = (int)std::min<int64_t>(max_items, sm_count);
  if (grid <= 0) return OSCAR_OK;
  if (hg == 4) return launch_f8<4>(T, grid, stream, priority);
  if (hg == 2) return launch_f8<2>(T, grid, stream, priority);
  return launch_f8<1>(T, grid, stream, priority);
}

}  // namespace oscar
