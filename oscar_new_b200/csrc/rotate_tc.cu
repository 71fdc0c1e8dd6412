// Rotation GEMM on the 5th-generation tensor cores (tcgen05) for large launches,
// with the INT2 clip / quantise / pack / scatter store as its epilogue.
// Reference: oscar_ascend/kernels.py:14-66 (rotate), :69-202 (clip, store_int2).
//
// One CTA = one tile of up to 128 rows (token-head vectors) of one job:
//   Y[128 x 256] = X[128 x 256] . R[256 x 256]   (bf16 operands, fp32 accumulator)
// * TMA brings X (3-D map over [tokens, heads, 256]) and R (2-D map) into shared
//   memory in two 48 KiB stages of K = 64, both with the 128-byte swizzle.  X is the
//   K-major A operand; row-major R is used as an MN-major B operand as it lies
//   (column-major R, e.g. a transposed view, as a K-major one).
// * Thread 0 issues 16 tcgen05.mma (M=128, N=256, K=16) into 256 TMEM columns and
//   commits each stage back to the producer through an mbarrier.
// * Epilogue: warps 0-7 read the accumulator from TMEM (warp w owns lanes 32(w%4)..,
//   column half w/4), round to bf16 and stage the rows in shared memory; then all 16
//   warps run the shared epilogue (rotate.cuh), which writes y and quantises K / V
//   rows, two per warp at a time.  The quantiser is latency-bound (dependent counting
//   passes), so the extra warps (at most 64 registers each) hide its latency: 16 warps
//   per CTA took config 2 from 106 to 89 us against 8.
// About 97 KiB of shared memory and 256 TMEM columns per CTA: two CTAs share an SM, so
// one CTA's epilogue overlaps the other's loads and MMAs.  No multicast anywhere.
// Every mbarrier wait is bounded; after a timeout the CTA lets its copies land, frees
// its TMEM and skips the tile's epilogue.
#include <cstring>

#include "rotate.cuh"
#include "tcgen05.cuh"

namespace oscar {
namespace {

constexpr int kThreads = 512;  // 8 warps drain the accumulator; all 16 quantise
constexpr int kTileM = 128;
constexpr int kChunkK = 64;                          // K per stage
constexpr int kChunks = kDim / kChunkK;              // 4
constexpr int kStagesTc = 2;
constexpr int kAStageBytes = kTileM * kChunkK * 2;   // 16 KiB
constexpr int kBStageBytes = kChunkK * kDim * 2;     // 32 KiB
constexpr int kStageBytesTc = kAStageBytes + kBStageBytes;
constexpr int kBarrierBytes = 64;
constexpr int kSlotBytes = kTileM * 8;             // prefetched slot base offset per token of the tile
constexpr int kSmemTc = kStagesTc * kStageBytesTc + kBarrierBytes + kSlotBytes + 1024;  // + alignment slack
constexpr uint32_t kTmemCols = 256;

struct TcJob {
  int64_t rows;       // n * h
  int64_t tiles;
  int32_t h;
  int32_t tile_rows;  // h * tokens_per_tile (128 when h divides 128)
  int32_t kv;         // -1 plain rotate, 0 K store, 1 V store
  int32_t bsel;       // which B map
  __nv_bfloat16 *y;
};

struct TcParams {
  CUtensorMap amap[3];
  CUtensorMap bmap[3];
  TcJob job[3];
  int32_t b_kmajor[3];
  int32_t njobs;
  RotateParams rp;  // epilogue view (jobs carry n, h, kv, y)
};

// Instruction descriptor, kind::f16: fp32 accumulator (bit 4), A and B bf16 (bits 7,
// 10), A K-major, B major at bit 16, N >> 3 at [17,23), M >> 4 at [24,29).
constexpr uint32_t idesc_bf16(bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(kDim >> 3) << 17) |
         ((uint32_t)(kTileM >> 4) << 24);
}

__global__ void __launch_bounds__(kThreads, 2) rotate_tc_kernel(const __grid_constant__ TcParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStagesTc * kStageBytesTc);
  uint64_t *empty = full + kStagesTc;
  uint64_t *done = empty + kStagesTc;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  int32_t *abort_flag = reinterpret_cast<int32_t *>(tmem_slot + 1);
  int64_t *tile_bases = reinterpret_cast<int64_t *>(smem + kStagesTc * kStageBytesTc + kBarrierBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  int64_t tile = blockIdx.x;
  int j = 0;
  while (j < P.njobs - 1 && tile >= P.job[j].tiles) {
    tile -= P.job[j].tiles;
    ++j;
  }
  const TcJob &job = P.job[j];

  if (tid == 0) {
    for (int s = 0; s < kStagesTc; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  if (job.kv >= 0 && tid >= 32 && tid < 32 + job.tile_rows / job.h) {
    // slot base offsets of the tile's tokens, computed while the GEMM runs (-1: not stored)
    const int64_t token = tile * (job.tile_rows / job.h) + (tid - 32);
    tile_bases[tid - 32] =
        token < P.rp.job[j].n && token < P.rp.counts[1] ? slot_base_offset(P.rp.slots[token], P.rp.geo) : -1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {
    // ---- producer + MMA issuer ----
    const CUtensorMap *amap = &P.amap[j];
    const CUtensorMap *bmap = &P.bmap[job.bsel];
    const bool bk = P.b_kmajor[job.bsel] != 0;
    const uint32_t idesc = idesc_bf16(!bk);
    const int tok0 = (int)(tile * (job.tile_rows / job.h));
    const uint32_t tx = (uint32_t)job.tile_rows * 128u + (uint32_t)kBStageBytes;
    auto load = [&](int c) {
      const int s = c % kStagesTc;
      uint8_t *st = smem + s * kStageBytesTc;
      mbar_arrive_expect_tx(&full[s], tx);
      tma_load_3d(smem_u32(st), amap, c * kChunkK, 0, tok0, &full[s]);
      if (bk) {
        tma_load_2d(smem_u32(st + kAStageBytes), bmap, c * kChunkK, 0, &full[s]);
      } else {
#pragma unroll
        for (int nb = 0; nb < kDim / 64; ++nb)
          tma_load_2d(smem_u32(st + kAStageBytes + nb * 8192), bmap, nb * 64, c * kChunkK, &full[s]);
      }
    };
    load(0);
    load(1);
    int issued = 2, consumed = 0;
    bool ok = true;
    for (int c = 0; c < kChunks; ++c) {
      const int s = c % kStagesTc;
      if (!mbar_wait_bounded(&full[s], (c / kStagesTc) & 1)) {
        ok = false;
        break;
      }
      consumed = c + 1;
      tc_fence_after();
      const uint32_t a0 = smem_u32(smem + s * kStageBytesTc);
      const uint32_t b0 = a0 + kAStageBytes;
#pragma unroll
      for (int kk = 0; kk < kChunkK / 16; ++kk) {
        // A: K-major rows of 128 B, 8-row groups 1024 B apart; K step = 32 B.
        const uint64_t ad = smem_desc(a0 + kk * 32, 16, 1024);
        // B row-major R (MN-major): n-blocks of 64 at 8 KiB, 8-k-row groups at 1 KiB;
        // K step = 16 rows = 2 KiB.  Column-major R (K-major): like A.
        const uint64_t bd = bk ? smem_desc(b0 + kk * 32, 16, 1024) : smem_desc(b0 + kk * 2048, 8192, 1024);
        umma_bf16(tmem, ad, bd, idesc, (c | kk) != 0 ? 1u : 0u);
      }
      umma_commit(&empty[s]);
      if (c + kStagesTc < kChunks) {
        if (!mbar_wait_bounded(&empty[s], 0)) {
          ok = false;
          break;
        }
        load(c + kStagesTc);
        ++issued;
      }
    }
    umma_commit(done);
    if (!ok) {
      *abort_flag = 1;
      // let copies still in flight land (bounded) before the CTA can exit
      for (int c = consumed; c < issued; ++c) (void)mbar_wait_bounded(&full[c % kStagesTc], (c / kStagesTc) & 1);
    }
  }
  // ---- epilogue ----
  const bool landed = mbar_wait_bounded(done, 0);
  tc_fence_after();
  __syncthreads();
  const bool ok = landed && *abort_flag == 0;
  if (!ok && tid == 0 && P.rp.status) atomicExch(P.rp.status, OSCAR_ERR_TIMEOUT);
  __nv_bfloat16 *stage_rows = reinterpret_cast<__nv_bfloat16 *>(smem);  // 64 KiB of the 96
  if (ok && warp < 8) {
    const int q = warp & 3, half = warp >> 2;
    const int r = 32 * q + lane;
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      const int col0 = half * 128 + cb * 32;
      uint32_t v[32];
      tmem_load32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)col0, v);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint4 w;
        w.x = pack_bf162(__uint_as_float(v[8 * ch + 0]), __uint_as_float(v[8 * ch + 1]));
        w.y = pack_bf162(__uint_as_float(v[8 * ch + 2]), __uint_as_float(v[8 * ch + 3]));
        w.z = pack_bf162(__uint_as_float(v[8 * ch + 4]), __uint_as_float(v[8 * ch + 5]));
        w.w = pack_bf162(__uint_as_float(v[8 * ch + 6]), __uint_as_float(v[8 * ch + 7]));
        const int chunk = (col0 >> 3) + ch;
        *reinterpret_cast<uint4 *>(stage_rows + r * kDim + ((chunk ^ (r & 7)) << 3)) = w;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (!ok) return;
  RotateJob rj = P.rp.job[j];
  rotate_epilogue(stage_rows, job.tile_rows, tile * job.tile_rows, rj, P.rp, kThreads / 32, tile_bases);
}

// ---- host side ---------------------------------------------------------------
// X rows (t, h) at x + t*s0 + h*s1: 3-D map {256, h, n}, box {64, h, tokens_per_tile}.
bool encode_rows(CUtensorMap *map, const RotateJob &jb, int tpt) {
  const int64_t s1 = jb.h == 1 ? kDim : jb.s1;
  if ((reinterpret_cast<uintptr_t>(jb.x) & 15) || s1 <= 0 || jb.s0 <= 0 || (s1 * 2) % 16 || (jb.s0 * 2) % 16)
    return false;
  cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)jb.h, (cuuint64_t)jb.n};
  cuuint64_t strides[2] = {(cuuint64_t)(s1 * 2), (cuuint64_t)(jb.s0 * 2)};
  cuuint32_t box[3] = {64u, (cuuint32_t)jb.h, (cuuint32_t)tpt};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<__nv_bfloat16 *>(jb.x), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// R: row-major (bs_n == 1) -> map {n, k} with box {64 n, 64 k} (MN-major operand);
// column-major (bs_k == 1) -> map {k, n} with box {64 k, 256 n} (K-major operand).
bool encode_rotation(CUtensorMap *map, const BMatrix &b, int32_t *kmajor) {
  if (reinterpret_cast<uintptr_t>(b.ptr) & 15) return false;
  const bool rowmajor = b.bs_n == 1;
  const int64_t ld = rowmajor ? b.bs_k : b.bs_n;
  if (ld < kDim || (ld * 2) % 16) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kDim, (cuuint64_t)kDim};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64u, rowmajor ? 64u : (cuuint32_t)kDim};
  cuuint32_t estr[2] = {1u, 1u};
  *kmajor = rowmajor ? 0 : 1;
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16 *>(b.ptr), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int launch_rotate_tc(const RotateParams &p, cudaStream_t stream) {
  if (encode_fn() == nullptr) return OSCAR_ERR_UNSUPPORTED;
  TcParams P;
  memset(&P, 0, sizeof(P));
  P.njobs = p.njobs;
  P.rp = p;
  int nb = 0;
  int64_t total = 0;
  for (int j = 0; j < p.njobs; ++j) {
    const RotateJob &jb = p.job[j];
    if (jb.h <= 0 || jb.h > kTileM) return OSCAR_ERR_UNSUPPORTED;
    const int tpt = kTileM / jb.h;
    if (!encode_rows(&P.amap[j], jb, tpt)) return OSCAR_ERR_UNSUPPORTED;
    int bsel = -1;
    for (int q = 0; q < j; ++q)
      if (p.job[q].r.ptr == jb.r.ptr && p.job[q].r.bs_k == jb.r.bs_k && p.job[q].r.bs_n == jb.r.bs_n)
        bsel = P.job[q].bsel;
    if (bsel < 0) {
      if (!encode_rotation(&P.bmap[nb], jb.r, &P.b_kmajor[nb])) return OSCAR_ERR_UNSUPPORTED;
      bsel = nb++;
    }
    TcJob &t = P.job[j];
    t.rows = jb.n * jb.h;
    t.h = jb.h;
    t.tile_rows = tpt * jb.h;
    t.tiles = (jb.n + tpt - 1) / tpt;
    t.kv = jb.kv;
    t.bsel = bsel;
    t.y = jb.y;
    P.rp.job[j].tiles = t.tiles;
    total += t.tiles;
  }
  if (total == 0) return OSCAR_OK;
  if (!ensure_dynamic_smem<rotate_tc_kernel>(kSmemTc)) return OSCAR_ERR_LAUNCH;
  rotate_tc_kernel<<<(unsigned)total, kThreads, kSmemTc, stream>>>(P);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

}  // namespace oscar
