// Covariance Gram accumulation on the 5th-generation tensor cores (tcgen05):
//   cov[g][i][j] += sum over the rows r of head group g of x_r[i] * y_r[j],
// y = x (query Grams) or y = w_r x_r (the SST-weighted value Grams), for bf16 rows x of
// 256 dims.  Reference: oscar_ascend/calibration_kernels.py:59-70 (accumulate_gram).
//
// One CTA = one head group x a range of tokens, accumulating the full 256 x 256 fp32
// Gram in all 512 tensor-memory columns (rows i as TMEM lanes: two M = 128 halves).
// * A producer thread brings 64-row blocks of X into shared memory with 3-D TMA copies
//   (map {256 dims, heads, tokens}, box {64 dims, heads of the group, tokens}, 128-byte
//   swizzle, no multicast): four 8 KiB boxes per block, one per 64 dims.  A group of
//   `hpg` heads fills hpg * floor(64 / hpg) rows of a block; the rows past that stay
//   zero (zeroed once) and add nothing.
// * The block is both operands as it lies: dims are contiguous, so X^T is an MN-major
//   A operand (M = dims of one half) and X an MN-major B operand (N = 256 dims); the
//   issuer thread runs, per 16 rows, tcgen05.mma M = 128, N = 256, K = 16 for both
//   halves (kind::f16, bf16 in, fp32 accumulate) and commits each stage back.
// * Weighted Grams: four converter warps write y = w x into two more buffers of the
//   same swizzled layout as bf16 hi + lo (hi = bf16(w x), lo = bf16(w x - hi)), and the
//   issuer runs the hi and lo products into the same accumulator.  bf16 x bf16 products
//   are exact in fp32, so this matches the mma.sync Gram's arithmetic.
// * Epilogue: the four converter / epilogue warps (one per TMEM lane quarter) read the
//   accumulator and add it into cov with vector atomics.
// Every mbarrier wait is bounded; on a timeout the CTA raises the status word (when
// given), lets its copies land and skips the epilogue.
#include <algorithm>
#include <cstring>

#include "tcgen05.cuh"

namespace oscar {
namespace {

constexpr int kGtRows = 64;                   // rows (K) per block
constexpr int kGtBoxBytes = kGtRows * 128;    // 64 rows x 64 dims bf16 = 8 KiB
constexpr int kGtXBytes = 4 * kGtBoxBytes;    // 32 KiB: 4 boxes of 64 dims
constexpr int kGtThreads = 192;               // warp 0 producer, warp 1 issuer, warps 2-5 convert / epilogue
constexpr uint32_t kGtCols = 512;

struct GramTcParams {
  CUtensorMap xmap;
  const float *w;     // nullable: per-row weights, index token * h + head
  float *cov;         // [groups][256][256]
  int64_t n;          // tokens
  int32_t h, hpg;     // heads, heads per group
  int32_t tpb;        // tokens per block (hpg * tpb <= 64)
  int32_t blocks_per_cta;
  int32_t ctas_per_group;
  int32_t *status;
};

template <int STAGES, bool WEIGHTED>
struct GtLayout {
  static constexpr int stage = WEIGHTED ? 3 * kGtXBytes : kGtXBytes;
  static constexpr int bars = STAGES * stage;
  static constexpr int bytes = bars + 256;
  static constexpr int smem = bytes + 1024;  // alignment slack
};

// kind::f16, fp32 accumulator (bit 4), A and B bf16 (bits 7, 10), both MN-major (bits
// 15, 16), N = 256 (>> 3 at [17, 23)), M = 128 (>> 4 at [24, 29)).
constexpr uint32_t kGtIdesc =
    (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

template <int STAGES, bool WEIGHTED>
__global__ void __launch_bounds__(kGtThreads, 1) gram_tc_kernel(const __grid_constant__ GramTcParams P) {
  using L = GtLayout<STAGES, WEIGHTED>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::bars);
  uint64_t *conv = full + STAGES;   // weighted: hi / lo parts written
  uint64_t *empty = conv + STAGES;  // the stage's MMAs have completed
  uint64_t *done = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  int32_t *abort_flag = reinterpret_cast<int32_t *>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int group = blockIdx.x / P.ctas_per_group;
  const int part = blockIdx.x % P.ctas_per_group;
  const int64_t blocks_total = (P.n + P.tpb - 1) / P.tpb;
  const int64_t b0 = (int64_t)part * P.blocks_per_cta;
  const int64_t left = blocks_total - b0;
  const int nblk = left <= 0 ? 0 : (int)(left < P.blocks_per_cta ? left : P.blocks_per_cta);

  // zero every buffer once: rows a block does not fill stay zero
  for (int i = tid; i < STAGES * L::stage / 16; i += kGtThreads)
    reinterpret_cast<uint4 *>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kGtCols);
  fence_async_smem();  // the zeroed buffers are visible to the async proxy (TMA, MMA)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int rows_per_block = P.hpg * P.tpb;
  const uint32_t tx = 4u * 128u * (uint32_t)rows_per_block;

  if (warp == 0 && lane == 0) {
    // ---- producer ----
    for (int b = 0; b < nblk; ++b) {
      const int s = b % STAGES;
      if (b >= STAGES && !mbar_wait_bounded(&empty[s], ((b / STAGES) - 1) & 1)) {
        atomicExch(abort_flag, 1);
        break;
      }
      if (*reinterpret_cast<volatile int32_t *>(abort_flag)) break;
      const uint32_t dst = smem_u32(smem + s * L::stage);
      mbar_arrive_expect_tx(&full[s], tx);
      const int tok = (int)((b0 + b) * P.tpb);
#pragma unroll
      for (int nb = 0; nb < 4; ++nb)
        tma_load_3d(dst + nb * kGtBoxBytes, &P.xmap, nb * 64, group * P.hpg, tok, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    bool ok = true;
    for (int b = 0; b < nblk && ok; ++b) {
      const int s = b % STAGES;
      ok = mbar_wait_bounded(&full[s], (b / STAGES) & 1) && (!WEIGHTED || mbar_wait_bounded(&conv[s], (b / STAGES) & 1));
      if (!ok || *reinterpret_cast<volatile int32_t *>(abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t x0 = smem_u32(smem + s * L::stage);
#pragma unroll
      for (int kk = 0; kk < kGtRows / 16; ++kk) {
        // MN-major operands: 64-element blocks 8 KiB apart, 8-row groups 1 KiB apart;
        // 16 rows of K = 2 KiB.
#pragma unroll
        for (int yp = 0; yp < (WEIGHTED ? 2 : 1); ++yp) {
          const uint32_t y0 = WEIGHTED ? x0 + (uint32_t)(1 + yp) * kGtXBytes : x0;
          const uint64_t bd = smem_desc(y0 + kk * 2048, 8192, 1024);
#pragma unroll
          for (int ti = 0; ti < 2; ++ti) {
            const uint64_t ad = smem_desc(x0 + ti * 16384 + kk * 2048, 8192, 1024);
            umma_bf16(tmem + (uint32_t)(ti * 256), ad, bd, kGtIdesc, (b | kk | yp) != 0 ? 1u : 0u);
          }
        }
      }
      umma_commit(&empty[s]);
    }
    if (!ok) atomicExch(abort_flag, 1);
    umma_commit(done);  // arrives once every MMA issued above has completed
  } else if (warp >= 2 && WEIGHTED) {
    // ---- converters: y = w x as bf16 hi + lo, same swizzled positions as x ----
    const int ct = tid - 64;  // 0..127
    for (int b = 0; b < nblk; ++b) {
      const int s = b % STAGES;
      if (!mbar_wait_bounded(&full[s], (b / STAGES) & 1)) {
        atomicExch(abort_flag, 1);
        break;
      }
      if (*reinterpret_cast<volatile int32_t *>(abort_flag)) break;
      uint8_t *xs = smem + s * L::stage;
      const int64_t tok0 = (b0 + b) * P.tpb;
      // 2048 chunks of 16 bytes: box nb, row r, chunk c (position XOR-swizzled by r & 7)
      for (int q = ct; q < 4 * kGtRows * 8; q += 128) {
        const int nb = q >> 9, r = (q >> 3) & 63;
        const int off = nb * kGtBoxBytes + r * 128 + (q & 7) * 16;
        float wt = 0.f;
        if (r < rows_per_block) {
          const int64_t t = tok0 + r / P.hpg;
          if (t < P.n) wt = P.w[t * P.h + group * P.hpg + r % P.hpg];
        }
        const uint4 xv = *reinterpret_cast<const uint4 *>(xs + off);
        const uint32_t vv[4] = {xv.x, xv.y, xv.z, xv.w};
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float y0 = wt * bf16_bits_to_float(vv[e] & 0xffffu);
          const float y1 = wt * bf16_bits_to_float(vv[e] >> 16);
          hi[e] = pack_bf162(y0, y1);
          lo[e] = pack_bf162(y0 - bf16_bits_to_float(hi[e] & 0xffffu), y1 - bf16_bits_to_float(hi[e] >> 16));
        }
        *reinterpret_cast<uint4 *>(xs + kGtXBytes + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4 *>(xs + 2 * kGtXBytes + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
      // the next write into this stage's hi / lo buffers follows the TMA of block
      // b + STAGES, which the producer issues only after these MMAs completed
    }
  }

  // ---- epilogue: warps 2-5, one TMEM lane quarter each ----
  __syncwarp();
  if (warp >= 2) {
    const bool landed = mbar_wait_bounded(done, 0);
    tc_fence_after();
    const bool ok = landed && *reinterpret_cast<volatile int32_t *>(abort_flag) == 0 && nblk > 0;
    if (!ok && nblk > 0 && lane == 0 && P.status) atomicExch(P.status, OSCAR_ERR_TIMEOUT);
    if (ok) {
      const int q = warp & 3;
      float *cov = P.cov + (size_t)group * kDim * kDim;
#pragma unroll 1
      for (int ti = 0; ti < 2; ++ti) {
        const int i = ti * 128 + 32 * q + lane;
#pragma unroll 1
        for (int cb = 0; cb < 8; ++cb) {
          uint32_t v[32];
          tmem_load32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(ti * 256 + cb * 32), v);
          float4 *dst = reinterpret_cast<float4 *>(cov + (size_t)i * kDim + cb * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            atomicAdd(dst + e, make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                           __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3])));
        }
      }
    }
  }
  // copies of an aborted run still land before the CTA exits
  if (warp == 0 && lane == 0 && *reinterpret_cast<volatile int32_t *>(abort_flag)) {
    for (int b = nblk > STAGES ? nblk - STAGES : 0; b < nblk; ++b)
      (void)mbar_wait_bounded(&full[b % STAGES], (b / STAGES) & 1, 4096);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kGtCols);
  }
}

template <int STAGES, bool WEIGHTED>
int launch_gram_tc(const GramTcParams &P, int grid, cudaStream_t stream) {
  using L = GtLayout<STAGES, WEIGHTED>;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(gram_tc_kernel<STAGES, WEIGHTED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                L::smem);
  });
  if (attr != cudaSuccess) return OSCAR_ERR_LAUNCH;
  gram_tc_kernel<STAGES, WEIGHTED><<<grid, kGtThreads, L::smem, stream>>>(P);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

}  // namespace

// Gram on tcgen05; OSCAR_ERR_UNSUPPORTED when the layout does not fit a tensor map
// (the caller then uses the mma.sync Gram).
int gram_tc_launch(const void *x, int64_t n, int32_t h, int64_t xs0, int64_t xs1, int32_t groups,
                   const float *weights, float *cov, int32_t *status, int sm_count, cudaStream_t stream) {
  const int hpg = h / groups;
  if (hpg > kGtRows || encode_fn() == nullptr || n > (int64_t)INT32_MAX) return OSCAR_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (xs0 * 2) % 16 || (xs1 * 2) % 16 || xs0 <= 0 || xs1 <= 0)
    return OSCAR_ERR_UNSUPPORTED;
  GramTcParams P;
  memset(&P, 0, sizeof(P));
  cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)h, (cuuint64_t)n};
  cuuint64_t strides[2] = {(cuuint64_t)(xs1 * 2), (cuuint64_t)(xs0 * 2)};
  P.tpb = kGtRows / hpg;
  cuuint32_t box[3] = {64u, (cuuint32_t)hpg, (cuuint32_t)P.tpb};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  if (encode_fn()(&P.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(x), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return OSCAR_ERR_UNSUPPORTED;
  P.w = weights;
  P.cov = cov;
  P.n = n;
  P.h = h;
  P.hpg = hpg;
  P.status = status;
  // At most one wave (about sm_count CTAs over the groups).  Query Grams: at least 8
  // blocks per CTA, since every CTA ends with 64 Ki atomic adds into the same 256 KiB of
  // cov and fewer, longer CTAs beat a full wave of short ones on small calls.  Weighted
  // Grams: the converter warps' w x split dominates a block, so the blocks spread over
  // the full wave (at 1024 tokens x 4 KV heads: 64 CTAs, 2.2x faster than 8 CTAs of 8
  // blocks, despite the atomics).
  const int64_t blocks = (n + P.tpb - 1) / P.tpb;
  const int64_t per_group = std::max<int64_t>(1, sm_count / groups);
  const int64_t min_blocks = weights ? 1 : 8;
  int64_t bpc = std::max<int64_t>(min_blocks, (blocks + per_group - 1) / per_group);
  P.blocks_per_cta = (int32_t)std::min<int64_t>(bpc, INT32_MAX);
  P.ctas_per_group = (int32_t)((blocks + bpc - 1) / bpc);
  const int grid = groups * P.ctas_per_group;
  if (grid <= 0) return OSCAR_OK;
  return weights ? launch_gram_tc<2, true>(P, grid, stream) : launch_gram_tc<4, false>(P, grid, stream);
}

}  // namespace oscar
