// SST weights on the 5th-generation tensor cores (tcgen05): w_r = max(k_r C_h k_r^T, 0)
// for the key rows r of each KV head h, and totals[h] += sum_r w_r (reference
// oscar_ascend/calibration_kernels.py:109-126, sst_weights).
//
// C_h (fp32) is split once per calibration pass into three bf16 parts whose sum is C_h
// exactly (hi + mid + lo carry its 24 significand bits: split_bf16x3_kernel).  A bf16 x
// bf16 product is exact in fp32, so D = K (C_hi + C_mid + C_lo)^T accumulated in fp32 is
// the fp32 product K C_h^T up to the order of the additions, as in the mma.sync SST
// kernel (calibration.cu).  k C k^T is a scalar, so C or C^T give the same weight.
//
// One CTA = 128 key rows of one head:
// * warp 0 (one thread): 3-D TMA copies, no multicast, 128-byte swizzle: the key tile
//   (four boxes of 128 rows x 64 dims) once, then the twelve [256 rows x 64 dims] blocks
//   of the three parts through a 3-stage ring;
// * warp 1 (one thread): tcgen05.mma kind::f16, M = 128 rows, N = 256, K = 16, both
//   operands K-major, all twelve blocks into one 256-column fp32 accumulator in tensor
//   memory, each stage committed back to the producer;
// * warps 2-5 (one TMEM lane quarter each): w_r = sum_j D[r][j] k_r[j] from the
//   accumulator and the key tile in shared memory, clamped at 0, stored, and summed into
//   totals[h].
// Rows past the last key row read the TMA's zero fill and are not stored.  Every wait is
// bounded; a timeout raises the status word (when given), lets the copies land and
// skips the stores.
#include <cstring>
#include <mutex>

#include "tcgen05.cuh"

namespace oscar {
namespace {

constexpr int kStRows = 128;                       // key rows per CTA (M)
constexpr int kStKBox = kStRows * 128;             // 128 rows x 64 dims bf16 = 16 KiB
constexpr int kStKBytes = 4 * kStKBox;             // 64 KiB: the key tile
constexpr int kStBBytes = 256 * 128;               // 256 rows x 64 dims bf16 = 32 KiB
constexpr int kStStages = 3;
constexpr int kStBlocks = 3 * 4;                   // (part, 64-dim block)
constexpr int kStThreads = 192;
constexpr uint32_t kStCols = 256;

struct SstTcParams {
  CUtensorMap kmap;  // {256 dims, heads, rows}
  CUtensorMap cmap;  // {256 dims, 256 rows of C, 3 * heads parts}
  float *w;          // [rows * heads], index row * heads + head
  float *totals;     // [heads]
  int64_t n;
  int32_t h;
  int32_t *status;
};

struct SstSmem {
  uint64_t kfull, full[kStStages], empty[kStStages], done;
  uint32_t tmem;
  int32_t abort;
};

// kind::f16, fp32 accumulator (bit 4), A and B bf16 (bits 7, 10), both K-major, N = 256
// (>> 3 at [17, 23)), M = 128 (>> 4 at [24, 29)).
constexpr uint32_t kStIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((128u >> 4) << 24);
constexpr int kStSmem = kStKBytes + kStStages * kStBBytes + 1024 /* SstSmem */ + 1024 /* alignment */;

__global__ void __launch_bounds__(kStThreads, 1) sst_tcgen05_kernel(const __grid_constant__ SstTcParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *ktile = smem;
  uint8_t *ring = smem + kStKBytes;
  SstSmem &S = *reinterpret_cast<SstSmem *>(ring + kStStages * kStBBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int head = blockIdx.y;
  const int64_t r0 = (int64_t)blockIdx.x * kStRows;

  if (tid == 0) {
    mbar_init(&S.kfull, 1);
    for (int s = 0; s < kStStages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    mbar_init(&S.done, 1);
    S.abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) tmem_alloc(&S.tmem, kStCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;

  if (warp == 0 && lane == 0) {
    // ---- producer ----
    mbar_arrive_expect_tx(&S.kfull, kStKBytes);
#pragma unroll
    for (int b = 0; b < 4; ++b) tma_load_3d(smem_u32(ktile + b * kStKBox), &P.kmap, 64 * b, head, (int)r0, &S.kfull);
    for (int i = 0; i < kStBlocks; ++i) {
      const int s = i % kStStages;
      if (i >= kStStages && !mbar_wait_bounded(&S.empty[s], ((i / kStStages) - 1) & 1)) {
        atomicExch(&S.abort, 1);
        break;
      }
      if (*reinterpret_cast<volatile int32_t *>(&S.abort)) break;
      mbar_arrive_expect_tx(&S.full[s], kStBBytes);
      tma_load_3d(smem_u32(ring + s * kStBBytes), &P.cmap, 64 * (i & 3), 0, 3 * head + (i >> 2), &S.full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: block i = part i / 4, dims 64 (i % 4) .. + 63 ----
    bool ok = mbar_wait_bounded(&S.kfull, 0);
    for (int i = 0; i < kStBlocks && ok; ++i) {
      const int s = i % kStStages;
      ok = mbar_wait_bounded(&S.full[s], (i / kStStages) & 1) && !*reinterpret_cast<volatile int32_t *>(&S.abort);
      if (!ok) break;
      tc_fence_after();
      const uint32_t a0 = smem_u32(ktile + (i & 3) * kStKBox), b0 = smem_u32(ring + s * kStBBytes);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16(tmem, smem_desc(a0 + kk * 32, 16, 1024), smem_desc(b0 + kk * 32, 16, 1024), kStIdesc,
                  (i | kk) != 0 ? 1u : 0u);
      umma_commit(&S.empty[s]);
    }
    if (!ok) atomicExch(&S.abort, 1);
    umma_commit(&S.done);  // arrives once every MMA issued above has completed
  }

  // ---- epilogue: warps 2-5, rows 32 (warp % 4) + lane ----
  __syncwarp();
  if (warp >= 2) {
    const bool landed = mbar_wait_bounded(&S.done, 0);
    tc_fence_after();
    const bool ok = landed && *reinterpret_cast<volatile int32_t *>(&S.abort) == 0;
    if (!ok && lane == 0 && P.status) atomicExch(P.status, OSCAR_ERR_TIMEOUT);
    const int q = warp & 3, row = 32 * q + lane;
    float sum = 0.f;
    if (ok) {
#pragma unroll 1
      for (int cb = 0; cb < 8; ++cb) {
        uint32_t v[32];
        tmem_load32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(32 * cb), v);
        // dims 32 cb .. 32 cb + 31 of the row: 64-dim box cb / 2, 16-byte chunks
        // 4 (cb % 2) .. + 3, each at its 128-byte-swizzle position
        const uint8_t *krow = ktile + (cb >> 1) * kStKBox + row * 128;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const int c = 4 * (cb & 1) + c4;
          const uint4 kv = *reinterpret_cast<const uint4 *>(krow + ((c ^ (row & 7)) << 4));
          const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            sum = fmaf(__uint_as_float(v[8 * c4 + 2 * e]), bf16_bits_to_float(kw[e] & 0xffffu), sum);
            sum = fmaf(__uint_as_float(v[8 * c4 + 2 * e + 1]), bf16_bits_to_float(kw[e] >> 16), sum);
          }
        }
      }
    }
    const int64_t r = r0 + row;
    const float wv = fmaxf(sum, 0.f);
    const bool store = ok && r < P.n;
    if (store) P.w[r * P.h + head] = wv;
    float tot = store ? wv : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if (lane == 0 && ok) atomicAdd(P.totals + head, tot);
  }
  // copies of an aborted run still land before the CTA exits
  if (warp == 0 && lane == 0 && *reinterpret_cast<volatile int32_t *>(&S.abort)) {
    (void)mbar_wait_bounded(&S.kfull, 0, 4096);
    for (int i = kStBlocks > kStStages ? kStBlocks - kStStages : 0; i < kStBlocks; ++i)
      (void)mbar_wait_bounded(&S.full[i % kStStages], (i / kStStages) & 1, 4096);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kStCols);
  }
}

// hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid): hi + mid + lo = x exactly
// for fp32 x (24 significand bits in three 8-bit pieces; each difference is exact).
// out holds [count / 65536 matrices][3 parts][65536] bf16.
__global__ void split_bf16x3_kernel(const float *__restrict__ x, int64_t count, __nv_bfloat16 *__restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float hv = round_bf16(v);
    const float r1 = v - hv;
    const float mv = round_bf16(r1);
    const float lv = round_bf16(r1 - mv);
    const int64_t m = i >> 16, e = i & 65535;
    __nv_bfloat16 *o = out + m * 3 * 65536 + e;
    o[0] = __float2bfloat16_rn(hv);
    o[65536] = __float2bfloat16_rn(mv);
    o[2 * 65536] = __float2bfloat16_rn(lv);
  }
}

}  // namespace

// Three exact bf16 parts of `matrices` fp32 256 x 256 matrices (the SST kernel's C).
int split_bf16x3_launch(const float *x, int32_t matrices, void *parts, cudaStream_t stream) {
  const int64_t count = (int64_t)matrices * 65536;
  if (count == 0) return OSCAR_OK;
  const int blocks = (int)((count + 255) / 256 < 4096 ? (count + 255) / 256 : 4096);
  split_bf16x3_kernel<<<blocks, 256, 0, stream>>>(x, count, reinterpret_cast<__nv_bfloat16 *>(parts));
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

// SST weights from pre-split covariances; OSCAR_ERR_UNSUPPORTED when the key layout does
// not fit a tensor map (16-byte aligned rows and strides).
int sst_tcgen05_launch(const void *key, int64_t n, int32_t h, int64_t ks0, int64_t ks1, const void *parts, float *w,
                       float *totals, int32_t *status, cudaStream_t stream) {
  if (encode_fn() == nullptr || n > (int64_t)INT32_MAX || h <= 0) return OSCAR_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(key) & 15) || (reinterpret_cast<uintptr_t>(parts) & 15) || (ks0 * 2) % 16 ||
      (ks1 * 2) % 16 || ks0 <= 0 || ks1 <= 0)
    return OSCAR_ERR_UNSUPPORTED;
  if (n == 0) return OSCAR_OK;
  SstTcParams P;
  memset(&P, 0, sizeof(P));
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)h, (cuuint64_t)n};
    cuuint64_t strides[2] = {(cuuint64_t)(ks1 * 2), (cuuint64_t)(ks0 * 2)};
    cuuint32_t box[3] = {64u, 1u, (cuuint32_t)kStRows};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    if (encode_fn()(&P.kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(key), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return OSCAR_ERR_UNSUPPORTED;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)kDim, (cuuint64_t)(3 * h)};
    cuuint64_t strides[2] = {(cuuint64_t)(kDim * 2), (cuuint64_t)(kDim * kDim * 2)};
    cuuint32_t box[3] = {64u, 256u, 1u};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    if (encode_fn()(&P.cmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(parts), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return OSCAR_ERR_UNSUPPORTED;
  }
  P.w = w;
  P.totals = totals;
  P.n = n;
  P.h = h;
  P.status = status;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(sst_tcgen05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kStSmem);
  });
  if (attr != cudaSuccess) return OSCAR_ERR_LAUNCH;
  const dim3 grid((unsigned)((n + kStRows - 1) / kStRows), (unsigned)h);
  sst_tcgen05_kernel<<<grid, kStThreads, kStSmem, stream>>>(P);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

}  // namespace oscar

extern "C" int oscar_split_bf16x3(const float *x, int32_t matrices, void *parts, void *stream) {
  if (matrices < 0 || (matrices > 0 && (!x || !parts))) return OSCAR_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(parts) & 15)) return OSCAR_ERR_INVALID;
  return oscar::split_bf16x3_launch(x, matrices, parts, (cudaStream_t)stream);
}

extern "C" int oscar_sst_weights_split(const void *key, int64_t n, int32_t h, int64_t ks0, int64_t ks1,
                                       const void *parts, float *weights, float *totals, int32_t *status,
                                       void *stream) {
  if (n < 0 || h <= 0 || !parts || !weights || !totals) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!key || (reinterpret_cast<uintptr_t>(key) & 15) || ks0 % 8 || ks1 % 8) return OSCAR_ERR_INVALID;
  return oscar::sst_tcgen05_launch(key, n, h, ks0, ks1, parts, weights, totals, status, (cudaStream_t)stream);
}
