// Causal BF16 attention of a first prefill on the 5th-generation tensor cores: the
// attention of the current tokens of requests that start at position 0 (no INT2 history
// and no BF16 window yet), D = 256, grouped-query heads, variable lengths.  The reference
// hands this case to the vendor's fused attention (oscar_ascend/backend.py:175-193);
// here it is a kernel of this library.
//
// One CTA = (request, query head, block of 128 query tokens); blocks with more keys run
// first.  Per key block of 64 tokens:
//   S = Q K^T   tcgen05.mma kind::f16, M = 128 query rows, N = 64 keys, K = 256, Q and
//               K from shared memory (TMA, 128-byte swizzle, K-major), S into tensor
//               memory (double-buffered);
//   softmax     one thread per query row (its TMEM lane): scale, causal mask on the
//               diagonal blocks, running max in the log2 domain re-based lazily (when a
//               row's max grows by more than 2^8 the row's O is rescaled in tensor
//               memory), P = 2^(s - m) as bf16 pairs stored into tensor memory;
//   O += P V    tcgen05.mma with A = P from tensor memory (TS form), B = V from shared
//               memory (MN-major), M = 128, N = 256, K = 64.
// Warp roles: warp 0 lane 0 issues the TMA copies (Q once, K / V in two stages, no
// multicast), warp 1 lane 0 issues the MMAs (S of block j ahead of P V of block j - 1),
// warps 2-5 run the softmax and the epilogue (O / l to bf16).  Tensor memory: O in 256
// columns, S 2 x 64, P 2 x 32.  Every mbarrier wait is bounded; a timeout sets the
// status word (when given) and the CTA skips its epilogue.
#include <cstring>

#include "tcgen05.cuh"

namespace oscar {
namespace {

constexpr int kPfQ = 128;                     // query rows per CTA
constexpr int kPfK = 64;                      // keys per block
constexpr int kPfQBytes = kPfQ * kDim * 2;    // 64 KiB: 4 boxes of 64 dims
constexpr int kPfKBytes = kPfK * kDim * 2;    // 32 KiB
constexpr int kPfStage = 2 * kPfKBytes;       // K and V of one block
constexpr int kPfThreads = 192;
constexpr uint32_t kColO = 0, kColS = 256, kColP = 384, kPfCols = 512;
constexpr float kPfSlack = 8.f;               // re-base a row when its max grows past 2^8

struct PfParams {
  CUtensorMap qmap, kmap, vmap;
  const int32_t *qstarts;  // [num_reqs + 1] device
  __nv_bfloat16 *out;
  int64_t os0, os1;
  int32_t num_reqs, group, nqb;
  float scale_log2;
  int32_t *status;
};

struct PfSmem {
  uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], s_empty[2], p_full[2], pv_done[2], o_done;
  uint32_t tmem;
  int32_t abort;
};

// kind::f16, fp32 accumulator, A and B bf16, M = 128; S: both K-major, N = 64;
// P V: B MN-major, N = 256.
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescPV =
    (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

OSCAR_DEVINL bool pf_wait(uint64_t *bar, uint32_t phase, PfSmem &S) {
  if (mbar_wait_bounded(bar, phase)) return true;
  atomicExch(&S.abort, 1);
  return false;
}

__global__ void __launch_bounds__(kPfThreads, 1) prefill_attention_kernel(const __grid_constant__ PfParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *qs = smem;
  uint8_t *kv = smem + kPfQBytes;
  PfSmem &S = *reinterpret_cast<PfSmem *>(kv + 2 * kPfStage);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int head = blockIdx.x, req = blockIdx.y, qb = P.nqb - 1 - (int)blockIdx.z;
  const int q0 = P.qstarts[req], len = P.qstarts[req + 1] - q0;
  if (qb * kPfQ >= len) return;
  const int last_q = min(qb * kPfQ + kPfQ - 1, len - 1);
  const int nkb = last_q / kPfK + 1;
  const int kvh = head / P.group;

  if (tid == 0) {
    mbar_init(&S.q_full, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.kv_full[b], 1);
      mbar_init(&S.kv_empty[b], 1);
      mbar_init(&S.s_full[b], 1);
      mbar_init(&S.s_empty[b], 4);
      mbar_init(&S.p_full[b], 4);
      mbar_init(&S.pv_done[b], 1);
    }
    mbar_init(&S.o_done, 1);
    S.abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) tmem_alloc(&S.tmem, kPfCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;

  if (warp == 0 && lane == 0) {
    // ---- producer ----
    mbar_arrive_expect_tx(&S.q_full, kPfQBytes);
    for (int b = 0; b < 4; ++b)
      tma_load_3d(smem_u32(qs + b * (kPfQBytes / 4)), &P.qmap, 64 * b, head, q0 + qb * kPfQ, &S.q_full);
    for (int j = 0; j < nkb; ++j) {
      const int st = j & 1;
      if (j >= 2 && !pf_wait(&S.kv_empty[st], ((j >> 1) - 1) & 1, S)) break;
      if (*reinterpret_cast<volatile int32_t *>(&S.abort)) break;
      uint8_t *ks = kv + st * kPfStage, *vs = ks + kPfKBytes;
      mbar_arrive_expect_tx(&S.kv_full[st], kPfStage);
      for (int b = 0; b < 4; ++b) {
        tma_load_3d(smem_u32(ks + b * (kPfKBytes / 4)), &P.kmap, 64 * b, kvh, q0 + j * kPfK, &S.kv_full[st]);
        tma_load_3d(smem_u32(vs + b * (kPfKBytes / 4)), &P.vmap, 64 * b, kvh, q0 + j * kPfK, &S.kv_full[st]);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    bool ok = pf_wait(&S.q_full, 0, S);
    auto pv = [&](int i) {
      if (!ok || !pf_wait(&S.p_full[i & 1], (i >> 1) & 1, S)) {
        ok = false;
        return;
      }
      tc_fence_after();
      const uint32_t v0 = smem_u32(kv + (i & 1) * kPfStage + kPfKBytes);
#pragma unroll
      for (int kk = 0; kk < kPfK / 16; ++kk)
        umma_f16_ts(tmem + kColO, tmem + kColP + 32 * (i & 1) + 8 * kk, smem_desc(v0 + kk * 2048, 8192, 1024),
                    kIdescPV, (i | kk) != 0 ? 1u : 0u);
      umma_commit(&S.kv_empty[i & 1]);
      umma_commit(&S.pv_done[i & 1]);
    };
    const uint32_t qa = smem_u32(qs);
    for (int j = 0; j < nkb && ok; ++j) {
      const int st = j & 1;
      if (!pf_wait(&S.kv_full[st], (j >> 1) & 1, S)) {
        ok = false;
        break;
      }
      if (j >= 2 && !pf_wait(&S.s_empty[st], ((j >> 1) - 1) & 1, S)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t k0 = smem_u32(kv + st * kPfStage);
#pragma unroll
      for (int b = 0; b < 4; ++b)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tmem + kColS + 64 * st, smem_desc(qa + b * (kPfQBytes / 4) + kk * 32, 16, 1024),
                    smem_desc(k0 + b * (kPfKBytes / 4) + kk * 32, 16, 1024), kIdescS, (b | kk) != 0 ? 1u : 0u);
      umma_commit(&S.s_full[st]);
      if (j >= 1) pv(j - 1);
    }
    if (ok) pv(nkb - 1);
    umma_commit(&S.o_done);
  } else if (warp >= 2) {
    // ---- softmax: thread = query row = TMEM lane ----
    const int quarter = warp & 3, row = 32 * quarter + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16);
    const int qi = qb * kPfQ + row;  // query index within the request
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      const int s = j & 1;
      ok = pf_wait(&S.s_full[s], (j >> 1) & 1, S);
      if (!ok) break;
      tc_fence_after();
      uint32_t a[32], b[32];
      tmem_load32x2(lane_base + kColS + 64 * s, a, lane_base + kColS + 64 * s + 32, b);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.s_empty[s]);
      float x[64];
#pragma unroll
      for (int c = 0; c < 32; ++c) x[c] = __uint_as_float(a[c]) * P.scale_log2;
#pragma unroll
      for (int c = 0; c < 32; ++c) x[32 + c] = __uint_as_float(b[c]) * P.scale_log2;
      if ((j + 1) * kPfK - 1 > qb * kPfQ) {  // keys past some query of the block: causal mask
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (j * kPfK + c > qi) x[c] = -INFINITY;
      }
      // tree reductions: no 64-long dependency chain
      float t32[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) t32[c] = fmaxf(x[c], x[c + 32]);
#pragma unroll
      for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
        for (int c = 0; c < w; ++c) t32[c] = fmaxf(t32[c], t32[c + w]);
      const float bmax = t32[0];
      const bool rebase = m != -INFINITY && bmax > m + kPfSlack;
      if (m == -INFINITY) m = bmax;
      if (__any_sync(0xffffffffu, rebase)) {
        // the warp's rows that re-base scale their O; P V of block j - 1 is complete first
        const float alpha = rebase ? ex2(m - bmax) : 1.f;
        if (rebase) {
          m = bmax;
          l *= alpha;
        }
        if (!pf_wait(&S.pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, S)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int cb = 0; cb < 8; ++cb) {
          uint32_t o[32];
          tmem_load32(lane_base + kColO + 32 * cb, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_store32(lane_base + kColO + 32 * cb, o);
        }
      }
      uint32_t pk[32];
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p0 = ex2(x[2 * c] - m), p1 = ex2(x[2 * c + 1] - m);
        acc[c & 3] += p0 + p1;
        pk[c] = pack_bf162(p0, p1);
      }
      l += (acc[0] + acc[1]) + (acc[2] + acc[3]);
      // P buffer s was read by P V of block j - 2
      if (j >= 2 && !pf_wait(&S.pv_done[s], ((j - 2) >> 1) & 1, S)) {
        ok = false;
        break;
      }
      tc_fence_after();
      tmem_store32(lane_base + kColP + 32 * s, pk);
      tmem_store_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.p_full[s]);
    }
    // ---- epilogue: O / l -> bf16 rows ----
    const bool done = ok && pf_wait(&S.o_done, 0, S);
    __syncwarp();
    const bool good = __all_sync(0xffffffffu, done) && *reinterpret_cast<volatile int32_t *>(&S.abort) == 0;
    if (!good) {
      if (lane == 0 && P.status) atomicExch(P.status, OSCAR_ERR_TIMEOUT);
    } else {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool store = qi < len;
      __nv_bfloat16 *dst = P.out + (int64_t)(q0 + qi) * P.os0 + (int64_t)head * P.os1;
#pragma unroll 1
      for (int cb = 0; cb < 8; ++cb) {
        uint32_t o[32];
        tmem_load32(lane_base + kColO + 32 * cb, o);
        if (store) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint4 w;
            w.x = pack_bf162(__uint_as_float(o[8 * e + 0]) * inv, __uint_as_float(o[8 * e + 1]) * inv);
            w.y = pack_bf162(__uint_as_float(o[8 * e + 2]) * inv, __uint_as_float(o[8 * e + 3]) * inv);
            w.z = pack_bf162(__uint_as_float(o[8 * e + 4]) * inv, __uint_as_float(o[8 * e + 5]) * inv);
            w.w = pack_bf162(__uint_as_float(o[8 * e + 6]) * inv, __uint_as_float(o[8 * e + 7]) * inv);
            *reinterpret_cast<uint4 *>(dst + 32 * cb + 8 * e) = w;
          }
        }
      }
    }
  }
  __syncwarp();
  // an aborted CTA lets its copies land before it exits
  if (warp == 0 && lane == 0 && *reinterpret_cast<volatile int32_t *>(&S.abort)) {
    (void)mbar_wait_bounded(&S.q_full, 0, 4096);
    for (int b = 0; b < 2; ++b) (void)mbar_wait_bounded(&S.kv_full[b], 0, 4096);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPfCols);
  }
}

bool encode_rows3(CUtensorMap *map, const void *base, int64_t n, int32_t heads, int64_t s0, int64_t s1, int box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (s0 * 2) % 16 || (s1 * 2) % 16 || s0 <= 0 || s1 <= 0) return false;
  cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)heads, (cuuint64_t)n};
  cuuint64_t strides[2] = {(cuuint64_t)(s1 * 2), (cuuint64_t)(s0 * 2)};
  cuuint32_t box[3] = {64u, 1u, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace
}  // namespace oscar

using namespace oscar;

extern "C" int oscar_prefill_attention(const void *query, int64_t qs0, int64_t qs1, const void *key, int64_t ks0,
                                       int64_t ks1, const void *value, int64_t vs0, int64_t vs1,
                                       const int32_t *qstarts, int32_t num_reqs, int32_t max_query_len, int64_t n,
                                       int32_t hq, int32_t hkv, float scale, void *out, int64_t os0, int64_t os1,
                                       int32_t *status, void *stream) {
  if (num_reqs < 0 || max_query_len < 0 || n < 0 || hq <= 0 || hkv <= 0 || hq % hkv || !(scale > 0.f))
    return OSCAR_ERR_INVALID;
  if (num_reqs == 0 || max_query_len == 0 || n == 0) return OSCAR_OK;
  if (!query || !key || !value || !qstarts || !out || n > INT32_MAX) return OSCAR_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || os0 % 8 || os1 % 8) return OSCAR_ERR_INVALID;
  if (encode_fn() == nullptr) return OSCAR_ERR_UNSUPPORTED;
  PfParams P;
  memset(&P, 0, sizeof(P));
  if (!encode_rows3(&P.qmap, query, n, hq, qs0, qs1, kPfQ) || !encode_rows3(&P.kmap, key, n, hkv, ks0, ks1, kPfK) ||
      !encode_rows3(&P.vmap, value, n, hkv, vs0, vs1, kPfK))
    return OSCAR_ERR_INVALID;
  P.qstarts = qstarts;
  P.out = reinterpret_cast<__nv_bfloat16 *>(out);
  P.os0 = os0;
  P.os1 = os1;
  P.num_reqs = num_reqs;
  P.group = hq / hkv;
  P.nqb = (max_query_len + kPfQ - 1) / kPfQ;
  P.scale_log2 = scale * 1.4426950408889634f;
  P.status = status;
  const int smem = kPfQBytes + 2 * kPfStage + (int)sizeof(PfSmem) + 1024;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [smem] {
    attr = cudaFuncSetAttribute(prefill_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  if (attr != cudaSuccess) return OSCAR_ERR_LAUNCH;
  dim3 grid((unsigned)hq, (unsigned)num_reqs, (unsigned)P.nqb);
  prefill_attention_kernel<<<grid, kPfThreads, smem, (cudaStream_t)stream>>>(P);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}
