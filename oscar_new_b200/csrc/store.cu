// Rotation GEMM, INT2 clip/pack/scatter store (standalone and fused), unpack.
//
// Reference: oscar_ascend/kernels.py:14-66 (rotate), :69-202 (clip, store_int2),
// :623-672 (unpack / dequant_inverse_rotate).
#include "rotate.cuh"

namespace oscar {

// ----------------------------------------------------------------------------
// standalone store: two (token, head) rows per warp, one per half-warp (the packed bf16
// quantiser of quant.cuh), K then V; a half whose row is absent or not stored still
// takes part in the reductions
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256) store_int2_kernel(const __nv_bfloat16 *__restrict__ krot,
                                                         const __nv_bfloat16 *__restrict__ vrot,
                                                         int64_t rows, uint8_t *__restrict__ history,
                                                         const int64_t *__restrict__ slots,
                                                         const int32_t *__restrict__ counts,
                                                         oscar_geometry geo, oscar_clip kc, oscar_clip vc) {
  const int lane = threadIdx.x & 31, l = lane & 15;
  const int64_t pair = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (2 * pair >= rows) return;  // warp-uniform
  const int64_t row = 2 * pair + (lane >> 4);
  bool live = row < rows;
  uint8_t *dst = nullptr;
  if (live) {
    const int64_t token = row / geo.kv_heads;
    const int head = (int)(row - token * geo.kv_heads);
    const int64_t slot = token < counts[1] ? slots[token] : -1;
    live = slot >= 0;
    if (live) dst = history + slot_byte_offset(slot, head, geo);
  }
  const int64_t rr = row < rows ? row : 2 * pair;
#pragma unroll 1
  for (int kv = 0; kv < 2; ++kv) {
    const uint4 *src = reinterpret_cast<const uint4 *>((kv == 0 ? krot : vrot) + rr * kDim + 16 * l);
    const uint4 r0 = src[0], r1 = src[1];
    const uint32_t w[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
    quantize_pack_half(w, kv == 0 ? kc : vc, live ? dst + kv * geo.vector_bytes : nullptr, live);
  }
}

// Decode-sized store jobs: 8 live rows on the 16-row GEMM tile, so that each of the 4
// warps quantises one pair of rows (the quantiser, not the GEMM, is the critical path).
constexpr int kSmallStoreRows = 8;

template <int ROWS>
__global__ void __launch_bounds__(ROWS == 64 ? 256 : 128) rotate_kernel(RotateParams p) {
  constexpr int MI = ROWS == 64 ? 2 : 1;
  constexpr int NT = ROWS == 64 ? 256 : 128;
  constexpr int NW = NT / 32;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16 *sA = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *sB = sA + ROWS * kDim;
  int64_t tile = blockIdx.x;
  int j = 0;
  while (j < p.njobs - 1 && tile >= p.job[j].tiles) {
    tile -= p.job[j].tiles;
    ++j;
  }
  const RotateJob job = p.job[j];
  const int64_t nrows = job.n * job.h;
  // store jobs of the 16-row kernel keep 8 live rows per tile (one quantise pass per warp)
  const int live = (ROWS == 16 && job.kv >= 0) ? kSmallStoreRows : ROWS;
  const int64_t row0 = tile * live;
  load_a_tile<ROWS, NT>(sA, row0, nrows, [&](int64_t r) {
    return job.x + (r / job.h) * job.s0 + (r % job.h) * job.s1;
  });
  cp_async_commit();
  float acc[MI][8][4];
  rowgemm_mainloop<MI, NT>(acc, sA, sB, job.r);
  // acc -> bf16 tile (rounded exactly once, as the reference rotate output)
  store_acc_bf16<MI>(sA, acc);
  __syncthreads();
  rotate_epilogue(sA, live, row0, job, p, NW);
}

// Large row counts go to the tcgen05 kernel; 16-row tiles (4x the CTAs of 64-row ones)
// serve launches whose 64-row grid would not fill two waves of the GPU (decode steps).
static int launch_rotate(RotateParams p, cudaStream_t stream) {
  int64_t rows64 = 0;
  for (int j = 0; j < p.njobs; ++j) rows64 += (p.job[j].n * p.job[j].h + 63) / 64;
  const bool small = rows64 < 2 * 148;
  if (!small) {
    // tcgen05 + TMA tiles; geometries the TMA unit cannot describe use 64-row tiles
    const int rc = launch_rotate_tc(p, stream);
    if (rc != OSCAR_ERR_UNSUPPORTED) return rc;
  }
  const int rows = small ? 16 : 64;
  int64_t total = 0;
  for (int j = 0; j < p.njobs; ++j) {
    const int jr = (small && p.job[j].kv >= 0) ? kSmallStoreRows : rows;
    p.job[j].tiles = (p.job[j].n * p.job[j].h + jr - 1) / jr;
    total += p.job[j].tiles;
  }
  const int smem = (rows * kDim + 2 * kBStageElems) * 2;
  if (small) {
    if (!ensure_dynamic_smem<rotate_kernel<16>>(smem)) return OSCAR_ERR_LAUNCH;
    rotate_kernel<16><<<(unsigned)total, 128, smem, stream>>>(p);
  } else {
    if (!ensure_dynamic_smem<rotate_kernel<64>>(smem)) return OSCAR_ERR_LAUNCH;
    rotate_kernel<64><<<(unsigned)total, 256, smem, stream>>>(p);
  }
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

// ----------------------------------------------------------------------------
// diagnostic unpack (reference _unpack_kernel): warp per (token, head)
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256) unpack_kernel(const uint8_t *__restrict__ history,
                                                     const int64_t *__restrict__ slots, int64_t n,
                                                     oscar_geometry geo, __nv_bfloat16 *__restrict__ kout,
                                                     __nv_bfloat16 *__restrict__ vout) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= n * geo.kv_heads) return;
  const int64_t token = row / geo.kv_heads;
  const int head = (int)(row % geo.kv_heads);
  const int64_t slot = slots[token];
#pragma unroll
  for (int kv = 0; kv < 2; ++kv) {
    uint32_t out[4] = {0, 0, 0, 0};
    if (slot >= 0) {
      const uint8_t *src = history + slot_byte_offset(slot, head, geo) + kv * geo.vector_bytes;
      const uint32_t codes = reinterpret_cast<const uint16_t *>(src)[lane];
      const uint32_t sz = *reinterpret_cast<const uint32_t *>(src + kDataBytes);
      const float s = half_bits_to_float(sz & 0xffffu), z = half_bits_to_float(sz >> 16);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float c0 = (float)((codes >> (4 * i)) & 3u), c1 = (float)((codes >> (4 * i + 2)) & 3u);
        out[i] = pack_bf162(__fadd_rn(__fmul_rn(c0, s), z), __fadd_rn(__fmul_rn(c1, s), z));
      }
    }
    __nv_bfloat16 *dst = (kv == 0 ? kout : vout) + row * kDim + lane * 8;
    *reinterpret_cast<uint4 *>(dst) = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

static bool rotation_ok(const void *r, int64_t rs0, int64_t rs1) {
  if (!r) return false;
  if (!((rs1 == 1 && rs0 % 8 == 0) || (rs0 == 1 && rs1 % 8 == 0))) return false;
  return (reinterpret_cast<uintptr_t>(r) & 15) == 0;
}

static bool rows_ok(const void *x, int64_t s0, int64_t s1) {
  return x && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && s0 % 8 == 0 && s1 % 8 == 0;
}

static bool geometry_ok(const oscar_geometry &g) {
  return g.head_dim == kDim && g.kv_heads > 0 && g.block_tokens > 0 && g.kernel_block == kKernelBlock &&
         g.block_tokens % kKernelBlock == 0 && g.slot_bytes % 16 == 0 && g.slot_bytes >= 2 * g.vector_bytes &&
         g.vector_bytes == kDataBytes + 4 && g.page_bytes == (int64_t)g.block_tokens * g.kv_heads * kDim * 2;
}

static bool clip_ok(const oscar_clip &c) {
  if (!c.enabled) return true;
  if (c.mode == 1) return c.factor > 0.f && c.factor <= 1.f;
  return c.mode == 0 && c.asc_lo >= 0 && c.asc_hi <= 255 && c.asc_lo <= c.asc_hi && c.asc_hi - c.asc_lo <= 1 &&
         c.weight >= 0.f && c.weight < 1.f;
}

}  // namespace oscar

using namespace oscar;

extern "C" int oscar_version(void) { return 100; }

// Bounded-wait self-test: one thread waits, with the bounded mbarrier wait that every
// kernel of this library uses, on a phase that nothing completes, and records
// OSCAR_ERR_TIMEOUT in *status when the wait gives up.
__global__ void bounded_wait_selftest_kernel(int32_t *status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival would complete phase 0; none ever comes
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_bounded(&bar, 0)) *status = OSCAR_ERR_TIMEOUT;
}

extern "C" int oscar_selftest_bounded_wait(int32_t *status, void *stream) {
  if (!status) return OSCAR_ERR_INVALID;
  bounded_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(status);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_rotate(const void *x, int64_t n, int32_t h, int64_t xs0, int64_t xs1, int64_t xs2,
                            const void *r, int64_t rs0, int64_t rs1, void *y, void *stream) {
  if (n < 0 || h <= 0 || xs2 != 1 || !y) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!rows_ok(x, xs0, xs1) || !rotation_ok(r, rs0, rs1)) return OSCAR_ERR_INVALID;
  RotateParams p{};
  p.njobs = 1;
  p.job[0] = RotateJob{reinterpret_cast<const __nv_bfloat16 *>(x), xs0, xs1, n, h,
                       BMatrix{reinterpret_cast<const __nv_bfloat16 *>(r), rs0, rs1},
                       reinterpret_cast<__nv_bfloat16 *>(y), -1, 0};
  return launch_rotate(p, (cudaStream_t)stream);
}

extern "C" int oscar_store_int2(const void *krot, const void *vrot, int64_t n, void *history,
                                const int64_t *slots, const int32_t *counts, oscar_geometry geo,
                                oscar_clip kclip, oscar_clip vclip, void *stream) {
  if (n < 0 || !geometry_ok(geo) || !clip_ok(kclip) || !clip_ok(vclip)) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!krot || !vrot || !history || !slots || !counts) return OSCAR_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(krot) | reinterpret_cast<uintptr_t>(vrot)) & 15) return OSCAR_ERR_INVALID;
  const int64_t rows = n * geo.kv_heads;
  store_int2_kernel<<<(unsigned)((rows + 15) / 16), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16 *>(krot), reinterpret_cast<const __nv_bfloat16 *>(vrot), rows,
      reinterpret_cast<uint8_t *>(history), slots, counts, geo, kclip, vclip);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_rotate_store(const void *key, int64_t ks0, int64_t ks1, const void *value, int64_t vs0,
                                  int64_t vs1, int64_t n, const void *rk, const void *rv, void *history,
                                  const int64_t *slots, const int32_t *counts, oscar_geometry geo,
                                  oscar_clip kclip, oscar_clip vclip, const void *query, int64_t qs0,
                                  int64_t qs1, int32_t hq, void *qrot_out, void *krot_out, void *vrot_out,
                                  int32_t *status, void *stream) {
  if (n < 0 || !geometry_ok(geo) || !clip_ok(kclip) || !clip_ok(vclip)) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!history || !slots || !counts) return OSCAR_ERR_INVALID;
  if (!rows_ok(key, ks0, ks1) || !rows_ok(value, vs0, vs1)) return OSCAR_ERR_INVALID;
  if (!rotation_ok(rk, 256, 1) || !rotation_ok(rv, 256, 1)) return OSCAR_ERR_INVALID;
  if (query && (!rows_ok(query, qs0, qs1) || hq <= 0 || !qrot_out)) return OSCAR_ERR_INVALID;
  const int64_t tiles = 0;  // set by launch_rotate
  RotateParams p{};
  p.history = reinterpret_cast<uint8_t *>(history);
  p.slots = slots;
  p.counts = counts;
  p.geo = geo;
  p.clip[0] = kclip;
  p.clip[1] = vclip;
  p.status = status;
  p.job[0] = RotateJob{reinterpret_cast<const __nv_bfloat16 *>(key), ks0, ks1, n, geo.kv_heads,
                       BMatrix{reinterpret_cast<const __nv_bfloat16 *>(rk), 256, 1},
                       reinterpret_cast<__nv_bfloat16 *>(krot_out), 0, tiles};
  p.job[1] = RotateJob{reinterpret_cast<const __nv_bfloat16 *>(value), vs0, vs1, n, geo.kv_heads,
                       BMatrix{reinterpret_cast<const __nv_bfloat16 *>(rv), 256, 1},
                       reinterpret_cast<__nv_bfloat16 *>(vrot_out), 1, tiles};
  p.njobs = 2;
  if (query) {
    p.job[2] = RotateJob{reinterpret_cast<const __nv_bfloat16 *>(query), qs0, qs1, n, hq,
                         BMatrix{reinterpret_cast<const __nv_bfloat16 *>(rk), 256, 1},
                         reinterpret_cast<__nv_bfloat16 *>(qrot_out), -1, 0};
    p.njobs = 3;
  }
  return launch_rotate(p, (cudaStream_t)stream);
}

extern "C" int oscar_unpack(const uint8_t *history, const int64_t *slots, int64_t n, oscar_geometry geo,
                            void *k_out, void *v_out, void *stream) {
  if (n < 0 || !geometry_ok(geo)) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!history || !slots || !k_out || !v_out) return OSCAR_ERR_INVALID;
  const int64_t rows = n * geo.kv_heads;
  unpack_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      history, slots, n, geo, reinterpret_cast<__nv_bfloat16 *>(k_out), reinterpret_cast<__nv_bfloat16 *>(v_out));
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}
