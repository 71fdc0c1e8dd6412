// Rotation jobs shared by the two rotation GEMM kernels (reference
// oscar_ascend/kernels.py:14-66 rotate, :104-202 store_int2):
//  * rotate_kernel (store.cu): warp-level mma.sync tiles of 16 rows for decode-sized
//    launches, where 128-row tiles would leave most SMs idle;
//  * rotate_tc_kernel (rotate_tc.cu): tcgen05 128-row tiles fed by TMA for large
//    launches (prefill chunks, bulk rotation + store).
// Both end in the same epilogue: the bf16-rounded rotated rows (the reference rounds
// the rotate output to bf16 once) are staged in shared memory, optionally copied to
// `y`, and, for K / V jobs, quantised and scattered into the paged history slots.
#pragma once

#include "quant.cuh"
#include "rowgemm.cuh"

namespace oscar {

struct RotateJob {
  const __nv_bfloat16 *x;  // rows (t, h) at x + t*s0 + h*s1, unit inner stride
  int64_t s0, s1;
  int64_t n;               // tokens
  int32_t h;               // heads per token
  BMatrix r;
  __nv_bfloat16 *y;        // contiguous [n*h, 256] output (nullable for store jobs)
  int32_t kv;              // -1: plain rotate, 0: K store, 1: V store
  int64_t tiles;
};

struct RotateParams {
  RotateJob job[3];
  int32_t njobs;
  uint8_t *history;
  const int64_t *slots;
  const int32_t *counts;
  oscar_geometry geo;
  oscar_clip clip[2];
  int32_t *status;  // nullable device word: OSCAR_ERR_TIMEOUT when a bounded wait gave up
};

// Byte offset of a slot's head-0 vector pair in the history stripes, -1 for slot < 0.
OSCAR_DEVINL int64_t slot_base_offset(int64_t slot, const oscar_geometry &g) {
  return slot < 0 ? -1 : slot_byte_offset(slot, 0, g);
}

// Epilogue over a staged tile of `rows` rotated rows (swizzled like the A tile, see
// a_index) starting at global row `row0` (valid while row < nrows): copy to y, then
// quantise + scatter K / V rows, two rows per warp.  `nw` warps of the CTA take part.
// `tile_bases` (optional, shared memory; row0 then a multiple of h) holds
// slot_base_offset of each token of the tile.
OSCAR_DEVINL void rotate_epilogue(const __nv_bfloat16 *sY, int rows, int64_t row0, const RotateJob &job,
                                  const RotateParams &p, int nw, const int64_t *tile_bases = nullptr) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nt = nw * 32;
  const int64_t nrows = job.n * job.h;
  if (job.y != nullptr) {
    for (int c = threadIdx.x; c < rows * 32; c += nt) {
      const int r = c >> 5, ch = c & 31;
      if (row0 + r < nrows)
        *reinterpret_cast<uint4 *>(job.y + (row0 + r) * kDim + ch * 8) =
            *reinterpret_cast<const uint4 *>(sY + r * kDim + ((ch ^ (r & 7)) << 3));
    }
  }
  if (job.kv < 0) return;
  const int32_t active = p.counts[1];
  // two rows per warp, one per half-warp (quantize_pack_half); a half whose row is
  // absent or not stored still takes part in the reductions
  const int half = lane >> 4, l = lane & 15;
  // token / head of row0 + r without a 64-bit division per row: one for the tile, then
  // floor(t / h) = umulhi(t, floor((2^32 - 1) / h) + 1), exact for t < 2^16
  const int64_t token0 = row0 / job.h;
  const int head0 = (int)(row0 - token0 * job.h);
  const uint32_t hm = job.h > 1 ? 0xffffffffu / (uint32_t)job.h + 1u : 0u;
#pragma unroll 1
  for (int pr = warp; 2 * pr < rows; pr += nw) {
    const int r = 2 * pr + half;
    const int64_t row = row0 + r;
    bool live = r < rows && row < nrows;
    int64_t base = -1;
    int head = 0;
    if (live) {
      const uint32_t t = (uint32_t)(head0 + r);
      const uint32_t tq = job.h > 1 ? __umulhi(t, hm) : t;
      const int64_t token = token0 + tq;
      head = (int)(t - tq * (uint32_t)job.h);
      if (tile_bases != nullptr)
        base = tile_bases[tq];  // prefetched for the tile's tokens (-1 when not stored)
      else
        base = token < active ? slot_base_offset(p.slots[token], p.geo) : -1;
      live = base >= 0;
    }
    if (!__any_sync(0xffffffffu, live)) continue;
    uint32_t w[8];  // dims 16l .. 16l+15 as bf16 pairs
    const int rr = r < rows ? r : 0;
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {
      const uint4 raw = *reinterpret_cast<const uint4 *>(sY + rr * kDim + (((2 * l + c2) ^ (rr & 7)) << 3));
      w[4 * c2] = raw.x, w[4 * c2 + 1] = raw.y, w[4 * c2 + 2] = raw.z, w[4 * c2 + 3] = raw.w;
    }
    uint8_t *dst = live ? p.history + base + (int64_t)head * p.geo.slot_bytes + job.kv * p.geo.vector_bytes : nullptr;
    quantize_pack_half(w, p.clip[job.kv], dst, live);
  }
}

// tcgen05 launch for large jobs (rotate_tc.cu).  Returns OSCAR_OK, or
// OSCAR_ERR_UNSUPPORTED when a job's geometry cannot be described to the TMA unit
// (the caller then uses the mma.sync tiles), or a launch error.
int launch_rotate_tc(const RotateParams &p, cudaStream_t stream);

}  // namespace oscar
