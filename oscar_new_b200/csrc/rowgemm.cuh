// Row-tile GEMM core: a CTA of 256 threads computes a [64 x 256] fp32 tile of
// A[64 x 256] @ B[256 x 256] with A staged in shared memory (filled by a caller
// prologue) and B streamed from global memory in four 64-deep stages.  bf16
// operands, fp32 accumulation on the warp-level tensor-core path (m16n8k16).
//
// Shared memory: A tile 32 KiB + 2 x 32 KiB B stages, 16-byte chunks XOR-swizzled
// by (row & 7) so that ldmatrix rows hit distinct banks.
#pragma once

#include "common.cuh"

namespace oscar {

constexpr int kTileRows = 64;
constexpr int kGemmThreads = 256;
constexpr int kStageK = 64;
constexpr int kAElems = kTileRows * kDim;        // 16384 bf16
constexpr int kBStageElems = kStageK * kDim;     // 16384 bf16
constexpr int kRowGemmSmem = (kAElems + 2 * kBStageElems) * 2;  // 98304 bytes

// A tile element (row, k) -> swizzled bf16 index
OSCAR_DEVINL int a_index(int row, int k) {
  return row * kDim + ((((k >> 3) ^ (row & 7))) << 3) + (k & 7);
}

// B matrix in global memory: element (k, n) at b[k * bs_k + n * bs_n]; exactly one of
// the strides is 1 (row-major: bs_n == 1, column-major: bs_k == 1).
struct BMatrix {
  const __nv_bfloat16 *ptr;
  int64_t bs_k;
  int64_t bs_n;
};

// Issue cp.async loads of B rows [k0, k0+64) into a stage (NT threads).
template <int NT = kGemmThreads>
OSCAR_DEVINL void load_b_stage(__nv_bfloat16 *stage, const BMatrix &b, int k0, int tid) {
  if (b.bs_n == 1) {
    // stage layout [64 k][256 n]: chunk (n/8) ^ (k&7)
#pragma unroll
    for (int i = 0; i < 2048 / NT; ++i) {
      const int c = tid + i * NT;  // 0..2047
      const int k = c >> 5, ch = c & 31;
      const __nv_bfloat16 *src = b.ptr + (int64_t)(k0 + k) * b.bs_k + ch * 8;
      cp_async_16(smem_u32(stage + k * kDim + ((ch ^ (k & 7)) << 3)), src);
    }
  } else {
    // stage layout [256 n][64 k]: chunk (k/8) ^ (n&7)
#pragma unroll
    for (int i = 0; i < 2048 / NT; ++i) {
      const int c = tid + i * NT;
      const int n = c >> 3, ch = c & 7;
      const __nv_bfloat16 *src = b.ptr + (int64_t)n * b.bs_n + k0 + ch * 8;
      cp_async_16(smem_u32(stage + n * kStageK + ((ch ^ (n & 7)) << 3)), src);
    }
  }
}

// acc[mi][nj][4]: warp tile (16*MI) rows x 64 cols (warp_m = warp / 4, warp_n = warp % 4).
// MI = 2: 64-row tile, 8 warps; MI = 1 with NT = 128: 16-row tile, 4 warps.
// The caller has issued (not necessarily completed) cp.async loads for the A tile in
// the most recent commit group, or written it synchronously; this function issues B
// stage 0 itself.
template <int MI = 2, int NT = kGemmThreads>
OSCAR_DEVINL void rowgemm_mainloop(float (&acc)[MI][8][4], const __nv_bfloat16 *sA, __nv_bfloat16 *sB,
                                   const BMatrix &b) {
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int wm = warp >> 2, wn = warp & 3;
#pragma unroll
  for (int i = 0; i < MI; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.f;

  load_b_stage<NT>(sB, b, 0, tid);
  cp_async_commit();
  const bool rowmajor = b.bs_n == 1;
#pragma unroll 1
  for (int s = 0; s < kDim / kStageK; ++s) {
    if (s + 1 < kDim / kStageK) {
      load_b_stage<NT>(sB + ((s + 1) & 1) * kBStageElems, b, (s + 1) * kStageK, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16 *stage = sB + (s & 1) * kBStageElems;
#pragma unroll
    for (int kk = 0; kk < kStageK / 16; ++kk) {
      const int kg = s * kStageK + kk * 16;  // global k of this step
      uint32_t a[MI][4];
#pragma unroll
      for (int mi = 0; mi < MI; ++mi) {
        const int row = wm * (16 * MI) + mi * 16 + (lane & 15);
        const int k = kg + (lane >> 4) * 8;
        ldmatrix_x4(a[mi], smem_u32(sA + a_index(row, k)));
      }
#pragma unroll
      for (int nj = 0; nj < 8; nj += 2) {
        uint32_t bf[4];
        if (rowmajor) {
          const int k = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int n = wn * 64 + (nj + (lane >> 4)) * 8;
          ldmatrix_x4_trans(bf, smem_u32(stage + k * kDim + (((n >> 3) ^ (k & 7)) << 3)));
        } else {
          const int n = wn * 64 + (nj + (lane >> 4)) * 8 + (lane & 7);
          const int k = kk * 16 + ((lane >> 3) & 1) * 8;
          ldmatrix_x4(bf, smem_u32(stage + n * kStageK + (((k >> 3) ^ (n & 7)) << 3)));
        }
#pragma unroll
        for (int mi = 0; mi < MI; ++mi) {
          mma_bf16_16816(acc[mi][nj], a[mi][0], a[mi][1], a[mi][2], a[mi][3], bf[0], bf[1]);
          mma_bf16_16816(acc[mi][nj + 1], a[mi][0], a[mi][1], a[mi][2], a[mi][3], bf[2], bf[3]);
        }
      }
    }
    __syncthreads();
  }
}

// Stage one row-block of X (bf16 rows with unit inner stride) into the A tile with
// cp.async; rows >= nrows are zero-filled.  row_ptr(r) gives the global row address.
template <int ROWS = kTileRows, int NT = kGemmThreads, typename RowPtr>
OSCAR_DEVINL void load_a_tile(__nv_bfloat16 *sA, int64_t row0, int64_t nrows, RowPtr row_ptr) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int i = 0; i < ROWS * 32 / NT; ++i) {
    const int c = tid + i * NT;  // ROWS rows x 32 chunks
    const int r = c >> 5, ch = c & 31;
    __nv_bfloat16 *dst = sA + r * kDim + ((ch ^ (r & 7)) << 3);
    if (row0 + r < nrows) {
      cp_async_16(smem_u32(dst), row_ptr(row0 + r) + ch * 8);
    } else {
      *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
}

// Write the fp32 accumulators as bf16 into a [rows][256] shared tile (same swizzle as A).
template <int MI = 2>
OSCAR_DEVINL void store_acc_bf16(__nv_bfloat16 *sY, const float (&acc)[MI][8][4]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wm = warp >> 2, wn = warp & 3;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mi = 0; mi < MI; ++mi)
#pragma unroll
    for (int nj = 0; nj < 8; ++nj) {
      const int row = wm * (16 * MI) + mi * 16 + g;
      const int col = wn * 64 + nj * 8 + 2 * t;
      *reinterpret_cast<uint32_t *>(sY + a_index(row, col)) = pack_bf162(acc[mi][nj][0], acc[mi][nj][1]);
      *reinterpret_cast<uint32_t *>(sY + a_index(row + 8, col)) = pack_bf162(acc[mi][nj][2], acc[mi][nj][3]);
    }
}

}  // namespace oscar
