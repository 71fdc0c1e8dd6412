// Compact (request, query offset) task table, built on the device by one block
// (reference oscar_ascend/kernels.py:222-287, _prepare_tasks_kernel): request r with
// q_r live query tokens (bounded by the active token count) owns ceil(q_r / tile)
// consecutive task slots (r, 0), (r, tile), ...  A block-wide scan over the requests
// gives each request its first slot; slots beyond `capacity` are dropped and the count
// is clamped to it.
#pragma once

#include "common.cuh"

namespace oscar {

// Called by every thread of one block (blockDim.x a multiple of 32, at most 1024).
OSCAR_DEVINL void build_task_table(const int32_t *__restrict__ qstarts, int nr, int active,
                                   int32_t *__restrict__ tasks, int32_t *__restrict__ task_count,
                                   int32_t capacity, int32_t query_tile) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int base = 0; base < nr; base += blockDim.x) {
    const int req = base + threadIdx.x;
    int tiles = 0;
    if (req < nr) {
      const int s = min(qstarts[req], active), e = min(qstarts[req + 1], active);
      tiles = (max(e - s, 0) + query_tile - 1) / query_tile;
    }
    int incl = tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int ws = lane < nwarps ? warp_sums[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, ws, o);
        if (lane >= o) ws += v;
      }
      warp_sums[lane] = ws;
    }
    __syncthreads();
    const int first = carry + (warp ? warp_sums[warp - 1] : 0) + incl - tiles;
    for (int i = 0; i < tiles; ++i) {
      const int slot = first + i;
      if (slot < capacity) {
        tasks[2 * slot] = req;
        tasks[2 * slot + 1] = i * query_tile;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_sums[nwarps - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) task_count[0] = min(carry, capacity);
}

}  // namespace oscar
