// One-launch staging of a decode / verify step's device metadata.
//
// The vLLM model runner hands the attention builder device tensors (query starts,
// sequence lengths, block table, slot mapping) whose addresses change from step to step.
// CUDA graphs need fixed addresses, so every step's values are staged into one fixed
// int32 arena (plus one int64 slot buffer) that recorded kernels read.  The reference
// builder does this with four tensor copies, two fills and its task-table kernel
// (oscar_ascend/metadata.py:108-145, kernels.py:222-287); here a single launch does all
// of it: block 0 writes the device counts, the query starts, the sequence lengths and
// the task table (built from the source query starts directly), the other blocks copy
// the reachable block-table columns and the slot mapping.
//
// A dummy step (graph capture, warm-up) stages zero requests and zero tokens with no
// sources: the counts and the task count become 0, which masks every cache access of
// the recorded kernels, and nothing else is read or written.  A real step of zero
// requests still copies its one query start.
#include <algorithm>

#include "common.cuh"
#include "tasks.cuh"

namespace oscar {

// Arena layout, in int32 words.  Words 0-1: device counts [requests, active tokens];
// word 2: task count; word 3: reserved.  Then, each segment 16-byte aligned: query
// starts [max_reqs + 1], sequence lengths [max_reqs], block table [max_reqs, columns],
// task table [capacity, 2].
struct ArenaLayout {
  int64_t qstarts, seq_lens, table, tasks, words;
};

static int64_t align4(int64_t w) { return (w + 3) & ~int64_t(3); }

static ArenaLayout arena_layout(int32_t max_reqs, int32_t columns, int32_t capacity) {
  ArenaLayout L;
  L.qstarts = 4;
  L.seq_lens = align4(L.qstarts + max_reqs + 1);
  L.table = align4(L.seq_lens + max_reqs);
  L.tasks = align4(L.table + (int64_t)max_reqs * columns);
  L.words = align4(L.tasks + 2 * (int64_t)capacity);
  return L;
}

struct StageArgs {
  const int32_t *qstarts, *seq_lens, *table;
  int64_t table_stride;
  const int64_t *slots;
  int32_t nr, nt, copy_columns, query_tile;
  int32_t *arena;
  ArenaLayout L;
  int32_t columns, capacity;
  int64_t *slot_out;
};

__global__ void __launch_bounds__(1024) stage_step_kernel(StageArgs a) {
  if (blockIdx.x == 0) {
    int32_t *q = a.arena + a.L.qstarts, *s = a.arena + a.L.seq_lens;
    if (threadIdx.x == 0) {
      a.arena[0] = a.nr;
      a.arena[1] = a.nt;
    }
    if (a.qstarts)
      for (int i = threadIdx.x; i <= a.nr; i += blockDim.x) q[i] = a.qstarts[i];
    for (int i = threadIdx.x; i < a.nr; i += blockDim.x) s[i] = a.seq_lens[i];
    build_task_table(a.qstarts, a.nr, a.nt, a.arena + a.L.tasks, a.arena + 2, a.capacity, a.query_tile);
    return;
  }
  const int64_t stride = (int64_t)(gridDim.x - 1) * blockDim.x;
  const int64_t first = (int64_t)(blockIdx.x - 1) * blockDim.x + threadIdx.x;
  const int64_t cells = (int64_t)a.nr * a.copy_columns;
  int32_t *t = a.arena + a.L.table;
  for (int64_t i = first; i < cells; i += stride) {
    const int64_t r = i / a.copy_columns, c = i - r * a.copy_columns;
    t[r * a.columns + c] = a.table[r * a.table_stride + c];
  }
  for (int64_t i = first; i < a.nt; i += stride) a.slot_out[i] = a.slots[i];
}

}  // namespace oscar

using namespace oscar;

extern "C" int oscar_step_arena_layout(int32_t max_reqs, int32_t columns, int32_t task_capacity,
                                       int64_t *offsets) {
  if (max_reqs <= 0 || columns <= 0 || task_capacity <= 0 || !offsets) return OSCAR_ERR_INVALID;
  const ArenaLayout L = arena_layout(max_reqs, columns, task_capacity);
  offsets[0] = L.qstarts;
  offsets[1] = L.seq_lens;
  offsets[2] = L.table;
  offsets[3] = L.tasks;
  offsets[4] = L.words;
  return OSCAR_OK;
}

extern "C" int oscar_stage_step_metadata(const int32_t *qstarts, const int32_t *seq_lens, const int32_t *table,
                                         int64_t table_stride, const int64_t *slots, int32_t num_reqs,
                                         int32_t num_tokens, int32_t copy_columns, int32_t query_tile,
                                         int32_t *arena, int32_t max_reqs, int32_t columns, int32_t task_capacity,
                                         int64_t *slot_out, int64_t slot_capacity, void *stream) {
  if (!arena || max_reqs <= 0 || columns <= 0 || task_capacity <= 0 || query_tile <= 0 || slot_capacity < 0)
    return OSCAR_ERR_INVALID;
  if (num_reqs < 0 || num_reqs > max_reqs || num_tokens < 0 || num_tokens > slot_capacity) return OSCAR_ERR_INVALID;
  if (copy_columns < 0 || copy_columns > columns) return OSCAR_ERR_INVALID;
  if (num_reqs > 0 && (!qstarts || !seq_lens)) return OSCAR_ERR_INVALID;
  if (num_reqs > 0 && copy_columns > 0 && (!table || table_stride < copy_columns)) return OSCAR_ERR_INVALID;
  if (num_tokens > 0 && (!slots || !slot_out)) return OSCAR_ERR_INVALID;
  StageArgs a;
  a.qstarts = qstarts;
  a.seq_lens = seq_lens;
  a.table = table;
  a.table_stride = table_stride;
  a.slots = slots;
  a.nr = num_reqs;
  a.nt = num_tokens;
  a.copy_columns = num_reqs > 0 ? copy_columns : 0;
  a.query_tile = query_tile;
  a.arena = arena;
  a.L = arena_layout(max_reqs, columns, task_capacity);
  a.columns = columns;
  a.capacity = task_capacity;
  a.slot_out = slot_out;
  const int64_t work = std::max<int64_t>((int64_t)a.nr * a.copy_columns, a.nt);
  const int copy_blocks = (int)std::min<int64_t>((work + 1023) / 1024, 296);
  stage_step_kernel<<<1 + copy_blocks, 1024, 0, (cudaStream_t)stream>>>(a);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}
