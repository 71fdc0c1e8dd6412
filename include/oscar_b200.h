/*
 * oscar_b200.h -- C ABI of the B200 (sm_100a) OSCAR INT2 KV-cache library.
 *
 * Every entry point takes raw device pointers, element strides, plain integer
 * geometry and a cudaStream_t (passed as void*), launches on that stream and
 * returns an int status (OSCAR_OK = 0).  Nothing throws across the ABI, nothing
 * synchronises the host, nothing reads device memory from the host, and nothing
 * allocates: every buffer is owned by the caller.  Entry points are safe to call
 * from several host threads on distinct streams and can be recorded in CUDA graphs
 * (all data-dependent bounds are read on the device from `counts`); the
 * no-allocation decode variant below carries its own notes instead.
 *
 * Tensor conventions (row-major unless strides are given):
 *   bf16/f16 are passed as raw 16-bit payloads (void*); D (head_dim) is 256.
 *   history : uint8 view of the native K stripe   [num_pages * page_bytes]
 *   window  : bf16 view of the native V stripe     [num_pages * page_bytes / 2]
 *   counts  : int32[2] = {num_reqs, num_actual_tokens}
 *   slots   : int64[n], -1 = do not store
 *   table   : int32 [max_reqs, table_stride] of 128-token kernel blocks
 */
#ifndef OSCAR_B200_H
#define OSCAR_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  OSCAR_OK = 0,
  OSCAR_ERR_INVALID = 1,   /* bad argument: null pointer, size, alignment, geometry */
  OSCAR_ERR_LAUNCH = 2,    /* CUDA launch error (cudaGetLastError after launch)     */
  OSCAR_ERR_UNSUPPORTED = 3,
  OSCAR_ERR_TIMEOUT = 4    /* a bounded device wait gave up (reported via status buffer) */
};

/* Device status word.  Entry points whose kernels wait on the device (mbarrier phases of
 * asynchronous copies and tensor-core work) take `int32_t *status`: a device int32, or
 * NULL.  Every such wait gives up after a fixed number of probes instead of hanging; the
 * kernel then stores OSCAR_ERR_TIMEOUT into *status, stops consuming, lets its copies in
 * flight land, frees its tensor memory and returns, leaving the context usable.  The
 * library never clears the word: the caller zeroes it, and reads it after synchronising
 * the stream (a nonzero value means the outputs of the calls since it was zeroed are not
 * valid).  Launch-time errors are still the return value. */

/* Cache geometry shared by the paged kernels (reference oscar_ascend/layout.py:8-95,
 * config.py:46-63).  page_bytes = physical_block_tokens * kv_heads * head_dim * 2. */
typedef struct oscar_geometry {
  int32_t kv_heads;           /* H                                  */
  int32_t group;              /* G = query heads per KV head        */
  int32_t head_dim;           /* D, must be 256                     */
  int32_t block_tokens;       /* Bp, physical page tokens           */
  int32_t kernel_block;       /* 128                                */
  int32_t slot_bytes;         /* 160                                */
  int32_t vector_bytes;       /* 68                                 */
  int32_t sink;               /* S                                  */
  int32_t recent;             /* R                                  */
  int32_t ring;               /* C = R + MTP + 1                    */
  int32_t table_stride;       /* row stride of the block table      */
  int32_t query_tile;         /* QT: queries per task               */
  int64_t page_bytes;         /* J                                  */
} oscar_geometry;

/* Percentile / factor clip parameters of one quantised stream (K or V).
 * mode 0 = percentile, 1 = factor; enabled 0 disables clipping.  For percentile mode
 * asc_lo/asc_hi are the ascending sorted indices floor/ceil((D-1)*ratio) and weight
 * the fp32 interpolation weight, i.e. torch.quantile(|x|, ratio) semantics
 * (reference tests/oracle.py:10-15, kernels.py:69-101). */
typedef struct oscar_clip {
  int32_t enabled;
  int32_t mode;
  int32_t asc_lo;
  int32_t asc_hi;
  float weight;
  float factor;
} oscar_clip;

/* Library/device identification. Returns the compiled SM arch (100 for sm_100a). */
int oscar_version(void);

/* Self-test of the bounded device waits (no counterpart in the reference, whose
 * attention kernel was seen to hang its device): launches one thread that waits, with
 * the same bounded mbarrier wait every kernel here uses, on a barrier phase that nothing
 * completes, and writes OSCAR_ERR_TIMEOUT to *status (device int32) when the wait gives
 * up.  A caller can run it to check that a wait which can never be satisfied ends with
 * an error status, not a hang, and that the context stays usable. */
int oscar_selftest_bounded_wait(int32_t *status, void *stream);

/* Causal BF16 attention of a first prefill (every request starts at position 0): the
 * current tokens only, D = 256, grouped-query heads (hq a multiple of hkv), variable
 * lengths from the device query starts [num_reqs + 1]; max_query_len is the host bound
 * that sizes the grid.  query [n, hq, 256], key / value [n, hkv, 256] bf16 rows with
 * element strides (token, head) that are multiples of 8; out [n, hq, 256] bf16.  A
 * tcgen05 kernel of this library where the reference hands the case to the vendor's fused
 * attention (backend.py:175-193). */
int oscar_prefill_attention(const void *query, int64_t qs0, int64_t qs1, const void *key, int64_t ks0, int64_t ks1,
                            const void *value, int64_t vs0, int64_t vs1, const int32_t *qstarts, int32_t num_reqs,
                            int32_t max_query_len, int64_t n, int32_t hq, int32_t hkv, float scale, void *out,
                            int64_t os0, int64_t os1, int32_t *status, void *stream);

/* Which history kernel the latest successful history launch of this process used
 * (a host-side record made at launch time; no device access): 0 none yet,
 * OSCAR_HISTORY_ATTENTION_KERNEL (mma.sync, decode and general rows),
 * OSCAR_HISTORY_MTP_KERNEL (mma.sync, MTP verify rows) or OSCAR_HISTORY_F8_KERNEL
 * (tcgen05 e4m3, opt-in with OSCAR_HISTORY_F8=1).  Diagnostics for tests and
 * deployments that need to know the dispatch; no reference counterpart. */
#define OSCAR_HISTORY_ATTENTION_KERNEL 1
#define OSCAR_HISTORY_MTP_KERNEL 2
#define OSCAR_HISTORY_F8_KERNEL 3
int oscar_last_history_kernel(void);

/* Test hook for the timeout path of the decode history kernels and the eigensolver (no
 * counterpart in the reference): from the next launch on, CTA (0, 0, 0) of every history
 * launch (the default mma.sync kernels and the opt-in tcgen05 kernel) never issues the
 * copy of its chunk / tile `withhold` (-1: none), CTA 0 of the first matrix's cluster of
 * every oscar_jacobi_rotations launch never pushes its partial sums of round `withhold`,
 * and every bounded device wait of those launches gives up after `wait_probes` probes (0:
 * the default limit of 2^20).  The consumers then time out: a history launch stores
 * OSCAR_ERR_TIMEOUT into its status word, marks the aborted CTA's rows empty (lse -inf),
 * lets its issued copies land and returns; the eigensolver reports info status 3 for that
 * matrix.  Process-wide; for tests only. */
int oscar_test_set_wait_fault(int32_t withhold, uint32_t wait_probes);

/* Y[n,h,:] = bf16( bf16(X[n,h,:]) @ bf16(R) ), fp32 accumulation.
 * Replaces reference oscar_ascend/kernels.py:51-66 (rotate / _rotate_kernel). */
int oscar_rotate(const void *x, int64_t n, int32_t h, int64_t xs0, int64_t xs1, int64_t xs2,
                 const void *r, int64_t rs0, int64_t rs1, void *y, void *stream);

/* Percentile clip + INT2 pack + masked scatter of pre-rotated K/V rows into the
 * history stripe.  krot/vrot: contiguous bf16 [n, H, 256].  Rows whose token index
 * >= counts[1] or whose slot is < 0 are skipped; bytes 136..159 of a slot are
 * never written.  Replaces reference kernels.py:140-202 (store_int2). */
int oscar_store_int2(const void *krot, const void *vrot, int64_t n, void *history,
                     const int64_t *slots, const int32_t *counts, oscar_geometry geo,
                     oscar_clip kclip, oscar_clip vclip, void *stream);

/* Fused: K and V rotation (bf16 GEMM, fp32 accumulation, bf16 rounding) followed by
 * the store_int2 epilogue, plus optionally Q rotation (qrot = Q @ Rk) in the same
 * launch.  key/value/query may be strided [n,H,256] / [n,Hq,256].  krot_out/vrot_out
 * (nullable) receive the bf16 rotated rows for debugging/parity.  Replaces the
 * reference's rotate(K,Rk), rotate(V,Rv), store_int2, rotate(Q,Rk) sequence
 * (backend.py:171-173,195). */
int oscar_rotate_store(const void *key, int64_t ks0, int64_t ks1, const void *value, int64_t vs0,
                       int64_t vs1, int64_t n, const void *rk, const void *rv, void *history,
                       const int64_t *slots, const int32_t *counts, oscar_geometry geo,
                       oscar_clip kclip, oscar_clip vclip, const void *query, int64_t qs0,
                       int64_t qs1, int32_t hq, void *qrot_out, void *krot_out, void *vrot_out,
                       int32_t *status, void *stream);

/* Compact (request, query-offset) task table + optional page-table column copy.
 * Replaces reference kernels.py:222-287 (prepare_tasks / _prepare_tasks_kernel).
 * tasks: int32 [capacity, 2]; task_count: int32[1]. */
int oscar_prepare_tasks(const int32_t *qstarts, const int32_t *counts, int32_t *tasks,
                        int32_t *task_count, int32_t capacity, int32_t max_reqs,
                        int32_t query_tile, const int32_t *source_table,
                        int64_t source_stride, int32_t *table, int64_t table_stride,
                        int32_t copy_columns, void *stream);

/* Fixed per-step metadata arena (int32 words) that CUDA graphs read: words 0-1 the
 * device counts [requests, active tokens], word 2 the task count, word 3 reserved; then,
 * each 16-byte aligned, query starts [max_reqs + 1], sequence lengths [max_reqs], block
 * table [max_reqs, columns] and task table [task_capacity, 2].  Writes the word offsets
 * of {query starts, sequence lengths, block table, tasks, total words} to offsets[0..4].
 * No reference counterpart: the reference keeps five separate device tensors
 * (metadata.py:59-75). */
int oscar_step_arena_layout(int32_t max_reqs, int32_t columns, int32_t task_capacity, int64_t *offsets);

/* Stage one step's metadata into the arena in one launch: counts = {num_reqs,
 * num_tokens}; query starts [0, num_reqs], sequence lengths [0, num_reqs); block-table
 * columns [0, copy_columns) of rows [0, num_reqs) (source rows `table_stride` apart);
 * slot_out[0, num_tokens) = slots; and the compact task table built from the source
 * query starts.  qstarts may be null only when num_reqs = 0: with num_tokens = 0 too
 * that is the dummy / capture step, whose counts and task count become 0 and nothing
 * else is touched.  Replaces the reference builder's copies,
 * fills and prepare_tasks call (metadata.py:108-145, kernels.py:222-287). */
int oscar_stage_step_metadata(const int32_t *qstarts, const int32_t *seq_lens, const int32_t *table,
                              int64_t table_stride, const int64_t *slots, int32_t num_reqs,
                              int32_t num_tokens, int32_t copy_columns, int32_t query_tile,
                              int32_t *arena, int32_t max_reqs, int32_t columns, int32_t task_capacity,
                              int64_t *slot_out, int64_t slot_capacity, void *stream);

/* Split-KV paged attention partials, reference kernels.py:290-482 semantics.
 * raw = 0: INT2 history [sink_len, recent_begin) with rotated query; raw = 1: BF16
 * sink + recent (window) + causal current tokens with the unrotated query, 1 split.
 * partials: fp32 [n, Hq, splits, 256]; lse: fp32 [n, Hq, splits]; rows that are not
 * live are left unwritten.  num_tasks = task slots to cover (attention_programs). */
int oscar_attention_partials(const void *query, int64_t qs0, int64_t qs1, const void *key,
                             int64_t ks0, int64_t ks1, const void *value, int64_t vs0,
                             int64_t vs1, const uint8_t *history, const void *window,
                             const int32_t *qstarts, const int32_t *seq_lens,
                             const int32_t *table, const int32_t *counts, const int32_t *tasks,
                             const int32_t *task_count, int32_t num_tasks, int64_t n,
                             float *partials, float *lse, oscar_geometry geo, float scale,
                             int32_t splits, int32_t raw, int32_t *status, void *stream);

/* LSE merge of split partials -> bf16 out [n,Hq,256] + fp32 logsum [n,Hq]; every row
 * is written (rows >= counts[1] get 0 / -inf).  Reference kernels.py:485-511. */
int oscar_merge_splits(const float *partials, const float *lse, int64_t n, int32_t hq,
                       int32_t splits, const int32_t *counts, void *out, float *logsum,
                       void *stream);

/* LSE merge of the (inverse-rotated) history output a (bf16 [n,Hq,256], la) with the
 * raw partial b (fp32, row stride b_row_stride elements, lb with stride lb_stride)
 * -> out bf16 [n, Hq*256].  Reference kernels.py:514-541. */
int oscar_merge_paths(const void *a, const float *la, const float *b, int64_t b_row_stride,
                      const float *lb, int64_t lb_stride, int64_t n, int32_t hq,
                      const int32_t *counts, void *out, void *stream);

/* Write current BF16 K/V into each request's sink/ring window (latest writer per
 * ring slot).  num_programs = min(n, max_reqs) as in reference kernels.py:598-620. */
int oscar_store_windows(const void *key, int64_t ks0, int64_t ks1, const void *value,
                        int64_t vs0, int64_t vs1, void *window, const int32_t *qstarts,
                        const int32_t *seq_lens, const int32_t *table, const int32_t *counts,
                        int32_t num_programs, oscar_geometry geo, void *stream);

/* Diagnostic unpack of slots into rotated bf16 K/V [n, H, 256] (reference
 * kernels.py:623-648, _unpack_kernel). */
int oscar_unpack(const uint8_t *history, const int64_t *slots, int64_t n, oscar_geometry geo,
                 void *k_out, void *v_out, void *stream);

/* One fused decode / MTP-verify attention step over the paged cache: INT2 history
 * split-KV attention (rotated space), BF16 sink/recent/current attention, split LSE
 * merge, inverse V rotation (hrot @ Rv^T) and path merge into `output` (bf16
 * [n, Hq*256]), then the window store of the current K/V.  Scratch: fp32 partials
 * [n*Hq*(splits+1)*256] and lse [n*Hq*(splits+1)] supplied by the caller.  `splits`
 * (1..64) is the most splits a request may use: each request gets a number of splits
 * proportional to its history, so that every split covers a similar span.
 * Replaces reference backend.py:195-226 (attention_partials x2, merge_splits,
 * rotate(hrot, Rv^T), merge_paths, store_windows). */
int oscar_decode_attention(const void *qrot, const void *query, int64_t qs0, int64_t qs1,
                           const void *key, int64_t ks0, int64_t ks1, const void *value,
                           int64_t vs0, int64_t vs1, const uint8_t *history, void *window,
                           const int32_t *qstarts, const int32_t *seq_lens,
                           const int32_t *table, const int32_t *counts, const int32_t *tasks,
                           const int32_t *task_count, int32_t num_tasks, int64_t n,
                           const void *rv, float *scratch_partials, float *scratch_lse,
                           void *output, oscar_geometry geo, float scale, int32_t splits,
                           int32_t window_programs, int32_t *status, void *stream);

/* oscar_decode_attention without caller scratch, for callers that cannot allocate
 * device memory during decode (an engine whose memory plan already gave all free
 * memory to the KV cache, or an FFI host with no device allocator).  No counterpart in
 * the reference.  The split scratch is a fixed file-scope device array of
 * oscar_decode_attention_noalloc_max_rows() rows (n * Hq * (splits + 1) <= 32768, i.e.
 * 32 MiB of partials) held by every GPU that loads the library; larger calls return
 * OSCAR_ERR_INVALID.  The first call on a device looks up the array's address (make it
 * before any stream capture; a first call on a capturing stream returns
 * OSCAR_ERR_INVALID).  The looked-up address belongs to the device's primary context.
 * All calls on a device share the array, so calls whose GPU work overlaps race;
 * sequential calls need no clearing.  Nothing is allocated. */
int oscar_decode_attention_noalloc(const void *qrot, const void *query, int64_t qs0, int64_t qs1,
                                   const void *key, int64_t ks0, int64_t ks1, const void *value,
                                   int64_t vs0, int64_t vs1, const uint8_t *history, void *window,
                                   const int32_t *qstarts, const int32_t *seq_lens,
                                   const int32_t *table, const int32_t *counts,
                                   const int32_t *tasks, const int32_t *task_count,
                                   int32_t num_tasks, int64_t n, const void *rv, void *output,
                                   oscar_geometry geo, float scale, int32_t splits,
                                   int32_t window_programs, int32_t *status, void *stream);

/* Row capacity of the built-in scratch of oscar_decode_attention_noalloc. */
int64_t oscar_decode_attention_noalloc_max_rows(void);

/* ---- calibration (reference oscar_ascend/calibration_kernels.py) -------------- */

/* cov[256,256] += X^T X over the n*h rows of bf16 X [n,h,256] (strided), or, when
 * weights (fp32 [n*h]) is non-null, += sum_t w_t x_t^T x_t.  Reference :14-70. */
int oscar_accumulate_gram(const void *x, int64_t n, int32_t h, int64_t xs0, int64_t xs1,
                          const float *weights, float *cov, void *stream);

/* w[t] = max(k_t C k_t^T, 0) for the n*h rows of bf16 K, and *total += sum w.
 * K 16-byte aligned with ks0, ks1 multiples of 8 elements (else OSCAR_ERR_INVALID);
 * C fp32, 16-byte aligned.  Reference :73-126 (generalised to any number of heads). */
int oscar_sst_weights(const void *key, int64_t n, int32_t h, int64_t ks0, int64_t ks1,
                      const float *q_cov, float *weights, float *total, void *stream);

/* Grouped Gram: the h heads form `groups` equal groups of consecutive heads; group g
 * accumulates into covs + g*65536 (rows of its heads only), weights as above (indexed
 * by token * h + head).  One launch for all KV heads of a layer where the reference
 * calls accumulate_gram per head (calibration_worker.py:75-82). */
int oscar_accumulate_gram_grouped(const void *x, int64_t n, int32_t h, int64_t xs0, int64_t xs1, int32_t groups,
                                  const float *weights, float *covs, void *stream);

/* Per-head SST weights: head h's rows use q_covs + h*65536 and add into totals[h];
 * weights is fp32 [n*h] indexed token * h + head.  Same arithmetic as
 * oscar_sst_weights, one launch for all heads. */
int oscar_sst_weights_per_head(const void *key, int64_t n, int32_t h, int64_t ks0, int64_t ks1,
                               const float *q_covs, float *weights, float *totals, void *stream);

/* parts (bf16 [matrices][3][256][256], 16-byte aligned) = three bf16 matrices whose sum
 * is each fp32 256x256 matrix of x exactly (hi, mid, lo).  Used once per calibration
 * pass to prepare the query covariances for oscar_sst_weights_split. */
int oscar_split_bf16x3(const float *x, int32_t matrices, void *parts, void *stream);

/* oscar_sst_weights_per_head from pre-split covariances (parts of h matrices, as made by
 * oscar_split_bf16x3) on the tcgen05 tensor cores; the same weights up to the order of
 * the fp32 additions.  OSCAR_ERR_UNSUPPORTED when the key layout does not fit a tensor
 * map (the caller then uses oscar_sst_weights_per_head); status (nullable) receives
 * OSCAR_ERR_TIMEOUT if a device wait gave up. */
int oscar_sst_weights_split(const void *key, int64_t n, int32_t h, int64_t ks0, int64_t ks1, const void *parts,
                            float *weights, float *totals, int32_t *status, void *stream);

/* out = x / max(denominator, 1e-30); the denominator is *device_denominator when
 * non-null, else host_denominator.  Reference :129-156. */
int oscar_normalize(const float *x, int64_t numel, const float *device_denominator,
                    float host_denominator, float *out, void *stream);

/* Batched symmetric EVD of cov [batch,256,256] by parallel cyclic (round-robin)
 * Jacobi, all sweeps in one launch (one thread-block cluster per matrix), then
 * ascending eigenpair sort and R = U * H * P_br.  info: fp32[4] = {sweeps,
 * relative_off_diagonal, status (0 ok, 1 not converged, 2 non-finite, 3 a device wait
 * for the cluster's partial sums timed out), 0}.  batch in [0, 2^20], max_sweeps in
 * [1, 64]; OSCAR_ERR_INVALID otherwise.  Reference :159-327. */
int oscar_jacobi_rotations(const float *cov, int32_t batch, int32_t max_sweeps, float tolerance,
                           float *rotations, float *eigenvalues, float *info, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* OSCAR_B200_H */
