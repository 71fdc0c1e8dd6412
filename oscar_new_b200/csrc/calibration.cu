// OSCAR calibration on device: covariance Gram accumulation, SST weights,
// normalisation and the batched symmetric eigensolver with U*H*P_br composition.
// Reference: oscar_ascend/calibration_kernels.py:14-327.
//
// Eigensolver: the parallel cyclic (round-robin) Jacobi of the reference, with all
// sweeps inside one launch.  A thread-block cluster of 8 CTAs owns one 256x256
// matrix; CTA r holds rows [32r, 32r+32) of W = C V and of V in registers (the column
// rotations are row-local), and the three dot products that define each rotation are
// summed across the cluster through distributed shared memory.  Cluster barriers are
// hardware barriers (no software spin), and the sweep count is bounded.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace oscar {

// ----------------------------------------------------------------------------
// Gram: cov[i][j] += sum_rows x[i] * x[j] (optionally * w_row).  CTA = 128 x 128
// output tile (blockIdx.y in 0..3) over a chunk of rows (blockIdx.x); fp32 partial
// tile reduced into cov with vector atomics.
// ----------------------------------------------------------------------------
constexpr int kGramRows = 32;  // rows per pipeline step

// blockIdx.z = output group: heads [z*hpg, (z+1)*hpg) accumulate into cov + z*D*D;
// blockIdx.x = a chunk of `chunk` rows (token, head-in-group) of that group.
__global__ void __launch_bounds__(256) gram_kernel(const __nv_bfloat16 *__restrict__ x, int64_t n, int32_t h,
                                                   int64_t xs0, int64_t xs1, const float *__restrict__ w,
                                                   float *__restrict__ cov_base, int32_t hpg, int32_t chunk) {
  __shared__ __align__(16) __nv_bfloat16 si[kGramRows * 128];   // x[row][i-range]
  __shared__ __align__(16) __nv_bfloat16 sj[kGramRows * 128];   // x[row][j-range] (or w*x hi)
  __shared__ __align__(16) __nv_bfloat16 sjl[kGramRows * 128];  // w*x lo part
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ti = blockIdx.y >> 1, tj = blockIdx.y & 1;
  const int group = blockIdx.z;
  float *cov = cov_base + (size_t)group * kDim * kDim;
  const int64_t rows = n * hpg;
  const int64_t r0 = (int64_t)blockIdx.x * chunk;
  const int64_t r1 = min(rows, r0 + chunk);
  const int wm = warp >> 2, wn = warp & 3;  // warp tile 64 (i) x 32 (j)
  float acc[4][4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;
  const bool weighted = w != nullptr;
  for (int64_t rb = r0; rb < r1; rb += kGramRows) {
    __syncthreads();
    // 32 rows x 16 chunks (of 8 bf16) per side
    for (int c = tid; c < kGramRows * 16; c += 256) {
      const int r = c >> 4, ch = c & 15;
      const int64_t row = rb + r;
      uint4 vi = make_uint4(0, 0, 0, 0), vj = vi;
      float wt = 0.f;
      if (row < r1) {
        const int64_t t = row / hpg;
        const int hh = group * hpg + (int)(row % hpg);
        const __nv_bfloat16 *src = x + t * xs0 + hh * xs1;
        vi = *reinterpret_cast<const uint4 *>(src + ti * 128 + ch * 8);
        vj = *reinterpret_cast<const uint4 *>(src + tj * 128 + ch * 8);
        if (weighted) wt = w[t * h + hh];
      }
      const int sw = ((ch ^ (r & 7)) << 3);
      *reinterpret_cast<uint4 *>(si + r * 128 + sw) = vi;
      if (!weighted) {
        *reinterpret_cast<uint4 *>(sj + r * 128 + sw) = vj;
      } else {
        const uint32_t vv[4] = {vj.x, vj.y, vj.z, vj.w};
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float y0 = wt * bf16_bits_to_float(vv[e] & 0xffffu);
          const float y1 = wt * bf16_bits_to_float(vv[e] >> 16);
          hi[e] = pack_bf162(y0, y1);
          lo[e] = pack_bf162(y0 - bf16_bits_to_float(hi[e] & 0xffffu), y1 - bf16_bits_to_float(hi[e] >> 16));
        }
        *reinterpret_cast<uint4 *>(sj + r * 128 + sw) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4 *>(sjl + r * 128 + sw) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kGramRows / 16; ++kk) {
      // A = X^T (i x rows): stored [row][i] -> ldmatrix.trans
      uint32_t a[4][4];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        const int r = kk * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int i = wm * 64 + mi * 16 + ((lane >> 3) & 1) * 8;
        ldmatrix_x4_trans(a[mi], smem_u32(si + r * 128 + (((i >> 3) ^ (r & 7)) << 3)));
      }
#pragma unroll
      for (int part = 0; part < (weighted ? 2 : 1); ++part) {
        const __nv_bfloat16 *sb = part ? sjl : sj;
        uint32_t b[4][2];
#pragma unroll
        for (int nj = 0; nj < 4; nj += 2) {
          uint32_t t4[4];
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int j = wn * 32 + (nj + (lane >> 4)) * 8;
          ldmatrix_x4_trans(t4, smem_u32(sb + r * 128 + (((j >> 3) ^ (r & 7)) << 3)));
          b[nj][0] = t4[0], b[nj][1] = t4[1], b[nj + 1][0] = t4[2], b[nj + 1][1] = t4[3];
        }
#pragma unroll
        for (int mi = 0; mi < 4; ++mi)
#pragma unroll
          for (int nj = 0; nj < 4; ++nj)
            mma_bf16_16816(acc[mi][nj], a[mi][0], a[mi][1], a[mi][2], a[mi][3], b[nj][0], b[nj][1]);
      }
    }
  }
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int nj = 0; nj < 4; ++nj) {
      const int i = ti * 128 + wm * 64 + mi * 16 + g;
      const int j = tj * 128 + wn * 32 + nj * 8 + 2 * t;
      atomicAdd(reinterpret_cast<float2 *>(cov + i * kDim + j), make_float2(acc[mi][nj][0], acc[mi][nj][1]));
      atomicAdd(reinterpret_cast<float2 *>(cov + (i + 8) * kDim + j), make_float2(acc[mi][nj][2], acc[mi][nj][3]));
    }
}

// ----------------------------------------------------------------------------
// SST weights on tensor cores: w_r = max(k_r C k_r^T, 0) for 64 rows per CTA.  C (fp32)
// is split exactly into three bf16 parts (hi + mid + lo carry its 24 significand bits),
// so each bf16 MMA product with the bf16 key is exact and accumulates in fp32, as the
// fp32 FMA form does.  C is taken in 64-row blocks: Y = K C_blk^T (C's rows as B's
// columns; k C k^T is a scalar, so C or C^T give the same sum), then
// w_r += sum_j Y[r][j] k_r[j].  The per-row partials of each (block, warp column) go to
// their own shared-memory slot and are added in a fixed order.
// ----------------------------------------------------------------------------
constexpr int kSstRows = 64;
constexpr int kSstTileBytes = kSstRows * kDim * 2;          // 64 rows of 256 bf16
constexpr int kSstSmem = 4 * kSstTileBytes + 8 * kSstRows * 4;  // K, 3 parts of C, partials

// byte offset of 16-byte chunk c of row r in a [rows][256] bf16 tile (XOR swizzle, so the
// eight rows of an ldmatrix land on distinct banks)
OSCAR_DEVINL uint32_t sst_swz(int r, int c) { return (uint32_t)(r * 512 + ((c ^ (r & 7)) << 4)); }

__global__ void __launch_bounds__(256, 1) sst_tc_kernel(const __nv_bfloat16 *__restrict__ k, int64_t n, int32_t h,
                                                        int64_t ks0, int64_t ks1, const float *__restrict__ c_base,
                                                        float *__restrict__ w, float *__restrict__ total_base,
                                                        int32_t per_head) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *ktile = smem;
  uint8_t *parts = smem + kSstTileBytes;  // [3][64 rows of C][256]
  float *wpart = reinterpret_cast<float *>(smem + 4 * kSstTileBytes);  // [4 blocks][2 halves][64 rows]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gi = lane >> 2, t = lane & 3;
  const int head = per_head ? (int)blockIdx.y : 0;
  const float *c = c_base + (size_t)head * kDim * kDim;
  const int64_t rows = per_head ? n : n * h;
  const int64_t r0 = (int64_t)blockIdx.x * kSstRows;
  auto out_index = [&](int64_t row) { return per_head ? row * h + head : row; };
  // key rows (zero beyond the last row)
  for (int e = tid; e < kSstRows * 32; e += 256) {
    const int r = e >> 5, ch = e & 31;
    const int64_t row = r0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < rows) {
      const __nv_bfloat16 *src = per_head ? k + row * ks0 + head * ks1 : k + (row / h) * ks0 + (row % h) * ks1;
      v = reinterpret_cast<const uint4 *>(src)[ch];
    }
    *reinterpret_cast<uint4 *>(ktile + sst_swz(r, ch)) = v;
  }
  const int wm = warp & 3, wn = warp >> 2;  // rows 16 wm.., columns 32 wn.. of a block
  const uint32_t kbase = smem_u32(ktile), pbase = smem_u32(parts);
#pragma unroll 1
  for (int nb = 0; nb < kDim / kSstRows; ++nb) {
    __syncthreads();  // the previous block's parts are no longer read
    for (int e = tid; e < kSstRows * 32; e += 256) {
      const int jr = e >> 5, ch = e & 31;
      const float4 *src = reinterpret_cast<const float4 *>(c + (size_t)(nb * kSstRows + jr) * kDim + ch * 8);
      const float4 f0 = src[0], f1 = src[1];
      const float x[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
      uint32_t hw[4], mw[4], lw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float hv[2], mv[2], lv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float v = x[2 * q + u];
          hv[u] = round_bf16(v);
          const float r1 = v - hv[u];
          mv[u] = round_bf16(r1);
          lv[u] = round_bf16(r1 - mv[u]);
        }
        hw[q] = pack_bf162(hv[0], hv[1]);
        mw[q] = pack_bf162(mv[0], mv[1]);
        lw[q] = pack_bf162(lv[0], lv[1]);
      }
      const uint32_t off = sst_swz(jr, ch);
      *reinterpret_cast<uint4 *>(parts + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4 *>(parts + kSstTileBytes + off) = make_uint4(mw[0], mw[1], mw[2], mw[3]);
      *reinterpret_cast<uint4 *>(parts + 2 * kSstTileBytes + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    __syncthreads();
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll 4
    for (int ks = 0; ks < kDim / 16; ++ks) {
      uint32_t a[4];
      ldmatrix_x4(a, kbase + sst_swz(16 * wm + (lane & 15), 2 * ks + (lane >> 4)));
#pragma unroll
      for (int part = 0; part < 3; ++part) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t b[4];
          const int nrow = 32 * wn + 16 * hf + ((lane >> 4) << 3) + (lane & 7);
          ldmatrix_x4(b, pbase + part * kSstTileBytes + sst_swz(nrow, 2 * ks + ((lane >> 3) & 1)));
          mma_bf16_16816(acc[2 * hf], a[0], a[1], a[2], a[3], b[0], b[1]);
          mma_bf16_16816(acc[2 * hf + 1], a[0], a[1], a[2], a[3], b[2], b[3]);
        }
      }
    }
    // partial w of rows 16 wm + gi (+8) over this warp's 32 columns
    float s0 = 0.f, s1 = 0.f;
    const int ra = 16 * wm + gi, rb = ra + 8;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int col = nb * kSstRows + 32 * wn + 8 * nt + 2 * t;
      const uint32_t ka = *reinterpret_cast<const uint32_t *>(ktile + sst_swz(ra, col >> 3) + (col & 7) * 2);
      const uint32_t kb = *reinterpret_cast<const uint32_t *>(ktile + sst_swz(rb, col >> 3) + (col & 7) * 2);
      s0 = fmaf(acc[nt][0], bf16_bits_to_float(ka & 0xffffu), s0);
      s0 = fmaf(acc[nt][1], bf16_bits_to_float(ka >> 16), s0);
      s1 = fmaf(acc[nt][2], bf16_bits_to_float(kb & 0xffffu), s1);
      s1 = fmaf(acc[nt][3], bf16_bits_to_float(kb >> 16), s1);
    }
    s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
    if (t == 0) {
      wpart[(nb * 2 + wn) * kSstRows + ra] = s0;
      wpart[(nb * 2 + wn) * kSstRows + rb] = s1;
    }
  }
  __syncthreads();
  if (warp < 2) {
    const int r = tid;  // 0..63
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) v += wpart[q * kSstRows + r];
    v = fmaxf(v, 0.f);
    const bool ok = r0 + r < rows;
    if (ok) w[out_index(r0 + r)] = v;
    float sum = ok ? v : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) atomicAdd(total_base + head, sum);
  }
}

__global__ void normalize_kernel(const float *__restrict__ x, int64_t numel, const float *__restrict__ dden,
                                 float hden, float *__restrict__ out) {
  const float den = fmaxf(dden ? dden[0] : hden, 1e-30f);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < numel; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = x[i] / den;
}

// ----------------------------------------------------------------------------
// Jacobi eigensolver, one 8-CTA cluster per matrix
// ----------------------------------------------------------------------------
constexpr int kJCtas = 8;
constexpr int kJRows = kDim / kJCtas;  // 32 rows per CTA
constexpr int kJGroups = kDim / 4;  // groups of two pairs of a round
constexpr int kJThreads = 4 * kJGroups;  // 8 warps: 4 lanes (8 rows each) per group
constexpr int kJWarps = kJThreads / 32;
constexpr int kJLaneRows = kJRows / 4;  // rows per lane
constexpr int kJPairStride = 4 * kJCtas + 2;  // doubles per pair in JacobiSmem::all

struct JacobiSmem {
  double a[kJRows][kDim];  // local rows of W = C V at the start and the end; epilogue scratch
  double u[kJRows][kDim];  // local rows of V (the accumulated rotations), likewise
  // every CTA's a_pp, a_qq, a_pq of each pair, pushed here (group m, pair k, CTA c at
  // [m][k * kJPairStride + 4c]); double-buffered by round.  The 560-byte group stride
  // keeps the 16-byte reads of a quarter warp (two groups x four lanes) on distinct banks.
  double all[2][kJGroups][2 * kJPairStride + 2];
  // (W, V) rows of the q columns leaving a warp's last group and of the p columns leaving
  // its first group, lane-interleaved: four lanes store 64 contiguous bytes per row
  double2 edge_q[kJWarps][kJLaneRows][4];
  double2 edge_p[kJWarps][kJLaneRows][4];
  double diag[kDim];
  double evpart[kDim];                    // this CTA's share of the Rayleigh quotients
  uint64_t xbar[2];                       // completes when all[b] holds every CTA's sums
  int32_t abort;                          // a wait for the sums gave up
  int32_t hook_round;                     // test hook: this CTA skips its pushes of this round
  uint32_t wait_probes;                   // probes of a wait before it gives up
};
constexpr uint32_t kJXBytes = kJCtas * kJGroups * 2 * 24;  // bytes pushed into a CTA per round

// shared::cluster address of `p` (this CTA's shared memory) in CTA `rank` of the cluster
OSCAR_DEVINL uint32_t cluster_addr(const void *p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

// stores into another CTA's shared memory that complete their bytes on its mbarrier;
// issued only when `on` is non-zero (a predicate, not a branch)
OSCAR_DEVINL void st_async_f64x2(uint32_t addr, double a, double b, uint32_t bar, uint32_t on) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
      " @p st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f64 [%0], {%1, %2}, [%3];\n}" ::"r"(addr),
      "d"(a), "d"(b), "r"(bar), "r"(on)
      : "memory");
}
OSCAR_DEVINL void st_async_f64(uint32_t addr, double a, uint32_t bar, uint32_t on) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %3, 0;\n"
      " @p st.async.shared::cluster.mbarrier::complete_tx::bytes.f64 [%0], %1, [%2];\n}" ::"r"(addr),
      "d"(a), "r"(bar), "r"(on)
      : "memory");
}

// bounded wait for a phase whose bytes other CTAs of the cluster wrote
OSCAR_DEVINL bool mbar_wait_cluster_bounded(uint64_t *bar, uint32_t phase, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.u32 "
        "%0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// x mod (D-1) for x in (-(D-1), 2(D-1)): two conditional corrections, no division.
OSCAR_DEVINL int mod_dm1(int x) {
  x += x < 0 ? (kDim - 1) : 0;
  return x >= kDim - 1 ? x - (kDim - 1) : x;
}

OSCAR_DEVINL void round_pair(int j, int r, int &p, int &q) {
  if (j == 0) {
    p = kDim - 1;
    q = r;
  } else {
    p = mod_dm1(r + j);
    q = mod_dm1(r - j);
  }
}

// Cyclic Jacobi with the reference's rotations (two-sided on A = V^T C V), carried out
// on columns only: V starts as I and W = C V as C, and every round applies the 128
// disjoint rotations of the reference's round-robin schedule to the columns of both.
// The rotation of pair (p, q) needs a_pp = v_p . w_p, a_qq = v_q . w_q and
// a_pq = v_p . w_q, the entries of the implicit A; its formula, skip rule and
// convergence test (max|a_pq| / max|a_pp| of a sweep) are the reference's.  Column
// updates are row-local, so a round needs only the cluster sums of the three dot
// products: each CTA pushes its sums over its 32 rows into every CTA of the cluster with
// st.async stores that complete on the receiving CTA's mbarrier, and waits (bounded) for
// the eight pushes it receives; there is no cluster barrier per round.  The eigenvalues
// are the Rayleigh quotients v_p . w_p.  fp64 arithmetic (the reference uses fp32).
//
// The columns live in registers.  Round r pairs seat k with seat 255 - k (pair k,
// k = 1..127; pair 0 = seat 0 with column 255), and column x sits at seat x - r mod 255:
// from one round to the next every column moves one seat down the ring.  Pairs 2m and
// 2m + 1 (group m) are held by lanes 4(m % 8) .. 4(m % 8) + 3 of warp m / 8, lane g of
// them holding rows 8g .. 8g + 7 of the four columns of W and V.  Half of the moves stay
// inside a group (register copies); the other half are a shuffle by 4 lanes, with the
// columns that cross a warp boundary staged in shared memory, so a round reads no
// matrix data from shared memory.
OSCAR_DEVINL double rsqrt_f64(double x) {
  // fp32 seed (about 23 bits), two Newton steps (about 46 bits, then fp64 precision)
  double y = (double)rsqrtf((float)x);
  y = y * fma(-0.5 * x, y * y, 1.5);
  y = y * fma(-0.5 * x, y * y, 1.5);
  return y;
}

OSCAR_DEVINL double rcp_f64(double x) {
  double y = (double)__frcp_rn((float)x);
  y = y * fma(-x, y, 2.0);
  y = y * fma(-x, y, 2.0);
  return y;
}

// withhold / wait_probes: the test hook of oscar_test_set_wait_fault (-1 / kWaitLimit
// outside tests)
__global__ void __launch_bounds__(kJThreads, 1) jacobi_kernel(const float *__restrict__ cov, int32_t max_sweeps,
                                                             float tol, float *__restrict__ rot,
                                                             float *__restrict__ evals, float *__restrict__ info,
                                                             int32_t withhold, uint32_t wait_probes) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  JacobiSmem &S = *reinterpret_cast<JacobiSmem *>(smem_raw);
  __shared__ double wo[kJWarps], wd[kJWarps];
  __shared__ int wf[kJWarps];
  __shared__ int rank_of[kDim];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int batch = blockIdx.x / kJCtas;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float *C = cov + (size_t)batch * kDim * kDim;
  const int row0 = rank * kJRows;
  if (tid == 0) {
    mbar_init(&S.xbar[0], 1);
    mbar_init(&S.xbar[1], 1);
    S.abort = 0;
    S.hook_round = batch == 0 && rank == 0 ? withhold : -1;
    S.wait_probes = wait_probes;
    fence_mbarrier_init();
  }
  for (int e = tid; e < kJRows * kDim; e += kJThreads) {
    const int r = e / kDim, c = e % kDim;
    const int gr = row0 + r;
    S.a[r][c] = ((double)C[gr * kDim + c] + (double)C[c * kDim + gr]) * 0.5;
    S.u[r][c] = gr == c ? 1.0 : 0.0;
  }
  cluster.sync();  // every CTA's barriers are initialised before the first push
  // this lane's two pairs (seats of round 0) and rows
  const int m = tid >> 2, g = tid & 3;
  double wp[2][kJLaneRows], wq[2][kJLaneRows], vp[2][kJLaneRows], vq[2][kJLaneRows];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    int p, q;
    round_pair(2 * m + k, 0, p, q);
#pragma unroll
    for (int i = 0; i < kJLaneRows; ++i) {
      const int lr = g * kJLaneRows + i;
      wp[k][i] = S.a[lr][p], wq[k][i] = S.a[lr][q], vp[k][i] = S.u[lr][p], vq[k][i] = S.u[lr][q];
    }
  }
  double residual = INFINITY;
  int sweeps_done = 0;
  bool finite = true, timed_out = false;
  uint32_t round_no = 0;  // rounds so far: buffer round_no & 1, its phase (round_no >> 1) & 1
  for (int sweep = 0; sweep < max_sweeps && !timed_out; ++sweep) {
    double smax = 0.0, dmax = 0.0;  // largest |a_pq| and |a_pp| seen in this sweep
    bool sfin = true;
#pragma unroll 1
    for (int r = 0; r < kDim - 1; ++r, ++round_no) {
      const int buf = (int)(round_no & 1u);
      if (tid == 0) mbar_arrive_expect_tx(&S.xbar[buf], kJXBytes);
      // (1) this CTA's a_pp, a_qq, a_pq of the lane's pairs over its 32 rows (each lane
      // 8 rows, then (g0 + g1) + (g2 + g3)); lane g pushes them into CTAs g, g + 4, whose
      // barrier for this buffer counts the bytes.  A CTA writes buffer b of round n + 2
      // only after every CTA's sums of round n + 1 reached it, and each CTA pushes those
      // after it has read its sums of round n, so double buffering needs no barrier.
      {
        double app[2] = {0.0, 0.0}, aqq[2] = {0.0, 0.0}, apq[2] = {0.0, 0.0};
#pragma unroll
        for (int k = 0; k < 2; ++k)
#pragma unroll
          for (int i = 0; i < kJLaneRows; ++i) {
            app[k] = fma(vp[k][i], wp[k][i], app[k]);
            aqq[k] = fma(vq[k][i], wq[k][i], aqq[k]);
            apq[k] = fma(vp[k][i], wq[k][i], apq[k]);
          }
#pragma unroll
        for (int s = 1; s <= 2; s <<= 1)
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            app[k] += __shfl_xor_sync(0xffffffffu, app[k], s);
            aqq[k] += __shfl_xor_sync(0xffffffffu, aqq[k], s);
            apq[k] += __shfl_xor_sync(0xffffffffu, apq[k], s);
          }
        const uint32_t on = (int32_t)round_no != S.hook_round;  // test hook: pushes skipped
#pragma unroll
        for (int c = g; c < kJCtas; c += 4) {
          const uint32_t dst = cluster_addr(S.all[buf][m] + 4 * rank, (uint32_t)c);
          const uint32_t bar = cluster_addr(&S.xbar[buf], (uint32_t)c);
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            st_async_f64x2(dst + 8u * (uint32_t)(k * kJPairStride), app[k], aqq[k], bar, on);
            st_async_f64(dst + 8u * (uint32_t)(k * kJPairStride + 2), apq[k], bar, on);
          }
        }
      }
      if (!mbar_wait_cluster_bounded(&S.xbar[buf], (round_no >> 1) & 1u, S.wait_probes)) S.abort = 1;
      // (2) cluster sums and the rotation of each pair: lane g adds CTAs g and g + 4, a
      // fixed shuffle tree adds the rest (the same order in every CTA, so every CTA and
      // every lane of the group derives the same rotations)
      double cs[2], sn[2];
      {
        double app[2], aqq[2], apq[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const double2 *x = reinterpret_cast<const double2 *>(S.all[buf][m] + k * kJPairStride + 4 * g);
          const double2 a01 = x[0], a2_ = x[1], b01 = x[8], b2_ = x[9];
          app[k] = a01.x + b01.x;
          aqq[k] = a01.y + b01.y;
          apq[k] = a2_.x + b2_.x;
        }
#pragma unroll
        for (int s = 1; s <= 2; s <<= 1)
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            app[k] += __shfl_xor_sync(0xffffffffu, app[k], s);
            aqq[k] += __shfl_xor_sync(0xffffffffu, aqq[k], s);
            apq[k] += __shfl_xor_sync(0xffffffffu, apq[k], s);
          }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (!isfinite(app[k]) || !isfinite(aqq[k]) || !isfinite(apq[k])) sfin = false;
          smax = fmax(smax, fabs(apq[k]));
          dmax = fmax(dmax, fmax(fabs(app[k]), fabs(aqq[k])));
          const double delta = (aqq[k] - app[k]) * 0.5;
          const double sgn = delta >= 0.0 ? 1.0 : -1.0;
          const double h2 = fma(delta, delta, apq[k] * apq[k]);
          const double h = h2 > 0.0 ? h2 * rsqrt_f64(h2) : 0.0;
          double tang = sgn * apq[k] * rcp_f64(fmax(fabs(delta) + h, 1e-300));
          if (!(fabs(apq[k]) > 1e-8 * (fabs(app[k]) + fabs(aqq[k])) + 1e-20)) tang = 0.0;
          cs[k] = rsqrt_f64(fma(tang, tang, 1.0));
          sn[k] = tang * cs[k];
        }
      }
      // (3) rotate columns p, q of the lane's rows of W and V
#pragma unroll
      for (int k = 0; k < 2; ++k)
#pragma unroll
        for (int i = 0; i < kJLaneRows; ++i) {
          const double w0 = wp[k][i], w1 = wq[k][i], u0 = vp[k][i], u1 = vq[k][i];
          wp[k][i] = w0 * cs[k] - w1 * sn[k];
          wq[k][i] = w0 * sn[k] + w1 * cs[k];
          vp[k][i] = u0 * cs[k] - u1 * sn[k];
          vq[k][i] = u0 * sn[k] + u1 * cs[k];
        }
      // (4) every column one seat down.  Within a group: pair 2m takes pair 2m + 1's p,
      // pair 2m + 1 takes pair 2m's q.  Across groups: pair 2m takes group m - 1's second
      // q, pair 2m + 1 group m + 1's first p.  Pair 0 keeps column 255 and takes pair 1's
      // p as its q; pair 127 turns its q into its p.  Columns crossing a warp boundary go
      // through shared memory (the previous round's readers are past this round's
      // cluster barrier).
      if (lane >= 28) {
#pragma unroll
        for (int i = 0; i < kJLaneRows; ++i) S.edge_q[warp][i][g] = make_double2(wq[1][i], vq[1][i]);
      }
      if (lane < 4) {
#pragma unroll
        for (int i = 0; i < kJLaneRows; ++i) S.edge_p[warp][i][g] = make_double2(wp[0][i], vp[0][i]);
      }
      __syncthreads();
      if (S.abort) {  // CTA-uniform after the barrier: stop the sweeps (others time out too)
        timed_out = true;
        break;
      }
#pragma unroll
      for (int i = 0; i < kJLaneRows; ++i) {
        const double wq_up = __shfl_up_sync(0xffffffffu, wq[1][i], 4);
        const double vq_up = __shfl_up_sync(0xffffffffu, vq[1][i], 4);
        const double wp_dn = __shfl_down_sync(0xffffffffu, wp[0][i], 4);
        const double vp_dn = __shfl_down_sync(0xffffffffu, vp[0][i], 4);
        double nwq0, nvq0, nwp1, nvp1;
        if (m == 0) {
          nwq0 = wp[1][i], nvq0 = vp[1][i];
        } else if (lane >= 4) {
          nwq0 = wq_up, nvq0 = vq_up;
        } else {
          const double2 e = S.edge_q[warp - 1][i][g];
          nwq0 = e.x, nvq0 = e.y;
        }
        if (m == kJGroups - 1) {
          nwp1 = wq[1][i], nvp1 = vq[1][i];
        } else if (lane < 28) {
          nwp1 = wp_dn, nvp1 = vp_dn;
        } else {
          const double2 e = S.edge_p[warp + 1][i][g];
          nwp1 = e.x, nvp1 = e.y;
        }
        if (m != 0) wp[0][i] = wp[1][i], vp[0][i] = vp[1][i];
        wq[1][i] = wq[0][i], vq[1][i] = vq[0][i];
        wq[0][i] = nwq0, vq[0][i] = nvq0;
        wp[1][i] = nwp1, vp[1][i] = nvp1;
      }
    }
    if (timed_out) break;
    sweeps_done = sweep + 1;
    // the sweep's residual (identical in every CTA: the same sums in the same order)
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      smax = fmax(smax, __shfl_xor_sync(0xffffffffu, smax, o));
      dmax = fmax(dmax, __shfl_xor_sync(0xffffffffu, dmax, o));
    }
    sfin = __all_sync(0xffffffffu, sfin);
    if (lane == 0) wo[warp] = smax, wd[warp] = dmax, wf[warp] = sfin;
    __syncthreads();
    double o = 0.0, d = 0.0;
    int f = 1;
    for (int w = 0; w < kJWarps; ++w) o = fmax(o, wo[w]), d = fmax(d, wd[w]), f &= wf[w];
    __syncthreads();
    finite = f != 0 && isfinite(o) && isfinite(d);
    residual = finite ? o / fmax(d, 1e-300) : INFINITY;
    if (!finite || residual < (double)tol) break;
  }
  // after whole sweeps the columns sit at their round-0 seats again
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    int p, q;
    round_pair(2 * m + k, 0, p, q);
#pragma unroll
    for (int i = 0; i < kJLaneRows; ++i) {
      const int lr = g * kJLaneRows + i;
      S.a[lr][p] = wp[k][i], S.a[lr][q] = wq[k][i], S.u[lr][p] = vp[k][i], S.u[lr][q] = vq[k][i];
    }
  }
  __syncthreads();
  // eigenvalues: Rayleigh quotients v_p . w_p, summed over the cluster's rows
  for (int i = tid; i < kDim; i += kJThreads) {
    double acc = 0.0;
    for (int lr = 0; lr < kJRows; ++lr) acc = fma(S.u[lr][i], S.a[lr][i], acc);
    S.evpart[i] = acc;
  }
  cluster.sync();
  for (int i = tid; i < kDim; i += kJThreads) {
    double acc = 0.0;
    for (int c = 0; c < kJCtas; ++c) acc += cluster.map_shared_rank(&S, c)->evpart[i];
    S.diag[i] = acc;
  }
  cluster.sync();
  for (int i = tid; i < kDim; i += kJThreads) {
    const double v = S.diag[i];
    int rk = 0;
    for (int k2 = 0; k2 < kDim; ++k2) {
      const double o = S.diag[k2];
      rk += (o < v) || (o == v && k2 < i);
    }
    rank_of[i] = rk;
    if (rank == 0) evals[(size_t)batch * kDim + rk] = (float)v;
  }
  __syncthreads();
  // sorted U rows (local), Hadamard butterfly, bit-reversed placement, / sqrt(256)
  for (int e = tid; e < kJRows * kDim; e += kJThreads) {
    const int lr = e / kDim, i = e % kDim;
    S.a[lr][rank_of[i]] = S.u[lr][i];
  }
  __syncthreads();
  for (int lr = warp; lr < kJRows; lr += kJWarps) {
    double v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = S.a[lr][8 * lane + e];
#pragma unroll
    for (int bit = 0; bit < 3; ++bit) {
      double nv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const double partner = v[e ^ (1 << bit)];
        nv[e] = (e & (1 << bit)) ? partner - v[e] : v[e] + partner;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = nv[e];
    }
#pragma unroll
    for (int bit = 3; bit < 8; ++bit) {
      const int lm = 1 << (bit - 3);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const double partner = __shfl_xor_sync(0xffffffffu, v[e], lm);
        v[e] = (lane & lm) ? partner - v[e] : v[e] + partner;
      }
    }
    float *dst = rot + ((size_t)batch * kDim + row0 + lr) * kDim;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = 8 * lane + e;
      const int rev = __brev((unsigned)(kDim - 1 - i)) >> 24;
      dst[rev] = (float)(v[e] * 0.0625);
    }
  }
  if (rank == 0 && tid == 0) {
    float *inf4 = info + (size_t)batch * 4;
    inf4[0] = (float)sweeps_done;
    inf4[1] = (float)residual;
    inf4[2] = timed_out ? 3.f : (!finite ? 2.f : (residual < (double)tol ? 0.f : 1.f));
    inf4[3] = 0.f;
  }
  cluster.sync();  // keep shared memory alive until every remote read is done
}

}  // namespace oscar

using namespace oscar;

namespace oscar {
int32_t test_hook_withhold();      // oscar_test_set_wait_fault state (attention.cu)
uint32_t test_hook_wait_probes();
int gram_tc_launch(const void *x, int64_t n, int32_t h, int64_t xs0, int64_t xs1, int32_t groups,
                   const float *weights, float *cov, int32_t *status, int sm_count, cudaStream_t stream);
}

// The tcgen05 Gram (gram_tc.cu) is the default; OSCAR_GRAM_MMA=1 (read at every call)
// selects the mma.sync gram_kernel, which also serves layouts a tensor map cannot take.
static bool gram_mma_forced() {
  const char *v = getenv("OSCAR_GRAM_MMA");
  return v != nullptr && v[0] == '1';
}

static int device_sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 148;
  return sms;
}

static int launch_gram(const void *x, int64_t n, int32_t h, int64_t xs0, int64_t xs1, int32_t groups,
                       const float *weights, float *cov, void *stream) {
  if (n < 0 || h <= 0 || groups <= 0 || h % groups || !cov) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!x || (reinterpret_cast<uintptr_t>(x) & 15) || xs0 % 8 || xs1 % 8) return OSCAR_ERR_INVALID;
  if (!gram_mma_forced()) {
    const int rc = gram_tc_launch(x, n, h, xs0, xs1, groups, weights, cov, nullptr, device_sm_count(),
                                  (cudaStream_t)stream);
    if (rc != OSCAR_ERR_UNSUPPORTED) return rc;
  }
  const int hpg = h / groups;
  const int64_t rows = n * hpg;
  // chunks sized so that the launch covers about two waves of 148 SMs
  const int64_t want = std::max<int64_t>(1, (2 * 148 + 4 * groups - 1) / (4 * groups));
  int64_t chunk = (rows + want - 1) / want;
  chunk = std::max<int64_t>(256, std::min<int64_t>(4096, (chunk + kGramRows - 1) / kGramRows * kGramRows));
  dim3 grid((unsigned)((rows + chunk - 1) / chunk), 4, (unsigned)groups);
  gram_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<const __nv_bfloat16 *>(x), n, h, xs0, xs1,
                                                      weights, cov, hpg, (int32_t)chunk);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_accumulate_gram(const void *x, int64_t n, int32_t h, int64_t xs0, int64_t xs1,
                                     const float *weights, float *cov, void *stream) {
  return launch_gram(x, n, h, xs0, xs1, 1, weights, cov, stream);
}

extern "C" int oscar_accumulate_gram_grouped(const void *x, int64_t n, int32_t h, int64_t xs0, int64_t xs1,
                                             int32_t groups, const float *weights, float *covs, void *stream) {
  return launch_gram(x, n, h, xs0, xs1, groups, weights, covs, stream);
}

extern "C" int oscar_sst_weights(const void *key, int64_t n, int32_t h, int64_t ks0, int64_t ks1, const float *q_cov,
                                 float *weights, float *total, void *stream) {
  if (n < 0 || h <= 0 || !q_cov || !weights || !total) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!key || (reinterpret_cast<uintptr_t>(key) & 15) || ks0 % 8 || ks1 % 8) return OSCAR_ERR_INVALID;
  const int64_t rows = n * h;
  if (!ensure_dynamic_smem<sst_tc_kernel>(kSstSmem)) return OSCAR_ERR_LAUNCH;
  sst_tc_kernel<<<(unsigned)((rows + kSstRows - 1) / kSstRows), 256, kSstSmem, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16 *>(key), n, h, ks0, ks1, q_cov, weights, total, 0);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_sst_weights_per_head(const void *key, int64_t n, int32_t h, int64_t ks0, int64_t ks1,
                                          const float *q_covs, float *weights, float *totals, void *stream) {
  if (n < 0 || h <= 0 || !q_covs || !weights || !totals) return OSCAR_ERR_INVALID;
  if (n == 0) return OSCAR_OK;
  if (!key || (reinterpret_cast<uintptr_t>(key) & 15) || ks0 % 8 || ks1 % 8) return OSCAR_ERR_INVALID;
  if (!ensure_dynamic_smem<sst_tc_kernel>(kSstSmem)) return OSCAR_ERR_LAUNCH;
  dim3 grid((unsigned)((n + kSstRows - 1) / kSstRows), (unsigned)h);
  sst_tc_kernel<<<grid, 256, kSstSmem, (cudaStream_t)stream>>>(reinterpret_cast<const __nv_bfloat16 *>(key), n, h,
                                                               ks0, ks1, q_covs, weights, totals, 1);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_normalize(const float *x, int64_t numel, const float *device_denominator, float host_denominator,
                               float *out, void *stream) {
  if (numel < 0 || !x || !out) return OSCAR_ERR_INVALID;
  if (numel == 0) return OSCAR_OK;
  const unsigned blocks = (unsigned)std::min<int64_t>((numel + 255) / 256, 4096);
  normalize_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(x, numel, device_denominator, host_denominator, out);
  OSCAR_CHECK_LAUNCH();
  return OSCAR_OK;
}

extern "C" int oscar_jacobi_rotations(const float *cov, int32_t batch, int32_t max_sweeps, float tolerance,
                                      float *rotations, float *eigenvalues, float *info, void *stream) {
  // batch <= 2^20 keeps the grid (8 CTAs per matrix) inside int range
  if (batch < 0 || batch > (1 << 20) || max_sweeps <= 0 || max_sweeps > 64 || !(tolerance > 0.f))
    return OSCAR_ERR_INVALID;
  if (batch == 0) return OSCAR_OK;
  if (!cov || !rotations || !eigenvalues || !info) return OSCAR_ERR_INVALID;
  const int smem = (int)sizeof(JacobiSmem);
  if (!ensure_dynamic_smem<jacobi_kernel>(smem)) return OSCAR_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kJCtas * batch);
  cfg.blockDim = dim3(kJThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kJCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, jacobi_kernel, cov, max_sweeps, tolerance, rotations, eigenvalues, info,
                         test_hook_withhold(), test_hook_wait_probes()) != cudaSuccess) {
    cudaGetLastError();
    return OSCAR_ERR_LAUNCH;
  }
  return OSCAR_OK;
}
