// Codebook-quantized (CQ) projections read straight from the `.cact` v3 blobs.
//
// Replaces the reference's batch-1 GEMV (`CqWeight::matvec_lut_impl` /
// `dot_group`, crates/needle-core/src/cq.rs:721-735, 838-873) and the batched
// GEMM (`matmul_rows_prepared_impl`, cq.rs:632-679). As in the reference the
// activation arrives already rotated by the per-group Walsh-Hadamard transform
// (`prepare_input`, cq.rs:264-274), so the inner loop is a dot product of
// codebook-decoded levels against the rotated activation with one FP16 norm
// per (row, group):  y[o] = sum_g norm[o,g] * sum_k level[idx[o,g,k]] * xh[g,k].
//
// Index unpacking is bit-exact with cq.rs:908-925 (LSB-first bitstream; a
// 2-bit byte holds indices 4b..4b+3 at bits 0-1, 2-3, 4-5, 6-7).
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.hpp"
#include "launch_util.hpp"

namespace nb {

// ----------------------------------------------------------------------------
// GEMV: MT activation rows at most (the batch-1 decode path and small batches).
//
// At these sizes the kernel is latency-bound, so it is ordered around the
// critical path: each lane first issues the 128-bit loads of its row chunks
// and their FP16 norms (weights never change, so this happens before waiting
// on the kernel that produced the activation), then the CTA builds the byte
// table of the codebook (one entry decodes every index of a packed byte, the
// GPU form of cq.rs:932-964; 4 KB for 2-bit, 2 KB for 4-bit), waits for the
// producer (programmatic dependent launch) and stages the activation rows.
// Each output row is split over LPR lanes: lane `sub` of a row takes the row's
// 16-byte chunks sub, sub+LPR, ... The activation rows sit in shared memory
// with a 4-float pad after every chunk-sized block so that lanes working on
// different chunks of the same row hit different banks. 128-thread CTAs keep
// the grid wide: a [3072, 768] 2-bit matrix spreads over 192 CTAs.
// ----------------------------------------------------------------------------
template <int BITS>
struct ChunkTraits;
template <>
struct ChunkTraits<2> {
  static constexpr int E = 64;  // elements per 16-byte chunk
  static constexpr int P = 4;   // levels per byte
};
template <>
struct ChunkTraits<4> {
  static constexpr int E = 32;
  static constexpr int P = 2;
};

constexpr int GV_THREADS = 128;
constexpr int GV_PRE = 2;  // chunks per lane fetched before the producer wait
constexpr int GV_MAX_CTAS = 148 * 8;  // grid cap: row blocks beyond it loop inside the CTAs

__host__ __device__ inline int padded_len(int in_pad, int E) { return in_pad + (in_pad / E) * 4; }

// Segment holding logical row r: walk the segments in order and stop at the
// first one whose end lies beyond r.
__device__ __forceinline__ int find_seg(const CqMat& W, int r, int* local) {
  int s = 0, base = 0;
#pragma unroll
  for (int i = 0; i < MAX_SEG - 1; ++i) {
    if (s == i && i < W.nseg - 1 && r >= base + W.seg[i].rows) {
      base += W.seg[i].rows;
      s = i + 1;
    }
  }
  *local = r - base;
  return s;
}

// Dot of one 16-byte chunk (chunk index c) with the MT staged activation rows.
template <int BITS, int MT>
__device__ __forceinline__ void gemv_chunk(const uint4 w, float nv, int c, const float* lut, const float* xs,
                                           int plen, int M, float (&acc)[MT]) {
  using T = ChunkTraits<BITS>;
  const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
  float part[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) part[m] = 0.f;
  const float* xc = xs + c * (T::E + 4);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
      const int byte = (wd[q] >> (8 * bb)) & 0xff;
      const int e0 = (q * 4 + bb) * T::P;
      if (BITS == 2) {
        const float4 lv = *reinterpret_cast<const float4*>(lut + byte * 4);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < M) {
            const float4 xv = *reinterpret_cast<const float4*>(xc + m * plen + e0);
            part[m] += lv.x * xv.x + lv.y * xv.y + lv.z * xv.z + lv.w * xv.w;
          }
        }
      } else {
        const float2 lv = *reinterpret_cast<const float2*>(lut + byte * 2);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < M) {
            const float2 xv = *reinterpret_cast<const float2*>(xc + m * plen + e0);
            part[m] += lv.x * xv.x + lv.y * xv.y;
          }
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] += nv * part[m];
}

template <int BITS, int LPR, int MT>
__global__ void __launch_bounds__(GV_THREADS) cq_gemv_kernel(CqMat W, const float* __restrict__ xh, int ldx,
                                                             int M, float* __restrict__ y, int ldy, int row0,
                                                             int nrows) {
  using T = ChunkTraits<BITS>;
  extern __shared__ __align__(16) float smem[];
  __shared__ float lev[16];
  const int plen = padded_len(W.in_pad, T::E);
  float* lut = smem;                // [256 * P]
  float* xs = smem + 256 * T::P;    // [MT][plen]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane % LPR;
  const int rows_per_block = (GV_THREADS / 32) * (32 / LPR);
  const int nblocks = (nrows + rows_per_block - 1) / rows_per_block;
  const int nchunks = W.row_bytes / 16;
  // This lane's row in row block `blk` and its first GV_PRE chunks and norms.
  auto fetch = [&](int blk, uint4 (&w)[GV_PRE], float (&nv)[GV_PRE], const uint8_t** row, const __half** nrm) {
    const int r = blk * rows_per_block + warp * (32 / LPR) + lane / LPR;
    *row = nullptr;
    *nrm = nullptr;
    if (blk < nblocks && r < nrows) {
      int local;
      const int s = find_seg(W, row0 + r, &local);
      *row = W.seg[s].packed + (size_t)local * W.row_bytes;
      *nrm = W.seg[s].norms + (size_t)local * W.groups;
    }
#pragma unroll
    for (int j = 0; j < GV_PRE; ++j) {
      const int c = sub + j * LPR;
      const bool ok = *row && c < nchunks;
      w[j] = ok ? __ldg(reinterpret_cast<const uint4*>(*row) + c) : make_uint4(0u, 0u, 0u, 0u);
      nv[j] = ok ? __half2float((*nrm)[c * T::E / W.group]) : 0.f;
    }
  };
  // 1. this lane's first chunks (weights never change, so they are fetched
  // before waiting on the producer of xh)
  uint4 wcur[GV_PRE];
  float ncur[GV_PRE];
  const uint8_t* row;
  const __half* nrm;
  fetch(blockIdx.x, wcur, ncur, &row, &nrm);
  // 2. byte table
  if (threadIdx.x < 16) lev[threadIdx.x] = W.levels[threadIdx.x];
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += GV_THREADS) {
#pragma unroll
    for (int j = 0; j < T::P; ++j) lut[i * T::P + j] = lev[(i >> (j * BITS)) & ((1 << BITS) - 1)];
  }
  // 3. the activation rows, written by the previous kernel
  pdl_wait();
  const int q4 = W.in_pad / 4;
  for (int m = 0; m < M; ++m)
    for (int i = threadIdx.x; i < q4; i += GV_THREADS) {
      const int k = i * 4;
      *reinterpret_cast<float4*>(xs + m * plen + k + (k / T::E) * 4) =
          *reinterpret_cast<const float4*>(xh + (size_t)m * ldx + k);
    }
  __syncthreads();
  pdl_trigger();

  // 4. row blocks blockIdx.x, + gridDim.x, ...: the next block's first chunks
  // are in flight while this block's dots run.
  for (int blk = blockIdx.x; blk < nblocks; blk += gridDim.x) {
    uint4 wnext[GV_PRE];
    float nnext[GV_PRE];
    const uint8_t* rnext;
    const __half* nrnext;
    fetch(blk + gridDim.x, wnext, nnext, &rnext, &nrnext);
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    if (row) {
#pragma unroll
      for (int j = 0; j < GV_PRE; ++j) {
        const int c = sub + j * LPR;
        if (c < nchunks) gemv_chunk<BITS, MT>(wcur[j], ncur[j], c, lut, xs, plen, M, acc);
      }
      for (int c = sub + GV_PRE * LPR; c < nchunks; c += LPR)
        gemv_chunk<BITS, MT>(__ldg(reinterpret_cast<const uint4*>(row) + c), __half2float(nrm[c * T::E / W.group]),
                             c, lut, xs, plen, M, acc);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    }
    const int r = blk * rows_per_block + warp * (32 / LPR) + lane / LPR;
    if (row && sub == 0) {
#pragma unroll
      for (int m = 0; m < MT; ++m)
        if (m < M) y[(size_t)m * ldy + r] = acc[m];
    }
#pragma unroll
    for (int j = 0; j < GV_PRE; ++j) {
      wcur[j] = wnext[j];
      ncur[j] = nnext[j];
    }
    row = rnext;
    nrm = nrnext;
  }
}

// ----------------------------------------------------------------------------
// GEMV for one activation row: partial-sum table per nibble position.
//
// After the activation arrives, the CTA builds, for every nibble position p of
// the packed row (2 codes of 2 bits, or 1 code of 4 bits) and every nibble
// value n, T[p][n] = sum_j level[code_j(n)] * xh[p * E + j] (16 floats per
// position: 24 KB for a 2-bit row of 768). Each lane then owns one output row:
// it reads its packed bytes 16 at a time and adds T[p][nibble] per nibble,
// applying the FP16 norm per quantisation group (cq.rs:666-672 structure). The
// lanes of a warp walk their rows in lockstep, so one table read touches one
// 16-float row of T: distinct nibbles fall in distinct banks and equal ones
// broadcast, so the table reads never conflict. Compared with decoding levels
// and re-reading the activation (32 B of shared memory per 4 codes), a nibble
// costs one 4-byte table read and one add.
// ----------------------------------------------------------------------------
constexpr int G1_THREADS = 128;

template <int BITS>
__global__ void __launch_bounds__(G1_THREADS) cq_gemv1_kernel(CqMat W, const float* __restrict__ xh,
                                                              float* __restrict__ y, int row0, int nrows) {
  constexpr int EN = 4 / BITS;                 // codes per nibble
  constexpr int CPG = 128 * BITS / 8 / 16;     // 16-byte chunks per quantisation group of 128
  extern __shared__ __align__(16) float T[];   // [npos][16]
  __shared__ float lev[16];
  const int npos = W.in_pad / EN;
  const int nchunks = W.row_bytes / 16;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nblocks = (nrows + G1_THREADS - 1) / G1_THREADS;
  if (threadIdx.x < 16) lev[threadIdx.x] = W.levels[threadIdx.x];
  __syncthreads();
  pdl_wait();  // xh is written by the previous kernel
  for (int e = threadIdx.x; e < npos * 16; e += G1_THREADS) {
    const int pos = e >> 4, n = e & 15;
    float v = 0.f;
#pragma unroll
    for (int j = 0; j < EN; ++j) v += lev[(n >> (j * BITS)) & ((1 << BITS) - 1)] * __ldg(xh + pos * EN + j);
    T[e] = v;
  }
  __syncthreads();
  pdl_trigger();
  for (int blk = blockIdx.x; blk < nblocks; blk += gridDim.x) {
    const int r = blk * G1_THREADS + warp * 32 + lane;
    if (r >= nrows) continue;
    int local;
    const int s = find_seg(W, row0 + r, &local);
    const uint4* row = reinterpret_cast<const uint4*>(W.seg[s].packed + (size_t)local * W.row_bytes);
    const __half* nrm = W.seg[s].norms + (size_t)local * W.groups;
    // Four independent partial sums (one per 32-bit word of a chunk) keep four
    // table reads and adds in flight per lane.
    float total = 0.f, gp[4] = {0.f, 0.f, 0.f, 0.f};
    uint4 w = __ldg(row);
    for (int c = 0; c < nchunks; ++c) {
      const uint4 cur = w;
      if (c + 1 < nchunks) w = __ldg(row + c + 1);
      const uint32_t wd[4] = {cur.x, cur.y, cur.z, cur.w};
      const float* tc = T + (size_t)c * 32 * 16;  // 32 nibble positions per chunk
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) gp[q] += tc[(q * 8 + i) * 16 + ((wd[q] >> (4 * i)) & 15)];
      if ((c + 1) % CPG == 0) {
        total += __half2float(nrm[c / CPG]) * ((gp[0] + gp[1]) + (gp[2] + gp[3]));
        gp[0] = gp[1] = gp[2] = gp[3] = 0.f;
      }
    }
    y[r] = total;
  }
}

template <int BITS>
static cudaError_t launch_gemv1(const CqMat& W, const float* xh, float* y, int row0, int nrows, cudaStream_t st) {
  const size_t smem = (size_t)(W.in_pad * BITS / 4) * 16 * sizeof(float);
  const int grid = std::min((nrows + G1_THREADS - 1) / G1_THREADS, GV_MAX_CTAS);
  auto kern = cq_gemv1_kernel<BITS>;
  cudaError_t e = allow_smem((const void*)kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(G1_THREADS), smem, st, W, xh, y, row0, nrows);
}

// Table size the one-row GEMV may stage (shared memory per CTA), and the row
// count from which it is used.
constexpr size_t G1_MAX_TABLE_BYTES = 100 * 1024;
constexpr int G1_MIN_ROWS = 16384;

// ----------------------------------------------------------------------------
// SIMT GEMM for many activation rows (prefill, batched decode).
// Tile: 64 weight rows x 64 activation rows, K stepped one quantisation group
// (128) at a time. The group's packed bytes are decoded once into shared memory
// (levels only; the FP16 norm is applied per group to the fp32 partial, as the
// reference applies `norm * group_dot` in cq.rs:666-672) and reused by every
// activation row of the tile.
// ----------------------------------------------------------------------------
constexpr int GB_N = 64, GB_M = 64, GB_K = 128, GB_KS = 64, GB_PAD = 4;

template <int BITS>
__global__ void __launch_bounds__(256) cq_gemm_simt_kernel(CqMat W, const float* __restrict__ xh,
                                                           int ldx, int M, float* __restrict__ y,
                                                           int ldy, int row0, int nrows) {
  // Half a group (64 of K) is staged at a time so the tiles fit static shared memory.
  __shared__ __align__(16) float Ws[GB_KS][GB_N + GB_PAD];
  __shared__ __align__(16) float Xs[GB_KS][GB_M + GB_PAD];
  __shared__ float Ns[GB_N];
  __shared__ float lev[16];
  const int tid = threadIdx.x;
  if (tid < 16) lev[tid] = W.levels[tid];
  const int n_base = blockIdx.x * GB_N, m_base = blockIdx.y * GB_M;
  const int tn = (tid % 16) * 4, tm = (tid / 16) * 4;
  constexpr int P = 8 / BITS;
  constexpr int BPG = GB_K * BITS / 8;   // packed bytes per group per row
  constexpr int BPS = GB_KS * BITS / 8;  // packed bytes per half group
  // Each thread decodes bytes of one fixed weight row (tid % 64).
  const int my_nl = tid % GB_N;
  const uint8_t* my_row = nullptr;
  const __half* my_norm = nullptr;
  if (n_base + my_nl < nrows) {
    int local;
    int s = find_seg(W, row0 + n_base + my_nl, &local);
    my_row = W.seg[s].packed + (size_t)local * W.row_bytes;
    my_norm = W.seg[s].norms + (size_t)local * W.groups;
  }
  float total[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) total[i][j] = 0.f;
  for (int g = 0; g < W.groups; ++g) {
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int hk = 0; hk < GB_K / GB_KS; ++hk) {
      __syncthreads();
      for (int bi = tid / GB_N; bi < BPS; bi += 256 / GB_N) {
        uint8_t byte = my_row ? my_row[(size_t)g * BPG + hk * BPS + bi] : 0;
#pragma unroll
        for (int j = 0; j < P; ++j) Ws[bi * P + j][my_nl] = lev[(byte >> (j * BITS)) & ((1 << BITS) - 1)];
      }
      if (hk == 0 && tid < GB_N) Ns[tid] = my_norm ? __half2float(my_norm[g]) : 0.f;
      for (int i = tid; i < GB_M * (GB_KS / 4); i += 256) {
        int ml = i % GB_M, k4 = (i / GB_M) * 4;
        int m = m_base + ml;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m < M) v = *reinterpret_cast<const float4*>(xh + (size_t)m * ldx + (size_t)g * GB_K + hk * GB_KS + k4);
        Xs[k4 + 0][ml] = v.x;
        Xs[k4 + 1][ml] = v.y;
        Xs[k4 + 2][ml] = v.z;
        Xs[k4 + 3][ml] = v.w;
      }
      __syncthreads();
#pragma unroll 8
      for (int k = 0; k < GB_KS; ++k) {
        float4 a = *reinterpret_cast<const float4*>(&Xs[k][tm]);
        float4 b = *reinterpret_cast<const float4*>(&Ws[k][tn]);
        float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float nv = Ns[tn + j];
#pragma unroll
      for (int i = 0; i < 4; ++i) total[i][j] += nv * acc[i][j];
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int m = m_base + tm + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int r = n_base + tn + j;
      if (r < nrows) y[(size_t)m * ldy + r] = total[i][j];
    }
  }
}

// ----------------------------------------------------------------------------
// Host dispatch
// ----------------------------------------------------------------------------
template <int BITS, int LPR, int MT>
static cudaError_t launch_gemv(const CqMat& W, const float* xh, int ldx, int M, float* y, int ldy,
                               int row0, int nrows, cudaStream_t st) {
  using T = ChunkTraits<BITS>;
  const int rows_per_cta = (GV_THREADS / 32) * (32 / LPR);
  // One row block per CTA for small matrices; large ones loop over row blocks
  // (the byte table and the activation are staged once per CTA).
  const int grid = std::min((nrows + rows_per_cta - 1) / rows_per_cta, GV_MAX_CTAS);
  const size_t smem = (size_t)(256 * T::P + MT * padded_len(W.in_pad, T::E)) * sizeof(float);
  auto kern = cq_gemv_kernel<BITS, LPR, MT>;
  cudaError_t e = allow_smem((const void*)kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(GV_THREADS), smem, st, W, xh, ldx, M, y, ldy, row0, nrows);
}

template <int BITS, int MT>
static cudaError_t gemv_lpr(const CqMat& W, const float* xh, int ldx, int M, float* y, int ldy,
                            int row0, int nrows, cudaStream_t st) {
  // Lanes per row: at most two chunks per lane, so every load is in flight
  // before the producer wait.
  const int nchunks = W.row_bytes / 16;
  if (nchunks <= 4) return launch_gemv<BITS, 2, MT>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  if (nchunks <= 8) return launch_gemv<BITS, 4, MT>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  if (nchunks <= 16) return launch_gemv<BITS, 8, MT>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  if (nchunks <= 32) return launch_gemv<BITS, 16, MT>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  return launch_gemv<BITS, 32, MT>(W, xh, ldx, M, y, ldy, row0, nrows, st);
}

template <int BITS>
static cudaError_t launch_gemm_simt(const CqMat& W, const float* xh, int ldx, int M, float* y,
                                    int ldy, int row0, int nrows, cudaStream_t st) {
  dim3 grid((nrows + GB_N - 1) / GB_N, (M + GB_M - 1) / GB_M);
  cq_gemm_simt_kernel<BITS><<<grid, 256, 0, st>>>(W, xh, ldx, M, y, ldy, row0, nrows);
  return cudaGetLastError();
}

template <int BITS>
static cudaError_t project_bits(const CqMat& W, const float* xh, int ldx, int M, float* y, int ldy,
                                int row0, int nrows, cudaStream_t st) {
  // Large one-row products stream through the table kernel; smaller ones are
  // latency-bound and take the kernel above, whose set-up is shorter.
  if (M == 1 && nrows >= G1_MIN_ROWS && (size_t)W.in_pad * BITS / 4 * 16 * sizeof(float) <= G1_MAX_TABLE_BYTES)
    return launch_gemv1<BITS>(W, xh, y, row0, nrows, st);
  if (M <= 1) return gemv_lpr<BITS, 1>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  if (M <= 2) return gemv_lpr<BITS, 2>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  if (M <= 4) return gemv_lpr<BITS, 4>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  if (M <= 8) return gemv_lpr<BITS, 8>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  return launch_gemm_simt<BITS>(W, xh, ldx, M, y, ldy, row0, nrows, st);
}

// Argument checks shared by every projection path: the kernels assume 16-byte
// aligned rows and activations and a group of 128.
static bool cq_args_ok(const CqMat& W, const float* xh, int ldx) {
  if (W.group != GB_K || (W.bits != 2 && W.bits != 4)) return false;
  if (W.row_bytes % 16 || W.in_pad % GB_K || ldx % 4 || (reinterpret_cast<uintptr_t>(xh) & 15)) return false;
  if (W.nseg < 1 || W.nseg > MAX_SEG) return false;
  for (int i = 0; i < W.nseg; ++i)
    if (reinterpret_cast<uintptr_t>(W.seg[i].packed) & 15) return false;
  return true;
}

// prepare_input (cq.rs:264-274): zero-pad to a multiple of 128 and rotate
// every group by the normalised Walsh-Hadamard transform. One warp per group.
__global__ void cq_prepare_kernel(const float* __restrict__ x, int in_feat, float* __restrict__ xh,
                                  int ld_out) {
  const int m = blockIdx.x, g = blockIdx.y, lane = threadIdx.x;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int k = g * 128 + lane * 4 + i;
    v[i] = k < in_feat ? x[(size_t)m * in_feat + k] : 0.f;
  }
  fwht128_warp(v);
  reinterpret_cast<float4*>(xh + (size_t)m * ld_out + g * 128)[lane] = make_float4(v[0], v[1], v[2], v[3]);
}

cudaError_t launch_cq_prepare(const float* x, int M, int in_feat, float* xh, int ld_out,
                              cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  const int in_pad = (in_feat + 127) / 128 * 128;
  if (!x || !xh || in_feat <= 0 || ld_out < in_pad || ld_out % 4 || (reinterpret_cast<uintptr_t>(xh) & 15))
    return cudaErrorInvalidValue;
  dim3 grid(M, in_pad / 128);
  cq_prepare_kernel<<<grid, 32, 0, st>>>(x, in_feat, xh, ld_out);
  return cudaGetLastError();
}

static bool umma_scratch_ok(const CqMat& W, int M, int nrows, const GemmScratch* gs) {
  return gs && gs->hi && gs->lo && gs->inv && gs->whi && gs->wlo && gs->elems >= (size_t)M * W.in_pad &&
         gs->rows >= (size_t)M && gs->welems >= (size_t)nrows * W.in_pad;
}

int cq_launches(const CqMat& W, int M, const GemmScratch* gs, int force_path) {
  if (M <= 0) return 0;
  if (force_path == 3 || (force_path == 0 && M > 8 && umma_scratch_ok(W, M, W.rows, gs) && umma_supported(W)))
    return 2;  // operand preparation + tensor-core GEMM
  return 1;
}

cudaError_t cq_project(const CqMat& W, const float* xh, int ldx, int M, float* y, int ldy, int row0,
                       int nrows, cudaStream_t st, int force_path, const GemmScratch* gs) {
  if (M <= 0 || nrows <= 0) return cudaSuccess;
  if (!cq_args_ok(W, xh, ldx) || row0 < 0 || row0 + nrows > W.rows) return cudaErrorInvalidValue;
  if (force_path == 1 && M > 8) return cudaErrorInvalidValue;
  if (force_path < 0 || force_path > 3) return cudaErrorInvalidValue;
  const bool scratch_ok = umma_scratch_ok(W, M, nrows, gs);
  if (force_path == 3) {
    if (!scratch_ok) return cudaErrorInvalidValue;
    return cq_project_umma(W, xh, ldx, M, y, ldy, row0, nrows, st, *gs);
  }
  if (force_path == 0 && M > 8 && scratch_ok && umma_supported(W))
    return cq_project_umma(W, xh, ldx, M, y, ldy, row0, nrows, st, *gs);
  if (force_path == 2)
    return W.bits == 2 ? launch_gemm_simt<2>(W, xh, ldx, M, y, ldy, row0, nrows, st)
                       : launch_gemm_simt<4>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  return W.bits == 2 ? project_bits<2>(W, xh, ldx, M, y, ldy, row0, nrows, st)
                     : project_bits<4>(W, xh, ldx, M, y, ldy, row0, nrows, st);
}

}  // namespace nb
