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
#include <cmath>

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
// Tensor-core GEMV: up to 8 activation rows on mma.sync m16n8k16 (f16 x f16
// -> f32), for codebooks whose levels (times a power of two) are f16 values.
//
// A warp owns tiles of 16 weight rows. Per 128-element quantisation group
// (cq.rs:666-672) it issues 8 MMAs of K = 16 into a fresh accumulator and adds
// norm * accumulator to an f32 total, so the tensor cores never accumulate
// across more than one group. The A operand is the levels of the packed
// codes, decoded in registers straight from the `.cact` bytes:
//   * 2-bit: half the bytes by byte_perm - a selector-byte table held in a
//     register maps four 2-bit codes at once to the byte selectors of their
//     f16 levels, and a second byte_perm picks two levels out of the 8-byte
//     level table (about 1.3 integer instructions per code) - and half by a
//     256-entry table of level quads (one 8-byte entry per packed byte, 16
//     copies so that each half-warp reads its own banks). The integer pipe
//     runs logical and permute instructions at half rate, and a table costs
//     shared-memory bandwidth per decoded value; splitting the decode between
//     them loads both pipes;
//   * 4-bit: a 256-entry table of level pairs (one f16x2 per packed byte),
//     replicated per lane so that every lane reads its own bank.
// The K order inside a group is the one the decode produces (the sum over a
// group does not depend on it); the activation is staged once per CTA in
// shared memory in that order, as the B fragments of each group and K step.
// The B operand's 8 columns carry each activation row split into an f16 high
// part and remainder (row scaled by a power of two first), so one MMA yields
// both halves: column 2m is x_hi * level, column 2m + 1 is x_lo * level, and
// every product is exact in f32 (about 22 bits of the activation kept).
// ----------------------------------------------------------------------------
constexpr int TG_THREADS = 128;
constexpr int TG_CTAS_PER_SM = 5;

template <int BITS>
struct TcTraits;
template <>
struct TcTraits<2> {
  static constexpr int GB = 4;     // groups per work item
  static constexpr int BYTES = 8;  // packed bytes of one group per lane and row
};
template <>
struct TcTraits<4> {
  static constexpr int GB = 2;
  static constexpr int BYTES = 16;
};

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Sixteen 2-bit codes c0..c15 of `w` (LSB first) -> eight f16x2 level pairs,
// in the order (c0,c2) (c4,c6) (c8,c10) (c12,c14) (c1,c3) (c5,c7) (c9,c11)
// (c13,c15). `la` holds the f16 levels 0 and 1, `lb` levels 2 and 3. The
// selector bytes of level c are (2c, 2c+1) = 34c + 16, which byte_perm reads
// out of 0x76543210 with the code itself as the selector nibble.
__device__ __forceinline__ void decode2(uint32_t w, uint32_t la, uint32_t lb, uint32_t (&v)[8]) {
  const uint32_t e = w & 0x33333333u, o = (w >> 2) & 0x33333333u;
  const uint32_t win[4] = {e, e >> 16, o, o >> 16};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t s = __byte_perm(0x76543210u, 0u, win[i]);
    v[2 * i] = __byte_perm(la, lb, s);
    v[2 * i + 1] = __byte_perm(la, lb, s >> 16);
  }
}

// Offset inside the lane's 32 codes of a group (2-bit: the lane's 8 packed
// bytes, two words of 16 codes) of element e (0..3 = a0.lo, a0.hi, a2.lo,
// a2.hi) of K step j: decode2's order for a word decoded by byte_perm (steps
// 0..3 always, steps 4..7 when `table` is false), the codes of byte j - 4 of
// the second word in order when it is decoded through the table.
__host__ __device__ __forceinline__ int tc_code_offset(int bits, int j, int e, bool table) {
  if (bits == 4 || (table && j >= 4)) return 4 * j + e;
  const int s = j & 3;
  return 16 * (j >> 2) + (s >> 1) + 8 * (s & 1) + 2 * e;
}

// The codebook levels times 2^le as f16 bit patterns, two per word (level 2i
// in the low half of h[i]).
struct TcLevels {
  uint32_t h[8];
};

// f16 high part (h = 0) or remainder (h = 1) of x.
__device__ __forceinline__ uint32_t f16_part(float x, int h) {
  const __half hi = __float2half_rn(x);
  return h ? (uint32_t)__half_as_ushort(__float2half_rn(x - __half2float(hi))) : (uint32_t)__half_as_ushort(hi);
}

// SPLIT = false: warps own whole tiles (warp-strided over the matrix), GB
// consecutive groups per work item. SPLIT = true (small matrices, where the
// latency of one warp walking every group of a tile dominates): a CTA owns a
// tile, warp w takes groups w, w + 4, ... (GB of them per item, the same item
// count for every warp) and the four partial sums meet in shared memory in a
// fixed order.
template <int BITS, int NT, bool SPLIT>
__global__ void __launch_bounds__(TG_THREADS) cq_gemv_tc_kernel(CqMat W, const float* __restrict__ xh, int ldx,
                                                                int M, float* __restrict__ y, int ldy, int row0,
                                                                int nrows, TcLevels L, float lsinv) {
  using T = TcTraits<BITS>;
  constexpr int GB = T::GB;
  constexpr int NWARP = TG_THREADS / 32;
  constexpr int GSTEP = SPLIT ? NWARP : 1;  // group stride between the slots of an item
  constexpr int NW = T::BYTES / 4;  // packed words per lane, row and group
  extern __shared__ __align__(16) unsigned char tsm[];
  // [ng][8][NT][32] B fragments, then (4-bit) the level-pair table [256][32].
  uint2* bs = reinterpret_cast<uint2*>(tsm);
  __shared__ float xsc[8], xinv[8];                // row scales (CTA-wide form)
  __shared__ float xsc_w[SPLIT ? 4 : 1][8], xinv_w[SPLIT ? 4 : 1][8];  // per warp (split form)
  const uint32_t la = L.h[0], lb = L.h[1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = lane & 3;
  const int ng = W.groups;
  uint32_t* ptab = reinterpret_cast<uint32_t*>(tsm + (size_t)ng * 8 * NT * 32 * sizeof(uint2));
  const int ntiles = (nrows + 15) >> 4;
  const int wstride = SPLIT ? gridDim.x : gridDim.x * NWARP;
  const int nit = SPLIT ? (ng + GB * NWARP - 1) / (GB * NWARP) : (ng + GB - 1) / GB;  // items per tile
  auto item_g0 = [&](int it) { return SPLIT ? warp + it * GB * NWARP : it * GB; };  // group of slot 0
  __shared__ float red[SPLIT ? NWARP : 1][32][4];

  // Rows g and g + 8 of tile t (null when outside the matrix).
  struct Rows {
    const uint8_t* p[2];
    const __half* n[2];
  };
  auto rows_of = [&](int t, Rows& R) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = t * 16 + (lane >> 2) + 8 * h;
      R.p[h] = nullptr;
      R.n[h] = nullptr;
      if (t < ntiles && r < nrows) {
        int local;
        const int s = find_seg(W, row0 + r, &local);
        R.p[h] = W.seg[s].packed + (size_t)local * W.row_bytes;
        R.n[h] = W.seg[s].norms + (size_t)local * W.groups;
      }
    }
  };
  // This lane's packed words of groups gb + q * GSTEP (q < GB) for both rows,
  // and (lane c < GB) the norms of group gb + c * GSTEP.
  auto load_item = [&](const Rows& R, int gb, uint32_t (&w)[GB][2][NW], float (&nv)[2]) {
#pragma unroll
    for (int q = 0; q < GB; ++q)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int G = gb + q * GSTEP;
        const bool ok = R.p[h] && G < ng;
        const uint8_t* src = ok ? R.p[h] + (size_t)G * (128 * BITS / 8) + c * T::BYTES : nullptr;
        if constexpr (BITS == 2) {
          const uint2 v = ok ? __ldg(reinterpret_cast<const uint2*>(src)) : make_uint2(0u, 0u);
          w[q][h][0] = v.x;
          w[q][h][1] = v.y;
        } else {
          const uint4 v = ok ? __ldg(reinterpret_cast<const uint4*>(src)) : make_uint4(0u, 0u, 0u, 0u);
          w[q][h][0] = v.x;
          w[q][h][1] = v.y;
          w[q][h][2] = v.z;
          w[q][h][3] = v.w;
        }
      }
#pragma unroll
    for (int h = 0; h < 2; ++h)
      nv[h] = (R.p[h] && c < GB && gb + c * GSTEP < ng) ? __half2float(R.n[h][gb + c * GSTEP]) : 0.f;
  };

  // 1. the first work item's weights, before waiting for the activation
  int tile = SPLIT ? blockIdx.x : blockIdx.x * NWARP + warp;
  Rows cur;
  rows_of(tile, cur);
  uint32_t cw[GB][2][NW];
  float cn[2];
  load_item(cur, item_g0(0), cw, cn);
  auto lev = [&](int i) { return (L.h[i >> 1] >> (16 * (i & 1))) & 0xFFFFu; };
  if constexpr (BITS == 4) {
    // Level pair of every packed byte (low nibble = the lower K index), one
    // copy per lane: entry b of lane l at word b * 32 + l, in bank l.
    for (int i = threadIdx.x; i < 256 * 32; i += TG_THREADS) {
      const int b = i >> 5;
      ptab[i] = lev(b & 15) | (lev(b >> 4) << 16);
    }
    if (SPLIT) __syncthreads();  // the split form has no CTA barrier before its tiles
  } else if (!SPLIT) {
    // Level quad of every packed byte (codes in K order as two f16x2), 16
    // copies: entry b of copy c at uint2 b * 16 + c, banks 2c and 2c + 1; the
    // two half-warps of an 8-byte access are served separately, lane l uses
    // copy l % 16.
    uint2* qtab = reinterpret_cast<uint2*>(ptab);
    for (int i = threadIdx.x; i < 256 * 16; i += TG_THREADS) {
      const int b = i >> 4;
      qtab[i] = make_uint2(lev(b & 3) | (lev((b >> 2) & 3) << 16), lev((b >> 4) & 3) | (lev(b >> 6) << 16));
    }
  }
  // 2. the activation rows: power-of-two row scales, then the B fragments
  // (split form: each warp the rows' scales and its own groups' fragments,
  // with no CTA barrier before its first tile)
  pdl_wait();
  float* xscw = SPLIT ? xsc_w[warp] : xsc;
  float* xinvw = SPLIT ? xinv_w[warp] : xinv;
  for (int m = SPLIT ? 0 : warp; m < M; m += SPLIT ? 1 : NWARP) {
    float amax = 0.f;
    for (int k = lane * 4; k < W.in_pad; k += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xh + (size_t)m * ldx + k);
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    amax = warp_max(amax);
    if (lane == 0) {
      int e = 0;
      if (amax > 0.f && isfinite(amax)) {
        frexpf(amax, &e);
        e = 14 - e;
      }
      xscw[m] = ldexpf(1.f, e);
      xinvw[m] = ldexpf(1.f, -e);
    }
  }
  if (SPLIT)
    __syncwarp();
  else
    __syncthreads();
  // Fragment slots (G, nt, lane): the lane's 32-element window of group G for
  // activation row m, loaded as eight independent float4 reads, gives its B
  // fragments of all 8 K steps. The split form fills the slots of its own
  // groups (warp, warp + 4, ...) itself.
  const int nslot = SPLIT ? ((ng - warp + NWARP - 1) / NWARP) * NT * 32 : ng * NT * 32;
  for (int i = SPLIT ? lane : (int)threadIdx.x; i < nslot; i += SPLIT ? 32 : TG_THREADS) {
    const int ln = i & 31, nt = (i >> 5) % NT;
    const int G = SPLIT ? warp + ((i >> 5) / NT) * NWARP : (i >> 5) / NT;
    const int n = ln >> 2, m = nt * 4 + (n >> 1), h = n & 1;
    uint2* dst = bs + (size_t)G * 8 * NT * 32 + nt * 32 + ln;
    if (m >= M) {  // unused column: zero, so every lane loads its fragments unconditionally
#pragma unroll
      for (int j = 0; j < 8; ++j) dst[j * NT * 32] = make_uint2(0u, 0u);
      continue;
    }
    const float4* xr = reinterpret_cast<const float4*>(xh + (size_t)m * ldx + G * 128 + 32 * (ln & 3));
    float xv[32];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 v = xr[k];
      xv[4 * k] = v.x;
      xv[4 * k + 1] = v.y;
      xv[4 * k + 2] = v.z;
      xv[4 * k + 3] = v.w;
    }
    const float sc = xscw[m];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t v0 = f16_part(xv[tc_code_offset(BITS, j, 0, !SPLIT)] * sc, h);
      const uint32_t v1 = f16_part(xv[tc_code_offset(BITS, j, 1, !SPLIT)] * sc, h);
      const uint32_t v2 = f16_part(xv[tc_code_offset(BITS, j, 2, !SPLIT)] * sc, h);
      const uint32_t v3 = f16_part(xv[tc_code_offset(BITS, j, 3, !SPLIT)] * sc, h);
      dst[j * NT * 32] = make_uint2(v0 | (v1 << 16), v2 | (v3 << 16));
    }
  }
  if (SPLIT)
    __syncwarp();
  else
    __syncthreads();
  pdl_trigger();

  // 3. tiles: warp-strided, GB groups per step, the next step's words in flight
  const uint32_t* ptl = ptab + lane;
  const uint2* qtl = reinterpret_cast<const uint2*>(ptab) + (lane & 15);
  float tot[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) tot[nt][0] = tot[nt][1] = 0.f;
  int it = 0;
  while (tile < ntiles) {
    const int gb = item_g0(it);
    int ntile = tile, nitn = it + 1;
    Rows nxt = cur;
    if (nitn >= nit) {
      nitn = 0;
      ntile = tile + wstride;
      rows_of(ntile, nxt);
    }
    uint32_t nw[GB][2][NW];
    float nn[2];
    load_item(nxt, item_g0(nitn), nw, nn);
    float acc[GB][NT][4];
#pragma unroll
    for (int q = 0; q < GB; ++q)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[q][nt][0] = acc[q][nt][1] = acc[q][nt][2] = acc[q][nt][3] = 0.f;
#pragma unroll
    for (int q = 0; q < GB; ++q) {
      if (gb + q * GSTEP >= ng) break;
      const uint2* bg = bs + (size_t)(gb + q * GSTEP) * 8 * NT * 32 + lane;
      if constexpr (BITS == 2) {
        {  // word 0: byte_perm decode, K steps 0..3
          uint32_t va[8], vb[8];
          decode2(cw[q][0][0], la, lb, va);
          decode2(cw[q][1][0], la, lb, vb);
#pragma unroll
          for (int s = 0; s < 4; ++s) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint2 b = bg[(s * NT + nt) * 32];
              mma16816(acc[q][nt], va[2 * s], vb[2 * s], va[2 * s + 1], vb[2 * s + 1], b.x, b.y);
            }
          }
        }
        if constexpr (SPLIT) {  // word 1 by byte_perm too (no table to build: latency first)
          uint32_t va[8], vb[8];
          decode2(cw[q][0][1], la, lb, va);
          decode2(cw[q][1][1], la, lb, vb);
#pragma unroll
          for (int s = 0; s < 4; ++s) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint2 b = bg[((4 + s) * NT + nt) * 32];
              mma16816(acc[q][nt], va[2 * s], vb[2 * s], va[2 * s + 1], vb[2 * s + 1], b.x, b.y);
            }
          }
        } else {
#pragma unroll
          for (int s = 0; s < 4; ++s) {  // word 1: table decode, K steps 4..7
            const uint2 ta = qtl[__byte_perm(cw[q][0][1], 0u, 0x4440u + s) * 16];
            const uint2 tb = qtl[__byte_perm(cw[q][1][1], 0u, 0x4440u + s) * 16];
            const int j = 4 + s;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint2 b = bg[(j * NT + nt) * 32];
              mma16816(acc[q][nt], ta.x, tb.x, ta.y, tb.y, b.x, b.y);
            }
          }
        }
      } else {
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          uint32_t va[4], vb[4];
#pragma unroll
          for (int bt = 0; bt < 4; ++bt) {
            va[bt] = ptl[__byte_perm(cw[q][0][wi], 0u, 0x4440u + bt) * 32];
            vb[bt] = ptl[__byte_perm(cw[q][1][wi], 0u, 0x4440u + bt) * 32];
          }
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const int j = 2 * wi + s;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint2 b = bg[(j * NT + nt) * 32];
              mma16816(acc[q][nt], va[2 * s], vb[2 * s], va[2 * s + 1], vb[2 * s + 1], b.x, b.y);
            }
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < GB; ++q) {
      if (gb + q * GSTEP >= ng) break;
      const float n0 = __shfl_sync(0xffffffffu, cn[0], (lane & ~3) | q);
      const float n1 = __shfl_sync(0xffffffffu, cn[1], (lane & ~3) | q);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        tot[nt][0] += n0 * (acc[q][nt][0] + acc[q][nt][1]);
        tot[nt][1] += n1 * (acc[q][nt][2] + acc[q][nt][3]);
      }
    }
    if (it + 1 == nit) {  // the tile is complete: rows g and g + 8, activation row c (+ 4)
      if constexpr (SPLIT) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          red[warp][lane][2 * nt] = tot[nt][0];
          red[warp][lane][2 * nt + 1] = tot[nt][1];
        }
        __syncthreads();
        if (warp == 0) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            tot[nt][0] = ((red[0][lane][2 * nt] + red[1][lane][2 * nt]) + red[2][lane][2 * nt]) + red[3][lane][2 * nt];
            tot[nt][1] = ((red[0][lane][2 * nt + 1] + red[1][lane][2 * nt + 1]) + red[2][lane][2 * nt + 1]) +
                         red[3][lane][2 * nt + 1];
          }
        }
      }
      if (!SPLIT || warp == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int m = nt * 4 + c;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int r = tile * 16 + (lane >> 2) + 8 * h;
            if (m < M && r < nrows) y[(size_t)m * ldy + r] = (tot[nt][h] * lsinv) * xinvw[m];
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) tot[nt][0] = tot[nt][1] = 0.f;
      if constexpr (SPLIT) __syncthreads();  // red is rewritten for the next tile
    }
    tile = ntile;
    it = nitn;
    cur = nxt;
#pragma unroll
    for (int q = 0; q < GB; ++q)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < NW; ++k) cw[q][h][k] = nw[q][h][k];
    cn[0] = nn[0];
    cn[1] = nn[1];
  }
}

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

// The codebook levels scaled by the power of two that puts max|level| in
// [2^13, 2^14), as f16 bit patterns, and the inverse scale; false when a
// scaled level is not an f16 value (such codebooks take the SIMT kernels).
static bool tc_levels(const CqMat& W, TcLevels* L, float* lsinv) {
  const int n = 1 << W.bits;
  float lmax = 0.f;
  for (int i = 0; i < n; ++i) lmax = std::max(lmax, std::fabs(W.levels[i]));
  if (!std::isfinite(lmax)) return false;
  int le = 0;
  if (lmax > 0.f) {
    int e;
    std::frexp(lmax, &e);
    le = 14 - e;
  }
  *L = TcLevels{};
  for (int i = 0; i < n; ++i) {
    const float v = std::ldexp(W.levels[i], le);
    const __half h = __float2half_rn(v);
    if (__half2float(h) != v) return false;
    L->h[i >> 1] |= (uint32_t)__half_as_ushort(h) << (16 * (i & 1));
  }
  *lsinv = std::ldexp(1.f, -le);
  return true;
}

// Tiles up to which the split-group form is used: a CTA per tile while that
// keeps under about 16 warps per SM.
constexpr int TG_SPLIT_MAX_TILES = 148 * 4;

template <int BITS, int NT>
static cudaError_t launch_gemv_tc(const CqMat& W, const TcLevels& L, float lsinv, const float* xh, int ldx, int M,
                                  float* y, int ldy, int row0, int nrows, cudaStream_t st) {
  // B fragments, then the 4-bit pair table (256 x 32 words) or the 2-bit quad
  // table (256 x 16 uint2): 32 KB either way.
  const size_t smem = (size_t)W.groups * 8 * NT * 32 * sizeof(uint2) + 256 * 32 * 4;
  const int ntiles = (nrows + 15) / 16;
  const bool split = ntiles <= TG_SPLIT_MAX_TILES;
  const int grid = split ? ntiles : std::min((ntiles + TG_THREADS / 32 - 1) / (TG_THREADS / 32), 148 * TG_CTAS_PER_SM);
  auto kern = split ? cq_gemv_tc_kernel<BITS, NT, true> : cq_gemv_tc_kernel<BITS, NT, false>;
  cudaError_t e = allow_smem((const void*)kern, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(TG_THREADS), smem, st, W, xh, ldx, M, y, ldy, row0, nrows, L, lsinv);
}

template <int BITS>
static cudaError_t launch_gemm_simt(const CqMat& W, const float* xh, int ldx, int M, float* y,
                                    int ldy, int row0, int nrows, cudaStream_t st) {
  dim3 grid((nrows + GB_N - 1) / GB_N, (M + GB_M - 1) / GB_M);
  cq_gemm_simt_kernel<BITS><<<grid, 256, 0, st>>>(W, xh, ldx, M, y, ldy, row0, nrows);
  return cudaGetLastError();
}

// gemv_kind (M <= 8 rows): 0 automatic, 1 the SIMT kernels, 2 the
// tensor-core GEMV (f16-exact levels only).
template <int BITS>
static cudaError_t project_bits(const CqMat& W, const float* xh, int ldx, int M, float* y, int ldy,
                                int row0, int nrows, cudaStream_t st, int gemv_kind = 0) {
  // Up to 8 rows on the tensor cores for matrices past the split-group size
  // when the levels are f16 values (the packer writes f16 codebooks): there
  // the tensor-core GEMV streams faster than the SIMT kernels (1.77 against
  // 1.26 TB/s for one row of a 300 MB 2-bit matrix on B200, 2.5x at two to
  // eight rows), while on the model's own matrices (768 to 8192 rows) the
  // latency-ordered SIMT GEMV finishes 0.6 to 6 us sooner. Otherwise the SIMT
  // kernels: large one-row products stream through the table kernel, smaller
  // ones take the latency-ordered GEMV.
  const bool large = (nrows + 15) / 16 > TG_SPLIT_MAX_TILES;
  if (M <= 8 && (gemv_kind == 2 || (gemv_kind == 0 && large))) {
    TcLevels L;
    float lsinv;
    if (tc_levels(W, &L, &lsinv))
      return M <= 4 ? launch_gemv_tc<BITS, 1>(W, L, lsinv, xh, ldx, M, y, ldy, row0, nrows, st)
                    : launch_gemv_tc<BITS, 2>(W, L, lsinv, xh, ldx, M, y, ldy, row0, nrows, st);
    if (gemv_kind == 2) return cudaErrorInvalidValue;
  }
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

bool cq_umma_takes(const CqMat& W, int M, const GemmScratch* gs) {
  return M > 8 && umma_scratch_ok(W, M, W.rows, gs) && umma_supported(W);
}

int cq_launches(const CqMat& W, int M, const GemmScratch* gs, int force_path, bool presplit) {
  if (M <= 0) return 0;
  if (force_path == 3 || (force_path == 0 && cq_umma_takes(W, M, gs)))
    return presplit && W.lvl_hi ? 1 : 2;  // (operand preparation +) tensor-core GEMM
  return 1;
}

cudaError_t cq_project(const CqMat& W, const float* xh, int ldx, int M, float* y, int ldy, int row0,
                       int nrows, cudaStream_t st, int force_path, const GemmScratch* gs, bool presplit) {
  if (M <= 0 || nrows <= 0) return cudaSuccess;
  if (!cq_args_ok(W, xh, ldx) || row0 < 0 || row0 + nrows > W.rows) return cudaErrorInvalidValue;
  if ((force_path == 1 || force_path >= 4) && M > 8) return cudaErrorInvalidValue;
  if (force_path < 0 || force_path > 5) return cudaErrorInvalidValue;
  if (force_path >= 4 && gs && gs->amax) return cudaErrorInvalidValue;
  if (force_path >= 4)  // one GEMV kernel by name: 4 the SIMT kernels, 5 the tensor-core GEMV
    return W.bits == 2 ? project_bits<2>(W, xh, ldx, M, y, ldy, row0, nrows, st, force_path - 3)
                       : project_bits<4>(W, xh, ldx, M, y, ldy, row0, nrows, st, force_path - 3);
  const bool scratch_ok = umma_scratch_ok(W, M, nrows, gs);
  if (force_path == 3) {
    if (!scratch_ok) return cudaErrorInvalidValue;
    return cq_project_umma(W, xh, ldx, M, y, ldy, row0, nrows, st, *gs, presplit);
  }
  if (force_path == 0 && M > 8 && scratch_ok && umma_supported(W))
    return cq_project_umma(W, xh, ldx, M, y, ldy, row0, nrows, st, *gs, presplit);
  // The input exists only in the split form, or the caller wants the greedy
  // pick, which only the tensor-core path computes.
  if (presplit || (gs && gs->amax)) return cudaErrorInvalidValue;
  if (force_path == 2)
    return W.bits == 2 ? launch_gemm_simt<2>(W, xh, ldx, M, y, ldy, row0, nrows, st)
                       : launch_gemm_simt<4>(W, xh, ldx, M, y, ldy, row0, nrows, st);
  return W.bits == 2 ? project_bits<2>(W, xh, ldx, M, y, ldy, row0, nrows, st)
                     : project_bits<4>(W, xh, ldx, M, y, ldy, row0, nrows, st);
}

}  // namespace nb
