// Block tail of a Needle-3 layer with the HadamardMLP on the tensor cores.
//
// model.rs:309-356: post_norm + gated residual, pre_hada norm, the
// HadamardMLP (v3/kernels.rs:119-180), MLP residual, y = block - u and
// scatter_up (mhc.rs:109-158) back into the lanes. One warp per activation row.
//
// Each Kronecker apply out = A^T Z B (kernels.rs:41-78; Z is the 1024-vector
// as a D x D matrix, D = 32 on the shipped geometry) runs as two D x D x D
// products on mma.sync m16n8k16 (f16 in, f32 accumulate):
//   stage 1   T^T[l][i] = sum_j B[j][l] Z[i][j]     (A operand B^T, B operand Z^T)
//   stage 2   out[k][l] = sum_i A[i][k] T[i][l]     (A operand A^T, B operand T)
// Computing stage 1 transposed makes its accumulator fragments exactly the B
// fragments of stage 2, so T never leaves registers. Every operand is split
// into an f16 high part and remainder (x_hi*w_hi + x_hi*w_lo + x_lo*w_hi) after
// a power-of-two scale that keeps the remainders normal; each accumulator sums
// only K = D products over 3 * D/16 MMAs, so the tensor cores' truncating
// accumulation stays at f32 rounding level. The weight fragments (high part
// and remainder, in mma lane order) are built once at load time.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "kernels.hpp"
#include "launch_util.hpp"

namespace nb {

namespace {

constexpr float EPS = 1e-6f;  // kernels.rs:11, norm.rs:6

__host__ __device__ inline int pow2_exp(float amax) {
  // Power of two that brings max|v| into [2^13, 2^14) (0 for an all-zero input).
  if (!(amax > 0.f) || !std::isfinite(amax)) return 0;
  int e;
  std::frexp(amax, &e);
  return 14 - e;
}

__device__ __forceinline__ uint32_t split_h2(float x, float y, uint32_t* lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const __half2 l = __floats2half2_rn(x - __low2float(h), y - __high2float(h));
  *lo = *reinterpret_cast<const uint32_t*>(&l);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Padded D x (D + 4) storage of a D x D matrix: element c = r * D + s at
// r * (D + 4) + s, so fragment loads of consecutive rows hit distinct banks.
template <int D>
__device__ __forceinline__ int pad_idx(int c) {
  return (c / D) * (D + 4) + c % D;
}

// One Kronecker apply for this warp. zb: the input, each element packed as
// (f16 high part | f16 remainder << 16) in padded layout, the true value being
// the stored one times invz. fb receives the f32 output in padded layout.
// fB / fA: weight fragments of B^T and A^T (true weight = fragment * inv).
template <int D>
__device__ void kron_tc(const uint32_t* __restrict__ fB, float invB, const uint32_t* __restrict__ fA,
                        float invA, const uint32_t* zb, float invz, float* fb) {
  constexpr int MT = D / 16, NT = D / 8, KS = D / 16, P = D + 4;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float c1[MT][NT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n) c1[m][n][0] = c1[m][n][1] = c1[m][n][2] = c1[m][n][3] = 0.f;
  // ---- stage 1: T^T[l][i] = sum_j Bt[l][j] Z^T[j][i]
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const uint32_t* zr = zb + (8 * n + g) * P + 16 * ks + 2 * t;
      const uint2 e01 = *reinterpret_cast<const uint2*>(zr);
      const uint2 e89 = *reinterpret_cast<const uint2*>(zr + 8);
      bh[n][0] = __byte_perm(e01.x, e01.y, 0x5410);
      bl[n][0] = __byte_perm(e01.x, e01.y, 0x7632);
      bh[n][1] = __byte_perm(e89.x, e89.y, 0x5410);
      bl[n][1] = __byte_perm(e89.x, e89.y, 0x7632);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint4* fr = reinterpret_cast<const uint4*>(fB + ((m * KS + ks) * 32 + lane) * 8);
      const uint4 h4 = __ldg(fr), l4 = __ldg(fr + 1);
      const uint32_t ah[4] = {h4.x, h4.y, h4.z, h4.w}, al[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
      for (int n = 0; n < NT; ++n) mma16816(c1[m][n], ah, bh[n][0], bh[n][1]);
#pragma unroll
      for (int n = 0; n < NT; ++n) mma16816(c1[m][n], ah, bl[n][0], bl[n][1]);
#pragma unroll
      for (int n = 0; n < NT; ++n) mma16816(c1[m][n], al, bh[n][0], bh[n][1]);
    }
  }
  // ---- rescale T for the f16 split of stage 2
  float amax = 0.f;
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) amax = fmaxf(amax, fabsf(c1[m][n][e]));
  amax = warp_max(amax);
  const int et = pow2_exp(amax);
  const float st = ldexpf(1.f, et);
  // ---- stage 2: out[k][l] = sum_i At[k][i] T[i][l]; B (i, l) = c1 tile (l/16, i/8)
  float c2[MT][NT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n) c2[m][n][0] = c2[m][n][1] = c2[m][n][2] = c2[m][n][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int m1 = n >> 1, h = (n & 1) * 2;  // rows l = 8n + g of c1 m-tile n/2
      bh[n][0] = split_h2(c1[m1][2 * ks][h] * st, c1[m1][2 * ks][h + 1] * st, &bl[n][0]);
      bh[n][1] = split_h2(c1[m1][2 * ks + 1][h] * st, c1[m1][2 * ks + 1][h + 1] * st, &bl[n][1]);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint4* fr = reinterpret_cast<const uint4*>(fA + ((m * KS + ks) * 32 + lane) * 8);
      const uint4 h4 = __ldg(fr), l4 = __ldg(fr + 1);
      const uint32_t ah[4] = {h4.x, h4.y, h4.z, h4.w}, al[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
      for (int n = 0; n < NT; ++n) mma16816(c2[m][n], ah, bh[n][0], bh[n][1]);
#pragma unroll
      for (int n = 0; n < NT; ++n) mma16816(c2[m][n], ah, bl[n][0], bl[n][1]);
#pragma unroll
      for (int n = 0; n < NT; ++n) mma16816(c2[m][n], al, bh[n][0], bh[n][1]);
    }
  }
  const float inv = invz * invB * ldexpf(1.f, -et) * invA;
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int k = 16 * m + g, l = 8 * n + 2 * t;
      *reinterpret_cast<float2*>(fb + k * P + l) = make_float2(c2[m][n][0] * inv, c2[m][n][1] * inv);
      *reinterpret_cast<float2*>(fb + (k + 8) * P + l) = make_float2(c2[m][n][2] * inv, c2[m][n][3] * inv);
    }
  __syncwarp();
}

// Converts this warp's row, held as f32 in zb (padded layout), to packed
// f16 high part | remainder with the power-of-two scale of `amax`; returns the
// inverse scale.
template <int D>
__device__ __forceinline__ float pack_row(uint32_t* zb, float amax) {
  constexpr int N = D * D;
  const int lane = threadIdx.x & 31;
  const int e = pow2_exp(amax);
  const float s = ldexpf(1.f, e);
  for (int c = lane; c < N; c += 32) {
    const int pi = pad_idx<D>(c);
    const float x = __uint_as_float(zb[pi]) * s;
    const __half h = __float2half_rn(x);
    const __half l = __float2half_rn(x - __half2float(h));
    zb[pi] = (uint32_t)__half_as_ushort(h) | ((uint32_t)__half_as_ushort(l) << 16);
  }
  __syncwarp();
  return ldexpf(1.f, -e);
}

// PW rows per CTA and NW warps: one warp per row (NW = PW: 8, 7, or 2 for
// mid-size batches, four times the CTAs so the SMs fill), or one row over
// eight warps (PW = 1, NW = 8: batch-1 and small batches, where each
// Kronecker product is spread over the warps).
template <int D, int PW, int NW>
struct __align__(16) PostSmem {
  static constexpr int P = D + 4;
  static constexpr bool PAR = PW == 1 && NW > 1;
  uint32_t zb[PW][D * P];  // Kronecker input (f32 while built, then f16 hi|lo)
  float fb[PW][D * P];     // Kronecker output
  float pr[PW][8];         // conditioning weights per row
  float part[NW][PW][8];   // per-warp partial sums: [warp][row][j]
  float amax[NW][PW];      // per-warp partial maxima: [warp][row]
  float inv2[PW];
  float gs[PW][24];        // gates per row: hpost [nl], hres [nl * nl]
  alignas(16) float tt[PAR ? D * (D + 8) : 1];  // one row over the warps: the intermediate T^T [D][D + 8]
  float wmax[NW];
};

// One halving step of a many-value warp sum: lanes with bit `o` set keep the
// upper H values of v[0 .. 2H), the others the lower H, each adding its
// partner's copy of the half it keeps.
template <int C, int H>
__device__ __forceinline__ void halve_sum(float (&v)[C], int lane, int o) {
  const bool up = (lane & o) != 0;
#pragma unroll
  for (int k = 0; k < H; ++k) {
    const float send = up ? v[k] : v[k + H];
    const float keep = up ? v[k + H] : v[k];
    v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
  }
}

// Warp sums of C = 64 or 16 values per lane by recursive halving (62 or 31
// shuffles instead of 5 per value). Afterwards lane l holds the sums of values
// 2l and 2l + 1 in v[0], v[1] (C = 64), or of value l / 2 in v[0] (C = 16).
template <int C>
__device__ __forceinline__ void warp_sum_many(float (&v)[C], int lane) {
  static_assert(C == 64 || C == 16, "64 or 16 values");
  if constexpr (C == 64) {
    halve_sum<64, 32>(v, lane, 16);
    halve_sum<64, 16>(v, lane, 8);
    halve_sum<64, 8>(v, lane, 4);
    halve_sum<64, 4>(v, lane, 2);
    halve_sum<64, 2>(v, lane, 1);
  } else {
    halve_sum<16, 8>(v, lane, 16);
    halve_sum<16, 4>(v, lane, 8);
    halve_sum<16, 2>(v, lane, 4);
    halve_sum<16, 1>(v, lane, 2);
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  }
}

// Block max over the NW warps of per-row partials red[warp][row].
template <int NW, int PW>
__device__ __forceinline__ float rows_max(float (*red)[PW], int row) {
  float m = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) m = fmaxf(m, red[w][row]);
  return m;
}

// pack_row for one row by every thread of the CTA (NW warps); returns the
// inverse scale. Contains __syncthreads.
template <int D, int NW>
__device__ __forceinline__ float pack_row_par(uint32_t* zb, float amax) {
  constexpr int N = D * D;
  const int e = pow2_exp(amax);
  const float s = ldexpf(1.f, e);
  for (int c = threadIdx.x; c < N; c += NW * 32) {
    const int pi = pad_idx<D>(c);
    const float x = __uint_as_float(zb[pi]) * s;
    const __half h = __float2half_rn(x);
    const __half l = __float2half_rn(x - __half2float(h));
    zb[pi] = (uint32_t)__half_as_ushort(h) | ((uint32_t)__half_as_ushort(l) << 16);
  }
  __syncthreads();
  return ldexpf(1.f, -e);
}

// Read-only weight loads: through the non-coherent cache from global memory,
// or plain loads when the weights were staged in shared memory (SM).
template <bool SM, typename T>
__device__ __forceinline__ T ldw(const T* p) {
  if constexpr (SM)
    return *p;
  else
    return __ldg(p);
}

// Shared-memory copies of one layer's tail parameters, staged by the one-row
// CTA before it waits for the previous kernel (none of them is written by a
// kernel), so that no phase after the first waits on an L2 round trip for a
// weight. Offsets in floats from `base`; d and N are multiples of 4.
struct PostStage {
  int post_norm, pre_hada, d1, d4, cond_v, cond_u, d2, b2, d3, p1, p2, hfrag, u, lanes, total;
  __host__ __device__ PostStage(int d, int N, int rk, int nl, int fr6) {
    int o = 0;
    post_norm = o; o += d;
    pre_hada = o; o += d;
    d1 = o; o += d;
    d4 = o; o += d;
    cond_v = o; o += d * rk;
    cond_u = o; o += rk * N;
    d2 = o; o += N;
    b2 = o; o += N;
    d3 = o; o += N;
    p1 = o; o += N;
    p2 = o; o += N;
    hfrag = o; o += fr6;
    u = o; o += d;
    lanes = o; o += nl * d;
    total = o;
  }
};

// cp.async of `floats` floats (a multiple of 4; both addresses 16-byte
// aligned) by every thread of the CTA.
__device__ __forceinline__ void stage_copy(float* dst, const void* src, int floats) {
  for (int i = 4 * threadIdx.x; i < floats; i += 4 * blockDim.x)
    cp_async16(dst + i, reinterpret_cast<const float*>(src) + i, true);
}

// kron_tc for one row by NW warps: warp w computes tiles w, w + NW, ... of
// both stages (D / 16 x D / 8 tiles of 16 x 8), with T^T exchanged through
// shared memory (tt [D][D + 8], 16-byte aligned; its float2 accesses are free
// of bank conflicts) and its maximum through wmax [NW]. The tiles, their K
// order and the scale are those of kron_tc, so the output is the same.
// Contains __syncthreads: every thread of the CTA calls it.
template <int D, int NW>
__device__ void kron_tc_par(const uint32_t* __restrict__ fB, float invB, const uint32_t* __restrict__ fA,
                            float invA, const uint32_t* zb, float invz, float* fb, float* tt, float* wmax) {
  constexpr int MT = D / 16, NT = D / 8, KS = D / 16, P = D + 4, TP = D + 8;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, w = threadIdx.x >> 5;
  float amax = 0.f;
  for (int q = w; q < MT * NT; q += NW) {  // stage 1: T^T[l][i] = sum_j Bt[l][j] Z^T[j][i]
    const int m = q / NT, n = q % NT;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const uint32_t* zr = zb + (8 * n + g) * P + 16 * ks + 2 * t;
      const uint2 e01 = *reinterpret_cast<const uint2*>(zr);
      const uint2 e89 = *reinterpret_cast<const uint2*>(zr + 8);
      const uint32_t bh0 = __byte_perm(e01.x, e01.y, 0x5410), bl0 = __byte_perm(e01.x, e01.y, 0x7632);
      const uint32_t bh1 = __byte_perm(e89.x, e89.y, 0x5410), bl1 = __byte_perm(e89.x, e89.y, 0x7632);
      const uint4* fr = reinterpret_cast<const uint4*>(fB + ((m * KS + ks) * 32 + lane) * 8);
      const uint4 h4 = fr[0], l4 = fr[1];
      const uint32_t ah[4] = {h4.x, h4.y, h4.z, h4.w}, al[4] = {l4.x, l4.y, l4.z, l4.w};
      mma16816(c, ah, bh0, bh1);
      mma16816(c, ah, bl0, bl1);
      mma16816(c, al, bh0, bh1);
    }
    const int l = 16 * m + g, i = 8 * n + 2 * t;
    *reinterpret_cast<float2*>(tt + l * TP + i) = make_float2(c[0], c[1]);
    *reinterpret_cast<float2*>(tt + (l + 8) * TP + i) = make_float2(c[2], c[3]);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(c[0]), fabsf(c[1])), fmaxf(fabsf(c[2]), fabsf(c[3]))));
  }
  amax = warp_max(amax);
  if (lane == 0) wmax[w] = amax;
  __syncthreads();
  float am = 0.f;
#pragma unroll
  for (int ww = 0; ww < NW; ++ww) am = fmaxf(am, wmax[ww]);
  const int et = pow2_exp(am);
  const float st = ldexpf(1.f, et);
  const float inv = invz * invB * ldexpf(1.f, -et) * invA;
  for (int q = w; q < MT * NT; q += NW) {  // stage 2: out[k][l] = sum_i At[k][i] T[i][l]
    const int m = q / NT, n = q % NT;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const float* tr = tt + (8 * n + g) * TP + 16 * ks + 2 * t;  // B (i, l) = T^T[l][i]
      const float2 t01 = *reinterpret_cast<const float2*>(tr), t89 = *reinterpret_cast<const float2*>(tr + 8);
      uint32_t bl0, bl1;
      const uint32_t bh0 = split_h2(t01.x * st, t01.y * st, &bl0);
      const uint32_t bh1 = split_h2(t89.x * st, t89.y * st, &bl1);
      const uint4* fr = reinterpret_cast<const uint4*>(fA + ((m * KS + ks) * 32 + lane) * 8);
      const uint4 h4 = fr[0], l4 = fr[1];
      const uint32_t ah[4] = {h4.x, h4.y, h4.z, h4.w}, al[4] = {l4.x, l4.y, l4.z, l4.w};
      mma16816(c, ah, bh0, bh1);
      mma16816(c, ah, bl0, bl1);
      mma16816(c, al, bh0, bh1);
    }
    const int k = 16 * m + g, l = 8 * n + 2 * t;
    *reinterpret_cast<float2*>(fb + k * P + l) = make_float2(c[0] * inv, c[1] * inv);
    *reinterpret_cast<float2*>(fb + (k + 8) * P + l) = make_float2(c[2] * inv, c[3] * inv);
  }
  __syncthreads();
}

// The CTA owns PW consecutive rows. Phases alternate between element-parallel
// work (thread tid covers elements tid, tid + PT, ... of every row, so each
// parameter element is loaded once per PW rows) and one Kronecker apply per
// warp on its own row.
template <int D, int PW, int NW>
__global__ void __launch_bounds__(NW * 32) layer_post_tc_kernel(Geo G, RowBatch rb, LayerParams lp,
                                                           const uint32_t* __restrict__ p1,
                                                           const uint32_t* __restrict__ p2,
                                                           const float* __restrict__ projo,
                                                           const float* __restrict__ u,
                                                           const float* __restrict__ bx_in,
                                                           const float* __restrict__ gates,
                                                           float* __restrict__ lanes) {
  constexpr int N = D * D;
  constexpr int PT = NW * 32;  // threads
  constexpr bool PAR = PostSmem<D, PW, NW>::PAR;
  extern __shared__ __align__(16) unsigned char post_smem[];
  auto& S = *reinterpret_cast<PostSmem<D, PW, NW>*>(post_smem);
  float* s1all = reinterpret_cast<float*>(post_smem + sizeof(PostSmem<D, PW, NW>));  // [PW][d]
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int r0 = blockIdx.x * PW;
  const int nrow = min(PW, rb.M - r0);
  const int d = G.d, nl = G.lanes, rk = G.cond_rank;
  constexpr int FR = (D / 16) * (D / 16) * 32 * 8;  // u32 per weight fragment block
  // Weight sources: global memory, or (one row over the warps) shared-memory
  // copies staged here, before the wait for the previous kernel; the row's u
  // and lanes follow right after the wait. WSRC picks the source at each use,
  // so the many-row variants keep reading the parameters in place.
  const PostStage so(d, N, rk, nl, 6 * FR);
  float* const stb = s1all + d;  // one row over the warps: the staged copies
#define WSRC(T, name) (PAR ? reinterpret_cast<const T*>(stb + so.name) : (const T*)(lp.name))
  if constexpr (PAR) {
    stage_copy(stb + so.post_norm, lp.post_norm, d);
    stage_copy(stb + so.pre_hada, lp.pre_hada, d);
    stage_copy(stb + so.d1, lp.d1, d);
    stage_copy(stb + so.d4, lp.d4, d);
    stage_copy(stb + so.cond_v, lp.cond_v, d * rk);
    stage_copy(stb + so.cond_u, lp.cond_u, rk * N);
    stage_copy(stb + so.d2, lp.d2, N);
    stage_copy(stb + so.b2, lp.b2, N);
    stage_copy(stb + so.d3, lp.d3, N);
    stage_copy(stb + so.p1, p1, N);
    stage_copy(stb + so.p2, p2, N);
    stage_copy(stb + so.hfrag, lp.hfrag, 6 * FR);
    cp_commit();
  }

  // The final phase re-reads this CTA's rows of u and of the lanes, which the
  // attention's KV stream has usually pushed out of L2: start bringing them
  // back now (a hint; nothing waits on it).
  if (tid == 0) {
    const unsigned ub = (unsigned)(nrow * d * 4), lb = (unsigned)(nrow * nl * d * 4);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(u + (size_t)r0 * d), "r"(ub) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lanes + (size_t)r0 * nl * d), "r"(lb) : "memory");
  }
  pdl_wait();  // everything below reads or writes what earlier kernels touch
  pdl_trigger();
  if constexpr (PAR) {
    stage_copy(stb + so.u, u + (size_t)r0 * d, d);
    stage_copy(stb + so.lanes, lanes + (size_t)r0 * nl * d, nl * d);
    cp_commit();
    cp_wait<1>();  // the weights
    __syncthreads();
  }
  // Gates of the CTA's rows: hpost [nl], hres [nl * nl] (written by layer_pre).
  if (tid < PW * 24) S.gs[tid / 24][tid % 24] = (tid / 24 < nrow) ? gates[(size_t)(r0 + tid / 24) * 24 + tid % 24] : 0.f;
  // ---- per row (warp w, or every warp on the one row): post_norm + gated
  // residual (model.rs:309-316), s1 and its rms
  if constexpr (PAR) {
    const float4* po = reinterpret_cast<const float4*>(projo + (size_t)r0 * d);
    const float4* bx = reinterpret_cast<const float4*>(bx_in + (size_t)r0 * d);
    const float4* pn = reinterpret_cast<const float4*>(WSRC(float, post_norm));
    float4* s1 = reinterpret_cast<float4*>(s1all);
    const int d4 = d / 4;
    float ss = 0.f;
    for (int c = tid; c < d4; c += PT) {
      const float4 v = po[c];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = block_sum(ss, S.tt);  // tt is free until the first Kronecker product
    const float inv = 1.0f / sqrtf(ss / (float)d + EPS);
    const float ag = sigmoidf_(lp.attn_gate);
    float s2 = 0.f;
    for (int c = tid; c < d4; c += PT) {
      const float4 p = po[c], x = bx[c], q = pn[c];
      const float4 v = make_float4(x.x + ag * ((1.0f + q.x) * p.x * inv), x.y + ag * ((1.0f + q.y) * p.y * inv),
                                   x.z + ag * ((1.0f + q.z) * p.z * inv), x.w + ag * ((1.0f + q.w) * p.w * inv));
      s1[c] = v;
      s2 += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    s2 = block_sum(s2, S.tt);
    if (tid == 0) S.inv2[0] = 1.0f / sqrtf(s2 / (float)d + EPS);
  } else if (w < nrow) {
    const int r = r0 + w;
    const float4* po = reinterpret_cast<const float4*>(projo + (size_t)r * d);
    const float4* bx = reinterpret_cast<const float4*>(bx_in + (size_t)r * d);
    const float4* pn = reinterpret_cast<const float4*>(lp.post_norm);
    float4* s1 = reinterpret_cast<float4*>(s1all + (size_t)w * d);
    const int d4 = d / 4;
    float ss = 0.f;
#pragma unroll 2
    for (int c = lane; c < d4; c += 32) {
      const float4 v = po[c];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)d + EPS);
    const float ag = sigmoidf_(lp.attn_gate);
    float s2 = 0.f;
#pragma unroll 2
    for (int c = lane; c < d4; c += 32) {
      const float4 p = po[c], x = bx[c], q = pn[c];
      const float4 v = make_float4(x.x + ag * ((1.0f + q.x) * p.x * inv), x.y + ag * ((1.0f + q.y) * p.y * inv),
                                   x.z + ag * ((1.0f + q.z) * p.z * inv), x.w + ag * ((1.0f + q.w) * p.w * inv));
      s1[c] = v;
      s2 += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    s2 = warp_sum(s2);
    if (lane == 0) S.inv2[w] = 1.0f / sqrtf(s2 / (float)d + EPS);
  }
  __syncthreads();
  // ---- element-parallel, four elements per thread: t = pre_hada norm,
  // z = t * d1, logits t . cond_v
  {
    float acc[PW][8], mz[PW];
#pragma unroll
    for (int i = 0; i < PW; ++i) {
      mz[i] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    }
    for (int c0 = 4 * tid; c0 < N; c0 += 4 * PT) {
      const int pi = pad_idx<D>(c0);  // c0..c0+3 stay in one padded row
      if (c0 < d) {
        const float4 ph4 = *reinterpret_cast<const float4*>(WSRC(float, pre_hada) + c0);
        const float4 d14 = *reinterpret_cast<const float4*>(WSRC(float, d1) + c0);
        const float ph[4] = {1.0f + ph4.x, 1.0f + ph4.y, 1.0f + ph4.z, 1.0f + ph4.w};
        const float dd[4] = {d14.x, d14.y, d14.z, d14.w};
        // cond_v rows c0..c0+3 ([d][rk] row-major): 4 * rk consecutive floats.
        float cv[4][8];
        if (rk == 8) {
          const float4* cv4 = reinterpret_cast<const float4*>(WSRC(float, cond_v) + (size_t)c0 * 8);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 a = ldw<PAR>(cv4 + 2 * e), b = ldw<PAR>(cv4 + 2 * e + 1);
            cv[e][0] = a.x, cv[e][1] = a.y, cv[e][2] = a.z, cv[e][3] = a.w;
            cv[e][4] = b.x, cv[e][5] = b.y, cv[e][6] = b.z, cv[e][7] = b.w;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int j = 0; j < 8; ++j) cv[e][j] = j < rk ? WSRC(float, cond_v)[(c0 + e) * rk + j] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < PW; ++i) {
          if (i >= nrow) break;
          const float4 sv = *reinterpret_cast<const float4*>(s1all + i * d + c0);
          const float s1v[4] = {sv.x, sv.y, sv.z, sv.w};
          float z[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float tc = ph[e] * s1v[e] * S.inv2[i];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i][j] += tc * cv[e][j];
            z[e] = tc * dd[e];
            mz[i] = fmaxf(mz[i], fabsf(z[e]));
          }
          *reinterpret_cast<uint4*>(&S.zb[i][pi]) =
              make_uint4(__float_as_uint(z[0]), __float_as_uint(z[1]), __float_as_uint(z[2]), __float_as_uint(z[3]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < PW; ++i) *reinterpret_cast<uint4*>(&S.zb[i][pi]) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int i = 0; i < PW; ++i) {
      if (i >= nrow) break;  // rows past the batch are never read
      const float m = warp_max(mz[i]);
      if (lane == 0) S.amax[w][i] = m;
    }
    // Conditioning logits: all PW x 8 partial sums of the warp at once (ranks
    // past rk and rows past the batch hold zeros).
    constexpr int NS = PW * 8 <= 16 ? 16 : 64;  // padded with zeros
    float sums[NS];
#pragma unroll
    for (int k = 0; k < NS; ++k) sums[k] = k < PW * 8 ? acc[k / 8 < PW ? k / 8 : 0][k % 8] : 0.f;
    warp_sum_many<NS>(sums, lane);
    if constexpr (NS == 64) {
      if ((lane >> 2) < PW) {
        S.part[w][lane >> 2][(2 * lane) & 7] = sums[0];
        S.part[w][lane >> 2][((2 * lane) & 7) + 1] = sums[1];
      }
    } else {
      if ((lane & 1) == 0 && (lane >> 4) < PW) S.part[w][lane >> 4][(lane >> 1) & 7] = sums[0];
    }
  }
  __syncthreads();
  // conditioning softmax per row (one lane per row)
  if (tid < nrow) {
    float lg[8], mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = 0.f;
#pragma unroll
      for (int ww = 0; ww < NW; ++ww) v += S.part[ww][tid][j];
      lg[j] = v;
      if (j < rk) mx = fmaxf(mx, v);
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < rk) {
        lg[j] = expf(lg[j] - mx);
        sum += lg[j];
      }
#pragma unroll
    for (int j = 0; j < 8; ++j) S.pr[tid][j] = j < rk ? lg[j] / sum : 0.f;
  }
  // ---- Kronecker 1 (warp per row, or every warp on the one row)
  if constexpr (PAR) {
    const float iz = pack_row_par<D, NW>(S.zb[0], rows_max<NW, PW>(S.amax, 0));
    kron_tc_par<D, NW>(WSRC(uint32_t, hfrag), lp.hinv[0], WSRC(uint32_t, hfrag) + FR, lp.hinv[1], S.zb[0], iz, S.fb[0], S.tt, S.wmax);
  } else if (w < nrow) {
    const float iz = pack_row<D>(S.zb[w], rows_max<NW, PW>(S.amax, w));
    kron_tc<D>(WSRC(uint32_t, hfrag), lp.hinv[0], WSRC(uint32_t, hfrag) + FR, lp.hinv[1], S.zb[w], iz, S.fb[w]);
  }
  __syncthreads();
  // ---- element-parallel: silu(d2 * cond * out[p1] + b2), cond = 1 + pr . cond_u
  // (kernels.rs:146-160; a conditioning rank whose weight is exactly zero is
  // skipped, as the reference skips it). A row's weights and their nonzero
  // mask are read once per row; silu(v) = v / (1 + e^-v) with the hardware
  // exponential and division (~2 ulp each).
  {
    float mz[PW];
#pragma unroll
    for (int i = 0; i < PW; ++i) mz[i] = 0.f;
    for (int c0 = 4 * tid; c0 < N; c0 += 4 * PT) {
      float cu[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 t =
            j < rk ? ldw<PAR>(reinterpret_cast<const float4*>(WSRC(float, cond_u) + j * N + c0)) : make_float4(0, 0, 0, 0);
        cu[j][0] = t.x;
        cu[j][1] = t.y;
        cu[j][2] = t.z;
        cu[j][3] = t.w;
      }
      const float4 d24 = ldw<PAR>(reinterpret_cast<const float4*>(WSRC(float, d2) + c0));
      const float4 b24 = ldw<PAR>(reinterpret_cast<const float4*>(WSRC(float, b2) + c0));
      const uint4 pp = ldw<PAR>(reinterpret_cast<const uint4*>((PAR ? reinterpret_cast<const uint32_t*>(stb + so.p1) : p1) + c0));
      const float d2[4] = {d24.x, d24.y, d24.z, d24.w}, b2[4] = {b24.x, b24.y, b24.z, b24.w};
      const int src[4] = {pad_idx<D>(pp.x), pad_idx<D>(pp.y), pad_idx<D>(pp.z), pad_idx<D>(pp.w)};
      const int pi = pad_idx<D>(c0);
#pragma unroll
      for (int i = 0; i < PW; ++i) {
        if (i >= nrow) break;
        float pr[8];
        unsigned nz = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          pr[j] = S.pr[i][j];
          nz |= (j < rk && pr[j] != 0.0f) ? 1u << j : 0u;
        }
        float cv[4] = {1.0f, 1.0f, 1.0f, 1.0f};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (nz & (1u << j)) {  // the same for every thread of the CTA
#pragma unroll
            for (int e = 0; e < 4; ++e) cv[e] += pr[j] * cu[j][e];
          }
        }
        float z[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float v = d2[e] * cv[e] * S.fb[i][src[e]] + b2[e];
          z[e] = __fdividef(v, 1.0f + __expf(-v));  // silu, ops.rs:118
          mz[i] = fmaxf(mz[i], fabsf(z[e]));
        }
        *reinterpret_cast<uint4*>(&S.zb[i][pi]) =
            make_uint4(__float_as_uint(z[0]), __float_as_uint(z[1]), __float_as_uint(z[2]), __float_as_uint(z[3]));
      }
    }
#pragma unroll
    for (int i = 0; i < PW; ++i) {
      if (i >= nrow) break;
      const float m = warp_max(mz[i]);
      if (lane == 0) S.amax[w][i] = m;
    }
  }
  __syncthreads();
  // ---- Kronecker 2
  if constexpr (PAR) {
    const float iz = pack_row_par<D, NW>(S.zb[0], rows_max<NW, PW>(S.amax, 0));
    kron_tc_par<D, NW>(WSRC(uint32_t, hfrag) + 2 * FR, lp.hinv[2], WSRC(uint32_t, hfrag) + 3 * FR, lp.hinv[3], S.zb[0], iz, S.fb[0], S.tt,
                       S.wmax);
  } else if (w < nrow) {
    const float iz = pack_row<D>(S.zb[w], rows_max<NW, PW>(S.amax, w));
    kron_tc<D>(WSRC(uint32_t, hfrag) + 2 * FR, lp.hinv[2], WSRC(uint32_t, hfrag) + 3 * FR, lp.hinv[3], S.zb[w], iz, S.fb[w]);
  }
  __syncthreads();
  // ---- element-parallel: out[p2] * d3
  {
    float mz[PW];
#pragma unroll
    for (int i = 0; i < PW; ++i) mz[i] = 0.f;
    for (int c0 = 4 * tid; c0 < N; c0 += 4 * PT) {
      const float4 d34 = *reinterpret_cast<const float4*>(WSRC(float, d3) + c0);
      const uint4 pp = *reinterpret_cast<const uint4*>((PAR ? reinterpret_cast<const uint32_t*>(stb + so.p2) : p2) + c0);
      const float d3[4] = {d34.x, d34.y, d34.z, d34.w};
      const int src[4] = {pad_idx<D>(pp.x), pad_idx<D>(pp.y), pad_idx<D>(pp.z), pad_idx<D>(pp.w)};
      const int pi = pad_idx<D>(c0);
#pragma unroll
      for (int i = 0; i < PW; ++i) {
        if (i >= nrow) break;
        float z[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          z[e] = S.fb[i][src[e]] * d3[e];
          mz[i] = fmaxf(mz[i], fabsf(z[e]));
        }
        *reinterpret_cast<uint4*>(&S.zb[i][pi]) =
            make_uint4(__float_as_uint(z[0]), __float_as_uint(z[1]), __float_as_uint(z[2]), __float_as_uint(z[3]));
      }
    }
#pragma unroll
    for (int i = 0; i < PW; ++i) {
      if (i >= nrow) break;
      const float m = warp_max(mz[i]);
      if (lane == 0) S.amax[w][i] = m;
    }
  }
  __syncthreads();
  // ---- Kronecker 3
  if constexpr (PAR) {
    const float iz = pack_row_par<D, NW>(S.zb[0], rows_max<NW, PW>(S.amax, 0));
    kron_tc_par<D, NW>(WSRC(uint32_t, hfrag) + 4 * FR, lp.hinv[4], WSRC(uint32_t, hfrag) + 5 * FR, lp.hinv[5], S.zb[0], iz, S.fb[0], S.tt,
                       S.wmax);
  } else if (w < nrow) {
    const float iz = pack_row<D>(S.zb[w], rows_max<NW, PW>(S.amax, w));
    kron_tc<D>(WSRC(uint32_t, hfrag) + 4 * FR, lp.hinv[4], WSRC(uint32_t, hfrag) + 5 * FR, lp.hinv[5], S.zb[w], iz, S.fb[w]);
  }
  __syncthreads();
  // ---- element-parallel: MLP residual, y = block - u, scatter_up into the lanes
  if constexpr (PAR) {
    cp_wait<0>();  // the row's u and lanes
    __syncthreads();
  }
  for (int c0 = 4 * tid; c0 < d; c0 += 4 * PT) {
    const float4 d44 = *reinterpret_cast<const float4*>(WSRC(float, d4) + c0);
    const int pi = pad_idx<D>(c0);
#pragma unroll
    for (int i = 0; i < PW; ++i) {
      if (i >= nrow) break;
      const int r = r0 + i;
      const float4 sv = *reinterpret_cast<const float4*>(s1all + i * d + c0);
      const float4 fv = *reinterpret_cast<const float4*>(&S.fb[i][pi]);
      const float4 uv = *reinterpret_cast<const float4*>((PAR ? stb + so.u : u + (size_t)r * d) + c0);
      const float y[4] = {sv.x + fv.x * d44.x - uv.x, sv.y + fv.y * d44.y - uv.y, sv.z + fv.z * d44.z - uv.z,
                          sv.w + fv.w * d44.w - uv.w};
      const float* lin = (PAR ? stb + so.lanes : lanes + (size_t)r * nl * d) + c0;
      float* lr = lanes + (size_t)r * nl * d + c0;
      float4 lv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) lv[j] = j < nl ? *reinterpret_cast<const float4*>(lin + j * d) : make_float4(0, 0, 0, 0);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        if (a >= nl) break;
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float accv = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j < nl) accv += S.gs[i][nl + a * nl + j] * (&lv[j].x)[e];
          o[e] = accv + S.gs[i][a] * y[e];
        }
        *reinterpret_cast<float4*>(lr + a * d) = make_float4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

#undef WSRC

// Weight fragments of one D x D matrix W used as the mma A operand with
// element (m, k) = W[k][m], scaled by 2^e: [D/16][D/16][32 lanes][4 hi, 4 lo].
void frag_block(const float* W, int D, int e, uint32_t* out) {
  const int MT = D / 16, KS = D / 16;
  const float s = std::ldexp(1.f, e);
  for (int mt = 0; mt < MT; ++mt)
    for (int ks = 0; ks < KS; ++ks)
      for (int lane = 0; lane < 32; ++lane) {
        const int g = lane >> 2, t = lane & 3;
        auto el = [&](int m, int k) { return W[k * D + m] * s; };
        const int m0 = 16 * mt + g, k0 = 16 * ks + 2 * t;
        const float v[8] = {el(m0, k0),     el(m0, k0 + 1),     el(m0 + 8, k0),     el(m0 + 8, k0 + 1),
                            el(m0, k0 + 8), el(m0, k0 + 9), el(m0 + 8, k0 + 8), el(m0 + 8, k0 + 9)};
        uint32_t* o = out + ((mt * KS + ks) * 32 + lane) * 8;
        for (int i = 0; i < 4; ++i) {
          const __half h0 = __float2half_rn(v[2 * i]), h1 = __float2half_rn(v[2 * i + 1]);
          const __half l0 = __float2half_rn(v[2 * i] - __half2float(h0));
          const __half l1 = __float2half_rn(v[2 * i + 1] - __half2float(h1));
          o[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
          o[4 + i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
      }
}

}  // namespace

bool hada_tc_supported(int ba, int bb) { return ba == bb && (ba == 16 || ba == 32); }

size_t hada_frag_words(int D) { return 6 * (size_t)(D / 16) * (D / 16) * 32 * 8; }

void hada_frags(const float* const* mats, int D, uint32_t* out, float* inv) {
  const size_t fr = hada_frag_words(D) / 6;
  for (int i = 0; i < 6; ++i) {
    float amax = 0.f;
    for (int k = 0; k < D * D; ++k) amax = std::fmax(amax, std::fabs(mats[i][k]));
    const int e = pow2_exp(amax);
    frag_block(mats[i], D, e, out + i * fr);
    inv[i] = std::ldexp(1.f, -e);
  }
}

template <int D, int PW, int NW = PW>
static cudaError_t post_tc(const Geo& G, const RowBatch& rb, const LayerParams& lp, const uint32_t* p1,
                           const uint32_t* p2, const float* projo, const float* u, float* bx, const float* gates,
                           float* lanes, cudaStream_t st) {
  constexpr int FR = (D / 16) * (D / 16) * 32 * 8;
  const size_t stage =
      PostSmem<D, PW, NW>::PAR ? (size_t)PostStage(G.d, D * D, G.cond_rank, G.lanes, 6 * FR).total * 4 : 0;
  const size_t smem = sizeof(PostSmem<D, PW, NW>) + (size_t)PW * G.d * 4 + stage;
  auto k = layer_post_tc_kernel<D, PW, NW>;
  cudaError_t e = allow_smem((const void*)k, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k, dim3((rb.M + PW - 1) / PW), dim3(NW * 32), smem, st, G, rb, lp, p1, p2, projo, u, bx, gates,
                    lanes);
}

cudaError_t launch_layer_post_tc(const Geo& G, const RowBatch& rb, const LayerParams& lp, const uint32_t* p1,
                                 const uint32_t* p2, const float* projo, const float* u, float* bx,
                                 const float* gates, float* lanes, cudaStream_t st) {
  if (rb.M <= 0) return cudaSuccess;
  if (!lp.hfrag || G.lanes > 4 || G.cond_rank > 8 || G.cond_rank < 1 || G.ba != G.bb || G.hada_n < G.d)
    return cudaErrorInvalidValue;
  // Below 128 rows, one row per CTA of 8 warps (the row's element phases and
  // Kronecker products spread over the warps, its weights staged in shared
  // memory while the previous kernel finishes); 2-row CTAs between 128 and 2048
  // rows fill the SMs; from 2048 rows, 8- or 7-row CTAs (two resident per SM),
  // whichever leaves the fewest rows on the busiest SM.
  const bool small = rb.M < 2048;
  auto busiest = [&](int pw) { return ((rb.M + pw - 1) / pw + 2 * 148 - 1) / (2 * 148) * pw; };
  const bool seven = !small && rb.M >= 2048 && busiest(7) < busiest(8);
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const bool stageable = G.d % 4 == 0 && al16(lp.post_norm) && al16(lp.pre_hada) && al16(lp.d1) && al16(lp.d4) &&
                         al16(lp.cond_v) && al16(lp.cond_u) && al16(lp.d2) && al16(lp.b2) && al16(lp.d3) &&
                         al16(p1) && al16(p2) && al16(lp.hfrag) && al16(u) && al16(lanes);
  if (rb.M < 128 && stageable) {
    if (G.ba == 32) return post_tc<32, 1, 8>(G, rb, lp, p1, p2, projo, u, bx, gates, lanes, st);
    if (G.ba == 16) return post_tc<16, 1, 8>(G, rb, lp, p1, p2, projo, u, bx, gates, lanes, st);
    return cudaErrorInvalidValue;
  }
  if (G.ba == 32) return small ? post_tc<32, 2>(G, rb, lp, p1, p2, projo, u, bx, gates, lanes, st)
                         : seven ? post_tc<32, 7>(G, rb, lp, p1, p2, projo, u, bx, gates, lanes, st)
                                 : post_tc<32, 8>(G, rb, lp, p1, p2, projo, u, bx, gates, lanes, st);
  if (G.ba == 16) return small ? post_tc<16, 2>(G, rb, lp, p1, p2, projo, u, bx, gates, lanes, st)
                         : seven ? post_tc<16, 7>(G, rb, lp, p1, p2, projo, u, bx, gates, lanes, st)
                                 : post_tc<16, 8>(G, rb, lp, p1, p2, projo, u, bx, gates, lanes, st);
  return cudaErrorInvalidValue;
}

}  // namespace nb
