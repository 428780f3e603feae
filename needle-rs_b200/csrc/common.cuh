// Shared device-side types and helpers for the Needle-3 B200 path.
//
// Data layout in HBM (one copy of the container per GPU):
//   * CQ tensors stay exactly as the `.cact` v3 blob stores them: `rows` packed
//     rows of `row_bytes` (LSB-first index bitstream, crates/needle-core/src/
//     cq.rs:908-925) followed by `rows * groups` FP16 norms. The whole container
//     is copied to the device once and kernels read those blobs in place.
//   * FP16/FP32 vectors (norm scales, taps, HadamardMLP factors, mHC scalars) are
//     widened to f32 once at load time into a parameter arena.
//   * Per-session state (KV rings, conv and Engram tails, token history) lives in
//     one device allocation per session, described by a `SessDesc` kept in device
//     memory so a captured CUDA graph can replay across decode steps.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace nb {

constexpr int WARP = 32;
constexpr int MAX_SEG = 4;

// One CQ tensor slice read in place from the container: `rows` packed rows
// followed by FP16 group norms (cq.rs:181-238).
struct CqSeg {
  const uint8_t* packed;
  const __half* norms;
  int rows;
};

// A logical projection = row-concatenation of up to MAX_SEG tensors that share
// in_feat, group and width (q|k|v|gate, Engram key|value).
struct CqMat {
  CqSeg seg[MAX_SEG];
  int nseg;
  int rows;       // total rows
  int in_feat;
  int in_pad;     // in_feat rounded up to the group
  int row_bytes;  // in_pad * bits / 8
  int groups;     // in_pad / group
  int group;      // 128 on every shipped tensor
  int bits;       // 2 or 4 (byte-aligned widths)
  float levels[16];
  // Every row's levels expanded once to f16 for the tensor-core projection
  // ([rows][in_pad], times the power of two umma_level_scale gives), or null:
  // the projection then expands the rows it needs on every call. lvl_lo holds
  // the remainders and is null when the scaled levels are exact in f16.
  const __half* lvl_hi;
  const __half* lvl_lo;
};

// Per-layer KV ring of one session. Device layout is head-major so one KV
// head's keys are contiguous: k [kv_heads][slots][qk] (f32 or i8),
// v [kv_heads][slots][vh], scales [kv_heads][slots] (int8 only).
struct LayerKV {
  void* k;
  void* v;
  float* ks;
  float* vs;
  int slots;
  int cap;
};

// Device-resident session descriptor (crates/needle-core/src/v3/cache.rs:148).
struct SessDesc {
  int pos;        // next position to write
  int int8;       // KvPrecision::Int8
  LayerKV* layers;
  float* qkv_tail;   // [layers][taps-1][q_dim+k_dim+v_dim], ring slot = pos % (taps-1)
  float* eng_tail;   // [sites][reach][d_model], ring slot = pos % reach
  uint32_t* toks;    // [4] token ring, slot = pos % 4
};

// One activation row of a batched forward: a (session, position) pair.
struct RowInfo {
  SessDesc* s;
  int pos;
  int base;  // prefill: row index of this session's position 0 in the launch; -1 for decode
  int len;   // prefill: prompt length of the session; -1 for decode
  int pad;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `red` is shared scratch of >= 32 floats. All threads get the
// result. Contains __syncthreads: call from every thread of the block.
__device__ __forceinline__ float block_sum(float v, float* red) {
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}
__device__ __forceinline__ float block_max(float v, float* red) {
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
  return warp_max(t);
}

// quant_into (crates/needle-core/src/v3/cache.rs:100-106, quant_scale
// :91-98) of one head vector held by a warp, two elements per lane (lanes past
// the vector's end hold 0): scale = absmax / 127 (1 for an all-zero vector),
// code = clamp(roundf(x * (1 / scale)), -128, 127). IEEE division for the
// scale and its reciprocal and roundf's half-away-from-zero rounding make it
// bit-exact with the reference on identical inputs. This is the only int8
// quantiser on the GPU: the KV append and the query fake-quant of qkv_post and
// the standalone nd_kv_quant all call it. Returns the scale; the codes come
// back as floats holding integers in [-128, 127]. Split in two steps
// (kv_quant_absmax_warp, kv_quant_codes) so that a warp holding several
// vectors can run their reductions back to back.
//
// The absolute maximum is one redux.sync over the IEEE bits: non-negative
// floats order as their bit patterns. A NaN lane counts as 0, as fmaxf
// ignores a NaN; an all-NaN vector gives 0 and scale 1 either way.
__device__ __forceinline__ float kv_quant_absmax_warp(float a, float b) {
  uint32_t u = __float_as_uint(fmaxf(fabsf(a), fabsf(b)));
  u = u > 0x7f800000u ? 0u : u;
  return __uint_as_float(__reduce_max_sync(0xffffffffu, u));
}
__device__ __forceinline__ float kv_quant_codes(float am, float a, float b, float* ca, float* cb) {
  const float scale = am > 0.0f ? __fdiv_rn(am, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, scale);
  *ca = fminf(fmaxf(roundf(__fmul_rn(a, inv)), -128.0f), 127.0f);
  *cb = fminf(fmaxf(roundf(__fmul_rn(b, inv)), -128.0f), 127.0f);
  return scale;
}
__device__ __forceinline__ float kv_quant_warp(float a, float b, float* ca, float* cb) {
  return kv_quant_codes(kv_quant_absmax_warp(a, b), a, b, ca, cb);
}

// Normalised Walsh-Hadamard transform of 128 floats held by one warp, 4 per
// lane (element e = lane*4 + i). Same butterfly pairs and operand order as
// crates/needle-core/src/hadamard.rs:24-55 (stride 1, 2, 4, ..., 64; a+b to the
// lower index, a-b to the upper), so the result is bit-identical; the
// 1/sqrt(128) scale (0x3db504f3 = 1.0f/sqrtf(128.f)) is applied at the end.
__device__ __forceinline__ void fwht128_warp(float (&x)[4]) {
  int lane = threadIdx.x & 31;
  float a0 = x[0] + x[1], a1 = x[0] - x[1], a2 = x[2] + x[3], a3 = x[2] - x[3];
  x[0] = a0 + a2;
  x[2] = a0 - a2;
  x[1] = a1 + a3;
  x[3] = a1 - a3;
#pragma unroll
  for (int b = 0; b < 5; ++b) {
    int m = 1 << b;
    bool upper = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float o = __shfl_xor_sync(0xffffffffu, x[i], m);
      x[i] = upper ? (o - x[i]) : (x[i] + o);
    }
  }
  const float s = __int_as_float(0x3db504f3);
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] *= s;
}

// FWHT of `n128` consecutive 128-float groups stored in shared (or global)
// memory, one warp per group, in place.
__device__ __forceinline__ void fwht_groups_warp(float* buf, int n128) {
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int g = wid; g < n128; g += nw) {
    float4 v = reinterpret_cast<float4*>(buf + g * 128)[lane];
    float x[4] = {v.x, v.y, v.z, v.w};
    fwht128_warp(x);
    reinterpret_cast<float4*>(buf + g * 128)[lane] = make_float4(x[0], x[1], x[2], x[3]);
  }
}

// x as an f16 high part (low half) and the f16 of the remainder (high half).
__device__ __forceinline__ uint32_t split_h16(float x) {
  const __half h = __float2half_rn(x);
  const __half l = __float2half_rn(x - __half2float(h));
  return (uint32_t)__half_as_ushort(h) | ((uint32_t)__half_as_ushort(l) << 16);
}

// Destination of a projection input written straight in the tensor-core
// projection's operand form: hi / lo [rows][K] f16 and inv [rows][K / 128]
// (the inverse scale of each 128-wide group). Null hi: the producer writes
// its f32 rows instead.
struct SplitOut {
  __half* hi;
  __half* lo;
  float* inv;
};

// One 128-wide group of an activation row held by a warp (element lane*4 + i
// in x[i]) in that form: scaled by the power of two 2^e that brings the
// group's max|x| into [2^13, 2^14) (e = 0 for an all-zero, denormal-only or
// non-finite max; e held at 126 for groups below 2^-112), each value split
// into an f16 high part and
// the f16 of its remainder (22 bits together), and the inverse scale. hi / lo
// point at the group's first element, inv at its scale.
__device__ __forceinline__ void split_group_store(const float (&x)[4], __half* hi, __half* lo, float* inv) {
  const int lane = threadIdx.x & 31;
  // The warp's max|x| in one instruction: non-negative floats order as their
  // bit patterns. (fmaxf skips a NaN; the NaN itself still reaches the
  // operands and the product.)
  const uint32_t mb = __float_as_uint(fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3]))));
  uint32_t wb;
  asm("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(wb) : "r"(mb));
  // e from the exponent field f of a normal max (max in [2^(f-127),
  // 2^(f-126))), and 2^e, 2^-e built from their bits.
  const int f = (int)(wb >> 23);
  const int e = (f == 0 || f >= 255) ? 0 : min(140 - f, 126);
  const float sc = __uint_as_float((uint32_t)(127 + e) << 23);
  const __half2 h01 = __floats2half2_rn(x[0] * sc, x[1] * sc), h23 = __floats2half2_rn(x[2] * sc, x[3] * sc);
  const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
  const __half2 l01 = __floats2half2_rn(x[0] * sc - f01.x, x[1] * sc - f01.y);
  const __half2 l23 = __floats2half2_rn(x[2] * sc - f23.x, x[3] * sc - f23.y);
  *reinterpret_cast<uint2*>(hi + lane * 4) =
      make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
  *reinterpret_cast<uint2*>(lo + lane * 4) =
      make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
  if (lane == 0) *inv = __uint_as_float((uint32_t)(127 - e) << 23);
}

// Greedy-pick key of output column `col` holding v (not a NaN): larger for a
// larger value and, among equal values, for a lower column, so the maximum key
// of a row is its first maximum, as argmax keeps it (v3_engine.rs:410-420);
// -0 counts as +0, as the comparison does. Never 0, which stands for a row
// whose outputs are all NaN (pick 0).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t col) {
  uint32_t b = __float_as_uint(v);
  if (b == 0x80000000u) b = 0u;
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (0xffffffffu - col);
}
__host__ __device__ __forceinline__ uint32_t argmax_pick(unsigned long long key) {
  return key ? 0xffffffffu - (uint32_t)key : 0u;
}

// cp.async copies global -> shared (src-size 0 when !valid: zero-fill, nothing read).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool valid) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  int n = valid ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialization attribute may start while the previous kernel in the
// stream is still running; pdl_wait() blocks until that kernel has completed
// and its memory is visible (a no-op for a normal launch), so everything a
// kernel reads or writes that another kernel touches comes after it.
// pdl_trigger() lets the next such kernel be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// Packed row and norms of logical row r of a (multi-segment) CQ matrix.
__device__ __forceinline__ void cq_row_ptr(const CqMat& W, int r, const uint8_t** row, const __half** nrm) {
  int s = 0, base = 0;
#pragma unroll
  for (int i = 0; i < MAX_SEG - 1; ++i) {
    if (s == i && i < W.nseg - 1 && r >= base + W.seg[i].rows) {
      base += W.seg[i].rows;
      s = i + 1;
    }
  }
  *row = W.seg[s].packed + (size_t)(r - base) * W.row_bytes;
  *nrm = W.seg[s].norms + (size_t)(r - base) * W.groups;
}

// Codes of elements g*128 + lane*4 .. +3 of a packed row, code i at bits
// [i*bits, (i+1)*bits) of the result (LSB-first bitstream, cq.rs:908-925):
// two bytes per lane at 4 bits, one byte at 2 bits.
__device__ __forceinline__ uint32_t cq_quad_codes(const uint8_t* row, int bits, int g, int lane) {
  if (bits == 4) return __ldg(reinterpret_cast<const uint16_t*>(row + g * 64) + lane);
  return __ldg(row + g * 32 + lane);
}

}  // namespace nb
