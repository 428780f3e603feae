// Grouped-query attention over the KV cache, f32 or int8.
//
// Restates attend_step_with (crates/needle-core/src/v3/attention.rs:327-377)
// for decode rows and attend_with (:241-287) for prefill rows: GQA with
// kv_head = h / repeat, scale 1/sqrt(qk_head_dim), softmax with max
// subtraction, then P.V. The int8 reader follows Int8View (:191-216): the
// per-(position, kv head) key scale multiplies the integer-valued dot and the
// value scale multiplies the softmax weight.
//
// Structure (split-position / "flash-decode"): one CTA per (row, KV head,
// split). A row's range [lo, hi] is cut into `nsplit` equal parts; each CTA
// streams its part in chunks of 128 positions through a double-buffered
// cp.async pipeline (keys, values and their scales in shared memory), keeps an
// online softmax per query head and writes an unnormalised partial
// (max, sum, P.V) per head. A combine step (fused into attn_finish for the
// forward, attn_combine for the standalone entry) merges the splits. All query
// heads of a KV head share one CTA, so each key/value byte is read from HBM
// once per row. Sums are reassociated relative to the reference's two-pass
// loop; results agree to f32 rounding.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.hpp"
#include "launch_util.hpp"

namespace nb {

constexpr int CH = 128;        // positions per chunk
constexpr int AT_THREADS = 128;
constexpr int AT_MAXREP = 8;

// Where keys/values of one (row, KV head) live: element (position n, KV head
// kh) of keys is at k + idx(n) * k_row + kh * k_head (elements), idx(n) = n %
// slots for a ring and base + n for the prefill scratch.
struct AttnSrc {
  const void* k;
  const void* v;
  const float* ks;
  const float* vs;
  long k_row, k_head, v_row, v_head, s_row, s_head;
  int slots;  // > 0: ring; 0: linear from `base`
  int base;
};


template <bool INT8, int QK, int VH>
struct AttnTile {
  static constexpr int ES = INT8 ? 1 : 4;
  static constexpr int KB = CH * QK * ES;  // key bytes per chunk
  static constexpr int VB = CH * VH * ES;  // value bytes per chunk
  static constexpr int KP = QK * ES / 16;  // 16-byte pieces per key row
  static constexpr int VP = VH * ES / 16;
  static constexpr int G = AT_THREADS / (VH / 4);  // position groups in P.V
};

template <bool INT8, int QK, int VH>
struct __align__(16) AttnSmem {
  using T = AttnTile<INT8, QK, VH>;
  uint8_t kbuf[2][T::KB];
  uint8_t vbuf[2][T::VB];
  float ksc[2][CH];
  float vsc[2][CH];
  float q[AT_MAXREP * QK];
  float P[CH][AT_MAXREP + 1];  // scores, then weights; padded row
  float m[AT_MAXREP], l[AT_MAXREP], corr[AT_MAXREP];
  float red[T::G][AT_MAXREP][VH];
};

// Issue the cp.async copies of one chunk [n0, n0 + CH) clipped at hi.
template <bool INT8, int QK, int VH>
__device__ __forceinline__ void issue_chunk(AttnSmem<INT8, QK, VH>& S, int buf, const AttnSrc& src,
                                            int kh, int n0, int hi) {
  using T = AttnTile<INT8, QK, VH>;
  const char* kb = (const char*)src.k;
  const char* vb = (const char*)src.v;
  // Storage index of position n0 + i: one modulo per chunk, then a wrap test.
  const int idx0 = src.slots > 0 ? n0 % src.slots : src.base + n0;
  auto index = [&](int i) -> long {
    if (src.slots == 0) return (long)idx0 + i;
    const int v = idx0 + i;
    if (src.slots >= CH) return v >= src.slots ? v - src.slots : v;
    return v % src.slots;
  };
  for (int j = threadIdx.x; j < CH * T::KP; j += AT_THREADS) {
    const int i = j / T::KP, pc = j % T::KP, n = n0 + i;
    const bool ok = n <= hi;
    const long idx = ok ? index(i) : 0;
    cp_async16(S.kbuf[buf] + i * QK * T::ES + pc * 16,
               kb + (idx * src.k_row + kh * src.k_head) * T::ES + pc * 16, ok);
  }
  for (int j = threadIdx.x; j < CH * T::VP; j += AT_THREADS) {
    const int i = j / T::VP, pc = j % T::VP, n = n0 + i;
    const bool ok = n <= hi;
    const long idx = ok ? index(i) : 0;
    cp_async16(S.vbuf[buf] + i * VH * T::ES + pc * 16,
               vb + (idx * src.v_row + kh * src.v_head) * T::ES + pc * 16, ok);
  }
  if (INT8) {
    for (int i = threadIdx.x; i < CH; i += AT_THREADS) {
      const int n = n0 + i;
      const bool ok = n <= hi;
      const long idx = ok ? index(i) : 0;
      cp_async4(&S.ksc[buf][i], src.ks + idx * src.s_row + kh * src.s_head, ok);
      cp_async4(&S.vsc[buf][i], src.vs + idx * src.s_row + kh * src.s_head, ok);
    }
  }
}

// One CTA: query heads [kh*rep, kh*rep + rep) of one row over positions
// [a, b] (inclusive; empty when a > b). Writes the partial to `part`:
// rep maxima, rep sums, rep x VH unnormalised outputs.
template <bool INT8, int QK, int VH>
__device__ void attend_part(AttnSmem<INT8, QK, VH>& S, const float* __restrict__ qrow, int rep,
                            const AttnSrc& src, int kh, int a, int b, float scale,
                            float* __restrict__ part) {
  using T = AttnTile<INT8, QK, VH>;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  for (int i = tid; i < rep * QK; i += AT_THREADS) S.q[i] = qrow[i];
  if (tid < AT_MAXREP) {
    S.m[tid] = -INFINITY;
    S.l[tid] = 0.f;
  }
  constexpr int DQ = VH / 4;  // d-quads
  const int dq = tid % DQ, grp = tid / DQ;
  float acc[AT_MAXREP][4];
#pragma unroll
  for (int h = 0; h < AT_MAXREP; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[h][e] = 0.f;
  const int nch = a <= b ? (b - a) / CH + 1 : 0;
  if (nch > 0) {
    issue_chunk<INT8, QK, VH>(S, 0, src, kh, a, b);
    cp_commit();
  }
  for (int c = 0; c < nch; ++c) {
    const int buf = c & 1;
    if (c + 1 < nch) {
      issue_chunk<INT8, QK, VH>(S, buf ^ 1, src, kh, a + (c + 1) * CH, b);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    // ---- scores: thread = position
    {
      const int n = a + c * CH + tid;
      float kv[QK];
      if (INT8) {
        const int8_t* kr = reinterpret_cast<const int8_t*>(S.kbuf[buf]) + tid * QK;
#pragma unroll
        for (int i = 0; i < QK; i += 16) {
          int4 w = *reinterpret_cast<const int4*>(kr + i);
          const int8_t* bb = reinterpret_cast<const int8_t*>(&w);
#pragma unroll
          for (int j = 0; j < 16; ++j) kv[i + j] = (float)bb[j];
        }
      } else {
        const float* kr = reinterpret_cast<const float*>(S.kbuf[buf]) + tid * QK;
#pragma unroll
        for (int i = 0; i < QK; i += 4) {
          float4 w = *reinterpret_cast<const float4*>(kr + i);
          kv[i] = w.x;
          kv[i + 1] = w.y;
          kv[i + 2] = w.z;
          kv[i + 3] = w.w;
        }
      }
      const float ksc = INT8 ? S.ksc[buf][tid] : 1.0f;
      const bool ok = n <= b;
#pragma unroll
      for (int h = 0; h < AT_MAXREP; ++h) {
        if (h < rep) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < QK; ++i) s += S.q[h * QK + i] * kv[i];
          if (INT8) s = s * ksc;
          S.P[tid][h] = ok ? s * scale : -INFINITY;
        }
      }
    }
    __syncthreads();
    // ---- online softmax per head (one warp per head)
    for (int h = wid; h < rep; h += AT_THREADS / 32) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < CH / 32; ++j) mx = fmaxf(mx, S.P[lane + 32 * j][h]);
      mx = warp_max(mx);
      const float mold = S.m[h], mnew = fmaxf(mold, mx);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < CH / 32; ++j) {
        const int i = lane + 32 * j;
        const float s = S.P[i][h];
        const float p = s == -INFINITY ? 0.f : expf(s - mnew);
        sum += p;
        S.P[i][h] = INT8 ? p * S.vsc[buf][i] : p;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float cr = mold == -INFINITY ? 0.f : expf(mold - mnew);
        S.corr[h] = cr;
        S.l[h] = S.l[h] * cr + sum;
        S.m[h] = mnew;
      }
    }
    __syncthreads();
    // ---- P.V: thread = (position group, d-quad), all heads
#pragma unroll
    for (int h = 0; h < AT_MAXREP; ++h)
      if (h < rep) {
        const float cr = S.corr[h];
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[h][e] *= cr;
      }
    for (int i = grp; i < CH; i += T::G) {
      float v4[4];
      if (INT8) {
        const int w = *reinterpret_cast<const int*>(S.vbuf[buf] + i * VH + dq * 4);
        v4[0] = (float)(int8_t)(w & 0xff);
        v4[1] = (float)(int8_t)((w >> 8) & 0xff);
        v4[2] = (float)(int8_t)((w >> 16) & 0xff);
        v4[3] = (float)(int8_t)((w >> 24) & 0xff);
      } else {
        const float4 w = *reinterpret_cast<const float4*>(S.vbuf[buf] + (i * VH + dq * 4) * 4);
        v4[0] = w.x;
        v4[1] = w.y;
        v4[2] = w.z;
        v4[3] = w.w;
      }
#pragma unroll
      for (int h = 0; h < AT_MAXREP; ++h)
        if (h < rep) {
          const float p = S.P[i][h];
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[h][e] += p * v4[e];
        }
    }
    __syncthreads();
  }
  // ---- reduce the position groups and write the partial
#pragma unroll
  for (int h = 0; h < AT_MAXREP; ++h)
    if (h < rep)
#pragma unroll
      for (int e = 0; e < 4; ++e) S.red[grp][h][dq * 4 + e] = acc[h][e];
  __syncthreads();
  for (int o = tid; o < rep * VH; o += AT_THREADS) {
    const int h = o / VH, d = o % VH;
    float s = 0.f;
    for (int g = 0; g < T::G; ++g) s += S.red[g][h][d];
    part[2 * rep + o] = s;
  }
  if (tid < rep) {
    part[tid] = S.m[tid];
    part[rep + tid] = S.l[tid];
  }
}

// Split z of `nsplit` equal, chunk-aligned parts of [lo, hi].
__device__ __forceinline__ void split_range(int lo, int hi, int nsplit, int z, int* a, int* b) {
  const int len = hi - lo + 1;
  int spl = (len + nsplit - 1) / nsplit;
  spl = (spl + CH - 1) / CH * CH;
  *a = lo + z * spl;
  *b = min(hi, lo + (z + 1) * spl - 1);
}

// Keys/values of row r for the forward pass: the prefill scratch ([row][kv
// head][dim], linear from the session's first row) or the session's head-major
// ring. Sets the first visible position lo (local window, ring floor) and the
// row's position p.
template <int QK, int VH>
__device__ __forceinline__ AttnSrc layer_src(const Geo& G, int li, const RowBatch& rb, int r, int window,
                                             const void* pk, const void* pv, const float* pks,
                                             const float* pvs, int* lo_out, int* p_out) {
  const RowInfo ri = rb.rows[r];
  const int p = ri.pos;
  int lo = (window > 0 && p + 1 > window) ? p + 1 - window : 0;
  AttnSrc src;
  if (rb.mode == MODE_PREFILL) {
    src.k = pk;
    src.v = pv;
    src.ks = pks;
    src.vs = pvs;
    src.k_row = (long)G.kvh * QK;
    src.k_head = QK;
    src.v_row = (long)G.kvh * VH;
    src.v_head = VH;
    src.s_row = G.kvh;
    src.s_head = 1;
    src.slots = 0;
    src.base = ri.base;
  } else {
    const LayerKV kv = ri.s->layers[li];
    src.k = kv.k;
    src.v = kv.v;
    src.ks = kv.ks;
    src.vs = kv.vs;
    src.k_row = QK;
    src.k_head = (long)kv.slots * QK;
    src.v_row = VH;
    src.v_head = (long)kv.slots * VH;
    src.s_row = 1;
    src.s_head = kv.slots;
    src.slots = kv.slots;
    src.base = 0;
    const int floor = p + 1 > kv.slots ? p + 1 - kv.slots : 0;  // cache.rs:322-331
    lo = max(lo, floor);
  }
  *lo_out = lo;
  *p_out = p;
  return src;
}

// Finish of one (row, KV head) once every split's partial is in ps (natural-
// log maxima): the softmax merge over the splits, the output gate
// (model.rs:305-308) and the rotation of the rep * VH outputs, whole 128-wide
// groups, into oh; the arithmetic of attn_finish_kernel with the splits of one
// KV head. F: shared scratch of FINISH_SCRATCH floats. Contains
// __syncthreads.
constexpr int FINISH_SCRATCH = AT_MAXREP * 64 + 8 + AT_MAXREP * 64 + 64 * 2 * AT_MAXREP;
template <int VH>
__device__ void finish_kvhead(const Geo& G, int r, int kh, int rep, int nsplit, const float* ps,
                              const float* __restrict__ proj, float* __restrict__ oh, float* F, const SplitOut& so) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  const int pw = rep * (VH + 2);
  float* Fw = F;              // [rep][64] split weights exp(m_z - M)
  float* FL = Fw + rep * 64;  // [rep] sums
  float* Fo = FL + 8;         // [rep * VH] gated outputs
  float* Fm = Fo + rep * VH;  // [nsplit][2 * rep] the splits' maxima and sums
  for (int i = tid; i < nsplit * 2 * rep; i += blockDim.x) Fm[i] = __ldcg(ps + (i / (2 * rep)) * pw + i % (2 * rep));
  __syncthreads();
  if (tid < rep) {
    const int h = tid;
    float M = -INFINITY;
    for (int z = 0; z < nsplit; ++z) M = fmaxf(M, Fm[z * 2 * rep + h]);
    float L = 0.f;
    for (int z = 0; z < nsplit; ++z) {
      const float mz = Fm[z * 2 * rep + h];
      const float wz = mz == -INFINITY ? 0.f : expf(mz - M);
      Fw[h * 64 + z] = wz;
      L += wz * Fm[z * 2 * rep + rep + h];
    }
    FL[h] = L;
  }
  __syncthreads();
  const float* gate = proj + (size_t)r * G.proj_dim + G.qkv_dim + (size_t)kh * rep * VH;
  for (int i = tid; i < rep * VH; i += blockDim.x) {
    const int h = i / VH;
    float o = 0.f;
#pragma unroll 4
    for (int z = 0; z < nsplit; ++z) o += Fw[h * 64 + z] * __ldcg(ps + z * pw + 2 * rep + i);
    Fo[i] = o / FL[h] * sigmoidf_(gate[i]);
  }
  __syncthreads();
  const int opad = (G.o_dim + 127) / 128 * 128;
  float* ohr = oh + (size_t)r * opad + (size_t)kh * rep * VH;
  for (int gg = wid; gg < rep * VH / 128; gg += nw) {
    const float4 v = reinterpret_cast<const float4*>(Fo + gg * 128)[lane];
    float x[4] = {v.x, v.y, v.z, v.w};
    fwht128_warp(x);
    if (so.hi) {  // out_proj's tensor-core operands
      const int g = kh * rep * VH / 128 + gg;
      split_group_store(x, so.hi + (size_t)r * opad + g * 128, so.lo + (size_t)r * opad + g * 128,
                        so.inv + (size_t)r * (opad / 128) + g);
    } else {
      reinterpret_cast<float4*>(ohr + gg * 128)[lane] = make_float4(x[0], x[1], x[2], x[3]);
    }
  }
}

// Forward-pass attention: grid (rows, kv_heads, nsplit). With oh (and proj,
// cnt: per-(row, KV head) counters, zero-initialised) the last CTA of each
// (row, KV head) to arrive also finishes it (finish_kvhead) and resets its
// counter; no CTA waits for another.
template <bool INT8, int QK, int VH>
__global__ void __launch_bounds__(AT_THREADS) layer_attn_kernel(Geo G, int li, RowBatch rb, int window,
                                                                int nsplit, const float* __restrict__ qpost,
                                                                const void* pk, const void* pv,
                                                                const float* pks, const float* pvs,
                                                                float* __restrict__ part,
                                                                const float* __restrict__ proj,
                                                                float* __restrict__ oh, int* __restrict__ cnt,
                                                                SplitOut so) {
  pdl_trigger();  // a PDL-launched projection after this kernel may start its weight prefetch
  pdl_wait();     // everything below reads or writes what earlier kernels touch
  extern __shared__ __align__(16) unsigned char smraw[];
  auto& S = *reinterpret_cast<AttnSmem<INT8, QK, VH>*>(smraw);
  const int r = blockIdx.x, kh = blockIdx.y, z = blockIdx.z;
  const int rep = G.heads / G.kvh;
  int lo, p;
  const AttnSrc src = layer_src<QK, VH>(G, li, rb, r, window, pk, pv, pks, pvs, &lo, &p);
  int a, b;
  split_range(lo, p, nsplit, z, &a, &b);
  const int pw = rep * (VH + 2);
  attend_part<INT8, QK, VH>(S, qpost + (size_t)r * G.q_dim + (size_t)kh * rep * QK, rep, src, kh, a, b,
                            1.0f / sqrtf((float)QK), part + (((size_t)r * G.kvh + kh) * nsplit + z) * pw);
  if (!oh) return;  // attn_finish combines and rotates
  static_assert(sizeof(AttnSmem<INT8, QK, VH>) >= FINISH_SCRATCH * sizeof(float), "finish scratch");
  __shared__ int last;
  __syncthreads();  // this CTA's partial is written; its shared memory is free
  if (nsplit > 1) {
    if (threadIdx.x == 0) {
      __threadfence();
      last = atomicAdd(&cnt[(size_t)r * G.kvh + kh], 1) == nsplit - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (threadIdx.x == 0) cnt[(size_t)r * G.kvh + kh] = 0;  // ready for the next launch
  }
  finish_kvhead<VH>(G, r, kh, rep, nsplit, part + ((size_t)r * G.kvh + kh) * nsplit * pw, proj, oh,
                    reinterpret_cast<float*>(smraw), so);
}

// ----------------------------------------------------------------------------
// int8 KV on the tensor cores.
//
// In int8 mode the query is fake-quantised (model.rs:289-293): q = code * qs
// with integer codes, so q.k = qs * sum(code * k8) and the key dot is an exact
// integer product, run as mma.sync s8 x s8 -> s32 (m16n8k32 / m16n8k16) with
// positions as the 16 rows (keys straight from shared memory as A) and the
// query heads of one KV head as the 8 columns (their codes held in registers
// as B; columns >= rep are zero). The score is then dot * (qs * scale) * ks,
// the reference's f32 dot times the key scale (attention.rs:191-216) up to
// f32 rounding of the products.
//
// P.V runs transposed, O^T = V^T P^T, as m16n8k16 f16 MMAs with f32
// accumulation: value dimensions are the 16 rows, heads the 8 columns. V^T
// comes straight from the int8 values in shared memory by ldmatrix.trans of
// byte pairs; each register splits into an even-dimension and an
// odd-dimension fragment, widened exactly to f16 (bias trick: byte ^ 0x80
// placed under exponent byte 0x64 is 1024 + u in f16; subtracting 1152 gives
// the signed value). Each weight p * vs is split into an f16 high part and an
// f16 remainder (two MMAs), which keeps about 22 bits of the weight. The
// weights leave the score fragment as [position][head] 8x8 blocks;
// movmatrix.trans turns each into the [head][position] pairs of the B
// fragment, so they never touch memory.
//
// Each of the four warps of a CTA owns every fourth 32-position block of the
// CTA's range with its own double block buffer and its own online softmax,
// so the main loop has no block-wide barrier; the warps merge at the end and
// the CTA writes the same (max, sum, P.V) partial as the f32 kernel.
// ----------------------------------------------------------------------------
constexpr int WB = 32;  // positions per warp block
constexpr int NJ = WB / 16;  // 16-position MMA tiles per warp block

template <int QK, int VH>
struct MmaTile {
  // Key row stride in shared memory: conflict-free 32-bit fragment loads.
  static constexpr int KS = QK == 16 ? 16 : (QK % 32 == 0 ? QK + 16 : QK);
  static constexpr int KP = QK / 16;   // 16-byte pieces per key row
  static constexpr int VP = VH / 16;   // 16-byte pieces per value row
  static constexpr int NT = VH / 8;    // P.V n-tiles
  static constexpr int NK32 = QK / 32; // m16n8k32 steps of the key dot
  static constexpr bool K16 = (QK % 32) != 0;
};

constexpr int NBUF = 2;  // per-warp block buffers: one block in flight while one is consumed (five CTAs per SM)

template <int QK, int VH>
struct __align__(16) MmaWarpSmem {
  using T = MmaTile<QK, VH>;
  int8_t k[NBUF][WB * T::KS];
  int8_t v[NBUF][WB * VH];
  float ks[NBUF][WB];
  float vs[NBUF][WB];
  uint64_t bar[NBUF];  // bulk-copy completion of each buffer
};

__device__ __forceinline__ void mma_s8_k32(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ void mma_f16_k16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Four (two) 8x8 b16 matrices from shared memory, lane l supplying the row
// address of row l & 7 of matrix l >> 3; as s8 data, the A fragment of an
// m16n8k32 (m16n8k16) integer MMA when the matrices are (rows 0-7, bytes
// 0-15), (rows 8-15, bytes 0-15), (rows 0-7, bytes 16-31), (rows 8-15, bytes
// 16-31) of the tile.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* smem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r[0]), "=r"(r[1]) : "r"(s));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* smem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

// 2^x by the hardware approximation (PTX ex2.approx.ftz.f32, relative error
// about 2^-22); used for softmax weights, whose arguments are <= 0 and whose
// sum is >= 1, so flushing denormal results to zero changes nothing material.
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Transpose of an 8x8 b16 matrix held in the accumulator-fragment layout
// (lane 4r + c/2 holds row r, columns c and c + 1). A register-only
// operation, so it is not volatile: the scheduler may interleave it with the
// value-fragment loads and conversions of the same block.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

// Offset-binary value bytes (code ^ 0x80, as the KV append stores them) (a0,
// a1, b0, b1) of two adjacent positions' dimension pair -> f16 code pairs
// (a0, b0) and (a1, b1) (exact: the byte is the low mantissa of 1024 + byte,
// less 1152), for V^T fragments read by ldmatrix.trans straight from the ring.
__device__ __forceinline__ void i8pairs_to_h2(uint32_t u, uint32_t* even, uint32_t* odd) {
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  uint32_t a = __byte_perm(u, 0x64646464u, 0x4240), b = __byte_perm(u, 0x64646464u, 0x4341);
  __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias);
  __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
  *even = *reinterpret_cast<uint32_t*>(&ha);
  *odd = *reinterpret_cast<uint32_t*>(&hb);
}

__device__ __forceinline__ uint32_t pack_h2(float x, float y) {
  __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Storage index of position n0 + i of a block, i in [0, WB): one modulo per
// block (idx0 = n0 mod slots), then a wrap test per position.
__device__ __forceinline__ long block_index(const AttnSrc& src, int idx0, int i) {
  if (src.slots == 0) return (long)idx0 + i;
  int v = idx0 + i;
  if (src.slots >= WB) return v >= src.slots ? v - src.slots : v;
  return v % src.slots;  // rings shorter than a block (tiny geometries only)
}

// cp.async of one warp block [n0, n0 + WB) clipped at hi (zero-filled beyond).
template <int QK, int VH>
__device__ __forceinline__ void mma_issue(MmaWarpSmem<QK, VH>& W, int buf, const AttnSrc& src, int kh,
                                          int n0, int hi, int lane) {
  using T = MmaTile<QK, VH>;
  const int8_t* kb = (const int8_t*)src.k + kh * src.k_head;
  const int8_t* vb = (const int8_t*)src.v + kh * src.v_head;
  const int idx0 = src.slots > 0 ? n0 % src.slots : src.base + n0;
#pragma unroll
  for (int j = lane; j < WB * T::KP; j += 32) {
    const int i = j / T::KP, pc = j % T::KP;
    const bool ok = n0 + i <= hi;
    const long idx = ok ? block_index(src, idx0, i) : 0;
    cp_async16(W.k[buf] + i * T::KS + pc * 16, kb + idx * src.k_row + pc * 16, ok);
  }
#pragma unroll
  for (int j = lane; j < WB * T::VP; j += 32) {
    const int i = j / T::VP, pc = j % T::VP;
    const bool ok = n0 + i <= hi;
    const long idx = ok ? block_index(src, idx0, i) : 0;
    cp_async16(W.v[buf] + i * VH + pc * 16, vb + idx * src.v_row + pc * 16, ok);
  }
#pragma unroll
  for (int i = lane; i < WB; i += 32) {
    const bool ok = n0 + i <= hi;
    const long idx = ok ? block_index(src, idx0, i) : 0;
    cp_async4(&W.ks[buf][i], src.ks + idx * src.s_row + kh * src.s_head, ok);
    cp_async4(&W.vs[buf][i], src.vs + idx * src.s_row + kh * src.s_head, ok);
  }
}

// ---- bulk copies for ring sources whose per-head rows are contiguous.
constexpr unsigned long long ATTN_WAIT_NS = 1000000000ull;  // bound of every wait: one second

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool mbar_try_parity(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread until the phase completes, for at most
// `hint_ns` (the hardware wakes it at completion), so a waiting warp issues no
// polling instructions meanwhile.
__device__ __forceinline__ bool mbar_try_parity_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar`, giving up after ATTN_WAIT_NS.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_parity(bar, parity)) return true;
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
    if (mbar_try_parity_sleep(bar, parity, 20000u)) return true;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > ATTN_WAIT_NS) return false;
  }
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Keys and values of one warp block [n0, n0 + WB) clipped at hi, as at most
// two contiguous pieces per operand (the ring wraps at most once: slots >= WB)
// copied by lane 0 and completing on W.bar[buf]; the scales go by cp.async
// (zero-filled past hi). Rows past hi keep stale bytes: their scores are
// masked and their value scales are zero, so they contribute nothing.
// idx0 = n0 mod slots (the caller steps it from block to block).
template <int QK, int VH>
__device__ __forceinline__ void mma_issue_bulk(MmaWarpSmem<QK, VH>& W, int buf, const AttnSrc& src, int kh,
                                               int n0, int idx0, int hi, int lane) {
  const int cnt = min(WB, hi - n0 + 1);
  if (lane == 0) {
    const int c1 = min(cnt, src.slots - idx0);
    const int8_t* kb = (const int8_t*)src.k + kh * src.k_head;
    const int8_t* vb = (const int8_t*)src.v + kh * src.v_head;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&W.bar[buf])),
                 "r"((uint32_t)cnt * (QK + VH))
                 : "memory");
    bulk_g2s(W.k[buf], kb + (long)idx0 * QK, (uint32_t)c1 * QK, &W.bar[buf]);
    bulk_g2s(W.v[buf], vb + (long)idx0 * VH, (uint32_t)c1 * VH, &W.bar[buf]);
    if (cnt > c1) {
      bulk_g2s(W.k[buf] + c1 * QK, kb, (uint32_t)(cnt - c1) * QK, &W.bar[buf]);
      bulk_g2s(W.v[buf] + c1 * VH, vb, (uint32_t)(cnt - c1) * VH, &W.bar[buf]);
    }
  }
#pragma unroll
  for (int i = lane; i < WB; i += 32) {
    const bool ok = i < cnt;
    int idx = idx0 + i;
    idx = idx >= src.slots ? idx - src.slots : idx;
    idx = ok ? idx : 0;
    cp_async4(&W.ks[buf][i], src.ks + kh * src.s_head + idx, ok);  // a ring's scales: [kv head][slot]
    cp_async4(&W.vs[buf][i], src.vs + kh * src.s_head + idx, ok);
  }
}

template <int QK, int VH>
__global__ void __launch_bounds__(128, 5) layer_attn_i8_kernel(Geo G, int li, RowBatch rb, int window, int nsplit,
                                                            const int8_t* __restrict__ q8,
                                                            const float* __restrict__ q8s, const void* pk,
                                                            const void* pv, const float* pks, const float* pvs,
                                                            float* __restrict__ part, const float* __restrict__ proj,
                                                            float* __restrict__ oh, int* __restrict__ cnt,
                                                            int* __restrict__ werr, SplitOut so) {
  pdl_trigger();  // a PDL-launched projection after this kernel may start its weight prefetch
  pdl_wait();     // everything below reads or writes what earlier kernels touch
  using T = MmaTile<QK, VH>;
  using WS = MmaWarpSmem<QK, VH>;
  extern __shared__ __align__(16) unsigned char smraw[];
  const int r = blockIdx.x, kh = blockIdx.y, z = blockIdx.z;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  WS& W = reinterpret_cast<WS*>(smraw)[wid];
  const int rep = G.heads / G.kvh;
  int lo, p;
  const AttnSrc src = layer_src<QK, VH>(G, li, rb, r, window, pk, pv, pks, pvs, &lo, &p);
  int a, b;
  split_range(lo, p, nsplit, z, &a, &b);
  // Scores are kept in base-2 units (times log2 e) so the softmax uses exp2f.
  const float scale = 1.0f / sqrtf((float)QK) * 1.44269504088896341f;

  // Query codes as the B operand of the key MMAs: column n of B is query head
  // kh * rep + n (columns >= rep are zero), so lane (g, t) holds head g's
  // codes at k = 4t.. of each 16-wide half of a 32-wide k step.
  const bool hv = g < rep;
  const int8_t* qr = q8 + (size_t)r * G.q_dim + (size_t)(kh * rep + (hv ? g : 0)) * QK;
  uint32_t qb[T::NK32 > 0 ? T::NK32 : 1][2];
  uint32_t qb16 = 0;
#pragma unroll
  for (int s = 0; s < T::NK32; ++s) {
    qb[s][0] = hv ? __ldg(reinterpret_cast<const uint32_t*>(qr + s * 32 + t * 4)) : 0u;
    qb[s][1] = hv ? __ldg(reinterpret_cast<const uint32_t*>(qr + s * 32 + 16 + t * 4)) : 0u;
  }
  if (T::K16) qb16 = hv ? __ldg(reinterpret_cast<const uint32_t*>(qr + T::NK32 * 32 + t * 4)) : 0u;
  // This lane's score columns are heads 2t and 2t + 1: the query scale times
  // the softmax scale for each (zero for padding columns).
  float qsc[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int h = 2 * t + e;
    qsc[e] = h < rep ? q8s[(size_t)r * G.heads + kh * rep + h] * scale : 0.f;
  }

  // Running max and this lane's share of the sum for heads 2t, 2t + 1.
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  // O^T accumulators: m-tile mt covers value dims mt*16 .. mt*16+15; lane
  // (g, t) holds dims mt*16+g (regs 0, 1) and mt*16+g+8 (regs 2, 3) of heads
  // 2t (regs 0, 2) and 2t + 1 (regs 1, 3).
  constexpr int MT = VH / 16;
  float o[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  const int nblk = a <= b ? (b - a) / WB + 1 : 0;
  const int mine = nblk > wid ? (nblk - wid + 3) / 4 : 0;  // blocks wid, wid + 4, ...
  // Ring rows of one KV head are contiguous: lane 0 moves a block with bulk
  // copies. Other sources (the prefill scratch interleaves KV heads) and padded
  // key rows go by per-lane cp.async.
  const bool bulk = src.slots >= WB && T::KS == QK;
  if (bulk) {
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < NBUF; ++i) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&W.bar[i])));
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
  }
  // Block c of this warp (position a + (wid + 4c) * WB) goes to buffer c % NBUF;
  // one cp.async commit group per block (empty past the last) keeps the
  // group count uniform. Blocks are issued in order, so the ring index of the
  // next one steps by 4 * WB instead of a modulo per block.
  int ring_idx = bulk ? (a + wid * WB) % src.slots : 0;
  auto issue = [&](int c) {
    if (c < mine) {
      const int n0 = a + (wid + 4 * c) * WB;
      if (bulk) {
        mma_issue_bulk<QK, VH>(W, c % NBUF, src, kh, n0, ring_idx, b, lane);
        ring_idx += 4 * WB;
        while (ring_idx >= src.slots) ring_idx -= src.slots;
      } else {
        mma_issue<QK, VH>(W, c % NBUF, src, kh, n0, b, lane);
      }
    }
    cp_commit();
  };
  bool failed = false;
#pragma unroll
  for (int c = 0; c < NBUF - 1; ++c) issue(c);
  for (int c = 0; c < mine; ++c) {
    const int buf = c % NBUF;
    const int n0 = a + (wid + 4 * c) * WB;
    issue(c + NBUF - 1);
    cp_wait<NBUF - 1>();
    if (bulk && !__all_sync(0xffffffffu, mbar_wait_bounded(&W.bar[buf], (uint32_t)(c / NBUF) & 1u))) {
      // The copy never completed: report it, let the copies in flight land
      // (bounded) and leave this warp's partial empty.
      if (lane == 0) atomicExch(werr, 2);
      for (int cc = c + 1; cc < c + NBUF && cc < mine; ++cc)
        mbar_wait_bounded(&W.bar[cc % NBUF], (uint32_t)(cc / NBUF) & 1u);
      failed = true;
      break;
    }
    __syncwarp();
    // ---- integer key dots, positions as rows: m-tile j covers positions
    // j*16 .. j*16+15; d[j] = (pos g, heads 2t, 2t+1), (pos g+8, same heads)
    int d[NJ][4];
#pragma unroll
    for (int j = 0; j < NJ; ++j) d[j][0] = d[j][1] = d[j][2] = d[j][3] = 0;
    // A fragments by ldmatrix: lane l addresses row (l >> 3 & 1) * 8 + (l & 7)
    // of the 16-position tile at byte offset (l >> 4) * 16 of the 32-byte step
    // (rows KS bytes apart: 16-byte aligned and bank-conflict free).
    const int8_t* krow = W.k[buf] + (((lane >> 3) & 1) * 8 + (lane & 7)) * T::KS + (lane >> 4) * 16;
#pragma unroll
    for (int s = 0; s < T::NK32; ++s)
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        uint32_t ka[4];
        ldsm_x4(ka, krow + j * 16 * T::KS + s * 32);
        mma_s8_k32(d[j], ka, qb[s][0], qb[s][1]);
      }
    if (T::K16) {
      const int8_t* krow16 = W.k[buf] + (((lane >> 3) & 1) * 8 + (lane & 7)) * T::KS + T::NK32 * 32;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        uint32_t ka[2];
        ldsm_x2(ka, krow16 + j * 16 * T::KS);
        mma_s8_k16(d[j], ka[0], ka[1], qb16);
      }
    }
    // Score i of this lane: position j*16 + g + 8*hf (i = 4j + 2hf + e), head 2t + e.
    float sc[4 * NJ];
    if (n0 + WB - 1 <= b) {  // a full block (warp-uniform): no position masked
#pragma unroll
      for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const float ksv = W.ks[buf][j * 16 + hf * 8 + g];
#pragma unroll
          for (int e = 0; e < 2; ++e) sc[4 * j + 2 * hf + e] = (float)d[j][2 * hf + e] * qsc[e] * ksv;
        }
    } else {
#pragma unroll
      for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int pi = j * 16 + hf * 8 + g;
          const float ksv = W.ks[buf][pi];
          const bool ok = n0 + pi <= b;
#pragma unroll
          for (int e = 0; e < 2; ++e)
            sc[4 * j + 2 * hf + e] = ok ? (float)d[j][2 * hf + e] * qsc[e] * ksv : -INFINITY;
        }
    }
    // ---- online softmax per head (column): the 8 lanes sharing t hold
    // the block's WB positions of heads 2t, 2t + 1
    // When no running max of the warp moved, every correction factor is
    // exp2(0) = 1 and the rescale of l and O is skipped (warp-uniform).
    float mold[2], mz[2];
    bool moved = false;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float mx = sc[e];
#pragma unroll
      for (int q = 1; q < 2 * NJ; ++q) mx = fmaxf(mx, sc[2 * q + e]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mnew = fmaxf(m[e], mx);
      moved |= mnew != m[e];
      mz[e] = mnew == -INFINITY ? 0.f : mnew;  // every position so far masked: weights are 0
      mold[e] = m[e];
      m[e] = mnew;
    }
    const bool rescale = __any_sync(0xffffffffu, moved);
    float pw[4 * NJ];
#pragma unroll
    for (int i = 0; i < 4 * NJ; ++i) pw[i] = ex2_fast(sc[i] - mz[i & 1]);
    float corr[2] = {1.f, 1.f};
    if (rescale) {
#pragma unroll
      for (int e = 0; e < 2; ++e) corr[e] = ex2_fast(mold[e] - mz[e]);
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < NJ; ++q) sum += pw[4 * q + e] + pw[4 * q + 2 + e];
      l[e] = rescale ? l[e] * corr[e] + sum : l[e] + sum;
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const float vsv = W.vs[buf][j * 16 + hf * 8 + g];
        pw[4 * j + 2 * hf] *= vsv;
        pw[4 * j + 2 * hf + 1] *= vsv;
      }
    if (rescale) {
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        o[i][0] *= corr[0];
        o[i][1] *= corr[1];
        o[i][2] *= corr[0];
        o[i][3] *= corr[1];
      }
    }
    __syncwarp();  // f16 values visible to every lane
    // ---- O^T += V^T P^T: k-step j covers positions j*16 .. j*16+15. The
    // weights (f16 high part and remainder) of 8 positions x 8 heads sit in
    // the score fragment as [position][head]; movmatrix.trans turns each into
    // the [head][position] pairs of the B fragment.
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      uint32_t bh[2], bl[2];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const float x0 = pw[4 * j + 2 * hf], x1 = pw[4 * j + 2 * hf + 1];
        const uint32_t h = pack_h2(x0, x1);
        const __half2 hh = *reinterpret_cast<const __half2*>(&h);
        const uint32_t lw = pack_h2(x0 - __low2float(hh), x1 - __high2float(hh));
        bh[hf] = movmatrix_t(h);
        bl[hf] = movmatrix_t(lw);
      }
      // V^T straight from the int8 values: ldmatrix.trans of 8x8 b16 tiles
      // (b16 = a pair of adjacent dimensions), matrix mi covering positions
      // j*16 + (mi >> 1)*8 .. +7 and dimension pairs hq*16 + (mi & 1)*8 .. +7.
      // Each register splits into an even-dimension and an odd-dimension A
      // fragment: m-tile 2hq + par has row g = dimension hq*32 + 2g + par and
      // row g + 8 = dimension hq*32 + 16 + 2g + par.
      const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
      for (int hq = 0; hq < VH / 32; ++hq) {
        uint32_t vr[4], ae[4], ao[4];
        ldsm_x4_trans(vr, W.v[buf] + (j * 16 + (mi >> 1) * 8 + ri) * VH + hq * 32 + (mi & 1) * 16);
#pragma unroll
        for (int k = 0; k < 4; ++k) i8pairs_to_h2(vr[k], &ae[k], &ao[k]);
        mma_f16_k16(o[2 * hq], ae, bh[0], bh[1]);
        mma_f16_k16(o[2 * hq], ae, bl[0], bl[1]);
        mma_f16_k16(o[2 * hq + 1], ao, bh[0], bh[1]);
        mma_f16_k16(o[2 * hq + 1], ao, bl[0], bl[1]);
      }
    }
    __syncwarp();  // before a later block overwrites this buffer
  }
  if (failed) {
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
  }
  if (bulk && lane == 0) {  // the barriers' memory is reused by the merge below
#pragma unroll
    for (int i = 0; i < NBUF; ++i)
      asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(&W.bar[i])) : "memory");
  }
  // Sum each head's share over the 8 lanes holding it.
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    l[e] += __shfl_xor_sync(0xffffffffu, l[e], 4);
    l[e] += __shfl_xor_sync(0xffffffffu, l[e], 8);
    l[e] += __shfl_xor_sync(0xffffffffu, l[e], 16);
  }

  // ---- merge the four warps (shared memory reused)
  __syncthreads();
  float* Wm = reinterpret_cast<float*>(smraw);  // [4][8]
  float* Wl = Wm + 32;                           // [4][8]
  float* Wo = Wl + 32;                           // [4][8][VH]
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int h = 2 * t + e;
    if (h >= rep) continue;
    if (g == 0) {
      Wm[wid * 8 + h] = m[e];
      Wl[wid * 8 + h] = l[e];
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int d0 = (mt >> 1) * 32 + 2 * g + (mt & 1);  // dimension of row g (row g + 8: d0 + 16)
      Wo[(wid * 8 + h) * VH + d0] = o[mt][e];
      Wo[(wid * 8 + h) * VH + d0 + 16] = o[mt][2 + e];
    }
  }
  __syncthreads();
  const int pwid = rep * (VH + 2);
  float* C = Wo + 4 * 8 * VH;  // this CTA's partial: rep maxima, rep sums, rep x VH outputs
  for (int i = threadIdx.x; i < pwid; i += blockDim.x) {
    const int h = i < 2 * rep ? i % rep : (i - 2 * rep) / VH;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, Wm[w * 8 + h]);
    float acc = 0.f;
    if (i < rep) {
      acc = M;
    } else if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float mw = Wm[w * 8 + h];
        if (mw == -INFINITY) continue;
        const float f = exp2f(mw - M);
        acc += f * (i < 2 * rep ? Wl[w * 8 + h] : Wo[(w * 8 + h) * VH + (i - 2 * rep) % VH]);
      }
    }
    C[i] = acc;
  }
  __syncthreads();
  float* out = part + (((size_t)r * G.kvh + kh) * nsplit + z) * pwid;
  // The separate attn_finish kernel expects natural-log maxima.
  if (!oh || nsplit > 1)
    for (int i = threadIdx.x; i < pwid; i += blockDim.x)
      out[i] = (!oh && i < rep && C[i] != -INFINITY) ? C[i] * 0.69314718055994531f : C[i];
  if (!oh) return;  // the separate attn_finish kernel combines and rotates
  // ---- finish this (row, KV head): softmax merge over the splits, output
  // gate, rotation of its rep * VH outputs (whole 128-wide groups) into oh.
  const float* ps = C;  // one split: this CTA's partial
  int ns = 1;
  if (nsplit > 1) {
    // The last CTA of the row's KV head to arrive combines all splits.
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      last = atomicAdd(&cnt[(size_t)r * G.kvh + kh], 1) == nsplit - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    ps = part + ((size_t)r * G.kvh + kh) * nsplit * pwid;
    ns = nsplit;
  }
  float* Fw = C + pwid;        // [rep][64] split weights exp(m_z - M)
  float* FL = Fw + rep * 64;   // [rep] 1 / sum
  float* Fo = FL + 8;          // [rep * VH] gated outputs
  if (threadIdx.x < rep) {
    const int h = threadIdx.x;
    float M = -INFINITY;
    for (int zz = 0; zz < ns; ++zz) M = fmaxf(M, ps[zz * pwid + h]);
    float L = 0.f;
    for (int zz = 0; zz < ns; ++zz) {
      const float mz = ps[zz * pwid + h];
      const float wz = mz == -INFINITY ? 0.f : exp2f(mz - M);
      Fw[h * 64 + zz] = wz;
      L += wz * ps[zz * pwid + rep + h];
    }
    FL[h] = 1.0f / L;
  }
  __syncthreads();
  const float* gate = proj + (size_t)r * G.proj_dim + G.qkv_dim + (size_t)kh * rep * VH;
#pragma unroll 3
  for (int i = threadIdx.x; i < rep * VH; i += blockDim.x) {
    const int h = i / VH;
    float acc = 0.f;
    for (int zz = 0; zz < ns; ++zz) acc += Fw[h * 64 + zz] * ps[zz * pwid + 2 * rep + i];
    Fo[i] = acc * FL[h] * sigmoidf_(gate[i]);
  }
  if (nsplit > 1 && threadIdx.x == 0) cnt[(size_t)r * G.kvh + kh] = 0;  // ready for the next launch
  __syncthreads();
  const int opad = (G.o_dim + 127) / 128 * 128;
  float* ohr = oh + (size_t)r * opad + (size_t)kh * rep * VH;
  for (int gg = wid; gg < rep * VH / 128; gg += 4) {
    const float4 v = reinterpret_cast<const float4*>(Fo + gg * 128)[lane];
    float x[4] = {v.x, v.y, v.z, v.w};
    fwht128_warp(x);
    if (so.hi) {  // out_proj's tensor-core operands
      const int g = kh * rep * VH / 128 + gg;
      split_group_store(x, so.hi + (size_t)r * opad + g * 128, so.lo + (size_t)r * opad + g * 128,
                        so.inv + (size_t)r * (opad / 128) + g);
    } else {
      reinterpret_cast<float4*>(ohr + gg * 128)[lane] = make_float4(x[0], x[1], x[2], x[3]);
    }
  }
}

template <int QK, int VH>
static cudaError_t launch_layer_attn_i8(const Geo& G, int li, const RowBatch& rb, int window, int nsplit,
                                        const int8_t* q8, const float* q8s, const void* pk, const void* pv,
                                        const float* pks, const float* pvs, float* part, const float* proj,
                                        float* oh, int* cnt, int* werr, SplitOut so, cudaStream_t st) {
  using WS = MmaWarpSmem<QK, VH>;
  const int rep = G.heads / G.kvh;
  const size_t fin = (size_t)(64 + 4 * 8 * VH + rep * (VH + 2) + rep * 64 + 8 + rep * VH) * sizeof(float);
  const size_t smem = std::max(4 * sizeof(WS), fin);
  auto k = layer_attn_i8_kernel<QK, VH>;
  cudaError_t e = allow_smem((const void*)k, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(rb.M, G.kvh, nsplit);
  return launch_pdl(k, grid, dim3(128), smem, st, G, li, rb, window, nsplit, q8, q8s, pk, pv, pks, pvs, part, proj,
                    oh, cnt, werr, so);
}

bool attn_fuses_finish(const Geo& G, int int8) {
  (void)int8;  // both kernels finish in place
  const int rep = G.heads / G.kvh;
  return (rep * G.vh) % 128 == 0 && rep <= 8;
}

// Attention CTAs a launch aims for: enough to cover the 148 SMs several times.
constexpr int AT_SPLIT_TARGET = 148 * 6;

int attn_nsplit(int rows, int kvh, int max_span) {
  // Split positions until the launch has AT_SPLIT_TARGET CTAs; never more
  // splits than chunks.
  const int target = AT_SPLIT_TARGET;
  int ns = (target + rows * kvh - 1) / (rows * kvh);
  ns = std::max(1, std::min(ns, (max_span + CH - 1) / CH));
  return std::min(ns, 64);
}

size_t attn_part_floats(int rows, int heads, int kvh, int vh, int nsplit) {
  return (size_t)rows * kvh * nsplit * (heads / kvh) * (vh + 2);
}

template <bool INT8, int QK, int VH>
static cudaError_t launch_layer_attn_t(const Geo& G, int li, const RowBatch& rb, int window, int nsplit,
                                       const float* qpost, const void* pk, const void* pv, const float* pks,
                                       const float* pvs, float* part, const float* proj, float* oh, int* cnt,
                                       SplitOut so, cudaStream_t st) {
  const size_t smem = sizeof(AttnSmem<INT8, QK, VH>);
  auto k = layer_attn_kernel<INT8, QK, VH>;
  cudaError_t e = allow_smem((const void*)k, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(rb.M, G.kvh, nsplit);
  return launch_pdl(k, grid, dim3(AT_THREADS), smem, st, G, li, rb, window, nsplit, qpost, pk, pv, pks, pvs, part,
                    proj, oh, cnt, so);
}

cudaError_t launch_attention(const Geo& G, int li, const RowBatch& rb, const LayerParams& lp, int nsplit,
                             const float* qpost, const int8_t* q8, const float* q8s, const void* pk,
                             const void* pv, const float* pks, const float* pvs, float* part,
                             cudaStream_t st, int int8, const float* proj, float* oh, int* cnt, int* werr,
                             SplitOut so) {
  if (rb.M <= 0) return cudaSuccess;
  const int rep = G.heads / G.kvh;
  if (rep > AT_MAXREP || nsplit < 1) return cudaErrorInvalidValue;
  if (int8) {
    if (!q8 || !q8s || !werr) return cudaErrorInvalidValue;
    // With proj, oh and cnt the kernel also finishes (attn_fuses_finish);
    // without them it leaves the partials to attn_finish.
    const bool fuse = proj && oh && cnt && attn_fuses_finish(G, int8) && nsplit <= 64;
    if (!fuse) proj = nullptr, oh = nullptr, cnt = nullptr, so = SplitOut{};
#define NB_ATI(Q, V)                                                                                         \
  return launch_layer_attn_i8<Q, V>(G, li, rb, lp.window, nsplit, q8, q8s, pk, pv, pks, pvs, part, proj, oh, \
                                    cnt, werr, so, st)
    if (G.vh == 64) {
      switch (G.qk) {
        case 16: NB_ATI(16, 64);
        case 32: NB_ATI(32, 64);
        case 48: NB_ATI(48, 64);
        case 64: NB_ATI(64, 64);
      }
    } else if (G.vh == 32) {
      switch (G.qk) {
        case 16: NB_ATI(16, 32);
        case 32: NB_ATI(32, 32);
        case 48: NB_ATI(48, 32);
        case 64: NB_ATI(64, 32);
      }
    }
#undef NB_ATI
    return cudaErrorInvalidValue;
  }
  // With proj, oh and cnt the kernel also finishes (attn_fuses_finish).
  if (!(proj && oh && cnt && attn_fuses_finish(G, int8) && nsplit <= 64))
    proj = nullptr, oh = nullptr, cnt = nullptr, so = SplitOut{};
#define NB_ATT(I8, Q, V)                                                                                          \
  return launch_layer_attn_t<I8, Q, V>(G, li, rb, lp.window, nsplit, qpost, pk, pv, pks, pvs, part, proj, oh, cnt, \
                                       so, st)
  const int key = G.qk * 2;  // f32 KV (int8 KV returned above)
  if (G.vh == 64) {
    switch (key) {
      case 32: NB_ATT(false, 16, 64);
      case 64: NB_ATT(false, 32, 64);
      case 96: NB_ATT(false, 48, 64);
      case 128: NB_ATT(false, 64, 64);
    }
  } else if (G.vh == 32) {
    switch (key) {
      case 32: NB_ATT(false, 16, 32);
      case 64: NB_ATT(false, 32, 32);
      case 96: NB_ATT(false, 48, 32);
      case 128: NB_ATT(false, 64, 32);
    }
  }
#undef NB_ATT
  return cudaErrorInvalidValue;
}

// Merge the split partials of one (row, head): softmax over all positions.
__device__ __forceinline__ float combine_head(const float* __restrict__ part, int nsplit, int rep, int vh,
                                              int hl, int d) {
  const int pw = rep * (vh + 2);
  float M = -INFINITY;
  for (int z = 0; z < nsplit; ++z) M = fmaxf(M, part[z * pw + hl]);
  float L = 0.f, o = 0.f;
  for (int z = 0; z < nsplit; ++z) {
    const float mz = part[z * pw + hl];
    if (mz == -INFINITY) continue;
    const float w = expf(mz - M);
    L += w * part[z * pw + rep + hl];
    o += w * part[z * pw + 2 * rep + hl * vh + d];
  }
  return o / L;
}

// Standalone batched decode attention: B independent
// sessions whose rings use the reference's layout k [slots][kv_heads][qk],
// v [slots][kv_heads][vh], scales [slots][kv_heads], session b at offset
// b * slots * kv_heads * (qk | vh | 1).
template <bool INT8, int QK, int VH>
__global__ void __launch_bounds__(AT_THREADS) attend_step_kernel(const float* __restrict__ q, const void* k,
                                                                 const void* v, const float* ks, const float* vs,
                                                                 int slots, const int* __restrict__ lo,
                                                                 const int* __restrict__ hi, int heads, int kvh,
                                                                 int nsplit, float* __restrict__ part) {
  extern __shared__ __align__(16) unsigned char smraw[];
  auto& S = *reinterpret_cast<AttnSmem<INT8, QK, VH>*>(smraw);
  const int bi = blockIdx.x, kh = blockIdx.y, z = blockIdx.z;
  const int rep = heads / kvh;
  const size_t es = INT8 ? 1 : 4;
  AttnSrc src;
  src.k = (const char*)k + (size_t)bi * slots * kvh * QK * es;
  src.v = (const char*)v + (size_t)bi * slots * kvh * VH * es;
  src.ks = INT8 ? ks + (size_t)bi * slots * kvh : nullptr;
  src.vs = INT8 ? vs + (size_t)bi * slots * kvh : nullptr;
  src.k_row = (long)kvh * QK;
  src.k_head = QK;
  src.v_row = (long)kvh * VH;
  src.v_head = VH;
  src.s_row = kvh;
  src.s_head = 1;
  src.slots = slots;
  src.base = 0;
  int a, b;
  split_range(lo[bi], hi[bi], nsplit, z, &a, &b);
  const int pw = rep * (VH + 2);
  attend_part<INT8, QK, VH>(S, q + (size_t)bi * heads * QK + (size_t)kh * rep * QK, rep, src, kh, a, b,
                            1.0f / sqrtf((float)QK), part + (((size_t)bi * kvh + kh) * nsplit + z) * pw);
}

__global__ void attn_combine_kernel(const float* __restrict__ part, int heads, int kvh, int vh, int nsplit,
                                    float* __restrict__ out) {
  const int bi = blockIdx.x, rep = heads / kvh, pw = rep * (vh + 2);
  for (int o = threadIdx.x; o < heads * vh; o += blockDim.x) {
    const int h = o / vh, d = o % vh, kh = h / rep, hl = h % rep;
    out[(size_t)bi * heads * vh + o] =
        combine_head(part + ((size_t)bi * kvh + kh) * nsplit * pw, nsplit, rep, vh, hl, d);
  }
}

template <bool INT8, int QK, int VH>
static cudaError_t launch_step_t(const float* q, const void* k, const void* v, const float* ks, const float* vs,
                                 int slots, const int* lo, const int* hi, int B, int heads, int kvh, int nsplit,
                                 float* part, cudaStream_t st) {
  const size_t smem = sizeof(AttnSmem<INT8, QK, VH>);
  auto kk = attend_step_kernel<INT8, QK, VH>;
  cudaError_t e = allow_smem((const void*)kk, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(B, kvh, nsplit);
  kk<<<grid, AT_THREADS, smem, st>>>(q, k, v, ks, vs, slots, lo, hi, heads, kvh, nsplit, part);
  return cudaGetLastError();
}

cudaError_t launch_attend_step(const float* q, const void* k, const void* v, const float* ks,
                               const float* vs, int int8, int slots, const int* lo, const int* hi,
                               int B, int heads, int kvh, int qk, int vh, int nsplit, float* part,
                               float* out, cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  if (kvh <= 0 || heads % kvh || heads / kvh > AT_MAXREP || slots <= 0 || nsplit < 1) return cudaErrorInvalidValue;
  cudaError_t e = cudaErrorInvalidValue;
#define NB_STEP(I8, Q, V) \
  e = launch_step_t<I8, Q, V>(q, k, v, ks, vs, slots, lo, hi, B, heads, kvh, nsplit, part, st)
  const int key = qk * 2 + (int8 ? 1 : 0);
  if (vh == 64) {
    if (key == 32) NB_STEP(false, 16, 64);
    else if (key == 33) NB_STEP(true, 16, 64);
    else if (key == 64) NB_STEP(false, 32, 64);
    else if (key == 65) NB_STEP(true, 32, 64);
    else if (key == 96) NB_STEP(false, 48, 64);
    else if (key == 97) NB_STEP(true, 48, 64);
    else if (key == 128) NB_STEP(false, 64, 64);
    else if (key == 129) NB_STEP(true, 64, 64);
  } else if (vh == 32) {
    if (key == 32) NB_STEP(false, 16, 32);
    else if (key == 33) NB_STEP(true, 16, 32);
    else if (key == 64) NB_STEP(false, 32, 32);
    else if (key == 65) NB_STEP(true, 32, 32);
    else if (key == 96) NB_STEP(false, 48, 32);
    else if (key == 97) NB_STEP(true, 48, 32);
    else if (key == 128) NB_STEP(false, 64, 32);
    else if (key == 129) NB_STEP(true, 64, 32);
  }
#undef NB_STEP
  if (e != cudaSuccess) return e;
  attn_combine_kernel<<<B, 256, 0, st>>>(part, heads, kvh, vh, nsplit, out);
  return cudaGetLastError();
}

// quant_into (crates/needle-core/src/v3/cache.rs:100-106) over `rows` vectors of
// `dim` <= 64: one warp per vector, through kv_quant_warp, the same quantiser
// the forward's KV append runs.
__global__ void kv_quant_kernel(const float* __restrict__ x, int rows, int dim, int8_t* __restrict__ q,
                                float* __restrict__ scales) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= rows) return;
  const float* xr = x + (size_t)w * dim;
  const float a = lane < dim ? xr[lane] : 0.f, b = lane + 32 < dim ? xr[lane + 32] : 0.f;
  float ca, cb;
  const float scale = kv_quant_warp(a, b, &ca, &cb);
  if (lane < dim) q[(size_t)w * dim + lane] = (int8_t)ca;
  if (lane + 32 < dim) q[(size_t)w * dim + lane + 32] = (int8_t)cb;
  if (lane == 0) scales[w] = scale;
}

cudaError_t launch_kv_quant(const float* x, int rows, int dim, int8_t* q, float* scales,
                            cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (dim <= 0 || dim > 64) return cudaErrorInvalidValue;
  const int warps = 8;
  kv_quant_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, st>>>(x, rows, dim, q, scales);
  return cudaGetLastError();
}

// Combine of the forward's attention partials, fused with the output gate
// (model.rs:305-308) and the rotation of out_proj's prepare_input.
__global__ void attn_finish_kernel(Geo G, int nsplit, const float* __restrict__ part,
                                   const float* __restrict__ proj, float* __restrict__ oh, SplitOut so) {
  pdl_trigger();  // a PDL-launched projection after this kernel may start its weight prefetch
  pdl_wait();     // everything below reads or writes what earlier kernels touch
  extern __shared__ __align__(16) float sm[];
  __shared__ float wsm[8][64];  // per-warp split weights (nsplit <= 64)
  const int r = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int od = G.o_dim, opad = (od + 127) / 128 * 128, rep = G.heads / G.kvh, pw = rep * (G.vh + 2);
  const float* gate = proj + (size_t)r * G.proj_dim + G.qkv_dim;
  // One warp per head: the split weights exp(m_z - M) and 1/L are formed once
  // per head (lanes over splits), then each lane merges its value dimensions.
  for (int h = wid; h < G.heads; h += nw) {
    const int kh = h / rep, hl = h % rep;
    const float* base = part + ((size_t)r * G.kvh + kh) * nsplit * pw;
    float M = -INFINITY;
    for (int z = lane; z < nsplit; z += 32) M = fmaxf(M, base[z * pw + hl]);
    M = warp_max(M);
    float L = 0.f;
    for (int z = lane; z < nsplit; z += 32) {
      const float mz = base[z * pw + hl];
      const float wz = mz == -INFINITY ? 0.f : expf(mz - M);  // split weight
      wsm[wid][z] = wz;
      L += wz * base[z * pw + rep + hl];
    }
    L = warp_sum(L);
    __syncwarp();
#pragma unroll 2
    for (int dd = lane; dd < G.vh; dd += 32) {
      float o = 0.f;
#pragma unroll 4
      for (int z = 0; z < nsplit; ++z) o += wsm[wid][z] * base[z * pw + 2 * rep + hl * G.vh + dd];
      const int i = h * G.vh + dd;
      sm[i] = o / L * sigmoidf_(gate[i]);
    }
    __syncwarp();
  }
  for (int i = od + threadIdx.x; i < opad; i += blockDim.x) sm[i] = 0.f;
  __syncthreads();
  if (so.hi) {  // rotation and out_proj's tensor-core operands, one warp per group
    for (int g = wid; g < opad / 128; g += nw) {
      const float4 v = reinterpret_cast<const float4*>(sm + g * 128)[lane];
      float x[4] = {v.x, v.y, v.z, v.w};
      fwht128_warp(x);
      split_group_store(x, so.hi + (size_t)r * opad + g * 128, so.lo + (size_t)r * opad + g * 128,
                        so.inv + (size_t)r * (opad / 128) + g);
    }
    return;
  }
  fwht_groups_warp(sm, opad / 128);
  __syncthreads();
  for (int i = threadIdx.x; i < opad; i += blockDim.x) oh[(size_t)r * opad + i] = sm[i];
}

cudaError_t launch_attn_finish(const Geo& G, const RowBatch& rb, int nsplit, const float* part,
                               const float* proj, float* oh, cudaStream_t st, SplitOut so) {
  if (rb.M <= 0) return cudaSuccess;
  const int opad = (G.o_dim + 127) / 128 * 128;
  if (nsplit > 64) return cudaErrorInvalidValue;  // the kernel's split-weight buffer
  return launch_pdl(attn_finish_kernel, dim3(rb.M), dim3(256), opad * sizeof(float), st, G, nsplit, part, proj, oh,
                    so);
}


// ---------------------------------------------------------------------------
// Allocation-free form of the standalone decode attention.
//
// Some callers cannot allocate device memory at all: a serving runtime that has
// reserved the GPU's memory for its own pool up front (so a cudaMalloc or
// cudaMallocAsync from inside a plugin fails, or fragments that pool), or code
// on a latency-critical path that must not make any allocation call. For them
// nd_attend_step_noalloc keeps the split partials in a fixed array compiled
// into this library instead of allocating them per call.
//
// The array holds NB_NOALLOC_SCRATCH_FLOATS floats (4 MiB). Every GPU that loads
// the library holds it until the process exits. All calls on a device share it
// and it keeps the last call's contents; each call overwrites every partial it
// later reads, so nothing has to start at zero. Calls whose kernels overlap on
// the GPU (different streams, or graphs replayed concurrently) race on the
// array: serialise them.
constexpr size_t NB_NOALLOC_SCRATCH_FLOATS = (size_t)1 << 20;
static __device__ __align__(256) float g_attn_noalloc_scratch[NB_NOALLOC_SCRATCH_FLOATS];

// attn_nsplit splits positions only while B * kv_heads < AT_SPLIT_TARGET, so a
// request with more than one split has B * kv_heads * splits < 2 *
// AT_SPLIT_TARGET rows of partials; with at most AT_MAXREP query heads per KV
// head and value heads of at most 64 floats those always fit the array. Only a
// single-split request (B * kv_heads >= AT_SPLIT_TARGET) can be too large.
static_assert((size_t)2 * AT_SPLIT_TARGET * AT_MAXREP * (64 + 2) <= NB_NOALLOC_SCRATCH_FLOATS,
              "split requests of nd_attend_step_noalloc must fit the fixed scratch");

namespace {
std::mutex g_noalloc_mu;
// Device address of the array per device ordinal, and the context it was
// looked up in.
struct NoallocSlot {
  CUcontext ctx;
  float* ptr;
};
NoallocSlot g_noalloc[256] = {};

PFN_cuCtxGetCurrent_v4000 ctx_get_current() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  });
  return fn;
}

// In host code the array's name stands for a host-side shadow, not a device
// address. The device address is looked up with that device current, once per
// device, and again when the device's context has changed since (a
// cudaDeviceReset reloads the module, which may move the array).
cudaError_t noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 256) return cudaErrorInvalidDevice;
  auto get_ctx = ctx_get_current();
  if (!get_ctx) return cudaErrorNotSupported;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return cudaErrorInvalidDevice;
  NoallocSlot& slot = g_noalloc[dev];
  if (!slot.ptr || !ctx || slot.ctx != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);  // also makes the primary context current
    if (e != cudaSuccess) return e;
    if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx) return cudaErrorInvalidDevice;
    slot.ctx = ctx;
    slot.ptr = static_cast<float*>(p);
  }
  *out = slot.ptr;
  return cudaSuccess;
}
}  // namespace

}  // namespace nb

extern "C" int nd_attend_step_noalloc(const float* q, const void* k, const void* v, const float* ks,
                                      const float* vs, int int8, int slots, const int* lo, const int* hi,
                                      int B, int heads, int kv_heads, int qk, int vh, float* out,
                                      void* stream) {
  using namespace nb;
  if (!q || !k || !v || !lo || !hi || !out || (int8 && (!ks || !vs)) || kv_heads <= 0 || heads % kv_heads ||
      heads / kv_heads > AT_MAXREP || slots <= 0 || (vh != 32 && vh != 64)) {
    nd_record_error(cudaErrorInvalidValue, "nd_attend_step_noalloc: invalid argument");
    return (int)cudaErrorInvalidValue;
  }
  if (B <= 0) return 0;
  // The split count of nd_attend_step; only a single-split request can exceed
  // the array (see the static_assert above).
  const int ns = attn_nsplit(B, kv_heads, slots);
  if (attn_part_floats(B, heads, kv_heads, vh, ns) > NB_NOALLOC_SCRATCH_FLOATS) {
    nd_record_error(cudaErrorInvalidValue,
                    "nd_attend_step_noalloc: B * heads * (v_head_dim + 2) floats exceed the fixed 4 MiB "
                    "scratch (1048576 floats); use nd_attend_step or a smaller batch");
    return (int)cudaErrorInvalidValue;
  }
  float* part = nullptr;
  cudaError_t e = noalloc_scratch(&part);
  if (e == cudaSuccess)
    e = launch_attend_step(q, k, v, ks, vs, int8, slots, lo, hi, B, heads, kv_heads, qk, vh, ns, part, out,
                           (cudaStream_t)stream);
  if (e != cudaSuccess) {
    nd_record_error(e, nullptr);
    return (int)e;
  }
  return 0;
}
