// Grouped-query attention over the KV cache, f32 or int8.
//
// Restates attend_step_with (crates/needle-core/src/v3/attention.rs:327-377)
// for decode rows and attend_with (:241-287) for prefill rows: GQA with
// kv_head = h / repeat, scale 1/sqrt(qk_head_dim), softmax with max
// subtraction, then P.V. The int8 reader follows Int8View (:191-216): the
// per-(position, kv head) key scale multiplies the integer-valued dot and the
// value scale multiplies the softmax weight. The softmax runs online over
// tiles of positions (one CTA per (row, kv head)), so sums are reassociated
// relative to the reference's two-pass loop; the result agrees to f32 rounding.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.hpp"
#include "launch_util.hpp"

namespace nb {

constexpr int AT_TILE = 128;
constexpr int AT_MAXREP = 8;

// Where keys/values of one (row, kv head) live. Element (position n, kv head
// kh) of keys is at k + idx(n) * k_row + kh * k_head (in elements), with
// idx(n) = n % slots for a ring and base + n for the prefill scratch.
struct AttnSrc {
  const void* k;
  const void* v;
  const float* ks;
  const float* vs;
  long k_row, k_head, v_row, v_head, s_row, s_head;
  int slots;  // > 0: ring; 0: linear from `base`
  int base;
};

template <bool INT8, int QK>
__device__ void attend_core(const float* qs, int rep, int vh, const AttnSrc& src, int kh,
                            int lo, int hi, float scale, float* __restrict__ out, float* sm) {
  float* S = sm;                          // [rep][AT_TILE]
  float* Vs = S + AT_MAXREP * AT_TILE;    // [AT_TILE][vh]
  float* vsc = Vs + AT_TILE * vh;         // [AT_TILE]
  float* mrun = vsc + AT_TILE;            // [AT_MAXREP]
  float* lrun = mrun + AT_MAXREP;
  float* cr = lrun + AT_MAXREP;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  if (tid < AT_MAXREP) {
    mrun[tid] = -INFINITY;
    lrun[tid] = 0.f;
  }
  const int nout = rep * vh;
  float acc0 = 0.f, acc1 = 0.f;  // outputs tid and tid + blockDim.x
  const int hsplit = (rep + 1) / 2;
  for (int n0 = lo; n0 <= hi; n0 += AT_TILE) {
    __syncthreads();
    // ---- scores: position n0 + (tid % TILE); head half tid / TILE.
    {
      const int t = tid % AT_TILE, half = tid / AT_TILE;
      const int n = n0 + t;
      const int h0 = half * hsplit, h1 = min(rep, h0 + hsplit);
      if (n <= hi) {
        const long idx = src.slots > 0 ? (long)(n % src.slots) : (long)(src.base + n);
        float kv[QK];
        if (INT8) {
          const int8_t* kp = (const int8_t*)src.k + idx * src.k_row + kh * src.k_head;
#pragma unroll
          for (int i = 0; i < QK; i += 16) {
            int4 w = *reinterpret_cast<const int4*>(kp + i);
            const int8_t* b = reinterpret_cast<const int8_t*>(&w);
#pragma unroll
            for (int j = 0; j < 16; ++j) kv[i + j] = (float)b[j];
          }
        } else {
          const float* kp = (const float*)src.k + idx * src.k_row + kh * src.k_head;
#pragma unroll
          for (int i = 0; i < QK; i += 4) {
            float4 w = *reinterpret_cast<const float4*>(kp + i);
            kv[i] = w.x;
            kv[i + 1] = w.y;
            kv[i + 2] = w.z;
            kv[i + 3] = w.w;
          }
        }
        const float ksc = INT8 ? src.ks[idx * src.s_row + kh * src.s_head] : 1.0f;
        for (int h = h0; h < h1; ++h) {
          float a = 0.f;
#pragma unroll
          for (int i = 0; i < QK; ++i) a += qs[h * QK + i] * kv[i];
          if (INT8) a = a * ksc;
          S[h * AT_TILE + t] = a * scale;
        }
      } else {
        for (int h = h0; h < h1; ++h) S[h * AT_TILE + t] = -INFINITY;
      }
    }
    // ---- value tile
    for (int e = tid; e < AT_TILE * vh; e += blockDim.x) {
      const int t = e / vh, dd = e % vh;
      const int n = n0 + t;
      float val = 0.f;
      if (n <= hi) {
        const long idx = src.slots > 0 ? (long)(n % src.slots) : (long)(src.base + n);
        if (INT8)
          val = (float)((const int8_t*)src.v)[idx * src.v_row + kh * src.v_head + dd];
        else
          val = ((const float*)src.v)[idx * src.v_row + kh * src.v_head + dd];
        if (INT8 && dd == 0) vsc[t] = src.vs[idx * src.s_row + kh * src.s_head];
      } else if (dd == 0) {
        vsc[t] = 0.f;
      }
      Vs[e] = val;
    }
    __syncthreads();
    // ---- online softmax update per head
    for (int h = wid; h < rep; h += nw) {
      float mx = -INFINITY;
      for (int t = lane; t < AT_TILE; t += 32) mx = fmaxf(mx, S[h * AT_TILE + t]);
      mx = warp_max(mx);
      const float mold = mrun[h];
      const float mnew = fmaxf(mold, mx);
      float sum = 0.f;
      for (int t = lane; t < AT_TILE; t += 32) {
        float s = S[h * AT_TILE + t];
        float pv = s == -INFINITY ? 0.f : expf(s - mnew);
        S[h * AT_TILE + t] = pv;
        sum += pv;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float c = mold == -INFINITY ? 0.f : expf(mold - mnew);
        cr[h] = c;
        lrun[h] = lrun[h] * c + sum;
        mrun[h] = mnew;
      }
    }
    __syncthreads();
    // ---- P.V
#pragma unroll
    for (int rep2 = 0; rep2 < 2; ++rep2) {
      const int o = tid + rep2 * blockDim.x;
      if (o < nout) {
        const int h = o / vh, dd = o % vh;
        float a = 0.f;
        const float* P = S + h * AT_TILE;
        if (INT8) {
          for (int t = 0; t < AT_TILE; ++t) a += (P[t] * vsc[t]) * Vs[t * vh + dd];
        } else {
          for (int t = 0; t < AT_TILE; ++t) a += P[t] * Vs[t * vh + dd];
        }
        if (rep2 == 0)
          acc0 = acc0 * cr[h] + a;
        else
          acc1 = acc1 * cr[h] + a;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int rep2 = 0; rep2 < 2; ++rep2) {
    const int o = tid + rep2 * blockDim.x;
    if (o < nout) {
      const int h = o / vh;
      out[o] = (rep2 == 0 ? acc0 : acc1) / lrun[h];
    }
  }
}

static size_t attn_smem(int vh) {
  return (size_t)(AT_MAXREP * AT_TILE + AT_TILE * vh + AT_TILE + 3 * AT_MAXREP + AT_MAXREP * 64) * sizeof(float);
}

// Forward-pass attention: one CTA per (row, kv head).
template <bool INT8, int QK>
__global__ void __launch_bounds__(256) layer_attn_kernel(Geo G, int li, RowBatch rb, int window,
                                                         const float* __restrict__ qpost,
                                                         const void* pk, const void* pv,
                                                         const float* pks, const float* pvs,
                                                         float* __restrict__ attn) {
  extern __shared__ __align__(16) float sm[];
  const int r = blockIdx.x, kh = blockIdx.y;
  const int rep = G.heads / G.kvh;
  const RowInfo ri = rb.rows[r];
  const int p = ri.pos;
  float* qs = sm;  // [rep][qk]
  float* rest = sm + AT_MAXREP * 64;
  for (int i = threadIdx.x; i < rep * G.qk; i += blockDim.x)
    qs[i] = qpost[(size_t)r * G.q_dim + (size_t)kh * rep * G.qk + i];
  int lo = (window > 0 && p + 1 > window) ? p + 1 - window : 0;
  AttnSrc src;
  if (rb.mode == MODE_PREFILL) {
    src.k = pk;
    src.v = pv;
    src.ks = pks;
    src.vs = pvs;
    src.k_row = (long)G.kvh * G.qk;
    src.k_head = G.qk;
    src.v_row = (long)G.kvh * G.vh;
    src.v_head = G.vh;
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
    src.k_row = G.qk;
    src.k_head = (long)kv.slots * G.qk;
    src.v_row = G.vh;
    src.v_head = (long)kv.slots * G.vh;
    src.s_row = 1;
    src.s_head = kv.slots;
    src.slots = kv.slots;
    src.base = 0;
    const int floor = p + 1 > kv.slots ? p + 1 - kv.slots : 0;  // cache.rs:322-331
    lo = max(lo, floor);
  }
  __syncthreads();
  const float scale = 1.0f / sqrtf((float)G.qk);
  attend_core<INT8, QK>(qs, rep, G.vh, src, kh, lo, p, scale,
                    attn + (size_t)r * G.o_dim + (size_t)kh * rep * G.vh, rest);
}

cudaError_t launch_attention(const Geo& G, int li, const RowBatch& rb, const LayerParams& lp,
                             const float* qpost, const void* pk, const void* pv, const float* pks,
                             const float* pvs, float* attn, cudaStream_t st, int int8) {
  if (rb.M <= 0) return cudaSuccess;
  const int rep = G.heads / G.kvh;
  if (rep > AT_MAXREP || G.qk > 64 || G.vh > 64 || G.qk % 16 || rep * G.vh > 512)
    return cudaErrorInvalidValue;
  const size_t smem = attn_smem(G.vh);
  dim3 grid(rb.M, G.kvh);
#define NB_ATTN_LAUNCH(I8, Q)                                                                   \
  {                                                                                            \
    auto k = layer_attn_kernel<I8, Q>;                                                         \
    cudaError_t e = allow_smem((const void*)k, smem);                                         \
    if (e != cudaSuccess) return e;                                                            \
    k<<<grid, 256, smem, st>>>(G, li, rb, lp.window, qpost, pk, pv, pks, pvs, attn);           \
  }
  switch (G.qk * 2 + (int8 ? 1 : 0)) {
    case 32: NB_ATTN_LAUNCH(false, 16) break;
    case 33: NB_ATTN_LAUNCH(true, 16) break;
    case 64: NB_ATTN_LAUNCH(false, 32) break;
    case 65: NB_ATTN_LAUNCH(true, 32) break;
    case 96: NB_ATTN_LAUNCH(false, 48) break;
    case 97: NB_ATTN_LAUNCH(true, 48) break;
    case 128: NB_ATTN_LAUNCH(false, 64) break;
    case 129: NB_ATTN_LAUNCH(true, 64) break;
    default: return cudaErrorInvalidValue;
  }
#undef NB_ATTN_LAUNCH
  return cudaGetLastError();
}

// Standalone batched decode attention: B independent
// sessions whose rings use the reference's layout k [slots][kv_heads][qk],
// v [slots][kv_heads][vh], scales [slots][kv_heads], session b at offset
// b * slots * kv_heads * (qk | vh | 1).
template <bool INT8, int QK>
__global__ void __launch_bounds__(256) attend_step_kernel(const float* __restrict__ q, const void* k,
                                                          const void* v, const float* ks,
                                                          const float* vs, int slots,
                                                          const int* __restrict__ lo,
                                                          const int* __restrict__ hi, int heads,
                                                          int kvh, int qk, int vh,
                                                          float* __restrict__ out) {
  extern __shared__ __align__(16) float sm[];
  const int b = blockIdx.x, kh = blockIdx.y;
  const int rep = heads / kvh;
  float* qs = sm;
  float* rest = sm + AT_MAXREP * 64;
  for (int i = threadIdx.x; i < rep * qk; i += blockDim.x)
    qs[i] = q[(size_t)b * heads * qk + (size_t)kh * rep * qk + i];
  AttnSrc src;
  const size_t esz = INT8 ? 1 : 4;
  src.k = (const char*)k + (size_t)b * slots * kvh * qk * esz;
  src.v = (const char*)v + (size_t)b * slots * kvh * vh * esz;
  src.ks = INT8 ? ks + (size_t)b * slots * kvh : nullptr;
  src.vs = INT8 ? vs + (size_t)b * slots * kvh : nullptr;
  src.k_row = (long)kvh * qk;
  src.k_head = qk;
  src.v_row = (long)kvh * vh;
  src.v_head = vh;
  src.s_row = kvh;
  src.s_head = 1;
  src.slots = slots;
  src.base = 0;
  __syncthreads();
  attend_core<INT8, QK>(qs, rep, vh, src, kh, lo[b], hi[b], 1.0f / sqrtf((float)qk),
                    out + (size_t)b * heads * vh + (size_t)kh * rep * vh, rest);
}

cudaError_t launch_attend_step(const float* q, const void* k, const void* v, const float* ks,
                               const float* vs, int int8, int slots, const int* lo, const int* hi,
                               int B, int heads, int kvh, int qk, int vh, float* out,
                               cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  if (kvh <= 0 || heads % kvh) return cudaErrorInvalidValue;
  const int rep = heads / kvh;
  if (rep > AT_MAXREP || qk > 64 || vh > 64 || qk % 16 || rep * vh > 512 || slots <= 0)
    return cudaErrorInvalidValue;
  const size_t smem = attn_smem(vh);
  dim3 grid(B, kvh);
#define NB_STEP_LAUNCH(I8, Q)                                                                   \
  {                                                                                            \
    auto kk = attend_step_kernel<I8, Q>;                                                       \
    cudaError_t e = allow_smem((const void*)kk, smem);                                        \
    if (e != cudaSuccess) return e;                                                            \
    kk<<<grid, 256, smem, st>>>(q, k, v, ks, vs, slots, lo, hi, heads, kvh, qk, vh, out);      \
  }
  switch (qk * 2 + (int8 ? 1 : 0)) {
    case 32: NB_STEP_LAUNCH(false, 16) break;
    case 33: NB_STEP_LAUNCH(true, 16) break;
    case 64: NB_STEP_LAUNCH(false, 32) break;
    case 65: NB_STEP_LAUNCH(true, 32) break;
    case 96: NB_STEP_LAUNCH(false, 48) break;
    case 97: NB_STEP_LAUNCH(true, 48) break;
    case 128: NB_STEP_LAUNCH(false, 64) break;
    case 129: NB_STEP_LAUNCH(true, 64) break;
    default: return cudaErrorInvalidValue;
  }
#undef NB_STEP_LAUNCH
  return cudaGetLastError();
}

// quant_into (crates/needle-core/src/v3/cache.rs:100-106) over `rows` head
// vectors of `dim` <= 64: one warp per vector. Bit-exact: IEEE division for
// the scale and its reciprocal, roundf half away from zero, clamp [-128, 127].
__global__ void kv_quant_kernel(const float* __restrict__ x, int rows, int dim, int8_t* __restrict__ q,
                                float* __restrict__ scales) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= rows) return;
  const float* xr = x + (size_t)w * dim;
  float a = lane < dim ? xr[lane] : 0.f, b = lane + 32 < dim ? xr[lane + 32] : 0.f;
  float am = warp_max(fmaxf(fabsf(a), fabsf(b)));
  float scale = am > 0.0f ? __fdiv_rn(am, 127.0f) : 1.0f;
  float inv = __fdiv_rn(1.0f, scale);
  if (lane < dim) q[(size_t)w * dim + lane] = (int8_t)fminf(fmaxf(roundf(__fmul_rn(a, inv)), -128.f), 127.f);
  if (lane + 32 < dim)
    q[(size_t)w * dim + lane + 32] = (int8_t)fminf(fmaxf(roundf(__fmul_rn(b, inv)), -128.f), 127.f);
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

}  // namespace nb
