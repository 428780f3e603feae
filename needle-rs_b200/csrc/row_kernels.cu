// Per-row kernels of the Needle-3 forward: one CTA per activation row, where a
// row is one (session, position) pair, so the same kernels serve batch-1
// decode, batched multi-session decode and whole-prompt prefill.
//
// Each kernel cites the reference function it restates. Reductions run as
// warp/block trees instead of the reference's sequential sums, so results
// match the CPU path to f32 rounding rather than bit for bit; the integer work
// (index unpacking, Engram hashing, int8 quantisation) is exact.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.hpp"
#include "launch_util.hpp"

namespace nb {

constexpr float EPS = 1e-6f;  // crates/needle-core/src/kernels.rs:11, norm.rs:6

// Decode one 128-element quantisation group of a CQ row into `out`
// (levels[idx] * norm, cq.rs:791-809); each lane writes elements lane*4..+3.
// `lev` is the tensor's level table in shared memory.
__device__ __forceinline__ void decode_group_lane(const CqMat& W, const float* lev, const uint8_t* row,
                                                  float norm, int g, float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  const int bits = W.bits, mask = (1 << bits) - 1;
  const uint32_t c = cq_quad_codes(row, bits, g, lane);
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = lev[(c >> (i * bits)) & mask] * norm;
}

__device__ __forceinline__ void load_levels(const CqMat& W, float* lev) {
  if (threadIdx.x < 16) lev[threadIdx.x] = W.levels[threadIdx.x];
  __syncthreads();
}

// ---------------------------------------------------------------- embedding
// model.rs:196-203: dequantize_row (levels*norm, inverse rotation) then
// * sqrt(d_model), broadcast into every mHC lane.
__global__ void embed_kernel(Geo G, CqMat emb, RowBatch rb, float* __restrict__ lanes) {
  pdl_wait();
  pdl_trigger();
  __shared__ float lev[16];
  load_levels(emb, lev);
  const int r = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t tok = rb.tokens[r];
  if (tok > (uint32_t)(G.vocab - 1)) tok = G.vocab - 1;  // clamp_token, model.rs:533
  const uint8_t* row = emb.seg[0].packed + (size_t)tok * emb.row_bytes;
  const __half* nrm = emb.seg[0].norms + (size_t)tok * emb.groups;
  float* out = lanes + (size_t)r * G.lanes * G.d;
  for (int g = wid; g < emb.groups; g += nw) {
    float v[4];
    decode_group_lane(emb, lev, row, __half2float(nrm[g]), g, v);
    fwht128_warp(v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int c = g * 128 + lane * 4 + i;
      if (c < G.d) {
        float x = v[i] * G.embed_scale;
        for (int l = 0; l < G.lanes; ++l) out[l * G.d + c] = x;
      }
    }
  }
}

cudaError_t launch_embed(const Geo& G, const CqMat& emb, const RowBatch& rb, float* lanes,
                         cudaStream_t st) {
  if (rb.M <= 0) return cudaSuccess;
  return launch_pdl(embed_kernel, dim3(rb.M), dim3(256), 0, st, G, emb, rb, lanes);
}

// ---------------------------------------------------------------- Engram
// engram.rs:31-61 (hash) and :66-69 (validity), model.rs:158-191 / :420-471
// (gather). The fetched row feeds key/value projections whose prepare_input
// rotates it again; the rotation is an involution, so the projection input is
// the decoded codes levels[idx]*norm directly and both rotations are skipped.
// One CTA per row, one warp per table (an order's hash head): the slot
// depends on the tokens and the table only, not on the site, so it is hashed
// once and the row of that slot is fetched from every site's table, EG_SITES
// sites' loads in flight together.
constexpr int EG_SITES = 8;
__global__ void __launch_bounds__(256) engram_gather_kernel(Geo G, const CqMat* __restrict__ tables, RowBatch rb,
                                                            float* __restrict__ fetched, SplitOut so) {
  pdl_trigger();  // a PDL-launched projection after this kernel may start its weight prefetch
  __shared__ float lev[16][16];
  for (int i = threadIdx.x; i < G.n_sites * 16; i += blockDim.x) lev[i >> 4][i & 15] = tables[i >> 4].levels[i & 15];
  pdl_wait();  // everything below reads or writes what earlier kernels touch
  const int r = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const RowInfo ri = rb.rows[r];
  const int p = ri.pos;
  __syncthreads();
  for (int t = wid; t < G.e_tables; t += nw) {
    const int oi = t / G.e_heads, h = t % G.e_heads;
    const int order = G.orders[oi];
    const bool valid = p + 1 >= order;  // ngram_valid
    uint32_t slot = 0;
    if (valid) {
      uint32_t acc = 0x9E3779B9u * (uint32_t)(oi * G.e_stride + h + 1);
      for (int j = 0; j < order; ++j) {
        uint32_t tok;
        if (j > p)
          tok = 0;
        else if (j == 0)
          tok = rb.tokens[r];
        else if (rb.mode == MODE_PREFILL)
          tok = rb.tokens[r - j];
        else
          tok = ri.s->toks[(p - j) & 3];
        acc = (acc ^ tok) * 0x01000193u;
      }
      acc ^= acc >> 15;
      slot = acc % (uint32_t)G.e_slots;
    }
    const size_t trow = (size_t)t * G.e_slots + slot;
    for (int s0 = 0; s0 < G.n_sites; s0 += EG_SITES) {
      uint32_t code[EG_SITES];
      float nrm[EG_SITES];
#pragma unroll
      for (int k = 0; k < EG_SITES; ++k) {
        code[k] = 0;
        nrm[k] = 0.f;
        const int site = s0 + k;
        if (!valid || site >= G.n_sites) continue;
        const CqMat& T = tables[site];
        code[k] = cq_quad_codes(T.seg[0].packed + trow * T.row_bytes, T.bits, 0, lane);
        nrm[k] = __half2float(T.seg[0].norms[trow * T.groups]);
      }
#pragma unroll
      for (int k = 0; k < EG_SITES; ++k) {
        const int site = s0 + k;
        if (site >= G.n_sites) break;
        const int bits = tables[site].bits, mask = (1 << bits) - 1;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = valid ? lev[site][(code[k] >> (i * bits)) & mask] * nrm[k] : 0.f;
        if (so.hi) {  // table t is the 128-wide group t of the site's projection input
          const size_t e0 = ((size_t)site * rb.M + r) * G.d + t * 128;
          split_group_store(v, so.hi + e0, so.lo + e0, so.inv + ((size_t)site * rb.M + r) * (G.d / 128) + t);
        } else {
          float* out = fetched + ((size_t)r * G.n_sites + site) * G.d;
          reinterpret_cast<float4*>(out + t * 128)[lane] = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
    }
  }
}

cudaError_t launch_engram_gather(const Geo& G, const CqMat* tables, const RowBatch& rb,
                                 float* fetched, cudaStream_t st, SplitOut so) {
  if (rb.M <= 0 || G.n_sites == 0) return cudaSuccess;
  if (G.n_sites > 16) return cudaErrorInvalidValue;
  const int warps = std::min(8, std::max(1, G.e_tables));
  return launch_pdl(engram_gather_kernel, dim3(rb.M), dim3(warps * 32), 0, st, G, tables, rb, fetched, so);
}

// value_conv (engram.rs:89-106) / engram_conv_step (cache.rs:444-479): dilated
// causal conv of the raw Engram values, gated until p >= j*max_order. Prefill
// rows read earlier raw values from the batch and seed the tail ring with the
// last `reach` raw rows; decode rows read the ring and then overwrite the slot
// of p-reach with this position's raw value.
struct EngTaps {
  const float* t[16];
};

// One CTA per row covering every site, four channels per thread-step (the
// row descriptor and the session's tail pointer are read once per row).
__global__ void __launch_bounds__(256, 5) engram_conv_kernel(Geo G, EngTaps taps, RowBatch rb, const float* __restrict__ ekv,
                                   float* __restrict__ evc) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const RowInfo ri = rb.rows[r];
  const int p = ri.pos, reach = G.e_reach, d = G.d, d4 = d / 4;
  const size_t kv_ld = (size_t)G.n_sites * 2 * d;
  float* tails = ri.s->eng_tail;
  const bool seed = reach > 0 && (rb.mode == MODE_DECODE || p >= ri.len - reach);
  const float* row_kv = ekv + (size_t)r * kv_ld;
  for (int i = threadIdx.x; i < G.n_sites * d4; i += blockDim.x) {
    const int site = i / d4, c = (i % d4) * 4;
    // Selected by compares, not indexed: a dynamic index into the parameter
    // array would copy it to local memory in every thread.
    const float* tp = taps.t[0];
#pragma unroll
    for (int k = 1; k < 16; ++k)
      if (k == site) tp = taps.t[k];
    const float4 raw = *reinterpret_cast<const float4*>(row_kv + (size_t)site * 2 * d + d + c);
    float* tail = tails + (size_t)site * reach * d;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < G.e_taps; ++j) {
      const int back = j * G.e_dil;
      if (back > p || p < j * G.e_maxorder) continue;
      float4 val;
      if (back == 0)
        val = raw;
      else if (rb.mode == MODE_PREFILL)
        val = *reinterpret_cast<const float4*>(ekv + (size_t)(r - back) * kv_ld + (size_t)site * 2 * d + d + c);
      else
        val = *reinterpret_cast<const float4*>(tail + (size_t)((p - back) % reach) * d + c);
      const float4 t = *reinterpret_cast<const float4*>(tp + (size_t)j * d + c);
      acc.x += t.x * val.x;
      acc.y += t.y * val.y;
      acc.z += t.z * val.z;
      acc.w += t.w * val.w;
    }
    *reinterpret_cast<float4*>(evc + ((size_t)r * G.n_sites + site) * d + c) = acc;
    // The slot written here is the one tap j = reach / dil read above (same
    // thread, same channels), so the read comes first.
    if (seed) *reinterpret_cast<float4*>(tail + (size_t)(p % reach) * d + c) = raw;
  }
}

cudaError_t launch_engram_conv(const Geo& G, const float* const* taps, const RowBatch& rb,
                               const float* ekv, float* evc, cudaStream_t st) {
  if (rb.M <= 0 || G.n_sites == 0) return cudaSuccess;
  if (G.n_sites > 16) return cudaErrorInvalidValue;
  EngTaps t;
  for (int i = 0; i < G.n_sites; ++i) t.t[i] = taps[i];
  if (G.d % 4) return cudaErrorInvalidValue;
  return launch_pdl(engram_conv_kernel, dim3(rb.M), dim3(256), 0, st, G, t, rb, ekv, evc);
}

// ---------------------------------------------------------------- mHC pre
// Sinkhorn (kernels.rs:46-85) in the log domain on an n x n matrix held one
// element per lane (n in {1, 2, 4}); rows are lane groups of n, columns lanes
// with stride n. The 20 dependent log-sum-exp rounds use the hardware
// exponential and logarithm (__expf/__logf, ~1e-6 relative).
// Two independent matrices per warp, one per 16-lane half (lanes 16.. hold the
// second); the shuffle distances (< n * n <= 16) stay inside a half.
__device__ __forceinline__ float sinkhorn_half_fast(float m, int n) {
  const int hl = threadIdx.x & 15;
  const bool in = hl < n * n;
  for (int it = 0; it < 20; ++it) {
    float mx = in ? m : -INFINITY;
    for (int o = 1; o < n; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float e = in ? __expf(m - mx) : 0.f;
    for (int o = 1; o < n; o <<= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    float lse = isfinite(mx) ? mx + __logf(e) : mx;
    m = m - lse;
    mx = in ? m : -INFINITY;
    for (int o = n; o < n * n; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    e = in ? __expf(m - mx) : 0.f;
    for (int o = n; o < n * n; o <<= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    m = m - (mx + __logf(e));
  }
  return __expf(m);
}

__device__ __forceinline__ float sinkhorn_lane_fast(float m, int n) {
  const int lane = threadIdx.x & 31;
  const bool in = lane < n * n;
  for (int it = 0; it < 20; ++it) {
    float mx = in ? m : -INFINITY;
    for (int o = 1; o < n; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float e = in ? __expf(m - mx) : 0.f;
    for (int o = 1; o < n; o <<= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    float lse = isfinite(mx) ? mx + __logf(e) : mx;
    m = m - lse;
    mx = in ? m : -INFINITY;
    for (int o = n; o < n * n; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    e = in ? __expf(m - mx) : 0.f;
    for (int o = n; o < n * n; o <<= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    m = m - (mx + __logf(e));
  }
  return __expf(m);
}


// Hardware reciprocal (MUFU, about 1 ulp): the Sinkhorn scalings sit in a
// 160-step dependency chain where an IEEE-rounded reciprocal sequence costs
// several times its latency.
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The same Sinkhorn iterations in the linear domain (n <= 4): with K =
// exp(m - max m), the log-domain iterate after t row/column steps is
// log(r_i K_ij c_j) for the scalings r_i = 1 / sum_j K_ij c_j and c_j = 1 /
// sum_i K_ij r_i, so each step is four dot products and four reciprocals
// instead of a logsumexp per row or column. Every lane holds the whole matrix.
// When a row or column maximum lies more than 60 below the overall maximum the
// scalings could leave the f32 range; the warp then takes the log-domain form.
// Lane l < n * n returns element l of the result.
__device__ __forceinline__ float sinkhorn_lane_lin(float m, int n) {
  const int lane = threadIdx.x & 31;
  float v[4][4];
  float M = -INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x = __shfl_sync(0xffffffffu, m, (i * n + j) & 31);
      v[i][j] = (i < n && j < n) ? x : -INFINITY;
      M = fmaxf(M, v[i][j]);
    }
  bool ok = isfinite(M);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float rm = -INFINITY, cm = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      rm = fmaxf(rm, v[i][j]);
      cm = fmaxf(cm, v[j][i]);
    }
    if (i < n) ok = ok && rm >= M - 60.0f && cm >= M - 60.0f;
  }
  if (!ok) return sinkhorn_lane_fast(m, n);  // the same decision in every lane
  float K[4][4], r[4], c[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    c[i] = i < n ? 1.0f : 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) K[i][j] = (i < n && j < n) ? __expf(v[i][j] - M) : 0.0f;
  }
  for (int it = 0; it < 20; ++it) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float sr = K[i][0] * c[0] + K[i][1] * c[1] + K[i][2] * c[2] + K[i][3] * c[3];
      r[i] = i < n ? rcp_approx(sr) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float sc = K[0][j] * r[0] + K[1][j] * r[1] + K[2][j] * r[2] + K[3][j] * r[3];
      c[j] = j < n ? rcp_approx(sc) : 0.0f;
    }
  }
  float out = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (i < n && j < n && lane == i * n + j) out = r[i] * K[i][j] * c[j];
  return out;
}

// Dot of one CQ row (4- or 2-bit) with a prepared activation in shared memory,
// one warp; lane l covers elements g*128 + l*4 .. +3 of every group, so the
// float4 reads of `xs` are conflict-free. `lev` is the matrix's level table in
// shared memory. The norm multiplies the lane's part of each group dot, as
// cq.rs:666-672 applies `norm * group_dot`. Returns the sum in every lane.
__device__ __forceinline__ float cq_row_dot_warp(const CqMat& W, int row_index, const float* lev,
                                                 const float* xs) {
  const int lane = threadIdx.x & 31;
  const uint8_t* row;
  const __half* nrm;
  cq_row_ptr(W, row_index, &row, &nrm);
  const int bits = W.bits, mask = (1 << bits) - 1;
  float acc = 0.f;
#pragma unroll 4
  for (int g = 0; g < W.groups; ++g) {
    const uint32_t c = cq_quad_codes(row, bits, g, lane);
    const float4 x = reinterpret_cast<const float4*>(xs + g * 128)[lane];
    float p = lev[c & mask] * x.x;
    p += lev[(c >> bits) & mask] * x.y;
    p += lev[(c >> (2 * bits)) & mask] * x.z;
    p += lev[(c >> (3 * bits)) & mask] * x.w;
    acc += __half2float(nrm[g]) * p;
  }
  return warp_sum(acc);
}

// cq_row_dot_warp over a packed row and its norms staged in shared memory.
__device__ __forceinline__ float cq_row_dot_staged(const unsigned char* row, const float* nrm, int bits,
                                                   int groups, const float* lev, const float* xs) {
  const int lane = threadIdx.x & 31, mask = (1 << bits) - 1;
  float acc = 0.f;
#pragma unroll 4
  for (int g = 0; g < groups; ++g) {
    const uint32_t c = bits == 4 ? (uint32_t)reinterpret_cast<const uint16_t*>(row + g * 64)[lane]
                                 : (uint32_t)row[g * 32 + lane];
    const float4 x = reinterpret_cast<const float4*>(xs + g * 128)[lane];
    float p = lev[c & mask] * x.x;
    p += lev[(c >> bits) & mask] * x.y;
    p += lev[(c >> (2 * bits)) & mask] * x.z;
    p += lev[(c >> (3 * bits)) & mask] * x.w;
    acc += nrm[g] * p;
  }
  return warp_sum(acc);
}

// The level tables of the three mHC projections, copied to shared memory so a
// lane-dependent lookup is a bank-parallel shared load.
__device__ __forceinline__ void load_phi_levels(const CqMat& a, const CqMat& b, const CqMat& c, float* lev) {
  const int t = threadIdx.x;
  if (t < 16)
    lev[t] = a.levels[t];
  else if (t < 32)
    lev[t] = b.levels[t - 16];
  else if (t < 48)
    lev[t] = c.levels[t - 32];
}

// Packed row, norms, row bytes and groups of projected row o of layer li:
// o < n phi_pre, o < 2n phi_post, else phi_res (mhc.rs:56-70).
__device__ __forceinline__ void phi_row(int o, int li, int n, const CqMat& a, const CqMat& b, const CqMat& c,
                                        const uint8_t** row, const __half** nrm, int* rb, int* groups) {
  if (o < n) {
    cq_row_ptr(a, li * n + o, row, nrm);
    *rb = a.row_bytes;
    *groups = a.groups;
  } else if (o < 2 * n) {
    cq_row_ptr(b, li * n + (o - n), row, nrm);
    *rb = b.row_bytes;
    *groups = b.groups;
  } else {
    cq_row_ptr(c, li * n * n + (o - 2 * n), row, nrm);
    *rb = c.row_bytes;
    *groups = c.groups;
  }
}

// The mHC pre-projection of row r after the 2n + n^2 projected values of
// rms_unit(lanes) are in phi[] (shared): the gates and Sinkhorn (mhc.rs:109-130;
// warp 0), mix_down (mhc.rs:79-102), the Engram gate (engram.rs:112-132) and
// the pre-attention norm + rotation of the q|k|v|gate input (model.rs:230-262)
// on the other warps. L: the row's lanes [lanes][d]; ek, ev: the row's Engram
// key and value at this layer's site (null without one); norm_in: the layer's
// input norm scale (each shared or global). gsm (24), red (32), bx (d) and hb
// (d rounded up to 128): shared scratch. Every thread of the CTA calls it last.
__device__ __forceinline__ void layer_pre_tail(const Geo& G, int li, int r, const MhcParams& mp,
                                               const float* phi, const float* L, float* gsm, float* red,
                                               float* bx, float* hb, const float* norm_in, const float* ek,
                                               const float* ev, float* __restrict__ u_out,
                                               float* __restrict__ bx_out, float* __restrict__ xh_out,
                                               float* __restrict__ gates, SplitOut so) {
  const int n = G.lanes, d = G.d;
  const int dpad = (d + 127) / 128 * 128;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  // Warp 0 forms the gates; the mix-down gate releases warps 1.. (named
  // barrier 1) while warp 0 runs Sinkhorn, which nothing below depends on.
  const int nwo = nw - 1, wo = wid - 1, to = tid - 32, NT = blockDim.x - 32;
  if (wid == 0) {
    const int act = li % n;
    float hpost = 0.f;
    if (lane < n) {
      const float pre_off = lane == act ? 4.0f : -4.0f;   // mhc.rs:56
      const float post_off = lane == act ? 0.0f : -4.0f;  // mhc.rs:65
      gsm[lane] = sigmoidf_(mp.a_pre * phi[lane] + mp.b_pre[lane] + pre_off);
      hpost = 2.0f * sigmoidf_(mp.a_post * phi[n + lane] + mp.b_post[lane] + post_off);
    }
    __syncwarp();
    asm volatile("bar.arrive 1, %0;" ::"r"(blockDim.x) : "memory");
    const float m = lane < n * n ? mp.a_res * phi[2 * n + lane] + mp.b_res[lane] : 0.f;
    const float hres = sinkhorn_lane_lin(m, n);
    float* gout = gates + (size_t)r * 24;
    if (lane < n) gout[lane] = hpost;
    if (lane < n * n) gout[n + lane] = hres;
    return;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(blockDim.x) : "memory");
  // Warps 1..: reductions over NT threads on named barrier 2.
  auto gsum = [&](float v) {
    v = warp_sum(v);
    asm volatile("bar.sync 2, %0;" ::"r"(NT) : "memory");
    if (lane == 0) red[wo] = v;
    asm volatile("bar.sync 2, %0;" ::"r"(NT) : "memory");
    return warp_sum(lane < nwo ? red[lane] : 0.f);
  };
  // Three sums at once (red holds 3 x 8 partials; nwo <= 8).
  auto gsum3 = [&](float& a, float& b, float& c) {
    a = warp_sum(a);
    b = warp_sum(b);
    c = warp_sum(c);
    asm volatile("bar.sync 2, %0;" ::"r"(NT) : "memory");
    if (lane == 0) red[wo] = a, red[8 + wo] = b, red[16 + wo] = c;
    asm volatile("bar.sync 2, %0;" ::"r"(NT) : "memory");
    a = warp_sum(lane < nwo ? red[lane] : 0.f);
    b = warp_sum(lane < nwo ? red[8 + lane] : 0.f);
    c = warp_sum(lane < nwo ? red[16 + lane] : 0.f);
  };
  // u = sum_i hpre_i * lane_i (mix_down), bx = u (+ Engram).
#pragma unroll 4
  for (int c = to; c < d; c += NT) {
    float acc = 0.f;
    for (int l = 0; l < n; ++l) acc += gsm[l] * L[l * d + c];
    bx[c] = acc;
    u_out[(size_t)r * d + c] = acc;
  }
  asm volatile("bar.sync 2, %0;" ::"r"(NT) : "memory");
  if (ek) {
    float sx = 0.f, sk = 0.f, sd = 0.f;
#pragma unroll 4
    for (int c = to; c < d; c += NT) {
      float x = bx[c], k = ek[c];
      sx += x * x;
      sk += k * k;
      sd += x * k;
    }
    gsum3(sx, sk, sd);
    const float ux = 1.0f / sqrtf(sx / (float)d + 1e-6f);
    const float uk = 1.0f / sqrtf(sk / (float)d + 1e-6f);
    const float alpha = sigmoidf_(sd * ux * uk / sqrtf((float)d));
#pragma unroll 4
    for (int c = to; c < d; c += NT) bx[c] += alpha * ev[c];
    asm volatile("bar.sync 2, %0;" ::"r"(NT) : "memory");
  }
  float s2 = 0.f;
  for (int c = to; c < d; c += NT) s2 += bx[c] * bx[c];
  s2 = gsum(s2);
  const float inv2 = 1.0f / sqrtf(s2 / (float)d + EPS);  // zc_rms_norm_vec, norm.rs:23
#pragma unroll 4
  for (int c = to; c < dpad; c += NT) {
    hb[c] = c < d ? (1.0f + norm_in[c]) * bx[c] * inv2 : 0.f;
    if (c < d) bx_out[(size_t)r * d + c] = bx[c];
  }
  asm volatile("bar.sync 2, %0;" ::"r"(NT) : "memory");
  for (int g = wo; g < dpad / 128; g += nwo) {
    float4 v = reinterpret_cast<float4*>(hb + g * 128)[lane];
    float x[4] = {v.x, v.y, v.z, v.w};
    fwht128_warp(x);
    if (so.hi)  // the q|k|v|gate projection's tensor-core operands
      split_group_store(x, so.hi + (size_t)r * dpad + g * 128, so.lo + (size_t)r * dpad + g * 128,
                        so.inv + (size_t)r * (dpad / 128) + g);
    else
      reinterpret_cast<float4*>(xh_out + (size_t)r * dpad + g * 128)[lane] = make_float4(x[0], x[1], x[2], x[3]);
  }
}

// mhc.rs:79-102 (mix_down) with the gate and Sinkhorn of mhc.rs:109-130, the
// Engram gate (engram.rs:112-132) and the pre-attention norm + rotation of the
// q|k|v|gate input (model.rs:230-262). phi_post / phi_res read the same
// rms_unit(lanes) as phi_pre (the lanes are unchanged until scatter_up,
// model.rs:241 vs :332), so all three projections run here.
__global__ void layer_pre_kernel(Geo G, int li, RowBatch rb, const float* __restrict__ lanes,
                                 CqMat phi_pre, CqMat phi_post, CqMat phi_res, MhcParams mp,
                                 const float* __restrict__ norm_in, int site,
                                 const float* __restrict__ ekv, const float* __restrict__ evc,
                                 float* __restrict__ u_out, float* __restrict__ bx_out,
                                 float* __restrict__ xh_out, float* __restrict__ gates, int rbmax,
                                 int gmax, SplitOut so) {
  pdl_trigger();  // a PDL-launched projection after this kernel may start its weight prefetch
  pdl_wait();     // everything below reads or writes what earlier kernels touch
  extern __shared__ __align__(16) float sm[];
  const int r = blockIdx.x;
  const int n = G.lanes, d = G.d, W = n * d;
  const int Wp = phi_pre.in_pad;
  float* L = sm;                 // [W]
  float* X = L + W;              // [Wp]
  float* bx = X + Wp;            // [d]
  float* hb = bx + d;            // [d] (h, rounded up to a multiple of 128)
  const int dpad = (d + 127) / 128 * 128;
  float* phi = hb + dpad;        // [32]
  float* red = phi + 32;         // [32]
  float* gsm = red + 32;         // [4 + 4 + 16]
  float* lev = gsm + 24;         // [3][16] level tables of phi_pre, phi_post, phi_res
  const int nrow = 2 * n + n * n;
  float* nsm = lev + 48;                                    // [nrow][gmax] norms
  unsigned char* csm = reinterpret_cast<unsigned char*>(  // [nrow][rbmax] codes, 16-byte aligned
      (reinterpret_cast<uintptr_t>(nsm + nrow * gmax) + 15) & ~uintptr_t(15));
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;

  load_phi_levels(phi_pre, phi_post, phi_res, lev);
  // The 2n + n^2 packed rows travel by cp.async while the lanes are normalised
  // and rotated below; every (row, chunk) and (row, group) is independent.
  {
    const int cpr = rbmax / 16;
    for (int i = tid; i < nrow * cpr; i += blockDim.x) {
      const int o = i / cpr, ch = i % cpr;
      const uint8_t* prow;
      const __half* pn;
      int rbo, go;
      phi_row(o, mp.phi_layer, n, phi_pre, phi_post, phi_res, &prow, &pn, &rbo, &go);
      if (ch * 16 < rbo) cp_async16(csm + (size_t)o * rbmax + ch * 16, prow + ch * 16, true);
    }
    cp_commit();
#pragma unroll 4
    for (int i = tid; i < nrow * gmax; i += blockDim.x) {
      const int o = i / gmax, g = i % gmax;
      const uint8_t* prow;
      const __half* pn;
      int rbo, go;
      phi_row(o, mp.phi_layer, n, phi_pre, phi_post, phi_res, &prow, &pn, &rbo, &go);
      nsm[i] = g < go ? __half2float(pn[g]) : 0.f;
    }
  }

  const float* lr = lanes + (size_t)r * W;
  float ss = 0.f;
#pragma unroll 4
  for (int i = tid; i < W; i += blockDim.x) {
    float v = lr[i];
    L[i] = v;
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)W + EPS);  // rms_unit_to, kernels.rs:32
  for (int i = tid; i < Wp; i += blockDim.x) X[i] = i < W ? L[i] * inv : 0.f;
  __syncthreads();
  fwht_groups_warp(X, Wp / 128);
  cp_wait<0>();
  __syncthreads();
  // 2n + n^2 projected gate rows of this layer, from the staged rows: warp w
  // dots rows w, w + nw, w + 2nw together, sharing each activation load.
  {
    float acc[3] = {0.f, 0.f, 0.f};
    int bits[3], lvo[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int k = wid + j * nw;
      bits[j] = k < n ? phi_pre.bits : (k < 2 * n ? phi_post.bits : phi_res.bits);
      lvo[j] = k < n ? 0 : (k < 2 * n ? 16 : 32);
    }
    const int groups = phi_pre.groups;  // the three mHC matrices share in_feat = lanes * d_model
#pragma unroll 2
    for (int g = 0; g < groups; ++g) {
      const float4 x = reinterpret_cast<const float4*>(X + g * 128)[lane];
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const int k = wid + j * nw;
        if (k >= nrow) continue;
        const unsigned char* row = csm + (size_t)k * rbmax;
        const int b = bits[j], mask = (1 << b) - 1;
        const uint32_t c = b == 4 ? (uint32_t)reinterpret_cast<const uint16_t*>(row + g * 64)[lane]
                                  : (uint32_t)row[g * 32 + lane];
        const float* lv = lev + lvo[j];
        float p = lv[c & mask] * x.x;
        p += lv[(c >> b) & mask] * x.y;
        p += lv[(c >> (2 * b)) & mask] * x.z;
        p += lv[(c >> (3 * b)) & mask] * x.w;
        acc[j] += nsm[k * gmax + g] * p;
      }
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float v = warp_sum(acc[j]);
      const int k = wid + j * nw;
      if (lane == 0 && k < nrow) phi[k] = v;
    }
  }
  __syncthreads();
  const float* ek = site >= 0 ? ekv + (size_t)r * G.n_sites * 2 * d + (size_t)site * 2 * d : nullptr;
  const float* ev = site >= 0 ? evc + ((size_t)r * G.n_sites + site) * d : nullptr;
  layer_pre_tail(G, li, r, mp, phi, L, gsm, red, bx, hb, norm_in, ek, ev, u_out, bx_out, xh_out, gates, so);
}

// The same computation for a few rows (batch-1 and small-batch decode), split
// over the 128-wide groups of the lanes so that one row occupies many SMs.
// CTA (g, r) rotates group g of row r's lanes, adds its sum of squares and its
// part of each of the 2n + n^2 dots (row k's group-g codes against the rotated
// group, times the group norm; cq.rs:666-672 sums norm * group_dot) into
// part[r][g][...]; the last CTA of the row to arrive (per-row counter, reset by
// that CTA) sums the groups in order, applies rms_unit (kernels.rs:32; a common
// factor of every dot, applied to the finished sums) and runs the tail. No CTA
// waits for another.
constexpr int PRE_SPLIT_MAX_GROUPS = 32;
__global__ void __launch_bounds__(256) layer_pre_split_kernel(
    Geo G, int li, RowBatch rb, const float* __restrict__ lanes, CqMat phi_pre, CqMat phi_post, CqMat phi_res,
    MhcParams mp, const float* __restrict__ norm_in, int site, const float* __restrict__ ekv,
    const float* __restrict__ evc, float* __restrict__ u_out, float* __restrict__ bx_out, float* __restrict__ xh_out,
    float* __restrict__ gates, float* __restrict__ part, int* __restrict__ cnt, SplitOut so) {
  pdl_trigger();  // a PDL-launched projection after this kernel may start its weight prefetch
  extern __shared__ __align__(16) float sm[];
  __shared__ __align__(16) float X[128];
  __shared__ float lev[48], phi[32], red[32], gsm[24];
  __shared__ int last;
  load_phi_levels(phi_pre, phi_post, phi_res, lev);  // kernel parameters only: before the wait
  pdl_wait();  // everything below reads or writes what earlier kernels touch
  const int g = blockIdx.x, r = blockIdx.y;
  const int n = G.lanes, d = G.d, W = n * d, ng = W / 128, nrow = 2 * n + n * n;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  const int dpad = (d + 127) / 128 * 128;
  float* bx = sm;              // [d]
  float* hb = sm + d;          // [dpad]
  float* Ls = hb + dpad;       // [W] the row's lanes (last CTA)
  float* eks = Ls + W;         // [d] Engram key (last CTA, with a site)
  float* evs = eks + d;        // [d] Engram value
  float* nis = evs + d;        // [d] norm_in
  float* pr = part + ((size_t)r * PRE_SPLIT_MAX_GROUPS + g) * 32;  // [0, nrow): dots; [31]: sum of squares
  if (wid == 0) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(lanes + (size_t)r * W + g * 128) + lane);
    float x[4] = {v.x, v.y, v.z, v.w};
    const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
    fwht128_warp(x);
    reinterpret_cast<float4*>(X)[lane] = make_float4(x[0], x[1], x[2], x[3]);
    if (lane == 0) pr[31] = ss;
  }
  __syncthreads();
  const float4 x = reinterpret_cast<const float4*>(X)[lane];
  // Rows wid, wid + 8, wid + 16 (nrow <= 24): every row's codes and norm are
  // loaded before any is used, one L2 round trip for the three.
  uint32_t cw[3] = {0u, 0u, 0u};
  float nw3[3] = {0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int k = wid + q * nw;
    if (k < nrow) {
      const uint8_t* row;
      const __half* nrm;
      int rbo, go;
      phi_row(k, mp.phi_layer, n, phi_pre, phi_post, phi_res, &row, &nrm, &rbo, &go);
      const int b = k < n ? phi_pre.bits : (k < 2 * n ? phi_post.bits : phi_res.bits);
      cw[q] = cq_quad_codes(row, b, g, lane);
      nw3[q] = __half2float(nrm[g]);
    }
  }
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int k = wid + q * nw;
    if (k < nrow) {
      const int b = k < n ? phi_pre.bits : (k < 2 * n ? phi_post.bits : phi_res.bits), mask = (1 << b) - 1;
      const float* lv = lev + (k < n ? 0 : (k < 2 * n ? 16 : 32));
      const uint32_t c = cw[q];
      float p = lv[c & mask] * x.x;
      p += lv[(c >> b) & mask] * x.y;
      p += lv[(c >> (2 * b)) & mask] * x.z;
      p += lv[(c >> (3 * b)) & mask] * x.w;
      p = warp_sum(p);
      if (lane == 0) pr[k] = nw3[q] * p;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&cnt[r], 1) == ng - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (tid == 0) cnt[r] = 0;  // ready for the next launch
  // The tail's inputs, copied while the partials are summed.
  const float* ek = site >= 0 ? ekv + (size_t)r * G.n_sites * 2 * d + (size_t)site * 2 * d : nullptr;
  const float* ev = site >= 0 ? evc + ((size_t)r * G.n_sites + site) * d : nullptr;
  for (int i = 4 * tid; i < W; i += 4 * blockDim.x) cp_async16(Ls + i, lanes + (size_t)r * W + i, true);
  for (int i = 4 * tid; i < d; i += 4 * blockDim.x) {
    cp_async16(nis + i, norm_in + i, true);
    if (ek) {
      cp_async16(eks + i, ek + i, true);
      cp_async16(evs + i, ev + i, true);
    }
  }
  cp_commit();
  if (tid < 32) {
    // All partials in flight at once (one L2 round trip), then summed in
    // group order.
    float pv[PRE_SPLIT_MAX_GROUPS];
    const bool used = tid < nrow || tid == 31;
#pragma unroll
    for (int gg = 0; gg < PRE_SPLIT_MAX_GROUPS; ++gg)
      pv[gg] = (used && gg < ng) ? __ldcg(part + ((size_t)r * PRE_SPLIT_MAX_GROUPS + gg) * 32 + tid) : 0.f;
    float v = 0.f;
#pragma unroll
    for (int gg = 0; gg < PRE_SPLIT_MAX_GROUPS; ++gg) v += pv[gg];
    const float inv = 1.0f / sqrtf(__shfl_sync(0xffffffffu, v, 31) / (float)W + EPS);  // rms_unit_to, kernels.rs:32
    if (tid < nrow) phi[tid] = v * inv;
  }
  cp_wait<0>();
  __syncthreads();
  layer_pre_tail(G, li, r, mp, phi, Ls, gsm, red, bx, hb, nis, ek ? eks : nullptr, ek ? evs : nullptr, u_out,
                 bx_out, xh_out, gates, so);
}

// The same computation for many rows: PT_M rows per CTA so each mHC weight
// row is read once for PT_M rows instead of once per row.
//
// Phase 1 streams the lanes of the tile one 128-wide group at a time through a
// PT_S-stage cp.async ring in shared memory, and warp w dots every row of the
// tile with outputs w, w+8 and w+16 of the 2n + n^2 projected rows, lane l
// covering group elements l*4..l*4+3. The weights are the mHC lane matrices
// dequantised and rotated once at load (MhcParams::phi_dense, f32): the CQ dot
// norm * (levels . H x) (cq.rs:666-672) equals (H (norm * levels)) . x for the
// symmetric group rotation H, so the lanes need no rotation here. The rms_unit
// scale (kernels.rs:32) is applied to the finished dot products rather than to
// the lanes first. Each warp keeps the next group's weights in flight.
// Phase 2 (one warp per row, no block barriers): gates and Sinkhorn, mix_down
// re-reading the tile's lanes (L2-resident), the Engram gate, the ZCRMS norm
// and the rotation of the attention input, exactly as the per-row kernel.
constexpr int PT_DQ = 8;   // d_model / 128 supported on this path
constexpr int PT_S = 4;    // lane-group stages in flight

// PT_M rows per CTA: 16 or 14 for large batches, 4 for small ones (four times
// the CTAs, shorter per-CTA loops).
template <int PT_M>
__global__ void __launch_bounds__(256, 2)
layer_pre_tiled_kernel(Geo G, int li, RowBatch rb, const float* __restrict__ lanes, MhcParams mp,
                       const float* __restrict__ norm_in, int site, const float* __restrict__ ekv,
                       const float* __restrict__ evc, float* __restrict__ u_out, float* __restrict__ bx_out,
                       float* __restrict__ xh_out, float* __restrict__ gates, SplitOut so) {
  pdl_trigger();  // a PDL-launched projection after this kernel may start its weight prefetch
  pdl_wait();     // everything below reads or writes what earlier kernels touch
  __shared__ __align__(16) float Xr[PT_S][PT_M][128];
  __shared__ float phi_s[PT_M][24];
  __shared__ float ss_s[PT_M];
  __shared__ float hp_s[PT_M][4];      // mix-down gates per row
  __shared__ float red3[8][PT_M][3];   // per-warp partial sums per row
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int n = G.lanes, d = G.d, W = n * d, nrow = 2 * n + n * n;
  const int m0 = blockIdx.x * PT_M;
  const int rows = min(PT_M, rb.M - m0);
  const int ngroups = W / 128;

  // Ring stage s <- group g of every tile row (rows past the batch zero-filled).
  auto issue = [&](int g) {
    if (g < ngroups)
      for (int i = tid; i < PT_M * 32; i += blockDim.x) {
        const int m = i >> 5, c = (i & 31) * 4;
        const float* src = lanes + (size_t)(m0 + (m < rows ? m : 0)) * W + g * 128 + c;
        cp_async16(&Xr[g % PT_S][m][c], src, m < rows);
      }
    cp_commit();  // one group per call, empty past the end, so the wait counts stay fixed
  };
#pragma unroll
  for (int g = 0; g < PT_S - 1; ++g) issue(g);

  // This warp's projected rows: o = wid + 8j, each a [W] row of dense weights.
  bool wok[3];
  const float* wrow[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int o = wid + 8 * j;
    wok[j] = o < nrow;
    wrow[j] = mp.phi_dense + (size_t)(wok[j] ? o : 0) * W + lane * 4;
  }
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 wn[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) wn[j] = wok[j] ? __ldg(reinterpret_cast<const float4*>(wrow[j])) : z4;
  float ssA = 0.f, ssB = 0.f;
  float acc[3][PT_M];
#pragma unroll
  for (int j = 0; j < 3; ++j)
#pragma unroll
    for (int m = 0; m < PT_M; ++m) acc[j][m] = 0.f;

  for (int g = 0; g < ngroups; ++g) {
    issue(g + PT_S - 1);
    float4 wc[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      wc[j] = wn[j];
      if (wok[j] && g + 1 < ngroups) wn[j] = __ldg(reinterpret_cast<const float4*>(wrow[j] + (g + 1) * 128));
    }
    cp_wait<PT_S - 1>();
    __syncthreads();
    const int s = g % PT_S;
    // Tile rows wid and wid + 8 exist only below PT_M (warp-uniform tests).
    if (wid < PT_M) {
      const float4 x = reinterpret_cast<const float4*>(Xr[s][wid])[lane];
      ssA += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
    if (wid + 8 < PT_M) {
      const float4 x = reinterpret_cast<const float4*>(Xr[s][wid + 8])[lane];
      ssB += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
#pragma unroll
    for (int m = 0; m < PT_M; ++m) {
      if (m < rows) {
        const float4 x = reinterpret_cast<const float4*>(Xr[s][m])[lane];
#pragma unroll
        for (int j = 0; j < 3; ++j)
          acc[j][m] += wc[j].x * x.x + wc[j].y * x.y + wc[j].z * x.z + wc[j].w * x.w;
      }
    }
    __syncthreads();  // stage s is refilled by the next iteration's issue
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
#pragma unroll
    for (int m = 0; m < PT_M; ++m) {
      const float v = warp_sum(acc[j][m]);
      if (lane == 0 && wok[j] && m < rows) phi_s[m][wid + 8 * j] = v;
    }
  }
  ssA = warp_sum(ssA);
  ssB = warp_sum(ssB);
  if (lane == 0) {
    if (wid < rows) ss_s[wid] = ssA;
    if (wid + 8 < rows) ss_s[wid + 8] = ssB;
  }
  __syncthreads();

  // ---- gates: warp w forms rows w and w + 8 at once, one per 16-lane half
  // (the Sinkhorn shuffles stay inside a half).
  {
    const int half = lane >> 4, hl = lane & 15;
    const int m = wid + 8 * half;
    const bool live = m < rows;
    const int act = li % n;
    const float inv = live ? 1.0f / sqrtf(ss_s[m] / (float)W + EPS) : 0.f;  // rms_unit_to, kernels.rs:32
    float hpre = 0.f, hpost = 0.f;
    if (live && hl < n) {
      const float pre_off = hl == act ? 4.0f : -4.0f;   // mhc.rs:56
      const float post_off = hl == act ? 0.0f : -4.0f;  // mhc.rs:65
      hpre = sigmoidf_(mp.a_pre * (phi_s[m][hl] * inv) + mp.b_pre[hl] + pre_off);
      hpost = 2.0f * sigmoidf_(mp.a_post * (phi_s[m][n + hl] * inv) + mp.b_post[hl] + post_off);
    }
    const float mres = (live && hl < n * n) ? mp.a_res * (phi_s[m][2 * n + hl] * inv) + mp.b_res[hl] : 0.f;
    const float hres = sinkhorn_half_fast(mres, n);
    if (live) {
      float* gout = gates + (size_t)(m0 + m) * 24;
      if (hl < n) {
        gout[hl] = hpost;
        hp_s[m][hl] = hpre;
      }
      if (hl < n * n) gout[n + hl] = hres;
    }
  }
  __syncthreads();
  // ---- element-parallel over the tile: warp w holds 128-wide group w of every
  // row (lane l elements 128w + 4l .. +3), so the final rotation needs no
  // shared memory. mix_down (mhc.rs:79-102), Engram gate (engram.rs:112-132),
  // ZCRMS norm (norm.rs:23) and the rotation of the attention input.
  const int nq = d / 128;
  const bool act_w = wid < nq;
  const int c0 = wid * 128 + lane * 4;
  float bxv[PT_M][4];
#pragma unroll
  for (int m = 0; m < PT_M; ++m) {
    bxv[m][0] = bxv[m][1] = bxv[m][2] = bxv[m][3] = 0.f;
    if (!act_w || m >= rows) continue;
    const float* lr = lanes + (size_t)(m0 + m) * W + c0;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int l = 0; l < n; ++l) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(lr + l * d));
      const float h = hp_s[m][l];
      a.x += h * t.x;
      a.y += h * t.y;
      a.z += h * t.z;
      a.w += h * t.w;
    }
    bxv[m][0] = a.x;
    bxv[m][1] = a.y;
    bxv[m][2] = a.z;
    bxv[m][3] = a.w;
    *reinterpret_cast<float4*>(u_out + (size_t)(m0 + m) * d + c0) = a;
  }
  if (site >= 0) {
    const size_t kv_ld = (size_t)G.n_sites * 2 * d;
#pragma unroll
    for (int m = 0; m < PT_M; ++m) {
      float sx = 0.f, sk = 0.f, sd = 0.f;
      if (act_w && m < rows) {
        const size_t r = m0 + m;
        const float4 kk = __ldg(reinterpret_cast<const float4*>(ekv + r * kv_ld + (size_t)site * 2 * d + c0));
        const float k4[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          sx += bxv[m][i] * bxv[m][i];
          sk += k4[i] * k4[i];
          sd += bxv[m][i] * k4[i];
        }
      }
      sx = warp_sum(sx);
      sk = warp_sum(sk);
      sd = warp_sum(sd);
      if (lane == 0) {
        red3[wid][m][0] = sx;
        red3[wid][m][1] = sk;
        red3[wid][m][2] = sd;
      }
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < PT_M; ++m) {
      if (!act_w || m >= rows) continue;
      float sx = 0.f, sk = 0.f, sd = 0.f;
      for (int w = 0; w < nq; ++w) {
        sx += red3[w][m][0];
        sk += red3[w][m][1];
        sd += red3[w][m][2];
      }
      const float ux = 1.0f / sqrtf(sx / (float)d + 1e-6f);
      const float uk = 1.0f / sqrtf(sk / (float)d + 1e-6f);
      const float alpha = sigmoidf_(sd * ux * uk / sqrtf((float)d));
      const float4 ev = __ldg(reinterpret_cast<const float4*>(evc + ((size_t)(m0 + m) * G.n_sites + site) * d + c0));
      bxv[m][0] += alpha * ev.x;
      bxv[m][1] += alpha * ev.y;
      bxv[m][2] += alpha * ev.z;
      bxv[m][3] += alpha * ev.w;
    }
    __syncthreads();
  }
#pragma unroll
  for (int m = 0; m < PT_M; ++m) {
    float s2 = bxv[m][0] * bxv[m][0] + bxv[m][1] * bxv[m][1] + bxv[m][2] * bxv[m][2] + bxv[m][3] * bxv[m][3];
    s2 = warp_sum(s2);
    if (lane == 0) red3[wid][m][0] = s2;
  }
  __syncthreads();
  if (!act_w) return;
  const float4 ni = __ldg(reinterpret_cast<const float4*>(norm_in + c0));
  // Rows are independent: predicated (not exited) so their latencies overlap.
#pragma unroll
  for (int m = 0; m < PT_M; ++m) {
    if (m >= rows) continue;
    float s2 = 0.f;
#pragma unroll
    for (int w = 0; w < PT_DQ; ++w) s2 += w < nq ? red3[w][m][0] : 0.f;
    const float inv2 = 1.0f / sqrtf(s2 / (float)d + EPS);  // zc_rms_norm_vec, norm.rs:23
    const size_t r = m0 + m;
    *reinterpret_cast<float4*>(bx_out + r * d + c0) = make_float4(bxv[m][0], bxv[m][1], bxv[m][2], bxv[m][3]);
    float h[4] = {(1.0f + ni.x) * bxv[m][0] * inv2, (1.0f + ni.y) * bxv[m][1] * inv2,
                  (1.0f + ni.z) * bxv[m][2] * inv2, (1.0f + ni.w) * bxv[m][3] * inv2};
    fwht128_warp(h);
    if (so.hi)  // the q|k|v|gate projection's tensor-core operands (d is a multiple of 128 here)
      split_group_store(h, so.hi + r * d + wid * 128, so.lo + r * d + wid * 128, so.inv + r * (d / 128) + wid);
    else
      *reinterpret_cast<float4*>(xh_out + r * d + c0) = make_float4(h[0], h[1], h[2], h[3]);
  }
}

// Rows at which the tiled kernel takes over from one CTA per row.
constexpr int PRE_TILED_MIN_ROWS = 2;

template <int PT_M>
static cudaError_t launch_pre_tiled(const Geo& G, int li, const RowBatch& rb, const float* lanes,
                                    const MhcParams& mp, const float* norm_in, int site, const float* ekv,
                                    const float* evc, float* u, float* bx, float* xh, float* gates,
                                    cudaStream_t st, SplitOut so) {
  return launch_pdl(layer_pre_tiled_kernel<PT_M>, dim3((rb.M + PT_M - 1) / PT_M), dim3(256), 0, st, G, li, rb, lanes,
                    mp, norm_in, site, ekv, evc, u, bx, xh, gates, so);
}

cudaError_t launch_layer_pre(const Geo& G, int li, const RowBatch& rb, const float* lanes,
                             const CqMat& phi_pre, const CqMat& phi_post, const CqMat& phi_res,
                             const MhcParams& mp, const float* norm_in, int site, const float* ekv,
                             const float* evc, float* u, float* bx, float* xh, float* gates,
                             cudaStream_t st, float* split_part, int* split_cnt, SplitOut so) {
  if (rb.M <= 0) return cudaSuccess;
  const int nrow = 2 * G.lanes + G.lanes * G.lanes;
  // Up to PRE_SPLIT_MAX_ROWS rows: every row over (lanes x d_model) / 128 CTAs.
  const int ngr = G.lanes * G.d / 128;
  if (split_part && split_cnt && rb.M <= PRE_SPLIT_MAX_ROWS && G.d % 128 == 0 && ngr <= PRE_SPLIT_MAX_GROUPS &&
      nrow <= 24 && phi_pre.groups == ngr && phi_post.groups == ngr && phi_res.groups == ngr &&
      (reinterpret_cast<uintptr_t>(norm_in) & 15) == 0 && (reinterpret_cast<uintptr_t>(lanes) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(ekv) & 15) == 0 && (reinterpret_cast<uintptr_t>(evc) & 15) == 0) {
    const size_t smem = (size_t)(G.d + G.d + ngr * 128 + 3 * G.d) * sizeof(float);
    cudaError_t e = allow_smem((const void*)layer_pre_split_kernel, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(layer_pre_split_kernel, dim3(ngr, rb.M), dim3(256), smem, st, G, li, rb, lanes, phi_pre,
                      phi_post, phi_res, mp, norm_in, site, ekv, evc, u, bx, xh, gates, split_part, split_cnt, so);
  }
  const int rbmax = std::max(phi_pre.row_bytes, std::max(phi_post.row_bytes, phi_res.row_bytes));
  const int gmax = std::max(phi_pre.groups, std::max(phi_post.groups, phi_res.groups));
  const bool tiled_ok = G.d % 128 == 0 && G.d / 128 <= PT_DQ && nrow <= 24 && G.lanes <= 4 &&
                        (reinterpret_cast<uintptr_t>(norm_in) & 15) == 0 && mp.phi_dense &&
                        (reinterpret_cast<uintptr_t>(mp.phi_dense) & 15) == 0;
  // From 2048 rows: 16- or 14-row tiles (two CTAs resident per SM), whichever
  // leaves the fewest rows on the busiest SM.
  auto busiest = [&](int pt) { return ((rb.M + pt - 1) / pt + 2 * 148 - 1) / (2 * 148) * pt; };
  if (tiled_ok && rb.M >= 2048)
    return busiest(14) < busiest(16)
               ? launch_pre_tiled<14>(G, li, rb, lanes, mp, norm_in, site, ekv, evc, u, bx, xh, gates, st, so)
               : launch_pre_tiled<16>(G, li, rb, lanes, mp, norm_in, site, ekv, evc, u, bx, xh, gates, st, so);
  if (tiled_ok && rb.M >= PRE_TILED_MIN_ROWS)
    return rb.M < 1024 ? launch_pre_tiled<2>(G, li, rb, lanes, mp, norm_in, site, ekv, evc, u, bx, xh, gates, st, so)
                       : launch_pre_tiled<4>(G, li, rb, lanes, mp, norm_in, site, ekv, evc, u, bx, xh, gates, st, so);
  const int W = G.lanes * G.d, dpad = (G.d + 127) / 128 * 128;
  const size_t smem = (size_t)(W + phi_pre.in_pad + G.d + dpad + 32 + 32 + 24 + 48 + nrow * gmax) * sizeof(float) +
                      (size_t)nrow * rbmax + 16;
  cudaError_t e = allow_smem((const void*)layer_pre_kernel, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(layer_pre_kernel, dim3(rb.M), dim3(256), smem, st, G, li, rb, lanes, phi_pre, phi_post, phi_res,
                    mp, norm_in, site, ekv, evc, u, bx, xh, gates, rbmax, gmax, so);
}

// ---------------------------------------------------------------- Q/K/V post-processing
// Causal depthwise conv (attention.rs:82-100, cache.rs:401-438), ZCRMS norm +
// half-split RoPE (attention.rs:107-143), int8 query fake-quant (model.rs:289-293)
// and quantize-on-append of K/V (cache.rs:346-377, quant_into :100-106).
//
// Every quantisation goes through kv_quant_warp (common.cuh), the one int8
// quantiser on the GPU, bit-exact with the reference on identical inputs.

// One activation row, handled by the whole CTA (WARP = false: the conv phase
// over every thread, the heads spread over the warps) or by one warp (WARP =
// true: many rows per CTA, for large batches). `sm` holds qkv_dim floats.
// Causal depthwise conv of channel c of row r (attention.rs:82-100,
// cache.rs:401-438): taps over the raw projections of the previous positions
// (the prompt's own rows in prefill, the session's tail ring in decode), and
// the raw value stored into the ring for the positions after it. The
// vectorised loop of qkv_post_row performs the same operations per channel.
__device__ __forceinline__ float qkv_conv_chan(const Geo& G, int li, const RowBatch& rb, const LayerParams& lp,
                                               const RowInfo& ri, const float* __restrict__ proj, int r, int c) {
  const int qd = G.q_dim, kd = G.k_dim, vd = G.v_dim, qkv = G.qkv_dim;
  const int taps = G.taps, tl = taps > 0 ? taps - 1 : 0, p = ri.pos;
  const float* tp;
  int dim, cc;
  if (c < qd) {
    tp = lp.q_taps; dim = qd; cc = c;
  } else if (c < qd + kd) {
    tp = lp.k_taps; dim = kd; cc = c - qd;
  } else {
    tp = lp.v_taps; dim = vd; cc = c - qd - kd;
  }
  const float x = proj[(size_t)r * G.proj_dim + c];
  if (taps <= 0) return x;
  float* tail = tl ? ri.s->qkv_tail + (size_t)li * tl * qkv : nullptr;
  float acc = tp[cc] * x;
#pragma unroll
  for (int j = 1; j < MAX_QKV_TAPS; ++j) {
    if (j >= taps || j > p) continue;
    const float prev = rb.mode == MODE_PREFILL ? proj[(size_t)(r - j) * G.proj_dim + c]
                                               : tail[(size_t)((p - j) % tl) * qkv + c];
    acc += tp[j * dim + cc] * prev;
  }
  if (tl && (rb.mode == MODE_DECODE || p >= ri.len - tl)) tail[(size_t)(p % tl) * qkv + c] = x;
  return acc;
}

// What every task of one row needs, read once per row: the layer's KV ring,
// the RoPE row of the position and where the new K/V go.
struct QkvRowCtx {
  LayerKV kv;
  const float* cs;  // cos
  const float* sn;  // sin
  int slot;
  bool int8, prefill, to_ring;
};
__device__ __forceinline__ QkvRowCtx qkv_row_ctx(const Geo& G, int li, const RowBatch& rb, const RowInfo& ri,
                                                 const float* __restrict__ rope_cs) {
  QkvRowCtx c;
  const int p = ri.pos, half = G.qk / 2;
  c.cs = rope_cs + (size_t)p * half;
  c.sn = rope_cs + (size_t)G.max_seq * half + (size_t)p * half;
  c.int8 = ri.s->int8 != 0;
  c.prefill = rb.mode == MODE_PREFILL;
  c.kv = ri.s->layers[li];
  c.slot = p % c.kv.slots;
  c.to_ring = !c.prefill || p >= ri.len - c.kv.slots;
  return c;
}

// Stores of task t of row r. x1, x2: the lane's two values after norm and
// RoPE (q, k) or the conv (v); in int8 mode c1, c2 are their codes and
// `scale` the head's scale (kv_quant_codes), and a q head stores the
// fake-quantised code * scale plus, for the integer score path of the int8
// attention, the codes and scale in q8out / q8s. Value codes are stored
// offset-binary (code ^ 0x80, the byte of code + 128): the attention widens
// them to f16 without a sign flip per byte, and the KV read-back flips them.
__device__ __forceinline__ void qkv_task_store(const Geo& G, float* __restrict__ qpost, void* pk, void* pv,
                                               float* pks, float* pvs, int8_t* __restrict__ q8out,
                                               float* __restrict__ q8s, int r, const QkvRowCtx& ctx, int t,
                                               float x1, float x2, float c1, float c2, float scale) {
  const int lane = threadIdx.x & 31;
  const int qd = G.q_dim;
  const bool int8 = ctx.int8, prefill = ctx.prefill, to_ring = ctx.to_ring;
  const LayerKV& kv = ctx.kv;
  const int slot = ctx.slot;
  if (t < G.heads) {
    const int h = t, half = G.qk / 2;
    if (int8) {
      if (q8out && lane < half) {
        q8out[(size_t)r * qd + h * G.qk + lane] = (int8_t)c1;
        q8out[(size_t)r * qd + h * G.qk + half + lane] = (int8_t)c2;
      }
      if (q8out && lane == 0) q8s[(size_t)r * G.heads + h] = scale;
      x1 = c1 * scale;
      x2 = c2 * scale;
    }
    if (lane < half) {
      qpost[(size_t)r * qd + h * G.qk + lane] = x1;
      qpost[(size_t)r * qd + h * G.qk + half + lane] = x2;
    }
    return;
  }
  const bool isk = t < G.heads + G.kvh;
  const int h = isk ? t - G.heads : t - G.heads - G.kvh;
  const int dim = isk ? G.qk : G.vh, hf = dim / 2;
  void* const scratch = isk ? pk : pv;
  void* const ring = isk ? kv.k : kv.v;
  if (int8) {
    const int x = isk ? 0 : 0x80;
    const int8_t a = (int8_t)((int)c1 ^ x), b = (int8_t)((int)c2 ^ x);
    if (lane < hf) {
      if (prefill) {
        int8_t* d8 = (int8_t*)scratch + ((size_t)r * G.kvh + h) * dim;
        d8[lane] = a;
        d8[hf + lane] = b;
      }
      if (to_ring) {
        int8_t* d8 = (int8_t*)ring + ((size_t)h * kv.slots + slot) * dim;
        d8[lane] = a;
        d8[hf + lane] = b;
      }
    }
    if (lane == 0) {
      if (prefill) (isk ? pks : pvs)[(size_t)r * G.kvh + h] = scale;
      if (to_ring) (isk ? kv.ks : kv.vs)[(size_t)h * kv.slots + slot] = scale;
    }
  } else if (lane < hf) {
    if (prefill) {
      float* df = (float*)scratch + ((size_t)r * G.kvh + h) * dim;
      df[lane] = x1;
      df[hf + lane] = x2;
    }
    if (to_ring) {
      float* df = (float*)ring + ((size_t)h * kv.slots + slot) * dim;
      df[lane] = x1;
      df[hf + lane] = x2;
    }
  }
}

// Task t of row r held by one warp: q head t (t < heads) or k head t - heads
// (norm + RoPE, attention.rs:107-143; int8 query fake-quant, model.rs:289-293)
// or v head t - heads - kvh, then the stores (quantize-on-append in int8
// mode, cache.rs:346-377). x1, x2: the lane's two conv outputs, channels
// qkv_task_chan gives (0 on lanes past the head's half).
__device__ __forceinline__ void qkv_task(const Geo& G, const LayerParams& lp, float* __restrict__ qpost, void* pk,
                                         void* pv, float* pks, float* pvs, int8_t* __restrict__ q8out,
                                         float* __restrict__ q8s, int r, const QkvRowCtx& ctx, int t, float x1,
                                         float x2) {
  const int lane = threadIdx.x & 31;
  if (t < G.heads + G.kvh) {
    const bool isq = t < G.heads;
    const int half = G.qk / 2;
    const float* sc = isq ? lp.q_norm : lp.k_norm;
    float sq = warp_sum(x1 * x1 + x2 * x2);
    float rms = sqrtf(sq / (float)G.qk + 1e-6f);
    if (lane < half) {
      x1 = (1.0f + sc[lane]) * x1 / rms;
      x2 = (1.0f + sc[half + lane]) * x2 / rms;
      float c = ctx.cs[lane], s = ctx.sn[lane];
      float y1 = x1 * c - x2 * s, y2 = x2 * c + x1 * s;
      x1 = y1;
      x2 = y2;
    }
  }
  float c1 = 0.f, c2 = 0.f, scale = 1.f;
  if (ctx.int8) scale = kv_quant_warp(x1, x2, &c1, &c2);
  qkv_task_store(G, qpost, pk, pv, pks, pvs, q8out, q8s, r, ctx, t, x1, x2, c1, c2, scale);
}

// The two channels (of the q|k|v conv output) lane `lane` holds in task t, or
// false on lanes past the head's half.
__device__ __forceinline__ bool qkv_task_chan(const Geo& G, int t, int lane, int* c1, int* c2) {
  int base, hf;
  if (t < G.heads + G.kvh) {
    base = t < G.heads ? t * G.qk : G.q_dim + (t - G.heads) * G.qk;
    hf = G.qk / 2;
  } else {
    base = G.q_dim + G.k_dim + (t - G.heads - G.kvh) * G.vh;
    hf = G.vh / 2;
  }
  *c1 = base + lane;
  *c2 = base + hf + lane;
  return lane < hf;
}

// One row over the CTA: the conv into `sm` ([qkv_dim] floats), then the heads
// over the warps.
__device__ __forceinline__ void qkv_post_row(const Geo& G, int li, const RowBatch& rb, const LayerParams& lp,
                                             const float* __restrict__ rope_cs, const float* __restrict__ proj,
                                             float* __restrict__ qpost, void* pk, void* pv, float* pks, float* pvs,
                                             int8_t* __restrict__ q8out, float* __restrict__ q8s, int r, float* sm) {
  const int tix = threadIdx.x, nthr = blockDim.x;
  const RowInfo ri = rb.rows[r];
  const int p = ri.pos;
  const int qd = G.q_dim, kd = G.k_dim, vd = G.v_dim, qkv = G.qkv_dim;
  const int taps = G.taps, tl = taps > 0 ? taps - 1 : 0;
  const float* raw = proj + (size_t)r * G.proj_dim;
  float* tail = tl ? ri.s->qkv_tail + (size_t)li * tl * qkv : nullptr;
  // Four channels per thread when every segment width is a multiple of 4.
  if ((qd | kd | vd) % 4 == 0) {
    const int slot_here = tl ? p % tl : 0;
    for (int c = 4 * tix; c < qkv; c += 4 * nthr) {
      const float* tp;
      int dim, cc;
      if (c < qd) {
        tp = lp.q_taps; dim = qd; cc = c;
      } else if (c < qd + kd) {
        tp = lp.k_taps; dim = kd; cc = c - qd;
      } else {
        tp = lp.v_taps; dim = vd; cc = c - qd - kd;
      }
      const float4 x = *reinterpret_cast<const float4*>(raw + c);
      float4 acc = x;
      if (taps > 0) {
        const float4 t0 = *reinterpret_cast<const float4*>(tp + cc);
        acc = make_float4(t0.x * x.x, t0.y * x.y, t0.z * x.z, t0.w * x.w);
        // Fixed trip count, predicated taps: every tap's loads are in flight
        // together instead of one tap per memory round trip.
#pragma unroll
        for (int j = 1; j < MAX_QKV_TAPS; ++j) {
          if (j >= taps || j > p) continue;
          const float4 pv = *reinterpret_cast<const float4*>(
              rb.mode == MODE_PREFILL ? proj + (size_t)(r - j) * G.proj_dim + c
                                      : tail + (size_t)((p - j) % tl) * qkv + c);
          const float4 tj = *reinterpret_cast<const float4*>(tp + j * dim + cc);
          acc.x += tj.x * pv.x;
          acc.y += tj.y * pv.y;
          acc.z += tj.z * pv.z;
          acc.w += tj.w * pv.w;
        }
        if (tl && (rb.mode == MODE_DECODE || p >= ri.len - tl))
          *reinterpret_cast<float4*>(tail + (size_t)slot_here * qkv + c) = x;
      }
      *reinterpret_cast<float4*>(sm + c) = acc;
    }
  } else {
#pragma unroll 4
    for (int c = tix; c < qkv; c += nthr) sm[c] = qkv_conv_chan(G, li, rb, lp, ri, proj, r, c);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int ntask = G.heads + 2 * G.kvh;
  const QkvRowCtx ctx = qkv_row_ctx(G, li, rb, ri, rope_cs);
  for (int t = wid; t < ntask; t += nw) {
    int c1, c2;
    const bool on = qkv_task_chan(G, t, lane, &c1, &c2);
    qkv_task(G, lp, qpost, pk, pv, pks, pvs, q8out, q8s, r, ctx, t, on ? sm[c1] : 0.f, on ? sm[c2] : 0.f);
  }
}

__global__ void qkv_post_kernel(Geo G, int li, RowBatch rb, LayerParams lp, const float* __restrict__ rope_cs,
                                const float* __restrict__ proj, float* __restrict__ qpost, void* pk, void* pv,
                                float* pks, float* pvs, int8_t* __restrict__ q8out, float* __restrict__ q8s) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float sm[];
  qkv_post_row(G, li, rb, lp, rope_cs, proj, qpost, pk, pv, pks, pvs, q8out, q8s, blockIdx.x, sm);
}

// Large batches: one warp per row, QP_ROWS rows per CTA, each warp with its
// own qkv_dim-float slice of shared memory for the conv output. The RoPE row
// and the norm scales are read once per row, and the heads run QP_CHUNK at a
// time with their reductions interleaved (each head's sums in the order
// qkv_task uses, so the results are the same). Needs q_dim, k_dim and v_dim
// multiples of 4. Seven rows: 4096 rows make 586 CTAs, four resident on each
// of the 148 SMs.
constexpr int QP_ROWS = 7;
constexpr int QP_CHUNK = 4;
__global__ void __launch_bounds__(QP_ROWS * 32, 4)
qkv_post_rows_kernel(Geo G, int li, RowBatch rb, LayerParams lp, const float* __restrict__ rope_cs,
                     const float* __restrict__ proj, float* __restrict__ qpost, void* pk, void* pv, float* pks,
                     float* pvs, int8_t* __restrict__ q8out, float* __restrict__ q8s) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float sm[];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, r = blockIdx.x * QP_ROWS + w;
  if (r >= rb.M) return;
  const int qd = G.q_dim, kd = G.k_dim, qkv = G.qkv_dim;
  float* const xs = sm + (size_t)w * ((qkv + 3) / 4 * 4);
  const RowInfo ri = rb.rows[r];
  const int p = ri.pos;
  const int taps = G.taps, tl = taps > 0 ? taps - 1 : 0;
  const float* raw = proj + (size_t)r * G.proj_dim;
  float* tail = tl ? ri.s->qkv_tail + (size_t)li * tl * qkv : nullptr;
  // Conv (the arithmetic of qkv_post_row).
  for (int c = 4 * lane; c < qkv; c += 128) {
    const float* tp;
    int dim, cc;
    if (c < qd) {
      tp = lp.q_taps; dim = qd; cc = c;
    } else if (c < qd + kd) {
      tp = lp.k_taps; dim = kd; cc = c - qd;
    } else {
      tp = lp.v_taps; dim = G.v_dim; cc = c - qd - kd;
    }
    const float4 x = *reinterpret_cast<const float4*>(raw + c);
    float4 acc = x;
    if (taps > 0) {
      const float4 t0 = *reinterpret_cast<const float4*>(tp + cc);
      acc = make_float4(t0.x * x.x, t0.y * x.y, t0.z * x.z, t0.w * x.w);
#pragma unroll
      for (int j = 1; j < MAX_QKV_TAPS; ++j) {
        if (j >= taps || j > p) continue;
        const float4 pv4 = *reinterpret_cast<const float4*>(
            rb.mode == MODE_PREFILL ? proj + (size_t)(r - j) * G.proj_dim + c : tail + (size_t)((p - j) % tl) * qkv + c);
        const float4 tj = *reinterpret_cast<const float4*>(tp + j * dim + cc);
        acc.x += tj.x * pv4.x;
        acc.y += tj.y * pv4.y;
        acc.z += tj.z * pv4.z;
        acc.w += tj.w * pv4.w;
      }
      if (tl && (rb.mode == MODE_DECODE || p >= ri.len - tl))
        *reinterpret_cast<float4*>(tail + (size_t)(p % tl) * qkv + c) = x;
    }
    *reinterpret_cast<float4*>(xs + c) = acc;
  }
  __syncwarp();
  const QkvRowCtx ctx = qkv_row_ctx(G, li, rb, ri, rope_cs);
  const int half = G.qk / 2;
  float qn1 = 0.f, qn2 = 0.f, kn1 = 0.f, kn2 = 0.f, rc = 0.f, rs = 0.f;
  if (lane < half) {
    qn1 = lp.q_norm[lane];
    qn2 = lp.q_norm[half + lane];
    kn1 = lp.k_norm[lane];
    kn2 = lp.k_norm[half + lane];
    rc = ctx.cs[lane];
    rs = ctx.sn[lane];
  }
  const int ntask = G.heads + 2 * G.kvh, nqk = G.heads + G.kvh;
  for (int t0 = 0; t0 < ntask; t0 += QP_CHUNK) {
    float x1[QP_CHUNK], x2[QP_CHUNK], sq[QP_CHUNK];
#pragma unroll
    for (int k = 0; k < QP_CHUNK; ++k) {
      int c1, c2;
      const bool on = t0 + k < ntask && qkv_task_chan(G, t0 + k, lane, &c1, &c2);
      x1[k] = on ? xs[c1] : 0.f;
      x2[k] = on ? xs[c2] : 0.f;
      sq[k] = x1[k] * x1[k] + x2[k] * x2[k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int k = 0; k < QP_CHUNK; ++k) sq[k] += __shfl_xor_sync(0xffffffffu, sq[k], o);
#pragma unroll
    for (int k = 0; k < QP_CHUNK; ++k) {
      const int t = t0 + k;
      if (t < nqk && lane < half) {  // q or k head: norm + RoPE
        const bool isq = t < G.heads;
        const float rms = sqrtf(sq[k] / (float)G.qk + 1e-6f);
        const float a = (1.0f + (isq ? qn1 : kn1)) * x1[k] / rms;
        const float b = (1.0f + (isq ? qn2 : kn2)) * x2[k] / rms;
        x1[k] = a * rc - b * rs;
        x2[k] = b * rc + a * rs;
      }
    }
    float c1[QP_CHUNK], c2[QP_CHUNK], scale[QP_CHUNK];
    if (ctx.int8) {
      float am[QP_CHUNK];
#pragma unroll
      for (int k = 0; k < QP_CHUNK; ++k) am[k] = kv_quant_absmax_warp(x1[k], x2[k]);
#pragma unroll
      for (int k = 0; k < QP_CHUNK; ++k) scale[k] = kv_quant_codes(am[k], x1[k], x2[k], &c1[k], &c2[k]);
    } else {
#pragma unroll
      for (int k = 0; k < QP_CHUNK; ++k) c1[k] = c2[k] = 0.f, scale[k] = 1.f;
    }
#pragma unroll
    for (int k = 0; k < QP_CHUNK; ++k)
      if (t0 + k < ntask)
        qkv_task_store(G, qpost, pk, pv, pks, pvs, q8out, q8s, r, ctx, t0 + k, x1[k], x2[k], c1[k], c2[k], scale[k]);
  }
}

// Small batches: one warp per task (q, k or v head) of a row, QH_TASKS tasks
// per CTA, each warp running the conv of its own channels, so that a row's
// heads spread over many SMs instead of queueing on one CTA's eight warps.
constexpr int QH_TASKS = 4;
constexpr int QH_MAX_ROWS = 128;
__global__ void __launch_bounds__(QH_TASKS * 32)
qkv_post_head_kernel(Geo G, int li, RowBatch rb, LayerParams lp, const float* __restrict__ rope_cs,
                     const float* __restrict__ proj, float* __restrict__ qpost, void* pk, void* pv, float* pks,
                     float* pvs, int8_t* __restrict__ q8out, float* __restrict__ q8s) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x, t = blockIdx.y * QH_TASKS + (int)(threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= G.heads + 2 * G.kvh) return;  // the whole warp
  const RowInfo ri = rb.rows[r];
  int c1, c2;
  float x1 = 0.f, x2 = 0.f;
  if (qkv_task_chan(G, t, lane, &c1, &c2)) {
    x1 = qkv_conv_chan(G, li, rb, lp, ri, proj, r, c1);
    x2 = qkv_conv_chan(G, li, rb, lp, ri, proj, r, c2);
  }
  qkv_task(G, lp, qpost, pk, pv, pks, pvs, q8out, q8s, r, qkv_row_ctx(G, li, rb, ri, rope_cs), t, x1, x2);
}

cudaError_t launch_qkv_post(const Geo& G, int li, const RowBatch& rb, const LayerParams& lp,
                            const float* rope_cs, const float* proj, float* qpost, void* pk,
                            void* pv, float* pks, float* pvs, int8_t* q8out, float* q8s, cudaStream_t st) {
  if (rb.M <= 0) return cudaSuccess;
  if (G.qk > 64 || G.vh > 64 || (G.qk & 1) || (G.vh & 1)) return cudaErrorInvalidValue;
  const bool rows_ok = (G.q_dim | G.k_dim | G.v_dim) % 4 == 0 && G.taps <= MAX_QKV_TAPS;
  if (rb.M >= 2048 && rows_ok) {  // enough rows to fill the SMs with one warp per row
    const size_t smem = (size_t)QP_ROWS * ((G.qkv_dim + 3) / 4 * 4) * sizeof(float);
    cudaError_t e = allow_smem((const void*)qkv_post_rows_kernel, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(qkv_post_rows_kernel, dim3((rb.M + QP_ROWS - 1) / QP_ROWS), dim3(QP_ROWS * 32), smem, st, G,
                      li, rb, lp, rope_cs, proj, qpost, pk, pv, pks, pvs, q8out, q8s);
  }
  if (rb.M <= QH_MAX_ROWS) {
    const int ntask = G.heads + 2 * G.kvh;
    return launch_pdl(qkv_post_head_kernel, dim3(rb.M, (ntask + QH_TASKS - 1) / QH_TASKS), dim3(QH_TASKS * 32), 0,
                      st, G, li, rb, lp, rope_cs, proj, qpost, pk, pv, pks, pvs, q8out, q8s);
  }
  const size_t smem = (size_t)G.qkv_dim * sizeof(float);
  return launch_pdl(qkv_post_kernel, dim3(rb.M), dim3(256), smem, st, G, li, rb, lp, rope_cs, proj, qpost, pk, pv,
                    pks, pvs, q8out, q8s);
}

// ---------------------------------------------------------------- block tail
// model.rs:309-356: post_norm + gated residual, pre_hada norm, HadamardMLP
// (v3/kernels.rs:119-180), MLP residual, y = block - u and scatter_up
// (mhc.rs:109-158) back into the lanes.
__device__ void kron_apply_block(const float* z, const float* __restrict__ a,
                                 const float* __restrict__ b, int ba, int bb, float* tmp, float* As,
                                 float* Bs, float* out) {
  // out[k][l] = sum_j (sum_i z[i][j] a[i][k]) b[j][l]  (kernels.rs:41-78)
  for (int i = threadIdx.x; i < ba * ba; i += blockDim.x) As[i] = a[i];
  for (int i = threadIdx.x; i < bb * bb; i += blockDim.x) Bs[i] = b[i];
  __syncthreads();
  for (int e = threadIdx.x; e < ba * bb; e += blockDim.x) {
    int k = e / bb, j = e % bb;
    float acc = 0.f;
    for (int i = 0; i < ba; ++i) acc += z[i * bb + j] * As[i * ba + k];
    tmp[e] = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ba * bb; e += blockDim.x) {
    int k = e / bb, l = e % bb;
    float acc = 0.f;
    for (int j = 0; j < bb; ++j) acc += tmp[k * bb + j] * Bs[j * bb + l];
    out[e] = acc;
  }
  __syncthreads();
}

// The same contraction register-tiled for ba, bb multiples of 4: each thread
// produces four consecutive k of one column j (stage 1) or l (stage 2), so a
// step reads one broadcast float4 and one per-lane float for four FMAs. The
// intermediate is stored transposed, tmpT[j][k] with row stride ba + 4 so the
// float4 stores of consecutive j hit distinct banks. Sums run over i and j in
// the same ascending order as kron_apply_block.
__device__ void kron_apply_block4(const float* z, const float* __restrict__ a,
                                  const float* __restrict__ b, int ba, int bb, float* tmpT, float* As,
                                  float* Bs, float* out) {
  for (int i = threadIdx.x; i < ba * ba; i += blockDim.x) As[i] = a[i];
  for (int i = threadIdx.x; i < bb * bb; i += blockDim.x) Bs[i] = b[i];
  __syncthreads();
  const int nq = (ba / 4) * bb, ts = ba + 4;
  for (int e = threadIdx.x; e < nq; e += blockDim.x) {
    const int j = e % bb, k0 = (e / bb) * 4;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 8
    for (int i = 0; i < ba; ++i) {
      const float zv = z[i * bb + j];
      const float4 av = *reinterpret_cast<const float4*>(As + i * ba + k0);
      a0 += zv * av.x;
      a1 += zv * av.y;
      a2 += zv * av.z;
      a3 += zv * av.w;
    }
    *reinterpret_cast<float4*>(tmpT + j * ts + k0) = make_float4(a0, a1, a2, a3);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < nq; e += blockDim.x) {
    const int l = e % bb, k0 = (e / bb) * 4;
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll 8
    for (int j = 0; j < bb; ++j) {
      const float bv = Bs[j * bb + l];
      const float4 tv = *reinterpret_cast<const float4*>(tmpT + j * ts + k0);
      o0 += tv.x * bv;
      o1 += tv.y * bv;
      o2 += tv.z * bv;
      o3 += tv.w * bv;
    }
    out[(k0 + 0) * bb + l] = o0;
    out[(k0 + 1) * bb + l] = o1;
    out[(k0 + 2) * bb + l] = o2;
    out[(k0 + 3) * bb + l] = o3;
  }
  __syncthreads();
}

__global__ void layer_post_kernel(Geo G, int li, RowBatch rb, LayerParams lp,
                                  const uint32_t* __restrict__ p1, const uint32_t* __restrict__ p2,
                                  const float* __restrict__ projo, const float* __restrict__ u,
                                  const float* __restrict__ bx_in, const float* __restrict__ gates,
                                  float* __restrict__ lanes) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float sm[];
  const int r = blockIdx.x;
  const int d = G.d, n = G.hada_n, nl = G.lanes;
  float* s1 = sm;             // [d]
  float* t = s1 + d;          // [d]
  float* cond = t + d;        // [n]
  float* z = cond + n;        // [n]
  float* buf = z + n;         // [n]
  float* tmp = buf + n;       // [n + 4*bb]
  float* As = tmp + n + 4 * G.bb;  // [ba*ba]
  float* Bs = As + G.ba * G.ba;  // [bb*bb]
  float* red = Bs + G.bb * G.bb; // [32]
  float* pr = red + 32;          // [8]
  float* gs = pr + 8;            // [24]
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const bool k4 = (G.ba % 4) == 0 && (G.bb % 4) == 0 && (d % 2) == 0;
  auto kron = [&](const float* a, const float* b) {
    if (k4)
      kron_apply_block4(z, a, b, G.ba, G.bb, tmp, As, Bs, buf);
    else
      kron_apply_block(z, a, b, G.ba, G.bb, tmp, As, Bs, buf);
  };
  const float* po = projo + (size_t)r * d;
  const float* bx = bx_in + (size_t)r * d;
  if (tid < nl + nl * nl) gs[tid] = gates[(size_t)r * 24 + tid];
  float ss = 0.f;
  for (int c = tid; c < d; c += blockDim.x) ss += po[c] * po[c];
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)d + EPS);
  const float ag = sigmoidf_(lp.attn_gate);
  for (int c = tid; c < d; c += blockDim.x) s1[c] = bx[c] + ag * ((1.0f + lp.post_norm[c]) * po[c] * inv);
  __syncthreads();
  float s2 = 0.f;
  for (int c = tid; c < d; c += blockDim.x) s2 += s1[c] * s1[c];
  s2 = block_sum(s2, red);
  const float inv2 = 1.0f / sqrtf(s2 / (float)d + EPS);
  for (int c = tid; c < d; c += blockDim.x) t[c] = (1.0f + lp.pre_hada[c]) * s1[c] * inv2;
  __syncthreads();
  // cond = 1 + softmax(t . cond_v) . cond_u   (rank <= 8)
  const int rk = G.cond_rank;
  if (wid < rk) {
    float acc = 0.f;
    for (int i = lane; i < d; i += 32) acc += t[i] * lp.cond_v[i * rk + wid];
    acc = warp_sum(acc);
    if (lane == 0) pr[wid] = acc;
  }
  __syncthreads();
  if (tid == 0) {
    float mx = -INFINITY;
    for (int j = 0; j < rk; ++j) mx = fmaxf(mx, pr[j]);
    float sum = 0.f;
    for (int j = 0; j < rk; ++j) {
      pr[j] = expf(pr[j] - mx);
      sum += pr[j];
    }
    for (int j = 0; j < rk; ++j) pr[j] = pr[j] / sum;
  }
  __syncthreads();
  for (int c = tid; c < n; c += blockDim.x) {
    float cv = 1.0f;
    for (int j = 0; j < rk; ++j)
      if (pr[j] != 0.0f) cv += pr[j] * lp.cond_u[j * n + c];
    cond[c] = cv;
    z[c] = (c < d ? t[c] : 0.f) * lp.d1[c];
  }
  __syncthreads();
  kron(lp.w1a, lp.w1b);
  for (int c = tid; c < n; c += blockDim.x) {
    float v = lp.d2[c] * cond[c] * buf[p1[c]] + lp.b2[c];
    z[c] = v * sigmoidf_(v);  // silu, ops.rs:118
  }
  __syncthreads();
  kron(lp.w2a, lp.w2b);
  for (int c = tid; c < n; c += blockDim.x) z[c] = buf[p2[c]] * lp.d3[c];
  __syncthreads();
  kron(lp.w3a, lp.w3b);
  // bx += mlp; y = bx - u; lanes' = hres . lanes + hpost * y
  float* lr = lanes + (size_t)r * nl * d;
  const float* ur = u + (size_t)r * d;
  for (int c = tid; c < d; c += blockDim.x) {
    float b2 = s1[c] + buf[c] * lp.d4[c];
    float y = b2 - ur[c];
    float lv[4];
    for (int j = 0; j < nl; ++j) lv[j] = lr[j * d + c];
    for (int i = 0; i < nl; ++i) {
      float acc = 0.f;
      for (int j = 0; j < nl; ++j) acc += gs[nl + i * nl + j] * lv[j];
      lr[i * d + c] = acc + gs[i] * y;
    }
  }
}

cudaError_t launch_layer_post(const Geo& G, int li, const RowBatch& rb, const LayerParams& lp,
                              const uint32_t* p1, const uint32_t* p2, const float* projo,
                              const float* u, float* bx, const float* gates, float* lanes,
                              cudaStream_t st) {
  if (rb.M <= 0) return cudaSuccess;
  if (lp.hfrag) return launch_layer_post_tc(G, rb, lp, p1, p2, projo, u, bx, gates, lanes, st);
  if (G.lanes > 4 || G.cond_rank > 8) return cudaErrorInvalidValue;
  const size_t smem =
      (size_t)(2 * G.d + 4 * G.hada_n + 4 * G.bb + G.ba * G.ba + G.bb * G.bb + 32 + 8 + 24) * sizeof(float);
  cudaError_t e = allow_smem((const void*)layer_post_kernel, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(layer_post_kernel, dim3(rb.M), dim3(256), smem, st, G, li, rb, lp, p1, p2, projo, u, bx, gates,
                    lanes);
}

// ---------------------------------------------------------------- head
// model.rs:358-374: lane mean, final ZCRMS norm, rotation for the tied head.
__global__ void final_kernel(Geo G, const float* __restrict__ lanes, const float* __restrict__ fnorm,
                             float* __restrict__ lm_in, SplitOut so, unsigned long long* __restrict__ keys) {
  pdl_trigger();  // a PDL-launched projection after this kernel may start its weight prefetch
  pdl_wait();     // everything below reads or writes what earlier kernels touch
  if (keys && threadIdx.x == 0) keys[blockIdx.x] = 0ull;  // the head's greedy pick starts empty
  extern __shared__ __align__(16) float sm[];
  float* red = sm;
  float* x = sm + 32;
  const int r = blockIdx.x, d = G.d, dpad = (d + 127) / 128 * 128;
  const float* lr = lanes + (size_t)r * G.lanes * d;
  float ss = 0.f;
#pragma unroll 4
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float a = 0.f;
    for (int l = 0; l < G.lanes; ++l) a += lr[l * d + c];
    a = a / (float)G.lanes;
    x[c] = a;
    ss += a * a;
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)d + EPS);
  for (int c = threadIdx.x; c < dpad; c += blockDim.x) x[c] = c < d ? (1.0f + fnorm[c]) * x[c] * inv : 0.f;
  __syncthreads();
  if (so.hi) {  // rotation and the LM head's tensor-core operands, one warp per group
    const int lane = threadIdx.x & 31;
    for (int g = threadIdx.x >> 5; g < dpad / 128; g += blockDim.x >> 5) {
      const float4 v = reinterpret_cast<const float4*>(x + g * 128)[lane];
      float h[4] = {v.x, v.y, v.z, v.w};
      fwht128_warp(h);
      split_group_store(h, so.hi + (size_t)r * dpad + g * 128, so.lo + (size_t)r * dpad + g * 128,
                        so.inv + (size_t)r * (dpad / 128) + g);
    }
    return;
  }
  fwht_groups_warp(x, dpad / 128);
  __syncthreads();
  for (int c = threadIdx.x; c < dpad; c += blockDim.x) lm_in[(size_t)r * dpad + c] = x[c];
}

cudaError_t launch_final(const Geo& G, const RowBatch& rb, const float* lanes,
                         const float* final_norm, float* lm_in, cudaStream_t st, SplitOut so,
                         unsigned long long* keys) {
  if (rb.M <= 0) return cudaSuccess;
  const int dpad = (G.d + 127) / 128 * 128;
  return launch_pdl(final_kernel, dim3(rb.M), dim3(256), (32 + dpad) * sizeof(float), st, G, lanes, final_norm,
                    lm_in, so, keys);
}

// Greedy pick: the first maximum, as argmax (v3_engine.rs:410-420) keeps the
// lowest index on ties and never picks a NaN.
__global__ void argmax_kernel(const float* __restrict__ logits, int n, int ld, uint32_t* out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int r = blockIdx.x;
  const float* x = logits + (size_t)r * ld;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = x[i];
    if (v > best || (v == best && i < idx)) {
      best = v;
      idx = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) {
    bv[wid] = best;
    bi[wid] = idx;
  }
  __syncthreads();
  if (wid == 0) {
    best = lane < nw ? bv[lane] : -INFINITY;
    idx = lane < nw ? bi[lane] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > best || (ov == best && oi < idx)) {
        best = ov;
        idx = oi;
      }
    }
    if (lane == 0) out[r] = idx == 0x7fffffff ? 0u : (uint32_t)idx;
  }
}

cudaError_t launch_argmax(const float* logits, int M, int n, int ld, uint32_t* out, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  return launch_pdl(argmax_kernel, dim3(M), dim3(256), 0, st, logits, n, ld, out);
}

__global__ void argmax_keys_kernel(const unsigned long long* __restrict__ keys, int M, uint32_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < M) out[r] = argmax_pick(keys[r]);
}

cudaError_t launch_argmax_keys(const unsigned long long* keys, int M, uint32_t* out, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  return launch_pdl(argmax_keys_kernel, dim3((M + 255) / 256), dim3(256), 0, st, keys, M, out);
}

// ---------------------------------------------------------------- step bookkeeping
__global__ void step_begin_kernel(RowInfo* rows, SessDesc* const* sess, int M) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M) return;
  SessDesc* s = sess[i];
  rows[i].s = s;
  rows[i].pos = s->pos;
  rows[i].base = -1;
  rows[i].len = -1;
}

cudaError_t launch_step_begin(const RowBatch& rb, SessDesc* const* sess, cudaStream_t st) {
  if (rb.M <= 0) return cudaSuccess;
  step_begin_kernel<<<(rb.M + 127) / 128, 128, 0, st>>>(rb.rows, sess, rb.M);
  return cudaGetLastError();
}

// Decode: record the token in the history ring and advance (cache.rs:276, :530).
// Prefill: seed the ring with the last tokens and set the position (cache.rs:505-520).
__global__ void step_end_kernel(RowBatch rb) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rb.M) return;
  RowInfo ri = rb.rows[i];
  if (rb.mode == MODE_DECODE) {
    ri.s->toks[ri.pos & 3] = rb.tokens[i];
    ri.s->pos = ri.pos + 1;
  } else {
    if (ri.pos >= ri.len - 4) ri.s->toks[ri.pos & 3] = rb.tokens[i];
    if (ri.pos == ri.len - 1) ri.s->pos = ri.len;
  }
}

cudaError_t launch_step_end(const RowBatch& rb, cudaStream_t st) {
  if (rb.M <= 0) return cudaSuccess;
  step_end_kernel<<<(rb.M + 127) / 128, 128, 0, st>>>(rb);
  return cudaGetLastError();
}

}  // namespace nb
