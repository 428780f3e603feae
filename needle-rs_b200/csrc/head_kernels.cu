// Probe heads over the per-layer cells (crates/needle-core/src/v3/heads.rs):
// the cells are captured during a forward (the scaled embedding, then each
// layer's lane stream meaned over lanes, model.rs:494-502, :910-926), pooled
// over positions per (cell, probe), then over (cell, probe) pairs per query,
// and projected. Used by the confidence head; a single sequence at a time.
#include "common.cuh"
#include "kernels.hpp"
#include "launch_util.hpp"

namespace nb {
namespace {

// out[r] = lane 0 of row r (copy0: cell 0, the embedding every lane holds), or
// the mean of its lanes, summed in lane order and divided by the lane count.
__global__ void lane_mean_kernel(const float* __restrict__ lanes, int n, int d, int copy0, float* __restrict__ out) {
  const int r = blockIdx.x;
  const float* lr = lanes + (size_t)r * n * d;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float a;
    if (copy0) {
      a = lr[c];
    } else {
      a = 0.f;
      for (int l = 0; l < n; ++l) a += lr[(size_t)l * d + c];
      a = a / (float)n;
    }
    out[(size_t)r * d + c] = a;
  }
}

constexpr int HP_THREADS = 256, HP_MAXC = 4;  // d_model <= 1024

// One CTA per (cell, probe) pair (heads.rs:72-111): scores probe . cell_t /
// sqrt(d) for every position t, their softmax, the weighted mean of the cells,
// rms_unit and the pair's gain.
__global__ void __launch_bounds__(HP_THREADS) probe_pool_kernel(const float* __restrict__ cells, int seq, int d,
                                                                int k, const float* __restrict__ probes,
                                                                const float* __restrict__ gain,
                                                                float* __restrict__ r) {
  extern __shared__ float sc[];  // [seq]
  __shared__ float red[32];
  const int pair = blockIdx.x, cell = pair / k;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  const float* C = cells + (size_t)cell * seq * d;
  const float* pr = probes + (size_t)pair * d;
  const float scale = 1.0f / sqrtf((float)d);
  for (int t = wid; t < seq; t += nw) {
    float acc = 0.f;
    for (int c = lane; c < d; c += 32) acc += C[(size_t)t * d + c] * pr[c];
    acc = warp_sum(acc);
    if (lane == 0) sc[t] = acc * scale;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int t = tid; t < seq; t += blockDim.x) mx = fmaxf(mx, sc[t]);
  mx = block_max(mx, red);
  float sum = 0.f;
  for (int t = tid; t < seq; t += blockDim.x) {
    const float e = expf(sc[t] - mx);
    sc[t] = e;
    sum += e;
  }
  sum = block_sum(sum, red);  // its barriers also publish sc
  const float inv = 1.0f / sum;
  float acc[HP_MAXC] = {0.f, 0.f, 0.f, 0.f};
  for (int t = 0; t < seq; ++t) {
    const float w = sc[t] * inv;
#pragma unroll
    for (int i = 0; i < HP_MAXC; ++i) {
      const int c = tid + i * HP_THREADS;
      if (c < d) acc[i] += w * C[(size_t)t * d + c];
    }
  }
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < HP_MAXC; ++i)
    if (tid + i * HP_THREADS < d) sq += acc[i] * acc[i];
  sq = block_sum(sq, red);
  const float g = 1.0f / sqrtf(sq / (float)d + 1e-6f);  // rms_unit, kernels.rs:22-28
  const float gn = gain[pair];
#pragma unroll
  for (int i = 0; i < HP_MAXC; ++i) {
    const int c = tid + i * HP_THREADS;
    if (c < d) r[(size_t)pair * d + c] = acc[i] * g * gn;
  }
}

// One CTA (heads.rs:120-177): per query a softmax over the m pairs of the
// scaled dot plus row bias, the weighted mean of the pairs, then the
// projection of the flattened (queries * d) vector plus the bias.
__global__ void __launch_bounds__(HP_THREADS) probe_finish_kernel(const float* __restrict__ r, int m, int d, int q,
                                                                  const float* __restrict__ query,
                                                                  const float* __restrict__ row_bias,
                                                                  const float* __restrict__ proj,
                                                                  const float* __restrict__ bias, int out_dim,
                                                                  float* __restrict__ out) {
  extern __shared__ float sm[];
  float* u = sm;             // [m]
  float* pooled = sm + m;    // [q * d]
  __shared__ float red[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  const float scale = 1.0f / sqrtf((float)d);
  for (int qi = 0; qi < q; ++qi) {
    const float* qv = query + (size_t)qi * d;
    for (int idx = wid; idx < m; idx += nw) {
      float acc = 0.f;
      for (int c = lane; c < d; c += 32) acc += r[(size_t)idx * d + c] * qv[c];
      acc = warp_sum(acc);
      if (lane == 0) u[idx] = acc * scale + row_bias[(size_t)qi * m + idx];
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int idx = tid; idx < m; idx += blockDim.x) mx = fmaxf(mx, u[idx]);
    mx = block_max(mx, red);
    float sum = 0.f;
    for (int idx = tid; idx < m; idx += blockDim.x) {
      const float e = expf(u[idx] - mx);
      u[idx] = e;
      sum += e;
    }
    sum = block_sum(sum, red);
    const float inv = 1.0f / sum;
    for (int c = tid; c < d; c += blockDim.x) {
      float a = 0.f;
      for (int idx = 0; idx < m; ++idx) a += (u[idx] * inv) * r[(size_t)idx * d + c];
      pooled[(size_t)qi * d + c] = a;
    }
    __syncthreads();  // u is rewritten by the next query
  }
  for (int o = 0; o < out_dim; ++o) {
    float acc = 0.f;
    for (int i = tid; i < q * d; i += blockDim.x) acc += proj[(size_t)o * q * d + i] * pooled[i];
    acc = block_sum(acc, red);
    if (tid == 0) out[o] = acc + bias[o];
  }
}

}  // namespace

cudaError_t launch_lane_mean(const float* lanes, int M, int n, int d, bool copy0, float* out, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  lane_mean_kernel<<<M, 256, 0, st>>>(lanes, n, d, copy0 ? 1 : 0, out);
  return cudaGetLastError();
}

cudaError_t launch_probe_head(const float* cells, int seq, int d, const ProbeHeadDev& h, float* r, float* out,
                              cudaStream_t st) {
  if (seq <= 0 || d > HP_THREADS * HP_MAXC || h.queries <= 0 || h.out_dim <= 0) return cudaErrorInvalidValue;
  const int m = h.cells * h.probes_per_cell;
  const size_t s1 = (size_t)seq * sizeof(float), s2 = ((size_t)m + (size_t)h.queries * d) * sizeof(float);
  cudaError_t e = allow_smem((const void*)probe_pool_kernel, s1);
  if (e == cudaSuccess) e = allow_smem((const void*)probe_finish_kernel, s2);
  if (e != cudaSuccess) return e;
  probe_pool_kernel<<<m, HP_THREADS, s1, st>>>(cells, seq, d, h.probes_per_cell, h.probes, h.gain, r);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  probe_finish_kernel<<<1, HP_THREADS, s2, st>>>(r, m, d, h.queries, h.query, h.row_bias, h.proj, h.bias,
                                                 h.out_dim, out);
  return cudaGetLastError();
}

}  // namespace nb
