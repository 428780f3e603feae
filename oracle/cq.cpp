// TEST INFRASTRUCTURE — CPU restatement of crates/needle-core/src/cq.rs,
// hadamard.rs, math.rs, kernels.rs, norm.rs and ops.rs (bynds/needle-rs).
// See oracle.hpp for the role of this code.
#include <cmath>
#include <cstring>
#include <omp.h>

#include "oracle.hpp"

namespace oracle {

// math.rs:53-68 — exact binary16 -> f32.
float f16_to_f32(uint16_t bits) {
  uint32_t sign = (uint32_t)(bits >> 15) << 31;
  uint32_t exp = (bits >> 10) & 0x1F;
  uint32_t mant = bits & 0x3FF;
  if (exp == 0) {
    float val = (float)mant / (float)(1u << 24);
    return sign ? -val : val;
  }
  uint32_t u;
  if (exp == 31) {
    u = sign | 0x7F800000u | (mant << 13);
  } else {
    u = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// cq.rs:107-115
size_t packed_row_bytes(size_t in_padded, uint8_t bits) {
  size_t eff = bits == TERNARY_RECORD_BITS ? 2 : bits;
  return in_padded * eff / 8;
}

// hadamard.rs:24-42 — Sylvester butterfly, unnormalised.
void fwht(float* x, size_t n) {
  size_t h = 1;
  while (h < n) {
    for (size_t i = 0; i < n; i += h << 1) {
      for (size_t j = i; j < i + h; ++j) {
        float a = x[j], b = x[j + h];
        x[j] = a + b;
        x[j + h] = a - b;
      }
    }
    h <<= 1;
  }
}

// hadamard.rs:48-55
void fwht_normalized(float* x, size_t n) {
  fwht(x, n);
  float inv = 1.0f / sqrtf((float)n);
  for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

// cq.rs:914-925 — LSB-first continuous bitstream per row.
static inline uint32_t read_bits(const uint8_t* row, size_t bit, size_t bits, uint32_t mask) {
  size_t byte = bit / 8, shift = bit % 8;
  uint32_t lo = row[byte];
  uint32_t hi = (shift + bits > 8) ? row[byte + 1] : 0;
  return ((lo | (hi << 8)) >> shift) & mask;
}

static inline size_t ternary_index(uint32_t code) {
  // cq.rs:948-955: crumb codes 3,0,1 are trit indices 0,1,2; 2 maps to zero.
  switch (code) {
    case 3: return 0;
    case 0: return 1;
    case 1: return 2;
    default: return 1;
  }
}

// cq.rs:932-964 — byte decode table for widths dividing a byte.
static void build_lut(uint8_t bits, const std::vector<float>& levels, size_t* per_byte_out,
                      std::vector<float>* lut) {
  bool ternary = bits == TERNARY_RECORD_BITS;
  size_t width = ternary ? 2 : bits;
  size_t per_byte;
  if (width == 2) per_byte = 4;
  else if (width == 4) per_byte = 2;
  else {
    *per_byte_out = 0;
    lut->clear();
    return;
  }
  uint32_t mask = (1u << width) - 1;
  lut->assign(256 * per_byte, 0.f);
  for (size_t byte = 0; byte < 256; ++byte) {
    for (size_t k = 0; k < per_byte; ++k) {
      uint32_t code = ((uint32_t)byte >> (k * width)) & mask;
      size_t idx = ternary ? ternary_index(code) : code;
      (*lut)[byte * per_byte + k] = levels[idx];
    }
  }
  *per_byte_out = per_byte;
}

// cq.rs:181-238
std::string CqWeight::from_blob(const uint8_t* blob, size_t blob_len, size_t out_feat,
                                size_t in_feat, size_t group, uint8_t bits,
                                const float* codebook, size_t codebook_len, CqWeight* w) {
  if (out_feat == 0 || in_feat == 0) return "cq: empty shape";
  if (group == 0 || group % 8 != 0 || (group & (group - 1)) != 0 || group > MAX_GROUP)
    return "cq: bad group " + std::to_string(group);
  std::vector<float> levels;
  if (bits == TERNARY_RECORD_BITS) {
    float s = TERNARY_CENTROID / sqrtf((float)group);
    levels = {-s, 0.0f, s};
  } else {
    if (codebook_len != CODEBOOK_LEN) return "cq: bad codebook length";
    if (bits == 2) levels.assign(codebook, codebook + 4);
    else if (bits == 3) levels.assign(codebook + 4, codebook + 12);
    else if (bits == 4) levels.assign(codebook + 12, codebook + 28);
    else return "cq: unsupported bits " + std::to_string(bits);
  }
  size_t in_padded = (in_feat + group - 1) / group * group;
  size_t num_groups = in_padded / group;
  size_t row_bytes = packed_row_bytes(in_padded, bits);
  size_t n_packed = out_feat * row_bytes;
  size_t n_norm = out_feat * num_groups * 2;
  if (blob_len < n_packed + n_norm) return "cq: short blob";
  w->packed.assign(blob, blob + n_packed);
  w->norms.resize(out_feat * num_groups);
  for (size_t i = 0; i < out_feat * num_groups; ++i) {
    uint16_t h = (uint16_t)blob[n_packed + 2 * i] | ((uint16_t)blob[n_packed + 2 * i + 1] << 8);
    w->norms[i] = f16_to_f32(h);
  }
  build_lut(bits, levels, &w->per_byte, &w->lut);
  w->row_bytes = row_bytes;
  w->num_groups = num_groups;
  w->out_feat = out_feat;
  w->in_feat = in_feat;
  w->in_padded = in_padded;
  w->group = group;
  w->bits = bits;
  w->levels = levels;
  return "";
}

// cq.rs:264-274
void CqWeight::prepare_input(const float* x, float* xh) const {
  std::memcpy(xh, x, in_feat * sizeof(float));
  for (size_t i = in_feat; i < in_padded; ++i) xh[i] = 0.0f;
  for (size_t g = 0; g < in_padded; g += group) fwht_normalized(xh + g, group);
}

void CqWeight::matvec(const float* x, float* y) const {
  std::vector<float> xh(in_padded);
  prepare_input(x, xh.data());
  matvec_rows_prepared(xh.data(), 0, y, out_feat);
}

// cq.rs:838-873 — one group, ACC_LANES lanes, P levels per byte.
template <size_t P>
static inline float dot_group(const float* lut, const uint8_t* gbytes, size_t nbytes,
                              const float* gx) {
  constexpr size_t per_iter = ACC_LANES / P;
  float lanes[ACC_LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t full = nbytes - nbytes % per_iter;
  size_t bi = 0;
  while (bi < full) {
    float vals[ACC_LANES];
    for (size_t t = 0; t < per_iter; ++t) {
      const float* e = lut + (size_t)gbytes[bi + t] * P;
      for (size_t k = 0; k < P; ++k) vals[t * P + k] = e[k];
    }
    const float* xs = gx + bi * P;
    for (size_t k = 0; k < ACC_LANES; ++k) lanes[k] += vals[k] * xs[k];
    bi += per_iter;
  }
  float acc = 0.0f;
  for (size_t k = 0; k < ACC_LANES; ++k) acc += lanes[k];
  for (size_t b = bi; b < nbytes; ++b) {
    const float* e = lut + (size_t)gbytes[b] * P;
    for (size_t k = 0; k < P; ++k) acc += e[k] * gx[b * P + k];
  }
  return acc;
}

// cq.rs:879-895 — same lane order over an already decoded group.
static inline float group_dot_lanes(const float* u, const float* x, size_t n) {
  size_t chunks = n / ACC_LANES;
  float lanes[ACC_LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t c = 0; c < chunks; ++c)
    for (size_t k = 0; k < ACC_LANES; ++k) lanes[k] += u[c * ACC_LANES + k] * x[c * ACC_LANES + k];
  float s = 0.0f;
  for (size_t k = 0; k < ACC_LANES; ++k) s += lanes[k];
  for (size_t k = chunks * ACC_LANES; k < n; ++k) s += u[k] * x[k];
  return s;
}

static inline float group_dot_serial(const float* u, const float* x, size_t n) {
  float s = 0.0f;
  for (size_t k = 0; k < n; ++k) s += u[k] * x[k];
  return s;
}

// cq.rs:325-334 dispatch + :721-735 (LUT path) + :738-757 (generic path).
void CqWeight::matvec_rows_serial(const float* xh, size_t row_start, float* y,
                                  size_t rows) const {
  if (per_byte == 4 || per_byte == 2) {
    size_t bpg = group / per_byte;
    for (size_t yi = 0; yi < rows; ++yi) {
      size_t o = row_start + yi;
      const uint8_t* row = packed.data() + o * row_bytes;
      const float* rn = norms.data() + o * num_groups;
      float total = 0.0f;
      for (size_t g = 0; g < num_groups; ++g) {
        float d = per_byte == 4 ? dot_group<4>(lut.data(), row + g * bpg, bpg, xh + g * group)
                                : dot_group<2>(lut.data(), row + g * bpg, bpg, xh + g * group);
        total += rn[g] * d;
      }
      y[yi] = total;
    }
  } else {
    uint32_t mask = (1u << bits) - 1;
    for (size_t yi = 0; yi < rows; ++yi) {
      size_t o = row_start + yi;
      const uint8_t* row = packed.data() + o * row_bytes;
      const float* rn = norms.data() + o * num_groups;
      float total = 0.0f;
      for (size_t g = 0; g < num_groups; ++g) {
        const float* gx = xh + g * group;
        float acc = 0.0f;
        for (size_t k = 0; k < group; ++k) {
          uint32_t idx = read_bits(row, (g * group + k) * bits, bits, mask);
          acc += levels[idx] * gx[k];
        }
        total += rn[g] * acc;
      }
      y[yi] = total;
    }
  }
}

// cq.rs:301-323 — the rayon row split, mirrored with OpenMP. Bit-identical to
// the serial path: each row is computed exactly as the serial path computes it.
static constexpr size_t MIN_PAR_ROWS = 64;    // cq.rs:812
static constexpr size_t MIN_PAR_BATCH = 8;    // cq.rs:816
static constexpr size_t PAR_MIN_MACS = 1u << 20;  // cq.rs:820

void CqWeight::matvec_rows_prepared(const float* xh, size_t row_start, float* y,
                                    size_t rows) const {
  int nt = omp_get_max_threads();
  if (nt > 1 && rows >= 2 * MIN_PAR_ROWS && rows * in_padded >= PAR_MIN_MACS) {
    size_t chunk = std::max((rows + nt - 1) / nt, MIN_PAR_ROWS);
    size_t nchunks = (rows + chunk - 1) / chunk;
#pragma omp parallel for schedule(static)
    for (long ci = 0; ci < (long)nchunks; ++ci) {
      size_t r0 = (size_t)ci * chunk;
      size_t n = std::min(chunk, rows - r0);
      matvec_rows_serial(xh, row_start + r0, y + r0, n);
    }
    return;
  }
  matvec_rows_serial(xh, row_start, y, rows);
}

// cq.rs:381-412 — the deliberately simple single-accumulator reference.
void CqWeight::matvec_prepared_reference(const float* xh, float* y) const {
  size_t b = bits == TERNARY_RECORD_BITS ? 2 : bits;
  uint32_t mask = (1u << b) - 1;
  for (size_t o = 0; o < out_feat; ++o) {
    const uint8_t* row = packed.data() + o * row_bytes;
    float total = 0.0f;
    for (size_t g = 0; g < num_groups; ++g) {
      float norm = norms[o * num_groups + g];
      float acc = 0.0f;
      for (size_t k = 0; k < group; ++k) {
        uint32_t code = read_bits(row, (g * group + k) * b, b, mask);
        size_t idx = bits == TERNARY_RECORD_BITS ? ternary_index(code) : code;
        acc += levels[idx] * xh[g * group + k];
      }
      total += norm * acc;
    }
    y[o] = total;
  }
}

// cq.rs:791-809
void CqWeight::decode_group(const uint8_t* row, size_t g, float norm, float* buf) const {
  if (per_byte != 0) {
    size_t p = per_byte, bpg = group / p;
    const uint8_t* gb = row + g * bpg;
    for (size_t bi = 0; bi < bpg; ++bi)
      for (size_t k = 0; k < p; ++k) buf[bi * p + k] = lut[(size_t)gb[bi] * p + k] * norm;
  } else {
    uint32_t mask = (1u << bits) - 1;
    for (size_t k = 0; k < group; ++k) {
      uint32_t idx = read_bits(row, (g * group + k) * bits, bits, mask);
      buf[k] = levels[idx] * norm;
    }
  }
}

// cq.rs:632-679 — decode each group once, apply to every batch row.
void CqWeight::matmul_rows_serial(const float* xh, size_t batch, size_t row_start, size_t rows,
                                  float* y) const {
  std::vector<float> ug(group), acc(batch);
  bool lanewise = per_byte != 0;
  size_t stride = in_padded;
  for (size_t r = 0; r < rows; ++r) {
    size_t o = row_start + r;
    const uint8_t* row = packed.data() + o * row_bytes;
    const float* rn = norms.data() + o * num_groups;
    std::fill(acc.begin(), acc.end(), 0.0f);
    for (size_t g = 0; g < num_groups; ++g) {
      decode_group(row, g, 1.0f, ug.data());
      size_t base = g * group;
      for (size_t b = 0; b < batch; ++b) {
        const float* gx = xh + b * stride + base;
        float s = lanewise ? group_dot_lanes(ug.data(), gx, group)
                           : group_dot_serial(ug.data(), gx, group);
        acc[b] += rn[g] * s;
      }
    }
    for (size_t b = 0; b < batch; ++b) y[b * rows + r] = acc[b];
  }
}

// cq.rs:446-472 with the row-band (:482) and batch-band (:549) splits.
void CqWeight::matmul_rows_prepared(const float* xh, size_t batch, size_t row_start,
                                    size_t rows, float* y) const {
  int nt = omp_get_max_threads();
  if (nt > 1 && rows * batch * in_padded >= PAR_MIN_MACS) {
    if (rows >= 2 * MIN_PAR_ROWS) {
      size_t chunk = std::max((rows + nt - 1) / nt, MIN_PAR_ROWS);
      size_t nb = (rows + chunk - 1) / chunk;
#pragma omp parallel for schedule(static)
      for (long bi = 0; bi < (long)nb; ++bi) {
        size_t r0 = (size_t)bi * chunk, band = std::min(chunk, rows - r0);
        std::vector<float> local(batch * band);
        matmul_rows_serial(xh, batch, row_start + r0, band, local.data());
        for (size_t b = 0; b < batch; ++b)
          std::memcpy(y + b * rows + r0, local.data() + b * band, band * sizeof(float));
      }
      return;
    }
    if (batch >= 2 * MIN_PAR_BATCH) {
      size_t band = std::max((batch + nt - 1) / nt, MIN_PAR_BATCH);
      size_t nb = (batch + band - 1) / band;
#pragma omp parallel for schedule(static)
      for (long ci = 0; ci < (long)nb; ++ci) {
        size_t b0 = (size_t)ci * band, n = std::min(band, batch - b0);
        matmul_rows_serial(xh + b0 * in_padded, n, row_start, rows, y + b0 * rows);
      }
      return;
    }
  }
  matmul_rows_serial(xh, batch, row_start, rows, y);
}

// cq.rs:763-779
void CqWeight::dequantize_row(size_t o, float* out) const {
  const uint8_t* row = packed.data() + o * row_bytes;
  const float* rn = norms.data() + o * num_groups;
  std::vector<float> buf(group);
  for (size_t g = 0; g < num_groups; ++g) {
    decode_group(row, g, rn[g], buf.data());
    fwht_normalized(buf.data(), group);
    size_t base = g * group;
    for (size_t k = 0; k < group; ++k)
      if (base + k < in_feat) out[base + k] = buf[k];
  }
}

// kernels.rs:32-40
void rms_unit_to(const float* x, float* out, size_t n) {
  float sq = 0.0f;
  for (size_t i = 0; i < n; ++i) sq += x[i] * x[i];
  float mean_sq = sq / (float)n;
  float inv = 1.0f / sqrtf(mean_sq + EPS);
  for (size_t i = 0; i < n; ++i) out[i] = x[i] * inv;
}

// norm.rs:23-30
void zc_rms_norm_vec(float* x, const float* scale, size_t n) {
  float sq = 0.0f;
  for (size_t i = 0; i < n; ++i) sq += x[i] * x[i];
  float mean_sq = sq / (float)n;
  float inv = 1.0f / sqrtf(mean_sq + EPS);
  for (size_t i = 0; i < n; ++i) x[i] = (1.0f + scale[i]) * x[i] * inv;
}

// kernels.rs:78-85
static float logsumexp(const float* x, size_t n) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, x[i]);
  if (!std::isfinite(mx)) return mx;
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) sum += expf(x[i] - mx);
  return mx + logf(sum);
}

// kernels.rs:46-76
void sinkhorn(float* m, size_t n) {
  for (int it = 0; it < SINKHORN_ITERS; ++it) {
    for (size_t i = 0; i < n; ++i) {
      float lse = logsumexp(m + i * n, n);
      for (size_t j = 0; j < n; ++j) m[i * n + j] -= lse;
    }
    for (size_t j = 0; j < n; ++j) {
      float mx = -INFINITY;
      for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, m[i * n + j]);
      float sum = 0.0f;
      for (size_t i = 0; i < n; ++i) sum += expf(m[i * n + j] - mx);
      float lse = mx + logf(sum);
      for (size_t i = 0; i < n; ++i) m[i * n + j] -= lse;
    }
  }
  for (size_t i = 0; i < n * n; ++i) m[i] = expf(m[i]);
}

float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }  // ops.rs:41
float silu(float x) { return x * sigmoid(x); }               // ops.rs:118

}  // namespace oracle
