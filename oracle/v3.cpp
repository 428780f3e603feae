// TEST INFRASTRUCTURE — CPU restatement of crates/needle-core/src/v3/*.rs
// (config, attention, cache, engram, mhc, kernels, model) of bynds/needle-rs.
// See oracle.hpp for the role of this code.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "oracle.hpp"

namespace oracle {

// ---------------------------------------------------------------- config.rs
int V3Engram::site_of(size_t layer) const {  // config.rs:38
  for (size_t i = 0; i < sites.size(); ++i)
    if (sites[i] == layer) return (int)i;
  return -1;
}
size_t V3Engram::max_order() const {
  size_t m = 0;
  for (size_t o : orders) m = std::max(m, o);
  return m == 0 ? 1 : m;
}
bool V3Config::is_global(size_t layer) const {  // config.rs:209
  return std::find(global_layers.begin(), global_layers.end(), layer) != global_layers.end();
}
size_t V3Config::attention_span(size_t layer) const {  // config.rs:216
  if (is_global(layer) || sliding_window == 0) return 0;
  return sliding_window;
}
size_t V3Config::kv_bytes(size_t seq_len, size_t bytes_per) const {  // config.rs:234
  size_t per_pos = num_kv_heads * (qk_head_dim + v_head_dim);
  size_t total = 0;
  for (size_t l = 0; l < num_layers; ++l) {
    size_t w = attention_span(l);
    size_t slots = w ? std::min(seq_len, w) : seq_len;
    total += slots * per_pos * bytes_per;
  }
  return total;
}
size_t V3Config::kv_bytes_at(size_t seq_len, KvPrecision p) const {  // config.rs:255
  if (p == KvPrecision::F32) return kv_bytes(seq_len, 4);
  size_t per_pos = num_kv_heads * (qk_head_dim + v_head_dim) + num_kv_heads * 8;
  size_t total = 0;
  for (size_t l = 0; l < num_layers; ++l) {
    size_t w = attention_span(l);
    size_t slots = w ? std::min(seq_len, w) : seq_len;
    total += slots * per_pos;
  }
  return total;
}

// ---------------------------------------------------------------- attention.rs
// attention.rs:82-100
void causal_depthwise_conv(float* buf, const float* taps, size_t seq, size_t dim,
                           size_t n_taps) {
  if (n_taps == 0) return;
  for (size_t tt = seq; tt-- > 0;) {
    for (size_t c = 0; c < dim; ++c) {
      float acc = 0.0f;
      for (size_t j = 0; j < n_taps; ++j) {
        if (j > tt) break;
        acc += taps[j * dim + c] * buf[(tt - j) * dim + c];
      }
      buf[tt * dim + c] = acc;
    }
  }
}

// attention.rs:107-143
void norm_and_rope(float* buf, const float* scale, const float* cos_t, const float* sin_t,
                   size_t seq, size_t heads, size_t head_dim) {
  size_t half = head_dim / 2;
  for (size_t t = 0; t < seq; ++t) {
    for (size_t h = 0; h < heads; ++h) {
      float* x = buf + (t * heads + h) * head_dim;
      float sq = 0.0f;
      for (size_t i = 0; i < head_dim; ++i) sq += x[i] * x[i];
      float rms = sqrtf(sq / (float)head_dim + 1e-6f);
      for (size_t i = 0; i < head_dim; ++i) x[i] = (1.0f + scale[i]) * x[i] / rms;
      for (size_t i = 0; i < half; ++i) {
        float c = cos_t[t * half + i], s = sin_t[t * half + i];
        float x1 = x[i], x2 = x[half + i];
        x[i] = x1 * c - x2 * s;
        x[half + i] = x2 * c + x1 * s;
      }
    }
  }
}

// attention.rs:177-216 — F32View / Int8View with the hoisted per-head scale.
static inline float kv_dot(const KvStore& kv, const float* q, size_t off, size_t len,
                           size_t scale_at) {
  float a = 0.0f;
  if (!kv.int8) {
    for (size_t i = 0; i < len; ++i) a += q[i] * kv.k[off + i];
    return a;
  }
  for (size_t i = 0; i < len; ++i) a += q[i] * (float)kv.kq[off + i];
  return a * kv.k_scale[scale_at];
}
static inline void kv_accum(const KvStore& kv, float w, size_t off, float* out, size_t n,
                            size_t scale_at) {
  if (!kv.int8) {
    for (size_t i = 0; i < n; ++i) out[i] += w * kv.v[off + i];
    return;
  }
  float ws = w * kv.v_scale[scale_at];
  for (size_t i = 0; i < n; ++i) out[i] += ws * (float)kv.vq[off + i];
}

// attention.rs:241-287
void attend(const float* q, const KvStore& kv, const AttnDims& d, size_t window, float* out) {
  float scale = 1.0f / sqrtf((float)d.qk_head_dim);
  size_t repeat = d.num_heads / d.num_kv_heads;
  std::vector<float> scores(d.seq);
  for (size_t t = 0; t < d.seq; ++t) {
    size_t lo = (window && t + 1 > window) ? t + 1 - window : 0;
    for (size_t h = 0; h < d.num_heads; ++h) {
      size_t kvh = h / repeat;
      const float* qv = q + (t * d.num_heads + h) * d.qk_head_dim;
      float mx = -INFINITY;
      for (size_t n = lo; n <= t; ++n) {
        size_t ko = (n * d.num_kv_heads + kvh) * d.qk_head_dim;
        float acc = kv_dot(kv, qv, ko, d.qk_head_dim, n * d.num_kv_heads + kvh);
        scores[n] = acc * scale;
        if (scores[n] > mx) mx = scores[n];
      }
      float sum = 0.0f;
      for (size_t n = lo; n <= t; ++n) {
        scores[n] = expf(scores[n] - mx);
        sum += scores[n];
      }
      float inv = 1.0f / sum;
      float* o = out + (t * d.num_heads + h) * d.v_head_dim;
      for (size_t i = 0; i < d.v_head_dim; ++i) o[i] = 0.0f;
      for (size_t n = lo; n <= t; ++n) {
        float w = scores[n] * inv;
        size_t vo = (n * d.num_kv_heads + kvh) * d.v_head_dim;
        kv_accum(kv, w, vo, o, d.v_head_dim, n * d.num_kv_heads + kvh);
      }
    }
  }
}

// attention.rs:327-377
void attend_step(const float* q, const KvStore& kv, size_t slots, size_t lo, size_t hi,
                 const AttnDims& d, float* out) {
  float scale = 1.0f / sqrtf((float)d.qk_head_dim);
  size_t repeat = d.num_heads / d.num_kv_heads;
  size_t span = hi - lo + 1;
  std::vector<float> scores(span);
  for (size_t h = 0; h < d.num_heads; ++h) {
    size_t kvh = h / repeat;
    const float* qv = q + h * d.qk_head_dim;
    float mx = -INFINITY;
    for (size_t i = 0; i < span; ++i) {
      size_t slot = (lo + i) % slots;
      size_t ko = (slot * d.num_kv_heads + kvh) * d.qk_head_dim;
      float acc = kv_dot(kv, qv, ko, d.qk_head_dim, slot * d.num_kv_heads + kvh);
      scores[i] = acc * scale;
      if (scores[i] > mx) mx = scores[i];
    }
    float sum = 0.0f;
    for (size_t i = 0; i < span; ++i) {
      scores[i] = expf(scores[i] - mx);
      sum += scores[i];
    }
    float inv = 1.0f / sum;
    float* o = out + h * d.v_head_dim;
    for (size_t i = 0; i < d.v_head_dim; ++i) o[i] = 0.0f;
    for (size_t i = 0; i < span; ++i) {
      float w = scores[i] * inv;
      size_t slot = (lo + i) % slots;
      size_t vo = (slot * d.num_kv_heads + kvh) * d.v_head_dim;
      kv_accum(kv, w, vo, o, d.v_head_dim, slot * d.num_kv_heads + kvh);
    }
  }
}

// ---------------------------------------------------------------- cache.rs
// cache.rs:81-93
static void quant_scale(const float* x, size_t n, uint32_t bits, float* scale, float* inv,
                        float* qmax) {
  *qmax = (float)((1u << (bits - 1)) - 1);
  float absmax = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float a = x[i] < 0.0f ? -x[i] : x[i];
    if (a > absmax) absmax = a;
  }
  *scale = absmax > 0.0f ? absmax / *qmax : 1.0f;
  *inv = 1.0f / *scale;
}

static inline float clampf(float v, float lo, float hi) {  // Rust f32::clamp
  if (v < lo) return lo;
  if (v > hi) return hi;
  return v;
}

// cache.rs:68-73 — roundf is half away from zero, as Rust's f32::round.
void fake_quant_vec(float* x, size_t n, uint32_t bits) {
  float scale, inv, qmax;
  quant_scale(x, n, bits, &scale, &inv, &qmax);
  for (size_t i = 0; i < n; ++i) x[i] = clampf(roundf(x[i] * inv), -qmax - 1.0f, qmax) * scale;
}

// cache.rs:100-106
float quant_into(const float* src, int8_t* dst, size_t n) {
  float scale, inv, qmax;
  quant_scale(src, n, 8, &scale, &inv, &qmax);
  for (size_t i = 0; i < n; ++i) dst[i] = (int8_t)clampf(roundf(src[i] * inv), -qmax - 1.0f, qmax);
  return scale;
}

// cache.rs:115-122
void quantize_rows(const float* x, size_t len, size_t head_dim, std::vector<int8_t>* ints,
                   std::vector<float>* scales) {
  size_t rows = len / head_dim;
  ints->assign(len, 0);
  scales->assign(rows, 1.0f);
  for (size_t r = 0; r < rows; ++r)
    (*scales)[r] = quant_into(x + r * head_dim, ints->data() + r * head_dim, head_dim);
}

// cache.rs:177-238
V3Cache::V3Cache(const V3Config& c, size_t hint, KvPrecision p) : cfg(c), precision(p) {
  hint = std::min(std::max(hint, (size_t)1), cfg.max_seq_len);
  size_t taps_tail = cfg.qkv_conv_taps > 0 ? cfg.qkv_conv_taps - 1 : 0;
  bool int8 = p == KvPrecision::Int8;
  layers.resize(cfg.num_layers);
  for (size_t li = 0; li < cfg.num_layers; ++li) {
    LayerCache& l = layers[li];
    size_t w = cfg.attention_span(li);
    l.cap = w ? std::min(w, cfg.max_seq_len) : cfg.max_seq_len;
    l.slots = std::min(hint, l.cap);
    size_t heads = l.slots * cfg.num_kv_heads;
    if (int8) {
      l.kq.assign(l.slots * cfg.k_dim(), 0);
      l.vq.assign(l.slots * cfg.v_dim(), 0);
      l.k_scale.assign(heads, 1.0f);
      l.v_scale.assign(heads, 1.0f);
    } else {
      l.k.assign(l.slots * cfg.k_dim(), 0.0f);
      l.v.assign(l.slots * cfg.v_dim(), 0.0f);
    }
    l.q_tail.assign(taps_tail * cfg.q_dim(), 0.0f);
    l.k_tail.assign(taps_tail * cfg.k_dim(), 0.0f);
    l.v_tail.assign(taps_tail * cfg.v_dim(), 0.0f);
  }
  size_t reach = (cfg.engram.conv_taps > 0 ? cfg.engram.conv_taps - 1 : 0) * cfg.engram.conv_dilation;
  engram_tail.assign(cfg.engram.sites.size(), std::vector<float>(reach * cfg.d_model, 0.0f));
  pos = 0;
}

size_t V3Cache::bytes() const {  // cache.rs:255-268
  size_t total = 0;
  for (const LayerCache& l : layers)
    total += (l.k.size() + l.v.size() + l.k_scale.size() + l.v_scale.size()) * 4 + l.kq.size() +
             l.vq.size() + (l.q_tail.size() + l.k_tail.size() + l.v_tail.size()) * 4;
  for (const auto& t : engram_tail) total += t.size() * 4;
  return total + tokens.size() * 4;
}

void V3Cache::push_token(uint32_t tok) {  // cache.rs:276-283
  size_t keep = cfg.engram.max_order();
  tokens.push_back(tok);
  if (tokens.size() > keep) tokens.erase(tokens.begin(), tokens.begin() + (tokens.size() - keep));
}

void V3Cache::ensure(size_t li, size_t p) {  // cache.rs:291-309
  LayerCache& l = layers[li];
  if (p < l.slots || l.slots >= l.cap) return;
  size_t want = std::min(std::max(l.slots * 2, p + 1), l.cap);
  if (l.kq.empty() && l.vq.empty()) {
    l.k.resize(want * cfg.k_dim(), 0.0f);
    l.v.resize(want * cfg.v_dim(), 0.0f);
  } else {
    l.kq.resize(want * cfg.k_dim(), 0);
    l.vq.resize(want * cfg.v_dim(), 0);
    l.k_scale.resize(want * cfg.num_kv_heads, 1.0f);
    l.v_scale.resize(want * cfg.num_kv_heads, 1.0f);
  }
  l.slots = want;
}

void V3Cache::span(size_t li, size_t p, size_t* lo, size_t* hi) const {  // cache.rs:322-331
  size_t slots = layers[li].slots;
  size_t w = cfg.attention_span(li);
  size_t l0 = (w && p + 1 > w) ? p + 1 - w : 0;
  size_t floor = p + 1 > slots ? p + 1 - slots : 0;
  *lo = std::max(l0, floor);
  *hi = p;
}

bool V3Cache::is_saturated() const {  // cache.rs:335-338
  for (size_t li = 0; li < cfg.num_layers; ++li)
    if (cfg.attention_span(li) == 0 && pos > layers[li].slots) return true;
  return false;
}

void V3Cache::write_kv(size_t li, size_t p, const float* k, const float* v) {  // cache.rs:346
  ensure(li, p);
  size_t kd = cfg.k_dim(), vd = cfg.v_dim(), qk = cfg.qk_head_dim, vh = cfg.v_head_dim;
  LayerCache& l = layers[li];
  size_t slot = p % l.slots;
  if (precision == KvPrecision::F32) {
    std::memcpy(l.k.data() + slot * kd, k, kd * 4);
    std::memcpy(l.v.data() + slot * vd, v, vd * 4);
    return;
  }
  size_t base = slot * cfg.num_kv_heads;
  for (size_t h = 0; h < cfg.num_kv_heads; ++h) {
    l.k_scale[base + h] = quant_into(k + h * qk, l.kq.data() + slot * kd + h * qk, qk);
    l.v_scale[base + h] = quant_into(v + h * vh, l.vq.data() + slot * vd + h * vh, vh);
  }
}

KvStore V3Cache::kv(size_t li) const {  // cache.rs:382-393
  const LayerCache& l = layers[li];
  KvStore s;
  if (precision == KvPrecision::F32) {
    s.k = l.k.data();
    s.v = l.v.data();
  } else {
    s.int8 = true;
    s.kq = l.kq.data();
    s.vq = l.vq.data();
    s.k_scale = l.k_scale.data();
    s.v_scale = l.v_scale.data();
  }
  return s;
}

// cache.rs:401-438
void V3Cache::conv_step(size_t li, Qkv which, const float* taps, float* raw, size_t dim) {
  size_t n_taps = cfg.qkv_conv_taps;
  if (n_taps == 0) return;
  LayerCache& l = layers[li];
  std::vector<float>& tail = which == Qkv::Q ? l.q_tail : (which == Qkv::K ? l.k_tail : l.v_tail);
  std::vector<float> out(dim);
  for (size_t c = 0; c < dim; ++c) {
    float acc = taps[c] * raw[c];
    for (size_t j = 1; j < n_taps; ++j) {
      if (j > pos) break;
      size_t slot = n_taps - 1 - j;
      acc += taps[j * dim + c] * tail[slot * dim + c];
    }
    out[c] = acc;
  }
  if (n_taps > 1) {
    std::memmove(tail.data(), tail.data() + dim, (tail.size() - dim) * 4);
    size_t last = (n_taps - 2) * dim;
    std::memcpy(tail.data() + last, raw, dim * 4);
  }
  std::memcpy(raw, out.data(), dim * 4);
}

// cache.rs:444-479
void V3Cache::engram_conv_step(size_t site, const float* taps, float* raw) {
  const V3Engram& e = cfg.engram;
  size_t n_taps = e.conv_taps, dil = e.conv_dilation, max_order = e.max_order();
  size_t d = cfg.d_model;
  size_t reach = (n_taps - 1) * dil;
  std::vector<float>& tail = engram_tail[site];
  std::vector<float> out(d);
  for (size_t c = 0; c < d; ++c) {
    float acc = 0.0f;
    for (size_t j = 0; j < n_taps; ++j) {
      size_t back = j * dil;
      if (back > pos || pos < j * max_order) continue;
      float val = j == 0 ? raw[c] : tail[(reach - back) * d + c];
      acc += taps[j * d + c] * val;
    }
    out[c] = acc;
  }
  if (reach > 0) {
    std::memmove(tail.data(), tail.data() + d, (tail.size() - d) * 4);
    std::memcpy(tail.data() + (reach - 1) * d, raw, d * 4);
  }
  std::memcpy(raw, out.data(), d * 4);
}

void V3Cache::seed_conv_tail(size_t li, Qkv which, const float* raw) {  // cache.rs:486
  LayerCache& l = layers[li];
  std::vector<float>& tail = which == Qkv::Q ? l.q_tail : (which == Qkv::K ? l.k_tail : l.v_tail);
  std::memcpy(tail.data(), raw, tail.size() * 4);
}
void V3Cache::seed_engram_tail(size_t site, const float* raw) {  // cache.rs:498
  std::memcpy(engram_tail[site].data(), raw, engram_tail[site].size() * 4);
}
void V3Cache::seed_tokens(const uint32_t* toks, size_t n) {  // cache.rs:505
  size_t keep = cfg.engram.max_order();
  tokens.clear();
  size_t start = n > keep ? n - keep : 0;
  tokens.assign(toks + start, toks + n);
}

// ---------------------------------------------------------------- engram.rs
static constexpr uint32_t ENGRAM_SEED = 0x9E3779B9u;   // engram.rs:19
static constexpr uint32_t ENGRAM_PRIME = 0x01000193u;  // engram.rs:20

std::vector<uint32_t> engram_indices(const uint32_t* tokens, size_t seq,
                                     const std::vector<size_t>& orders, size_t heads,
                                     uint32_t slots, size_t seed_heads) {  // engram.rs:31-61
  size_t stride = seed_heads == 0 ? heads : seed_heads;
  size_t nt = orders.size() * heads;
  std::vector<uint32_t> out(seq * nt, 0);
  for (size_t oi = 0; oi < orders.size(); ++oi) {
    size_t order = orders[oi];
    for (size_t h = 0; h < heads; ++h) {
      size_t table = oi * heads + h;
      uint32_t seed = ENGRAM_SEED * (uint32_t)(oi * stride + h + 1);
      for (size_t p = 0; p < seq; ++p) {
        uint32_t acc = seed;
        for (size_t j = 0; j < order; ++j) {
          uint32_t tok = j > p ? 0u : tokens[p - j];
          acc = (acc ^ tok) * ENGRAM_PRIME;
        }
        acc ^= acc >> 15;
        out[p * nt + table] = acc % slots;
      }
    }
  }
  return out;
}

bool ngram_valid(size_t p, size_t table, const std::vector<size_t>& orders, size_t heads) {
  return p + 1 >= orders[table / heads];  // engram.rs:66-69
}

void value_conv(float* buf, const float* taps, size_t seq, size_t dim, size_t conv_taps,
                size_t conv_dilation, size_t max_order) {  // engram.rs:89-106
  for (size_t p = seq; p-- > 0;) {
    for (size_t c = 0; c < dim; ++c) {
      float acc = 0.0f;
      for (size_t j = 0; j < conv_taps; ++j) {
        size_t back = j * conv_dilation;
        if (back > p || p < j * max_order) continue;
        acc += taps[j * dim + c] * buf[(p - back) * dim + c];
      }
      buf[p * dim + c] = acc;
    }
  }
}

void apply_site(float* x, const float* k, const float* v, size_t d) {  // engram.rs:112-132
  auto unit = [d](const float* z) {
    float sq = 0.0f;
    for (size_t i = 0; i < d; ++i) sq += z[i] * z[i];
    return 1.0f / sqrtf(sq / (float)d + 1e-6f);
  };
  float ux = unit(x), uk = unit(k);
  float dot = 0.0f;
  for (size_t i = 0; i < d; ++i) dot += x[i] * k[i];
  float alpha = sigmoid(dot * ux * uk / sqrtf((float)d));
  for (size_t i = 0; i < d; ++i) x[i] += alpha * v[i];
}

// ---------------------------------------------------------------- mhc.rs
float pre_off(size_t layer, size_t lane, size_t lanes) { return lane == layer % lanes ? 4.0f : -4.0f; }
float post_off(size_t layer, size_t lane, size_t lanes) { return lane == layer % lanes ? 0.0f : -4.0f; }

void mix_down(const float* lanes_buf, float* rows, const MhcLayer& m, size_t layer,
              size_t lanes, size_t d, float* u) {  // mhc.rs:79-102
  for (size_t lane = 0; lane < lanes; ++lane)
    rows[lane] = sigmoid(m.a_pre * rows[lane] + m.b_pre[lane] + pre_off(layer, lane, lanes));
  for (size_t c = 0; c < d; ++c) {
    float acc = 0.0f;
    for (size_t lane = 0; lane < lanes; ++lane) acc += rows[lane] * lanes_buf[lane * d + c];
    u[c] = acc;
  }
}

void scatter_up(float* lanes_buf, float* post, float* res, const float* y, const MhcLayer& m,
                size_t layer, size_t lanes, size_t d) {  // mhc.rs:109-158
  for (size_t lane = 0; lane < lanes; ++lane)
    post[lane] = 2.0f * sigmoid(m.a_post * post[lane] + m.b_post[lane] + post_off(layer, lane, lanes));
  for (size_t idx = 0; idx < lanes * lanes; ++idx) res[idx] = m.a_res * res[idx] + m.b_res[idx];
  sinkhorn(res, lanes);
  std::vector<float> scratch(lanes_buf, lanes_buf + lanes * d);
  for (size_t i = 0; i < lanes; ++i) {
    float hp = post[i];
    for (size_t c = 0; c < d; ++c) {
      float acc = 0.0f;
      for (size_t j = 0; j < lanes; ++j) acc += res[i * lanes + j] * scratch[j * d + c];
      lanes_buf[i * d + c] = acc + hp * y[c];
    }
  }
}

// ---------------------------------------------------------------- v3/kernels.rs
void hada_blocks(size_t n, size_t* ba, size_t* bb) {  // kernels.rs:26-34
  size_t v = n - 1, bits = 0;
  while (v) {
    ++bits;
    v >>= 1;
  }
  *ba = (size_t)1 << (bits / 2);
  *bb = n / *ba;
}

void kron_apply(const float* z, const float* a, const float* b, size_t ba, size_t bb,
                float* out) {  // kernels.rs:41-78
  std::vector<float> t(ba * bb, 0.0f);
  for (size_t i = 0; i < ba; ++i) {
    const float* zi = z + i * bb;
    const float* ai = a + i * ba;
    for (size_t k = 0; k < ba; ++k) {
      float aik = ai[k];
      if (aik == 0.0f) continue;
      float* tk = t.data() + k * bb;
      for (size_t j = 0; j < bb; ++j) tk[j] += zi[j] * aik;
    }
  }
  for (size_t k = 0; k < ba; ++k) {
    const float* tk = t.data() + k * bb;
    float* ok = out + k * bb;
    for (size_t l = 0; l < bb; ++l) ok[l] = 0.0f;
    for (size_t j = 0; j < bb; ++j) {
      float tkj = tk[j];
      if (tkj == 0.0f) continue;
      const float* bj = b + j * bb;
      for (size_t l = 0; l < bb; ++l) ok[l] += tkj * bj[l];
    }
  }
}

void hadamard_mlp(const float* x, size_t d_model, const HadaMlp& w, const HadaPerms& perms,
                  size_t n, float* out) {  // kernels.rs:119-180
  size_t ba, bb;
  hada_blocks(n, &ba, &bb);
  size_t r = w.cond_rank;
  std::vector<float> proj(r);
  for (size_t j = 0; j < r; ++j) {
    float acc = 0.0f;
    for (size_t i = 0; i < d_model; ++i) acc += x[i] * w.cond_v[i * r + j];
    proj[j] = acc;
  }
  float mx = -INFINITY;
  for (size_t j = 0; j < r; ++j) mx = std::fmax(mx, proj[j]);
  float sum = 0.0f;
  for (size_t j = 0; j < r; ++j) {
    proj[j] = expf(proj[j] - mx);
    sum += proj[j];
  }
  for (size_t j = 0; j < r; ++j) proj[j] /= sum;
  std::vector<float> cond(n, 1.0f);
  for (size_t j = 0; j < r; ++j) {
    float pj = proj[j];
    if (pj == 0.0f) continue;
    const float* row = w.cond_u.data() + j * n;
    for (size_t c = 0; c < n; ++c) cond[c] += pj * row[c];
  }
  std::vector<float> z(n, 0.0f), buf(n);
  std::memcpy(z.data(), x, d_model * 4);
  for (size_t i = 0; i < n; ++i) z[i] *= w.d1[i];
  kron_apply(z.data(), w.w1a.data(), w.w1b.data(), ba, bb, buf.data());
  for (size_t i = 0; i < n; ++i) z[i] = buf[perms.p1[i]];
  for (size_t i = 0; i < n; ++i) z[i] = silu(w.d2[i] * cond[i] * z[i] + w.b2[i]);
  kron_apply(z.data(), w.w2a.data(), w.w2b.data(), ba, bb, buf.data());
  for (size_t i = 0; i < n; ++i) z[i] = buf[perms.p2[i]];
  for (size_t i = 0; i < n; ++i) z[i] *= w.d3[i];
  kron_apply(z.data(), w.w3a.data(), w.w3b.data(), ba, bb, buf.data());
  for (size_t i = 0; i < d_model; ++i) out[i] = buf[i] * w.d4[i];
}

// ---------------------------------------------------------------- model.rs
size_t V3Model::clamp_token(uint32_t t) const {  // model.rs:533-535
  return std::min((size_t)t, cfg.vocab_size - 1);
}

void V3Model::rope_at(size_t pos, float* c, float* s) const {  // model.rs:378-393
  size_t half = cfg.qk_head_dim / 2;
  for (size_t i = 0; i < half; ++i) {
    float freq = 1.0f / powf(cfg.rope_theta, (float)(2 * i) / (float)cfg.qk_head_dim);
    float angle = (float)pos * freq;
    c[i] = cosf(angle);
    s[i] = sinf(angle);
  }
}

void V3Model::rope(size_t seq, std::vector<float>* c, std::vector<float>* s) const {  // :396
  size_t half = cfg.qk_head_dim / 2;
  c->assign(seq * half, 0.0f);
  s->assign(seq * half, 0.0f);
  for (size_t t = 0; t < seq; ++t) rope_at(t, c->data() + t * half, s->data() + t * half);
}

// quant_rows, model.rs:94-106
static void quant_rows(float* x, size_t seq, size_t heads, size_t head_dim) {
  for (size_t t = 0; t < seq; ++t)
    for (size_t h = 0; h < heads; ++h) fake_quant_vec(x + (t * heads + h) * head_dim, head_dim, 8);
}

// model.rs:150-375
std::vector<float> V3Model::decode_step(V3Cache& cache, uint32_t token) const {
  const V3Config& c = cfg;
  size_t d = c.d_model, n = c.mhc_lanes, pos = cache.pos, rows = c.logit_rows();
  cache.push_token(token);
  const V3Engram& e = c.engram;
  std::vector<uint32_t> hist = cache.tokens;
  size_t here = hist.size() - 1;
  std::vector<uint32_t> idx =
      engram_indices(hist.data(), hist.size(), e.orders, e.heads, (uint32_t)e.slots, e.seed_heads);
  size_t nt = e.num_tables();
  size_t ns = e.sites.size();
  std::vector<float> ek(ns * d), ev(ns * d), fetched(nt * e.sub_dim), row(e.sub_dim);
  for (size_t s = 0; s < ns; ++s) {
    const V3EngramSite& site = engrams[s];
    for (size_t t = 0; t < nt; ++t) {
      float* dst = fetched.data() + t * e.sub_dim;
      if (ngram_valid(pos, t, e.orders, e.heads)) {
        size_t slot = idx[here * nt + t];
        site.tables.dequantize_row(t * e.slots + slot, row.data());
        std::memcpy(dst, row.data(), e.sub_dim * 4);
      } else {
        std::fill(dst, dst + e.sub_dim, 0.0f);
      }
    }
    site.key_proj.matvec(fetched.data(), ek.data() + s * d);
    site.value_proj.matvec(fetched.data(), ev.data() + s * d);
    cache.engram_conv_step(s, site.taps.data(), ev.data() + s * d);
  }

  std::vector<float> lanes(n * d), emb(d);
  embedding.dequantize_row(clamp_token(token), emb.data());
  for (float& x : emb) x *= embed_scale;
  for (size_t l = 0; l < n; ++l) std::memcpy(lanes.data() + l * d, emb.data(), d * 4);

  AttnDims dims{1, c.num_heads, c.num_kv_heads, c.qk_head_dim, c.v_head_dim};
  size_t half = c.qk_head_dim / 2;
  std::vector<float> rc(half), rs(half);
  rope_at(pos, rc.data(), rs.data());

  std::vector<float> nx(n * d), nx_prep(mhc.phi_pre.prepared_len()), hpre(n), hpost(n),
      hres(n * n), u(d), q(c.q_dim()), k(c.k_dim()), v(c.v_dim()), attn(c.attn_out_dim()),
      gate(c.attn_out_dim()), proj(d), mlp_out(d), bx(d), h(d), y(d);

  for (size_t li = 0; li < c.num_layers; ++li) {
    const V3Layer& layer = layers[li];
    MhcLayer m{mhc.a_pre[li], mhc.a_post[li], mhc.a_res[li], mhc.b_pre.data() + li * n,
               mhc.b_post.data() + li * n, mhc.b_res.data() + li * n * n};
    rms_unit_to(lanes.data(), nx.data(), n * d);
    mhc.phi_pre.prepare_input(nx.data(), nx_prep.data());
    mhc.phi_pre.matvec_rows_prepared(nx_prep.data(), li * n, hpre.data(), n);
    mix_down(lanes.data(), hpre.data(), m, li, n, d, u.data());

    bx = u;
    int site = c.engram.site_of(li);
    if (site >= 0) apply_site(bx.data(), ek.data() + site * d, ev.data() + site * d, d);

    h = bx;
    zc_rms_norm_vec(h.data(), layer.norm_in.data(), d);
    layer.q_proj.matvec(h.data(), q.data());
    layer.k_proj.matvec(h.data(), k.data());
    layer.v_proj.matvec(h.data(), v.data());
    if (c.qkv_conv_taps > 0) {
      cache.conv_step(li, Qkv::Q, layer.q_taps.data(), q.data(), c.q_dim());
      cache.conv_step(li, Qkv::K, layer.k_taps.data(), k.data(), c.k_dim());
      cache.conv_step(li, Qkv::V, layer.v_taps.data(), v.data(), c.v_dim());
    }
    norm_and_rope(q.data(), layer.q_norm.data(), rc.data(), rs.data(), 1, c.num_heads, c.qk_head_dim);
    norm_and_rope(k.data(), layer.k_norm.data(), rc.data(), rs.data(), 1, c.num_kv_heads,
                  c.qk_head_dim);
    if (cache.precision == KvPrecision::Int8) quant_rows(q.data(), 1, c.num_heads, c.qk_head_dim);
    cache.write_kv(li, pos, k.data(), v.data());
    size_t lo, hi;
    cache.span(li, pos, &lo, &hi);
    attend_step(q.data(), cache.kv(li), cache.layers[li].slots, lo, hi, dims, attn.data());

    layer.gate_proj.matvec(h.data(), gate.data());
    for (size_t i = 0; i < attn.size(); ++i) attn[i] *= sigmoid(gate[i]);
    layer.out_proj.matvec(attn.data(), proj.data());
    zc_rms_norm_vec(proj.data(), layer.post_norm.data(), d);
    float agate = sigmoid(layer.attn_gate);
    for (size_t i = 0; i < d; ++i) bx[i] += agate * proj[i];

    proj = bx;
    zc_rms_norm_vec(proj.data(), layer.pre_hada.data(), d);
    hadamard_mlp(proj.data(), d, layer.mlp, perms, c.hada_n, mlp_out.data());
    for (size_t i = 0; i < d; ++i) bx[i] += mlp_out[i];
    for (size_t i = 0; i < d; ++i) y[i] = bx[i] - u[i];

    rms_unit_to(lanes.data(), nx.data(), n * d);
    mhc.phi_post.prepare_input(nx.data(), nx_prep.data());
    mhc.phi_post.matvec_rows_prepared(nx_prep.data(), li * n, hpost.data(), n);
    mhc.phi_res.prepare_input(nx.data(), nx_prep.data());
    mhc.phi_res.matvec_rows_prepared(nx_prep.data(), li * n * n, hres.data(), n * n);
    scatter_up(lanes.data(), hpost.data(), hres.data(), y.data(), m, li, n, d);
  }
  cache.pos += 1;

  std::vector<float> x(d);
  for (size_t ch = 0; ch < d; ++ch) {
    float acc = 0.0f;
    for (size_t l = 0; l < n; ++l) acc += lanes[l * d + ch];
    x[ch] = acc / (float)n;
  }
  zc_rms_norm_vec(x.data(), final_norm.data(), d);
  std::vector<float> lm_prep(embedding.prepared_len()), full(c.vocab_size);
  embedding.prepare_input(x.data(), lm_prep.data());
  embedding.matvec_rows_prepared(lm_prep.data(), 0, full.data(), c.vocab_size);
  full.resize(rows);
  return full;
}

// model.rs:420-471
void V3Model::engram_kv_with_raw(const uint32_t* tokens, size_t seq, bool want_raw,
                                 std::vector<float>* ks, std::vector<float>* vs,
                                 std::vector<float>* raw) const {
  const V3Engram& e = cfg.engram;
  size_t d = cfg.d_model, nt = e.num_tables(), ns = e.sites.size();
  std::vector<uint32_t> idx =
      engram_indices(tokens, seq, e.orders, e.heads, (uint32_t)e.slots, e.seed_heads);
  ks->assign(ns * seq * d, 0.0f);
  vs->assign(ns * seq * d, 0.0f);
  if (want_raw) raw->assign(ns * seq * d, 0.0f);
  std::vector<float> fetched(nt * e.sub_dim), row(e.sub_dim);
  for (size_t s = 0; s < ns; ++s) {
    const V3EngramSite& site = engrams[s];
    for (size_t p = 0; p < seq; ++p) {
      for (size_t t = 0; t < nt; ++t) {
        float* dst = fetched.data() + t * e.sub_dim;
        if (ngram_valid(p, t, e.orders, e.heads)) {
          site.tables.dequantize_row(t * e.slots + idx[p * nt + t], row.data());
          std::memcpy(dst, row.data(), e.sub_dim * 4);
        } else {
          std::fill(dst, dst + e.sub_dim, 0.0f);
        }
      }
      size_t base = (s * seq + p) * d;
      site.key_proj.matvec(fetched.data(), ks->data() + base);
      site.value_proj.matvec(fetched.data(), vs->data() + base);
    }
    size_t off = s * seq * d;
    if (want_raw) std::memcpy(raw->data() + off, vs->data() + off, seq * d * 4);
    value_conv(vs->data() + off, site.taps.data(), seq, d, e.conv_taps, e.conv_dilation,
               e.max_order());
  }
}

// model.rs:1000 — last_rows: the last n rows of (seq, dim), oldest first,
// zero-padded at the front when seq < n.
static std::vector<float> last_rows(const float* buf, size_t seq, size_t dim, size_t n) {
  std::vector<float> out(n * dim, 0.0f);
  size_t m = std::min(n, seq);
  for (size_t j = 0; j < m; ++j) {
    size_t src = seq - m + j, dst = n - m + j;
    std::memcpy(out.data() + dst * dim, buf + src * dim, dim * 4);
  }
  return out;
}

std::vector<float> V3Model::forward_sequence(const uint32_t* tokens, size_t n) const {
  return forward_impl(tokens, n, nullptr);
}

std::vector<float> V3Model::prefill(const uint32_t* tokens, size_t n, V3Cache& cache) const {
  if (n == 0) return {};  // model.rs:516-518
  size_t rows = cfg.logit_rows();
  std::vector<float> all = forward_impl(tokens, n, &cache);
  return std::vector<float>(all.begin() + (n - 1) * rows, all.begin() + n * rows);
}

// model.rs:550-980 (forward_impl_pooled without cells / probe pool).
std::vector<float> V3Model::forward_cells(const uint32_t* tokens, size_t n) const {
  std::vector<float> cells;
  forward_impl(tokens, n, nullptr, &cells);
  return cells;
}

// heads.rs:65-177: per (cell, probe) a softmax over positions of the scaled
// probe dot, the weighted mean of the cells, rms_unit and the gain; per query a
// softmax over all (cell, probe) pairs with the row bias, the weighted mean,
// then the projection of the flattened (queries * d) vector plus the bias.
std::vector<float> ProbeHead::forward(const float* cs, size_t seq, size_t d) const {
  const size_t l1 = cells, k = probes_per_cell, q = queries, m = l1 * k;
  const float scale = 1.0f / sqrtf((float)d);
  std::vector<float> r(m * d, 0.f), sc(seq);
  for (size_t l = 0; l < l1; ++l)
    for (size_t kk = 0; kk < k; ++kk) {
      const float* pr = probes.data() + (l * k + kk) * d;
      float mx = -INFINITY;
      for (size_t t = 0; t < seq; ++t) {
        const float* cell = cs + (t * l1 + l) * d;
        float acc = 0.f;
        for (size_t i = 0; i < d; ++i) acc += cell[i] * pr[i];
        sc[t] = acc * scale;
        if (sc[t] > mx) mx = sc[t];
      }
      float sum = 0.f;
      for (size_t t = 0; t < seq; ++t) {
        sc[t] = expf(sc[t] - mx);
        sum += sc[t];
      }
      const float inv = 1.0f / sum;
      float* dst = r.data() + (l * k + kk) * d;
      for (size_t t = 0; t < seq; ++t) {
        const float w = sc[t] * inv;
        const float* cell = cs + (t * l1 + l) * d;
        for (size_t i = 0; i < d; ++i) dst[i] += w * cell[i];
      }
      rms_unit_to(dst, dst, d);
      const float g = gain[l * k + kk];
      for (size_t i = 0; i < d; ++i) dst[i] *= g;
    }
  std::vector<float> pooled(q * d, 0.f), u(m);
  for (size_t qi = 0; qi < q; ++qi) {
    const float* qv = query.data() + qi * d;
    float mx = -INFINITY;
    for (size_t idx = 0; idx < m; ++idx) {
      float acc = 0.f;
      for (size_t i = 0; i < d; ++i) acc += r[idx * d + i] * qv[i];
      u[idx] = acc * scale + row_bias[qi * m + idx];
      if (u[idx] > mx) mx = u[idx];
    }
    float sum = 0.f;
    for (size_t idx = 0; idx < m; ++idx) {
      u[idx] = expf(u[idx] - mx);
      sum += u[idx];
    }
    const float inv = 1.0f / sum;
    for (size_t idx = 0; idx < m; ++idx) {
      const float w = u[idx] * inv;
      for (size_t i = 0; i < d; ++i) pooled[qi * d + i] += w * r[idx * d + i];
    }
  }
  std::vector<float> out(out_dim);
  for (size_t o = 0; o < out_dim; ++o) {
    float acc = 0.f;
    for (size_t i = 0; i < q * d; ++i) acc += proj[o * q * d + i] * pooled[i];
    out[o] = acc + (o < bias.size() ? bias[o] : 0.f);
  }
  return out;
}

std::vector<float> V3Model::forward_impl(const uint32_t* tokens, size_t seq, V3Cache* cache,
                                         std::vector<float>* cells) const {
  const V3Config& c = cfg;
  size_t d = c.d_model, n = c.mhc_lanes, rows = c.logit_rows();
  bool quantised = cache && cache->precision == KvPrecision::Int8;
  std::vector<float> rc, rs;
  rope(seq, &rc, &rs);
  std::vector<float> ek, ev, ev_raw;
  engram_kv_with_raw(tokens, seq, cache != nullptr, &ek, &ev, &ev_raw);

  std::vector<float> lanes(seq * n * d), emb(d);
  const size_t l1 = c.num_layers + 1;
  if (cells) cells->assign(seq * l1 * d, 0.f);
  for (size_t t = 0; t < seq; ++t) {
    embedding.dequantize_row(clamp_token(tokens[t]), emb.data());
    for (float& x : emb) x *= embed_scale;
    if (cells) std::memcpy(cells->data() + t * l1 * d, emb.data(), d * 4);  // cell 0
    for (size_t l = 0; l < n; ++l) std::memcpy(lanes.data() + (t * n + l) * d, emb.data(), d * 4);
  }
  AttnDims dims{seq, c.num_heads, c.num_kv_heads, c.qk_head_dim, c.v_head_dim};
  size_t qd = c.q_dim(), kd = c.k_dim(), vd = c.v_dim(), od = c.attn_out_dim();
  std::vector<float> nx(n * d), nx_prep(mhc.phi_pre.prepared_len()), hpre(n), hpost(n), hres(n * n);
  std::vector<float> u(seq * d), bx(seq * d), q(seq * qd), k(seq * kd), v(seq * vd),
      attn(seq * od), gates(seq * od);
  const size_t DEFAULT_CHUNK = 64;  // model.rs:23
  size_t chunk = std::min(DEFAULT_CHUNK, std::max(seq, (size_t)1));
  size_t prep_len = layers[0].q_proj.prepared_len();
  std::vector<float> xh(chunk * prep_len);
  size_t out_prep = layers[0].out_proj.prepared_len();
  std::vector<float> oh(chunk * out_prep), projected(seq * d), mlp_out(d), y(d);

  for (size_t li = 0; li < c.num_layers; ++li) {
    const V3Layer& layer = layers[li];
    MhcLayer m{mhc.a_pre[li], mhc.a_post[li], mhc.a_res[li], mhc.b_pre.data() + li * n,
               mhc.b_post.data() + li * n, mhc.b_res.data() + li * n * n};
    for (size_t t = 0; t < seq; ++t) {
      const float* ls = lanes.data() + t * n * d;
      rms_unit_to(ls, nx.data(), n * d);
      mhc.phi_pre.prepare_input(nx.data(), nx_prep.data());
      mhc.phi_pre.matvec_rows_prepared(nx_prep.data(), li * n, hpre.data(), n);
      mix_down(ls, hpre.data(), m, li, n, d, u.data() + t * d);
    }
    bx = u;
    int site = c.engram.site_of(li);
    if (site >= 0)
      for (size_t t = 0; t < seq; ++t) {
        size_t base = ((size_t)site * seq + t) * d;
        apply_site(bx.data() + t * d, ek.data() + base, ev.data() + base, d);
      }
    std::vector<float> h = bx;
    for (size_t t = 0; t < seq; ++t) zc_rms_norm_vec(h.data() + t * d, layer.norm_in.data(), d);
    for (size_t c0 = 0; c0 < seq; c0 += chunk) {
      size_t b = std::min(seq - c0, chunk);
      for (size_t i = 0; i < b; ++i)
        layer.q_proj.prepare_input(h.data() + (c0 + i) * d, xh.data() + i * prep_len);
      layer.q_proj.matmul_rows_prepared(xh.data(), b, 0, qd, q.data() + c0 * qd);
      layer.k_proj.matmul_rows_prepared(xh.data(), b, 0, kd, k.data() + c0 * kd);
      layer.v_proj.matmul_rows_prepared(xh.data(), b, 0, vd, v.data() + c0 * vd);
      layer.gate_proj.matmul_rows_prepared(xh.data(), b, 0, od, gates.data() + c0 * od);
    }
    std::vector<float> qt, kt, vt;
    if (cache && c.qkv_conv_taps > 0) {
      size_t nn = c.qkv_conv_taps - 1;
      qt = last_rows(q.data(), seq, qd, nn);
      kt = last_rows(k.data(), seq, kd, nn);
      vt = last_rows(v.data(), seq, vd, nn);
    }
    if (c.qkv_conv_taps > 0) {
      causal_depthwise_conv(q.data(), layer.q_taps.data(), seq, qd, c.qkv_conv_taps);
      causal_depthwise_conv(k.data(), layer.k_taps.data(), seq, kd, c.qkv_conv_taps);
      causal_depthwise_conv(v.data(), layer.v_taps.data(), seq, vd, c.qkv_conv_taps);
    }
    norm_and_rope(q.data(), layer.q_norm.data(), rc.data(), rs.data(), seq, c.num_heads, c.qk_head_dim);
    norm_and_rope(k.data(), layer.k_norm.data(), rc.data(), rs.data(), seq, c.num_kv_heads,
                  c.qk_head_dim);
    if (quantised) {
      quant_rows(q.data(), seq, c.num_heads, c.qk_head_dim);
      quant_rows(k.data(), seq, c.num_kv_heads, c.qk_head_dim);
      quant_rows(v.data(), seq, c.num_kv_heads, c.v_head_dim);
    }
    if (cache) {
      for (size_t t = 0; t < seq; ++t) cache->write_kv(li, t, k.data() + t * kd, v.data() + t * vd);
      if (c.qkv_conv_taps > 0) {
        cache->seed_conv_tail(li, Qkv::Q, qt.data());
        cache->seed_conv_tail(li, Qkv::K, kt.data());
        cache->seed_conv_tail(li, Qkv::V, vt.data());
      }
    }
    std::vector<int8_t> kq, vq;
    std::vector<float> ksc, vsc;
    KvStore store;
    if (quantised) {
      quantize_rows(k.data(), k.size(), c.qk_head_dim, &kq, &ksc);
      quantize_rows(v.data(), v.size(), c.v_head_dim, &vq, &vsc);
      store.int8 = true;
      store.kq = kq.data();
      store.k_scale = ksc.data();
      store.vq = vq.data();
      store.v_scale = vsc.data();
    } else {
      store.k = k.data();
      store.v = v.data();
    }
    attend(q.data(), store, dims, c.attention_span(li), attn.data());

    float agate = sigmoid(layer.attn_gate);
    for (size_t t = 0; t < seq; ++t)
      for (size_t i = 0; i < od; ++i) attn[t * od + i] *= sigmoid(gates[t * od + i]);
    for (size_t c0 = 0; c0 < seq; c0 += chunk) {
      size_t b = std::min(seq - c0, chunk);
      for (size_t i = 0; i < b; ++i)
        layer.out_proj.prepare_input(attn.data() + (c0 + i) * od, oh.data() + i * out_prep);
      layer.out_proj.matmul_rows_prepared(oh.data(), b, 0, d, projected.data() + c0 * d);
    }
    for (size_t t = 0; t < seq; ++t) {
      float* proj = projected.data() + t * d;
      zc_rms_norm_vec(proj, layer.post_norm.data(), d);
      float* s1 = bx.data() + t * d;
      for (size_t i = 0; i < d; ++i) s1[i] += agate * proj[i];
      std::memcpy(proj, s1, d * 4);
      zc_rms_norm_vec(proj, layer.pre_hada.data(), d);
      hadamard_mlp(proj, d, layer.mlp, perms, c.hada_n, mlp_out.data());
      for (size_t i = 0; i < d; ++i) s1[i] += mlp_out[i];
    }
    for (size_t t = 0; t < seq; ++t) {
      float* ls = lanes.data() + t * n * d;
      rms_unit_to(ls, nx.data(), n * d);
      mhc.phi_post.prepare_input(nx.data(), nx_prep.data());
      mhc.phi_post.matvec_rows_prepared(nx_prep.data(), li * n, hpost.data(), n);
      mhc.phi_res.prepare_input(nx.data(), nx_prep.data());
      mhc.phi_res.matvec_rows_prepared(nx_prep.data(), li * n * n, hres.data(), n * n);
      for (size_t i = 0; i < d; ++i) y[i] = bx[t * d + i] - u[t * d + i];
      scatter_up(ls, hpost.data(), hres.data(), y.data(), m, li, n, d);
    }
    if (cells)  // cell li + 1: the lane stream after this layer, meaned over lanes (model.rs:910-926)
      for (size_t t = 0; t < seq; ++t)
        for (size_t i = 0; i < d; ++i) {
          float a = 0.f;
          for (size_t l = 0; l < n; ++l) a += lanes[(t * n + l) * d + i];
          (*cells)[(t * l1 + li + 1) * d + i] = a / (float)n;
        }
  }

  if (cache) {
    cache->pos = seq;
    cache->seed_tokens(tokens, seq);
    size_t reach = (c.engram.conv_taps > 0 ? c.engram.conv_taps - 1 : 0) * c.engram.conv_dilation;
    if (reach > 0)
      for (size_t s = 0; s < c.engram.sites.size(); ++s) {
        std::vector<float> lr = last_rows(ev_raw.data() + s * seq * d, seq, d, reach);
        cache->seed_engram_tail(s, lr.data());
      }
  }

  std::vector<float> logits(seq * rows), pooled(seq * d);
  for (size_t t = 0; t < seq; ++t) {
    float* o = pooled.data() + t * d;
    for (size_t ch = 0; ch < d; ++ch) {
      float a = 0.0f;
      for (size_t l = 0; l < n; ++l) a += lanes[(t * n + l) * d + ch];
      o[ch] = a / (float)n;
    }
    zc_rms_norm_vec(o, final_norm.data(), d);
  }
  size_t lm_prep = embedding.prepared_len();
  std::vector<float> lh(chunk * lm_prep);
  for (size_t c0 = 0; c0 < seq; c0 += chunk) {
    size_t b = std::min(seq - c0, chunk);
    for (size_t i = 0; i < b; ++i)
      embedding.prepare_input(pooled.data() + (c0 + i) * d, lh.data() + i * lm_prep);
    embedding.matmul_rows_prepared(lh.data(), b, 0, rows, logits.data() + c0 * rows);
  }
  return logits;
}

}  // namespace oracle
