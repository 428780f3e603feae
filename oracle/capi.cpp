// TEST INFRASTRUCTURE — a flat C interface over the oracle, loaded with ctypes
// by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg only.
#include <omp.h>

#include <cmath>
#include <cstring>
#include <string>

#include "oracle.hpp"

using namespace oracle;

static void put_err(char* err, size_t errlen, const std::string& s) {
  if (!err || errlen == 0) return;
  size_t n = std::min(errlen - 1, s.size());
  std::memcpy(err, s.data(), n);
  err[n] = 0;
}

extern "C" {

int orc_version() { return 1; }
void orc_set_threads(int n) { omp_set_num_threads(n); }
int orc_max_threads() { return omp_get_max_threads(); }

// ---------------------------------------------------------------- CQ weights
void* orc_cq_new(const uint8_t* blob, size_t blob_len, size_t out_feat, size_t in_feat,
                 size_t group, int bits, const float* codebook, char* err, size_t errlen) {
  CqWeight* w = new CqWeight();
  std::string e = CqWeight::from_blob(blob, blob_len, out_feat, in_feat, group, (uint8_t)bits,
                                      codebook, CODEBOOK_LEN, w);
  if (!e.empty()) {
    put_err(err, errlen, e);
    delete w;
    return nullptr;
  }
  return w;
}
void orc_cq_free(void* w) { delete (CqWeight*)w; }
void orc_cq_prepare(void* w, const float* x, float* xh) { ((CqWeight*)w)->prepare_input(x, xh); }
void orc_cq_matvec(void* w, const float* x, float* y) { ((CqWeight*)w)->matvec(x, y); }
void orc_cq_matvec_rows_prepared(void* w, const float* xh, size_t row_start, size_t rows,
                                 float* y) {
  ((CqWeight*)w)->matvec_rows_prepared(xh, row_start, y, rows);
}
void orc_cq_matvec_reference(void* w, const float* xh, float* y) {
  ((CqWeight*)w)->matvec_prepared_reference(xh, y);
}
void orc_cq_matmul_prepared(void* w, const float* xh, size_t batch, size_t row_start,
                            size_t rows, float* y) {
  ((CqWeight*)w)->matmul_rows_prepared(xh, batch, row_start, rows, y);
}
void orc_cq_dequant_row(void* w, size_t o, float* out) { ((CqWeight*)w)->dequantize_row(o, out); }
// Decoded level indices of one row (in_padded entries), for unpack parity.
void orc_cq_row_indices(void* w, size_t o, uint8_t* out) {
  CqWeight* q = (CqWeight*)w;
  size_t b = q->bits == TERNARY_RECORD_BITS ? 2 : q->bits;
  const uint8_t* row = q->packed.data() + o * q->row_bytes;
  for (size_t k = 0; k < q->in_padded; ++k) {
    size_t bit = k * b, byte = bit / 8, sh = bit % 8;
    uint32_t lo = row[byte], hi = (sh + b > 8) ? row[byte + 1] : 0;
    out[k] = (uint8_t)(((lo | (hi << 8)) >> sh) & ((1u << b) - 1));
  }
}
size_t orc_cq_in_padded(void* w) { return ((CqWeight*)w)->in_padded; }
float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

// ---------------------------------------------------------------- primitives
void orc_fwht_normalized(float* x, size_t n) { fwht_normalized(x, n); }
void orc_fake_quant(float* x, size_t n, uint32_t bits) { fake_quant_vec(x, n, bits); }
float orc_quant_into(const float* src, int8_t* dst, size_t n) { return quant_into(src, dst, n); }
void orc_rms_unit(const float* x, float* out, size_t n) { rms_unit_to(x, out, n); }
void orc_zc_rms_norm(float* x, const float* scale, size_t n) { zc_rms_norm_vec(x, scale, n); }
void orc_sinkhorn(float* m, size_t n) { sinkhorn(m, n); }
void orc_causal_conv(float* buf, const float* taps, size_t seq, size_t dim, size_t n_taps) {
  causal_depthwise_conv(buf, taps, seq, dim, n_taps);
}
void orc_kron_apply(const float* z, const float* a, const float* b, size_t ba, size_t bb,
                    float* out) {
  kron_apply(z, a, b, ba, bb, out);
}
void orc_hada_blocks(size_t n, size_t* ba, size_t* bb) { hada_blocks(n, ba, bb); }
void orc_engram_indices(const uint32_t* tokens, size_t seq, const size_t* orders, size_t n_orders,
                        size_t heads, uint32_t slots, size_t seed_heads, uint32_t* out) {
  std::vector<size_t> o(orders, orders + n_orders);
  std::vector<uint32_t> r = engram_indices(tokens, seq, o, heads, slots, seed_heads);
  std::memcpy(out, r.data(), r.size() * 4);
}
int orc_ngram_valid(size_t p, size_t table, const size_t* orders, size_t n_orders, size_t heads) {
  std::vector<size_t> o(orders, orders + n_orders);
  return ngram_valid(p, table, o, heads) ? 1 : 0;
}
void orc_value_conv(float* buf, const float* taps, size_t seq, size_t dim, size_t conv_taps,
                    size_t dil, size_t max_order) {
  value_conv(buf, taps, seq, dim, conv_taps, dil, max_order);
}
void orc_apply_site(float* x, const float* k, const float* v, size_t d) { apply_site(x, k, v, d); }
void orc_mix_down(const float* lanes, float* rows, float a_pre, const float* b_pre, size_t layer,
                  size_t n, size_t d, float* u) {
  MhcLayer m{a_pre, 0.f, 0.f, b_pre, nullptr, nullptr};
  mix_down(lanes, rows, m, layer, n, d, u);
}
void orc_scatter_up(float* lanes, float* post, float* res, const float* y, float a_post,
                    float a_res, const float* b_post, const float* b_res, size_t layer, size_t n,
                    size_t d) {
  MhcLayer m{0.f, a_post, a_res, nullptr, b_post, b_res};
  scatter_up(lanes, post, res, y, m, layer, n, d);
}
void orc_norm_and_rope(float* buf, const float* scale, const float* c, const float* s, size_t seq,
                       size_t heads, size_t hd) {
  norm_and_rope(buf, scale, c, s, seq, heads, hd);
}
// F32 store when kq == NULL.
void orc_attend_step(const float* q, const float* k, const float* v, const int8_t* kq,
                     const float* ks, const int8_t* vq, const float* vs, size_t slots, size_t lo,
                     size_t hi, size_t heads, size_t kv_heads, size_t qk, size_t vh, float* out) {
  KvStore st;
  if (kq) {
    st.int8 = true;
    st.kq = kq;
    st.k_scale = ks;
    st.vq = vq;
    st.v_scale = vs;
  } else {
    st.k = k;
    st.v = v;
  }
  AttnDims d{1, heads, kv_heads, qk, vh};
  attend_step(q, st, slots, lo, hi, d, out);
}
void orc_attend(const float* q, const float* k, const float* v, const int8_t* kq, const float* ks,
                const int8_t* vq, const float* vs, size_t seq, size_t heads, size_t kv_heads,
                size_t qk, size_t vh, size_t window, float* out) {
  KvStore st;
  if (kq) {
    st.int8 = true;
    st.kq = kq;
    st.k_scale = ks;
    st.vq = vq;
    st.v_scale = vs;
  } else {
    st.k = k;
    st.v = v;
  }
  AttnDims d{seq, heads, kv_heads, qk, vh};
  attend(q, st, d, window, out);
}

// ---------------------------------------------------------------- model and sessions
void* orc_model_load(const uint8_t* data, size_t len, char* err, size_t errlen) {
  V3Model* m = new V3Model();
  std::string e = load_model(data, len, m);
  if (!e.empty()) {
    put_err(err, errlen, e);
    delete m;
    return nullptr;
  }
  return m;
}
void orc_model_free(void* m) { delete (V3Model*)m; }
// The `depth`-block rung of a full-depth container (v3.rs:656-745).
void* orc_model_load_depth(const uint8_t* data, size_t len, size_t depth, char* err, size_t errlen) {
  V3Model* m = new V3Model();
  std::string e = load_model(data, len, m);
  if (e.empty()) e = slice_to_depth(m, depth);
  if (!e.empty()) {
    put_err(err, errlen, e);
    delete m;
    return nullptr;
  }
  return m;
}
int orc_model_has_confidence(void* mp) { return ((V3Model*)mp)->has_confidence ? 1 : 0; }
// The confidence head's first logit over the sequence (v3_engine.rs:351-368
// before the sigmoid); 0 when the model has no head.
int orc_confidence_logit(void* mp, const uint32_t* ids, size_t n, float* out) {
  const V3Model* m = (const V3Model*)mp;
  if (!m->has_confidence || n == 0) return 0;
  std::vector<float> cells = m->forward_cells(ids, n);
  *out = m->confidence.forward(cells.data(), n, m->cfg.d_model)[0];
  return 1;
}
// ProbeHead::forward on explicit weights (heads.rs:65-118).
void orc_probe_forward(const float* cells, size_t seq, size_t d, const float* probes, const float* gain,
                       const float* query, const float* row_bias, const float* proj, const float* bias,
                       size_t ncells, size_t k, size_t q, size_t out_dim, float* out) {
  ProbeHead h;
  h.probes.assign(probes, probes + ncells * k * d);
  h.gain.assign(gain, gain + ncells * k);
  h.query.assign(query, query + q * d);
  h.row_bias.assign(row_bias, row_bias + q * ncells * k);
  h.proj.assign(proj, proj + out_dim * q * d);
  h.bias.assign(bias, bias + out_dim);
  h.cells = ncells;
  h.probes_per_cell = k;
  h.queries = q;
  h.out_dim = out_dim;
  std::vector<float> r = h.forward(cells, seq, d);
  for (size_t o = 0; o < out_dim; ++o) out[o] = r[o];
}
// ladder.rs:28: writes num_layers entries.
void orc_ladder_order(size_t num_layers, int64_t* out) {
  std::vector<size_t> o = ladder_order(num_layers);
  for (size_t i = 0; i < o.size(); ++i) out[i] = (int64_t)o[i];
}
// ladder.rs:67: writes depth entries and returns 1, or returns 0 outside the ladder.
int orc_ladder_layers(size_t num_layers, size_t depth, int64_t* out) {
  std::vector<size_t> k;
  if (!ladder_layer_indices(num_layers, depth, &k)) return 0;
  for (size_t i = 0; i < k.size(); ++i) out[i] = (int64_t)k[i];
  return 1;
}
// Global layers and Engram sites of the model (rungs renumber them): counts
// first, then the lists; returns the number of entries written.
int orc_model_layer_roles(void* mp, int64_t* out, int cap) {
  const V3Config& c = ((V3Model*)mp)->cfg;
  int w = 0;
  if (cap < 2) return 0;
  out[w++] = (int64_t)c.global_layers.size();
  out[w++] = (int64_t)c.engram.sites.size();
  for (size_t l : c.global_layers)
    if (w < cap) out[w++] = (int64_t)l;
  for (size_t l : c.engram.sites)
    if (w < cap) out[w++] = (int64_t)l;
  return w;
}
// vocab, out_vocab, d_model, heads, kv_heads, layers, qk, vh, max_seq, hada_n, lanes,
// window, conv_taps, logit_rows
void orc_model_geom(void* mp, int64_t* out) {
  const V3Config& c = ((V3Model*)mp)->cfg;
  int64_t v[14] = {(int64_t)c.vocab_size, (int64_t)c.out_vocab, (int64_t)c.d_model,
                   (int64_t)c.num_heads, (int64_t)c.num_kv_heads, (int64_t)c.num_layers,
                   (int64_t)c.qk_head_dim, (int64_t)c.v_head_dim, (int64_t)c.max_seq_len,
                   (int64_t)c.hada_n, (int64_t)c.mhc_lanes, (int64_t)c.sliding_window,
                   (int64_t)c.qkv_conv_taps, (int64_t)c.logit_rows()};
  std::memcpy(out, v, sizeof(v));
}
size_t orc_model_kv_bytes(void* mp, size_t seq_len, int int8) {
  return ((V3Model*)mp)->cfg.kv_bytes_at(seq_len, int8 ? KvPrecision::Int8 : KvPrecision::F32);
}
void orc_model_mlp(void* mp, size_t layer, const float* x, float* out) {
  V3Model* m = (V3Model*)mp;
  hadamard_mlp(x, m->cfg.d_model, m->layers[layer].mlp, m->perms, m->cfg.hada_n, out);
}
void* orc_session_new(void* mp, size_t hint, int int8) {
  return new V3Cache(((V3Model*)mp)->cfg, hint, int8 ? KvPrecision::Int8 : KvPrecision::F32);
}
void orc_session_free(void* s) { delete (V3Cache*)s; }
void* orc_session_clone(void* s) { return new V3Cache(*(V3Cache*)s); }
size_t orc_session_pos(void* s) { return ((V3Cache*)s)->pos; }
size_t orc_session_bytes(void* s) { return ((V3Cache*)s)->bytes(); }
size_t orc_session_slots(void* s, size_t li) { return ((V3Cache*)s)->layers[li].slots; }
int orc_session_saturated(void* s) { return ((V3Cache*)s)->is_saturated() ? 1 : 0; }
// Copies the stored KV of one layer: f32 (k, v) or int8 (kq, ks, vq, vs); NULL pointers skip.
void orc_session_kv(void* sp, size_t li, float* k, float* v, int8_t* kq, float* ks, int8_t* vq,
                    float* vs) {
  const LayerCache& l = ((V3Cache*)sp)->layers[li];
  if (k && !l.k.empty()) std::memcpy(k, l.k.data(), l.k.size() * 4);
  if (v && !l.v.empty()) std::memcpy(v, l.v.data(), l.v.size() * 4);
  if (kq && !l.kq.empty()) std::memcpy(kq, l.kq.data(), l.kq.size());
  if (vq && !l.vq.empty()) std::memcpy(vq, l.vq.data(), l.vq.size());
  if (ks && !l.k_scale.empty()) std::memcpy(ks, l.k_scale.data(), l.k_scale.size() * 4);
  if (vs && !l.v_scale.empty()) std::memcpy(vs, l.v_scale.data(), l.v_scale.size() * 4);
}
void orc_session_span(void* sp, size_t li, size_t pos, size_t* lo, size_t* hi) {
  ((V3Cache*)sp)->span(li, pos, lo, hi);
}
void orc_session_write_kv(void* sp, size_t li, size_t pos, const float* k, const float* v) {
  ((V3Cache*)sp)->write_kv(li, pos, k, v);
}
void orc_session_advance(void* sp) { ((V3Cache*)sp)->pos += 1; }
void orc_session_conv_step(void* sp, size_t li, int which, const float* taps, float* raw,
                           size_t dim) {
  ((V3Cache*)sp)->conv_step(li, which == 0 ? Qkv::Q : (which == 1 ? Qkv::K : Qkv::V), taps, raw,
                            dim);
}
void orc_session_engram_conv_step(void* sp, size_t site, const float* taps, float* raw) {
  ((V3Cache*)sp)->engram_conv_step(site, taps, raw);
}
// Returns the number of logits written (logit_rows), 0 for an empty prompt.
size_t orc_prefill(void* mp, void* sp, const uint32_t* ids, size_t n, float* logits) {
  std::vector<float> r = ((V3Model*)mp)->prefill(ids, n, *(V3Cache*)sp);
  if (!r.empty()) std::memcpy(logits, r.data(), r.size() * 4);
  return r.size();
}
size_t orc_decode_step(void* mp, void* sp, uint32_t tok, float* logits) {
  std::vector<float> r = ((V3Model*)mp)->decode_step(*(V3Cache*)sp, tok);
  std::memcpy(logits, r.data(), r.size() * 4);
  return r.size();
}
// SplitMix64::next_u64 (crates/needle-infer/src/v3_engine.rs:446-459).
uint64_t orc_splitmix64_next(uint64_t* state) {
  *state += 0x9E3779B97F4A7C15ull;
  uint64_t z = *state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// SplitMix64::next_f64 (v3_engine.rs:461-463): the top 53 bits over 2^53.
double orc_splitmix64_next_f64(uint64_t* state) {
  return (double)(orc_splitmix64_next(state) >> 11) / (double)(1ull << 53);
}
// sample (v3_engine.rs:422-443): softmax weights exp((v - max) / T) in f32,
// summed in f64; the first index whose running subtraction from
// next_f64 * sum reaches <= 0, else the last index.
uint32_t orc_sample(const float* logits, size_t n, float temperature, uint64_t* state) {
  const float inv = 1.0f / temperature;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i)
    if (logits[i] > mx) mx = logits[i];
  double sum = 0.0;
  for (size_t i = 0; i < n; ++i) sum += (double)std::exp((logits[i] - mx) * inv);
  double target = orc_splitmix64_next_f64(state) * sum;
  for (size_t i = 0; i < n; ++i) {
    target -= (double)std::exp((logits[i] - mx) * inv);
    if (target <= 0.0) return (uint32_t)i;
  }
  return (uint32_t)(n - 1);
}

void orc_forward_sequence(void* mp, const uint32_t* ids, size_t n, float* logits) {
  std::vector<float> r = ((V3Model*)mp)->forward_sequence(ids, n);
  std::memcpy(logits, r.data(), r.size() * 4);
}

}  // extern "C"
