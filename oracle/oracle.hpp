// TEST INFRASTRUCTURE — not product code.
//
// A CPU restatement of the Needle-3 forward path of bynds/needle-rs
// (`crates/needle-core`, `crates/needle-infer/src/cact.rs`, `v3.rs`), written in
// C++ because the reference is Rust and no Rust toolchain exists here. It is the
// parity oracle for the CUDA path and the timed CPU baseline in bench.py. Only
// the test suite, `__graft_entry__.smoke()` and bench.py's cpu_baseline leg load
// it, always as the checker, never as the thing measured or shipped.
//
// Numerics follow the reference's summation orders (8 accumulator lanes per CQ
// group, group norm applied after the group dot, sequential f32 sums) and its
// float semantics: compiled with -ffp-contract=off so no multiply-add is fused,
// glibc libm for exp/log/sin/cos/pow/round (the reference uses the `libm` crate;
// transcendental ulp behaviour is not pinned by any reference test).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace oracle {

// ---------------------------------------------------------------- cq.rs
// Record width that marks a ternary tensor (crates/needle-core/src/cq.rs:57).
constexpr uint8_t TERNARY_RECORD_BITS = 5;
// Ternary centroid before 1/sqrt(group) (cq.rs:61).
constexpr float TERNARY_CENTROID = 1.2240064f;
// cb2|cb3|cb4 = 4+8+16 (cq.rs:68).
constexpr size_t CODEBOOK_LEN = 28;
constexpr size_t MAX_GROUP = 1024;  // cq.rs:73
constexpr size_t ACC_LANES = 8;     // cq.rs:830

float f16_to_f32(uint16_t bits);  // math.rs:53-68

// Packed row bytes (cq.rs:107-115).
size_t packed_row_bytes(size_t in_padded, uint8_t bits);

// In-place normalised fast Walsh-Hadamard transform (hadamard.rs:24-55).
void fwht(float* x, size_t n);
void fwht_normalized(float* x, size_t n);

struct CqWeight {  // cq.rs:117-141
  std::vector<uint8_t> packed;
  std::vector<float> norms;
  std::vector<float> lut;
  size_t per_byte = 0, row_bytes = 0, num_groups = 0;
  size_t out_feat = 0, in_feat = 0, in_padded = 0, group = 0;
  uint8_t bits = 0;
  std::vector<float> levels;

  // cq.rs:181-238. Returns an empty string on success, else the error.
  static std::string from_blob(const uint8_t* blob, size_t blob_len, size_t out_feat,
                               size_t in_feat, size_t group, uint8_t bits,
                               const float* codebook, size_t codebook_len, CqWeight* out);
  size_t prepared_len() const { return in_padded; }
  void prepare_input(const float* x, float* xh) const;                         // cq.rs:264
  void matvec(const float* x, float* y) const;                                 // cq.rs:283
  void matvec_rows_prepared(const float* xh, size_t row_start, float* y,
                            size_t rows) const;                                // cq.rs:301
  void matvec_prepared_reference(const float* xh, float* y) const;             // cq.rs:381
  void matmul_rows_prepared(const float* xh, size_t batch, size_t row_start, size_t rows,
                            float* y) const;                                   // cq.rs:446
  void dequantize_row(size_t o, float* out) const;                             // cq.rs:763
  void decode_group(const uint8_t* row, size_t g, float norm, float* buf) const;  // cq.rs:791
  bool select_rows(const std::vector<size_t>& rows, CqWeight* out) const;          // cq.rs:151

 private:
  void matvec_rows_serial(const float* xh, size_t row_start, float* y, size_t rows) const;
  void matmul_rows_serial(const float* xh, size_t batch, size_t row_start, size_t rows,
                          float* y) const;
};

// ---------------------------------------------------------------- kernels.rs / norm.rs / ops.rs
constexpr float EPS = 1e-6f;
constexpr int SINKHORN_ITERS = 20;
void rms_unit_to(const float* x, float* out, size_t n);        // kernels.rs:32
void zc_rms_norm_vec(float* x, const float* scale, size_t n);  // norm.rs:23
void sinkhorn(float* m, size_t n);                             // kernels.rs:46
float sigmoid(float x);                                        // ops.rs:41
float silu(float x);                                           // ops.rs:118

// ---------------------------------------------------------------- v3/config.rs
struct V3Engram {
  std::vector<size_t> orders;
  size_t heads = 0, slots = 0, sub_dim = 0;
  std::vector<size_t> sites;
  size_t conv_taps = 0, conv_dilation = 0, seed_heads = 0;
  size_t num_tables() const { return orders.size() * heads; }
  int site_of(size_t layer) const;
  size_t max_order() const;
};

enum class KvPrecision { F32 = 0, Int8 = 1 };

struct V3Config {  // v3/config.rs:44-73
  size_t vocab_size = 0, out_vocab = 0, d_model = 0, num_heads = 0, num_kv_heads = 0,
         num_layers = 0, qk_head_dim = 0, v_head_dim = 0, max_seq_len = 0, hada_n = 0,
         mhc_lanes = 0;
  float rope_theta = 0.f;
  size_t sliding_window = 0;
  std::vector<size_t> global_layers;
  size_t qkv_conv_taps = 0;
  V3Engram engram;
  size_t q_dim() const { return num_heads * qk_head_dim; }
  size_t k_dim() const { return num_kv_heads * qk_head_dim; }
  size_t v_dim() const { return num_kv_heads * v_head_dim; }
  size_t attn_out_dim() const { return num_heads * v_head_dim; }
  size_t kv_repeat() const { return num_heads / num_kv_heads; }
  size_t logit_rows() const { return out_vocab == 0 ? vocab_size : out_vocab; }
  bool is_global(size_t layer) const;
  // 0 means unbounded (config.rs:216 returns None).
  size_t attention_span(size_t layer) const;
  size_t kv_bytes(size_t seq_len, size_t bytes_per) const;          // config.rs:234
  size_t kv_bytes_at(size_t seq_len, KvPrecision p) const;          // config.rs:255
};

// ---------------------------------------------------------------- v3/attention.rs
struct AttnDims {
  size_t seq, num_heads, num_kv_heads, qk_head_dim, v_head_dim;
};
// One KV store view. For F32 k/v are float; for Int8 kq/vq + scales.
struct KvStore {
  bool int8 = false;
  const float* k = nullptr;
  const float* v = nullptr;
  const int8_t* kq = nullptr;
  const float* k_scale = nullptr;
  const int8_t* vq = nullptr;
  const float* v_scale = nullptr;
};
void causal_depthwise_conv(float* buf, const float* taps, size_t seq, size_t dim,
                           size_t n_taps);                                   // attention.rs:82
void norm_and_rope(float* buf, const float* scale, const float* cos, const float* sin,
                   size_t seq, size_t heads, size_t head_dim);               // attention.rs:107
// window 0 = unbounded.
void attend(const float* q, const KvStore& kv, const AttnDims& d, size_t window,
            float* out);                                                     // attention.rs:218
void attend_step(const float* q, const KvStore& kv, size_t slots, size_t lo, size_t hi,
                 const AttnDims& d, float* out);                             // attention.rs:300

// ---------------------------------------------------------------- v3/cache.rs
void fake_quant_vec(float* x, size_t n, uint32_t bits);                        // cache.rs:68
float quant_into(const float* src, int8_t* dst, size_t n);                     // cache.rs:100
void quantize_rows(const float* x, size_t len, size_t head_dim, std::vector<int8_t>* ints,
                   std::vector<float>* scales);                                // cache.rs:115

struct LayerCache {
  std::vector<float> k, v;
  std::vector<int8_t> kq, vq;
  std::vector<float> k_scale, v_scale;
  size_t slots = 0, cap = 0;
  std::vector<float> q_tail, k_tail, v_tail;
};

enum class Qkv { Q, K, V };

struct V3Cache {  // cache.rs:148
  V3Config cfg;
  KvPrecision precision = KvPrecision::F32;
  std::vector<LayerCache> layers;
  std::vector<uint32_t> tokens;
  std::vector<std::vector<float>> engram_tail;
  size_t pos = 0;

  V3Cache(const V3Config& cfg, size_t hint, KvPrecision p);  // cache.rs:177
  size_t bytes() const;                                       // cache.rs:255
  void push_token(uint32_t tok);                              // cache.rs:276
  void ensure(size_t li, size_t pos);                         // cache.rs:291
  void span(size_t li, size_t pos, size_t* lo, size_t* hi) const;  // cache.rs:322
  bool is_saturated() const;                                  // cache.rs:335
  void write_kv(size_t li, size_t pos, const float* k, const float* v);  // cache.rs:346
  KvStore kv(size_t li) const;                                // cache.rs:382
  void conv_step(size_t li, Qkv which, const float* taps, float* raw, size_t dim);  // :401
  void engram_conv_step(size_t site, const float* taps, float* raw);                 // :444
  void seed_conv_tail(size_t li, Qkv which, const float* raw);                       // :486
  void seed_engram_tail(size_t site, const float* raw);                              // :498
  void seed_tokens(const uint32_t* toks, size_t n);                                  // :505
};

// ---------------------------------------------------------------- v3/engram.rs
std::vector<uint32_t> engram_indices(const uint32_t* tokens, size_t seq,
                                     const std::vector<size_t>& orders, size_t heads,
                                     uint32_t slots, size_t seed_heads);  // engram.rs:31
bool ngram_valid(size_t p, size_t table, const std::vector<size_t>& orders,
                 size_t heads);                                           // engram.rs:66
void value_conv(float* buf, const float* taps, size_t seq, size_t dim, size_t conv_taps,
                size_t conv_dilation, size_t max_order);                  // engram.rs:89
void apply_site(float* x, const float* k, const float* v, size_t d_model);  // engram.rs:112

// ---------------------------------------------------------------- v3/mhc.rs
struct MhcLayer {
  float a_pre, a_post, a_res;
  const float* b_pre;
  const float* b_post;
  const float* b_res;
};
float pre_off(size_t layer, size_t lane, size_t lanes);   // mhc.rs:56
float post_off(size_t layer, size_t lane, size_t lanes);  // mhc.rs:65
void mix_down(const float* lanes_buf, float* phi_pre_rows, const MhcLayer& m, size_t layer,
              size_t lanes, size_t d_model, float* u);    // mhc.rs:79
void scatter_up(float* lanes_buf, float* post, float* res, const float* y, const MhcLayer& m,
                size_t layer, size_t lanes, size_t d_model);  // mhc.rs:109

// ---------------------------------------------------------------- v3/kernels.rs
void hada_blocks(size_t n, size_t* ba, size_t* bb);  // kernels.rs:26
void kron_apply(const float* z, const float* a, const float* b, size_t ba, size_t bb,
                float* out);                          // kernels.rs:41
struct HadaMlp {                                      // kernels.rs:83
  std::vector<float> d1, d2, b2, d3, d4, w1a, w1b, w2a, w2b, w3a, w3b, cond_v, cond_u;
  size_t cond_rank = 0;
};
struct HadaPerms {
  std::vector<uint32_t> p1, p2;
};
void hadamard_mlp(const float* x, size_t d_model, const HadaMlp& w, const HadaPerms& perms,
                  size_t hada_n, float* out);  // kernels.rs:119

// ---------------------------------------------------------------- v3/model.rs
struct V3Layer {
  std::vector<float> norm_in;
  CqWeight q_proj, k_proj, v_proj;
  std::vector<float> q_taps, k_taps, v_taps, q_norm, k_norm;
  CqWeight gate_proj, out_proj;
  std::vector<float> post_norm;
  float attn_gate = 0.f;
  std::vector<float> pre_hada;
  HadaMlp mlp;
};
struct V3Mhc {
  std::vector<float> a_pre, a_post, a_res, b_pre, b_post, b_res;
  CqWeight phi_pre, phi_post, phi_res;
};
struct V3EngramSite {
  CqWeight tables, key_proj, value_proj;
  std::vector<float> taps;
};

// heads.rs:41-118: a probe head over the per-layer cells, dense weights.
struct ProbeHead {
  std::vector<float> probes, gain, query, row_bias, proj, bias;
  size_t cells = 0, probes_per_cell = 0, queries = 0, out_dim = 0;
  // `cells` shaped (seq, this->cells, d): out_dim logits (the two-pass form).
  std::vector<float> forward(const float* cells, size_t seq, size_t d) const;
};

struct V3Model {
  V3Config cfg;
  CqWeight embedding;
  std::vector<V3Layer> layers;
  V3Mhc mhc;
  std::vector<V3EngramSite> engrams;
  std::vector<float> final_norm;
  HadaPerms perms;
  float embed_scale = 0.f;

  std::vector<float> decode_step(V3Cache& cache, uint32_t token) const;        // model.rs:150
  std::vector<float> prefill(const uint32_t* tokens, size_t n, V3Cache& cache) const;  // :512
  std::vector<float> forward_sequence(const uint32_t* tokens, size_t n) const;  // :478
  std::vector<float> forward_impl(const uint32_t* tokens, size_t n, V3Cache* cache,
                                  std::vector<float>* cells = nullptr) const;  // :550
  // (seq, num_layers + 1, d): the scaled embedding, then each layer's lane mean (model.rs:494-502).
  std::vector<float> forward_cells(const uint32_t* tokens, size_t n) const;
  bool has_confidence = false;
  ProbeHead confidence;  // heads.rs HEAD_CONFIDENCE (code 2), when the container exports it
  size_t clamp_token(uint32_t t) const;
  void rope_at(size_t pos, float* c, float* s) const;
  void rope(size_t seq, std::vector<float>* c, std::vector<float>* s) const;
  void engram_kv_with_raw(const uint32_t* tokens, size_t seq, bool want_raw,
                          std::vector<float>* ks, std::vector<float>* vs,
                          std::vector<float>* raw) const;
};

// ---------------------------------------------------------------- cact.rs / v3.rs
struct Record {
  uint8_t dtype = 0, ndim = 0;
  size_t shape[4] = {0, 0, 0, 0};
  uint64_t offset = 0, nbytes = 0;
  size_t group = 0;
  uint8_t bits = 0;
};
constexpr uint32_t TAG_V3 = 0x05E12A84u;
constexpr size_t HEADER_BYTES_V3 = 49 * 4;
constexpr size_t REC_BYTES = 44;
constexpr uint8_t DT_FP16 = 1, DT_FP32 = 2, DT_CQ = 3, DT_RAW = 4;

// Parse container bytes and build the model (cact.rs:990-1030, v3.rs:25-484).
// Returns an empty string on success, else a message.
std::string load_model(const uint8_t* raw, size_t len, V3Model* out);

// ---------------------------------------------------------------- v3/ladder.rs, v3.rs:620-745
std::vector<size_t> ladder_order(size_t num_layers);                                   // ladder.rs:28
bool ladder_layer_indices(size_t num_layers, size_t depth, std::vector<size_t>* kept);  // ladder.rs:67
std::string slice_to_depth(V3Model* m, size_t depth);  // v3.rs:656, on a model loaded at full depth

}  // namespace oracle
