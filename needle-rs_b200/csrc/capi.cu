// extern "C" surface of libneedle_b200.so (declared in include/needle.h).
//
// Error model as crates/needle-c/src/lib.rs:27-40: a thread-local last error,
// cleared at the start of every needle_* call and set on failure; pointer
// results are NULL on failure, boolean results false, sizes 0.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/needle.h"
#include "constrained.hpp"
#include "engine.hpp"

struct NeedleV3Handle {
  std::shared_ptr<nb::Engine> eng;
};
struct NeedleV3Session {
  std::shared_ptr<nb::Engine> eng;  // keeps the engine alive until this object is freed
  std::unique_ptr<nb::Session> s;
};
struct NeedleV3Batch {
  std::shared_ptr<nb::Engine> eng;  // keeps the engine alive until this object is freed
  std::unique_ptr<nb::Batch> b;
};

namespace {
thread_local std::string g_err;
thread_local bool g_has_err = false;
thread_local std::string g_nd_err;

void clear_err() {
  g_has_err = false;
  g_err.clear();
}
void set_err(const std::string& m) {
  g_err = m;
  g_has_err = true;
}

NeedleV3Handle* load_engine(const uint8_t* data, size_t len, const std::string& what, size_t depth = 0) {
  std::string err;
  nb::Engine* e = nb::Engine::load(data, len, &err, depth);
  if (!e) {
    set_err(what + err);
    return nullptr;
  }
  NeedleV3Handle* h = new NeedleV3Handle();
  h->eng.reset(e);
  return h;
}

bool read_file(const char* path, std::vector<uint8_t>* out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  f.seekg(0, std::ios::end);
  std::streamoff n = f.tellg();
  if (n < 0) return false;
  f.seekg(0, std::ios::beg);
  out->resize((size_t)n);
  return (bool)f.read(reinterpret_cast<char*>(out->data()), n) || n == 0;
}

char* out_string(const std::string& s) {
  char* p = (char*)std::malloc(s.size() + 1);
  if (!p) {
    set_err("out of host memory");
    return nullptr;
  }
  std::memcpy(p, s.c_str(), s.size() + 1);
  return p;
}

const char* kNoTokenizer =
    "the container has no tokenizer record, so text-level calls cannot run; use the token-level API "
    "(needle_v3_prefill / needle_v3_decode_step / needle_v3_generate_ids)";

// Defaults of V3Options (v3_engine.rs:26, :65-76) and the ids upstream fixes
// for the stop and start tokens (v3_engine.rs:175-178).
constexpr size_t kDefaultMaxNewTokens = 256;
constexpr uint32_t kEosId = 1, kBosId = 2;

bool utf8_ok(const char* s) {
  if (!s) return false;
  const std::string t(s);
  return nb::utf8_lossy(t) == t;
}

// compact_json (prompt.rs): whitespace outside JSON strings removed.
std::string compact_json(const std::string& s) {
  std::string out;
  bool in_str = false, esc = false;
  for (char c : s) {
    if (in_str) {
      out += c;
      if (esc) esc = false;
      else if (c == '\\') esc = true;
      else if (c == '"') in_str = false;
      continue;
    }
    if (c == '"') {
      in_str = true;
      out += c;
    } else if (c != ' ' && c != '\t' && c != '\n' && c != '\r') {
      out += c;
    }
  }
  return out;
}

// build_prompt (prompt.rs), no system turn: the user turn carries the compact
// tool list between <tools> markers, then the assistant turn is opened.
std::string build_prompt(const std::string& query, const std::string& tools_json) {
  return "<|im_start|>user\n<tools>" + compact_json(tools_json) + "</tools>\n" + query +
         "<|im_end|>\n<|im_start|>assistant\n";
}

// The text between `open` and `close` (to the end when unterminated), or
// false when `open` is absent (v3_engine.rs:392-401).
bool between(const std::string& text, const char* open, const char* close, std::string* out) {
  size_t a = text.find(open);
  if (a == std::string::npos) return false;
  a += std::strlen(open);
  const size_t b = text.find(close, a);
  *out = text.substr(a, b == std::string::npos ? std::string::npos : b - a);
  return true;
}

// Unicode White_Space (what Rust's str::trim removes).
bool unicode_ws(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F ||
         c == 0x3000;
}

// Code point of the well-formed UTF-8 sequence of `n` bytes at p.
uint32_t code_point(const char* p, size_t n) {
  const unsigned char* u = reinterpret_cast<const unsigned char*>(p);
  if (n == 1) return u[0];
  uint32_t c = u[0] & (0xFF >> (n + 1));
  for (size_t k = 1; k < n; ++k) c = (c << 6) | (u[k] & 0x3F);
  return c;
}

// Leading and trailing Unicode white space removed from UTF-8 text.
std::string trim(const std::string& s) {
  auto seq_len = [](unsigned char b) -> size_t { return b < 0x80 ? 1 : b < 0xE0 ? 2 : b < 0xF0 ? 3 : 4; };
  size_t i = 0, j = s.size();
  while (i < j) {
    const size_t n = std::min(seq_len((unsigned char)s[i]), j - i);
    if (!unicode_ws(code_point(s.data() + i, n))) break;
    i += n;
  }
  while (j > i) {
    size_t k = j - 1;
    while (k > i && ((unsigned char)s[k] & 0xC0) == 0x80) --k;
    if (!unicode_ws(code_point(s.data() + k, j - k))) break;
    j = k;
  }
  return s.substr(i, j - i);
}

int nd_status(cudaError_t e) {
  if (e == cudaSuccess) return 0;
  g_nd_err = std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e);
  return (int)e;
}

nb::CqMat make_cq(const void* packed, const void* norms, int rows, int in_feat, int bits,
                  const float* levels) {
  nb::CqMat W;
  std::memset(&W, 0, sizeof(W));
  const int in_pad = (in_feat + 127) / 128 * 128;
  W.seg[0].packed = (const uint8_t*)packed;
  W.seg[0].norms = (const __half*)norms;
  W.seg[0].rows = rows;
  W.nseg = 1;
  W.rows = rows;
  W.in_feat = in_feat;
  W.in_pad = in_pad;
  W.row_bytes = in_pad * bits / 8;
  W.groups = in_pad / 128;
  W.group = 128;
  W.bits = bits;
  for (int i = 0; i < (1 << bits) && i < 16; ++i) W.levels[i] = levels[i];
  return W;
}

// Stream-ordered scratch of the nd_* entry points comes from a library-owned
// memory pool per device whose release threshold keeps freed memory reserved,
// so repeated calls reuse it instead of mapping new memory each time.
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st) {
  static std::mutex mu;
  static std::vector<cudaMemPool_t> pools;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  cudaMemPool_t pool = nullptr;
  {
    std::lock_guard<std::mutex> lk(mu);
    if ((int)pools.size() <= dev) pools.resize(dev + 1, nullptr);
    if (!pools[dev]) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      e = cudaMemPoolCreate(&pools[dev], &props);
      if (e != cudaSuccess) {
        pools[dev] = nullptr;
        return e;
      }
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
    }
    pool = pools[dev];
  }
  return cudaMallocFromPoolAsync(p, bytes, pool, st);
}

// SplitMix64 and temperature sampling as crates/needle-infer/src/v3_engine.rs:422-464.
struct SplitMix64 {
  uint64_t s;
  uint64_t next_u64() {
    s += 0x9E3779B97F4A7C15ull;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  double next_f64() { return (double)(next_u64() >> 11) / (double)(1ull << 53); }
};
uint32_t sample(const float* logits, size_t n, float temperature, SplitMix64* rng) {
  const float inv = 1.0f / temperature;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i)
    if (logits[i] > mx) mx = logits[i];
  double sum = 0.0;
  for (size_t i = 0; i < n; ++i) sum += (double)expf((logits[i] - mx) * inv);
  double target = rng->next_f64() * sum;
  for (size_t i = 0; i < n; ++i) {
    target -= (double)expf((logits[i] - mx) * inv);
    if (target <= 0.0) return (uint32_t)i;
  }
  return (uint32_t)(n - 1);
}

struct TextOptions {
  size_t max_new_tokens = kDefaultMaxNewTokens;
  float temperature = 0.f;
  uint64_t seed = 0;
  bool kv_int8 = false;
  bool constrain = false;
};

// First maximum, as argmax (v3_engine.rs:410-420).
uint32_t host_argmax(const float* v, size_t n) {
  size_t best = 0;
  float top = -INFINITY;
  for (size_t i = 0; i < n; ++i)
    if (v[i] > top) {
      top = v[i];
      best = i;
    }
  return (uint32_t)best;
}

// V3Engine::generate_with (v3_engine.rs:193-305): the chat prompt as [bos] +
// encode(prompt), truncated to the context; one batched prefill, then greedy
// or temperature sampling until </s>, <|im_end|>, the token budget or the end
// of the context. With `constrain` and at least one declared tool, the logits
// inside a <tool_call> span get the grammar mask first. Every step's newly
// decoded text goes to `cb` (the whole run is re-decoded so byte-fallback
// characters split over several tokens arrive whole). False with *err set on
// failure.
bool generate_text(nb::Engine* E, const std::string& query, const std::string& tools, const TextOptions& o,
                   void (*cb)(const char*, void*), void* ud, std::string* text, std::string* err) {
  if (!E->tok) {
    *err = kNoTokenizer;
    return false;
  }
  const nb::Tokenizer& T = *E->tok;
  uint32_t im_end = UINT32_MAX;
  T.id_of("<|im_end|>", &im_end);
  std::vector<uint32_t> ids = {kBosId};
  const std::vector<uint32_t> enc = T.encode(build_prompt(query, tools));
  ids.insert(ids.end(), enc.begin(), enc.end());
  const size_t max = E->cfg.max_seq;
  if (ids.size() > max) ids.resize(max);
  const size_t budget = std::min(max - ids.size(), o.max_new_tokens);
  std::vector<uint32_t> out;
  text->clear();
  if (budget == 0) return true;
  std::unique_ptr<nb::Session> s(E->new_session(ids.size() + budget, o.kv_int8, err));
  if (!s) return false;
  const size_t rows = E->cfg.logit_rows();
  std::unique_ptr<nb::ConstrainedDecoder> grammar;
  if (o.constrain) {
    const std::vector<nb::ToolDef> defs = nb::parse_tools_json(tools);
    if (!defs.empty()) grammar.reset(new nb::ConstrainedDecoder(defs, T.token_bytes(), true));
  }
  uint32_t tc_start = 0, tc_end = 0;
  const bool has_start = T.id_of("<tool_call>", &tc_start), has_end = T.id_of("</tool_call>", &tc_end);
  bool in_call = false;
  std::vector<float> logits(rows);
  float* lp = o.temperature > 0.f || grammar ? logits.data() : nullptr;
  nb::Session* sp = s.get();
  const uint32_t* idp[1] = {ids.data()};
  size_t lens[1] = {ids.size()};
  uint32_t pick = 0;
  if (!E->prefill(&sp, idp, lens, 1, lp, &pick, err)) return false;
  SplitMix64 rng{o.seed};
  std::string emitted;
  for (size_t t = 0; t < budget; ++t) {
    if (in_call && grammar) {
      const std::vector<float> mask = grammar->logit_mask(rows);
      for (size_t i = 0; i < rows; ++i) logits[i] += mask[i];
    }
    const uint32_t next = o.temperature > 0.f ? sample(logits.data(), rows, o.temperature, &rng)
                          : lp                ? host_argmax(logits.data(), rows)
                                              : pick;
    if (next == kEosId || next == im_end) break;
    out.push_back(next);
    if (grammar) {
      if (has_start && next == tc_start) in_call = true;
      else if (has_end && next == tc_end) in_call = false;
      else if (in_call) grammar->update(next);
    }
    const std::string full = T.decode(out.data(), out.size());
    if (full.size() > emitted.size()) {
      const std::string delta = full.substr(emitted.size());
      if (cb && delta.find('\0') == std::string::npos) cb(delta.c_str(), ud);
      emitted = full;
    }
    if (sp->pos >= max) break;
    if (!E->decode(&sp, &next, 1, lp, &pick, err)) return false;
  }
  *text = T.decode(out.data(), out.size());
  return true;
}

// Shared argument checks of the text calls (v3.rs:131-150): NULL or
// non-UTF-8 strings fail with the reference's messages.
bool text_args(NeedleV3Handle* h, const char* query, const char* tools_json) {
  if (!h) {
    set_err("handle was null");
    return false;
  }
  if (!utf8_ok(query)) {
    set_err("query was null or not UTF-8");
    return false;
  }
  if (!utf8_ok(tools_json)) {
    set_err("tools_json was null or not UTF-8");
    return false;
  }
  return true;
}

char* text_call(NeedleV3Handle* h, const char* query, const char* tools_json, const TextOptions& o,
                void (*cb)(const char*, void*), void* ud) {
  if (!text_args(h, query, tools_json)) return nullptr;
  std::string text, err;
  if (!generate_text(h->eng.get(), query, tools_json, o, cb, ud, &text, &err)) {
    set_err(err);
    return nullptr;
  }
  return out_string(text);
}
}  // namespace

extern "C" {

// ------------------------------------------------------------------ Part 1
NeedleV3Handle* needle_v3_load(const char* cact_path) {
  clear_err();
  if (!cact_path) {
    set_err("cact_path was null or not UTF-8");
    return nullptr;
  }
  std::vector<uint8_t> raw;
  if (!read_file(cact_path, &raw)) {
    set_err(std::string("failed to load ") + cact_path + ": cannot read file");
    return nullptr;
  }
  return load_engine(raw.data(), raw.size(), std::string("failed to load ") + cact_path + ": ");
}

NeedleV3Handle* needle_v3_load_bytes(const unsigned char* data, size_t len) {
  clear_err();
  if (!data) {
    set_err("data was null");
    return nullptr;
  }
  return load_engine(data, len, "failed to load container: ");
}

NeedleV3Handle* needle_v3_load_bytes_with_depth(const unsigned char* data, size_t len, size_t layers) {
  clear_err();
  if (!data) {
    set_err("data was null");
    return nullptr;
  }
  const std::string what = "failed to load container at " + std::to_string(layers) + " layers: ";
  if (layers == 0) {
    set_err(what + "depth is outside the ladder");
    return nullptr;
  }
  return load_engine(data, len, what, layers);
}

NeedleV3Handle* needle_v3_load_with_depth(const char* cact_path, size_t layers) {
  clear_err();
  if (!cact_path) {
    set_err("cact_path was null or not UTF-8");
    return nullptr;
  }
  const std::string what = std::string("failed to load ") + cact_path + " at " + std::to_string(layers) + " layers: ";
  std::vector<uint8_t> raw;
  if (!read_file(cact_path, &raw)) {
    set_err(what + "cannot read file");
    return nullptr;
  }
  // 0 is not a rung (the engine reads 0 as "every block").
  if (layers == 0) {
    set_err(what + "depth is outside the ladder");
    return nullptr;
  }
  return load_engine(raw.data(), raw.size(), what, layers);
}

size_t needle_v3_num_layers(NeedleV3Handle* h) {
  clear_err();
  if (!h) {
    set_err("handle was null");
    return 0;
  }
  return h->eng->cfg.layers;
}

char* needle_v3_run(NeedleV3Handle* h, const char* query, const char* tools_json) {
  clear_err();
  return text_call(h, query, tools_json, TextOptions(), nullptr, nullptr);
}

// The <tool_call> payload of run(), trimmed; an empty string when the model
// emitted no call (v3.rs:171-181 returns unwrap_or_default()).
char* needle_v3_run_json(NeedleV3Handle* h, const char* query, const char* tools_json) {
  clear_err();
  if (!text_args(h, query, tools_json)) return nullptr;
  std::string text, err, call;
  if (!generate_text(h->eng.get(), query, tools_json, TextOptions(), nullptr, nullptr, &text, &err)) {
    set_err(err);
    return nullptr;
  }
  return out_string(between(text, "<tool_call>", "</tool_call>", &call) ? trim(call) : std::string());
}

// V3Engine::reasoning (v3_engine.rs:382-401): the text between <think> and
// </think> (or to the end when unterminated), trimmed; NULL when absent.
char* needle_v3_reasoning(NeedleV3Handle* h, const char* text) {
  clear_err();
  if (!h) {
    set_err("handle was null");
    return nullptr;
  }
  if (!utf8_ok(text)) {
    set_err("text was null or not UTF-8");
    return nullptr;
  }
  std::string mid;
  if (!between(text, "<think>", "</think>", &mid)) return nullptr;
  return out_string(trim(mid));
}

char* needle_v3_generate(NeedleV3Handle* h, const char* query, const char* tools_json,
                         size_t max_new_tokens, float temperature, uint64_t seed, bool constrain,
                         bool kv_int8) {
  clear_err();
  TextOptions o;
  o.constrain = constrain;
  o.max_new_tokens = max_new_tokens == 0 ? kDefaultMaxNewTokens : max_new_tokens;
  o.temperature = temperature;
  o.seed = seed;
  o.kv_int8 = kv_int8;
  return text_call(h, query, tools_json, o, nullptr, nullptr);
}

char* needle_v3_run_stream(NeedleV3Handle* h, const char* query, const char* tools_json,
                           void (*cb)(const char*, void*), void* userdata) {
  clear_err();
  return text_call(h, query, tools_json, TextOptions(), cb, userdata);
}

bool needle_v3_has_confidence(NeedleV3Handle* h) {
  clear_err();
  if (!h) {
    set_err("handle was null");
    return false;
  }
  return h->eng->cfg.has_heads;
}

bool needle_v3_confidence_for(NeedleV3Handle* h, const char* query, const char* tools_json,
                              const char* completion, float* out) {
  clear_err();
  if (!h) set_err("handle was null");
  else if (!utf8_ok(query) || !utf8_ok(tools_json) || !utf8_ok(completion))
    set_err("an argument was null or not UTF-8");
  else if (!out) set_err("out was null");
  else if (!h->eng->cfg.has_heads) set_err("this container exports no confidence head");
  else if (!h->eng->tok) set_err(kNoTokenizer);
  else {
    // V3Engine::confidence_for (v3_engine.rs:351-368): the prompt plus the
    // completion, [bos] + encode(), truncated to the context; the sigmoid of
    // the head's first logit.
    nb::Engine* E = h->eng.get();
    std::vector<uint32_t> ids = {kBosId};
    const std::vector<uint32_t> enc = E->tok->encode(build_prompt(query, tools_json) + completion);
    ids.insert(ids.end(), enc.begin(), enc.end());
    if (ids.size() > E->cfg.max_seq) ids.resize(E->cfg.max_seq);
    float logit = 0.f;
    std::string err;
    if (!E->confidence(ids.data(), ids.size(), &logit, &err)) {
      set_err(err);
      return false;
    }
    *out = 1.0f / (1.0f + expf(-logit));
    return true;
  }
  return false;
}

size_t needle_v3_kv_bytes(NeedleV3Handle* h, size_t seq_len, bool kv_int8) {
  clear_err();
  if (!h) {
    set_err("handle was null");
    return 0;
  }
  return h->eng->cfg.kv_bytes_at(seq_len, kv_int8);
}

size_t needle_v3_max_seq_len(NeedleV3Handle* h) {
  clear_err();
  if (!h) {
    set_err("handle was null");
    return 0;
  }
  return h->eng->cfg.max_seq;
}

void needle_v3_free(NeedleV3Handle* h) { delete h; }

void needle_free_str(char* s) { std::free(s); }

const char* needle_last_error(void) { return g_has_err ? g_err.c_str() : nullptr; }

// ------------------------------------------------------------------ Part 2
NeedleV3Session* needle_v3_session_new(NeedleV3Handle* h, size_t hint, bool kv_int8) {
  clear_err();
  if (!h) {
    set_err("handle was null");
    return nullptr;
  }
  std::string err;
  nb::Session* s = h->eng->new_session(hint, kv_int8, &err);
  if (!s) {
    set_err(err);
    return nullptr;
  }
  NeedleV3Session* r = new NeedleV3Session();
  r->eng = h->eng;
  r->s.reset(s);
  return r;
}

void needle_v3_session_free(NeedleV3Session* s) { delete s; }

size_t needle_v3_session_pos(NeedleV3Session* s) {
  clear_err();
  if (!s) {
    set_err("session was null");
    return 0;
  }
  return s->s->pos;
}

size_t needle_v3_session_bytes(NeedleV3Session* s) {
  clear_err();
  if (!s) {
    set_err("session was null");
    return 0;
  }
  return s->s->bytes();
}

size_t needle_v3_session_slots(NeedleV3Session* s, size_t layer) {
  clear_err();
  if (!s || layer >= s->s->layers.size()) {
    set_err("session was null or layer out of range");
    return 0;
  }
  return (size_t)s->s->layers[layer].slots;
}

uint32_t needle_v3_sample(const float* logits, size_t n, float temperature, uint64_t* rng_state) {
  clear_err();
  if (!logits || !rng_state || n == 0) {
    set_err("logits or rng_state was null, or n was 0");
    return UINT32_MAX;
  }
  if (!(temperature > 0.f)) {
    set_err("temperature must be positive");
    return UINT32_MAX;
  }
  SplitMix64 rng{*rng_state};
  const uint32_t pick = sample(logits, n, temperature, &rng);
  *rng_state = rng.s;
  return pick;
}

bool needle_v3_session_kv(NeedleV3Session* s, size_t layer, void* k, void* v, float* k_scale,
                          float* v_scale) {
  clear_err();
  if (!s) {
    set_err("session was null");
    return false;
  }
  if (s->s->int8 && (!!k_scale != !!k || !!v_scale != !!v)) {
    set_err("an int8 ring is read with its scales");
    return false;
  }
  std::string err;
  if (!s->eng->read_kv(s->s.get(), layer, k, v, k_scale, v_scale, &err)) {
    set_err(err);
    return false;
  }
  return true;
}

static bool check_sessions(NeedleV3Handle* h, NeedleV3Session* const* ss, size_t n,
                           std::vector<nb::Session*>* out) {
  if (!h) {
    set_err("handle was null");
    return false;
  }
  if (n && !ss) {
    set_err("sessions was null");
    return false;
  }
  out->resize(n);
  for (size_t i = 0; i < n; ++i) {
    if (!ss[i] || ss[i]->eng != h->eng) {
      set_err("session was null or belongs to another handle");
      return false;
    }
    (*out)[i] = ss[i]->s.get();
  }
  return true;
}

bool needle_v3_prefill(NeedleV3Handle* h, NeedleV3Session* s, const uint32_t* ids, size_t n,
                       float* logits) {
  clear_err();
  std::vector<nb::Session*> v;
  if (!check_sessions(h, &s, 1, &v)) return false;
  if (!ids && n) {
    set_err("ids was null");
    return false;
  }
  if (n == 0) return true;  // empty prompt: nothing to report (model.rs:516-518)
  std::string err;
  const uint32_t* idp[1] = {ids};
  size_t lens[1] = {n};
  if (!h->eng->prefill(v.data(), idp, lens, 1, logits, nullptr, &err)) {
    set_err(err);
    return false;
  }
  return true;
}

bool needle_v3_decode_step(NeedleV3Handle* h, NeedleV3Session* s, uint32_t token, float* logits) {
  clear_err();
  std::vector<nb::Session*> v;
  if (!check_sessions(h, &s, 1, &v)) return false;
  std::string err;
  if (!h->eng->decode(v.data(), &token, 1, logits, nullptr, &err)) {
    set_err(err);
    return false;
  }
  return true;
}

bool needle_v3_prefill_batch(NeedleV3Handle* h, NeedleV3Session* const* ss, const uint32_t* ids,
                             const size_t* lens, size_t n, float* last_logits, uint32_t* picks) {
  clear_err();
  std::vector<nb::Session*> v;
  if (!check_sessions(h, ss, n, &v)) return false;
  if (n && (!ids || !lens)) {
    set_err("ids or lens was null");
    return false;
  }
  std::vector<const uint32_t*> idp(n);
  size_t off = 0;
  for (size_t i = 0; i < n; ++i) {
    idp[i] = ids + off;
    off += lens[i];
  }
  std::string err;
  if (!h->eng->prefill(v.data(), idp.data(), lens, n, last_logits, picks, &err)) {
    set_err(err);
    return false;
  }
  return true;
}

bool needle_v3_decode_batch(NeedleV3Handle* h, NeedleV3Session* const* ss, const uint32_t* tokens,
                            size_t n, float* logits, uint32_t* picks) {
  clear_err();
  std::vector<nb::Session*> v;
  if (!check_sessions(h, ss, n, &v)) return false;
  if (n && !tokens) {
    set_err("tokens was null");
    return false;
  }
  std::string err;
  if (!h->eng->decode(v.data(), tokens, n, logits, picks, &err)) {
    set_err(err);
    return false;
  }
  return true;
}

size_t needle_v3_generate_ids(NeedleV3Handle* h, const uint32_t* prompt, size_t n,
                              size_t max_new_tokens, float temperature, uint64_t seed, bool kv_int8,
                              uint32_t eos_id, uint32_t* out_ids) {
  clear_err();
  const size_t FAIL = (size_t)-1;
  if (!h) {
    set_err("handle was null");
    return FAIL;
  }
  if ((!prompt && n) || (!out_ids && max_new_tokens)) {
    set_err("prompt or out_ids was null");
    return FAIL;
  }
  if (n == 0 || max_new_tokens == 0) return 0;
  nb::Engine* E = h->eng.get();
  const size_t max = E->cfg.max_seq;
  if (n > max) n = max;  // prompt truncation, v3_engine.rs:206-214
  const size_t budget = std::min(max - n, max_new_tokens);
  std::string err;
  std::unique_ptr<nb::Session> s(E->new_session(n + budget, kv_int8, &err));
  if (!s) {
    set_err(err);
    return FAIL;
  }
  const size_t rows = E->cfg.logit_rows();
  std::vector<float> logits(rows);
  nb::Session* sp = s.get();
  const uint32_t* idp[1] = {prompt};
  size_t lens[1] = {n};
  uint32_t pick = 0;
  if (!E->prefill(&sp, idp, lens, 1, temperature > 0.f ? logits.data() : nullptr, &pick, &err)) {
    set_err(err);
    return FAIL;
  }
  SplitMix64 rng{seed};
  size_t count = 0;
  for (size_t t = 0; t < budget; ++t) {
    uint32_t next = temperature > 0.f ? sample(logits.data(), rows, temperature, &rng) : pick;
    if (eos_id != UINT32_MAX && next == eos_id) break;
    out_ids[count++] = next;
    if (sp->pos >= max) break;
    if (!E->decode(&sp, &next, 1, temperature > 0.f ? logits.data() : nullptr, &pick, &err)) {
      set_err(err);
      return FAIL;
    }
  }
  return count;
}

NeedleV3Batch* needle_v3_batch_new(NeedleV3Handle* h, NeedleV3Session* const* ss, size_t n) {
  clear_err();
  std::vector<nb::Session*> v;
  if (!check_sessions(h, ss, n, &v)) return nullptr;
  std::string err;
  nb::Batch* b = h->eng->new_batch(v.data(), n, &err);
  if (!b) {
    set_err(err);
    return nullptr;
  }
  NeedleV3Batch* r = new NeedleV3Batch();
  r->eng = h->eng;
  r->b.reset(b);
  return r;
}

void needle_v3_batch_free(NeedleV3Batch* b) { delete b; }

uint32_t* needle_v3_batch_tokens(NeedleV3Batch* b) {
  clear_err();
  if (!b) {
    set_err("batch was null");
    return nullptr;
  }
  return b->b->d_tok;
}

uint32_t* needle_v3_batch_next(NeedleV3Batch* b) {
  clear_err();
  if (!b) {
    set_err("batch was null");
    return nullptr;
  }
  return b->b->d_next;
}

bool needle_v3_batch_step(NeedleV3Batch* b, float* d_logits, void* stream, bool use_graph) {
  clear_err();
  if (!b) {
    set_err("batch was null");
    return false;
  }
  nb::Engine* E = b->eng.get();
  cudaStream_t st = stream ? (cudaStream_t)stream : E->stream;
  std::string err;
  if (!E->decode_batch_device(b->b.get(), d_logits, st, use_graph, &err)) {
    set_err(err);
    return false;
  }
  return true;
}

bool needle_v3_batch_feed_next(NeedleV3Batch* b, void* stream) {
  clear_err();
  if (!b) {
    set_err("batch was null");
    return false;
  }
  nb::Engine* E = b->eng.get();
  cudaStream_t st = stream ? (cudaStream_t)stream : E->stream;
  cudaError_t e = cudaMemcpyAsync(b->b->d_tok, b->b->d_next, b->b->sessions.size() * 4,
                                  cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) {
    set_err(std::string("feeding tokens: ") + cudaGetErrorString(e));
    return false;
  }
  return true;
}

bool needle_v3_batch_profile(NeedleV3Batch* b, float* ms, int* launches) {
  clear_err();
  if (!b || !ms || !launches) {
    set_err("batch, ms or launches was null");
    return false;
  }
  std::string err;
  if (!b->eng->profile_batch_step(b->b.get(), ms, launches, &err)) {
    set_err(err);
    return false;
  }
  return true;
}

static bool batch_copy(NeedleV3Batch* b, void* dst, const void* src, cudaMemcpyKind kind) {
  nb::Engine* E = b->eng.get();
  cudaError_t e = cudaMemcpyAsync(dst, src, b->b->sessions.size() * 4, kind, E->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(E->stream);
  if (e != cudaSuccess) {
    set_err(std::string("batch token copy: ") + cudaGetErrorString(e));
    return false;
  }
  return true;
}

bool needle_v3_batch_set_tokens(NeedleV3Batch* b, const uint32_t* tokens) {
  clear_err();
  if (!b || !tokens) {
    set_err("batch or tokens was null");
    return false;
  }
  // The batch's previous step may run on another stream: wait for the device.
  cudaDeviceSynchronize();
  return batch_copy(b, b->b->d_tok, tokens, cudaMemcpyHostToDevice);
}

bool needle_v3_batch_get_next(NeedleV3Batch* b, uint32_t* next) {
  clear_err();
  if (!b || !next) {
    set_err("batch or next was null");
    return false;
  }
  cudaSetDevice(b->eng->device);
  cudaDeviceSynchronize();
  if (b->eng->take_wait_flag() == cudaErrorTimeout) {
    set_err("a kernel of an earlier step gave up a bounded wait; its results are invalid");
    return false;
  }
  return batch_copy(b, next, b->b->d_next, cudaMemcpyDeviceToHost);
}

struct NeedleTokenizer {
  std::unique_ptr<nb::Tokenizer> t;
};

NeedleTokenizer* needle_tokenizer_new(const unsigned char* blob, size_t len) {
  clear_err();
  if (!blob) {
    set_err("blob was null");
    return nullptr;
  }
  std::string err;
  nb::Tokenizer* t = nb::Tokenizer::from_blob(blob, len, &err);
  if (!t) {
    set_err(err);
    return nullptr;
  }
  NeedleTokenizer* r = new NeedleTokenizer();
  r->t.reset(t);
  return r;
}

void needle_tokenizer_free(NeedleTokenizer* t) { delete t; }

size_t needle_tokenizer_encode(NeedleTokenizer* t, const char* text, uint32_t* out, size_t cap) {
  clear_err();
  if (!t) {
    set_err("tokenizer was null");
    return (size_t)-1;
  }
  if (!utf8_ok(text)) {
    set_err("text was null or not UTF-8");
    return (size_t)-1;
  }
  const std::vector<uint32_t> ids = t->t->encode(text);
  if (out)
    for (size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
  return ids.size();
}

char* needle_tokenizer_decode(NeedleTokenizer* t, const uint32_t* ids, size_t n) {
  clear_err();
  if (!t) {
    set_err("tokenizer was null");
    return nullptr;
  }
  if (!ids && n) {
    set_err("ids was null");
    return nullptr;
  }
  return out_string(t->t->decode(ids, n));
}

bool needle_tokenizer_tool_mask(NeedleTokenizer* t, const char* tools_json, const unsigned char* out_bytes,
                                size_t n, bool unique_keys, float* mask, size_t vocab) {
  clear_err();
  if (!t || !mask || (!out_bytes && n)) {
    set_err("tokenizer, out_bytes or mask was null");
    return false;
  }
  if (!utf8_ok(tools_json)) {
    set_err("tools_json was null or not UTF-8");
    return false;
  }
  nb::ConstrainedDecoder g(nb::parse_tools_json(tools_json), t->t->token_bytes(), unique_keys);
  g.feed_bytes(std::string(reinterpret_cast<const char*>(out_bytes), n));
  const std::vector<float> m = g.logit_mask(vocab);
  std::copy(m.begin(), m.end(), mask);
  return true;
}

bool needle_v3_geometry(NeedleV3Handle* h, int64_t* out) {
  clear_err();
  if (!h || !out) {
    set_err("handle or out was null");
    return false;
  }
  const nb::HostConfig& c = h->eng->cfg;
  int64_t v[14] = {(int64_t)c.vocab, (int64_t)c.out_vocab, (int64_t)c.d,       (int64_t)c.heads,
                   (int64_t)c.kvh,   (int64_t)c.layers,    (int64_t)c.qk,      (int64_t)c.vh,
                   (int64_t)c.max_seq, (int64_t)c.hada_n,  (int64_t)c.lanes,   (int64_t)c.window,
                   (int64_t)c.taps,  (int64_t)c.logit_rows()};
  std::memcpy(out, v, sizeof(v));
  return true;
}

int needle_v3_device(NeedleV3Handle* h) { return h ? h->eng->device : -1; }

// Copies one engine workspace buffer (the last forward's intermediates) to the
// host, for debugging and tests: 0 xh, 1 proj, 2 qpost, 3 int8 query scales, 4 oh, 5 projo,
// 6 prefill keys (f32), 7 prefill values (f32), 8 lanes, 9 u, 10 bx, 11 lm_in.
bool needle_v3_debug_buffer(NeedleV3Handle* h, int which, float* out, size_t count) {
  clear_err();
  if (!h || !out) {
    set_err("handle or out was null");
    return false;
  }
  nb::Workspace& w = h->eng->ws;
  const void* src[] = {w.xh, w.proj, w.qpost, w.q8s, w.oh, w.projo, w.pk, w.pv, w.lanes, w.u, w.bx, w.lm_in};
  if (which < 0 || which >= (int)(sizeof(src) / sizeof(src[0])) || !src[which]) {
    set_err("no such buffer");
    return false;
  }
  cudaError_t e = cudaStreamSynchronize(h->eng->stream);
  if (e == cudaSuccess) e = cudaMemcpy(out, src[which], count * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    set_err(cudaGetErrorString(e));
    return false;
  }
  return true;
}

// ------------------------------------------------------------------ Part 3
// One projection of a built matrix: the tensor-core path gets stream-ordered
// scratch, the others run directly.
static int project_mat(const nb::CqMat& W, const float* xh, int ldx, int M, float* y, int ldy, int row0, int nrows,
                       int path, cudaStream_t st) {
  const int rows = W.rows;
  const bool tensor_cores = path == 3 || (path == 0 && M > 8 && nb::umma_supported(W));
  if (!tensor_cores || M <= 0) return nd_status(nb::cq_project(W, xh, ldx, M, y, ldy, row0, nrows, st, path));
  // The split activations live in stream-ordered scratch, released on `stream`.
  if (nrows <= 0 || row0 < 0 || row0 + nrows > rows) return nd_status(cudaErrorInvalidValue);
  nb::GemmScratch gs;
  gs.elems = (size_t)M * W.in_pad;
  gs.welems = (size_t)nrows * W.in_pad;
  void* mem = nullptr;
  // hi / lo [M][in_pad], the level tiles, and one inverse scale per 128-wide group.
  cudaError_t e = scratch_alloc(
      &mem, (gs.elems + gs.welems) * 2 * sizeof(__half) + (size_t)M * (W.in_pad / 128) * sizeof(float), st);
  if (e != cudaSuccess) return nd_status(e);
  gs.hi = (__half*)mem;
  gs.lo = gs.hi + gs.elems;
  gs.whi = gs.lo + gs.elems;
  gs.wlo = gs.whi + gs.welems;
  gs.inv = reinterpret_cast<float*>(gs.wlo + gs.welems);
  gs.rows = (size_t)M;
  e = nb::cq_project(W, xh, ldx, M, y, ldy, row0, nrows, st, path, &gs);
  cudaError_t f = cudaFreeAsync(mem, st);
  return nd_status(e != cudaSuccess ? e : f);
}

int nd_cq_project(const void* packed, const void* norms, int rows, int in_feat, int bits,
                  const float* levels, const float* xh, int ldx, int M, float* y, int ldy, int row0,
                  int nrows, int path, void* stream) {
  if (!packed || !norms || !levels || !xh || !y || rows <= 0 || in_feat <= 0 || (bits != 2 && bits != 4))
    return nd_status(cudaErrorInvalidValue);
  const nb::CqMat W = make_cq(packed, norms, rows, in_feat, bits, levels);
  return project_mat(W, xh, ldx, M, y, ldy, row0, nrows, path, (cudaStream_t)stream);
}

int nd_cq_project_grouped(int count, const void* const* packed, const void* const* norms, const int* rows,
                          int in_feat, int bits, const float* levels, const float* xh, int ldx, int M, float* y,
                          int ldy, int path, void* stream) {
  if (count < 1 || count > nb::MAX_SEG || !packed || !norms || !rows || !levels || !xh || !y || in_feat <= 0 ||
      (bits != 2 && bits != 4))
    return nd_status(cudaErrorInvalidValue);
  for (int i = 0; i < count; ++i)
    if (!packed[i] || !norms[i] || rows[i] <= 0) return nd_status(cudaErrorInvalidValue);
  // One matrix whose row segments are the given matrices (the form the engine
  // gives a block's q|k|v|gate).
  nb::CqMat W = make_cq(packed[0], norms[0], rows[0], in_feat, bits, levels);
  for (int i = 1; i < count; ++i) {
    W.seg[i].packed = (const uint8_t*)packed[i];
    W.seg[i].norms = (const __half*)norms[i];
    W.seg[i].rows = rows[i];
    W.rows += rows[i];
  }
  W.nseg = count;
  return project_mat(W, xh, ldx, M, y, ldy, 0, W.rows, path, (cudaStream_t)stream);
}

int nd_cq_prepare(const float* x, int M, int in_feat, float* xh, int ld_out, void* stream) {
  return nd_status(nb::launch_cq_prepare(x, M, in_feat, xh, ld_out, (cudaStream_t)stream));
}

int nd_kv_quant(const float* x, int rows, int dim, int8_t* q, float* scales, void* stream) {
  if (!x || !q || !scales) return nd_status(cudaErrorInvalidValue);
  return nd_status(nb::launch_kv_quant(x, rows, dim, q, scales, (cudaStream_t)stream));
}

int nd_attend_step(const float* q, const void* k, const void* v, const float* ks, const float* vs,
                   int int8, int slots, const int* lo, const int* hi, int B, int heads, int kv_heads,
                   int qk, int vh, float* out, void* stream) {
  if (!q || !k || !v || !lo || !hi || !out || (int8 && (!ks || !vs))) return nd_status(cudaErrorInvalidValue);
  if (B <= 0) return 0;
  if (kv_heads <= 0 || heads % kv_heads || slots <= 0) return nd_status(cudaErrorInvalidValue);
  // Split partials live in stream-ordered scratch: allocated and released on
  // `stream`, so concurrent calls on different streams never share it.
  cudaStream_t st = (cudaStream_t)stream;
  const int ns = nb::attn_nsplit(B, kv_heads, slots);
  float* part = nullptr;
  cudaError_t e = scratch_alloc((void**)&part, nb::attn_part_floats(B, heads, kv_heads, vh, ns) * 4, st);
  if (e != cudaSuccess) return nd_status(e);
  e = nb::launch_attend_step(q, k, v, ks, vs, int8, slots, lo, hi, B, heads, kv_heads, qk, vh, ns, part, out, st);
  cudaError_t f = cudaFreeAsync(part, st);
  return nd_status(e != cudaSuccess ? e : f);
}

const char* nd_last_error(void) { return g_nd_err.c_str(); }

}  // extern "C"

namespace nb {
void nd_record_error(cudaError_t e, const char* msg) {
  g_nd_err = msg ? std::string(msg) : std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e);
}
}  // namespace nb

extern "C" {

}  // extern "C"
