// Needle-3 engine on one B200: container upload, sessions, batched forward.
//
// The container is parsed as crates/needle-infer/src/cact.rs:306-525 and
// 981-1100 read it, the canon is walked as v3.rs:236-332 walks it and shapes
// are validated as v3.rs:336-383 validates them. The whole container is then
// copied to the device once and CQ tensors are read in place.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cmath>
#include <cstring>

#include "engine.hpp"

namespace nb {

#define NB_TRY(expr)                                        \
  do {                                                      \
    cudaError_t _e = (expr);                                \
    if (_e != cudaSuccess) return _e;                       \
  } while (0)

static std::string cuda_msg(const char* what, cudaError_t e) {
  return std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
}

static uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }

static float half_to_float(uint16_t h) {  // exact binary16 -> f32 (math.rs:53-68)
  uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1F, mant = h & 0x3FF, u;
  if (exp == 0) {
    float v = (float)mant / (float)(1u << 24);
    return sign ? -v : v;
  }
  u = exp == 31 ? (sign | 0x7F800000u | (mant << 13)) : (sign | ((exp + 112) << 23) | (mant << 13));
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

bool HostConfig::is_global(size_t l) const {
  return std::find(global_layers.begin(), global_layers.end(), (int)l) != global_layers.end();
}
size_t HostConfig::span(size_t l) const { return (is_global(l) || window == 0) ? 0 : window; }
size_t HostConfig::kv_bytes_at(size_t seq_len, bool int8) const {
  size_t per_pos = int8 ? kvh * (qk + vh) + kvh * 8 : kvh * (qk + vh) * 4;
  size_t total = 0;
  for (size_t l = 0; l < layers; ++l) {
    size_t w = span(l);
    total += (w ? std::min(seq_len, w) : seq_len) * per_pos;
  }
  return total;
}

// ------------------------------------------------------------------ workspace
void Workspace::release() {
  void* ps[] = {lanes, u, bx, xh, proj, qpost, q8s, q8, ahi, alo, ainv, ehi, elo, einv, whi, wlo, cnt, keys, oh, projo, gates,
                fetched, ekv, evc, lm_in, pks, pvs, pk, pv, rows, tokens, next, last_rows, pre_part, pre_cnt};
  for (void* p : ps)
    if (p) cudaFree(p);
  if (logits) cudaFree(logits);
  if (part) cudaFree(part);
  if (lm_last) cudaFree(lm_last);
  for (void* h : {(void*)h_rows, (void*)h_tok, (void*)h_pick})
    if (h) cudaFreeHost(h);
  *this = Workspace();
}

bool Engine::ensure_ws(Workspace& w, size_t rows, std::string* err) {
  if (rows <= w.cap) return true;
  cudaStreamSynchronize(stream);
  size_t cap = std::max(rows, w.cap * 2);
  w.release();
  const size_t d = G.d, dpad = (d + 127) / 128 * 128, opad = (G.o_dim + 127) / 128 * 128;
  const size_t S = std::max(1, G.n_sites);
  const size_t kmax = std::max(dpad, opad);  // widest input of a projection
  const size_t wmax = std::max<size_t>(std::max<size_t>(G.logit_rows, G.proj_dim), 2 * d);  // most weight rows
  const size_t pre_rows = std::min<size_t>(cap, PRE_SPLIT_MAX_ROWS);  // rows of the split mHC pre-projection
  struct A {
    void** p;
    size_t bytes;
  } allocs[] = {
      {(void**)&w.lanes, cap * G.lanes * d * 4},   {(void**)&w.u, cap * d * 4},
      {(void**)&w.bx, cap * d * 4},                {(void**)&w.xh, cap * dpad * 4},
      {(void**)&w.proj, cap * G.proj_dim * 4},     {(void**)&w.qpost, cap * G.q_dim * 4},
      {(void**)&w.q8s, cap * G.heads * 4},         {(void**)&w.q8, cap * G.q_dim},
      {(void**)&w.ahi, cap * kmax * 2},            {(void**)&w.alo, cap * kmax * 2},
      {(void**)&w.ainv, cap * 32 * 4},                  {(void**)&w.cnt, cap * G.kvh * 4},
      {(void**)&w.ehi, cap * S * dpad * 2},        {(void**)&w.elo, cap * S * dpad * 2},
      {(void**)&w.einv, cap * S * (dpad / 128) * 4}, {(void**)&w.keys, cap * 8},
      {(void**)&w.whi, wmax * kmax * 2},           {(void**)&w.wlo, wmax * kmax * 2},
      {(void**)&w.oh, cap * opad * 4},
      {(void**)&w.projo, cap * d * 4},             {(void**)&w.gates, cap * 24 * 4},
      {(void**)&w.fetched, cap * S * d * 4},       {(void**)&w.ekv, cap * S * 2 * d * 4},
      {(void**)&w.evc, cap * S * d * 4},           {(void**)&w.lm_in, cap * dpad * 4},
      {(void**)&w.pk, cap * G.kvh * G.qk * 4},     {(void**)&w.pv, cap * G.kvh * G.vh * 4},
      {(void**)&w.pks, cap * G.kvh * 4},           {(void**)&w.pvs, cap * G.kvh * 4},
      {(void**)&w.rows, cap * sizeof(RowInfo)},    {(void**)&w.tokens, cap * 4},
      {(void**)&w.next, cap * 4},                  {(void**)&w.last_rows, cap * 4},
      {(void**)&w.pre_part, pre_rows * 32 * 32 * 4}, {(void**)&w.pre_cnt, pre_rows * 4},
  };
  for (auto& a : allocs) {
    cudaError_t e = cudaMalloc(a.p, std::max<size_t>(a.bytes, 256));
    if (e != cudaSuccess) {
      w.release();
      *err = cuda_msg("workspace allocation", e);
      return false;
    }
  }
  {
    cudaError_t e = cudaMallocHost((void**)&w.h_rows, cap * sizeof(RowInfo));
    if (e == cudaSuccess) e = cudaMallocHost((void**)&w.h_tok, cap * 4);
    if (e == cudaSuccess) e = cudaMallocHost((void**)&w.h_pick, cap * 4);
    if (e != cudaSuccess) {
      w.release();
      *err = cuda_msg("pinned staging allocation", e);
      return false;
    }
  }
  {
    cudaError_t e = cudaMemset(w.cnt, 0, cap * G.kvh * 4);  // attention split counters start at zero
    if (e == cudaSuccess) e = cudaMemset(w.pre_cnt, 0, pre_rows * 4);
    if (e != cudaSuccess) {
      w.release();
      *err = cuda_msg("workspace initialisation", e);
      return false;
    }
  }
  w.gs.hi = w.ahi;
  w.gs.lo = w.alo;
  w.gs.inv = w.ainv;
  w.gs.elems = cap * kmax;
  w.gs.rows = cap;
  w.gs.whi = w.whi;
  w.gs.wlo = w.wlo;
  w.gs.welems = wmax * kmax;
  w.gs.werr = d_wait_flag;
  w.cap = cap;
  epoch++;
  return true;
}

bool Engine::ensure_part(Workspace& w, size_t rows, int nsplit, std::string* err) {
  const size_t need = attn_part_floats((int)rows, G.heads, G.kvh, G.vh, nsplit);
  if (need <= w.part_cap) return true;
  cudaStreamSynchronize(stream);
  if (w.part) cudaFree(w.part);
  w.part = nullptr;
  const size_t cap = std::max(need, w.part_cap * 2);
  cudaError_t e = cudaMalloc(&w.part, cap * 4);
  if (e != cudaSuccess) {
    w.part_cap = 0;
    *err = cuda_msg("allocating attention partials", e);
    return false;
  }
  w.part_cap = cap;
  epoch++;
  return true;
}

// ------------------------------------------------------------------ loading
namespace {
// Widths of a CQ record: 2, 3 or 4 bits against the header codebook, or 5 for
// ternary (four signed 2-bit crumbs per byte, cq.rs:55-61).
constexpr int CQ_TERNARY = 5;

// Level table of a record's width, 16 entries (unused ones zero): the header
// codebook slice cb2 | cb3 | cb4, or the analytic ternary levels {-s, 0, +s}
// with s = centroid / sqrt(group) (cq.rs:197-203).
void cq_levels(int bits, int group, const float* codebook, float* lv) {
  std::fill(lv, lv + 16, 0.f);
  if (bits == CQ_TERNARY) {
    const float s = 1.2240064f / sqrtf((float)group);
    lv[0] = -s;
    lv[2] = s;
    return;
  }
  const float* src = bits == 2 ? codebook : bits == 3 ? codebook + 4 : codebook + 12;
  for (int k = 0; k < (1 << bits); ++k) lv[k] = src[k];
}

// Level indices of the first n codes of a packed row: an LSB-first bitstream
// of 2-, 3- or 4-bit codes, ternary crumbs 3, 0, 1 (2) meaning levels 0, 1, 2
// (1) (cq.rs:395-420, :908-925).
void cq_row_codes(const uint8_t* row, size_t n, int bits, uint8_t* idx) {
  const bool ter = bits == CQ_TERNARY;
  const int w = ter ? 2 : bits;
  const uint32_t mask = (1u << w) - 1;
  for (size_t k = 0; k < n; ++k) {
    const size_t bit = k * w, byte = bit / 8, shift = bit % 8;
    const uint32_t v = row[byte] | (shift + w > 8 ? (uint32_t)row[byte + 1] << 8 : 0u);
    const uint32_t code = (v >> shift) & mask;
    idx[k] = ter ? (uint8_t)(code == 3 ? 0 : code == 1 ? 2 : 1) : (uint8_t)code;
  }
}

struct Loader {
  const uint8_t* raw;
  size_t len;
  std::vector<Record> recs;
  float codebook[28];
  std::vector<float> arena;  // f32 parameters, each tensor 16-byte aligned
  std::string err;
  std::vector<void*>* owned = nullptr;  // device buffers of widened tensors, freed with the engine

  // FP16/FP32 record -> offset (floats) into the arena (cact.rs:494-524).
  long floats(size_t i, size_t expect = 0) {
    const Record& r = recs[i];
    size_t n;
    if (r.dtype == 1) {
      if (r.nbytes % 2) return fail("ragged fp16 blob", i);
      n = r.nbytes / 2;
    } else if (r.dtype == 2) {
      if (r.nbytes % 4) return fail("ragged fp32 blob", i);
      n = r.nbytes / 4;
    } else {
      return fail("expected an fp16/fp32 tensor", i);
    }
    if (expect && n != expect) return fail("unexpected element count", i);
    long off = (long)arena.size();
    const uint8_t* b = raw + r.offset;
    for (size_t k = 0; k < n; ++k) {
      if (r.dtype == 1)
        arena.push_back(half_to_float((uint16_t)(b[2 * k] | (b[2 * k + 1] << 8))));
      else {
        float f;
        std::memcpy(&f, b + 4 * k, 4);
        arena.push_back(f);
      }
    }
    while (arena.size() % 4) arena.push_back(0.f);
    return off;
  }
  long fail(const char* m, size_t i) {
    err = std::string(m) + " (tensor " + std::to_string(i) + ")";
    return -1;
  }
  // CQ record -> CqMat with one segment pointing into the device copy.
  bool cq(size_t i, const uint8_t* d_blob, CqMat* W) {
    const Record& r = recs[i];
    if (r.dtype != 3) return fail("expected a CQ tensor", i) >= 0;
    if (r.group != 128) return fail("GPU path supports CQ group 128 only", i) >= 0;
    if (r.bits < 2 || r.bits > 5) return fail("CQ width must be 2, 3, 4 bits or ternary", i) >= 0;
    size_t out = r.shape[0], in = r.shape[1];
    if (!out || !in) return fail("empty CQ shape", i) >= 0;
    const int w = r.bits == CQ_TERNARY ? 2 : (int)r.bits;
    size_t in_pad = (in + 127) / 128 * 128, groups = in_pad / 128, rb = in_pad * w / 8;
    if (r.nbytes < out * rb + out * groups * 2) return fail("short CQ blob", i) >= 0;
    if (r.offset % 16) return fail("CQ blob not 16-byte aligned", i) >= 0;
    std::memset(W, 0, sizeof(*W));
    W->seg[0].packed = d_blob + r.offset;
    W->seg[0].norms = reinterpret_cast<const __half*>(d_blob + r.offset + out * rb);
    W->seg[0].rows = (int)out;
    W->nseg = 1;
    W->rows = (int)out;
    W->in_feat = (int)in;
    W->in_pad = (int)in_pad;
    W->row_bytes = (int)rb;
    W->groups = (int)groups;
    W->group = 128;
    W->bits = (int)r.bits;
    cq_levels((int)r.bits, 128, codebook, W->levels);
    if (r.bits == 3 || r.bits == CQ_TERNARY) {
      // The kernels read byte-aligned 2- and 4-bit codes: 3-bit and ternary
      // tensors are widened once to 4-bit codes indexing the same levels, so
      // every product sees exactly the reference's dequantised values.
      if (!owned) return fail("internal: no owner for a widened tensor", i) >= 0;
      const size_t rb4 = in_pad / 2;
      std::vector<uint8_t> idx(in_pad), packed(out * rb4);
      for (size_t o = 0; o < out; ++o) {
        cq_row_codes(raw + r.offset + o * rb, in_pad, (int)r.bits, idx.data());
        for (size_t k = 0; k < in_pad; k += 2) packed[o * rb4 + k / 2] = (uint8_t)(idx[k] | (idx[k + 1] << 4));
      }
      void* d = nullptr;
      cudaError_t e = cudaMalloc(&d, packed.size());
      if (e == cudaSuccess) e = cudaMemcpy(d, packed.data(), packed.size(), cudaMemcpyHostToDevice);
      if (e != cudaSuccess) {
        if (d) cudaFree(d);
        return fail("widening a CQ tensor failed on the device", i) >= 0;
      }
      owned->push_back(d);
      W->seg[0].packed = static_cast<const uint8_t*>(d);
      W->row_bytes = (int)rb4;
      W->bits = 4;
    }
    return true;
  }
};

bool concat(CqMat* dst, const CqMat& add, std::string* err) {
  if (dst->nseg == 0) {
    *dst = add;
    return true;
  }
  if (dst->nseg >= MAX_SEG || dst->in_feat != add.in_feat || dst->bits != add.bits) {
    *err = "projections to fuse disagree in width or input";
    return false;
  }
  dst->seg[dst->nseg++] = add.seg[0];
  dst->rows += add.rows;
  return true;
}
}  // namespace

// The intelligence ladder (ladder.rs:28-74): block 0 and the last block, then
// repeatedly the midpoint of the widest gap between chosen blocks (the leftmost
// gap on ties); the rung of depth k keeps the first k blocks of that order, in
// stack order. Depths outside 2..layers are not rungs.
// One row of a CQ record as dense f32 weights, each 128-group rotated:
// H (norm_g * levels[codes]) with H the normalised Walsh-Hadamard matrix of
// the group (natural order, symmetric), so that dense . x == norm_g * (levels
// . H x), the CQ dot of cq.rs:666-672. Computed in double from the
// container's host bytes and rounded once.
static void cq_dense_row(const uint8_t* raw, const Record& r, const float* codebook, size_t row, float* out) {
  const int w = r.bits == CQ_TERNARY ? 2 : (int)r.bits;
  const size_t in_pad = (r.shape[1] + 127) / 128 * 128, groups = in_pad / 128, rb = in_pad * w / 8;
  const uint8_t* codes = raw + r.offset + row * rb;
  const uint8_t* nb = raw + r.offset + r.shape[0] * rb + row * groups * 2;
  float lv[16];
  cq_levels((int)r.bits, 128, codebook, lv);
  std::vector<uint8_t> idx(in_pad);
  cq_row_codes(codes, in_pad, (int)r.bits, idx.data());
  double v[128];
  for (size_t g = 0; g < groups; ++g) {
    __half_raw hr;
    hr.x = (unsigned short)(nb[2 * g] | (nb[2 * g + 1] << 8));
    const double norm = (double)__half2float(__half(hr));
    for (int j = 0; j < 128; ++j) v[j] = (double)lv[idx[g * 128 + j]] * norm;
    for (int h = 1; h < 128; h <<= 1)
      for (int i = 0; i < 128; i += 2 * h)
        for (int j = i; j < i + h; ++j) {
          const double a = v[j], b = v[j + h];
          v[j] = a + b;
          v[j + h] = a - b;
        }
    const double sc = 1.0 / std::sqrt(128.0);
    for (int j = 0; j < 128; ++j) out[g * 128 + j] = (float)(v[j] * sc);
  }
}

static bool ladder_kept(size_t layers, size_t depth, std::vector<int>* kept) {
  if (depth < 2 || depth > layers) return false;
  std::vector<int> sel = {0, (int)layers - 1};
  while (sel.size() < depth) {
    std::vector<int> s = sel;
    std::sort(s.begin(), s.end());
    int at = -1, widest = 1;
    for (size_t i = 0; i + 1 < s.size(); ++i)
      if (s[i + 1] - s[i] > widest) {
        widest = s[i + 1] - s[i];
        at = (int)i;
      }
    if (at < 0) break;
    sel.push_back((s[at] + s[at + 1]) / 2);
  }
  std::sort(sel.begin(), sel.end());
  *kept = sel;
  return sel.size() == depth;
}

Engine* Engine::load(const uint8_t* raw, size_t len, std::string* err, size_t depth) {
  if (!raw) {
    *err = "data was null";
    return nullptr;
  }
  if (len < 196) {
    *err = "container too short for a v3 header";
    return nullptr;
  }
  uint32_t w[49];
  for (int i = 0; i < 49; ++i) w[i] = rd32(raw + 4 * i);
  if (w[0] != 0x05E12A84u) {  // TAG_V3, cact.rs:29-31
    *err = "not a Needle 3 container (bad tag)";
    return nullptr;
  }
  if (w[2] != 28) {
    *err = "bad codebook length";
    return nullptr;
  }
  Loader L{raw, len, {}, {}, {}, ""};
  std::memcpy(L.codebook, raw + 196, 28 * 4);
  const size_t nt = w[1], dir = 196 + 28 * 4;
  if (len < dir + nt * 44) {
    *err = "container too short for its directory";
    return nullptr;
  }
  for (size_t i = 0; i < nt; ++i) {
    const uint8_t* b = raw + dir + i * 44;
    Record r;
    r.dtype = b[0];
    r.ndim = b[1];
    if (r.ndim > 4) {
      *err = "bad ndim in directory";
      return nullptr;
    }
    for (int k = 0; k < 4; ++k) r.shape[k] = rd32(b + 4 + 4 * k);
    r.offset = rd64(b + 20);
    r.nbytes = rd64(b + 28);
    r.group = rd32(b + 36);
    r.bits = rd32(b + 40);
    if (r.offset + r.nbytes > len || r.offset + r.nbytes < r.offset) {
      *err = "blob out of range (tensor " + std::to_string(i) + ")";
      return nullptr;
    }
    L.recs.push_back(r);
  }
  std::unique_ptr<Engine> E(new Engine());
  L.owned = &E->d_owned;
  // The tokenizer travels as the container's RAW record (cact.rs:1068-1075).
  // A malformed one fails the load; a container without one still serves the
  // token-level API.
  for (size_t i = 0; i < nt; ++i)
    if (L.recs[i].dtype == 4) {
      std::string terr;
      E->tok.reset(Tokenizer::from_blob(raw + L.recs[i].offset, L.recs[i].nbytes, &terr));
      if (!E->tok) {
        *err = "bad tokenizer record: " + terr;
        return nullptr;
      }
      break;
    }
  HostConfig& c = E->cfg;
  c.num_tensors = nt;
  c.kv_window = w[3];
  c.kv_bits = w[4];
  c.vocab = w[5];
  c.out_vocab = w[6];
  c.d = w[7];
  c.heads = w[8];
  c.kvh = w[9];
  c.layers = w[10];
  c.qk = w[11];
  c.vh = w[12];
  c.max_seq = w[13];
  c.hada_n = w[14];
  c.lanes = w[15];
  c.window = w[16];
  uint64_t gmask = (uint64_t)w[17] | ((uint64_t)w[18] << 32);
  for (size_t i = 0; i < c.layers && i < 64; ++i)
    if ((gmask >> i) & 1) c.global_layers.push_back((int)i);
  c.taps = w[19];
  c.e_slots = w[20];
  c.e_sub = w[21];
  c.e_tables = w[22];
  c.e_taps = w[23];
  c.e_dil = w[24];
  c.e_seed_heads = w[25];
  for (size_t k = 0; k < std::min<size_t>(w[26], 4); ++k) c.orders.push_back((int)w[27 + k]);
  for (size_t k = 0; k < std::min<size_t>(w[31], 16); ++k) c.sites.push_back((int)w[32 + k]);
  std::memcpy(&c.rope_theta, &w[48], 4);
  // config_from_geometry (v3.rs:25-70)
  if (c.orders.empty()) {
    *err = "container declares no engram orders";
    return nullptr;
  }
  if (c.e_tables % c.orders.size()) {
    *err = "engram tables not divisible by orders";
    return nullptr;
  }
  c.e_heads = c.e_tables / c.orders.size();
  if (c.e_heads == 0 || c.d / (c.orders.size() * c.e_heads) != c.e_sub) {
    *err = "engram sub_dim disagrees with d_model / (orders * heads)";
    return nullptr;
  }
  if (c.kvh == 0 || c.heads % c.kvh) {
    *err = "query heads do not divide into kv heads";
    return nullptr;
  }
  // Limits of this GPU path (checked, not assumed).
  if (c.d % 128 || c.e_sub != 128 || c.e_tables * 128 != c.d || (c.lanes != 1 && c.lanes != 2 && c.lanes != 4) ||
      c.heads / c.kvh > 8 || (c.qk != 16 && c.qk != 32 && c.qk != 48 && c.qk != 64) || c.vh > 64 ||
      c.vh % 2 || (c.heads / c.kvh) * c.vh > 512 || c.hada_n > 1024 || c.hada_n < c.d ||
      (c.hada_n & (c.hada_n - 1)) || c.sites.size() > 16 || c.max_seq == 0 ||
      c.heads * c.vh % 128 || c.out_vocab > c.vocab || c.taps > (size_t)MAX_QKV_TAPS) {
    *err = "geometry outside what this GPU path supports";
    return nullptr;
  }
  // Blocks this engine runs, by source block in the container: all of them, or
  // a ladder rung. Tensors are read at the container's depth and selected
  // below; nothing is re-quantised.
  std::vector<int> src;
  const bool rung = depth != 0 && depth != c.layers;
  if (rung) {
    if (!ladder_kept(c.layers, depth, &src)) {
      *err = "depth is outside the ladder";
      return nullptr;
    }
  } else {
    for (size_t l = 0; l < c.layers; ++l) src.push_back((int)l);
  }

  // Canon walk (v3.rs:236-332).
  size_t cur = 0;
  auto take = [&](size_t* idx) -> bool {
    if (cur >= nt) return false;
    *idx = cur++;
    return true;
  };
  auto shape2 = [&](size_t i, size_t a, size_t b) { return L.recs[i].shape[0] == a && L.recs[i].shape[1] == b; };
  const size_t qd = c.heads * c.qk, kd = c.kvh * c.qk, vd = c.kvh * c.vh, od = c.heads * c.vh, d = c.d;
  struct LayerIdx {
    size_t norm_in, q, k, v, qt, kt, vt, qn, kn, gate, out, post, agate, pre, mlp[13];
  };
  std::vector<LayerIdx> li(c.layers);
  size_t emb;
  bool ok = take(&emb);
  for (size_t l = 0; ok && l < c.layers; ++l) {
    LayerIdx& x = li[l];
    ok = take(&x.norm_in) && take(&x.q) && take(&x.k) && take(&x.v);
    if (ok && c.taps) ok = take(&x.qt) && take(&x.kt) && take(&x.vt);
    ok = ok && take(&x.qn) && take(&x.kn) && take(&x.gate) && take(&x.out) && take(&x.post) &&
         take(&x.agate) && take(&x.pre);
    for (int j = 0; ok && j < 13; ++j) ok = take(&x.mlp[j]);
  }
  size_t sc[6], phi[3], perm[2];
  for (int j = 0; ok && j < 6; ++j) ok = take(&sc[j]);
  for (int j = 0; ok && j < 3; ++j) ok = take(&phi[j]);
  for (int j = 0; ok && j < 2; ++j) ok = take(&perm[j]);
  std::vector<size_t> et(c.sites.size()), ek(c.sites.size()), ev(c.sites.size()), etap(c.sites.size());
  for (size_t s = 0; ok && s < c.sites.size(); ++s) ok = take(&et[s]) && take(&ek[s]) && take(&ev[s]) && take(&etap[s]);
  size_t fn = 0;
  ok = ok && take(&fn);
  if (!ok) {
    *err = "directory has fewer tensors than the canon needs";
    return nullptr;
  }
  // Probe heads (v3.rs:300-316, :486-560): the records between the final norm
  // and the RAW tokenizer are a manifest of head codes, then six tensors per
  // head (seven for the router) — probes, gain, query, row_bias, proj, bias.
  // Only the confidence head (code 2) is kept.
  size_t head_end = nt, conf_i = 0;
  long conf_gain = -1, conf_rb = -1, conf_bias = -1;
  for (size_t i = 0; i < nt; ++i)
    if (L.recs[i].dtype == 4) {
      head_end = i;
      break;
    }
  c.has_heads = false;
  if (cur < head_end) {
    const size_t mi = cur++;
    const long mo = L.floats(mi);
    if (mo < 0) {
      *err = L.err;
      return nullptr;
    }
    const size_t ncodes = (size_t)L.recs[mi].nbytes / (L.recs[mi].dtype == 1 ? 2 : 4);  // the arena pads
    for (size_t k = 0; k < ncodes; ++k) {
      const int code = (int)(uint8_t)L.arena[mo + k];
      const size_t need = code == 3 ? 7 : 6;
      if (cur + need > head_end) {
        *err = "head tensors ran out";
        return nullptr;
      }
      if (code == 2 && !c.has_heads) {
        conf_i = cur;
        conf_gain = L.floats(cur + 1);
        conf_rb = L.floats(cur + 3);
        conf_bias = L.floats(cur + 5);
        if (conf_gain < 0 || conf_rb < 0 || conf_bias < 0) {
          *err = L.err;
          return nullptr;
        }
        c.has_heads = true;
      }
      cur += need;
    }
  }
  // Shape validation (v3.rs:336-383).
  const char* bad = nullptr;
  if (!shape2(emb, c.vocab, d)) bad = "embedding";
  for (size_t l = 0; !bad && l < c.layers; ++l) {
    if (!shape2(li[l].q, qd, d)) bad = "q_proj";
    else if (!shape2(li[l].k, kd, d)) bad = "k_proj";
    else if (!shape2(li[l].v, vd, d)) bad = "v_proj";
    else if (!shape2(li[l].gate, od, d)) bad = "gate_proj";
    else if (!shape2(li[l].out, d, od)) bad = "out_proj";
  }
  for (size_t s = 0; !bad && s < c.sites.size(); ++s) {
    if (!shape2(et[s], c.e_tables * c.e_slots, c.e_sub)) bad = "engram tables";
    else if (!shape2(ek[s], d, d)) bad = "engram key_proj";
    else if (!shape2(ev[s], d, d)) bad = "engram value_proj";
  }
  if (!bad && !(shape2(phi[0], c.layers * c.lanes, c.lanes * d) && shape2(phi[1], c.layers * c.lanes, c.lanes * d) &&
                shape2(phi[2], c.layers * c.lanes * c.lanes, c.lanes * d)))
    bad = "mhc phi";
  if (bad) {
    *err = std::string("tensor shape does not match the geometry: ") + bad;
    return nullptr;
  }

  // Device upload of the container.
  cudaError_t e = cudaGetDevice(&E->device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&E->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&E->d_wait_flag, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(E->d_wait_flag, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaMallocHost(&E->h_wait_flag, sizeof(int));
  if (e == cudaSuccess) *E->h_wait_flag = 0;
  if (e == cudaSuccess) e = cudaMalloc(&E->d_blob, len);
  if (e == cudaSuccess) e = cudaMemcpy(E->d_blob, raw, len, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    *err = cuda_msg("uploading the container", e);
    return nullptr;
  }
  // f32 parameter arena.
  struct LOff {
    long norm_in, qt, kt, vt, qn, kn, post, pre, mlp[13];
    float agate;
  };
  std::vector<LOff> lo(c.layers);
  const size_t n = c.hada_n;
  size_t ba, bb;
  {
    size_t v = n - 1, bits = 0;
    while (v) {
      ++bits;
      v >>= 1;
    }
    ba = (size_t)1 << (bits / 2);  // hada_blocks, v3/kernels.rs:26-34
    bb = n / ba;
  }
  for (size_t l = 0; l < c.layers && L.err.empty(); ++l) {
    LOff& o = lo[l];
    o.norm_in = L.floats(li[l].norm_in, d);
    if (c.taps) {
      o.qt = L.floats(li[l].qt, c.taps * qd);
      o.kt = L.floats(li[l].kt, c.taps * kd);
      o.vt = L.floats(li[l].vt, c.taps * vd);
    }
    o.qn = L.floats(li[l].qn, c.qk);
    o.kn = L.floats(li[l].kn, c.qk);
    o.post = L.floats(li[l].post, d);
    long ag = L.floats(li[l].agate);
    o.agate = ag >= 0 ? L.arena[ag] : 0.f;
    o.pre = L.floats(li[l].pre, d);
    const size_t expect[13] = {n, n, n, n, n, ba * ba, bb * bb, ba * ba, bb * bb, ba * ba, bb * bb, 0, 0};
    for (int j = 0; j < 13; ++j) o.mlp[j] = L.floats(li[l].mlp[j], expect[j]);
  }
  size_t rank = c.layers ? L.recs[li[0].mlp[11]].shape[1] : 0;
  if (rank == 0 || rank > 8) L.err = L.err.empty() ? "HadamardMLP conditioning rank outside 1..8" : L.err;
  long a_pre = L.floats(sc[0], c.layers), a_post = L.floats(sc[1], c.layers), a_res = L.floats(sc[2], c.layers);
  long b_pre = L.floats(sc[3], c.layers * c.lanes), b_post = L.floats(sc[4], c.layers * c.lanes);
  long b_res = L.floats(sc[5], c.layers * c.lanes * c.lanes);
  std::vector<long> etaps(c.sites.size());
  for (size_t s = 0; s < c.sites.size(); ++s) etaps[s] = L.floats(etap[s], c.e_taps * d);
  long fnorm = L.floats(fn, d);
  long p1 = L.floats(perm[0], n), p2 = L.floats(perm[1], n);
  if (!L.err.empty()) {
    *err = L.err;
    return nullptr;
  }
  std::vector<uint32_t> perms(2 * n);
  for (size_t i = 0; i < n; ++i) {
    perms[i] = (uint32_t)L.arena[p1 + i];  // `x as u32`, v3.rs:474-478
    perms[n + i] = (uint32_t)L.arena[p2 + i];
    if (perms[i] >= n || perms[n + i] >= n) {
      *err = "hadamard permutation entry out of range";
      return nullptr;
    }
  }
  // RoPE table [2][max_seq][half] with the reference's f32 formula (model.rs:378-393).
  const size_t half = c.qk / 2;
  std::vector<float> rope(2 * c.max_seq * half);
  for (size_t i = 0; i < half; ++i) {
    float freq = 1.0f / powf(c.rope_theta, (float)(2 * i) / (float)c.qk);
    for (size_t p = 0; p < c.max_seq; ++p) {
      float ang = (float)p * freq;
      rope[p * half + i] = cosf(ang);
      rope[c.max_seq * half + p * half + i] = sinf(ang);
    }
  }
  e = cudaMalloc(&E->d_params, L.arena.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(E->d_params, L.arena.data(), L.arena.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&E->d_perm, perms.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(E->d_perm, perms.data(), perms.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&E->d_rope, rope.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(E->d_rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    *err = cuda_msg("uploading parameters", e);
    return nullptr;
  }
  // config_at_depth (v3.rs:620-640): kept blocks renumbered contiguously; the
  // global layers and Engram sites follow them, a site surviving exactly when
  // its block does. ssrc maps each kept site to its source site.
  std::vector<int> ssrc;
  if (rung) {
    auto pos = [&](int l) {
      auto it = std::find(src.begin(), src.end(), l);
      return it == src.end() ? -1 : (int)(it - src.begin());
    };
    std::vector<int> gl, st;
    for (int l : c.global_layers)
      if (pos(l) >= 0) gl.push_back(pos(l));
    for (size_t s = 0; s < c.sites.size(); ++s)
      if (pos(c.sites[s]) >= 0) {
        st.push_back(pos(c.sites[s]));
        ssrc.push_back((int)s);
      }
    c.layers = src.size();
    c.global_layers = gl;
    c.sites = st;
  } else {
    for (size_t s = 0; s < c.sites.size(); ++s) ssrc.push_back((int)s);
  }
  const float* P = E->d_params;
  auto pp = [&](long off) -> const float* { return off >= 0 ? P + off : nullptr; };
  // CQ tensors.
  bool okc = L.cq(emb, E->d_blob, &E->emb) && L.cq(phi[0], E->d_blob, &E->phi_pre) &&
             L.cq(phi[1], E->d_blob, &E->phi_post) && L.cq(phi[2], E->d_blob, &E->phi_res);
  E->qkvg.resize(c.layers);
  E->outp.resize(c.layers);
  for (size_t l = 0; okc && l < c.layers; ++l) {
    CqMat q, k, v, g;
    const LayerIdx& x = li[src[l]];
    okc = L.cq(x.q, E->d_blob, &q) && L.cq(x.k, E->d_blob, &k) && L.cq(x.v, E->d_blob, &v) &&
          L.cq(x.gate, E->d_blob, &g) && L.cq(x.out, E->d_blob, &E->outp[l]);
    std::memset(&E->qkvg[l], 0, sizeof(CqMat));
    okc = okc && concat(&E->qkvg[l], q, err) && concat(&E->qkvg[l], k, err) && concat(&E->qkvg[l], v, err) &&
          concat(&E->qkvg[l], g, err);
  }
  E->eng_kv.resize(c.sites.size());
  E->eng_tables.resize(c.sites.size());
  for (size_t s = 0; okc && s < c.sites.size(); ++s) {
    CqMat k, v;
    const int o = ssrc[s];
    okc = L.cq(et[o], E->d_blob, &E->eng_tables[s]) && L.cq(ek[o], E->d_blob, &k) && L.cq(ev[o], E->d_blob, &v);
    std::memset(&E->eng_kv[s], 0, sizeof(CqMat));
    okc = okc && concat(&E->eng_kv[s], k, err) && concat(&E->eng_kv[s], v, err);
  }
  if (!okc) {
    if (err->empty()) *err = L.err;
    return nullptr;
  }
  // The projections that run on the tensor cores (batches past 8 rows) read
  // f16 level tiles: expanded once here instead of on every call.
  {
    cudaError_t ec = umma_cache_levels(&E->emb, &E->d_owned, 0);
    for (size_t l = 0; ec == cudaSuccess && l < c.layers; ++l) {
      ec = umma_cache_levels(&E->qkvg[l], &E->d_owned, 0);
      if (ec == cudaSuccess) ec = umma_cache_levels(&E->outp[l], &E->d_owned, 0);
    }
    for (size_t s = 0; ec == cudaSuccess && s < c.sites.size(); ++s) ec = umma_cache_levels(&E->eng_kv[s], &E->d_owned, 0);
    if (ec == cudaSuccess) ec = cudaStreamSynchronize(0);
    if (ec != cudaSuccess) {
      *err = cuda_msg("expanding the projection levels", ec);
      return nullptr;
    }
  }
  if (!c.sites.empty()) {
    e = cudaMalloc(&E->d_tables, c.sites.size() * sizeof(CqMat));
    if (e == cudaSuccess)
      e = cudaMemcpy(E->d_tables, E->eng_tables.data(), c.sites.size() * sizeof(CqMat), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      *err = cuda_msg("uploading engram tables", e);
      return nullptr;
    }
  }
  E->lp.resize(c.layers);
  E->mp.resize(c.layers);
  E->site_of.assign(c.layers, -1);
  for (size_t s = 0; s < c.sites.size(); ++s)
    if ((size_t)c.sites[s] < c.layers) E->site_of[c.sites[s]] = (int)s;
  for (size_t l = 0; l < c.layers; ++l) {
    LayerParams& x = E->lp[l];
    const LOff& o = lo[src[l]];
    x.norm_in = pp(o.norm_in);
    x.q_taps = c.taps ? pp(o.qt) : nullptr;
    x.k_taps = c.taps ? pp(o.kt) : nullptr;
    x.v_taps = c.taps ? pp(o.vt) : nullptr;
    x.q_norm = pp(o.qn);
    x.k_norm = pp(o.kn);
    x.post_norm = pp(o.post);
    x.pre_hada = pp(o.pre);
    x.attn_gate = o.agate;
    x.d1 = pp(o.mlp[0]);
    x.d2 = pp(o.mlp[1]);
    x.b2 = pp(o.mlp[2]);
    x.d3 = pp(o.mlp[3]);
    x.d4 = pp(o.mlp[4]);
    x.w1a = pp(o.mlp[5]);
    x.w1b = pp(o.mlp[6]);
    x.w2a = pp(o.mlp[7]);
    x.w2b = pp(o.mlp[8]);
    x.w3a = pp(o.mlp[9]);
    x.w3b = pp(o.mlp[10]);
    x.cond_v = pp(o.mlp[11]);
    x.cond_u = pp(o.mlp[12]);
    x.window = (int)c.span(l);
    MhcParams& m = E->mp[l];
    const size_t sl = (size_t)src[l];
    m.a_pre = L.arena[a_pre + sl];
    m.a_post = L.arena[a_post + sl];
    m.a_res = L.arena[a_res + sl];
    m.b_pre = P + b_pre + sl * c.lanes;
    m.b_post = P + b_post + sl * c.lanes;
    m.b_res = P + b_res + sl * c.lanes * c.lanes;
    m.phi_layer = src[l];  // the lane matrices keep the container's rows
  }
  // Dense rotated mHC lane-matrix rows for the tiled layer-pre kernel, every
  // container layer (a rung addresses them through its source blocks).
  {
    const size_t nr = 2 * c.lanes + c.lanes * c.lanes, Wd = c.lanes * d, PL = (size_t)E->phi_pre.rows / c.lanes;
    std::vector<float> dense(PL * nr * Wd);
    for (size_t l = 0; l < PL; ++l)
      for (size_t o = 0; o < nr; ++o) {
        float* dst = dense.data() + (l * nr + o) * Wd;
        if (o < c.lanes) cq_dense_row(raw, L.recs[phi[0]], L.codebook, l * c.lanes + o, dst);
        else if (o < 2 * c.lanes) cq_dense_row(raw, L.recs[phi[1]], L.codebook, l * c.lanes + o - c.lanes, dst);
        else cq_dense_row(raw, L.recs[phi[2]], L.codebook, l * c.lanes * c.lanes + o - 2 * c.lanes, dst);
      }
    e = cudaMalloc(&E->d_phid, dense.size() * 4);
    if (e == cudaSuccess) e = cudaMemcpy(E->d_phid, dense.data(), dense.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      *err = cuda_msg("uploading the mHC lane matrices", e);
      return nullptr;
    }
    for (size_t l = 0; l < c.layers; ++l) E->mp[l].phi_dense = E->d_phid + (size_t)src[l] * nr * Wd;
  }
  for (size_t s = 0; s < c.sites.size(); ++s) E->eng_taps.push_back(P + etaps[ssrc[s]]);
  // The confidence head, dense, with the cells of this engine's blocks
  // (confidence_head_at_depth, v3.rs:745-787: cell 0 and 1 + each kept block).
  if (c.has_heads) {
    CqMat pm, qm, jm;
    if (!(L.cq(conf_i, E->d_blob, &pm) && L.cq(conf_i + 2, E->d_blob, &qm) && L.cq(conf_i + 4, E->d_blob, &jm))) {
      *err = L.err;
      return nullptr;
    }
    const size_t PL1 = (size_t)E->phi_pre.rows / c.lanes + 1, prow = (size_t)pm.rows;
    const size_t ngain = (size_t)L.recs[conf_i + 1].nbytes / (L.recs[conf_i + 1].dtype == 1 ? 2 : 4);
    if (prow % PL1 || ngain != prow || pm.in_feat != (int)d || qm.in_feat != (int)d ||
        jm.in_feat != qm.rows * (int)d) {
      *err = "probe head shapes disagree with num_layers + 1 cells";
      return nullptr;
    }
    const size_t K = prow / PL1, Q = qm.rows, OD = jm.rows, mm = PL1 * K;
    auto count = [&](size_t i) { return (size_t)L.recs[i].nbytes / (L.recs[i].dtype == 1 ? 2 : 4); };
    if (count(conf_i + 3) != Q * mm || count(conf_i + 5) < OD) {
      *err = "probe head row_bias or bias disagrees with its shapes";
      return nullptr;
    }
    std::vector<size_t> cl = {0};
    for (int sl : src) cl.push_back((size_t)sl + 1);
    const size_t cells = cl.size(), m = cells * K;
    std::vector<float> probes(m * d), gain(m), query(Q * d), rb(Q * m), proj(OD * Q * d), bias(OD);
    for (size_t i = 0; i < cells; ++i)
      for (size_t k = 0; k < K; ++k) {
        cq_dense_row(raw, L.recs[conf_i], L.codebook, cl[i] * K + k, probes.data() + (i * K + k) * d);
        gain[i * K + k] = L.arena[conf_gain + cl[i] * K + k];
        for (size_t qi = 0; qi < Q; ++qi) rb[qi * m + i * K + k] = L.arena[conf_rb + qi * mm + cl[i] * K + k];
      }
    for (size_t qi = 0; qi < Q; ++qi) cq_dense_row(raw, L.recs[conf_i + 2], L.codebook, qi, query.data() + qi * d);
    for (size_t o = 0; o < OD; ++o) {
      cq_dense_row(raw, L.recs[conf_i + 4], L.codebook, o, proj.data() + o * Q * d);
      bias[o] = L.arena[conf_bias + o];
    }
    std::vector<float> all;
    for (const auto* v : {&probes, &gain, &query, &rb, &proj, &bias}) all.insert(all.end(), v->begin(), v->end());
    e = cudaMalloc(&E->d_conf, all.size() * 4);
    if (e == cudaSuccess) e = cudaMemcpy(E->d_conf, all.data(), all.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      *err = cuda_msg("uploading the confidence head", e);
      return nullptr;
    }
    ProbeHeadDev& h = E->conf;
    h.probes = E->d_conf;
    h.gain = h.probes + probes.size();
    h.query = h.gain + gain.size();
    h.row_bias = h.query + query.size();
    h.proj = h.row_bias + rb.size();
    h.bias = h.proj + proj.size();
    h.cells = (int)cells;
    h.probes_per_cell = (int)K;
    h.queries = (int)Q;
    h.out_dim = (int)OD;
  }
  E->final_norm = P + fnorm;
  // HadamardMLP weight fragments for the tensor-core block tail.
  for (size_t l = 0; l < c.layers; ++l) E->lp[l].hfrag = nullptr;
  if (hada_tc_supported((int)ba, (int)bb)) {
    const size_t fw = hada_frag_words((int)ba);
    std::vector<uint32_t> frags(fw * c.layers);
    for (size_t l = 0; l < c.layers; ++l) {
      const LOff& o = lo[src[l]];
      // Stage order per Kronecker pair: B^T (w*b) then A^T (w*a).
      const float* mats[6] = {&L.arena[o.mlp[6]], &L.arena[o.mlp[5]], &L.arena[o.mlp[8]],
                              &L.arena[o.mlp[7]], &L.arena[o.mlp[10]], &L.arena[o.mlp[9]]};
      hada_frags(mats, (int)ba, frags.data() + l * fw, E->lp[l].hinv);
    }
    e = cudaMalloc(&E->d_hfrag, frags.size() * 4);
    if (e == cudaSuccess) e = cudaMemcpy(E->d_hfrag, frags.data(), frags.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      *err = cuda_msg("uploading HadamardMLP fragments", e);
      return nullptr;
    }
    for (size_t l = 0; l < c.layers; ++l) E->lp[l].hfrag = E->d_hfrag + l * fw;
  }

  Geo& g = E->G;
  g.d = (int)d;
  g.heads = (int)c.heads;
  g.kvh = (int)c.kvh;
  g.qk = (int)c.qk;
  g.vh = (int)c.vh;
  g.layers = (int)c.layers;
  g.lanes = (int)c.lanes;
  g.hada_n = (int)n;
  g.ba = (int)ba;
  g.bb = (int)bb;
  g.taps = (int)c.taps;
  g.window = (int)c.window;
  g.max_seq = (int)c.max_seq;
  g.vocab = (int)c.vocab;
  g.logit_rows = (int)c.logit_rows();
  g.q_dim = (int)qd;
  g.k_dim = (int)kd;
  g.v_dim = (int)vd;
  g.o_dim = (int)od;
  g.qkv_dim = (int)(qd + kd + vd);
  g.proj_dim = (int)(qd + kd + vd + od);
  g.e_tables = (int)c.e_tables;
  g.e_heads = (int)c.e_heads;
  g.e_slots = (int)c.e_slots;
  g.e_sub = (int)c.e_sub;
  g.e_taps = (int)c.e_taps;
  g.e_dil = (int)c.e_dil;
  int mo = 1;
  for (int o : c.orders) mo = std::max(mo, o);
  g.e_maxorder = mo;
  g.e_reach = (int)((c.e_taps > 0 ? c.e_taps - 1 : 0) * c.e_dil);
  g.e_stride = (int)(c.e_seed_heads == 0 ? c.e_heads : c.e_seed_heads);
  g.n_orders = (int)c.orders.size();
  g.n_sites = (int)c.sites.size();
  for (int k = 0; k < 4; ++k) g.orders[k] = k < (int)c.orders.size() ? c.orders[k] : 0;
  g.cond_rank = (int)rank;
  g.embed_scale = sqrtf((float)d);  // model.rs:131
  if (mo > 4) {
    *err = "engram order above 4 exceeds the token ring";
    return nullptr;
  }
  return E.release();
}

Engine::~Engine() {
  if (stream) cudaStreamSynchronize(stream);
  if (dec_graph) cudaGraphExecDestroy(dec_graph);
  ws.release();
  if (d_blob) cudaFree(d_blob);
  if (d_params) cudaFree(d_params);
  if (d_perm) cudaFree(d_perm);
  if (d_rope) cudaFree(d_rope);
  if (d_hfrag) cudaFree(d_hfrag);
  if (d_phid) cudaFree(d_phid);
  if (d_conf) cudaFree(d_conf);
  for (void* p : d_owned) cudaFree(p);
  if (d_tables) cudaFree(d_tables);
  if (h_wait_flag) cudaFreeHost(h_wait_flag);
  if (d_wait_flag) cudaFree(d_wait_flag);
  if (stream) cudaStreamDestroy(stream);
}

cudaError_t Engine::queue_wait_flag(cudaStream_t st) {
  return cudaMemcpyAsync(h_wait_flag, d_wait_flag, sizeof(int), cudaMemcpyDeviceToHost, st);
}

cudaError_t Engine::wait_status(cudaStream_t st) {
  if (!*h_wait_flag) return cudaSuccess;
  *h_wait_flag = 0;
  cudaError_t e = cudaMemsetAsync(d_wait_flag, 0, sizeof(int), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e == cudaSuccess ? cudaErrorTimeout : e;
}

cudaError_t Engine::take_wait_flag() {
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, d_wait_flag, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess || !v) return e;
  e = cudaMemset(d_wait_flag, 0, sizeof(int));
  return e == cudaSuccess ? cudaErrorTimeout : e;
}

// ------------------------------------------------------------------ sessions
static size_t kv_elem_bytes(const Session* s) { return s->int8 ? 1 : 4; }

// Bytes of one layer's KV ring at `slots` (each array 256-byte aligned).
static size_t layer_bytes(const Geo& g, bool int8, int slots) {
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t eb = int8 ? 1 : 4;
  size_t b = al((size_t)g.kvh * slots * g.qk * eb) + al((size_t)g.kvh * slots * g.vh * eb);
  if (int8) b += 2 * al((size_t)g.kvh * slots * 4);
  return b;
}

// Point L's arrays into `base` (layer_bytes(...) bytes, zeroed by the caller).
static void carve_layer(const Geo& g, bool int8, int slots, int cap, uint8_t* base, LayerKV* L) {
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t eb = int8 ? 1 : 4;
  std::memset(L, 0, sizeof(*L));
  L->slots = slots;
  L->cap = cap;
  L->k = base;
  base += al((size_t)g.kvh * slots * g.qk * eb);
  L->v = base;
  base += al((size_t)g.kvh * slots * g.vh * eb);
  if (int8) {
    L->ks = (float*)base;
    base += al((size_t)g.kvh * slots * 4);
    L->vs = (float*)base;
  }
}

Session::~Session() {
  if (eng) cudaStreamSynchronize(eng->stream);
  for (size_t l = 0; l < layers.size(); ++l)
    if (l < owned.size() && owned[l] && layers[l].k) cudaFree(layers[l].k);
  if (d_arena) cudaFree(d_arena);
}

size_t Session::bytes() const {  // as V3Cache::bytes counts (cache.rs:255-268)
  size_t t = state_bytes;
  const Geo& g = eng->G;
  for (const LayerKV& l : layers)
    t += (size_t)g.kvh * l.slots * (g.qk + g.vh) * kv_elem_bytes(this) + (int8 ? (size_t)g.kvh * l.slots * 8 : 0);
  return t;
}

Session* Engine::new_session(size_t hint, bool int8, std::string* err) {
  std::lock_guard<std::mutex> lk(mu);
  cudaSetDevice(device);
  std::unique_ptr<Session> s(new Session());
  s->eng = this;
  s->int8 = int8;
  hint = std::min(std::max<size_t>(hint, 1), cfg.max_seq);  // cache.rs:178
  s->hint = hint;
  s->layers.resize(cfg.layers);
  s->owned.assign(cfg.layers, 0);
  // One device arena per session: every layer's ring, the conv/Engram tails and
  // token ring, the per-layer descriptor array and the session descriptor.
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  std::vector<int> slots(cfg.layers), caps(cfg.layers);
  size_t total = 0;
  for (size_t l = 0; l < cfg.layers; ++l) {
    size_t w = cfg.span(l);
    caps[l] = (int)(w ? std::min(w, cfg.max_seq) : cfg.max_seq);
    slots[l] = (int)std::min<size_t>(hint, (size_t)caps[l]);
    total += layer_bytes(G, int8, slots[l]);
  }
  const size_t tl = G.taps > 0 ? G.taps - 1 : 0;
  // The Engram tails start at the Q/K/V tail count rounded up to four floats
  // (16-byte aligned for float4 access); the byte count (V3Cache::bytes)
  // excludes that padding.
  const size_t qkv_n = cfg.layers * tl * G.qkv_dim, eng_tail = (size_t)G.n_sites * G.e_reach * G.d;
  const size_t qkv_tail = (qkv_n + 3) / 4 * 4;
  s->state_bytes = (qkv_n + eng_tail) * 4 + 4 * 4;
  const size_t state_off = total;
  total += al((qkv_tail + eng_tail) * 4 + 4 * 4);
  const size_t layers_off = total;
  total += al(cfg.layers * sizeof(LayerKV));
  const size_t desc_off = total;
  total += al(sizeof(SessDesc));
  cudaError_t e = cudaMalloc(&s->d_arena, total);
  if (e == cudaSuccess) e = cudaMemsetAsync(s->d_arena, 0, total, stream);
  if (e != cudaSuccess) {
    *err = cuda_msg("allocating the session", e);
    return nullptr;
  }
  uint8_t* base = (uint8_t*)s->d_arena;
  size_t off = 0;
  for (size_t l = 0; l < cfg.layers; ++l) {
    carve_layer(G, int8, slots[l], caps[l], base + off, &s->layers[l]);
    off += layer_bytes(G, int8, slots[l]);
  }
  s->d_state = base + state_off;
  s->d_layers = (LayerKV*)(base + layers_off);
  s->d_desc = (SessDesc*)(base + desc_off);
  SessDesc h{};
  h.pos = 0;
  h.int8 = int8 ? 1 : 0;
  h.layers = s->d_layers;
  h.qkv_tail = (float*)s->d_state;
  h.eng_tail = (float*)s->d_state + qkv_tail;
  h.toks = (uint32_t*)((float*)s->d_state + qkv_tail + eng_tail);
  e = cudaMemcpyAsync(s->d_layers, s->layers.data(), cfg.layers * sizeof(LayerKV), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(s->d_desc, &h, sizeof(h), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) {
    *err = cuda_msg("writing the session descriptor", e);
    return nullptr;
  }
  return s.release();
}

// Grow every layer ring so `pos` is addressable, doubling up to the layer's
// cap exactly as V3Cache::ensure does (cache.rs:291-309); a local layer at its
// window wraps instead. Old contents are kept: while a ring is below its cap
// the slot of position p is p itself.
bool Engine::ensure_slots(Session* s, size_t pos, std::string* err) {
  if (pos < s->grow_at) return true;
  bool changed = false;
  const size_t eb = kv_elem_bytes(s);
  for (size_t l = 0; l < cfg.layers; ++l) {
    LayerKV& L = s->layers[l];
    if ((int)pos < L.slots || L.slots >= L.cap) continue;
    int want = L.slots;
    while ((int)pos >= want && want < L.cap) want = std::min(std::max(want * 2, want + 1), L.cap);
    LayerKV N;
    void* mem = nullptr;
    const size_t nb_ = layer_bytes(G, s->int8, want);
    cudaError_t e = cudaMalloc(&mem, nb_);
    if (e == cudaSuccess) e = cudaMemsetAsync(mem, 0, nb_, stream);
    if (e == cudaSuccess) carve_layer(G, s->int8, want, L.cap, (uint8_t*)mem, &N);
    auto copy2d = [&](void* dst, const void* src, size_t row) {
      return cudaMemcpy2DAsync(dst, want * row, src, L.slots * row, L.slots * row, G.kvh,
                               cudaMemcpyDeviceToDevice, stream);
    };
    if (e == cudaSuccess) e = copy2d(N.k, L.k, G.qk * eb);
    if (e == cudaSuccess) e = copy2d(N.v, L.v, G.vh * eb);
    if (e == cudaSuccess && s->int8) e = copy2d(N.ks, L.ks, 4);
    if (e == cudaSuccess && s->int8) e = copy2d(N.vs, L.vs, 4);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
      if (mem) cudaFree(mem);
      *err = cuda_msg("growing the KV ring", e);
      return false;
    }
    if (s->owned[l]) cudaFree(L.k);  // a ring grown earlier owns its allocation
    L = N;
    s->owned[l] = 1;
    changed = true;
  }
  if (changed) {
    cudaError_t e = cudaMemcpyAsync(s->d_layers, s->layers.data(), cfg.layers * sizeof(LayerKV),
                                    cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
      *err = cuda_msg("updating the session descriptor", e);
      return false;
    }
    epoch++;
  }
  size_t next = SIZE_MAX;
  for (size_t l = 0; l < cfg.layers; ++l)
    if (s->layers[l].slots < s->layers[l].cap) next = std::min(next, (size_t)s->layers[l].slots);
  s->grow_at = next;
  return true;
}

bool Engine::read_kv(Session* s, size_t li, void* k, void* v, float* ks, float* vs, std::string* err) {
  std::lock_guard<std::mutex> lk(mu);
  cudaSetDevice(device);
  if (li >= s->layers.size()) {
    *err = "layer out of range";
    return false;
  }
  const LayerKV& L = s->layers[li];
  const size_t eb = kv_elem_bytes(s), S = (size_t)L.slots, H = (size_t)G.kvh;
  std::vector<uint8_t> hk(H * S * G.qk * eb), hv(H * S * G.vh * eb);
  std::vector<float> hks(s->int8 ? H * S : 0), hvs(s->int8 ? H * S : 0);
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess) e = cudaMemcpy(hk.data(), L.k, hk.size(), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(hv.data(), L.v, hv.size(), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && s->int8) e = cudaMemcpy(hks.data(), L.ks, hks.size() * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && s->int8) e = cudaMemcpy(hvs.data(), L.vs, hvs.size() * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    *err = cuda_msg("reading the KV ring", e);
    return false;
  }
  // Head-major [kv_heads][slots][dim] on the device -> [slots][kv_heads][dim].
  // Slots no position has reached yet (slot t >= pos while the ring is not
  // full) hold zero codes and report the reference's initial scale of 1
  // (cache.rs:214-215, :305-306); the device arena leaves them 0, which
  // attention never reads.
  const size_t kr = G.qk * eb, vr = G.vh * eb;
  // int8 value codes sit offset-binary in the ring (code ^ 0x80): flip back.
  if (s->int8)
    for (uint8_t& c : hv) c ^= 0x80;
  for (size_t h = 0; h < H; ++h)
    for (size_t t = 0; t < S; ++t) {
      const bool written = t < s->pos;
      if (k) std::memcpy((uint8_t*)k + (t * H + h) * kr, hk.data() + (h * S + t) * kr, kr);
      if (v) {
        uint8_t* dv = (uint8_t*)v + (t * H + h) * vr;
        if (s->int8 && !written)
          std::memset(dv, 0, vr);  // never written: the reference's zero codes
        else
          std::memcpy(dv, hv.data() + (h * S + t) * vr, vr);
      }
      if (ks && s->int8) ks[t * H + h] = written ? hks[h * S + t] : 1.0f;
      if (vs && s->int8) vs[t * H + h] = written ? hvs[h * S + t] : 1.0f;
    }
  return true;
}

// ------------------------------------------------------------------ forward
cudaError_t Prof::mark(int kind, cudaStream_t st, int nlaunch) {
  launches += nlaunch;
  if (used == marks.size()) {
    cudaEvent_t ev;
    NB_TRY(cudaEventCreate(&ev));
    marks.push_back({kind, ev});
  }
  marks[used].first = kind;
  NB_TRY(cudaEventRecord(marks[used].second, st));
  ++used;
  return cudaSuccess;
}

#define NB_MARK(kind, n) \
  if (prof) NB_TRY(prof->mark(kind, st, n))

cudaError_t Engine::forward(Workspace& w, const RowBatch& rb, cudaStream_t st, bool int8, int nsplit, Prof* prof,
                            bool split_head) {
  const int M = rb.M, d = G.d, S = G.n_sites;
  const int dpad = (d + 127) / 128 * 128, opad = (G.o_dim + 127) / 128 * 128;
  if (S > 0) {
    // On the tensor cores the gather writes every site's projection operands
    // in the split form, so each projection is a single launch.
    bool pre = d == dpad;
    for (int s = 0; s < S; ++s) pre = pre && cq_umma_takes(eng_kv[s], M, &w.gs);
    NB_TRY(launch_engram_gather(G, d_tables, rb, w.fetched, st, pre ? SplitOut{w.ehi, w.elo, w.einv} : SplitOut{}));
    for (int s = 0; s < S; ++s) {
      GemmScratch gs = w.gs;
      if (pre) {
        gs.hi = w.ehi + (size_t)s * M * d;
        gs.lo = w.elo + (size_t)s * M * d;
        gs.inv = w.einv + (size_t)s * M * (d / 128);
      }
      NB_TRY(cq_project(eng_kv[s], w.fetched + (size_t)s * d, S * d, M, w.ekv + (size_t)s * 2 * d, S * 2 * d, 0,
                        2 * d, st, 0, &gs, pre));
    }
    NB_TRY(launch_engram_conv(G, eng_taps.data(), rb, w.ekv, w.evc, st));
    NB_MARK(PK_ENGRAM, S * cq_launches(eng_kv[0], M, &w.gs, 0, pre) + 2);
  }
  NB_TRY(launch_embed(G, emb, rb, w.lanes, st));
  if (w.cells) NB_TRY(launch_lane_mean(w.lanes, M, G.lanes, d, true, w.cells, st));
  NB_MARK(PK_EMBED, 1);
  // Inputs of tensor-core projections are written by their producers in the
  // split form, straight into the projection scratch.
  const SplitOut to_gs{w.gs.hi, w.gs.lo, w.gs.inv};
  for (int l = 0; l < G.layers; ++l) {
    const SplitOut sq = cq_umma_takes(qkvg[l], M, &w.gs) ? to_gs : SplitOut{};
    NB_TRY(launch_layer_pre(G, l, rb, w.lanes, phi_pre, phi_post, phi_res, mp[l], lp[l].norm_in,
                            site_of[l], w.ekv, w.evc, w.u, w.bx, w.xh, w.gates, st, w.pre_part, w.pre_cnt, sq));
    NB_MARK(PK_LAYER_PRE, 1);
    NB_TRY(cq_project(qkvg[l], w.xh, dpad, M, w.proj, G.proj_dim, 0, G.proj_dim, st, 0, &w.gs, sq.hi != nullptr));
    NB_MARK(PK_QKVG, cq_launches(qkvg[l], M, &w.gs, 0, sq.hi != nullptr));
    NB_TRY(launch_qkv_post(G, l, rb, lp[l], d_rope, w.proj, w.qpost, w.pk, w.pv, w.pks, w.pvs,
                           int8 ? w.q8 : nullptr, int8 ? w.q8s : nullptr, st));
    NB_MARK(PK_QKV_POST, 1);
    const bool fused = attn_fuses_finish(G, int8 ? 1 : 0) && nsplit <= 64;
    const SplitOut so = cq_umma_takes(outp[l], M, &w.gs) ? to_gs : SplitOut{};
    NB_TRY(launch_attention(G, l, rb, lp[l], nsplit, w.qpost, w.q8, w.q8s, w.pk, w.pv, w.pks, w.pvs,
                            w.part, st, int8 ? 1 : 0, w.proj, w.oh, w.cnt, d_wait_flag, so));
    NB_MARK(PK_ATTN, 1);
    if (!fused) NB_TRY(launch_attn_finish(G, rb, nsplit, w.part, w.proj, w.oh, st, so));
    NB_MARK(PK_ATTN_FINISH, fused ? 0 : 1);
    NB_TRY(cq_project(outp[l], w.oh, opad, M, w.projo, d, 0, d, st, 0, &w.gs, so.hi != nullptr));
    NB_MARK(PK_OUT_PROJ, cq_launches(outp[l], M, &w.gs, 0, so.hi != nullptr));
    NB_TRY(launch_layer_post(G, l, rb, lp[l], d_perm, d_perm + G.hada_n, w.projo, w.u, w.bx,
                             w.gates, w.lanes, st));
    if (w.cells) NB_TRY(launch_lane_mean(w.lanes, M, G.lanes, d, false, w.cells + (size_t)(l + 1) * M * d, st));
    NB_MARK(PK_LAYER_POST, 1);
  }
  const SplitOut sh = split_head && cq_umma_takes(emb, M, &w.gs) ? to_gs : SplitOut{};
  NB_TRY(launch_final(G, rb, w.lanes, final_norm, w.lm_in, st, sh, sh.hi ? w.keys : nullptr));
  w.head_presplit = sh.hi != nullptr;
  NB_MARK(PK_FINAL, 1);
  return cudaSuccess;
}

// Tied head over logit_rows (model.rs:358-374, :942-978) and the greedy pick.
cudaError_t Engine::head(Workspace& w, const float* lm_in, int ldx, int M, float* logits, uint32_t* picks,
                         cudaStream_t st, Prof* prof, bool need_logits) {
  // The last forward's final kernel may have written this input split (lm_in
  // itself then holds nothing).
  const bool presplit = lm_in == w.lm_in && w.head_presplit;
  if (picks && !need_logits && presplit) {
    // The split input means the tensor-core path, and the final kernel zeroed
    // the rows' keys: the projection keeps each row's first maximum only.
    GemmScratch gs = w.gs;
    gs.amax = w.keys;
    NB_TRY(cq_project(emb, lm_in, ldx, M, logits, G.logit_rows, 0, G.logit_rows, st, 0, &gs, true));
    NB_MARK(PK_HEAD, cq_launches(emb, M, &w.gs, 0, true));
    NB_TRY(launch_argmax_keys(w.keys, M, picks, st));
    NB_MARK(PK_BOOK, 1);
    return cudaSuccess;
  }
  NB_TRY(cq_project(emb, lm_in, ldx, M, logits, G.logit_rows, 0, G.logit_rows, st, 0, &w.gs, presplit));
  NB_MARK(PK_HEAD, cq_launches(emb, M, &w.gs, 0, presplit));
  if (picks) NB_TRY(launch_argmax(logits, M, G.logit_rows, G.logit_rows, picks, st));
  NB_MARK(PK_BOOK, picks ? 1 : 0);
  return cudaSuccess;
}

static bool ensure_logits(Engine* E, Workspace& w, size_t rows, std::string* err) {
  if (rows <= w.last_cap) return true;
  if (w.logits) cudaFree(w.logits);
  if (w.lm_last) cudaFree(w.lm_last);
  w.logits = nullptr;
  w.lm_last = nullptr;
  size_t cap = std::max(rows, w.last_cap * 2);
  cudaError_t e = cudaMalloc(&w.logits, cap * E->G.logit_rows * 4);
  if (e == cudaSuccess) e = cudaMalloc(&w.lm_last, cap * ((E->G.d + 127) / 128 * 128) * 4);
  if (e != cudaSuccess) {
    *err = cuda_msg("allocating logits", e);
    w.last_cap = 0;
    return false;
  }
  w.last_cap = cap;
  E->epoch++;
  return true;
}

static constexpr size_t MAX_PREFILL_ROWS = 16384;

bool Engine::prefill(Session* const* ss, const uint32_t* const* ids, const size_t* lens, size_t n,
                     float* logits, uint32_t* picks, std::string* err, float* d_cells) {
  std::lock_guard<std::mutex> lk(mu);
  cudaSetDevice(device);
  if (n == 0) return true;
  if (d_cells && n != 1) {
    *err = "cells are captured for one prompt at a time";
    return false;
  }
  for (size_t i = 0; i < n; ++i) {
    if (!ss[i] || ss[i]->eng != this) {
      *err = "session does not belong to this handle";
      return false;
    }
    if (ss[i]->pos != 0) {
      *err = "prefill needs a fresh session (position 0)";
      return false;
    }
    if (lens[i] == 0 || lens[i] > cfg.max_seq) {
      *err = "prompt length must be in 1..max_seq_len";
      return false;
    }
    if (ss[i]->int8 != ss[0]->int8) {
      *err = "a batch must share one KV precision";
      return false;
    }
  }
  const int dpad = (G.d + 127) / 128 * 128;
  size_t i0 = 0;
  while (i0 < n) {
    // Group whole prompts so one forward holds at most MAX_PREFILL_ROWS rows.
    size_t i1 = i0, rows = 0;
    while (i1 < n && (i1 == i0 || rows + lens[i1] <= MAX_PREFILL_ROWS)) rows += lens[i1++];
    for (size_t i = i0; i < i1; ++i)
      if (!ensure_slots(ss[i], lens[i] - 1, err)) return false;
    size_t maxlen = 0;
    for (size_t i = i0; i < i1; ++i) maxlen = std::max(maxlen, lens[i]);
    const int ns = attn_nsplit((int)rows, G.kvh, (int)maxlen);
    if (!ensure_ws(ws, rows, err) || !ensure_logits(this, ws, i1 - i0, err) || !ensure_part(ws, rows, ns, err)) return false;
    std::vector<RowInfo> ri(rows);
    std::vector<uint32_t> tok(rows);
    std::vector<int> last(i1 - i0);
    size_t r = 0;
    for (size_t i = i0; i < i1; ++i) {
      for (size_t p = 0; p < lens[i]; ++p, ++r) {
        ri[r] = RowInfo{ss[i]->d_desc, (int)p, (int)(r - p), (int)lens[i], 0};
        tok[r] = ids[i][p];
      }
      last[i - i0] = (int)(r - 1);
    }
    cudaError_t e = cudaMemcpyAsync(ws.rows, ri.data(), rows * sizeof(RowInfo), cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ws.tokens, tok.data(), rows * 4, cudaMemcpyHostToDevice, stream);
    RowBatch rb{ws.rows, ws.tokens, (int)rows, MODE_PREFILL};
    ws.cells = d_cells;
    if (e == cudaSuccess) e = forward(ws, rb, stream, ss[i0]->int8, ns);
    ws.cells = nullptr;
    if (e == cudaSuccess) e = launch_step_end(rb, stream);
    for (size_t i = 0; e == cudaSuccess && i < i1 - i0; ++i)
      e = cudaMemcpyAsync(ws.lm_last + i * dpad, ws.lm_in + (size_t)last[i] * dpad, dpad * 4,
                          cudaMemcpyDeviceToDevice, stream);
    if (e == cudaSuccess) e = head(ws, ws.lm_last, dpad, (int)(i1 - i0), ws.logits, ws.next, stream);
    if (e == cudaSuccess && logits)
      e = cudaMemcpyAsync(logits + i0 * G.logit_rows, ws.logits, (i1 - i0) * G.logit_rows * 4,
                          cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess && picks)
      e = cudaMemcpyAsync(picks + i0, ws.next, (i1 - i0) * 4, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = queue_wait_flag(stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess) e = wait_status(stream);
    if (e != cudaSuccess) {
      *err = cuda_msg("prefill", e);
      return false;
    }
    for (size_t i = i0; i < i1; ++i) ss[i]->pos = lens[i];
    i0 = i1;
  }
  return true;
}

// model.rs:482-492 forward_head with the confidence head: a prefill of `ids`
// on a scratch f32 session that also captures the cells, then the head.
bool Engine::confidence(const uint32_t* ids, size_t n, float* logit, std::string* err) {
  if (!cfg.has_heads) {
    *err = "this container exports no confidence head";
    return false;
  }
  if (n == 0 || n > cfg.max_seq) {
    *err = "input length must be in 1..max_seq_len";
    return false;
  }
  std::unique_ptr<Session> s(new_session(n, false, err));
  if (!s) return false;
  const size_t d = G.d, cells = conf.cells, m = cells * conf.probes_per_cell;
  float* buf = nullptr;
  {
    std::lock_guard<std::mutex> lk(mu);
    cudaSetDevice(device);
    cudaError_t e = cudaMalloc(&buf, (cells * n * d + m * d + conf.out_dim) * sizeof(float));
    if (e != cudaSuccess) {
      *err = cuda_msg("allocating the head cells", e);
      return false;
    }
  }
  Session* sp = s.get();
  const uint32_t* idp[1] = {ids};
  size_t lens[1] = {n};
  bool ok = prefill(&sp, idp, lens, 1, nullptr, nullptr, err, buf);
  if (ok) {
    std::lock_guard<std::mutex> lk(mu);
    cudaSetDevice(device);
    float* r = buf + cells * n * d;
    cudaError_t e = launch_probe_head(buf, (int)n, (int)d, conf, r, r + m * d, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(logit, r + m * d, sizeof(float), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
      *err = cuda_msg("confidence head", e);
      ok = false;
    }
  }
  {
    std::lock_guard<std::mutex> lk(mu);
    cudaSetDevice(device);
    cudaFree(buf);
  }
  return ok;
}

bool Engine::decode(Session* const* ss, const uint32_t* tokens, size_t n, float* logits,
                    uint32_t* picks, std::string* err) {
  std::lock_guard<std::mutex> lk(mu);
  cudaSetDevice(device);
  if (n == 0) return true;
  for (size_t i = 0; i < n; ++i) {
    if (!ss[i] || ss[i]->eng != this) {
      *err = "session does not belong to this handle";
      return false;
    }
    if (ss[i]->int8 != ss[0]->int8) {
      *err = "a batch must share one KV precision";
      return false;
    }
    if (ss[i]->pos >= cfg.max_seq) {
      *err = "session reached max_seq_len";
      return false;
    }
    if (!ensure_slots(ss[i], ss[i]->pos, err)) return false;
  }
  // A session twice in one batch: every session carries the stamp of the last
  // call that saw it (one pass instead of a sort of the list).
  ++batch_stamp;
  for (size_t i = 0; i < n; ++i) {
    if (ss[i]->seen == batch_stamp) {
      *err = "a session appears twice in one decode batch";
      return false;
    }
    ss[i]->seen = batch_stamp;
  }
  size_t maxpos = 0;
  for (size_t i = 0; i < n; ++i) maxpos = std::max(maxpos, ss[i]->pos);
  const int ns = attn_nsplit((int)n, G.kvh, (int)maxpos + 1);
  if (!ensure_ws(ws, n, err) || !ensure_logits(this, ws, n, err) || !ensure_part(ws, n, ns, err)) return false;
  // The stream is idle here (every call ends synchronised), so the pinned
  // staging buffers are free to refill.
  for (size_t i = 0; i < n; ++i) ws.h_rows[i] = RowInfo{ss[i]->d_desc, (int)ss[i]->pos, -1, -1, 0};
  std::memcpy(ws.h_tok, tokens, n * 4);
  const int dpad = (G.d + 127) / 128 * 128;
  cudaError_t e = cudaMemcpyAsync(ws.rows, ws.h_rows, n * sizeof(RowInfo), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(ws.tokens, ws.h_tok, n * 4, cudaMemcpyHostToDevice, stream);
  RowBatch rb{ws.rows, ws.tokens, (int)n, MODE_DECODE};
  const int int8 = ss[0]->int8 ? 1 : 0;
  auto body = [&](cudaStream_t s) -> cudaError_t {
    NB_TRY(forward(ws, rb, s, int8, ns, nullptr, true));
    NB_TRY(launch_step_end(rb, s));
    return head(ws, ws.lm_in, dpad, (int)n, ws.logits, ws.next, s, nullptr, logits != nullptr);
  };
  // Replay the captured step while its shapes and buffers are unchanged; a
  // new shape or epoch first runs one eager step (one-time set-up such as
  // shared-memory opt-ins happens outside any capture), then captures.
  const bool same = dec_n == n && dec_ns == ns && dec_int8 == int8 && dec_logits == (logits ? 1 : 0);
  if (e == cudaSuccess) {
    if (dec_graph && same && dec_graph_epoch == epoch) {
      e = cudaGraphLaunch(dec_graph, stream);
    } else if (same && dec_warm_epoch == epoch) {
      if (dec_graph) {
        cudaGraphExecDestroy(dec_graph);
        dec_graph = nullptr;
      }
      cudaGraph_t g = nullptr;
      e = cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal);
      if (e == cudaSuccess) {
        const cudaError_t eb = body(stream);
        e = cudaStreamEndCapture(stream, &g);
        if (eb != cudaSuccess) e = eb;
      }
      if (e == cudaSuccess) e = cudaGraphInstantiate(&dec_graph, g, 0);
      if (g) cudaGraphDestroy(g);
      if (e == cudaSuccess) {
        dec_graph_epoch = epoch;
        e = cudaGraphLaunch(dec_graph, stream);
      }
    } else {
      // A different shape: the captured graph (if any) belongs to the old key.
      if (dec_graph && !same) {
        cudaGraphExecDestroy(dec_graph);
        dec_graph = nullptr;
        dec_graph_epoch = 0;
      }
      e = body(stream);
      dec_n = n;
      dec_ns = ns;
      dec_int8 = int8;
      dec_logits = logits ? 1 : 0;
      dec_warm_epoch = epoch;
    }
  }
  if (e == cudaSuccess && logits)
    e = cudaMemcpyAsync(logits, ws.logits, n * G.logit_rows * 4, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess && picks) e = cudaMemcpyAsync(ws.h_pick, ws.next, n * 4, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = queue_wait_flag(stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess) e = wait_status(stream);
  if (e != cudaSuccess) {
    *err = cuda_msg("decode step", e);
    return false;
  }
  if (picks) std::memcpy(picks, ws.h_pick, n * 4);
  for (size_t i = 0; i < n; ++i) ss[i]->pos += 1;
  return true;
}

// ------------------------------------------------------------------ batches
Batch::~Batch() {
  if (graph) cudaGraphExecDestroy(graph);
  if (d_sess) cudaFree(d_sess);
  if (d_tok) cudaFree(d_tok);
  if (d_next) cudaFree(d_next);
}

Batch* Engine::new_batch(Session* const* ss, size_t n, std::string* err) {
  std::lock_guard<std::mutex> lk(mu);
  cudaSetDevice(device);
  if (n == 0) {
    *err = "empty batch";
    return nullptr;
  }
  std::unique_ptr<Batch> b(new Batch());
  b->eng = this;
  std::vector<SessDesc*> descs(n);
  for (size_t i = 0; i < n; ++i) {
    if (!ss[i] || ss[i]->eng != this) {
      *err = "session does not belong to this handle";
      return nullptr;
    }
    if (ss[i]->int8 != ss[0]->int8) {
      *err = "a batch must share one KV precision";
      return nullptr;
    }
    for (size_t j = 0; j < i; ++j)
      if (ss[j] == ss[i]) {
        *err = "a session appears twice in one batch";
        return nullptr;
      }
    descs[i] = ss[i]->d_desc;
  }
  b->sessions.assign(ss, ss + n);
  b->int8 = ss[0]->int8;
  cudaError_t e = cudaMalloc(&b->d_sess, n * sizeof(SessDesc*));
  if (e == cudaSuccess) e = cudaMemcpy(b->d_sess, descs.data(), n * sizeof(SessDesc*), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_tok, n * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_next, n * 4);
  if (e == cudaSuccess) e = cudaMemset(b->d_tok, 0, n * 4);
  if (e != cudaSuccess) {
    *err = cuda_msg("allocating the batch", e);
    return nullptr;
  }
  return b.release();
}

bool Engine::decode_batch_device(Batch* b, float* d_logits, cudaStream_t st, bool use_graph,
                                 std::string* err) {
  std::lock_guard<std::mutex> lk(mu);
  cudaSetDevice(device);
  const size_t n = b->sessions.size();
  for (Session* s : b->sessions) {
    if (s->pos >= cfg.max_seq) {
      *err = "session reached max_seq_len";
      return false;
    }
    if (!ensure_slots(s, s->pos, err)) return false;
  }
  size_t maxpos = 0;
  for (Session* s : b->sessions) maxpos = std::max(maxpos, s->pos);
  const int ns = attn_nsplit((int)n, G.kvh, (int)maxpos + 1);
  if (ns != b->nsplit) {  // a different split count changes the launch shapes
    b->nsplit = ns;
    b->graph_epoch = 0;
  }
  if (!ensure_ws(ws, n, err) || !ensure_part(ws, n, ns, err)) return false;
  const int dpad = (G.d + 127) / 128 * 128;
  float* lg = d_logits;
  if (!lg) {
    if (!ensure_logits(this, ws, n, err)) return false;
    lg = ws.logits;
  }
  RowBatch rb{ws.rows, b->d_tok, (int)n, MODE_DECODE};
  auto body = [&](cudaStream_t s) -> cudaError_t {
    NB_TRY(launch_step_begin(rb, b->d_sess, s));
    NB_TRY(forward(ws, rb, s, b->int8, ns, nullptr, true));
    NB_TRY(launch_step_end(rb, s));
    NB_TRY(head(ws, ws.lm_in, dpad, (int)n, lg, b->d_next, s, nullptr, d_logits != nullptr));
    return cudaSuccess;
  };
  cudaError_t e = cudaSuccess;
  // The graph bakes in workspace and ring pointers: it is rebuilt whenever one
  // of them changed (epoch) or the logits target changed. A rebuild is preceded
  // by one eager step at the same epoch, so every one-time setup (shared-memory
  // opt-ins) has happened before capture begins.
  const bool graph_ok = b->graph && b->graph_epoch == epoch && b->graph_logits == (d_logits != nullptr);
  if (use_graph && graph_ok) {
    e = cudaGraphLaunch(b->graph, st);
  } else if (use_graph && b->warm_epoch == epoch) {
    if (b->graph) {
      cudaGraphExecDestroy(b->graph);
      b->graph = nullptr;
    }
    cudaGraph_t g = nullptr;
    e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      cudaError_t eb = body(st);
      e = cudaStreamEndCapture(st, &g);
      if (eb != cudaSuccess) e = eb;
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&b->graph, g, 0);
    if (g) cudaGraphDestroy(g);
    if (e == cudaSuccess) {
      b->graph_epoch = epoch;
      b->graph_logits = d_logits != nullptr;
      e = cudaGraphLaunch(b->graph, st);
    }
  } else {
    e = body(st);
    if (use_graph) b->warm_epoch = epoch;
  }
  if (e != cudaSuccess) {
    *err = cuda_msg("batched decode step", e);
    return false;
  }
  for (Session* s : b->sessions) s->pos += 1;
  return true;
}

bool Engine::profile_batch_step(Batch* b, float* ms, int* launches, std::string* err) {
  std::lock_guard<std::mutex> lk(mu);
  cudaSetDevice(device);
  const size_t n = b->sessions.size();
  for (Session* s : b->sessions) {
    if (s->pos >= cfg.max_seq) {
      *err = "session reached max_seq_len";
      return false;
    }
    if (!ensure_slots(s, s->pos, err)) return false;
  }
  size_t maxpos = 0;
  for (Session* s : b->sessions) maxpos = std::max(maxpos, s->pos);
  const int ns = attn_nsplit((int)n, G.kvh, (int)maxpos + 1);
  if (!ensure_ws(ws, n, err) || !ensure_logits(this, ws, n, err) || !ensure_part(ws, n, ns, err)) return false;
  const int dpad = (G.d + 127) / 128 * 128;
  RowBatch rb{ws.rows, b->d_tok, (int)n, MODE_DECODE};
  Prof prof;
  cudaStream_t st = stream;
  auto run = [&]() -> cudaError_t {
    Prof* p = &prof;
    NB_TRY(p->mark(PK_BOOK, st, 0));
    NB_TRY(launch_step_begin(rb, b->d_sess, st));
    NB_TRY(p->mark(PK_BOOK, st, 1));
    NB_TRY(forward(ws, rb, st, b->int8, ns, p, true));
    NB_TRY(launch_step_end(rb, st));
    NB_TRY(p->mark(PK_BOOK, st, 1));
    NB_TRY(head(ws, ws.lm_in, dpad, (int)n, ws.logits, b->d_next, st, p, false));
    return cudaStreamSynchronize(st);
  };
  cudaError_t e = run();
  for (int k = 0; k < PK_COUNT; ++k) ms[k] = 0.f;
  for (size_t i = 1; e == cudaSuccess && i < prof.used; ++i) {
    float t = 0.f;
    e = cudaEventElapsedTime(&t, prof.marks[i - 1].second, prof.marks[i].second);
    ms[prof.marks[i].first] += t;
  }
  for (auto& m : prof.marks) cudaEventDestroy(m.second);
  if (e != cudaSuccess) {
    *err = cuda_msg("profiled decode step", e);
    return false;
  }
  *launches = prof.launches;
  for (Session* s : b->sessions) s->pos += 1;
  return true;
}

}  // namespace nb
