// TEST INFRASTRUCTURE — CPU restatement of the `.cact` v3 reader
// (crates/needle-infer/src/cact.rs:306-525, 981-1100) and the v3 loader
// (crates/needle-infer/src/v3.rs:25-484) of bynds/needle-rs.
#include <cmath>
#include <cstring>

#include "oracle.hpp"

namespace oracle {

static uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }

namespace {
struct Loader {
  const uint8_t* raw;
  size_t len;
  std::vector<Record> recs;
  std::vector<float> codebook;
  std::string err;

  bool floats(size_t i, std::vector<float>* out) {  // cact.rs:494-524
    if (i >= recs.size()) {
      err = "tensor index out of range";
      return false;
    }
    const Record& r = recs[i];
    const uint8_t* b = raw + r.offset;
    if (r.dtype == DT_FP16) {
      if (r.nbytes % 2) {
        err = "ragged fp16 blob " + std::to_string(i);
        return false;
      }
      out->resize(r.nbytes / 2);
      for (size_t k = 0; k < out->size(); ++k)
        (*out)[k] = f16_to_f32((uint16_t)(b[2 * k] | (b[2 * k + 1] << 8)));
      return true;
    }
    if (r.dtype == DT_FP32) {
      if (r.nbytes % 4) {
        err = "ragged fp32 blob " + std::to_string(i);
        return false;
      }
      out->resize(r.nbytes / 4);
      std::memcpy(out->data(), b, r.nbytes);
      return true;
    }
    err = "tensor " + std::to_string(i) + ": expected dtype 1, got " + std::to_string(r.dtype);
    return false;
  }
  bool cq(size_t i, CqWeight* w) {  // cact.rs:1073-1091
    const Record& r = recs[i];
    if (r.dtype != DT_CQ) {
      err = "tensor " + std::to_string(i) + ": expected dtype 3, got " + std::to_string(r.dtype);
      return false;
    }
    std::string e = CqWeight::from_blob(raw + r.offset, r.nbytes, r.shape[0], r.shape[1], r.group,
                                        r.bits, codebook.data(), codebook.size(), w);
    if (!e.empty()) {
      err = "tensor " + std::to_string(i) + ": " + e;
      return false;
    }
    return true;
  }
};
}  // namespace

std::string load_model(const uint8_t* raw, size_t len, V3Model* m) {
  if (len < HEADER_BYTES_V3) return "container too short";
  uint32_t w[49];
  for (int i = 0; i < 49; ++i) w[i] = rd32(raw + 4 * i);
  if (w[0] != TAG_V3) return "bad tag";  // cact.rs:351
  size_t num_tensors = w[1], codebook_len = w[2];
  if (codebook_len != CODEBOOK_LEN) return "bad codebook length";
  size_t dir_start = HEADER_BYTES_V3 + codebook_len * 4;
  size_t dir_end = dir_start + num_tensors * REC_BYTES;
  if (len < dir_end) return "container too short for directory";
  Loader L{raw, len, {}, {}, ""};
  L.codebook.resize(codebook_len);
  std::memcpy(L.codebook.data(), raw + HEADER_BYTES_V3, codebook_len * 4);
  for (size_t i = 0; i < num_tensors; ++i) {  // cact.rs:398-425
    const uint8_t* b = raw + dir_start + i * REC_BYTES;
    Record r;
    r.dtype = b[0];
    r.ndim = b[1];
    if (r.ndim > 4) return "bad ndim";
    for (int k = 0; k < 4; ++k) r.shape[k] = rd32(b + 4 + 4 * k);
    r.offset = rd64(b + 20);
    r.nbytes = rd64(b + 28);
    r.group = rd32(b + 36);
    r.bits = (uint8_t)rd32(b + 40);
    if (r.offset + r.nbytes > len) return "blob out of range";
    L.recs.push_back(r);
  }

  // v3.rs:25-70 config_from_geometry
  V3Config& c = m->cfg;
  size_t num_orders = w[26], num_sites = w[31];
  c.engram.orders.clear();
  for (size_t k = 0; k < std::min<size_t>(num_orders, 4); ++k) c.engram.orders.push_back(w[27 + k]);
  c.engram.sites.clear();
  for (size_t k = 0; k < std::min<size_t>(num_sites, 16); ++k) c.engram.sites.push_back(w[32 + k]);
  if (c.engram.orders.empty()) return "container declares no engram orders";
  size_t tables = w[22];
  if (tables % c.engram.orders.size()) return "engram tables not divisible by orders";
  size_t eheads = tables / c.engram.orders.size();
  c.vocab_size = w[5];
  c.out_vocab = w[6];
  c.d_model = w[7];
  c.num_heads = w[8];
  c.num_kv_heads = w[9];
  c.num_layers = w[10];
  c.qk_head_dim = w[11];
  c.v_head_dim = w[12];
  c.max_seq_len = w[13];
  c.hada_n = w[14];
  c.mhc_lanes = w[15];
  c.sliding_window = w[16];
  uint64_t gmask = (uint64_t)w[17] | ((uint64_t)w[18] << 32);
  c.global_layers.clear();
  for (size_t i = 0; i < c.num_layers; ++i)
    if (i < 64 && ((gmask >> i) & 1)) c.global_layers.push_back(i);
  c.qkv_conv_taps = w[19];
  c.engram.slots = w[20];
  c.engram.sub_dim = w[21];
  c.engram.heads = eheads;
  c.engram.conv_taps = w[23];
  c.engram.conv_dilation = w[24];
  c.engram.seed_heads = w[25];
  float theta;
  std::memcpy(&theta, &w[48], 4);
  c.rope_theta = theta;
  if (c.d_model / (c.engram.orders.size() * eheads) != c.engram.sub_dim) return "engram sub_dim mismatch";
  if (c.num_kv_heads == 0 || c.num_heads % c.num_kv_heads) return "heads not divisible";

  // v3.rs:236-332 canon walk + :336-383 validation.
  size_t cur = 0;
  auto take = [&](size_t* idx) {
    if (cur >= num_tensors) return false;
    *idx = cur++;
    return true;
  };
  auto shape_is = [&](size_t i, size_t a, size_t b) {
    return L.recs[i].shape[0] == a && L.recs[i].shape[1] == b;
  };
  size_t emb;
  if (!take(&emb)) return "too few tensors";
  if (!shape_is(emb, c.vocab_size, c.d_model)) return "embedding shape";
  if (!L.cq(emb, &m->embedding)) return L.err;
  m->layers.assign(c.num_layers, V3Layer());
  for (size_t li = 0; li < c.num_layers; ++li) {
    V3Layer& ly = m->layers[li];
    size_t ix[27];
    size_t count = 24 + (c.qkv_conv_taps ? 3 : 0);
    for (size_t k = 0; k < count; ++k)
      if (!take(&ix[k])) return "too few tensors";
    size_t p = 0;
    size_t norm_in = ix[p++], q = ix[p++], k = ix[p++], v = ix[p++];
    size_t qt = 0, kt = 0, vt = 0;
    if (c.qkv_conv_taps) {
      qt = ix[p++];
      kt = ix[p++];
      vt = ix[p++];
    }
    size_t qn = ix[p++], kn = ix[p++], gate = ix[p++], out = ix[p++], post = ix[p++],
           agate = ix[p++], pre = ix[p++];
    size_t mlp[13];
    for (int j = 0; j < 13; ++j) mlp[j] = ix[p++];
    if (!shape_is(q, c.q_dim(), c.d_model)) return "q_proj shape";
    if (!shape_is(k, c.k_dim(), c.d_model)) return "k_proj shape";
    if (!shape_is(v, c.v_dim(), c.d_model)) return "v_proj shape";
    if (!shape_is(gate, c.attn_out_dim(), c.d_model)) return "gate_proj shape";
    if (!shape_is(out, c.d_model, c.attn_out_dim())) return "out_proj shape";
    std::vector<float> ag;
    bool ok = L.floats(norm_in, &ly.norm_in) && L.cq(q, &ly.q_proj) && L.cq(k, &ly.k_proj) &&
              L.cq(v, &ly.v_proj) && L.floats(qn, &ly.q_norm) && L.floats(kn, &ly.k_norm) &&
              L.cq(gate, &ly.gate_proj) && L.cq(out, &ly.out_proj) &&
              L.floats(post, &ly.post_norm) && L.floats(agate, &ag) && L.floats(pre, &ly.pre_hada);
    if (ok && c.qkv_conv_taps)
      ok = L.floats(qt, &ly.q_taps) && L.floats(kt, &ly.k_taps) && L.floats(vt, &ly.v_taps);
    HadaMlp& h = ly.mlp;
    if (ok)
      ok = L.floats(mlp[0], &h.d1) && L.floats(mlp[1], &h.d2) && L.floats(mlp[2], &h.b2) &&
           L.floats(mlp[3], &h.d3) && L.floats(mlp[4], &h.d4) && L.floats(mlp[5], &h.w1a) &&
           L.floats(mlp[6], &h.w1b) && L.floats(mlp[7], &h.w2a) && L.floats(mlp[8], &h.w2b) &&
           L.floats(mlp[9], &h.w3a) && L.floats(mlp[10], &h.w3b) && L.floats(mlp[11], &h.cond_v) &&
           L.floats(mlp[12], &h.cond_u);
    if (!ok) return L.err;
    if (ag.empty()) return "empty attn_gate";
    ly.attn_gate = ag[0];
    h.cond_rank = L.recs[mlp[11]].shape[1];
  }
  size_t sc[6], phi[3], perm[2];
  for (int j = 0; j < 6; ++j)
    if (!take(&sc[j])) return "too few tensors";
  for (int j = 0; j < 3; ++j)
    if (!take(&phi[j])) return "too few tensors";
  for (int j = 0; j < 2; ++j)
    if (!take(&perm[j])) return "too few tensors";
  V3Mhc& mh = m->mhc;
  if (!(L.floats(sc[0], &mh.a_pre) && L.floats(sc[1], &mh.a_post) && L.floats(sc[2], &mh.a_res) &&
        L.floats(sc[3], &mh.b_pre) && L.floats(sc[4], &mh.b_post) && L.floats(sc[5], &mh.b_res) &&
        L.cq(phi[0], &mh.phi_pre) && L.cq(phi[1], &mh.phi_post) && L.cq(phi[2], &mh.phi_res)))
    return L.err;
  m->engrams.assign(c.engram.sites.size(), V3EngramSite());
  for (size_t s = 0; s < c.engram.sites.size(); ++s) {
    size_t t, kp, vp, tp;
    if (!(take(&t) && take(&kp) && take(&vp) && take(&tp))) return "too few tensors";
    if (!shape_is(t, c.engram.num_tables() * c.engram.slots, c.engram.sub_dim)) return "engram tables shape";
    if (!shape_is(kp, c.d_model, c.d_model)) return "engram key_proj shape";
    if (!shape_is(vp, c.d_model, c.d_model)) return "engram value_proj shape";
    V3EngramSite& es = m->engrams[s];
    if (!(L.cq(t, &es.tables) && L.cq(kp, &es.key_proj) && L.cq(vp, &es.value_proj) &&
          L.floats(tp, &es.taps)))
      return L.err;
  }
  size_t fn;
  if (!take(&fn)) return "too few tensors";
  if (!L.floats(fn, &m->final_norm)) return L.err;
  std::vector<float> p1, p2;
  if (!(L.floats(perm[0], &p1) && L.floats(perm[1], &p2))) return L.err;
  m->perms.p1.resize(p1.size());
  m->perms.p2.resize(p2.size());
  for (size_t i = 0; i < p1.size(); ++i) m->perms.p1[i] = (uint32_t)p1[i];
  for (size_t i = 0; i < p2.size(); ++i) m->perms.p2[i] = (uint32_t)p2[i];
  // Probe heads (v3.rs:300-316, :486-560): the records between the final norm
  // and the RAW tokenizer are a manifest of head codes, then six tensors per
  // head (seven for the router): probes, gain, query, row_bias, proj, bias.
  size_t head_end = num_tensors;
  for (size_t i = 0; i < num_tensors; ++i)
    if (L.recs[i].dtype == DT_RAW) {
      head_end = i;
      break;
    }
  if (cur < head_end) {
    std::vector<float> codes;
    if (!L.floats(cur++, &codes)) return L.err;
    for (float code : codes) {
      const size_t need = (uint8_t)code == 3 ? 7 : 6;
      if (cur + need > head_end) return "head tensors ran out";
      const size_t pi = cur, gi = cur + 1, qi = cur + 2, ri = cur + 3, ji = cur + 4, bi = cur + 5;
      cur += need;
      if ((uint8_t)code != 2) continue;
      ProbeHead& h = m->confidence;
      auto dense = [&](size_t i, std::vector<float>* out) {
        CqWeight w;
        if (!L.cq(i, &w)) return false;
        out->assign(w.out_feat * w.in_feat, 0.f);
        for (size_t o = 0; o < w.out_feat; ++o) w.dequantize_row(o, out->data() + o * w.in_feat);
        return true;
      };
      if (!(dense(pi, &h.probes) && L.floats(gi, &h.gain) && dense(qi, &h.query) && L.floats(ri, &h.row_bias) &&
            dense(ji, &h.proj) && L.floats(bi, &h.bias)))
        return L.err;
      h.cells = c.num_layers + 1;
      const size_t prow = L.recs[pi].shape[0];
      if (prow % h.cells || h.gain.size() != prow) return "probe head shapes disagree with num_layers + 1 cells";
      h.probes_per_cell = prow / h.cells;
      h.queries = L.recs[qi].shape[0];
      h.out_dim = L.recs[ji].shape[0];
      m->has_confidence = true;
    }
  }
  // model.rs:110-136 V3Model::new
  if (m->embedding.out_feat != c.vocab_size || m->embedding.in_feat != c.d_model)
    return "embedding shape does not match geometry";
  m->embed_scale = sqrtf((float)c.d_model);
  return "";
}

}  // namespace oracle
