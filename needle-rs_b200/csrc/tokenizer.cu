// SentencePiece BPE tokenizer of the container (host code); see tokenizer.hpp.
#include <algorithm>
#include <cstring>

#include "tokenizer.hpp"

namespace nb {
namespace {

const char kMetaSpace[] = "\xE2\x96\x81";  // U+2581, SentencePiece's visible space

uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }

// Length of the well-formed UTF-8 sequence at s[i], or 0 when ill-formed;
// *bad receives how many bytes form the maximal ill-formed prefix (>= 1).
size_t utf8_seq(const std::string& s, size_t i, size_t* bad) {
  const unsigned char b0 = (unsigned char)s[i];
  if (b0 < 0x80) return 1;
  size_t len;
  unsigned char lo = 0x80, hi = 0xBF;  // range of the second byte
  if (b0 >= 0xC2 && b0 <= 0xDF) len = 2;
  else if (b0 == 0xE0) len = 3, lo = 0xA0;
  else if ((b0 >= 0xE1 && b0 <= 0xEC) || b0 == 0xEE || b0 == 0xEF) len = 3;
  else if (b0 == 0xED) len = 3, hi = 0x9F;
  else if (b0 == 0xF0) len = 4, lo = 0x90;
  else if (b0 >= 0xF1 && b0 <= 0xF3) len = 4;
  else if (b0 == 0xF4) len = 4, hi = 0x8F;
  else {
    *bad = 1;
    return 0;
  }
  for (size_t k = 1; k < len; ++k) {
    if (i + k >= s.size()) {
      *bad = k;
      return 0;
    }
    const unsigned char c = (unsigned char)s[i + k];
    const bool ok = k == 1 ? (c >= lo && c <= hi) : (c >= 0x80 && c <= 0xBF);
    if (!ok) {
      *bad = k;
      return 0;
    }
  }
  return len;
}

bool valid_utf8(const std::string& s) {
  for (size_t i = 0; i < s.size();) {
    size_t bad = 0, n = utf8_seq(s, i, &bad);
    if (!n) return false;
    i += n;
  }
  return true;
}

int hexval(char c) {
  if (c >= '0' && c <= '9') return c - '0';
  if (c >= 'a' && c <= 'f') return c - 'a' + 10;
  if (c >= 'A' && c <= 'F') return c - 'A' + 10;
  return -1;
}

// The byte of a `<0xNN>` piece: characters 3..5 of the surface read as a
// base-16 number (an optional '+' sign, as an unsigned integer parse allows).
bool byte_of(const std::string& p, int* b) {
  if (p.size() < 5) return false;
  const char c0 = p[3], c1 = p[4];
  if (c0 == '+') {
    const int v = hexval(c1);
    if (v < 0) return false;
    *b = v;
    return true;
  }
  const int h = hexval(c0), l = hexval(c1);
  if (h < 0 || l < 0) return false;
  *b = h * 16 + l;
  return true;
}

}  // namespace

std::string utf8_lossy(const std::string& s) {
  std::string out;
  out.reserve(s.size());
  for (size_t i = 0; i < s.size();) {
    size_t bad = 0, n = utf8_seq(s, i, &bad);
    if (n) {
      out.append(s, i, n);
      i += n;
    } else {
      out += "\xEF\xBF\xBD";
      i += bad;
    }
  }
  return out;
}

Tokenizer* Tokenizer::from_blob(const uint8_t* blob, size_t len, std::string* err) {
  if (!blob || len < 24) {
    *err = "tokenizer blob truncated: need 24 bytes, got " + std::to_string(blob ? len : 0);
    return nullptr;
  }
  const size_t n = rd32(blob);
  if (n == 0) {
    *err = "tokenizer blob declares zero pieces";
    return nullptr;
  }
  Tokenizer* t = new Tokenizer();
  t->pad_id = rd32(blob + 4);
  t->eos_id = rd32(blob + 8);
  t->bos_id = rd32(blob + 12);
  t->unk_id = rd32(blob + 16);
  t->add_dummy_prefix = blob[20] != 0;
  t->byte_fallback = blob[21] != 0;
  auto fail = [&](const std::string& m) -> Tokenizer* {
    *err = m;
    delete t;
    return nullptr;
  };
  size_t off = 24;
  for (size_t i = 0; i < n; ++i) {
    if (off + 7 > len)
      return fail("tokenizer blob truncated: need " + std::to_string(off + 7) + " bytes, got " + std::to_string(len));
    float score;
    std::memcpy(&score, blob + off, 4);
    const uint8_t ty = blob[off + 4];
    const size_t sl = (size_t)blob[off + 5] | (size_t)blob[off + 6] << 8;
    off += 7;
    if (off + sl > len)
      return fail("tokenizer blob truncated: need " + std::to_string(off + sl) + " bytes, got " + std::to_string(len));
    std::string surface(reinterpret_cast<const char*>(blob + off), sl);
    off += sl;
    if (!valid_utf8(surface)) return fail("piece " + std::to_string(i) + " is not valid UTF-8");
    t->pieces_.push_back(std::move(surface));
    t->scores_.push_back(score);
    t->types_.push_back(ty);
  }
  const std::pair<const char*, uint32_t> specials[4] = {
      {"pad", t->pad_id}, {"eos", t->eos_id}, {"bos", t->bos_id}, {"unk", t->unk_id}};
  for (const auto& sp : specials)
    if (sp.second >= n)
      return fail(std::string(sp.first) + " id " + std::to_string(sp.second) + " is past the " + std::to_string(n) +
                  " pieces");
  for (size_t i = 0; i < n; ++i) t->to_id_[t->pieces_[i]] = (uint32_t)i;
  std::fill(t->byte_id_, t->byte_id_ + 256, -1);
  for (size_t i = 0; i < n; ++i) {
    if (t->types_[i] != BYTE) continue;
    int b;
    if (!byte_of(t->pieces_[i], &b)) return fail("byte piece " + std::to_string(i) + " is not of the form <0xNN>");
    t->byte_id_[b] = (int32_t)i;
  }
  for (size_t i = 0; i < n; ++i)
    if (t->types_[i] == USER_DEFINED) t->markers_.push_back({t->pieces_[i], (uint32_t)i});
  std::stable_sort(t->markers_.begin(), t->markers_.end(),
                   [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
  return t;
}

bool Tokenizer::id_of(const std::string& surface, uint32_t* id) const {
  auto it = to_id_.find(surface);
  if (it == to_id_.end()) return false;
  *id = it->second;
  return true;
}

// Greedy pairwise merging over the characters of one segment: each round
// merges the adjacent pair whose concatenation is the highest-scoring piece
// (the leftmost such pair on ties), until no adjacent pair is a piece
// (sp_tokenizer.rs:292-368). Unknown symbols fall back to byte pieces.
void Tokenizer::bpe(const std::string& seg, std::vector<uint32_t>* out) const {
  if (seg.empty()) return;
  std::vector<size_t> st, en;
  for (size_t i = 0; i < seg.size();) {
    size_t bad = 0, n = utf8_seq(seg, i, &bad);
    if (!n) n = bad;  // inputs are validated; keep going on a malformed byte
    st.push_back(i);
    en.push_back(i + n);
    i += n;
  }
  const int m = (int)st.size();
  std::vector<int> nx(m);
  for (int i = 0; i < m; ++i) nx[i] = i + 1 < m ? i + 1 : -1;
  std::string key;
  for (int live = m; live > 1; --live) {
    int best = -1;
    float best_score = 0.f;
    for (int j = 0; j >= 0 && nx[j] >= 0; j = nx[j]) {
      const int k = nx[j];
      key.assign(seg, st[j], en[k] - st[j]);
      auto it = to_id_.find(key);
      if (it == to_id_.end()) continue;
      const float s = scores_[it->second];
      if (best < 0 || s > best_score) {
        best = j;
        best_score = s;
      }
    }
    if (best < 0) break;
    const int k = nx[best];
    en[best] = en[k];
    nx[best] = nx[k];
  }
  for (int j = 0; j >= 0; j = nx[j]) {
    key.assign(seg, st[j], en[j] - st[j]);
    auto it = to_id_.find(key);
    if (it != to_id_.end()) {
      out->push_back(it->second);
    } else if (byte_fallback) {
      for (size_t b = st[j]; b < en[j]; ++b) {
        const int id = byte_id_[(unsigned char)seg[b]];
        out->push_back(id >= 0 ? (uint32_t)id : unk_id);
      }
    } else {
      out->push_back(unk_id);
    }
  }
}

// Spaces become the meta space (and one is prepended with add_dummy_prefix);
// user-defined markers split the text, longest marker first at each
// position, and every stretch between them is merged by bpe
// (sp_tokenizer.rs:253-295).
std::vector<uint32_t> Tokenizer::encode(const std::string& text) const {
  std::vector<uint32_t> ids;
  if (text.empty()) return ids;
  std::string esc = add_dummy_prefix ? kMetaSpace : "";
  for (char c : text) {
    if (c == ' ') esc += kMetaSpace;
    else esc += c;
  }
  std::string buf;
  for (size_t i = 0; i < esc.size();) {
    bool hit = false;
    for (const auto& mk : markers_) {
      if (esc.compare(i, mk.first.size(), mk.first) == 0 && !mk.first.empty()) {
        bpe(buf, &ids);
        buf.clear();
        ids.push_back(mk.second);
        i += mk.first.size();
        hit = true;
        break;
      }
    }
    if (hit) continue;
    size_t bad = 0, n = utf8_seq(esc, i, &bad);
    if (!n) n = bad;
    buf.append(esc, i, n);
    i += n;
  }
  bpe(buf, &ids);
  return ids;
}

// Byte pieces contribute their byte, control and unknown pieces nothing,
// others their surface; the bytes are read as UTF-8 (ill-formed runs become
// U+FFFD), meta spaces become spaces and one leading space is dropped under
// add_dummy_prefix (sp_tokenizer.rs:390-414).
std::string Tokenizer::decode(const uint32_t* ids, size_t n) const {
  std::string buf;
  for (size_t i = 0; i < n; ++i) {
    const uint32_t id = ids[i];
    if (id >= pieces_.size()) continue;
    const uint8_t ty = types_[id];
    if (ty == BYTE) {
      int b;
      if (byte_of(pieces_[id], &b)) buf += (char)b;
    } else if (ty != CONTROL && ty != UNKNOWN) {
      buf += pieces_[id];
    }
  }
  const std::string text = utf8_lossy(buf);
  std::string out;
  out.reserve(text.size());
  for (size_t i = 0; i < text.size();) {
    if (text.compare(i, 3, kMetaSpace) == 0) {
      out += ' ';
      i += 3;
    } else {
      out += text[i++];
    }
  }
  if (add_dummy_prefix && !out.empty() && out[0] == ' ') out.erase(0, 1);
  return out;
}

std::vector<std::string> Tokenizer::token_bytes() const {
  std::vector<std::string> out(pieces_.size());
  for (size_t id = 0; id < pieces_.size(); ++id) {
    const uint8_t ty = types_[id];
    if (ty == BYTE) {
      int b;
      if (byte_of(pieces_[id], &b)) out[id] = std::string(1, (char)b);
    } else if (ty != CONTROL && ty != UNKNOWN) {
      const std::string& p = pieces_[id];
      for (size_t i = 0; i < p.size();) {
        if (p.compare(i, 3, kMetaSpace) == 0) {
          out[id] += ' ';
          i += 3;
        } else {
          out[id] += p[i++];
        }
      }
    }
  }
  return out;
}

}  // namespace nb
