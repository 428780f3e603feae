// SentencePiece BPE tokenizer read from the RAW tokenizer record of a `.cact`
// container (the encoder/decoder that upstream ships as the normative spec of
// the blob, restated by crates/needle-infer/src/sp_tokenizer.rs). Host code:
// text in, ids out, and back.
//
// Blob (little-endian): header of 24 bytes — u32 n_pieces, pad_id, eos_id,
// bos_id, unk_id; u8 add_dummy_prefix, u8 byte_fallback, u16 padding — then
// n_pieces records in id order: f32 score, u8 type, u16 length, UTF-8 bytes.
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace nb {

class Tokenizer {
 public:
  // Piece types (sp_tokenizer.rs:27-32).
  enum : uint8_t { NORMAL = 0, UNKNOWN = 1, CONTROL = 2, USER_DEFINED = 3, BYTE = 4 };

  // nullptr with *err set when the blob is malformed (sp_tokenizer.rs:116-223).
  static Tokenizer* from_blob(const uint8_t* blob, size_t len, std::string* err);

  std::vector<uint32_t> encode(const std::string& text) const;
  std::string decode(const uint32_t* ids, size_t n) const;
  // Exact surface -> id; false when absent.
  bool id_of(const std::string& surface, uint32_t* id) const;
  size_t size() const { return pieces_.size(); }
  // Bytes each token contributes to decoded output, by id: a byte piece its
  // byte, control and unknown pieces nothing, others their surface with the
  // meta space as a space (sp_tokenizer.rs:370-388).
  std::vector<std::string> token_bytes() const;

  uint32_t pad_id = 0, eos_id = 0, bos_id = 0, unk_id = 0;
  bool add_dummy_prefix = false, byte_fallback = false;

 private:
  void bpe(const std::string& seg, std::vector<uint32_t>* out) const;

  std::vector<std::string> pieces_;
  std::vector<float> scores_;
  std::vector<uint8_t> types_;
  std::unordered_map<std::string, uint32_t> to_id_;  // later duplicates win
  int32_t byte_id_[256];                              // -1 when absent
  std::vector<std::pair<std::string, uint32_t>> markers_;  // user-defined, longest first
};

// Bytes as UTF-8 text, each maximal ill-formed subsequence replaced by U+FFFD
// (the substitution that Rust's String::from_utf8_lossy applies).
std::string utf8_lossy(const std::string& bytes);

}  // namespace nb
