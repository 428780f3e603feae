// Grammar-constrained decoding of tool calls (host code): the restatement of
// crates/needle-infer/src/constrained.rs. Inside a <tool_call> span the model's
// compact JSON is followed byte by byte; while it writes a tool name or an
// argument key, only tokens that continue a declared name or key stay
// possible (the others get -1e9 added to their logits).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace nb {

// A byte trie of the allowed names or keys (constrained.rs:20-75).
struct ByteTrie {
  struct Node {
    std::map<uint8_t, int> kids;
    bool terminal = false;
  };
  std::vector<Node> nodes{Node()};
  void insert(const std::string& s);
  int advance(int node, const std::string& bytes) const;  // -1 when it leaves the trie
  int child(int node, uint8_t b) const;
};

// A declared tool: its name, the snake_case form the model writes, and its
// argument keys (constrained.rs:317-327, :463-537).
struct ToolDef {
  std::string name, snake_name;
  std::vector<std::string> param_keys;
};
std::vector<ToolDef> parse_tools_json(const std::string& json);
std::string to_snake_case(const std::string& name);  // tokenizer.rs:250-292

// Position in the model's compact JSON output (constrained.rs:119-315).
struct JsonMachine {
  enum State { FREE, IN_NAME, IN_ARG_KEY };
  State state = FREE;
  std::string current_function, buf;
  std::vector<std::string> used_keys;
  bool in_arguments = false, in_string = false, prev_escape = false;
  size_t arguments_depth = 0, nesting_depth = 0;
  std::string tail;  // the last 13 output bytes
  void feed_byte(uint8_t b);
  void feed(const std::string& bytes) {
    for (char c : bytes) feed_byte((uint8_t)c);
  }
};

class ConstrainedDecoder {
 public:
  // token_texts[id]: the bytes token id adds to the output.
  ConstrainedDecoder(const std::vector<ToolDef>& tools, std::vector<std::string> token_texts, bool unique_keys);
  void update(uint32_t token);  // after emitting a token inside a call
  void feed_bytes(const std::string& bytes) { sm_.feed(bytes); }
  // Additive logit mask over `vocab` ids for the current state.
  std::vector<float> logit_mask(size_t vocab) const;

 private:
  std::vector<float> mask_from(const ByteTrie& trie, int node, size_t vocab) const;
  ByteTrie names_;
  std::map<std::string, ByteTrie> key_tries_;
  std::map<std::string, std::vector<std::string>> keys_;
  JsonMachine sm_;
  std::vector<std::string> texts_;
  bool unique_;
};

}  // namespace nb
