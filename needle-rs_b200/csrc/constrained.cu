// Grammar-constrained decoding of tool calls (host code); see constrained.hpp.
#include <algorithm>

#include "constrained.hpp"

namespace nb {
namespace {

const char kNameTrigger[] = "\"name\":\"";         // enters a tool name
const char kArgsTrigger[] = "\"arguments\":{";     // opens the arguments object
constexpr size_t kTail = 13;                        // longest trigger

bool ends_with(const std::string& s, const char* t) {
  const size_t n = std::char_traits<char>::length(t);
  return s.size() >= n && s.compare(s.size() - n, n, t) == 0;
}

bool ascii_ws(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\f'; }

// Unicode White_Space at the start of s (what str::trim_start removes).
size_t skip_unicode_ws(const std::string& s, size_t i) {
  while (i < s.size()) {
    const unsigned char b = (unsigned char)s[i];
    if (b < 0x80) {
      if ((b >= 0x09 && b <= 0x0D) || b == 0x20) {
        ++i;
        continue;
      }
      return i;
    }
    // Multi-byte white space: U+0085, U+00A0, U+1680, U+2000-200A, U+2028,
    // U+2029, U+202F, U+205F, U+3000.
    uint32_t c = 0;
    size_t n = b < 0xE0 ? 2 : b < 0xF0 ? 3 : 4;
    if (i + n > s.size()) return i;
    c = b & (0xFF >> (n + 1));
    for (size_t k = 1; k < n; ++k) c = (c << 6) | ((unsigned char)s[i + k] & 0x3F);
    const bool ws = c == 0x85 || c == 0xA0 || c == 0x1680 || (c >= 0x2000 && c <= 0x200A) || c == 0x2028 ||
                    c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
    if (!ws) return i;
    i += n;
  }
  return i;
}

// Index of the delimiter closing the one at `start`, skipping quoted strings;
// the last index when unmatched (constrained.rs:539-568).
size_t find_matching(const std::string& s, size_t start, char open, char close) {
  size_t depth = 0;
  bool in_str = false, esc = false;
  for (size_t i = start; i < s.size(); ++i) {
    const char b = s[i];
    if (in_str) {
      if (esc) esc = false;
      else if (b == '\\') esc = true;
      else if (b == '"') in_str = false;
    } else if (b == '"') {
      in_str = true;
    } else if (b == open) {
      ++depth;
    } else if (b == close) {
      depth = depth ? depth - 1 : 0;
      if (depth == 0) return i;
    }
  }
  return s.empty() ? 0 : s.size() - 1;
}

// `"field":"value"` -> value (escapes kept as written).
bool extract_string(const std::string& obj, const std::string& field, std::string* out) {
  const std::string needle = "\"" + field + "\":\"";
  const size_t pos = obj.find(needle);
  if (pos == std::string::npos) return false;
  const size_t a = pos + needle.size();
  bool esc = false;
  for (size_t i = a; i < obj.size(); ++i) {
    if (esc) esc = false;
    else if (obj[i] == '\\') esc = true;
    else if (obj[i] == '"') {
      *out = obj.substr(a, i - a);
      return true;
    }
  }
  return false;
}

// `"field":{...}` -> {...}.
bool extract_object(const std::string& obj, const std::string& field, std::string* out) {
  const std::string needle = "\"" + field + "\":";
  const size_t pos = obj.find(needle);
  if (pos == std::string::npos) return false;
  const std::string after = obj.substr(skip_unicode_ws(obj, pos + needle.size()));
  if (after.empty() || after[0] != '{') return false;
  *out = after.substr(0, find_matching(after, 0, '{', '}') + 1);
  return true;
}

size_t skip_value(const std::string& s, size_t i) {
  if (i >= s.size()) return i;
  if (s[i] == '{') return find_matching(s, i, '{', '}') + 1;
  if (s[i] == '[') return find_matching(s, i, '[', ']') + 1;
  if (s[i] == '"') {
    bool esc = false;
    for (++i; i < s.size(); ++i) {
      if (esc) esc = false;
      else if (s[i] == '\\') esc = true;
      else if (s[i] == '"') return i + 1;
    }
    return i;
  }
  while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']') ++i;
  return i;
}

// Top-level keys of an object; with `objects_only`, those whose value is an
// object (constrained.rs:604-724).
std::vector<std::string> object_keys(const std::string& obj, bool objects_only) {
  std::vector<std::string> keys;
  size_t i = 0;
  if (!obj.empty() && obj[0] == '{') i = 1;
  while (i < obj.size()) {
    while (i < obj.size() && (obj[i] == ',' || ascii_ws(obj[i]))) ++i;
    if (i >= obj.size() || obj[i] == '}') break;
    if (obj[i] != '"') {
      ++i;
      continue;
    }
    const size_t ks = ++i;
    bool esc = false;
    for (; i < obj.size(); ++i) {
      if (esc) esc = false;
      else if (obj[i] == '\\') esc = true;
      else if (obj[i] == '"') break;
    }
    const std::string key = obj.substr(ks, i - ks);
    ++i;
    while (i < obj.size() && obj[i] != ':') ++i;
    ++i;
    while (i < obj.size() && ascii_ws(obj[i])) ++i;
    if (objects_only) {
      if (i < obj.size() && obj[i] == '{') {
        if (!key.empty()) keys.push_back(key);
        i = find_matching(obj, i, '{', '}') + 1;
      } else {
        i = skip_value(obj, i);
      }
    } else {
      if (!key.empty()) keys.push_back(key);
      i = skip_value(obj, i);
    }
  }
  return keys;
}

// ASCII character classes (tool names are ASCII in practice; other code
// points count as alphanumeric and caseless).
bool is_upper(uint32_t c) { return c >= 'A' && c <= 'Z'; }
bool is_lower(uint32_t c) { return c >= 'a' && c <= 'z'; }
bool is_alnum(uint32_t c) { return is_upper(c) || is_lower(c) || (c >= '0' && c <= '9') || c >= 0x80; }

}  // namespace

void ByteTrie::insert(const std::string& s) {
  int cur = 0;
  for (char ch : s) {
    const uint8_t b = (uint8_t)ch;
    auto it = nodes[cur].kids.find(b);
    if (it != nodes[cur].kids.end()) {
      cur = it->second;
    } else {
      const int n = (int)nodes.size();
      nodes.push_back(Node());
      nodes[cur].kids[b] = n;
      cur = n;
    }
  }
  nodes[cur].terminal = true;
}

int ByteTrie::child(int node, uint8_t b) const {
  if (node < 0 || node >= (int)nodes.size()) return -1;
  auto it = nodes[node].kids.find(b);
  return it == nodes[node].kids.end() ? -1 : it->second;
}

int ByteTrie::advance(int node, const std::string& bytes) const {
  for (char ch : bytes) {
    node = child(node, (uint8_t)ch);
    if (node < 0) return -1;
  }
  return node;
}

// Separators (anything not alphanumeric or '_') become single underscores, a
// lower-to-upper or acronym-to-word boundary gains one, letters are
// lowercased, and trailing underscores go (tokenizer.rs:250-292).
std::string to_snake_case(const std::string& name) {
  std::vector<uint32_t> cs;
  std::vector<std::string> raw;
  for (size_t i = 0; i < name.size();) {
    const unsigned char b = (unsigned char)name[i];
    size_t n = b < 0x80 ? 1 : b < 0xE0 ? 2 : b < 0xF0 ? 3 : 4;
    n = std::min(n, name.size() - i);
    uint32_t c = n == 1 ? b : (b & (0xFF >> (n + 1)));
    for (size_t k = 1; k < n; ++k) c = (c << 6) | ((unsigned char)name[i + k] & 0x3F);
    cs.push_back(c);
    raw.push_back(name.substr(i, n));
    i += n;
  }
  std::string out;
  bool prev_us = false, prev_up = false;
  for (size_t i = 0; i < cs.size(); ++i) {
    const uint32_t c = cs[i];
    if (is_alnum(c) || c == '_') {
      if (c == '_') {
        if (!prev_us && !out.empty()) {
          out += '_';
          prev_us = true;
        }
        prev_up = false;
      } else if (is_upper(c)) {
        const bool prev_low = i > 0 && (is_lower(cs[i - 1]) || (cs[i - 1] >= '0' && cs[i - 1] <= '9'));
        const bool next_low = i + 1 < cs.size() && is_lower(cs[i + 1]);
        if (i > 0 && !prev_us && (prev_low || (prev_up && next_low))) out += '_';
        out += (char)(c - 'A' + 'a');
        prev_us = false;
        prev_up = true;
      } else {
        out += raw[i];
        prev_us = false;
        prev_up = false;
      }
    } else {
      if (!prev_us && !out.empty()) {
        out += '_';
        prev_us = true;
      }
      prev_up = false;
    }
  }
  while (!out.empty() && out.back() == '_') out.pop_back();
  return out;
}

// A list (or a single object) of tool objects: each with a string "name" and
// argument keys from "parameters" — the keys of its "properties" object in
// JSON-Schema form, else its keys whose values are objects
// (constrained.rs:463-537).
std::vector<ToolDef> parse_tools_json(const std::string& json) {
  std::vector<ToolDef> tools;
  size_t i = 0;
  while (i < json.size() && json[i] != '[' && json[i] != '{') ++i;
  if (i >= json.size()) return tools;
  if (json[i] == '[') ++i;
  while (i < json.size()) {
    while (i < json.size() && (json[i] == ',' || ascii_ws(json[i]))) ++i;
    if (i >= json.size() || json[i] == ']') break;
    if (json[i] != '{') {
      ++i;
      continue;
    }
    const size_t end = find_matching(json, i, '{', '}');
    const std::string obj = json.substr(i, end + 1 - i);
    ToolDef t;
    if (extract_string(obj, "name", &t.name)) {
      t.snake_name = to_snake_case(t.name);
      std::string params, props;
      if (extract_object(obj, "parameters", &params))
        t.param_keys = extract_object(params, "properties", &props) ? object_keys(props, false)
                                                                     : object_keys(params, true);
      tools.push_back(std::move(t));
    }
    i = end + 1;
  }
  return tools;
}

// constrained.rs:189-283. Inside a tool name or an argument key the bytes are
// collected until the closing quote; elsewhere value strings are skipped,
// brace depth is tracked, and the recent bytes are matched against the
// triggers that open a name, the arguments object and each key.
void JsonMachine::feed_byte(uint8_t b) {
  if (state == IN_NAME) {
    if (b == '"') {
      current_function = buf;
      buf.clear();
      state = FREE;
    } else {
      buf += (char)b;
    }
    return;
  }
  if (state == IN_ARG_KEY) {
    if (b == '"') {
      if (!buf.empty() && std::find(used_keys.begin(), used_keys.end(), buf) == used_keys.end())
        used_keys.push_back(buf);
      buf.clear();
      state = FREE;
    } else {
      buf += (char)b;
    }
    return;
  }
  tail += (char)b;
  if (tail.size() > kTail) tail.erase(0, tail.size() - kTail);
  if (in_string) {
    if (prev_escape) prev_escape = false;
    else if (b == '\\') prev_escape = true;
    else if (b == '"') in_string = false;
    return;
  }
  if (b == '{' || b == '[') {
    ++nesting_depth;
  } else if (b == '}' || b == ']') {
    nesting_depth = nesting_depth ? nesting_depth - 1 : 0;
    if (b == '}' && in_arguments && nesting_depth < arguments_depth) in_arguments = false;
    return;
  }
  if (!in_arguments && ends_with(tail, kNameTrigger)) {
    state = IN_NAME;
    buf.clear();
    used_keys.clear();  // a new call starts with no keys written
    return;
  }
  if (ends_with(tail, kArgsTrigger)) {
    in_arguments = true;
    arguments_depth = nesting_depth;
    return;
  }
  const size_t n = tail.size();
  if (in_arguments && nesting_depth == arguments_depth && n >= 2 && (tail[n - 2] == '{' || tail[n - 2] == ',') &&
      tail[n - 1] == '"') {
    state = IN_ARG_KEY;
    buf.clear();
    return;
  }
  if (b == '"' && n >= 2 && tail[n - 2] == ':') in_string = true;
}

ConstrainedDecoder::ConstrainedDecoder(const std::vector<ToolDef>& tools, std::vector<std::string> token_texts,
                                       bool unique_keys)
    : texts_(std::move(token_texts)), unique_(unique_keys) {
  for (const ToolDef& t : tools) {
    names_.insert(t.snake_name);
    ByteTrie keys;
    for (const std::string& k : t.param_keys) keys.insert(k);
    key_tries_[t.snake_name] = keys;
    keys_[t.snake_name] = t.param_keys;
  }
}

void ConstrainedDecoder::update(uint32_t token) {
  if (token < texts_.size()) sm_.feed(texts_[token]);
}

// A token is allowed when its bytes walk the trie from `node`, a quote being
// allowed only at the end of a name or key (what follows it is the state
// machine's business); when no token is allowed the mask is lifted
// (constrained.rs:81-116).
std::vector<float> ConstrainedDecoder::mask_from(const ByteTrie& trie, int node, size_t vocab) const {
  std::vector<float> mask(vocab, -1e9f);
  bool any = false;
  for (size_t id = 0; id < texts_.size() && id < vocab; ++id) {
    int cur = node;
    bool ok = true;
    for (char ch : texts_[id]) {
      if (ch == '"') {
        ok = trie.nodes[cur].terminal;
        break;
      }
      cur = trie.child(cur, (uint8_t)ch);
      if (cur < 0) {
        ok = false;
        break;
      }
    }
    if (ok) {
      mask[id] = 0.f;
      any = true;
    }
  }
  if (!any) std::fill(mask.begin(), mask.end(), 0.f);
  return mask;
}

// constrained.rs:431-461: no mask outside a name or key; inside one, the
// declared names, or the current tool's keys (minus those already written in
// this call when unique keys are asked for and some remain).
std::vector<float> ConstrainedDecoder::logit_mask(size_t vocab) const {
  if (sm_.state == JsonMachine::FREE) return std::vector<float>(vocab, 0.f);
  if (sm_.state == JsonMachine::IN_NAME) {
    const int node = names_.advance(0, sm_.buf);
    return node < 0 ? std::vector<float>(vocab, 0.f) : mask_from(names_, node, vocab);
  }
  ByteTrie remaining;
  const ByteTrie* trie = nullptr;
  if (unique_) {
    auto it = keys_.find(sm_.current_function);
    if (it != keys_.end()) {
      bool any = false;
      for (const std::string& k : it->second)
        if (std::find(sm_.used_keys.begin(), sm_.used_keys.end(), k) == sm_.used_keys.end()) {
          remaining.insert(k);
          any = true;
        }
      if (any) trie = &remaining;
    }
  }
  if (!trie) {
    auto it = key_tries_.find(sm_.current_function);
    if (it == key_tries_.end()) return std::vector<float>(vocab, 0.f);
    trie = &it->second;
  }
  const int node = trie->advance(0, sm_.buf);
  return node < 0 ? std::vector<float>(vocab, 0.f) : mask_from(*trie, node, vocab);
}

}  // namespace nb
