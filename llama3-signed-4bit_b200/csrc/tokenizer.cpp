// Byte-level BPE tokenizer behind llama_tokenizer_* (src/llama_engine.h:59-62).
//
// Host code, off the GPU path.  Behaviour follows the reference's LLaMATokenizer
// (src/llama_engine.cpp:526-739): bytes map to printable code points with the GPT-2 byte table;
// text is split on single spaces (every space becomes its own token); each non-space run is
// merged pair-by-pair by lowest merge rank (one merge per round, leftmost pair among equal
// ranks); pieces missing from the vocabulary are dropped.  Decoding maps code points back to
// bytes.  The tokenizer.json reader here is a small JSON parser of its own; it reads
// model.vocab and model.merges, with merges given either as "a b" strings or as ["a", "b"] pairs.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "llama_engine.h"

#define LE_API extern "C" __attribute__((visibility("default")))

namespace {

void append_utf8(std::string& out, uint32_t cp) {
  if (cp < 0x80) {
    out += static_cast<char>(cp);
  } else if (cp < 0x800) {
    out += static_cast<char>(0xC0 | (cp >> 6));
    out += static_cast<char>(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    out += static_cast<char>(0xE0 | (cp >> 12));
    out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
    out += static_cast<char>(0x80 | (cp & 0x3F));
  } else {
    out += static_cast<char>(0xF0 | (cp >> 18));
    out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
    out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
    out += static_cast<char>(0x80 | (cp & 0x3F));
  }
}

size_t utf8_len(unsigned char c) {
  if ((c & 0xE0) == 0xC0) return 2;
  if ((c & 0xF0) == 0xE0) return 3;
  if ((c & 0xF8) == 0xF0) return 4;
  return 1;
}

// Minimal JSON reader: enough to walk tokenizer.json and pull out strings and integers.
class Json {
 public:
  explicit Json(const std::string& s) : s_(s) {}
  bool ok() const { return ok_; }

  void ws() {
    while (p_ < s_.size() && (s_[p_] == ' ' || s_[p_] == '\n' || s_[p_] == '\r' || s_[p_] == '\t')) ++p_;
  }
  bool eat(char c) {
    ws();
    if (p_ < s_.size() && s_[p_] == c) { ++p_; return true; }
    return false;
  }
  char peek() {
    ws();
    return p_ < s_.size() ? s_[p_] : '\0';
  }
  bool str(std::string& out) {
    out.clear();
    if (!eat('"')) return fail();
    while (p_ < s_.size()) {
      char c = s_[p_++];
      if (c == '"') return true;
      if (c != '\\') { out += c; continue; }
      if (p_ >= s_.size()) return fail();
      char e = s_[p_++];
      switch (e) {
        case 'n': out += '\n'; break;
        case 't': out += '\t'; break;
        case 'r': out += '\r'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'u': {
          uint32_t cp = 0;
          if (!hex4(cp)) return fail();
          if (cp >= 0xD800 && cp < 0xDC00 && p_ + 6 <= s_.size() && s_[p_] == '\\' && s_[p_ + 1] == 'u') {
            p_ += 2;
            uint32_t lo = 0;
            if (!hex4(lo)) return fail();
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          append_utf8(out, cp);
          break;
        }
        default: out += e; break;  // \" \\ \/
      }
    }
    return fail();
  }
  bool integer(int64_t& v) {
    ws();
    size_t q = p_;
    bool neg = false;
    if (q < s_.size() && s_[q] == '-') { neg = true; ++q; }
    if (q >= s_.size() || s_[q] < '0' || s_[q] > '9') return fail();
    v = 0;
    while (q < s_.size() && s_[q] >= '0' && s_[q] <= '9') v = v * 10 + (s_[q++] - '0');
    // skip fraction / exponent if any
    while (q < s_.size() && (s_[q] == '.' || s_[q] == 'e' || s_[q] == 'E' || s_[q] == '+' || s_[q] == '-' ||
                             (s_[q] >= '0' && s_[q] <= '9')))
      ++q;
    p_ = q;
    if (neg) v = -v;
    return true;
  }
  // Skips any JSON value.
  bool skip() {
    char c = peek();
    if (c == '"') { std::string t; return str(t); }
    if (c == '{') {
      eat('{');
      if (eat('}')) return true;
      do {
        std::string k;
        if (!str(k) || !eat(':') || !skip()) return fail();
      } while (eat(','));
      return eat('}') || fail();
    }
    if (c == '[') {
      eat('[');
      if (eat(']')) return true;
      do {
        if (!skip()) return fail();
      } while (eat(','));
      return eat(']') || fail();
    }
    if (c == '-' || (c >= '0' && c <= '9')) { int64_t v; return integer(v); }
    for (const char* lit : {"true", "false", "null"}) {
      size_t n = std::strlen(lit);
      if (s_.compare(p_, n, lit) == 0) { p_ += n; return true; }
    }
    return fail();
  }

 private:
  bool hex4(uint32_t& cp) {
    if (p_ + 4 > s_.size()) return false;
    cp = 0;
    for (int i = 0; i < 4; ++i) {
      char h = s_[p_++];
      cp <<= 4;
      if (h >= '0' && h <= '9') cp |= h - '0';
      else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
      else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
      else return false;
    }
    return true;
  }
  bool fail() { ok_ = false; return false; }
  const std::string& s_;
  size_t p_ = 0;
  bool ok_ = true;
};

struct PairHash {
  size_t operator()(const std::pair<std::string, std::string>& p) const {
    return std::hash<std::string>()(p.first) * 1000003u ^ std::hash<std::string>()(p.second);
  }
};

class Tokenizer {
 public:
  bool load(const std::string& path) {
    build_byte_table();
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string text = ss.str();
    Json j(text);
    if (!j.eat('{')) return false;
    if (j.eat('}')) return false;
    do {
      std::string key;
      if (!j.str(key) || !j.eat(':')) return false;
      if (key == "model") {
        if (!read_model(j)) return false;
      } else if (!j.skip()) {
        return false;
      }
    } while (j.eat(','));
    return j.ok() && !vocab_.empty();
  }

  std::vector<int32_t> encode(const std::string& text) const {
    std::vector<int32_t> ids;
    size_t i = 0;
    while (i < text.size()) {
      if (text[i] == ' ') {
        auto it = vocab_.find(byte_to_cp_str_[static_cast<unsigned char>(' ')]);
        if (it != vocab_.end()) ids.push_back(it->second);
        ++i;
        continue;
      }
      size_t j = i;
      while (j < text.size() && text[j] != ' ') ++j;
      std::string mapped;
      for (size_t k = i; k < j; ++k) mapped += byte_to_cp_str_[static_cast<unsigned char>(text[k])];
      for (const auto& piece : merge(mapped)) {
        auto it = vocab_.find(piece);
        if (it != vocab_.end()) ids.push_back(it->second);
      }
      i = j;
    }
    return ids;
  }

  std::string decode(int32_t id) const {
    auto it = id_to_piece_.find(id);
    if (it == id_to_piece_.end()) return "";
    const std::string& s = it->second;
    std::string out;
    for (size_t i = 0; i < s.size();) {
      size_t n = utf8_len(static_cast<unsigned char>(s[i]));
      std::string ch = s.substr(i, n);
      auto b = cp_str_to_byte_.find(ch);
      if (b != cp_str_to_byte_.end()) out += static_cast<char>(b->second);
      else out += ch;
      i += n;
    }
    return out;
  }

  std::string last;

 private:
  void build_byte_table() {
    std::vector<int> printable;
    for (int b = '!'; b <= '~'; ++b) printable.push_back(b);
    for (int b = 161; b <= 172; ++b) printable.push_back(b);
    for (int b = 174; b <= 255; ++b) printable.push_back(b);
    std::vector<bool> is_printable(256, false);
    for (int b : printable) is_printable[b] = true;
    int extra = 0;
    for (int b = 0; b < 256; ++b) {
      uint32_t cp = is_printable[b] ? (uint32_t)b : (uint32_t)(256 + extra++);
      std::string u;
      append_utf8(u, cp);
      byte_to_cp_str_[b] = u;
      cp_str_to_byte_[u] = static_cast<uint8_t>(b);
    }
  }

  bool read_model(Json& j) {
    if (!j.eat('{')) return false;
    if (j.eat('}')) return true;
    do {
      std::string key;
      if (!j.str(key) || !j.eat(':')) return false;
      if (key == "vocab") {
        if (!j.eat('{')) return false;
        if (!j.eat('}')) {
          do {
            std::string piece;
            int64_t id;
            if (!j.str(piece) || !j.eat(':') || !j.integer(id)) return false;
            vocab_[piece] = (int32_t)id;
            id_to_piece_[(int32_t)id] = piece;
          } while (j.eat(','));
          if (!j.eat('}')) return false;
        }
      } else if (key == "merges") {
        if (!j.eat('[')) return false;
        int32_t rank = 0;
        if (!j.eat(']')) {
          do {
            std::string a, b;
            if (j.peek() == '[') {
              j.eat('[');
              if (!j.str(a) || !j.eat(',') || !j.str(b) || !j.eat(']')) return false;
            } else {
              std::string m;
              if (!j.str(m)) return false;
              size_t sp = m.find(' ');
              if (sp == std::string::npos) continue;  // not a pair: ignored, rank not consumed
              a = m.substr(0, sp);
              b = m.substr(sp + 1);
            }
            ranks_[std::make_pair(a, b)] = rank++;  // a repeated pair keeps its last rank
          } while (j.eat(','));
          if (!j.eat(']')) return false;
        }
      } else if (!j.skip()) {
        return false;
      }
    } while (j.eat(','));
    return j.eat('}');
  }

  std::vector<std::string> merge(const std::string& s) const {
    std::vector<std::string> w;
    for (size_t i = 0; i < s.size();) {
      size_t n = utf8_len(static_cast<unsigned char>(s[i]));
      w.push_back(s.substr(i, n));
      i += n;
    }
    while (w.size() > 1) {
      int32_t best = INT32_MAX;
      size_t at = SIZE_MAX;
      for (size_t i = 0; i + 1 < w.size(); ++i) {
        auto it = ranks_.find({w[i], w[i + 1]});
        if (it != ranks_.end() && it->second < best) { best = it->second; at = i; }
      }
      if (at == SIZE_MAX) break;
      w[at] += w[at + 1];
      w.erase(w.begin() + (long)at + 1);
    }
    return w;
  }

  std::string byte_to_cp_str_[256];
  std::unordered_map<std::string, uint8_t> cp_str_to_byte_;
  std::unordered_map<std::string, int32_t> vocab_;
  std::unordered_map<int32_t, std::string> id_to_piece_;
  std::unordered_map<std::pair<std::string, std::string>, int32_t, PairHash> ranks_;
};

}  // namespace

LE_API llama_tokenizer_t llama_tokenizer_create(const char* tokenizer_path) {
  if (!tokenizer_path) return nullptr;
  auto* t = new Tokenizer();
  if (!t->load(tokenizer_path)) {
    delete t;
    return nullptr;
  }
  return t;
}

LE_API void llama_tokenizer_free(llama_tokenizer_t tokenizer) { delete static_cast<Tokenizer*>(tokenizer); }

LE_API int llama_tokenizer_encode(llama_tokenizer_t tokenizer, const char* text, int32_t* out_tokens, int max_tokens) {
  if (!tokenizer || !text || !out_tokens || max_tokens <= 0) return 0;
  auto ids = static_cast<Tokenizer*>(tokenizer)->encode(text);
  int n = (int)std::min<size_t>((size_t)max_tokens, ids.size());
  for (int i = 0; i < n; ++i) out_tokens[i] = ids[i];
  return n;
}

LE_API const char* llama_tokenizer_decode(llama_tokenizer_t tokenizer, int32_t token_id) {
  if (!tokenizer) return "";
  auto* t = static_cast<Tokenizer*>(tokenizer);
  t->last = t->decode(token_id);
  return t->last.c_str();
}
