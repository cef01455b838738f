// Byte-level BPE tokenizer behind llama_tokenizer_* (src/llama_engine.h:59-62).
//
// Host code, off the GPU path.  Behaviour follows the reference's LLaMATokenizer
// (src/llama_engine.cpp:526-739) exactly, including how it reads tokenizer.json:
// * the vocabulary is the run of "piece": id entries between the first `"vocab": {` and the
//   following `"merges": [` of the file; in a piece only the escapes \" and \\ are undone
//   (every other backslash sequence stays as written, :594-603);
// * merges are the quoted strings from there to the file's last `]`, taken verbatim (no escape
//   is undone), split at their first space; strings without a space are skipped and consume no
//   rank, and a repeated pair keeps its last rank (:623-647);
// * bytes map to printable code points with the GPT-2 byte table; text is split on single
//   spaces (every space becomes its own token); each non-space run is merged pair by pair by
//   lowest merge rank (one merge per round, leftmost pair among equal ranks); pieces missing from
//   the vocabulary are dropped; decoding maps code points back to bytes.
// The scanning code here is this library's own; it keeps those rules because a drop-in must
// produce the same ids from the same tokenizer.json.
#include <algorithm>
#include <cctype>
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

// End of the quoted string whose opening quote is at q1: the next quote before `limit` that is
// preceded by an even number of backslashes; `limit` when there is none.
size_t quote_end(const std::string& s, size_t q1, size_t limit) {
  size_t q2 = q1 + 1;
  for (; q2 < limit; ++q2) {
    if (s[q2] != '"') continue;
    size_t bs = 0;
    for (size_t k = q2; k > q1 && s[k - 1] == '\\'; --k) ++bs;
    if (bs % 2 == 0) break;
  }
  return q2;
}

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
    const size_t npos = std::string::npos;
    const size_t vb = text.find("\"vocab\": {");
    const size_t mb = text.find("\"merges\": [", vb);
    if (vb != npos && mb != npos) read_vocab(text, vb + 10, mb);
    if (mb != npos) read_merges(text, mb + 11, text.rfind(']'));
    return true;  // like the reference: a file without these sections gives an empty tokenizer
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

  // "piece": id entries in [cur, end)
  void read_vocab(const std::string& t, size_t cur, size_t end) {
    while (cur < end) {
      const size_t q1 = t.find('"', cur);
      if (q1 == std::string::npos || q1 >= end) return;
      const size_t q2 = quote_end(t, q1, end);
      if (q2 >= end) return;
      std::string piece;
      for (size_t i = q1 + 1; i < q2; ++i) {
        if (t[i] == '\\' && i + 1 < q2 && (t[i + 1] == '"' || t[i + 1] == '\\')) {
          piece += t[++i];
          continue;
        }
        piece += t[i];
      }
      const size_t colon = t.find(':', q2);
      if (colon == std::string::npos || colon >= end) return;
      size_t d0 = colon + 1;
      while (d0 < end && !std::isdigit(static_cast<unsigned char>(t[d0]))) ++d0;
      size_t d1 = d0;
      int32_t id = 0;
      for (; d1 < end && std::isdigit(static_cast<unsigned char>(t[d1])); ++d1) id = id * 10 + (t[d1] - '0');
      if (d1 > d0) {
        vocab_[piece] = id;
        id_to_piece_[id] = piece;
      }
      cur = d1;
    }
  }

  // quoted "a b" strings in [cur, end), verbatim
  void read_merges(const std::string& t, size_t cur, size_t end) {
    if (end == std::string::npos) return;
    int32_t rank = 0;
    while (cur < end) {
      const size_t q1 = t.find('"', cur);
      if (q1 == std::string::npos || q1 >= end) return;
      const size_t q2 = quote_end(t, q1, end);
      if (q2 >= end) return;
      const std::string m = t.substr(q1 + 1, q2 - q1 - 1);
      const size_t sp = m.find(' ');
      if (sp != std::string::npos) ranks_[std::make_pair(m.substr(0, sp), m.substr(sp + 1))] = rank++;
      cur = q2 + 1;
    }
  }

  std::vector<std::string> merge(const std::string& s) const {
    std::vector<std::string> w;
    for (size_t i = 0; i < s.size();) {
      size_t n = utf8_len(static_cast<unsigned char>(s[i]));
      w.push_back(s.substr(i, n));
      i += n;
    }
    while (w.size() > 1) {
      int32_t best = 1000000000;  // ranks at or above 1e9 never merge (src/llama_engine.cpp:668)
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
