// ec_tokenizer.cu -- tokenizer.lisp in C++ (host code): WordPiece, byte-level
// BPE and Unigram behind the C ABI, so a host can turn texts into the token
// ids ec_embed_batch takes at the rates the GPU consumes them.
//
// The pipeline is tk-encode's (tokenizer.lisp:201-244): optional lowercase
// -> pre-tokenizer -> model -> truncation to max-len - 2 -> BOS / CLS / body
// / SEP / EOS.  Text is decoded from UTF-8 into code points and every step
// works on code points, as the Lisp works on characters:
//   * whitespace-p, punctuation-p (:30-43) are restated as code-point tests;
//     alpha-char-p / digit-char-p / sb-unicode:lowercase come from
//     ec_unicode_tables.h (general category L*, Nd, the full lowercase
//     mapping; final sigma: a capital sigma after a letter and not before
//     one lowers to the final form);
//   * pretokenize-wordpiece (:258-270), pretokenize-gpt2 (:280-327),
//     pretokenize-llama3 (:329-377) and pretokenize-metaspace (:386-391) are
//     hand-written scanners with the same branches in the same order;
//   * wordpiece-tokenize-word (:395-415): greedy longest match with "##",
//     words over 100 characters -> the unknown token, and the match advances
//     by the matched piece's length including the "##" (as the Lisp does);
//   * bpe-merge (:417-434): repeatedly merge the adjacent pair of lowest rank
//     (leftmost among equal ranks) over byte-level mapped characters
//     (bytes_to_unicode, :74-93);
//   * unigram-viterbi (:436-458): best-score segmentation over pieces of up to
//     20 characters, scores added in double; tk-encode then looks its ids up
//     in the string-keyed vocabulary, so each piece comes out as the unknown
//     token's id (reproduced).
// Loading follows make-tokenizer (:119-197) and make-tokenizer-from-json
// (:515-552) including json-specials (:465-498) and pretok-mode (:500-513).
// Tokenizers are read-only after loading, so batches are encoded on several
// host threads.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <new>
#include <sstream>
#include <stdexcept>
#include <string>
#include <system_error>
#include <thread>
#include <unordered_map>
#include <vector>

#include "ec_json.h"
#include "ec_state.h"
#include "ec_unicode_tables.h"

namespace ec {
namespace tok {
namespace {

using U32 = std::u32string;

// ---------------------------------------------------------------- unicode --
template <size_t N>
bool in_ranges(const uni::Range (&r)[N], uint32_t cp) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (r[mid].hi < cp) lo = mid + 1;
    else hi = mid;
  }
  return lo < N && r[lo].lo <= cp && cp <= r[lo].hi;
}

bool whitespace_p(char32_t c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == 0x0C; }
bool punctuation_p(char32_t c) {
  return (c >= 33 && c <= 47) || (c >= 58 && c <= 64) || (c >= 91 && c <= 96) ||
         (c >= 123 && c <= 126) || (c >= 0x2000 && c <= 0x206F) || (c >= 0x3000 && c <= 0x303F);
}
bool alpha_p(char32_t c) {
  if (c < 128) return (c | 32) >= 'a' && (c | 32) <= 'z';
  return in_ranges(uni::kLetters, c);
}
bool digit_p(char32_t c) {
  if (c < 128) return c >= '0' && c <= '9';
  return in_ranges(uni::kDigits, c);
}

void lower_into(char32_t c, U32& out) {
  if (c < 128) {
    out.push_back(c >= 'A' && c <= 'Z' ? c + 32 : c);
    return;
  }
  for (const uni::MapN& m : uni::kLowerN)
    if (m.from == c) {
      for (uint32_t k = 0; k < m.n; ++k) out.push_back(m.to[k]);
      return;
    }
  const uni::Map1* b = std::begin(uni::kLower1);
  const uni::Map1* e = std::end(uni::kLower1);
  const uni::Map1* it = std::lower_bound(b, e, static_cast<uint32_t>(c),
                                         [](const uni::Map1& m, uint32_t v) { return m.from < v; });
  out.push_back(it != e && it->from == c ? it->to : c);
}

U32 lowercase(const U32& s) {
  U32 out;
  out.reserve(s.size());
  for (size_t i = 0; i < s.size(); ++i) {
    if (s[i] == 0x03A3) {
      const bool prev = i > 0 && alpha_p(s[i - 1]);
      const bool next = i + 1 < s.size() && alpha_p(s[i + 1]);
      out.push_back(prev && !next ? 0x03C2 : 0x03C3);
    } else {
      lower_into(s[i], out);
    }
  }
  return out;
}

// UTF-8 <-> code points; malformed UTF-8 is rejected (the Lisp reads texts
// through a UTF-8 external format, which signals on malformed input)
bool utf8_decode(const char* p, size_t n, U32& out) {
  out.clear();
  out.reserve(n);
  size_t i = 0;
  while (i < n) {
    const unsigned char c = static_cast<unsigned char>(p[i]);
    uint32_t cp;
    int len;
    if (c < 0x80) { cp = c; len = 1; }
    else if ((c >> 5) == 6) { cp = c & 0x1F; len = 2; }
    else if ((c >> 4) == 14) { cp = c & 0x0F; len = 3; }
    else if ((c >> 3) == 30) { cp = c & 0x07; len = 4; }
    else return false;
    if (i + len > n) return false;
    for (int k = 1; k < len; ++k) {
      const unsigned char cc = static_cast<unsigned char>(p[i + k]);
      if ((cc >> 6) != 2) return false;
      cp = (cp << 6) | (cc & 0x3F);
    }
    out.push_back(cp);
    i += len;
  }
  return true;
}

void utf8_append(char32_t cp, std::string& out) {
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

std::string utf8(const U32& s, size_t b = 0, size_t e = std::u32string::npos) {
  std::string out;
  if (e > s.size()) e = s.size();
  out.reserve(e - b);
  for (size_t i = b; i < e; ++i) utf8_append(s[i], out);
  return out;
}

// GPT-2 bytes_to_unicode: printable bytes keep their code, the rest shift
// into 256.. in byte order (tokenizer.lisp:74-86)
struct ByteMap {
  char32_t to[256];
  ByteMap() {
    int n = 0;
    for (int b = 0; b < 256; ++b) {
      const bool keep = (b >= 33 && b <= 126 && b != 92) || (b >= 161 && b <= 172) || (b >= 174);
      to[b] = keep ? static_cast<char32_t>(b) : static_cast<char32_t>(256 + n++);
    }
  }
};
const ByteMap& byte_map() {
  static const ByteMap m;
  return m;
}

// ----------------------------------------------------------- tokenizer ---
enum Kind { kWordPiece, kBpe, kUnigram };

struct Tokenizer {
  Kind kind = kWordPiece;
  std::unordered_map<std::string, int> vocab;
  std::vector<std::string> inv;
  std::unordered_map<std::string, int> merges;  // "a\x01b" -> rank
  std::vector<std::pair<std::string, std::string>> merge_list;  // (a, b) in file order
  std::unordered_map<std::string, double> scores;
  bool lowercase = true;
  int max_len = 512;
  std::string cls = "[CLS]", sep = "[SEP]", unk = "[UNK]";
  bool byte_level = false;
  bool llama3 = false;
  int bos = -1, eos = -1;  // -1: none

  int id_of(const std::string& t) const {
    auto it = vocab.find(t);
    return it == vocab.end() ? -1 : it->second;
  }

  // WordPiece: byte tries of every token (root 0: the candidates of a word's
  // first piece are matched as they are) and of the "##" tokens without the
  // "##" (root 1: continuation candidates); edge (node << 8 | byte) -> child
  // while building, node -> id of the token ending there (-1: none).  For
  // matching, the two roots get direct 256-entry child tables and every other
  // node its children as a byte-sorted run (few children each).
  std::unordered_map<uint64_t, int> edge;
  std::vector<int> node_id;
  std::vector<int> root_child;            // [2 * 256]
  std::vector<uint32_t> kid_off;          // [nodes + 1]
  std::vector<unsigned char> kid_byte;
  std::vector<int> kid_node;
  // BPE on integers: every vocabulary and merge string interned as a symbol;
  // (left, right) -> (rank, merged symbol) with the rank merges[] gives the
  // pair's string key; characters without a symbol take part in no merge and
  // have no id
  std::unordered_map<std::string, int> sym;
  std::vector<int> sym_id;                                 // vocab id or -1
  std::unordered_map<uint64_t, std::pair<int, int>> pair_rank;
  std::vector<int> char_sym;                               // code points < 0x10000
  int intern(const std::string& str) {
    auto it = sym.find(str);
    if (it != sym.end()) return it->second;
    const int s = static_cast<int>(sym_id.size());
    sym.emplace(str, s);
    auto v = vocab.find(str);
    sym_id.push_back(v == vocab.end() ? -1 : v->second);
    return s;
  }
  void add_merge(const std::string& a, const std::string& b, int rank);
  void build_bpe();
  int symbol_of(char32_t c) const;
  int child(int node, unsigned char b) const {
    if (node < 2) return root_child[static_cast<size_t>(node) * 256 + b];
    const uint32_t e = kid_off[static_cast<size_t>(node) + 1];
    for (uint32_t i = kid_off[static_cast<size_t>(node)]; i < e; ++i)
      if (kid_byte[i] >= b) return kid_byte[i] == b ? kid_node[i] : -1;
    return -1;
  }
  void trie_insert(int root, const std::string& t, size_t from, int id) {
    int node = root;
    for (size_t b = from; b < t.size(); ++b) {
      const uint64_t key = (static_cast<uint64_t>(node) << 8) | static_cast<unsigned char>(t[b]);
      auto it = edge.find(key);
      if (it == edge.end()) {
        node_id.push_back(-1);
        node = static_cast<int>(node_id.size()) - 1;
        edge.emplace(key, node);
      } else {
        node = it->second;
      }
    }
    if (node > 1) node_id[static_cast<size_t>(node)] = id;
  }
  void build_trie() {
    edge.clear();
    node_id.assign(2, -1);
    for (const auto& kv : vocab) {
      trie_insert(0, kv.first, 0, kv.second);
      if (kv.first.size() > 2 && kv.first[0] == '#' && kv.first[1] == '#')
        trie_insert(1, kv.first, 2, kv.second);
    }
    // flatten: (parent, byte, child) sorted by parent then byte
    std::vector<std::pair<uint64_t, int>> es(edge.begin(), edge.end());
    std::sort(es.begin(), es.end());
    const size_t nn = node_id.size();
    root_child.assign(2 * 256, -1);
    kid_off.assign(nn + 1, 0);
    kid_byte.clear();
    kid_node.clear();
    for (const auto& e : es) {
      const size_t parent = static_cast<size_t>(e.first >> 8);
      const unsigned char b = static_cast<unsigned char>(e.first & 0xff);
      if (parent < 2) {
        root_child[parent * 256 + b] = e.second;
      } else {
        ++kid_off[parent + 1];
        kid_byte.push_back(b);
        kid_node.push_back(e.second);
      }
    }
    for (size_t i = 0; i < nn; ++i) kid_off[i + 1] += kid_off[i];
    edge.clear();
  }
};

std::string merge_key(const std::string& a, const std::string& b) {
  std::string k;
  k.reserve(a.size() + b.size() + 1);
  k += a;
  k += '\x01';
  k += b;
  return k;
}

void Tokenizer::add_merge(const std::string& a, const std::string& b, int rank) {
  merges[merge_key(a, b)] = rank;
  merge_list.emplace_back(a, b);
}

void Tokenizer::build_bpe() {
  sym.clear();
  sym_id.clear();
  pair_rank.clear();
  for (const auto& kv : vocab) intern(kv.first);
  for (const auto& m : merge_list) {
    const int a = intern(m.first), b = intern(m.second);
    const int ab = intern(m.first + m.second);
    pair_rank[(static_cast<uint64_t>(a) << 32) | static_cast<uint32_t>(b)] =
        std::make_pair(merges.at(merge_key(m.first, m.second)), ab);
  }
  char_sym.assign(0x10000, -1);
  std::string u;
  for (uint32_t c = 0; c < 0x10000; ++c) {
    u.clear();
    utf8_append(static_cast<char32_t>(c), u);
    auto it = sym.find(u);
    if (it != sym.end()) char_sym[c] = it->second;
  }
}

int Tokenizer::symbol_of(char32_t c) const {
  if (c < 0x10000) return char_sym[c];
  std::string u;
  utf8_append(c, u);
  auto it = sym.find(u);
  return it == sym.end() ? -1 : it->second;
}

std::vector<U32> split_spaces(const U32& s) {
  std::vector<U32> out;
  size_t start = 0;
  for (size_t i = 0; i < s.size(); ++i)
    if (whitespace_p(s[i])) {
      if (i > start) out.emplace_back(s, start, i - start);
      start = i + 1;
    }
  if (s.size() > start) out.emplace_back(s, start, s.size() - start);
  return out;
}

// pretokenize-gpt2 / pretokenize-llama3: same branches, same order
// the pieces as (start, length) spans of s, in order
using Spans = std::vector<std::pair<size_t, size_t>>;
void pretokenize_bytelevel(const U32& s, bool llama3, Spans& out) {
  static const char* kContr[] = {"s", "t", "m", "d", "re", "ve", "ll"};
  out.clear();
  const size_t n = s.size();
  auto alpha_at = [&](size_t j) { return j < n && alpha_p(s[j]); };
  auto digit_at = [&](size_t j) { return j < n && digit_p(s[j]); };
  auto punct_at = [&](size_t j) {
    return j < n && !whitespace_p(s[j]) && !alpha_p(s[j]) && !digit_p(s[j]);
  };
  size_t i = 0;
  while (i < n) {
    const char32_t c = s[i];
    if (c == '\'' && i + 1 < n) {
      const size_t rl = std::min(n, i + 3) - (i + 1);
      int m = -1;
      for (int q = 0; q < 7 && m < 0; ++q) {
        const size_t L = std::strlen(kContr[q]);
        if (L > rl) continue;
        bool eq = true;
        for (size_t k = 0; k < L; ++k) eq = eq && s[i + 1 + k] == static_cast<char32_t>(kContr[q][k]);
        if (eq) m = q;
      }
      if (m >= 0) {
        const size_t L = std::strlen(kContr[m]);
        out.emplace_back(i, 1 + L);
        i += 1 + L;
      } else {
        out.emplace_back(i, 1);
        i += 1;
      }
      continue;
    }
    if (!llama3 ? (alpha_at(i) || (c == ' ' && alpha_at(i + 1)))
                : (alpha_at(i) || (c != '\r' && c != '\n' && !digit_at(i) && alpha_at(i + 1)))) {
      size_t k = !llama3 ? (c == ' ' ? i + 1 : i) : (alpha_at(i) ? i : i + 1);
      while (alpha_at(k)) ++k;
      out.emplace_back(i, k - i);
      i = k;
      continue;
    }
    if (!llama3 && (digit_at(i) || (c == ' ' && digit_at(i + 1)))) {
      size_t k = c == ' ' ? i + 1 : i;
      while (digit_at(k)) ++k;
      out.emplace_back(i, k - i);
      i = k;
      continue;
    }
    if (llama3 && digit_at(i)) {
      out.emplace_back(i, 1);
      i += 1;
      continue;
    }
    if (punct_at(i) || (c == ' ' && punct_at(i + 1))) {
      size_t k = c == ' ' ? i + 1 : i;
      while (punct_at(k)) ++k;
      out.emplace_back(i, k - i);
      i = k;
      continue;
    }
    size_t k = i;
    while (k < n && whitespace_p(s[k])) ++k;
    out.emplace_back(i, k - i);
    i = k;
  }
}

std::vector<U32> pretokenize_metaspace(const U32& s) {
  std::vector<U32> out = split_spaces(s);
  for (size_t i = 1; i < out.size(); ++i) out[i].insert(out[i].begin(), ' ');
  return out;
}

// ids of one word's pieces (-1: the unknown token's name, whose id may not
// exist); the word is w[0..len).  The greedy longest match is one walk down
// the byte trie from each start, remembering the last complete piece.
void wordpiece_word(const Tokenizer& tk, const char32_t* w, size_t len, std::vector<int>& out) {
  if (len > 100) {
    out.push_back(-1);
    return;
  }
  thread_local std::string u8;
  thread_local std::vector<size_t> bo;
  u8.clear();
  bo.assign(1, 0);
  for (size_t i = 0; i < len; ++i) {
    utf8_append(w[i], u8);
    bo.push_back(u8.size());
  }
  size_t start = 0;
  while (start < len) {
    int node = start == 0 ? 0 : 1;
    int best_id = -1;
    size_t best_end = start;
    size_t c = start;
    for (size_t b = bo[start]; b < u8.size(); ++b) {
      node = tk.child(node, static_cast<unsigned char>(u8[b]));
      if (node < 0) break;
      if (b + 1 == bo[c + 1]) {  // a character boundary: a piece may end here
        ++c;
        const int id = tk.node_id[static_cast<size_t>(node)];
        if (id >= 0) {
          best_id = id;
          best_end = c;
        }
      }
    }
    if (best_id >= 0) {
      // the Lisp advances by (length found): the characters matched, plus 2
      // for the "##" of a continuation piece
      start += (best_end - start) + (start > 0 ? 2 : 0);
      out.push_back(best_id);
    } else {
      out.push_back(-1);
      start = len;
    }
  }
}

// wordpiece_word for an ASCII word (every byte a character)
void wordpiece_word_ascii(const Tokenizer& tk, const unsigned char* w, size_t len, std::vector<int>& out) {
  if (len > 100) {
    out.push_back(-1);
    return;
  }
  size_t start = 0;
  while (start < len) {
    int node = start == 0 ? 0 : 1;
    int best_id = -1;
    size_t best_end = start;
    for (size_t b = start; b < len; ++b) {
      node = tk.child(node, w[b]);
      if (node < 0) break;
      const int id = tk.node_id[static_cast<size_t>(node)];
      if (id >= 0) {
        best_id = id;
        best_end = b + 1;
      }
    }
    if (best_id >= 0) {
      start += (best_end - start) + (start > 0 ? 2 : 0);
      out.push_back(best_id);
    } else {
      out.push_back(-1);
      start = len;
    }
  }
}

// ids of the merged parts (-1: not in the vocabulary)
void bpe_word(const Tokenizer& tk, const char32_t* word, size_t len, std::vector<int>& out) {
  // the parts as symbols (-1: a character with no symbol)
  thread_local std::vector<int> parts;
  thread_local std::vector<int> rank;
  parts.clear();
  for (size_t i = 0; i < len; ++i) parts.push_back(tk.symbol_of(word[i]));
  // rank of each adjacent pair (-1: none), recomputed only next to a merge;
  // merged[i]: the symbol a merge of pair i makes
  thread_local std::vector<int> merged;
  auto rank_of = [&](size_t i) {
    merged[i] = -1;
    if (parts[i] < 0 || parts[i + 1] < 0) return -1;
    auto it = tk.pair_rank.find((static_cast<uint64_t>(parts[i]) << 32) | static_cast<uint32_t>(parts[i + 1]));
    if (it == tk.pair_rank.end()) return -1;
    merged[i] = it->second.second;
    return it->second.first;
  };
  const size_t np = parts.empty() ? 0 : parts.size() - 1;
  rank.assign(np, -1);
  merged.assign(np, -1);
  for (size_t i = 0; i < np; ++i) rank[i] = rank_of(i);
  while (parts.size() > 1) {
    int best = -1;
    size_t bi = 0;
    for (size_t i = 0; i + 1 < parts.size(); ++i)
      if (rank[i] >= 0 && (best < 0 || rank[i] < best)) {
        best = rank[i];
        bi = i;
      }
    if (best < 0) break;
    parts[bi] = merged[bi];
    parts.erase(parts.begin() + static_cast<long>(bi) + 1);
    rank.erase(rank.begin() + static_cast<long>(bi));
    merged.erase(merged.begin() + static_cast<long>(bi));
    if (bi < rank.size()) rank[bi] = rank_of(bi);
    if (bi > 0) rank[bi - 1] = rank_of(bi - 1);
  }
  for (const int p : parts) out.push_back(p >= 0 ? tk.sym_id[static_cast<size_t>(p)] : -1);
}

bool unigram_word(const Tokenizer& tk, const U32& s, std::vector<int>& ids) {
  const size_t len = s.size();
  std::vector<double> best(len + 1, -1.7976931348623157e308);
  std::vector<long> back(len + 1, -1);
  best[0] = 0.0;
  for (size_t i = 0; i < len; ++i)
    for (size_t j = i + 1; j <= std::min(len, i + 20); ++j) {
      auto it = tk.scores.find(utf8(s, i, j));
      if (it == tk.scores.end()) continue;
      const double cand = best[i] + it->second;
      if (cand > best[j]) {
        best[j] = cand;
        back[j] = static_cast<long>(i);
      }
    }
  std::vector<int> rev;
  size_t j = len;
  while (j > 0) {
    if (back[j] < 0) return false;  // no segmentation (the Lisp signals an error)
    const size_t i = static_cast<size_t>(back[j]);
    const int id = tk.id_of(utf8(s, i, j));
    if (id < 0) return false;
    rev.push_back(id);
    j = i;
  }
  ids.insert(ids.end(), rev.rbegin(), rev.rend());
  return true;
}

// tk-encode; false when a token has no id and there is no unknown token
bool finish(const Tokenizer& tk, const std::vector<int>& pid, size_t keep, std::vector<int32_t>& out);

bool encode(const Tokenizer& tk, const char* text, size_t n, std::vector<int32_t>& out) {
  thread_local U32 raw, s;
  thread_local std::vector<int> pid;
  const size_t keep = static_cast<size_t>(std::max(0, tk.max_len - 2));
  bool ascii = tk.kind == kWordPiece;
  for (size_t i = 0; ascii && i < n; ++i) ascii = static_cast<unsigned char>(text[i]) < 0x80;
  if (ascii) {
    // the same pieces as below for a pure-ASCII text, on its bytes: ASCII
    // lowering, whitespace runs split, punctuation single pieces
    thread_local std::string low;
    low.assign(text, n);
    if (tk.lowercase)
      for (char& c : low)
        if (c >= 'A' && c <= 'Z') c = static_cast<char>(c + 32);
    const unsigned char* p = reinterpret_cast<const unsigned char*>(low.data());
    pid.clear();
    size_t start = 0;
    bool full = false;
    auto piece = [&](size_t b, size_t len) {
      if (pid.size() >= keep) {
        full = true;
        return;
      }
      wordpiece_word_ascii(tk, p + b, len, pid);
    };
    for (size_t i = 0; i < n && !full; ++i) {
      if (whitespace_p(p[i])) {
        if (i > start) piece(start, i - start);
        start = i + 1;
      } else if (punctuation_p(p[i])) {
        if (i > start) piece(start, i - start);
        if (!full) piece(i, 1);
        start = i + 1;
      }
    }
    if (!full && n > start) piece(start, n - start);
    return finish(tk, pid, keep, out);
  }
  if (!utf8_decode(text, n, raw)) return false;
  if (tk.lowercase) s = lowercase(raw);
  else s.swap(raw);
  // piece ids before the unknown-token substitution (-1: no id); pieces past
  // the truncation point cannot change the result for WordPiece and BPE, so
  // their words are skipped (unigram words are all scanned: the Lisp signals
  // on a word it cannot segment anywhere in the text)
  pid.clear();
  if (tk.kind == kWordPiece) {
    // pretokenize-wordpiece's pieces, in order, as spans of s: runs between
    // whitespace, each punctuation character a piece of its own
    const char32_t* p = s.data();
    const size_t n = s.size();
    size_t start = 0;
    bool full = false;
    auto piece = [&](size_t b, size_t len) {
      if (pid.size() >= keep) {
        full = true;
        return;
      }
      wordpiece_word(tk, p + b, len, pid);
    };
    for (size_t i = 0; i < n && !full; ++i) {
      if (whitespace_p(p[i])) {
        if (i > start) piece(start, i - start);
        start = i + 1;
      } else if (punctuation_p(p[i])) {
        if (i > start) piece(start, i - start);
        if (!full) piece(i, 1);
        start = i + 1;
      }
    }
    if (!full && n > start) piece(start, n - start);
  } else if (tk.kind == kBpe) {
    thread_local Spans spans;
    pretokenize_bytelevel(s, tk.llama3, spans);
    for (const auto& sp : spans) {
      if (pid.size() >= keep) break;
      const char32_t* w = s.data() + sp.first;
      if (tk.byte_level) {
        thread_local std::string b;
        thread_local U32 mapped;
        b.clear();
        for (size_t i = 0; i < sp.second; ++i) utf8_append(w[i], b);
        mapped.clear();
        const ByteMap& bm = byte_map();
        for (unsigned char ch : b) mapped.push_back(bm.to[ch]);
        bpe_word(tk, mapped.data(), mapped.size(), pid);
      } else {
        bpe_word(tk, w, sp.second, pid);
      }
    }
  } else {
    // unigram-viterbi returns ids, which tk-encode then looks up in the
    // string-keyed vocabulary (tokenizer.lisp:228): every piece becomes the
    // unknown token
    std::vector<int> uni;
    for (const U32& w : pretokenize_metaspace(s))
      if (!unigram_word(tk, w, uni)) return false;
    pid.assign(uni.size(), -1);
  }
  return finish(tk, pid, keep, out);
}

// specials around the first `keep` piece ids, unknown pieces -> the unknown
// token (false: an unknown piece and no unknown token)
bool finish(const Tokenizer& tk, const std::vector<int>& pid, size_t keep, std::vector<int32_t>& out) {
  const size_t nb = std::min(pid.size(), keep);
  const int unk = tk.id_of(tk.unk), cls = tk.id_of(tk.cls), sep = tk.id_of(tk.sep);
  out.clear();
  out.reserve(nb + 4);
  if (tk.bos >= 0) out.push_back(tk.bos);
  if (cls >= 0) out.push_back(cls);
  for (size_t i = 0; i < nb; ++i) {
    const int id = pid[i] >= 0 ? pid[i] : unk;
    if (id < 0) return false;
    out.push_back(id);
  }
  if (sep >= 0) out.push_back(sep);
  if (tk.eos >= 0) out.push_back(tk.eos);
  return true;
}

// ------------------------------------------------------------- loading ---
int read_file(const char* path, std::string& out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return set_error(EC_EINVAL, "cannot open %s", path);
  std::ostringstream ss;
  ss << f.rdbuf();
  out = ss.str();
  return EC_OK;
}

int parse_json(const char* path, JVal& v) {
  std::string text;
  int rc = read_file(path, text);
  if (rc) return rc;
  std::string err;
  JParser p(text);
  if (!p.parse(v, err)) return set_error(EC_EINVAL, "%s: %s", path, err.c_str());
  return EC_OK;
}

// read-line over the whole file
std::vector<std::string> file_lines(const std::string& text) {
  std::vector<std::string> lines;
  size_t s = 0;
  while (s < text.size()) {
    size_t e = text.find('\n', s);
    if (e == std::string::npos) e = text.size();
    lines.push_back(text.substr(s, e - s));
    s = e + 1;
  }
  return lines;
}

std::string trim_cr_space(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && (s[a] == '\r' || s[a] == ' ')) ++a;
  while (b > a && (s[b - 1] == '\r' || s[b - 1] == ' ')) --b;
  return s.substr(a, b - a);
}

constexpr int kMaxVocabId = 1 << 24;

void build_inv(Tokenizer& t) {
  int maxid = -1;
  for (auto& kv : t.vocab) maxid = std::max(maxid, kv.second);
  t.inv.assign(static_cast<size_t>(maxid + 1), std::string());
  for (auto& kv : t.vocab)
    if (kv.second >= 0) t.inv[static_cast<size_t>(kv.second)] = kv.first;
}

int vocab_from(const JVal& v, Tokenizer& t, const char* what) {
  if (v.kind != JVal::Obj) return set_error(EC_EINVAL, "%s: vocab is not an object", what);
  for (const auto& kv : v.o) {
    if (kv.second.kind != JVal::Int) return set_error(EC_EINVAL, "%s: non-integer id", what);
    // ids index the decode table: bounded well above any real vocabulary
    if (kv.second.i < 0 || kv.second.i >= kMaxVocabId)
      return set_error(EC_EINVAL, "%s: id %lld of %s outside [0, %d)", what,
                       static_cast<long long>(kv.second.i), kv.first.c_str(), kMaxVocabId);
    t.vocab[kv.first] = static_cast<int>(kv.second.i);
  }
  build_inv(t);
  return EC_OK;
}

// json-specials (tokenizer.lisp:465-498)
void json_specials(const JVal& tj, int* bos, int* eos) {
  *bos = *eos = -1;
  std::unordered_map<std::string, int> by_name;
  if (const JVal* at = tj.get("added_tokens"))
    if (at->kind == JVal::Arr)
      for (const JVal& a : at->a) {
        const JVal* c = a.get("content");
        const JVal* id = a.get("id");
        if (c && c->kind == JVal::Str && id && id->kind == JVal::Int)
          by_name[c->s] = static_cast<int>(id->i);
      }
  const JVal* pp = tj.get("post_processor");
  if (!pp || pp->kind != JVal::Obj) return;
  const JVal* pt = pp->get("type");
  const std::string ptype = pt && pt->kind == JVal::Str ? pt->s : "";
  if (ptype == "RobertaProcessing" || ptype == "BertProcessing") {
    const JVal* cls = pp->get("cls");
    const JVal* sep = pp->get("sep");
    if (cls && cls->kind == JVal::Arr && cls->a.size() >= 2 && cls->a[1].kind == JVal::Int)
      *bos = static_cast<int>(cls->a[1].i);
    if (sep && sep->kind == JVal::Arr && sep->a.size() >= 2 && sep->a[1].kind == JVal::Int)
      *eos = static_cast<int>(sep->a[1].i);
    return;
  }
  const JVal* procs = pp->get("processors");
  if (!procs || procs->kind != JVal::Arr) return;
  for (const JVal& p : procs->a) {
    const JVal* ty = p.get("type");
    if (!ty || ty->kind != JVal::Str || ty->s != "TemplateProcessing") continue;
    bool seen_seq = false;
    if (const JVal* single = p.get("single"))
      if (single->kind == JVal::Arr)
        for (const JVal& item : single->a) {
          if (const JVal* st = item.get("SpecialToken")) {
            const JVal* idn = st->get("id");
            int id = -1;
            if (idn && idn->kind == JVal::Str) {
              auto it = by_name.find(idn->s);
              if (it != by_name.end()) id = it->second;
            }
            if (seen_seq) *eos = id;
            else *bos = id;
          }
          if (item.get("Sequence")) seen_seq = true;
        }
    return;  // the first TemplateProcessing only
  }
}

// pretok-mode (tokenizer.lisp:500-513)
bool pretok_llama3(const JVal& tj) {
  const JVal* pre = tj.get("pre_tokenizer");
  if (!pre || pre->kind != JVal::Obj) return false;
  std::string pat;
  bool have = false;
  auto look = [&](const JVal& p) {
    if (const JVal* split = p.get("pattern"))
      if (const JVal* rx = split->get("Regex"))
        if (rx->kind == JVal::Str) {
          pat = rx->s;
          have = true;
        }
  };
  const JVal* procs = pre->get("pretokenizers");
  if (procs && procs->kind == JVal::Arr && !procs->a.empty()) {
    for (const JVal& p : procs->a) look(p);
  } else {
    look(*pre);
  }
  return have && pat.find("\\r\\n") != std::string::npos;
}

int from_json(const char* path, Tokenizer& t) {
  JVal tj;
  int rc = parse_json(path, tj);
  if (rc) return rc;
  const JVal* model = tj.get("model");
  if (!model || model->kind != JVal::Obj) return set_error(EC_EINVAL, "%s: no model", path);
  const JVal* mt = model->get("type");
  const std::string mtype = mt && mt->kind == JVal::Str ? mt->s : "";
  const JVal* vocab = model->get("vocab");
  if (!vocab) return set_error(EC_EINVAL, "%s: no vocab", path);
  if ((rc = vocab_from(*vocab, t, path))) return rc;
  const JVal* norm = tj.get("normalizer");
  const JVal* lc = norm && norm->kind == JVal::Obj ? norm->get("lowercase") : nullptr;
  const bool lowercase = lc && lc->truthy();
  json_specials(tj, &t.bos, &t.eos);
  t.max_len = 512;
  if (mtype == "WordPiece") {
    t.kind = kWordPiece;
    t.build_trie();
    t.lowercase = lowercase;
    t.cls = t.bos >= 0 ? "" : "[CLS]";
    t.sep = t.eos >= 0 ? "" : "[SEP]";
    t.unk = "[UNK]";
    return EC_OK;
  }
  if (mtype == "BPE") {
    t.kind = kBpe;
    t.lowercase = false;
    t.cls = t.sep = "";
    t.unk = "<unk>";
    t.byte_level = true;
    t.llama3 = pretok_llama3(tj);
    int rank = 0;
    if (const JVal* ms = model->get("merges"))
      if (ms->kind == JVal::Arr)
        for (const JVal& m : ms->a) {
          if (m.kind == JVal::Arr && m.a.size() >= 2 && m.a[0].kind == JVal::Str &&
              m.a[1].kind == JVal::Str) {
            t.add_merge(m.a[0].s, m.a[1].s, rank++);
          } else if (m.kind == JVal::Str) {
            const size_t sp = m.s.find(' ');
            if (sp != std::string::npos) t.add_merge(m.s.substr(0, sp), m.s.substr(sp + 1), rank++);
          }
        }
    return EC_OK;
  }
  return set_error(EC_EUNSUPPORTED, "%s: unsupported tokenizer.json model type %s", path, mtype.c_str());
}

// ------------------------------------------------------------- registry --
// Shared ownership: a call holds its tokenizer until it returns, so an
// ec_tokenizer_free from another thread only drops the registry's share.
std::mutex g_mu;
std::vector<std::shared_ptr<const Tokenizer>> g_tok;

int add(std::unique_ptr<Tokenizer> t, int* handle) {
  if (t->kind == kBpe) t->build_bpe();
  std::shared_ptr<const Tokenizer> s(std::move(t));
  std::lock_guard<std::mutex> lk(g_mu);
  for (size_t i = 0; i < g_tok.size(); ++i)
    if (!g_tok[i]) {
      g_tok[i] = std::move(s);
      *handle = static_cast<int>(i) + 1;
      return EC_OK;
    }
  g_tok.push_back(std::move(s));
  *handle = static_cast<int>(g_tok.size());
  return EC_OK;
}

std::shared_ptr<const Tokenizer> get(int handle) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (handle < 1 || handle > static_cast<int>(g_tok.size())) return nullptr;
  return g_tok[static_cast<size_t>(handle) - 1];
}

// No C++ exception leaves the C ABI: allocation failures become EC_ENOMEM,
// anything else from the standard library EC_EINVAL.
template <class F>
int guarded(const char* what, F&& f) {
  try {
    return f();
  } catch (const std::bad_alloc&) {
    return set_error(EC_ENOMEM, "%s: out of host memory", what);
  } catch (const std::exception& e) {
    return set_error(EC_EINVAL, "%s: %s", what, e.what());
  }
}

}  // namespace
}  // namespace tok
}  // namespace ec

using namespace ec;
using namespace ec::tok;

extern "C" {

int ec_tokenizer_from_json(const char* path, int* handle) {
  clear_error();
  if (!path || !handle) return set_error(EC_EINVAL, "bad tokenizer arguments");
  return guarded(path, [&]() -> int {
    auto t = std::make_unique<Tokenizer>();
    int rc = from_json(path, *t);
    if (rc) return rc;
    return add(std::move(t), handle);
  });
}

int ec_tokenizer_wordpiece(const char* vocab_txt, int lowercase, int* handle) {
  clear_error();
  if (!vocab_txt || !handle) return set_error(EC_EINVAL, "bad tokenizer arguments");
  return guarded(vocab_txt, [&]() -> int {
    std::string text;
    int rc = read_file(vocab_txt, text);
    if (rc) return rc;
    auto t = std::make_unique<Tokenizer>();
    t->kind = kWordPiece;
    t->lowercase = lowercase != 0;
    for (const std::string& line : file_lines(text)) {
      const std::string tokn = trim_cr_space(line);
      t->vocab[tokn] = static_cast<int>(t->inv.size());
      t->inv.push_back(tokn);
    }
    t->build_trie();
    return add(std::move(t), handle);
  });
}

int ec_tokenizer_bpe(const char* vocab_json, const char* merges_txt, int lowercase,
                     int byte_level, int llama3, const char* cls_token, const char* sep_token,
                     const char* unk_token, int bos_id, int eos_id, int* handle) {
  clear_error();
  if (!vocab_json || !merges_txt || !handle) return set_error(EC_EINVAL, "bad tokenizer arguments");
  return guarded(vocab_json, [&]() -> int {
    auto t = std::make_unique<Tokenizer>();
    t->kind = kBpe;
    JVal v;
    int rc = parse_json(vocab_json, v);
    if (rc) return rc;
    if ((rc = vocab_from(v, *t, vocab_json))) return rc;
    std::string text;
    if ((rc = read_file(merges_txt, text))) return rc;
    const std::vector<std::string> lines = file_lines(text);
    int rank = 0;
    for (size_t i = 1; i < lines.size(); ++i) {  // the first line is the version line
      const std::string& l = lines[i];
      if (l.empty() || l[0] == '#') continue;
      const size_t sp = l.find(' ');
      if (sp == std::string::npos) continue;
      t->add_merge(l.substr(0, sp), l.substr(sp + 1), rank++);
    }
    t->lowercase = lowercase != 0;
    t->byte_level = byte_level != 0;
    t->llama3 = llama3 != 0;
    if (cls_token) t->cls = cls_token;
    if (sep_token) t->sep = sep_token;
    if (unk_token) t->unk = unk_token;
    t->bos = bos_id;
    t->eos = eos_id;
    return add(std::move(t), handle);
  });
}

int ec_tokenizer_unigram(const char* scores_json, int lowercase, int* handle) {
  clear_error();
  if (!scores_json || !handle) return set_error(EC_EINVAL, "bad tokenizer arguments");
  return guarded(scores_json, [&]() -> int {
    JVal v;
    int rc = parse_json(scores_json, v);
    if (rc) return rc;
    if (v.kind != JVal::Obj) return set_error(EC_EINVAL, "%s: not an object", scores_json);
    auto t = std::make_unique<Tokenizer>();
    t->kind = kUnigram;
    t->lowercase = lowercase != 0;
    for (const std::string& k : v.keys) {
      const JVal& sv = v.o.at(k);
      if (!sv.is_num()) return set_error(EC_EINVAL, "%s: score of %s is not a number", scores_json, k.c_str());
      t->vocab[k] = static_cast<int>(t->inv.size());
      t->inv.push_back(k);
      t->scores[k] = sv.num();
    }
    return add(std::move(t), handle);
  });
}

int ec_tokenizer_free(int handle) {
  clear_error();
  std::lock_guard<std::mutex> lk(g_mu);
  if (handle < 1 || handle > static_cast<int>(g_tok.size()) || !g_tok[static_cast<size_t>(handle) - 1])
    return set_error(EC_EINVAL, "no tokenizer %d", handle);
  g_tok[static_cast<size_t>(handle) - 1].reset();
  return EC_OK;
}

int ec_tokenizer_vocab_size(int handle) {
  clear_error();
  const auto t = get(handle);
  if (!t) return set_error(EC_EINVAL, "no tokenizer %d", handle);
  return static_cast<int>(t->inv.size());
}

int ec_tokenize(int handle, const char* const* texts, const int64_t* lengths, int ntexts,
                int32_t* ids, int64_t cap, int64_t* offsets, int nthreads) {
  clear_error();
  const auto t = get(handle);
  if (!t) return set_error(EC_EINVAL, "no tokenizer %d", handle);
  if (ntexts < 0 || (ntexts > 0 && (!texts || !offsets))) return set_error(EC_EINVAL, "bad tokenize arguments");
  return guarded("ec_tokenize", [&]() -> int {
    std::vector<std::vector<int32_t>> res(static_cast<size_t>(ntexts));
    std::vector<int> bad(static_cast<size_t>(std::max(ntexts, 1)), 0);
    int nt = nthreads > 0 ? nthreads : static_cast<int>(std::thread::hardware_concurrency());
    nt = std::max(1, std::min(nt, std::max(1, ntexts / 4)));
    auto work = [&](int w) {
      for (int i = w; i < ntexts; i += nt) {
        // a NULL text is only accepted as an empty one (length given as 0)
        const char* s = texts[i];
        const int64_t n = lengths ? lengths[i] : (s ? static_cast<int64_t>(std::strlen(s)) : -1);
        if (n < 0 || (!s && n > 0)) {
          bad[static_cast<size_t>(i)] = 2;
          continue;
        }
        try {  // an exception must not leave a worker thread
          if (!encode(*t, s ? s : "", static_cast<size_t>(n), res[static_cast<size_t>(i)]))
            bad[static_cast<size_t>(i)] = 1;
        } catch (const std::exception&) {
          bad[static_cast<size_t>(i)] = 3;
        }
      }
    };
    // reserved up front, so that once a thread runs nothing here can throw
    // before it is joined; a worker whose thread cannot start runs here
    std::vector<std::thread> th;
    std::vector<int> here;
    th.reserve(static_cast<size_t>(nt));
    here.reserve(static_cast<size_t>(nt));
    for (int w = 1; w < nt; ++w) {
      try {
        th.emplace_back(work, w);
      } catch (const std::system_error&) {
        here.push_back(w);
      }
    }
    work(0);
    for (int w : here) work(w);
    for (auto& x : th) x.join();
    offsets[0] = 0;
    for (int i = 0; i < ntexts; ++i) {
      const int b = bad[static_cast<size_t>(i)];
      if (b == 2) return set_error(EC_EINVAL, "text %d: NULL pointer or negative length", i);
      if (b == 3) return set_error(EC_ENOMEM, "text %d: out of host memory", i);
      if (b) return set_error(EC_EINVAL, "text %d: invalid UTF-8, or a piece with no id and no unknown token", i);
      offsets[i + 1] = offsets[i] + static_cast<int64_t>(res[static_cast<size_t>(i)].size());
    }
    if (offsets[ntexts] > cap || (offsets[ntexts] > 0 && !ids))
      return set_error(EC_EINVAL, "%lld ids do not fit the buffer of %lld", static_cast<long long>(offsets[ntexts]),
                       static_cast<long long>(cap));
    for (int i = 0; i < ntexts; ++i)
      std::memcpy(ids + offsets[i], res[static_cast<size_t>(i)].data(), res[static_cast<size_t>(i)].size() * 4);
    return EC_OK;
  });
}

int ec_tokenizer_decode(int handle, const int32_t* ids, int n, char* out, int64_t cap, int64_t* len) {
  clear_error();
  const auto t = get(handle);
  if (!t) return set_error(EC_EINVAL, "no tokenizer %d", handle);
  if (n < 0 || (n > 0 && !ids)) return set_error(EC_EINVAL, "bad decode arguments");
  return guarded("ec_tokenizer_decode", [&]() -> int {
    std::string s;
    for (int i = 0; i < n; ++i)
      if (ids[i] >= 0 && ids[i] < static_cast<int>(t->inv.size())) s += t->inv[static_cast<size_t>(ids[i])];
    if (len) *len = static_cast<int64_t>(s.size());
    if (static_cast<int64_t>(s.size()) > cap || (!out && !s.empty()))
      return set_error(EC_EINVAL, "%zu bytes do not fit the buffer of %lld", s.size(), static_cast<long long>(cap));
    if (!s.empty()) std::memcpy(out, s.data(), s.size());
    return EC_OK;
  });
}

}  // extern "C"
