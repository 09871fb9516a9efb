// ec_json.h -- minimal JSON reader for config.json / 1_Pooling/config.json /
// tokenizer.json.
//
// Numbers with '.', 'e' or 'E' are converted exactly the way json.lisp's
// parse-number does (json.lisp:79-113): integer digits accumulated in a
// double, fraction digits added as digit * scale with scale starting at 0.1
// and divided by 10 per digit, then multiplied by 10^exp computed by
// repeated multiplication; so rms_norm_eps / rope_theta come out as the same
// doubles the Lisp loaders see.  Other numbers are integers.
#pragma once

#include <cstdint>
#include <exception>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace ec {

struct JVal {
  enum Kind { Null, Bool, Int, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  int64_t i = 0;
  double d = 0.0;
  std::string s;
  std::vector<JVal> a;
  std::map<std::string, JVal> o;
  std::vector<std::string> keys;  // object keys in file order (first occurrence)

  const JVal* get(const std::string& k) const {
    if (kind != Obj) return nullptr;
    auto it = o.find(k);
    return it == o.end() ? nullptr : &it->second;
  }
  bool is_num() const { return kind == Int || kind == Num; }
  double num() const { return kind == Int ? static_cast<double>(i) : d; }
  bool truthy() const {  // Lisp truthiness of gethash: anything but false/null
    return !(kind == Null || (kind == Bool && !b));
  }
};

class JParser {
 public:
  explicit JParser(const std::string& s) : s_(s) {}
  bool parse(JVal& out, std::string& err) {
    try {
      ws();
      value(out);
      return true;
    } catch (const std::string& e) {
      err = e;
      return false;
    } catch (const std::exception& e) {  // e.g. std::bad_alloc: no exception leaves the C ABI
      err = std::string("json: ") + e.what();
      return false;
    }
  }

 private:
  // nesting limit: a deeper file is refused before the recursion can
  // exhaust the calling thread's stack
  static constexpr int kMaxDepth = 256;
  const std::string& s_;
  size_t p_ = 0;
  int depth_ = 0;

  char peek() const { return p_ < s_.size() ? s_[p_] : '\0'; }
  char next() {
    if (p_ >= s_.size()) throw std::string("json: unexpected end");
    return s_[p_++];
  }
  void ws() {
    while (p_ < s_.size() && (s_[p_] == ' ' || s_[p_] == '\n' || s_[p_] == '\r' || s_[p_] == '\t'))
      ++p_;
  }
  void value(JVal& v) {
    ws();
    char c = peek();
    if (c == '{' || c == '[') {
      if (++depth_ > kMaxDepth) throw std::string("json: nested too deeply");
      if (c == '{')
        obj(v);
      else
        arr(v);
      --depth_;
    } else if (c == '"') {
      v.kind = JVal::Str;
      str(v.s);
    } else if (c == 't') {
      word("true");
      v.kind = JVal::Bool;
      v.b = true;
    } else if (c == 'f') {
      word("false");
      v.kind = JVal::Bool;
      v.b = false;
    } else if (c == 'n') {
      word("null");
      v.kind = JVal::Null;
    } else {
      num(v);
    }
  }
  void word(const char* w) {
    for (const char* q = w; *q; ++q)
      if (next() != *q) throw std::string("json: bad literal");
  }
  void obj(JVal& v) {
    v.kind = JVal::Obj;
    next();
    ws();
    if (peek() == '}') {
      next();
      return;
    }
    while (true) {
      ws();
      std::string k;
      str(k);
      ws();
      if (next() != ':') throw std::string("json: expected ':'");
      JVal x;
      value(x);
      if (v.o.find(k) == v.o.end()) v.keys.push_back(k);
      v.o[k] = std::move(x);
      ws();
      char c = next();
      if (c == '}') return;
      if (c != ',') throw std::string("json: expected ',' or '}'");
    }
  }
  void arr(JVal& v) {
    v.kind = JVal::Arr;
    next();
    ws();
    if (peek() == ']') {
      next();
      return;
    }
    while (true) {
      JVal x;
      value(x);
      v.a.push_back(std::move(x));
      ws();
      char c = next();
      if (c == ']') return;
      if (c != ',') throw std::string("json: expected ',' or ']'");
    }
  }
  unsigned hex4() {
    unsigned cp = 0;
    for (int k = 0; k < 4; ++k) {
      char h = next();
      cp <<= 4;
      if (h >= '0' && h <= '9') cp |= h - '0';
      else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
      else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
      else throw std::string("json: bad \\u escape");
    }
    return cp;
  }
  void str(std::string& out) {
    if (next() != '"') throw std::string("json: expected string");
    while (true) {
      char c = next();
      if (c == '"') return;
      if (c == '\\') {
        char e = next();
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            unsigned cp = hex4();
            // a high surrogate followed by an escaped low one is one
            // supplementary character
            if (cp >= 0xD800 && cp < 0xDC00 && p_ + 1 < s_.size() && s_[p_] == '\\' &&
                s_[p_ + 1] == 'u') {
              const size_t save = p_;
              p_ += 2;
              const unsigned lo = hex4();
              if (lo >= 0xDC00 && lo < 0xE000)
                cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
              else
                p_ = save;
            }
            if (cp < 0x80) out += static_cast<char>(cp);
            else if (cp < 0x800) {
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
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
  }
  void num(JVal& v) {
    size_t st = p_;
    while (p_ < s_.size()) {
      char c = s_[p_];
      if ((c >= '0' && c <= '9') || c == '-' || c == '+' || c == '.' || c == 'e' || c == 'E')
        ++p_;
      else
        break;
    }
    std::string t = s_.substr(st, p_ - st);
    if (t.empty()) throw std::string("json: bad value");
    if (t.find_first_of(".eE") == std::string::npos) {
      // an optional '-' and digits; a value outside int64 is an error
      const bool neg = t[0] == '-';
      size_t i = neg ? 1 : 0;
      if (i == t.size()) throw std::string("json: bad number");
      uint64_t mag = 0;
      for (; i < t.size(); ++i) {
        if (t[i] < '0' || t[i] > '9') throw std::string("json: bad number");
        const uint64_t dg = static_cast<uint64_t>(t[i] - '0');
        if (mag > (UINT64_MAX - dg) / 10) throw std::string("json: integer out of range");
        mag = mag * 10 + dg;
      }
      const uint64_t lim = neg ? (uint64_t{1} << 63) : static_cast<uint64_t>(INT64_MAX);
      if (mag > lim) throw std::string("json: integer out of range");
      v.kind = JVal::Int;
      v.i = neg ? static_cast<int64_t>(0 - mag) : static_cast<int64_t>(mag);
      return;
    }
    // json.lisp:85-113
    double mant = 0.0, sign = 1.0;
    size_t i = 0, n = t.size();
    if (t[0] == '-') {
      sign = -1.0;
      i = 1;
    }
    while (i < n && t[i] >= '0' && t[i] <= '9') {
      mant = mant * 10 + (t[i] - '0');
      ++i;
    }
    if (i < n && t[i] == '.') {
      ++i;
      double scale = 0.1;
      while (i < n && t[i] >= '0' && t[i] <= '9') {
        mant = mant + scale * (t[i] - '0');
        scale = scale / 10.0;
        ++i;
      }
    }
    if (i < n && (t[i] == 'e' || t[i] == 'E')) {
      ++i;
      int esign = 1;
      long e = 0;
      if (i < n && t[i] == '-') {
        esign = -1;
        ++i;
      }
      if (i < n && t[i] == '+') ++i;
      while (i < n && t[i] >= '0' && t[i] <= '9') {
        e = e * 10 + (t[i] - '0');
        ++i;
      }
      // (expt 10d0 k) for integer k: repeated squaring; 1/10^|k| for k < 0
      double base = 10.0, r = 1.0;
      long k = e;
      while (k > 0) {
        if (k & 1) r *= base;
        base *= base;
        k >>= 1;
      }
      mant = esign > 0 ? mant * r : mant * (1.0 / r);
    }
    v.kind = JVal::Num;
    v.d = sign * mant;
  }
};

}  // namespace ec
