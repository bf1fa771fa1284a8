// Minimal JSON reader for the Plan the C ABI receives (src/plan/ir.ts:41-60 serialised).
// Objects, arrays, numbers (kept as double), strings (with \" \\ \/ \b \f \n \r \t \uXXXX
// escapes, ASCII only for \u), true/false/null. Errors throw std::runtime_error with the
// byte offset.
#pragma once

#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace kh {

struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  bool has(const std::string& k) const { return kind == Obj && obj.count(k) > 0; }
  const Json& operator[](const std::string& k) const {
    auto it = obj.find(k);
    if (kind != Obj || it == obj.end()) throw std::runtime_error("plan json: missing key '" + k + "'");
    return it->second;
  }
  const Json& operator[](size_t i) const {
    if (kind != Arr || i >= arr.size()) throw std::runtime_error("plan json: index out of range");
    return arr[i];
  }
  size_t size() const { return kind == Arr ? arr.size() : obj.size(); }
  double as_num() const {
    if (kind != Num) throw std::runtime_error("plan json: expected a number");
    return num;
  }
  long long as_int() const { return (long long)as_num(); }
  const std::string& as_str() const {
    if (kind != Str) throw std::runtime_error("plan json: expected a string");
    return str;
  }
  bool as_bool() const {
    if (kind != Bool) throw std::runtime_error("plan json: expected a boolean");
    return b;
  }
  bool is_num() const { return kind == Num; }
  bool is_str() const { return kind == Str; }
};

class JsonReader {
 public:
  JsonReader(const char* s, size_t n) : s_(s), n_(n) {}
  Json parse() {
    Json v = value();
    ws();
    if (i_ != n_) fail("trailing characters");
    return v;
  }

 private:
  const char* s_;
  size_t n_;
  size_t i_ = 0;

  [[noreturn]] void fail(const char* why) {
    throw std::runtime_error(std::string("plan json: ") + why + " at byte " + std::to_string(i_));
  }
  void ws() {
    while (i_ < n_ && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
  }
  char peek() {
    ws();
    if (i_ >= n_) fail("unexpected end");
    return s_[i_];
  }
  void expect(char c) {
    if (peek() != c) fail("unexpected character");
    ++i_;
  }
  Json value() {
    char c = peek();
    Json v;
    if (c == '{') {
      v.kind = Json::Obj;
      ++i_;
      if (peek() == '}') { ++i_; return v; }
      for (;;) {
        if (peek() != '"') fail("expected a key");
        std::string k = string();
        expect(':');
        v.obj[k] = value();
        char d = peek();
        ++i_;
        if (d == '}') break;
        if (d != ',') fail("expected , or }");
      }
    } else if (c == '[') {
      v.kind = Json::Arr;
      ++i_;
      if (peek() == ']') { ++i_; return v; }
      for (;;) {
        v.arr.push_back(value());
        char d = peek();
        ++i_;
        if (d == ']') break;
        if (d != ',') fail("expected , or ]");
      }
    } else if (c == '"') {
      v.kind = Json::Str;
      v.str = string();
    } else if (c == 't' || c == 'f' || c == 'n') {
      auto lit = [&](const char* w) {
        size_t l = std::char_traits<char>::length(w);
        if (i_ + l > n_ || std::string(s_ + i_, l) != w) fail("bad literal");
        i_ += l;
      };
      if (c == 't') { lit("true"); v.kind = Json::Bool; v.b = true; }
      else if (c == 'f') { lit("false"); v.kind = Json::Bool; v.b = false; }
      else { lit("null"); v.kind = Json::Null; }
    } else {
      size_t st = i_;
      while (i_ < n_ && (std::isdigit((unsigned char)s_[i_]) || s_[i_] == '-' || s_[i_] == '+' || s_[i_] == '.' ||
                         s_[i_] == 'e' || s_[i_] == 'E'))
        ++i_;
      if (st == i_) fail("unexpected character");
      std::string tok(s_ + st, i_ - st);
      char* end = nullptr;
      v.kind = Json::Num;
      v.num = std::strtod(tok.c_str(), &end);
      if (!end || *end) fail("bad number");
    }
    return v;
  }
  std::string string() {
    expect('"');
    std::string out;
    while (i_ < n_ && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= n_) fail("bad escape");
        char e = s_[i_++];
        switch (e) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (i_ + 4 > n_) fail("bad \\u escape");
            unsigned code = std::stoul(std::string(s_ + i_, 4), nullptr, 16);
            i_ += 4;
            if (code > 0x7f) fail("non-ASCII \\u escape");
            out += char(code);
            break;
          }
          default: fail("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (i_ >= n_) fail("unterminated string");
    ++i_;
    return out;
  }
};

inline Json parse_json(const char* s, size_t n) { return JsonReader(s, n).parse(); }

inline std::vector<unsigned char> base64_decode(const std::string& in) {
  static int T[256];
  static bool init = false;
  if (!init) {
    for (int& t : T) t = -1;
    const char* a = "ABCDEFGHIJKLMNOPQRSTUVWXYZabcdefghijklmnopqrstuvwxyz0123456789+/";
    for (int i = 0; i < 64; ++i) T[(unsigned char)a[i]] = i;
    init = true;
  }
  std::vector<unsigned char> out;
  out.reserve(in.size() * 3 / 4);
  int val = 0, bits = -8;
  for (unsigned char c : in) {
    if (c == '=') break;
    if (T[c] < 0) throw std::runtime_error("plan json: bad base64");
    val = (val << 6) + T[c];
    bits += 6;
    if (bits >= 0) {
      out.push_back((unsigned char)((val >> bits) & 0xff));
      bits -= 8;
    }
  }
  return out;
}

}  // namespace kh
