// Minimal JSON reader for the runtime manifest (manifest.json written by the
// reference's scripts/extract-qwen-runtime-assets.mjs:14-101). Objects, arrays,
// strings (with \" \\ \/ \b \f \n \r \t escapes; \u is kept verbatim), numbers,
// true/false/null. Throws std::runtime_error on malformed input.
#pragma once

#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace qd {

struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  const Json& at(const std::string& k) const {
    auto it = obj.find(k);
    if (kind != Obj || it == obj.end()) throw std::runtime_error("manifest: missing key '" + k + "'");
    return it->second;
  }
  const Json* find(const std::string& k) const {
    auto it = obj.find(k);
    return (kind == Obj && it != obj.end()) ? &it->second : nullptr;
  }
  const Json& at(size_t i) const {
    if (kind != Arr || i >= arr.size()) throw std::runtime_error("manifest: index out of range");
    return arr[i];
  }
  long long as_int() const {
    if (kind != Num) throw std::runtime_error("manifest: expected a number");
    return (long long)num;
  }
  double as_num() const {
    if (kind != Num) throw std::runtime_error("manifest: expected a number");
    return num;
  }
  const std::string& as_str() const {
    if (kind != Str) throw std::runtime_error("manifest: expected a string");
    return str;
  }
  size_t size() const { return kind == Arr ? arr.size() : obj.size(); }
};

class JsonParser {
 public:
  explicit JsonParser(const std::string& s) : s_(s) {}
  Json parse() {
    Json v = value();
    ws();
    if (i_ != s_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;
  [[noreturn]] void fail(const char* what) {
    throw std::runtime_error(std::string("manifest.json: ") + what + " at offset " + std::to_string(i_));
  }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
  }
  bool eat(char c) {
    ws();
    if (i_ < s_.size() && s_[i_] == c) { ++i_; return true; }
    return false;
  }
  Json value() {
    ws();
    if (i_ >= s_.size()) fail("unexpected end");
    const char c = s_[i_];
    Json v;
    if (c == '{') {
      ++i_;
      v.kind = Json::Obj;
      if (eat('}')) return v;
      do {
        ws();
        std::string k = string();
        if (!eat(':')) fail("expected ':'");
        v.obj[k] = value();
      } while (eat(','));
      if (!eat('}')) fail("expected '}'");
    } else if (c == '[') {
      ++i_;
      v.kind = Json::Arr;
      if (eat(']')) return v;
      do { v.arr.push_back(value()); } while (eat(','));
      if (!eat(']')) fail("expected ']'");
    } else if (c == '"') {
      v.kind = Json::Str;
      v.str = string();
    } else if (s_.compare(i_, 4, "true") == 0) {
      v.kind = Json::Bool; v.b = true; i_ += 4;
    } else if (s_.compare(i_, 5, "false") == 0) {
      v.kind = Json::Bool; v.b = false; i_ += 5;
    } else if (s_.compare(i_, 4, "null") == 0) {
      i_ += 4;
    } else {
      const char* start = s_.c_str() + i_;
      char* end = nullptr;
      v.num = std::strtod(start, &end);
      if (end == start) fail("bad value");
      v.kind = Json::Num;
      i_ += (size_t)(end - start);
    }
    return v;
  }
  std::string string() {
    if (i_ >= s_.size() || s_[i_] != '"') fail("expected string");
    ++i_;
    std::string out;
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= s_.size()) fail("bad escape");
        const char e = s_[i_++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': out += "\\u"; break;
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (i_ >= s_.size()) fail("unterminated string");
    ++i_;
    return out;
  }
};

inline Json parse_json(const std::string& s) { return JsonParser(s).parse(); }

}  // namespace qd
