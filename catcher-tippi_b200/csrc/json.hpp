// Minimal JSON reader for the release artifact's manifest, the safetensors
// header and the tokenizer's tokenizer.json: objects keep their key order,
// numbers are doubles, strings are UTF-8 (\\u escapes, surrogate pairs
// included, become UTF-8).  Errors throw CQ_INVALID_ARGUMENT with the text
// "invalid <what>: <reason>".
#pragma once

#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "qlinear.hpp"

namespace nemotron_cuda {

struct Json {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& key) const {
    if (kind != kObj) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JsonParser {
 public:
  JsonParser(const char* p, size_t n, const std::string& what) : p_(p), end_(p + n), what_(what) {}
  Json parse() {
    Json v = value();
    ws();
    if (p_ != end_) fail("trailing characters");
    return v;
  }

 private:
  [[noreturn]] void fail(const std::string& msg) { throw_invalid("invalid " + what_ + ": " + msg); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char* s) {
    const size_t n = std::strlen(s);
    if (static_cast<size_t>(end_ - p_) >= n && std::memcmp(p_, s, n) == 0) {
      p_ += n;
      return true;
    }
    return false;
  }
  Json value() {
    ws();
    if (p_ >= end_) fail("unexpected end");
    Json v;
    const char c = *p_;
    if (c == '{') {
      v.kind = Json::kObj;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return v;
      }
      while (true) {
        ws();
        if (p_ >= end_ || *p_ != '"') fail("expected a key");
        std::string k = string();
        ws();
        if (p_ >= end_ || *p_ != ':') fail("expected ':'");
        ++p_;
        v.obj.emplace_back(std::move(k), value());
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return v;
        }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Json::kArr;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return v;
      }
      while (true) {
        v.arr.push_back(value());
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return v;
        }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Json::kStr;
      v.str = string();
      return v;
    }
    if (lit("true")) {
      v.kind = Json::kBool;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.kind = Json::kBool;
      return v;
    }
    if (lit("null")) return v;
    // number
    const char* s = p_;
    while (p_ < end_ && (std::strchr("+-0123456789.eE", *p_) != nullptr)) ++p_;
    if (s == p_) fail("unexpected character");
    v.kind = Json::kNum;
    v.num = std::strtod(std::string(s, p_).c_str(), nullptr);
    return v;
  }
  unsigned hex4() {
    if (end_ - p_ < 4) fail("bad \\u escape");
    unsigned v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= static_cast<unsigned>(c - '0');
      else if (c >= 'a' && c <= 'f') v |= static_cast<unsigned>(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= static_cast<unsigned>(c - 'A' + 10);
      else fail("bad \\u escape");
    }
    return v;
  }
  static void utf8(unsigned cp, std::string& out) {
    if (cp < 0x80) {
      out.push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
      out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
      out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
  }
  std::string string() {
    ++p_;  // opening quote
    std::string out;
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (p_ >= end_) fail("bad escape");
      c = *p_++;
      switch (c) {
        case 'n': out.push_back('\n'); break;
        case 't': out.push_back('\t'); break;
        case 'r': out.push_back('\r'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'u': {
          unsigned cp = hex4();
          // a UTF-16 surrogate pair encodes one code point above U+FFFF
          if (cp >= 0xD800 && cp < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
            p_ += 2;
            const unsigned lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(cp, out);
          break;
        }
        default: out.push_back(c);  // \" \\ \/
      }
    }
    if (p_ >= end_) fail("unterminated string");
    ++p_;
    return out;
  }

  const char* p_;
  const char* end_;
  std::string what_;
};

}  // namespace nemotron_cuda
