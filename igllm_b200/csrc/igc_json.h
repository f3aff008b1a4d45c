// igc_json.h - a small JSON reader for config.json and safetensors headers.
#pragma once

#include <cctype>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace igc {

struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json *get(const char *key) const {
    if (kind != OBJ) return nullptr;
    for (auto &kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  double number(const char *key, double spare) const {
    const Json *j = get(key);
    if (!j) return spare;
    if (j->kind == NUM) return j->num;
    if (j->kind == BOOL) return j->b ? 1.0 : 0.0;
    if (j->kind == ARR && !j->arr.empty() && j->arr[0].kind == NUM) return j->arr[0].num;
    return spare;
  }
  bool flag(const char *key, bool spare) const {
    const Json *j = get(key);
    if (!j) return spare;
    if (j->kind == BOOL) return j->b;
    if (j->kind == NUM) return j->num != 0.0;
    return spare;
  }
  std::string text(const char *key, const char *spare) const {
    const Json *j = get(key);
    return (j && j->kind == STR) ? j->str : std::string(spare ? spare : "");
  }
};

class JsonReader {
 public:
  JsonReader(const char *text, size_t len) : p_(text), end_(text + len) {}
  bool parse(Json &out) {
    skip();
    if (!value(out, 0)) return false;
    return true;
  }

 private:
  const char *p_, *end_;
  void skip() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char *w) {
    size_t n = 0;
    while (w[n]) ++n;
    if ((size_t)(end_ - p_) < n) return false;
    for (size_t i = 0; i < n; ++i)
      if (p_[i] != w[i]) return false;
    p_ += n;
    return true;
  }
  static void put_utf8(std::string &s, uint32_t cp) {
    if (cp < 0x80) s += (char)cp;
    else if (cp < 0x800) { s += (char)(0xC0 | (cp >> 6)); s += (char)(0x80 | (cp & 63)); }
    else if (cp < 0x10000) {
      s += (char)(0xE0 | (cp >> 12)); s += (char)(0x80 | ((cp >> 6) & 63)); s += (char)(0x80 | (cp & 63));
    } else {
      s += (char)(0xF0 | (cp >> 18)); s += (char)(0x80 | ((cp >> 12) & 63));
      s += (char)(0x80 | ((cp >> 6) & 63)); s += (char)(0x80 | (cp & 63));
    }
  }
  bool string(std::string &s) {
    if (p_ >= end_ || *p_ != '"') return false;
    ++p_;
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if (c != '\\') { s += c; continue; }
      if (p_ >= end_) return false;
      char e = *p_++;
      switch (e) {
        case 'n': s += '\n'; break;
        case 't': s += '\t'; break;
        case 'r': s += '\r'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'u': {
          if (end_ - p_ < 4) return false;
          uint32_t cp = (uint32_t)strtoul(std::string(p_, 4).c_str(), nullptr, 16);
          p_ += 4;
          put_utf8(s, cp);
          break;
        }
        default: s += e;
      }
    }
    if (p_ >= end_) return false;
    ++p_;
    return true;
  }
  bool value(Json &out, int depth) {
    if (depth > 64 || p_ >= end_) return false;
    char c = *p_;
    if (c == '{') {
      out.kind = Json::OBJ;
      ++p_;
      skip();
      if (p_ < end_ && *p_ == '}') { ++p_; return true; }
      for (;;) {
        skip();
        std::string key;
        if (!string(key)) return false;
        skip();
        if (p_ >= end_ || *p_ != ':') return false;
        ++p_;
        skip();
        out.obj.emplace_back(std::move(key), Json());
        if (!value(out.obj.back().second, depth + 1)) return false;
        skip();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == '}') { ++p_; return true; }
        return false;
      }
    }
    if (c == '[') {
      out.kind = Json::ARR;
      ++p_;
      skip();
      if (p_ < end_ && *p_ == ']') { ++p_; return true; }
      for (;;) {
        skip();
        out.arr.emplace_back();
        if (!value(out.arr.back(), depth + 1)) return false;
        skip();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == ']') { ++p_; return true; }
        return false;
      }
    }
    if (c == '"') { out.kind = Json::STR; return string(out.str); }
    if (lit("true")) { out.kind = Json::BOOL; out.b = true; return true; }
    if (lit("false")) { out.kind = Json::BOOL; out.b = false; return true; }
    if (lit("null")) { out.kind = Json::NUL; return true; }
    {
      char *stop = nullptr;
      std::string num;
      while (p_ < end_ && (std::isdigit((unsigned char)*p_) || *p_ == '-' || *p_ == '+' || *p_ == '.' ||
                           *p_ == 'e' || *p_ == 'E'))
        num += *p_++;
      if (num.empty()) return false;
      out.kind = Json::NUM;
      out.num = strtod(num.c_str(), &stop);
      return true;
    }
  }
};

}  // namespace igc
