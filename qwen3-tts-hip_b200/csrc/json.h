// Minimal JSON reader for config.json and safetensors headers.
#pragma once

#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace qtts {

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  bool has(const std::string& k) const { return kind == Object && obj.count(k); }
  const Json& at(const std::string& k) const {
    auto it = obj.find(k);
    if (kind != Object || it == obj.end()) throw std::runtime_error("missing json field: " + k);
    return it->second;
  }
  double number(const std::string& k) const {
    const Json& v = at(k);
    if (v.kind != Number) throw std::runtime_error("json field is not a number: " + k);
    return v.num;
  }
  long long integer(const std::string& k) const { return (long long)number(k); }
  const std::string& string(const std::string& k) const {
    const Json& v = at(k);
    if (v.kind != String) throw std::runtime_error("json field is not a string: " + k);
    return v.str;
  }

  static Json parse(const char* p, size_t n) {
    Parser ps{p, p + n};
    Json v = ps.value();
    ps.ws();
    if (ps.p != ps.end) throw std::runtime_error("trailing characters after json value");
    return v;
  }

 private:
  struct Parser {
    const char* p;
    const char* end;
    void ws() {
      while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    [[noreturn]] void fail(const char* what) { throw std::runtime_error(std::string("json: ") + what); }
    char peek() {
      ws();
      if (p >= end) fail("unexpected end");
      return *p;
    }
    void expect(char c) {
      if (peek() != c) fail("unexpected character");
      ++p;
    }
    bool lit(const char* s) {
      const char* q = p;
      while (*s) {
        if (q >= end || *q != *s) return false;
        ++q, ++s;
      }
      p = q;
      return true;
    }
    std::string str() {
      expect('"');
      std::string out;
      while (true) {
        if (p >= end) fail("unterminated string");
        char c = *p++;
        if (c == '"') break;
        if (c != '\\') {
          out.push_back(c);
          continue;
        }
        if (p >= end) fail("bad escape");
        char e = *p++;
        switch (e) {
          case '"': out.push_back('"'); break;
          case '\\': out.push_back('\\'); break;
          case '/': out.push_back('/'); break;
          case 'b': out.push_back('\b'); break;
          case 'f': out.push_back('\f'); break;
          case 'n': out.push_back('\n'); break;
          case 'r': out.push_back('\r'); break;
          case 't': out.push_back('\t'); break;
          case 'u': {
            if (end - p < 4) fail("bad unicode escape");
            unsigned cp = (unsigned)std::strtoul(std::string(p, p + 4).c_str(), nullptr, 16);
            p += 4;
            if (cp < 0x80) {
              out.push_back((char)cp);
            } else if (cp < 0x800) {
              out.push_back((char)(0xC0 | (cp >> 6)));
              out.push_back((char)(0x80 | (cp & 0x3F)));
            } else {
              out.push_back((char)(0xE0 | (cp >> 12)));
              out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
              out.push_back((char)(0x80 | (cp & 0x3F)));
            }
            break;
          }
          default: fail("bad escape");
        }
      }
      return out;
    }
    Json value() {
      Json v;
      char c = peek();
      if (c == '{') {
        ++p;
        v.kind = Object;
        if (peek() == '}') { ++p; return v; }
        while (true) {
          std::string k = str();
          expect(':');
          v.obj[k] = value();
          char d = peek();
          ++p;
          if (d == '}') break;
          if (d != ',') fail("expected , or }");
        }
      } else if (c == '[') {
        ++p;
        v.kind = Array;
        if (peek() == ']') { ++p; return v; }
        while (true) {
          v.arr.push_back(value());
          char d = peek();
          ++p;
          if (d == ']') break;
          if (d != ',') fail("expected , or ]");
        }
      } else if (c == '"') {
        v.kind = String;
        v.str = str();
      } else if (lit("true")) {
        v.kind = Bool;
        v.b = true;
      } else if (lit("false")) {
        v.kind = Bool;
      } else if (lit("null")) {
        v.kind = Null;
      } else {
        char* q = nullptr;
        std::string tmp(p, std::min<size_t>(64, end - p));
        v.num = std::strtod(tmp.c_str(), &q);
        if (q == tmp.c_str()) fail("bad value");
        p += (q - tmp.c_str());
        v.kind = Number;
      }
      return v;
    }
  };
};

}  // namespace qtts
